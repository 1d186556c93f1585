"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def built():
    """Builds the oracle and libcortex.so if they are missing."""
    import subprocess
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    if not os.path.exists(os.path.join(ROOT, "snai_b200", "libcortex.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "snai_b200", "csrc")], check=True)
    return True


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def make_model(model_dir, name, vocab, dim, ctx, layers, seed=1234, std=0.02):
    from snai_b200 import modelgen
    p = os.path.join(str(model_dir), name)
    if not os.path.exists(p):
        modelgen.random_model(p, vocab, dim, ctx, layers, seed=seed, std=std)
    return p


@pytest.fixture(scope="session")
def small_model(model_dir):
    """d=128, 2 layers, ctx 96, V=1000 (heads = d/64 = 2)."""
    return make_model(model_dir, "small.snai", 1000, 128, 96, 2, seed=7)


def rel_err(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(1e-30, np.max(np.abs(b))))
