"""CPU tests of the C ABI library: it loads, exports every declared symbol,
and fails loudly (no fallback) when there is no GPU."""
import ctypes
import math
import os
import re

import pytest

from conftest import ROOT, gpu_available

HEADER = os.path.join(ROOT, "include", "cortex.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^CORTEX_API\s+[\w\s\*]*?\b(\w+)\(", src, re.M)))


def test_header_declares_reference_boundary():
    names = declared_functions()
    reference = ["cortex_init", "cortex_load_stream", "cortex_forward", "cortex_reset_cache", "cortex_free",
                 "cortex_init_gpu", "get_vocab_size", "get_ctx_size", "cortex_load_layer", "cortex_extract_layer",
                 "cortex_load_adam_layer", "cortex_extract_adam_layer", "cortex_train_step"]
    for n in reference:
        assert n in names


def test_library_exports_every_declared_symbol(built):
    from snai_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_functions():
        assert hasattr(lib, name), name
    # the Python binding declares the same set
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_null_state_is_safe(built):
    from snai_b200 import load
    lib = load()
    assert lib.get_vocab_size(None) == 0
    assert lib.get_ctx_size(None) == 0
    lib.cortex_free(None)
    lib.cortex_reset_cache(None)
    assert math.isnan(lib.cortex_train_step(None, None, None, 0, 0.1))
    assert "NULL state" in lib.cortex_last_error().decode()
    assert lib.cortex_train_apply(None, 0.1, 1.0) != 0


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_no_gpu_fails_loudly(built, small_model):
    from snai_b200 import Cortex, CortexError, load
    lib = load()
    assert not lib.cortex_load_stream(small_model.encode(), 2)
    assert "CUDA" in lib.cortex_last_error().decode()
    with pytest.raises(CortexError):
        Cortex(small_model, num_heads=2)
