"""cortex_forward_batch_noalloc: the forward pass for callers that cannot
allocate GPU memory while they run (their device memory is owned by another
allocator or a fixed pool).  Its activation scratch is a static array in the
library, so its results must match cortex_forward_batch's exactly: this
test drives both entry points through the C ABI on two separate states of
the same model, two calls in a row (a prompt, then one more token), and
compares the logits and the per-slot positions.

The file is named to run last, so a failure here cannot hide other tests."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import PREC_BF16, PREC_FP32, Cortex, load  # noqa: E402
from conftest import make_model, rel_err  # noqa: E402


def _call(lib, fn, eng, tokens):
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    B, n = t.shape
    out = np.zeros((B, eng.vocab), dtype=np.float32)
    rc = fn(eng.h, t.ctypes.data_as(ctypes.c_void_p), B, n, None, out.ctypes.data_as(ctypes.c_void_p), 0)
    assert rc == 0, lib.cortex_last_error()
    return out


@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
def test_noalloc_forward_matches_forward_batch(prec, model_dir, built):
    path = make_model(model_dir, "noalloc.snai", 1000, 128, 96, 2, seed=17)
    lib = load()
    rng = np.random.default_rng(prec)
    B = 3
    prompts = rng.integers(0, 1000, (B, 40)).astype(np.int32)  # 120 rows: tensor cores in BF16 mode
    nxt = rng.integers(0, 1000, (B, 1)).astype(np.int32)
    ref = Cortex(path, num_heads=2, max_seqs=B, precision=prec)
    tst = Cortex(path, num_heads=2, max_seqs=B, precision=prec)
    tol = 2e-5 if prec == PREC_FP32 else 3e-2
    for step, toks in enumerate((prompts, nxt)):
        a = _call(lib, lib.cortex_forward_batch, ref, toks)
        b = _call(lib, lib.cortex_forward_batch_noalloc, tst, toks)
        assert rel_err(b, a) <= tol, step
        assert [tst.pos(s) for s in range(B)] == [ref.pos(s) for s in range(B)]
    ref.close()
    tst.close()
