"""cortex_forward_batch_noalloc: the forward pass for callers that cannot
allocate GPU memory while they run (their device memory is owned by another
allocator or a fixed pool).  Its activation scratch is a static array in the
library.  It runs the same kernels as cortex_forward_batch on the same rows,
so with the same chunking its logits are identical bit for bit: this test
drives both entry points through the C ABI on two separate states of the
same model, two calls in a row (a prompt, then one more token), and
compares the logits (np.array_equal) and the per-slot positions.

The d=1024 case needs several chunks of the 8 MiB array (128 rows each):
4 sequences x 100 prompt tokens are chunks of 128, 128, 128 and 16 rows
(a partial last chunk).  The reference state is made with the same chunk
size (SNAI_CHUNK_ROWS) so both entry points split the rows alike.

The file is named to run last, so a failure here cannot hide other tests."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import PREC_BF16, PREC_FP32, Cortex, load  # noqa: E402
from conftest import make_model  # noqa: E402

SCRATCH = 8 << 20  # bytes of the library's static array


def _call(lib, fn, eng, tokens):
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    B, n = t.shape
    out = np.zeros((B, eng.vocab), dtype=np.float32)
    rc = fn(eng.h, t.ctypes.data_as(ctypes.c_void_p), B, n, None, out.ctypes.data_as(ctypes.c_void_p), 0)
    assert rc == 0, lib.cortex_last_error()
    return out


def _carve(rows, D, att_ch):
    """Bytes the library carves for `rows` rows: row and logits-row
    descriptors, h, x, q, staged K/V, attention output, MLP intermediate and
    normed logits rows (fp32), each rounded up to 256 bytes."""
    off = 0
    for b in (16, 8, 4 * D, 4 * D, 4 * att_ch, 8 * att_ch, 4 * D, 16 * D, 4 * D):
        off = (off + rows * b + 255) // 256 * 256
    return off


def _chunk_rows(D, att_ch, m_max=256):
    rows = min(m_max, SCRATCH // _carve(1, D, att_ch))
    while rows > 0 and _carve(rows, D, att_ch) > SCRATCH:
        rows -= 1
    return rows // 128 * 128 if rows > 128 else rows


def _engines(path, heads, B, prec, chunk):
    old = os.environ.get("SNAI_CHUNK_ROWS")
    os.environ["SNAI_CHUNK_ROWS"] = str(chunk)
    try:
        ref = Cortex(path, num_heads=heads, max_seqs=B, precision=prec)
    finally:
        if old is None:
            del os.environ["SNAI_CHUNK_ROWS"]
        else:
            os.environ["SNAI_CHUNK_ROWS"] = old
    tst = Cortex(path, num_heads=heads, max_seqs=B, precision=prec)
    return ref, tst


@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
@pytest.mark.parametrize("shape", ["d128", "d1024"])
def test_noalloc_forward_matches_forward_batch(shape, prec, model_dir, built):
    if shape == "d128":
        path = make_model(model_dir, "noalloc.snai", 1000, 128, 96, 2, seed=17)
        heads, D, B, plen = 2, 128, 3, 40  # 120 rows: one chunk (tensor cores in BF16 mode)
    else:
        path = make_model(model_dir, "noalloc1024.snai", 2000, 1024, 128, 1, seed=18)
        heads, D, B, plen = 16, 1024, 4, 100  # 400 rows: chunks of 128, 128, 128, 16
    chunk = _chunk_rows(D, D)
    assert shape == "d128" or chunk == 128, chunk
    lib = load()
    rng = np.random.default_rng(prec + 10 * D)
    prompts = rng.integers(0, 1000, (B, plen)).astype(np.int32)
    nxt = rng.integers(0, 1000, (B, 1)).astype(np.int32)
    ref, tst = _engines(path, heads, B, prec, chunk)
    for step, toks in enumerate((prompts, nxt)):
        a = _call(lib, lib.cortex_forward_batch, ref, toks)
        b = _call(lib, lib.cortex_forward_batch_noalloc, tst, toks)
        assert np.isfinite(a).all() and np.abs(a).max() > 0, step
        assert np.array_equal(b, a), (step, float(np.abs(b - a).max()))
        assert [tst.pos(s) for s in range(B)] == [ref.pos(s) for s in range(B)]
    ref.close()
    tst.close()

