"""Parity at the shapes the throughput benchmark runs.

The decode benchmark's two models (seeded SNAI_V4, V=16384, ctx 1024,
L=2): d=1024 with 16 heads and d=512 with 8 heads.  Four distinct
sequences get a 960-token prompt, so attention reads up to 964 cached
positions, then three teacher-forced decode steps; each sequence is
replicated over 2048 slots, so a decode step's projections run at 2048 rows
(one GPU's share of the benchmark at N=2: the CTA-pair tensor-core GEMM for
QKV (N=3D), W_up (N=4D), W_down (N=D, K=4D) and the logits (N=16384), the
128 x 64 single-CTA tiles for Wo), and the prompts as 1024-row chunks.
Checked against the oracle (the CPU restatement of core/cortex.nim:487-563,
teacher-forced on the same tokens):

* logits after the prompt and after every forced token, per precision,
  max |gpu - oracle| / max |oracle| within the stated tolerance;
* the replicas of a sequence get bit-identical logits, and a second engine
  with one slot per sequence (passes of 4 rows: single-CTA tiles
  throughout; its attention held to the whole-row kernel with
  SNAI_ATTENTION_SPLIT=0, as passes of many rows use) gets the same bits (a
  row's result does not depend on the other rows of the pass or on the
  projection tile shape);
* one more step through the fused decode (cortex_decode_batch: sample, then
  feed) gives, row by row, exactly the id the oracle's sampler picks from
  the GPU's logits with the same history and uniform
  (src/tensor_ffi_adapter.php:168-204, T 0.7, top-k 40, top-p 0.9,
  rep 1.1);
* the same for one sequence on the fp32 path (one-row projections),
  with the PHP inference script's sampler (src/snai_inference.php:151-195,
  T 0.25, rep 1.15).
"""
import functools

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import PREC_BF16, PREC_FP32, PREC_TF32, Cortex, VARIANT_A, VARIANT_B, sample_params  # noqa: E402
from conftest import make_model, rel_err  # noqa: E402

# logits tolerance: max |gpu - oracle| / max |oracle|
TOL = {PREC_FP32: 2e-5, PREC_TF32: 4e-3, PREC_BF16: 3e-2}

CASES = {
    # the benchmark's models: d=1024 (16 heads) and d=512 (8 heads)
    "d1024": dict(V=16384, D=1024, L=2, heads=16, ctx=1024),
    "d512": dict(V=16384, D=512, L=2, heads=8, ctx=1024),
}
S, P, T, R = 4, 960, 3, 2048  # sequences, prompt length, forced steps, slots


@functools.lru_cache(maxsize=None)
def _oracle(case, model_dir):
    c = CASES[case]
    path = make_model(model_dir, f"bench_{case}.snai", c["V"], c["D"], c["ctx"], c["L"], seed=1234, std=0.02)
    rng = np.random.default_rng(c["D"])
    prompts = rng.integers(0, c["V"], (S, P)).astype(np.int32)
    forced = rng.integers(0, c["V"], (S, T)).astype(np.int32)
    o = O.Oracle(path, num_heads=c["heads"])
    _, ref, _ = o.generate(prompts, T, np.zeros((S, T), np.float32), VARIANT_B, 0.7, 1.1, forced=forced,
                           want_logits=True, nthreads=S)
    o.close()
    return path, prompts, forced, ref


@pytest.mark.parametrize("prec", [PREC_TF32, PREC_BF16])
@pytest.mark.parametrize("case", ["d1024", "d512"])
def test_bench_shapes_logits_and_ids(case, prec, model_dir, built):
    c = CASES[case]
    path, prompts, forced, ref = _oracle(case, str(model_dir))
    seq = np.arange(R) % S
    e = Cortex(path, num_heads=c["heads"], max_seqs=R, precision=prec)
    got = [e.forward(prompts[seq])]
    for s in range(T):
        got.append(e.forward(forced[seq, s:s + 1]))
    errs = []
    for s in range(T + 1):
        g = got[s]
        assert np.isfinite(g).all()
        for r in range(S):
            assert np.array_equal(g[seq == r], np.broadcast_to(g[r], (R // S, c["V"]))), (s, r)
        err = max(rel_err(g[r], ref[r, s]) for r in range(S))
        errs.append(err)
        assert err < TOL[prec], (s, err)
    print(f"{case} prec {prec}: max rel err per step {errs}")
    assert e.pos(0) == P + T
    import os
    os.environ["SNAI_ATTENTION_SPLIT"] = "0"
    try:
        small = Cortex(path, num_heads=c["heads"], max_seqs=S, precision=prec)
    finally:
        del os.environ["SNAI_ATTENTION_SPLIT"]
    mine = [small.forward(prompts)] + [small.forward(forced[:, s:s + 1]) for s in range(T)]
    for s in range(T + 1):
        assert np.array_equal(mine[s], got[s][:S]), s
    small.close()
    # one decode step through the fused path: ids vs the oracle sampler on the GPU logits
    lg = e.logits(np.arange(R))
    rng = np.random.default_rng(5 + prec)
    U = rng.random(S).astype(np.float32)[seq]
    ids = e.decode(U, sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9))
    for r in range(S):  # the replicas share logits, history and uniform, so their ids too
        hist = list(prompts[r]) + list(forced[r])
        want = O.sample_b(lg[r], hist, 0.7, 40, 0.9, 1.1, U[r])
        assert ids[r] == want, (r, ids[r], want)
        assert (ids[seq == r] == want).all(), r
    e.close()


@pytest.mark.parametrize("case", ["d1024", "d512"])
def test_bench_shapes_fp32_one_sequence(case, model_dir, built):
    c = CASES[case]
    path, prompts, forced, ref = _oracle(case, str(model_dir))
    e = Cortex(path, num_heads=c["heads"], max_seqs=1, precision=PREC_FP32)
    errs = [rel_err(e.forward(prompts[:1])[0], ref[0, 0])]
    for s in range(T):
        errs.append(rel_err(e.forward(forced[:1, s:s + 1])[0], ref[0, s + 1]))
    print(f"{case} fp32: max rel err per step {errs}")
    assert max(errs) < TOL[PREC_FP32], errs
    lg = e.logits([0])[0]
    ids = e.decode(np.asarray([0.37], np.float32), sample_params(VARIANT_A, 0.25, 1.15))
    want = O.sample_a(lg, list(prompts[0]) + list(forced[0]), 0.25, 1.15, np.float32(0.37))
    assert ids[0] == want
    e.close()
