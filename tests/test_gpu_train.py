"""GPU training step (core/cortex.nim:565-822) through the C ABI vs the oracle.

* gradients of forward + backward, per tensor within an fp32 tolerance
  (the GPU sums in GEMM order, the reference sequentially);
* the clip and Adam given the same gradients: bit for bit when the clip does
  not apply, within a few ulps when it does (the gradient norm is summed in
  another order);
* whole steps (cortex_train_step): losses, and the weights, moments and the
  forward pass that follow them;
* the reference's side effects: K/V rows of the training sequence left in the
  cache, the position unchanged; ctx cut-off; zero tokens.
"""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import PREC_BF16, PREC_FP32, PREC_TF32, Cortex, SnaiCortexBridge, load  # noqa: E402
from conftest import make_model, rel_err  # noqa: E402

TYPES = (10, 11, 12, 13, 14, 15, 16, 17)
# max |gpu - oracle| / max |oracle| per gradient tensor.  FP32 engines run
# the training GEMMs in fp32 (only the summation order differs: 2.5e-6
# measured); TF32 and BF16 engines on the TF32 tensor cores (10-bit operand
# mantissas, fp32 accumulation).
GRAD_TOL = {PREC_FP32: 2e-5, PREC_TF32: 1e-2, PREC_BF16: 1e-2}
LOSS_TOL = {PREC_FP32: 2e-5, PREC_TF32: 2e-3, PREC_BF16: 2e-3}  # relative, mean loss


def keys(layers):
    return [(-1, 0), (-1, 1), (-1, 2)] + [(l, t) for l in range(layers) for t in TYPES]


def seq(rng, V, n):
    x = rng.integers(0, V, n).astype(np.int32)
    y = rng.integers(0, V, n).astype(np.int32)
    x[n // 3] = x[n // 2] = x[1]  # a repeated token
    x[2] = V + 3                  # out of range: row 0
    y[4] = -1                     # out of range target: 0
    return x, y


@pytest.mark.parametrize("precision", [PREC_FP32, PREC_TF32])
@pytest.mark.parametrize("shape", [
    # name, vocab, dim, ctx, layers, heads, tokens
    ("tr_a", 1001, 128, 140, 2, 2, 131),  # hs 64, two row tiles, V and act not multiples of 4
    ("tr_b", 3001, 256, 300, 1, 4, 290),  # three row tiles, 24 logits column tiles
    ("tr_c", 203, 24, 40, 2, 4, 37),      # head size 6: unaligned head slices (scalar GEMM loads)
    ("tr_d", 16384, 512, 300, 1, 8, 260), # the benchmark vocabulary and head size: K=16384 split-K products
])
def test_train_gradients_vs_oracle(model_dir, built, shape, precision):
    name, V, D, ctx, L, heads, n = shape
    p = make_model(model_dir, name + ".snai", V, D, ctx, L, seed=21, std=0.08)
    rng = np.random.default_rng(3)
    x, y = seq(rng, V, n)
    e = Cortex(p, num_heads=heads, precision=precision)
    o = O.Oracle(p, num_heads=heads)
    lg = e.train_grads(x, y)
    lo = o.train_grads(x, y)
    assert abs(lg - lo) <= LOSS_TOL[precision] * abs(lo), (lg, lo)
    worst = 0.0
    for k in keys(L):
        gg = e.tensor(k[0], k[1], "grad")
        go = o.tensor(k[0], k[1], "grad")
        err = rel_err(gg, go)
        worst = max(worst, err)
        assert err < GRAD_TOL[precision], (k, err)
    # the weights are untouched by the gradient pass
    assert np.array_equal(e.tensor(0, 12), o.tensor(0, 12))
    print(f"{name} precision {precision}: loss {lg:.6f} vs {lo:.6f}, worst gradient error {worst:.2e}")
    e.close()
    o.close()


def _load_grads(e, o, rng, L, scale):
    for k in keys(L):
        n = o.tensor_size(*k)
        g = (rng.standard_normal(n) * scale).astype(np.float32)
        if k == (-1, 0):
            g[: n // 3] = 0  # embedding rows without gradient: the sparse rule skips them
        o.set_tensor(k[0], k[1], g, "grad")
        e.set_tensor(k[0], k[1], g, "grad")


def test_adam_bit_exact_given_gradients(model_dir, built):
    p = make_model(model_dir, "tr_a.snai", 1001, 128, 140, 2, seed=21, std=0.08)
    e = Cortex(p, num_heads=2)
    o = O.Oracle(p, num_heads=2)
    rng = np.random.default_rng(9)
    # step 1 from zero moments, step 2 from loaded moments (cortex_load_adam_layer)
    for step, lr in ((1, 0.01), (2, 0.003)):
        if step == 2:
            for k in keys(2):
                for which in ("m", "v"):
                    vals = np.abs(rng.standard_normal(o.tensor_size(*k))).astype(np.float32) * 1e-4
                    o.set_tensor(k[0], k[1], vals, which)
                    e.set_tensor(k[0], k[1], vals, which)
        _load_grads(e, o, rng, 2, 1e-5)  # global norm below 1: no clip
        e.train_apply(lr, 7.0)
        o.train_apply(lr, 7.0)
        info = e.train_info()
        assert info["adam_steps"] == step == o.adam_steps
        assert not info["clipped"]
        for k in keys(2):
            for which in ("weight", "m", "v"):
                assert np.array_equal(e.tensor(k[0], k[1], which), o.tensor(k[0], k[1], which)), (step, k, which)
    e.close()
    o.close()


def test_adam_with_clip(model_dir, built):
    p = make_model(model_dir, "tr_a.snai", 1001, 128, 140, 2, seed=21, std=0.08)
    e = Cortex(p, num_heads=2)
    o = O.Oracle(p, num_heads=2)
    rng = np.random.default_rng(10)
    _load_grads(e, o, rng, 2, 1e-2)  # global norm far above 1
    e.train_apply(0.01, 5.0)
    o.train_apply(0.01, 5.0)
    info = e.train_info()
    assert info["clipped"] and info["grad_norm"] > 1
    # the reference sums the 3.7 M squares sequentially in fp32, the GPU in
    # double: the clip factors differ by about 1e-5 relative, m follows it
    # and v its square; a weight moves by lr * x / (x + 1e-8), x = |clipped
    # gradient| / scale, so only gradients near 1e-8 feel the factor: at most
    # about lr * 1e-5 (the weights' atol below is lr * 2e-4)
    for k in keys(2):
        for which in ("m", "v"):
            a, b = e.tensor(k[0], k[1], which), o.tensor(k[0], k[1], which)
            assert np.allclose(a, b, rtol=1e-4, atol=0), (k, which)
        a, b = e.tensor(k[0], k[1]), o.tensor(k[0], k[1])
        assert np.allclose(a, b, rtol=1e-6, atol=0.01 * 2e-4), (k, float(np.abs(a - b).max()))
    e.close()
    o.close()


@pytest.mark.parametrize("precision", [PREC_FP32, PREC_TF32, PREC_BF16])
def test_train_steps_then_forward(model_dir, built, precision):
    p = make_model(model_dir, "tr_a.snai", 1001, 128, 140, 2, seed=21, std=0.08)
    e = Cortex(p, num_heads=2, precision=precision)
    o = O.Oracle(p, num_heads=2)
    rng = np.random.default_rng(4)
    lr = 0.002
    # BF16 engines train on the TF32 tensor cores: looser bounds
    loss_tol, min_cos = (1e-4, 0.9999) if precision == PREC_FP32 else (3e-3, 0.95)
    W0 = {k: e.tensor(k[0], k[1]).astype(np.float64) for k in keys(2)}
    for step in range(3):
        x, y = seq(rng, 1001, 100 + 7 * step)
        lg = e.train_step(x, y, lr)
        lo = o.train_step(x, y, lr)
        assert abs(lg - lo) <= loss_tol * abs(lo), (step, lg, lo)
    assert e.train_info()["adam_steps"] == 3
    worst = 1.0
    for k in keys(2):
        a, b = e.tensor(k[0], k[1]).astype(np.float64), o.tensor(k[0], k[1]).astype(np.float64)
        # Adam's first steps move a weight by about lr whatever the gradient's
        # size, so a gradient below the GEMMs' rounding may move the other
        # way on the GPU: bound each move, and compare the update directions
        assert np.abs(a - b).max() <= 2 * 3 * lr + 1e-6, k
        da, db = a - W0[k], b - W0[k]
        if not db.any():
            assert not da.any(), k
            continue
        cos = float(da @ db / (np.linalg.norm(da) * np.linalg.norm(db)))
        worst = min(worst, cos)
        assert cos > min_cos, (k, cos)
    print(f"precision {precision}: lowest cosine of the weight updates vs the oracle's: {worst:.5f}")
    # the forward pass runs on the updated weights (in BF16 mode through the
    # refreshed bf16 copies): the oracle given the GPU's weights agrees
    o2 = O.Oracle(p, num_heads=2)
    for k in keys(2):
        o2.set_tensor(k[0], k[1], e.tensor(k[0], k[1]))
    e.reset()
    t = rng.integers(0, 1001, 30).astype(np.int32)
    ref = o2.forward(t)
    got = e.forward([t])[0]
    assert rel_err(got, ref) < {PREC_FP32: 2e-5, PREC_TF32: 4e-3, PREC_BF16: 3e-2}[precision]
    e.close()
    o.close()
    o2.close()


def test_train_leaves_kv_rows_and_position(model_dir, built):
    """core/cortex.nim:509-510: the training forward writes the K/V cache rows
    of its positions; cachedTokens is not changed, so a forward that follows
    without a reset attends over them."""
    p = make_model(model_dir, "tr_a.snai", 1001, 128, 140, 2, seed=21, std=0.08)
    lib = load()
    s = lib.cortex_load_stream(p.encode(), 2)
    o = O.Oracle(p, num_heads=2)
    rng = np.random.default_rng(8)
    V = 1001
    buf = np.zeros(V, dtype=np.float32)
    pre = rng.integers(0, V, 5).astype(np.int32)
    lib.cortex_forward(s, pre.ctypes.data_as(ctypes.c_void_p), 5, buf.ctypes.data_as(ctypes.c_void_p))
    o.forward(pre)
    x, y = seq(rng, V, 12)
    lg = lib.cortex_train_step(s, x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), 12, 0.0)
    lo = o.train_step(x, y, 0.0)
    assert abs(lg - lo) <= LOSS_TOL[PREC_FP32] * abs(lo)
    nxt = np.array([17], dtype=np.int32)
    lib.cortex_forward(s, nxt.ctypes.data_as(ctypes.c_void_p), 1, buf.ctypes.data_as(ctypes.c_void_p))
    ref = o.forward(nxt)  # position 5, over the training K/V of positions 0..4
    assert o.pos == 6
    assert rel_err(buf, ref) < 2e-5
    lib.cortex_free(s)
    o.close()


def test_train_zero_tokens_and_ctx_cut(model_dir, built):
    p = make_model(model_dir, "tr_c.snai", 203, 24, 40, 2, seed=21, std=0.08)
    e = Cortex(p, num_heads=4)
    o = O.Oracle(p, num_heads=4)
    assert e.train_step([], [], 0.1) == 0.0
    assert e.train_info()["adam_steps"] == 0
    x = (np.arange(55) % 203).astype(np.int32)  # 55 > ctx 40: the first 40 are used
    y = ((x + 5) % 203).astype(np.int32)
    lg = e.train_step(x, y, 0.01)
    lo = o.train_step(x, y, 0.01)
    assert abs(lg - lo) <= LOSS_TOL[PREC_FP32] * abs(lo)
    # the PHP bridge passes the last ctx tokens (src/tensor_ffi_adapter.php:135-151)
    b = SnaiCortexBridge(p, num_heads=4)
    lb = b.train_step(list(x), list(y), 0.01)
    o2 = O.Oracle(p, num_heads=4)
    assert abs(lb - o2.train_step(x[-40:], y[-40:], 0.01)) <= LOSS_TOL[PREC_FP32] * abs(lb)
    b.close()
    e.close()
    o.close()
    o2.close()


def test_training_cluster_round(model_dir, built):
    """The reference's training-cluster round (src/train_cluster.php:144-224
    with src/train_worker.php:113-145): each worker trains its own copy of
    the model on its own text, then the workers' weights are averaged.  Here
    two FP32 engines take two steps each on different sequences, then
    cortex_average_states averages them on the GPU; the oracle does the same
    with two oracle states and the merge restatement.  Every averaged weight
    is within two Adam steps of the oracle's (a gradient below the GEMMs'
    rounding may step the other way), and the update directions agree."""
    from snai_b200 import average_states
    p = make_model(model_dir, "tr_a.snai", 1001, 128, 140, 2, seed=21, std=0.08)
    rng = np.random.default_rng(12)
    lr = 0.003
    data = [[seq(rng, 1001, 120) for _ in range(2)] for _ in range(2)]
    engines = [Cortex(p, num_heads=2) for _ in range(2)]
    oracles = [O.Oracle(p, num_heads=2) for _ in range(2)]
    W0 = {k: oracles[0].tensor(k[0], k[1]).astype(np.float64) for k in keys(2)}
    for w in range(2):
        for x, y in data[w]:
            lg = engines[w].train_step(x, y, lr)
            lo = oracles[w].train_step(x, y, lr)
            assert abs(lg - lo) <= 1e-4 * abs(lo), (w, lg, lo)
    average_states(engines)
    for k in keys(2):
        a = engines[0].tensor(k[0], k[1]).astype(np.float64)
        assert np.array_equal(a, engines[1].tensor(k[0], k[1]))  # every engine holds the average
        # src/train_cluster.php:188-205: sum in worker order (double), divide, store fp32
        b = ((oracles[0].tensor(k[0], k[1]).astype(np.float64) + oracles[1].tensor(k[0], k[1])) / 2.0)
        b = b.astype(np.float32).astype(np.float64)
        assert np.abs(a - b).max() <= 2 * lr + 1e-6, k
        da, db = a - W0[k], b - W0[k]
        if db.any():
            cos = float(da @ db / (np.linalg.norm(da) * np.linalg.norm(db)))
            assert cos > 0.999, (k, cos)
    for e in engines:
        e.close()
    for o in oracles:
        o.close()
