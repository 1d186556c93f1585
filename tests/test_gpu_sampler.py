"""GPU sampler (cortex_sample through the C ABI) vs the oracle: sampled ids
must be bit-identical for the same logits and uniforms."""
import json
import os

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import VARIANT_A, VARIANT_B, sample_device, sample_params  # noqa: E402
from test_oracle import load_kats, random_rows  # noqa: E402


def gpu_sample(L, hist, U, params, hist_len=None, ld=None):
    dev = torch.device("cuda")
    L = np.ascontiguousarray(L, dtype=np.float32)
    R, V = L.shape
    if ld is not None and ld > V:
        big = np.zeros((R, ld), dtype=np.float32)
        big[:, :V] = L
        lt = torch.from_numpy(big).to(dev)[:, :V]
    else:
        lt = torch.from_numpy(L).to(dev)
    H = np.ascontiguousarray(hist, dtype=np.int32).reshape(R, -1)
    ht = torch.from_numpy(H).to(dev) if H.shape[1] > 0 else None
    hl = None if hist_len is None else torch.from_numpy(np.ascontiguousarray(hist_len, dtype=np.int32)).to(dev)
    ut = torch.from_numpy(np.ascontiguousarray(U, dtype=np.float32)).to(dev)
    out = torch.full((R,), -7, dtype=torch.int32, device=dev)
    sample_device(lt, ut, params, ht, hl, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def stream_batch(L, hist, U):
    """The rows tiled (uniforms varied) to a batch large enough (4 rows per
    SM) for the one-warp-per-row kernels; smaller batches take the
    CTA-per-row kernels."""
    need = 4 * torch.cuda.get_device_properties(0).multi_processor_count
    reps = -(-need // L.shape[0])
    rng = np.random.default_rng(L.shape[0] * 7 + L.shape[1])
    U2 = np.concatenate([U] + [rng.random(len(U)).astype(np.float32) for _ in range(reps - 1)])
    return np.tile(L, (reps, 1)), np.tile(hist, (reps, 1)), U2


def oracle_ids(L, hist, U, variant, T, rep, k=40, p=0.9, exp_mode=1, hist_len=None):
    ids = []
    for r in range(L.shape[0]):
        h = hist[r] if hist_len is None else hist[r][:hist_len[r]]
        if variant == VARIANT_A:
            ids.append(O.sample_a(L[r], h, T, rep, U[r], exp_mode))
        else:
            ids.append(O.sample_b(L[r], h, T, k, p, rep, U[r], exp_mode))
    return np.asarray(ids, dtype=np.int32)


@pytest.mark.parametrize("case", load_kats(), ids=lambda c: c["name"])
def test_gpu_sampler_kats(case, built):
    L = np.asarray([case["logits"]], dtype=np.float32)
    hist = np.asarray([case["hist"]], dtype=np.int32).reshape(1, -1)
    if case["variant"] == 0:
        prm = sample_params(VARIANT_A, case["T"], case["rep"], nan_guard=0)
    else:
        prm = sample_params(VARIANT_B, case["T"], case["rep"], case["top_k"], case["top_p"])
    got = gpu_sample(L, hist, [case["u"]], prm)
    assert got[0] == case["expect"], case["why"]


def synth(rng, R, V, H=256, spikes=True):
    L = rng.normal(0, 4, (R, V)).astype(np.float32)
    if spikes:
        L[rng.random((R, V)) < 0.01] += 12.0
    hist = rng.integers(0, V, (R, H)).astype(np.int32)
    U = rng.random(R).astype(np.float32)
    return L, hist, U


@pytest.mark.parametrize("V", [1000, 1001, 16384, 32000])
@pytest.mark.parametrize("T", [0.01, 0.25, 0.7, 2.0])
def test_variant_a_matches_oracle(V, T, built):
    rng = np.random.default_rng(V + int(T * 100))
    L, hist, U = synth(rng, 48, V)
    prm = sample_params(VARIANT_A, T, 1.15, nan_guard=0)
    got = gpu_sample(L, hist, U, prm)
    assert np.array_equal(got, oracle_ids(L, hist, U, VARIANT_A, T, 1.15, exp_mode=1))
    # libm exp (what PHP calls) gives the same ids on these rows
    assert np.array_equal(got, oracle_ids(L, hist, U, VARIANT_A, T, 1.15, exp_mode=0))


@pytest.mark.parametrize("V", [1000, 1001, 16384, 32000])
@pytest.mark.parametrize("cfg", [(0.0, 40, 0.9), (0.7, 40, 0.9), (0.7, 50, 0.95), (1.0, 1, 0.9), (0.9, 512, 1.0)])
def test_variant_b_matches_oracle(V, cfg, built):
    T, k, p = cfg
    rng = np.random.default_rng(V + k)
    L, hist, U = synth(rng, 48, V)
    prm = sample_params(VARIANT_B, T, 1.1, k, p)
    got = gpu_sample(L, hist, U, prm)
    assert np.array_equal(got, oracle_ids(L, hist, U, VARIANT_B, T, 1.1, k, p, exp_mode=1))
    assert np.array_equal(got, oracle_ids(L, hist, U, VARIANT_B, T, 1.1, k, p, exp_mode=0))


@pytest.mark.parametrize("V", [50000, 131072, 229380])
def test_large_vocab_both_variants(V, built):
    """Rows longer than one CTA's register row: a cluster of CTAs per row
    (2, 4 and 7 slices; the first and last with a partial final slice)."""
    rng = np.random.default_rng(5 + V)
    L, hist, U = synth(rng, 16, V)
    for prm, args in [(sample_params(VARIANT_A, 0.7, 1.15, nan_guard=0), (VARIANT_A, 0.7, 1.15)),
                      (sample_params(VARIANT_A, 0.01, 1.15, nan_guard=0), (VARIANT_A, 0.01, 1.15)),
                      (sample_params(VARIANT_B, 0.7, 1.1, 50, 0.95), (VARIANT_B, 0.7, 1.1, 50, 0.95))]:
        got = gpu_sample(L, hist, U, prm)
        assert np.array_equal(got, oracle_ids(L, hist, U, *args))


def test_ties_and_edge_uniforms(built):
    """Whole rows of equal logits (variant B's tie path), quantised logits,
    u = 0 and u = 1, history shorter per row, a padded row stride."""
    rng = np.random.default_rng(9)
    R, V = 24, 16384
    L = np.round(rng.normal(0, 1, (R, V)) * 2).astype(np.float32) / 2
    L[0:4] = 0.25  # all equal
    L[4:6] = -3.0
    U = rng.random(R).astype(np.float32)
    U[0::3] = 0.0
    U[1::3] = 1.0
    hist = rng.integers(0, V, (R, 300)).astype(np.int32)
    hist_len = rng.integers(0, 301, R).astype(np.int32)
    for prm, args in [(sample_params(VARIANT_A, 0.9, 1.3, nan_guard=0), (VARIANT_A, 0.9, 1.3)),
                      (sample_params(VARIANT_A, 0.005, 1.3, nan_guard=0), (VARIANT_A, 0.005, 1.3)),
                      (sample_params(VARIANT_B, 0.7, 0.5, 40, 0.9), (VARIANT_B, 0.7, 0.5, 40, 0.9)),
                      (sample_params(VARIANT_B, 0.0, 0.5, 40, 0.9), (VARIANT_B, 0.0, 0.5, 40, 0.9)),
                      (sample_params(VARIANT_B, 1.0, 0.0, 512, 1.0), (VARIANT_B, 1.0, 0.0, 512, 1.0))]:
        got = gpu_sample(L, hist, U, prm, hist_len=hist_len, ld=V + 36)
        assert np.array_equal(got, oracle_ids(L, hist, U, *args, hist_len=hist_len))


def test_variant_b_tail_edges(built):
    """Variant B's top-p tail where the warp's certified sums cannot decide
    and the exact sequential arithmetic takes over: running sums that land
    on top_p exactly (k equal logits: 1/2, 1/4 steps), exponentials that
    overflow to inf (PHP then keeps order[0]), u = 1 (r equal to the last
    running sum), and T exactly at the greedy threshold."""
    rng = np.random.default_rng(21)
    R, V = 32, 4096
    L = rng.normal(0, 1, (R, V)).astype(np.float32)
    top = rng.choice(V, (R, 4), replace=True)
    for r in range(R):
        L[r, top[r]] = 30.0
    L[8:12, :4] = 800.0  # exp(800 / T) overflows
    U = rng.random(R).astype(np.float32)
    U[0::4] = 1.0
    U[1::4] = 0.5
    hist = rng.integers(0, V, (R, 64)).astype(np.int32)
    Lb, Hb, Ub = stream_batch(L, hist, U)
    for T, rep, k, p in [(0.7, 0.0, 2, 0.5), (0.7, 0.0, 4, 0.5), (1.0, 0.0, 4, 1.0), (0.7, 0.0, 4, 0.75),
                         (0.01, 0.0, 4, 0.9), (0.7, 1.5, 40, 0.9)]:
        for LL, HH, UU in ((L, hist, U), (Lb, Hb, Ub)):
            got = gpu_sample(LL, HH, UU, sample_params(VARIANT_B, T, rep, k, p))
            assert np.array_equal(got, oracle_ids(LL, HH, UU, VARIANT_B, T, rep, k, p)), (len(LL), T, rep, k, p)


def test_variant_a_stream_edges(built):
    """Variant A through the one-warp-per-row kernel: logits of magnitude 1e4
    (wide error bounds: the exact tiers), a history covering a quarter of
    the vocabulary with penalties above and below 1, rows of -inf but for a
    few ids, a NaN entry (the sequential tier), u = 0 and 1, a partial last
    chunk."""
    rng = np.random.default_rng(41)
    R, V = 24, 4096 + 1024 + 8
    L = rng.normal(0, 3, (R, V)).astype(np.float32)
    L[0:3] *= 3000.0
    L[3:5] = -np.inf
    L[3, [7, 900, 5000]] = [1.0, 2.0, 1.5]
    L[4, V - 1] = 0.0
    L[5, 1234] = np.nan
    L[6:8, rng.choice(V, 40, replace=False)] += 15.0
    U = rng.random(R).astype(np.float32)
    U[8] = 0.0
    U[9] = 1.0
    U[10] = np.float32(np.nextafter(np.float32(1.0), np.float32(0.0)))
    hist = rng.integers(0, V, (R, 1024)).astype(np.int32)
    Lb, Hb, Ub = stream_batch(L, hist, U)
    for T, rep in [(0.7, 1.15), (0.25, 0.5), (2.0, 1.0), (0.011, 3.0), (0.01, 1.15), (0.004, 0.5)]:
        for LL, HH, UU in ((L, hist, U), (Lb, Hb, Ub)):
            got = gpu_sample(LL, HH, UU, sample_params(VARIANT_A, T, rep, nan_guard=0))
            assert np.array_equal(got, oracle_ids(LL, HH, UU, VARIANT_A, T, rep)), (len(LL), T, rep)


def test_variant_b_ordered_and_clustered_rows(built):
    """Rows whose largest logits all sit at the start (descending order) or
    the end (ascending), rows where a few hundred entries share the top
    values, and rows with NaN and -inf entries: the opening threshold of
    the one-warp-per-row kernel is then far off, and the row is regathered
    or selected exactly."""
    rng = np.random.default_rng(31)
    R, V = 16, 16384
    L = rng.normal(0, 2, (R, V)).astype(np.float32)
    L[0:4] = -np.sort(-L[0:4], axis=1)
    L[4:8] = np.sort(L[4:8], axis=1)
    L[8:10, rng.choice(V, 300, replace=False)] = 9.5
    L[10, ::7] = np.nan
    L[11, ::3] = -np.inf
    L[12, :V - 20] = np.nan
    U = rng.random(R).astype(np.float32)
    hist = rng.integers(0, V, (R, 128)).astype(np.int32)
    Lb, Hb, Ub = stream_batch(L, hist, U)
    for T, rep, k, p in [(0.7, 1.1, 50, 0.95), (0.0, 1.1, 40, 0.9), (1.3, 0.0, 128, 0.99), (0.7, -0.5, 40, 0.9)]:
        for LL, HH, UU in ((L, hist, U), (Lb, Hb, Ub)):
            got = gpu_sample(LL, HH, UU, sample_params(VARIANT_B, T, rep, k, p))
            assert np.array_equal(got, oracle_ids(LL, HH, UU, VARIANT_B, T, rep, k, p)), (len(LL), T, rep, k, p)


@pytest.mark.parametrize("V", [16384, 32000, 131072])
def test_streaming_kernels_large_batch(V, built):
    """A batch of 4 rows per SM (the one-warp-per-row kernels) of the sampler
    benchmark's kind of rows, both variants, with a ragged history."""
    rng = np.random.default_rng(3 * V)
    need = 4 * torch.cuda.get_device_properties(0).multi_processor_count
    L, hist, U = synth(rng, need, V)
    hist_len = rng.integers(0, hist.shape[1] + 1, need).astype(np.int32)
    for variant, T, rep, k, p in [(VARIANT_A, 0.7, 1.15, 40, 0.9), (VARIANT_A, 0.01, 1.15, 40, 0.9),
                                  (VARIANT_B, 0.7, 1.15, 50, 0.95), (VARIANT_B, 0.0, 1.1, 40, 0.9)]:
        prm = (sample_params(VARIANT_A, T, rep, nan_guard=0) if variant == VARIANT_A
               else sample_params(VARIANT_B, T, rep, k, p))
        got = gpu_sample(L, hist, U, prm, hist_len=hist_len)
        want = oracle_ids(L, hist, U, variant, T, rep, k, p, hist_len=hist_len)
        assert np.array_equal(got, want), (variant, T)


@pytest.mark.parametrize("kind", ["spiky", "flat"])
def test_variant_a_every_row_of_a_large_batch(kind, built):
    """Variant A over 4096 rows of V=16384 against the oracle, every row: the
    rows the streaming kernel cannot certify (a few per thousand of the
    benchmark's spiky rows, many more of near-uniform ones) go through the
    CTA-per-row kernel's mixed tier (exact exponentials for the entries that
    carry the row's mass) and, failing that, the exact tiers."""
    R, V, H = 4096, 16384, 256
    rng = np.random.default_rng(11 if kind == "spiky" else 12)
    if kind == "spiky":
        L = (rng.standard_normal((R, V)) * 2.0).astype(np.float32)
        L += (rng.random((R, V)) < 0.01).astype(np.float32) * 12.0
    else:
        L = (rng.standard_normal((R, V)) * 0.05).astype(np.float32)
    hist = rng.integers(0, V, (R, H)).astype(np.int32)
    U = rng.random(R).astype(np.float32)
    got = gpu_sample(L, hist, U, sample_params(VARIANT_A, 0.7, 1.15, nan_guard=0))
    want, _ = O.sample_rows(L, hist, U, VARIANT_A, 0.7, 1.15, exp_mode=1, nthreads=os.cpu_count() or 1)
    bad = np.flatnonzero(got != want)
    assert bad.size == 0, (kind, bad[:8], got[bad[:8]], want[bad[:8]])


def test_nan_guard_and_argument_errors(built):
    from snai_b200 import CortexError
    rng = np.random.default_rng(1)
    L, hist, U = synth(rng, 4, 2048)
    L[1, 0] = np.nan
    got = gpu_sample(L, hist, U, sample_params(VARIANT_A, 0.8, 1.15, nan_guard=1))
    assert got[1] == -1 and got[0] >= 0 and got[2] >= 0
    with pytest.raises(CortexError):
        gpu_sample(L, hist, U, sample_params(VARIANT_A, 0.0, 1.15))  # PHP: division by zero
    with pytest.raises(CortexError):
        gpu_sample(L, hist, U, sample_params(VARIANT_B, 0.7, 1.1, 0, 0.9))
    with pytest.raises(CortexError):
        gpu_sample(L, hist, U, sample_params(VARIANT_B, 0.7, 1.1, 513, 0.9))
