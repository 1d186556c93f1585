"""GPU forward pass through the C ABI vs the oracle (teacher-forced logits,
fp32-relative tolerance per GEMM precision) and the fused decode step's ids
vs the oracle sampler applied to the GPU's own logits (bit-exact)."""
import ctypes
import math

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import (PREC_BF16, PREC_FP32, PREC_TF32, Cortex, SnaiCortexBridge, VARIANT_A,  # noqa: E402
                       VARIANT_B, load, run_inference, sample_params)
from conftest import make_model, rel_err  # noqa: E402

# logits tolerance: max |gpu - oracle| / max |oracle|
TOL = {PREC_FP32: 2e-5, PREC_TF32: 4e-3, PREC_BF16: 3e-2}


def oracle_logits_seq(path, heads, tokens_steps):
    """Feeds each list in tokens_steps in turn; returns the logits after each."""
    o = O.Oracle(path, num_heads=heads)
    out = [o.forward(t).copy() for t in tokens_steps]
    o.close()
    return out


def test_legacy_api_prompt_and_steps(small_model, built):
    lib = load()
    s = lib.cortex_load_stream(small_model.encode(), 2)
    assert s, lib.cortex_last_error()
    V = lib.get_vocab_size(s)
    assert V == 1000 and lib.get_ctx_size(s) == 96
    rng = np.random.default_rng(0)
    steps = [list(rng.integers(0, V, 40))] + [[int(x)] for x in rng.integers(-5, V + 5, 12)]
    ref = oracle_logits_seq(small_model, 2, steps)
    buf = np.zeros(V, dtype=np.float32)
    for i, t in enumerate(steps):
        a = np.ascontiguousarray(t, dtype=np.int32)
        lib.cortex_forward(s, a.ctypes.data_as(ctypes.c_void_p), len(a), buf.ctypes.data_as(ctypes.c_void_p))
        assert rel_err(buf, ref[i]) < TOL[PREC_FP32], i
    lib.cortex_free(s)


def test_ctx_cutoff_reset_and_clamp(model_dir, built):
    p = make_model(model_dir, "ctx16.snai", 300, 64, 16, 1, seed=3, std=0.1)
    e = Cortex(p, num_heads=1)
    assert e.head_size == 64
    o = O.Oracle(p, num_heads=1)
    toks = np.arange(10, 24, dtype=np.int32)
    a = e.forward([toks])
    b = o.forward(toks)
    assert rel_err(a[0], b) < TOL[PREC_FP32]
    # positions 14, 15 then ctx: the last token is dropped -> no logits written
    lib = load()
    sentinel = np.full(300, 5.0, dtype=np.float32)
    t2 = np.asarray([1, 2, 3], dtype=np.int32)
    lib.cortex_forward(e.h, t2.ctypes.data_as(ctypes.c_void_p), 3, sentinel.ctypes.data_as(ctypes.c_void_p))
    assert e.pos(0) == 16 and np.all(sentinel == 5.0)
    e.reset([0])
    assert e.pos(0) == 0
    o.reset()
    bad = np.asarray([-4, 299, 300, 12345], dtype=np.int32)  # out-of-range ids read row 0
    assert rel_err(e.forward([bad])[0], o.forward(bad)) < TOL[PREC_FP32]
    e.close()


def test_load_extract_adam_train(small_model, built):
    lib = load()
    s = lib.cortex_load_stream(small_model.encode(), 2)
    D, V = 128, 1000
    w = np.zeros(D * D, dtype=np.float32)
    lib.cortex_extract_layer(s, 1, 13, w.ctypes.data_as(ctypes.c_void_p), D * D)
    from snai_b200 import modelgen
    _, t = modelgen.read_model(small_model)
    assert np.array_equal(w.reshape(D, D), t["1.w_k"])
    neww = (np.arange(D * D, dtype=np.float32) * 1e-4).astype(np.float32)
    lib.cortex_load_layer(s, 1, 13, neww.ctypes.data_as(ctypes.c_void_p), D * D)
    lib.cortex_extract_layer(s, 1, 13, w.ctypes.data_as(ctypes.c_void_p), D * D)
    assert np.array_equal(w, neww)
    junk = np.ones(7, dtype=np.float32)
    lib.cortex_load_layer(s, 1, 13, junk.ctypes.data_as(ctypes.c_void_p), 7)  # size mismatch: no-op
    lib.cortex_extract_layer(s, 1, 13, w.ctypes.data_as(ctypes.c_void_p), D * D)
    assert np.array_equal(w, neww)
    m = np.zeros(V * D, dtype=np.float32)
    lib.cortex_extract_adam_layer(s, -1, 0, False, m.ctypes.data_as(ctypes.c_void_p), V * D)
    assert not m.any()
    m[:] = 0.5
    lib.cortex_load_adam_layer(s, -1, 0, True, m.ctypes.data_as(ctypes.c_void_p), V * D)
    m2 = np.zeros_like(m)
    lib.cortex_extract_adam_layer(s, -1, 0, True, m2.ctypes.data_as(ctypes.c_void_p), V * D)
    assert np.array_equal(m, m2)
    assert lib.cortex_train_step(s, None, None, 0, 0.01) == 0.0  # act <= 0: nothing to do (core/cortex.nim:567)
    lib.cortex_free(s)
    # cortex_init: zero weights, unit RMSNorm weights -> zero logits
    z = lib.cortex_init(50, 32, 8, 1, 1)
    assert z
    buf = np.full(50, 3.0, dtype=np.float32)
    a = np.asarray([3], dtype=np.int32)
    lib.cortex_forward(z, a.ctypes.data_as(ctypes.c_void_p), 1, buf.ctypes.data_as(ctypes.c_void_p))
    assert not buf.any()
    r = np.zeros(32, dtype=np.float32)
    lib.cortex_extract_layer(z, 0, 10, r.ctypes.data_as(ctypes.c_void_p), 32)
    assert np.all(r == 1.0)
    lib.cortex_free(z)


def test_bad_files(tmp_path, small_model, built):
    lib = load()
    data = open(small_model, "rb").read()
    (tmp_path / "short.snai").write_bytes(data[:-8])
    (tmp_path / "magic.snai").write_bytes(b"SNAI_V5\x00" + data[8:])
    assert not lib.cortex_load_stream(str(tmp_path / "short.snai").encode(), 2)
    assert not lib.cortex_load_stream(str(tmp_path / "magic.snai").encode(), 2)
    assert not lib.cortex_load_stream(b"/nonexistent/x.snai", 2)


@pytest.mark.parametrize("prec", [PREC_FP32, PREC_TF32, PREC_BF16])
def test_batched_teacher_forced(prec, small_model, built):
    """B slots with a shared prompt length, then teacher-forced decode steps;
    B=70 puts >= 64 rows through the tensor-core path in TF32/BF16 mode."""
    B, plen, steps = 70, 20, 4
    rng = np.random.default_rng(prec)
    prompts = rng.integers(0, 1000, (B, plen)).astype(np.int32)
    forced = rng.integers(0, 1000, (B, steps)).astype(np.int32)
    e = Cortex(small_model, num_heads=2, max_seqs=B, precision=prec)
    got = [e.forward(prompts)]
    for s in range(steps):
        got.append(e.forward(forced[:, s:s + 1]))
    o = O.Oracle(small_model, num_heads=2)
    _, ref, _ = o.generate(prompts, steps, np.zeros((B, steps), np.float32), VARIANT_A, 0.8, 1.15,
                           forced=forced, want_logits=True)
    for s in range(steps + 1):
        err = max(rel_err(got[s][b], ref[b, s]) for b in range(B))
        assert err < TOL[prec], (s, err)
    e.close()


@pytest.mark.parametrize("prec", [PREC_TF32, PREC_BF16])
def test_pair_tiles_prefill_and_decode(prec, model_dir, built):
    """Shapes for the CTA-pair tensor-core GEMM: 300 sequences (a partial
    256-row pair tile), d=256 (N=768/256/1024 projections, K=256/1024) and
    V=3000 (a partial 256-wide logits tile), prompt rows 2400, then
    teacher-forced decode steps of 300 rows that also take the logits GEMM."""
    path = make_model(model_dir, "pair.snai", 3000, 256, 32, 2, seed=21)
    B, plen, steps = 300, 8, 2
    rng = np.random.default_rng(11 + prec)
    prompts = rng.integers(0, 3000, (B, plen)).astype(np.int32)
    forced = rng.integers(0, 3000, (B, steps)).astype(np.int32)
    e = Cortex(path, num_heads=4, max_seqs=B, precision=prec)
    got = [e.forward(prompts)]
    for s in range(steps):
        got.append(e.forward(forced[:, s:s + 1]))
    o = O.Oracle(path, num_heads=4)
    _, ref, _ = o.generate(prompts, steps, np.zeros((B, steps), np.float32), VARIANT_A, 0.8, 1.15,
                           forced=forced, want_logits=True)
    for s in range(steps + 1):
        err = max(rel_err(got[s][b], ref[b, s]) for b in range(B))
        assert err < TOL[prec], (s, err)
    e.close()


@pytest.mark.parametrize("B", [1, 2, 3, 5, 9])
def test_gemv_shapes(B, model_dir, built):
    """fp32 GEMV edges: d=1040 (K=1040 in three 384-column slices; W_down's
    K=4160 in eight 640-column slices of two passes, the last slice empty),
    V=1001 (a last row quad of one row), 16 heads of 64 channels (16 unused
    channels), and row counts that fill activation groups of 1, 2, 4 and 8
    partly (prompt rows 3B, decode rows B)."""
    path = make_model(model_dir, "gemv.snai", 1001, 1040, 16, 1, seed=33)
    plen, steps = 3, 2
    rng = np.random.default_rng(40 + B)
    prompts = rng.integers(0, 1001, (B, plen)).astype(np.int32)
    forced = rng.integers(0, 1001, (B, steps)).astype(np.int32)
    e = Cortex(path, num_heads=16, max_seqs=B, precision=PREC_FP32)
    got = [e.forward(prompts)]
    for s in range(steps):
        got.append(e.forward(forced[:, s:s + 1]))
    o = O.Oracle(path, num_heads=16)
    _, ref, _ = o.generate(prompts, steps, np.zeros((B, steps), np.float32), VARIANT_A, 0.8, 1.15,
                           forced=forced, want_logits=True)
    for s in range(steps + 1):
        err = max(rel_err(got[s][b], ref[b, s]) for b in range(B))
        assert err < TOL[PREC_FP32], (s, err)
    e.close()


@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
def test_single_sequence_long_prompt(prec, small_model, built):
    """A 90-token prompt of one sequence: 90 rows in one pass (tensor cores in
    BF16 mode) with causal attention inside the pass."""
    rng = np.random.default_rng(4)
    toks = rng.integers(0, 1000, 90).astype(np.int32)
    e = Cortex(small_model, num_heads=2, precision=prec)
    a = e.forward([toks])[0]
    b = O.Oracle(small_model, num_heads=2).forward(toks)
    assert rel_err(a, b) < TOL[prec]
    e.close()


@pytest.mark.parametrize("variant", [VARIANT_A, VARIANT_B])
@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
def test_decode_batch_ids_exact(variant, prec, small_model, built):
    """cortex_decode_batch: each sampled id equals the oracle sampler applied to
    the GPU's logits with the slot's history (every token fed so far)."""
    B, plen, steps = 66, 12, 5
    rng = np.random.default_rng(10 + variant)
    prompts = rng.integers(0, 1000, (B, plen)).astype(np.int32)
    e = Cortex(small_model, num_heads=2, max_seqs=B, precision=prec)
    e.forward(prompts, want_logits=False)
    hist = [list(p) for p in prompts]
    if variant == VARIANT_A:
        prm, args = sample_params(VARIANT_A, 0.8, 1.15), dict(T=0.8, rep=1.15)
    else:
        prm, args = sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9), dict(T=0.7, rep=1.1)
    for s in range(steps):
        lg = e.logits(np.arange(B))
        U = rng.random(B).astype(np.float32)
        ids = e.decode(U, prm)
        for b in range(B):
            if variant == VARIANT_A:
                want = O.sample_a(lg[b], hist[b], args["T"], args["rep"], U[b])
            else:
                want = O.sample_b(lg[b], hist[b], args["T"], 40, 0.9, args["rep"], U[b])
            assert ids[b] == want, (s, b)
            hist[b].append(int(ids[b]))
    e.close()


@pytest.mark.parametrize("variant", [VARIANT_A, VARIANT_B])
@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
def test_decode_steps_graph_equals_decode_batch(variant, prec, small_model, built):
    """cortex_decode_steps (one captured step replayed as a CUDA graph) gives
    the ids and final logits of the same number of cortex_decode_batch calls,
    for a slot subset in a permuted order, host and device pointers, a second
    call that reuses the graph, and the context-limit fallback."""
    B, plen = 70, 10
    rng = np.random.default_rng(30 + variant + 2 * prec)
    prompts = rng.integers(0, 1000, (B, plen)).astype(np.int32)
    prm = sample_params(VARIANT_A, 0.8, 1.15) if variant == VARIANT_A else sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9)
    slots = rng.permutation(B)[:67].astype(np.int32)
    a = Cortex(small_model, num_heads=2, max_seqs=B, precision=prec)
    g = Cortex(small_model, num_heads=2, max_seqs=B, precision=prec)
    a.forward(prompts, want_logits=False)
    g.forward(prompts, want_logits=False)
    for call, steps in enumerate((9, 6)):
        U = rng.random((steps, len(slots))).astype(np.float32)
        want = np.stack([a.decode(U[k], prm, slots=slots) for k in range(steps)])
        if call == 0:
            got = g.decode_steps(U, prm, slots=slots)
        else:
            ud = torch.from_numpy(U).cuda()
            idd = torch.zeros((steps, len(slots)), dtype=torch.int32, device="cuda")
            g.decode_steps_dev(ud, prm, idd, slots=slots)
            g.synchronize()
            got = idd.cpu().numpy()
        assert np.array_equal(got, want), call
        assert np.array_equal(g.logits(slots), a.logits(slots))
        assert [g.pos(int(s)) for s in slots] == [a.pos(int(s)) for s in slots]
    # past the context (96): the per-step fallback, same results
    steps = 96 - plen - 15 + 4
    U = rng.random((steps, len(slots))).astype(np.float32)
    want = np.stack([a.decode(U[k], prm, slots=slots) for k in range(steps)])
    got = g.decode_steps(U, prm, slots=slots)
    assert np.array_equal(got, want)
    a.close()
    g.close()


def test_decode_matches_oracle_trajectory(small_model, built):
    """Full generation (FP32): ids of GPU and oracle agree step by step while
    their logits agree to fp32 tolerance (a flip needs a near-tie)."""
    B, plen, steps = 8, 16, 24
    rng = np.random.default_rng(21)
    prompts = rng.integers(0, 1000, (B, plen)).astype(np.int32)
    U = rng.random((B, steps)).astype(np.float32)
    e = Cortex(small_model, num_heads=2, max_seqs=B)
    e.forward(prompts, want_logits=False)
    prm = sample_params(VARIANT_A, 0.25, 1.15)
    got = np.stack([e.decode(U[:, s], prm) for s in range(steps)], axis=1)
    ids, _, _ = O.Oracle(small_model, num_heads=2).generate(prompts, steps, U, VARIANT_A, 0.25, 1.15)
    agree = (got == ids).mean()
    assert agree > 0.95, agree
    e.close()


def test_run_inference_and_bridge(small_model, built):
    rng = np.random.default_rng(2)
    prompt = list(rng.integers(3, 1000, 20))
    U = rng.random(64).astype(np.float32)
    out, why = run_inference(small_model, prompt, U, max_new_tokens=30, stop_tokens=())
    assert why == "max" and len(out) == 30
    br = SnaiCortexBridge(small_model, num_heads=1)
    window = list(rng.integers(0, 1000, 30))
    tok = br.generate_next_token(window, 0.7, 40, 0.9, 1.15, u=0.37)
    o = O.Oracle(small_model, num_heads=1)
    lg = o.forward(window)
    # same id as the oracle sampler on the GPU logits, and (tolerance permitting) on the oracle's
    assert tok == O.sample_b(br.cached_c_logits, window, 0.7, 40, 0.9, 1.15, 0.37)
    assert rel_err(br.cached_c_logits, lg) < TOL[PREC_FP32]
    st = br.extract_state()
    assert len(st["tensors"]["layers"]) == 2
    br.close()


def test_device_pointer_path(small_model, built):
    """SNAI_DEVICE_PTRS: tokens, uniforms and ids in device memory, work on a
    torch stream; same ids as the host-pointer path."""
    B = 16
    rng = np.random.default_rng(8)
    prompts = rng.integers(0, 1000, (B, 10)).astype(np.int32)
    U = rng.random(B).astype(np.float32)
    prm = sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9)
    e1 = Cortex(small_model, num_heads=2, max_seqs=B)
    e1.forward(prompts, want_logits=False)
    ids_host = e1.decode(U, prm)
    e2 = Cortex(small_model, num_heads=2, max_seqs=B)
    st = torch.cuda.Stream()
    e2.set_stream(st.cuda_stream)
    with torch.cuda.stream(st):
        tok = torch.from_numpy(prompts.ravel()).cuda()
        e2.forward_dev(tok, B, 10)
        ut = torch.from_numpy(U).cuda()
        ids = torch.zeros(B, dtype=torch.int32, device="cuda")
        e2.decode_dev(ut, prm, ids)
    st.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_host)
    e1.close()
    e2.close()


@pytest.mark.parametrize("prec", [PREC_FP32, PREC_BF16])
def test_split_attention_ragged_positions(prec, model_dir, built):
    """Passes of few rows split each (row, head)'s positions over several
    CTAs and merge their partial softmax terms.  Three slots at very
    different positions (899, 499, 36: some splits of the short rows are
    empty) and one slot at position 0, then one more token each, against
    the oracle at every step (a one-row pass, a two-row and a four-row
    pass)."""
    path = make_model(model_dir, "split.snai", 2000, 128, 1024, 2, seed=51)
    lens = [899, 499, 36, 0]
    rng = np.random.default_rng(60 + prec)
    toks = [rng.integers(0, 2000, n + 3).astype(np.int32) for n in lens]
    e = Cortex(path, num_heads=2, max_seqs=4, precision=prec)
    refs = []
    for s, n in enumerate(lens):
        o = O.Oracle(path, num_heads=2)
        r = [o.forward(toks[s][:n]) if n else None]
        for i in range(3):
            r.append(o.forward(toks[s][n + i:n + i + 1]))
        refs.append(r)
        o.close()
        if n:
            e.forward([toks[s][:n]], slots=[s], want_logits=False)
    tol = TOL[prec]  # the prompts ran through the tensor cores in BF16 mode
    for group in ([0], [1, 2], [0, 1, 2, 3]):
        t = np.asarray([[toks[s][e.pos(s)]] for s in group], dtype=np.int32)
        got = e.forward(t, slots=np.asarray(group, dtype=np.int32))
        for j, s in enumerate(group):
            k = e.pos(s) - lens[s]  # tokens fed after the prompt
            assert rel_err(got[j], refs[s][k]) < tol, (group, s, k)
    e.close()


@pytest.mark.parametrize("dim", [512, 1024])
def test_pass_kernel_bits_equal_kernel_per_stage(dim, model_dir, built):
    """FP32 decode passes of one and two rows run as one persistent kernel
    (weights streamed through a shared-memory ring, grid barriers between
    the stages).  Its arithmetic is the per-stage kernels' operation for
    operation, so its logits equal those of an engine with the persistent
    kernel off (SNAI_PASS_KERNEL=0) bit for bit, and the oracle's within the
    fp32 tolerance, over a few steps at positions up to ~700.  (The
    persistent kernel is opt-in, SNAI_PASS_KERNEL=1.)"""
    import os
    path = make_model(model_dir, f"pass{dim}.snai", 2000, dim, 1024, 2, seed=61)
    heads = dim // 64
    rng = np.random.default_rng(dim)
    prompts = rng.integers(0, 2000, (2, 700)).astype(np.int32)
    steps = rng.integers(0, 2000, (2, 4)).astype(np.int32)
    engines = []
    for flag in ("1", "0"):
        os.environ["SNAI_PASS_KERNEL"] = flag
        try:
            engines.append(Cortex(path, num_heads=heads, max_seqs=2, precision=PREC_FP32))
        finally:
            del os.environ["SNAI_PASS_KERNEL"]
    fused, staged = engines
    oracles = [O.Oracle(path, num_heads=heads) for _ in range(2)]
    for e in engines:
        e.forward(prompts, want_logits=False)
    for s in range(2):
        oracles[s].forward(prompts[s])
    for k in range(4):
        group = [0] if k % 2 == 0 else [0, 1]
        t = steps[group, k:k + 1]
        a = fused.forward(t, slots=np.asarray(group, np.int32))
        b = staged.forward(t, slots=np.asarray(group, np.int32))
        assert np.array_equal(a, b), (k, float(np.abs(a - b).max()))
        for j, s in enumerate(group):
            assert rel_err(a[j], oracles[s].forward(t[j])) < TOL[PREC_FP32]
    # a decode step (sampler, then the one-row pass) through both engines
    prm = sample_params(VARIANT_A, 0.8, 1.15)
    u = np.asarray([0.3], np.float32)
    assert np.array_equal(fused.decode(u, prm, slots=[1]), staged.decode(u, prm, slots=[1]))
    assert np.array_equal(fused.logits([1]), staged.logits([1]))
    for e in engines:
        e.close()
    for o in oracles:
        o.close()
