"""CPU tests of the oracle (the checker) against hand-derived known answers,
an independent transliteration of the PHP samplers, and a float64 numpy
restatement of the forward step.  No GPU."""
import json
import math
import os

import numpy as np
import pytest

import oracle as O
from snai_b200 import modelgen
from conftest import make_model, rel_err

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sampler_kats.json")


def load_kats():
    with open(GOLDEN) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        c["logits"] = [float("-inf") if x == "-inf" else x for x in c["logits"]]
    return cases


@pytest.mark.parametrize("case", load_kats(), ids=lambda c: c["name"])
@pytest.mark.parametrize("exp_mode", [0, 1])
def test_sampler_kats(case, exp_mode, built):
    L = np.asarray(case["logits"], dtype=np.float32)
    if case["variant"] == 0:
        got = O.sample_a(L, case["hist"], case["T"], case["rep"], case["u"], exp_mode)
    else:
        got = O.sample_b(L, case["hist"], case["T"], case["top_k"], case["top_p"], case["rep"], case["u"], exp_mode)
    assert got == case["expect"], case["why"]


# --- a second, independent restatement: the PHP code transliterated -------

def f32(x):
    return float(np.float32(x))


def php_variant_a(logits, history, T, rep, u, exp=math.exp):
    """src/snai_inference.php:140-195, line by line (PHP floats are doubles;
    writes into the FFI float buffer round to float)."""
    c = [float(x) for x in np.asarray(logits, dtype=np.float32)]
    V = len(c)
    best = 0
    for v in range(V):
        c[v] = f32(c[v] / T)
    for t in dict.fromkeys(history):  # array_unique keeps first occurrences
        if 0 <= t < V:
            if c[t] > 0:
                c[t] = f32(c[t] / rep)
            else:
                c[t] = f32(c[t] * rep)
    mx = -math.inf
    for v in range(V):
        if c[v] > mx:
            mx = c[v]
            if T <= 0.01:
                best = v
    if T > 0.01:
        probs = []
        s = 0.0
        for v in range(V):
            p = exp(c[v] - mx)
            probs.append(p)
            s += p
        r = u * s
        cum = 0.0
        for v in range(V):
            cum += probs[v]
            if cum >= r:
                best = v
                break
    return best


def php_variant_b(logits, input_tokens, T, top_k, top_p, rep, u, exp=math.exp):
    """src/tensor_ffi_adapter.php:168-204."""
    c = [float(x) for x in np.asarray(logits, dtype=np.float32)]
    inset = set(input_tokens)
    vals = [(c[i] - rep) if i in inset else c[i] for i in range(len(c))]
    order = sorted(range(len(c)), key=lambda i: (-vals[i], i))[:top_k]  # stable arsort
    if T < 0.01:
        return order[0]
    probs = [exp(vals[i] / T) for i in order]
    s = 0.0
    for p in probs:
        s += p
    cum = 0.0
    filt = []
    for i, p in zip(order, probs):
        pn = p / s
        filt.append((i, pn))
        cum += pn
        if cum >= top_p:
            break
    r = u * cum
    cc = 0.0
    for i, p in filt:
        cc += p
        if r <= cc:
            return i
    return filt[0][0]


def contract_exp(x):
    return float(O.exp_contract(np.asarray([x]))[0])


def random_rows(rng, n, V):
    rows = []
    for i in range(n):
        kind = i % 4
        if kind == 0:
            L = rng.normal(0, 4, V)
        elif kind == 1:
            L = rng.normal(0, 0.3, V)
        elif kind == 2:
            L = np.round(rng.normal(0, 2, V) * 4) / 4  # many exact ties
        else:
            L = rng.normal(0, 4, V)
            L[rng.random(V) < 0.01] += 12.0
        rows.append(L.astype(np.float32))
    return rows


@pytest.mark.parametrize("exp_mode", [0, 1])
def test_oracle_samplers_match_transliteration(exp_mode, built):
    rng = np.random.default_rng(11)
    exp = math.exp if exp_mode == 0 else contract_exp
    V = 300
    for i, L in enumerate(random_rows(rng, 24, V)):
        hist = list(rng.integers(-2, V + 2, 40))
        u = float(np.float32(rng.random()))
        for T in (0.005, 0.25, 0.8, 1.7):
            a = O.sample_a(L, hist, T, 1.15, u, exp_mode)
            assert a == php_variant_a(L, hist, T, 1.15, u, exp), (i, T)
        for (T, k, p) in ((0.0, 40, 0.9), (0.7, 40, 0.9), (0.7, 50, 0.95), (1.3, 5, 0.5), (0.7, 400, 1.0)):
            b = O.sample_b(L, hist, T, k, p, 1.1, u, exp_mode)
            assert b == php_variant_b(L, hist, T, k, p, 1.1, u, exp), (i, T, k, p)


def test_oracle_samplers_match_transliteration_benchmark_vocab(built):
    """The same check at the benchmark's vocabulary (V=16384), the sampler
    benchmark's settings, one row of each kind."""
    rng = np.random.default_rng(12)
    V = 16384
    for i, L in enumerate(random_rows(rng, 4, V)):
        hist = list(rng.integers(0, V, 256))
        u = float(np.float32(rng.random()))
        for exp_mode, exp in ((0, math.exp), (1, contract_exp)):
            assert O.sample_a(L, hist, 0.7, 1.15, u, exp_mode) == php_variant_a(L, hist, 0.7, 1.15, u, exp), i
            b = O.sample_b(L, hist, 0.7, 50, 0.95, 1.15, u, exp_mode)
            assert b == php_variant_b(L, hist, 0.7, 50, 0.95, 1.15, u, exp), i


def test_exp_contract_accuracy(built):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-745, 709, 300000), rng.uniform(-60, 0, 300000), rng.uniform(-1, 1, 100000)])
    a, b = O.exp_contract(x), O.exp_libm(x)
    ok = (b > 0) & np.isfinite(b)
    ulps = np.abs(a[ok].view(np.int64) - b[ok].view(np.int64))
    assert ulps.max() <= 1
    special = np.array([0.0, -0.0, np.inf, -np.inf, 710.0, -746.0, 1e-300, -1e-300])
    ys = O.exp_contract(special)
    assert ys[0] == 1.0 and ys[1] == 1.0 and ys[2] == np.inf and ys[3] == 0.0
    assert ys[4] == np.inf and ys[5] == 0.0 and ys[6] == 1.0 and ys[7] == 1.0
    assert np.isnan(O.exp_contract(np.array([np.nan]))[0])


# --- forward -------------------------------------------------------------

def np_forward(h, t, tokens, heads):
    """float64 numpy restatement of core/cortex.nim:487-563 for one sequence
    from position 0; returns logits of the last token."""
    V, D, L, ctx = h["vocab_size"], h["hidden_dim"], h["num_layers"], h["ctx_size"]
    F = 4 * D
    hs = D // max(1, heads)
    hs -= hs % 2
    hs = max(hs, 2)
    nh = max(1, heads)
    kc = np.zeros((L, ctx, D))
    vc = np.zeros((L, ctx, D))

    def rms(x, w):
        return x / np.sqrt(np.mean(x * x) + 1e-5) * w

    def rope(vec, pos):
        vec = vec.copy()
        for hh in range(D // hs):
            for i in range(0, hs, 2):
                fr = 1.0 / 10000.0 ** (i / hs)
                th = pos * fr
                a, b = vec[hh * hs + i], vec[hh * hs + i + 1]
                vec[hh * hs + i] = a * math.cos(th) - b * math.sin(th)
                vec[hh * hs + i + 1] = a * math.sin(th) + b * math.cos(th)
        return vec

    g = lambda k: t[k].astype(np.float64)
    logits = None
    for pos, tok in enumerate(tokens):
        tok = tok if 0 <= tok < V else 0
        x = g("embeddings")[tok].copy()
        for l in range(L):
            n = rms(x, g(f"{l}.rms_att"))
            q = rope(g(f"{l}.w_q") @ n, pos)
            kc[l, pos] = rope(g(f"{l}.w_k") @ n, pos)
            vc[l, pos] = g(f"{l}.w_v") @ n
            att = np.zeros(D)
            for hh in range(nh):
                o = hh * hs
                s = kc[l, :pos + 1, o:o + hs] @ q[o:o + hs] / math.sqrt(hs)
                m = max(-9999.0, s.max())
                e = np.exp(s - m)
                att[o:o + hs] = (e / e.sum()) @ vc[l, :pos + 1, o:o + hs]
            x = x + g(f"{l}.w_o") @ att
            n = rms(x, g(f"{l}.rms_ffn"))
            u = g(f"{l}.w_up")[:F] @ n
            u = u / (1 + np.exp(-u))
            x = x + g(f"{l}.w_down") @ u
        logits = g("w_out") @ rms(x, g("rms_final"))
    return logits


@pytest.mark.parametrize("heads", [1, 2, 3])
def test_oracle_forward_matches_numpy(heads, model_dir, built):
    p = make_model(model_dir, "tiny.snai", 61, 16, 12, 2, seed=5, std=0.3)
    h, t = modelgen.read_model(p)
    rng = np.random.default_rng(heads)
    toks = list(rng.integers(-3, 64, 9))  # includes out-of-range ids (read as 0)
    o = O.Oracle(p, num_heads=heads)
    lg = o.forward(toks)
    ref = np_forward(h, t, toks, heads)
    assert rel_err(lg, ref) < 2e-5


@pytest.mark.parametrize("dim,heads", [(1024, 16), (512, 8)])
def test_oracle_forward_matches_numpy_headline_shape(dim, heads, model_dir, built):
    """The benchmarked models' widths and heads (d=1024 with 16 heads and
    d=512 with 8, heads of 64, two layers, N(0, 0.02) weights; a small
    vocabulary) over 40 positions."""
    p = make_model(model_dir, f"d{dim}.snai", 512, dim, 48, 2, seed=9, std=0.02)
    h, t = modelgen.read_model(p)
    toks = list(np.random.default_rng(9).integers(0, 512, 40))
    o = O.Oracle(p, num_heads=heads)
    lg = o.forward(toks)
    assert rel_err(lg, np_forward(h, t, toks, heads)) < 2e-5


def test_oracle_one_position_attention_returns_v(model_dir, built):
    """At position 0 softmax has one term, so attention returns v exactly;
    with Wo = I and a zero MLP, h = e + Wv*RMSNorm(e)."""
    V, D = 40, 16
    o = O.Oracle(shape=(V, D, 8, 1), num_heads=2)
    rng = np.random.default_rng(0)
    emb = rng.normal(0, 1, (V, D)).astype(np.float32)
    wv = rng.normal(0, 0.3, (D, D)).astype(np.float32)
    wout = rng.normal(0, 0.3, (V, D)).astype(np.float32)
    L = O.lib()
    for layer, typ, arr in [(-1, 0, emb), (-1, 1, wout), (0, 14, wv), (0, 15, np.eye(D, dtype=np.float32))]:
        a = np.ascontiguousarray(arr.ravel())
        L.oracle_load_layer(o.h, layer, typ, a.ctypes.data, a.size)
    lg = o.forward([7])
    e = emb[7].astype(np.float64)
    n = e / np.sqrt(np.mean(e * e) + 1e-5)
    h = e + wv.astype(np.float64) @ n
    ref = wout.astype(np.float64) @ (h / np.sqrt(np.mean(h * h) + 1e-5))
    assert rel_err(lg, ref) < 1e-5


def test_oracle_ctx_cutoff_and_reset(model_dir, built):
    p = make_model(model_dir, "tiny.snai", 61, 16, 12, 2, seed=5, std=0.3)
    o = O.Oracle(p, num_heads=2)
    o.forward(list(range(10)))
    assert o.pos == 10
    sentinel = np.full(o.vocab, 7.0, dtype=np.float32)
    o.forward([1, 2, 3, 4], logits=sentinel)  # positions 10, 11, then ctx
    assert o.pos == 12
    assert np.all(sentinel == 7.0)  # last token not processed: buffer untouched
    o.reset()
    assert o.pos == 0


def test_file_format(model_dir, built, tmp_path):
    p = make_model(model_dir, "tiny.snai", 61, 16, 12, 2, seed=5, std=0.3)
    assert os.path.getsize(p) == modelgen.expected_size(61, 16, 64, 2)
    hdr = modelgen.read_header(p)
    assert hdr == {"vocab_size": 61, "hidden_dim": 16, "ffn_dim": 64, "ctx_size": 12, "num_layers": 2}
    bad = tmp_path / "bad.snai"
    data = bytearray(open(p, "rb").read())
    data[:8] = b"SNAI_V3\x00"
    bad.write_bytes(bytes(data))
    assert modelgen.read_header(str(bad)) is None
    assert not O.lib().oracle_load_stream(str(bad).encode(), 1)
    short = tmp_path / "short.snai"
    short.write_bytes(open(p, "rb").read()[:-4])
    assert not O.lib().oracle_load_stream(str(short).encode(), 1)
