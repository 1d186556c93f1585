"""CPU checks of the oracle's training step (core/cortex.nim:565-822).

The reference ships no training fixtures, so the restatement is pinned here
by (1) central finite differences of an independent float64 numpy forward
pass and loss, against the oracle's backpropagated gradients, and (2) a
numpy float32 restatement of the clip and Adam (core/cortex.nim:145-258),
bit for bit.
"""
import numpy as np
import pytest

import oracle as O
from snai_b200 import modelgen

TYPES = (12, 13, 14, 15, 16, 17, 10, 11)


def weights64(o):
    W = {(-1, t): o.tensor(-1, t).astype(np.float64) for t in (0, 1, 2)}
    for l in range(o.layers):
        for t in TYPES:
            W[(l, t)] = o.tensor(l, t).astype(np.float64)
    return W


def loss64(W, tokens, targets, D, L, heads, hs):
    """Sum over positions of -ln softmax(logits)[target], float64, every
    position at once (causal attention, RoPE at the row's position)."""
    V = W[(-1, 0)].size // D
    tok = np.where((tokens < 0) | (tokens >= V), 0, tokens)
    tgt = np.where((targets < 0) | (targets >= V), 0, targets)
    M = len(tok)
    E = W[(-1, 0)].reshape(V, D)
    h = E[tok].copy()
    pos = np.arange(M, dtype=np.float64)[:, None]
    i = np.arange(0, hs, 2, dtype=np.float64)
    theta = pos / (10000.0 ** (i / hs))[None, :]
    c, s = np.cos(theta), np.sin(theta)

    def rope(x):
        x = x.copy()
        for hh in range(D // hs):
            a = x[:, hh * hs:(hh + 1) * hs:2].copy()
            b = x[:, hh * hs + 1:(hh + 1) * hs:2].copy()
            x[:, hh * hs:(hh + 1) * hs:2] = a * c - b * s
            x[:, hh * hs + 1:(hh + 1) * hs:2] = a * s + b * c
        return x

    def rms(x, w):
        return x / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-5) * w[None, :]

    mask = np.tril(np.ones((M, M), dtype=bool))
    for l in range(L):
        n = rms(h, W[(l, 10)])
        q = rope(n @ W[(l, 12)].reshape(D, D).T)
        k = rope(n @ W[(l, 13)].reshape(D, D).T)
        v = n @ W[(l, 14)].reshape(D, D).T
        att = np.zeros_like(h)
        for hh in range(heads):
            sl = slice(hh * hs, (hh + 1) * hs)
            sc = q[:, sl] @ k[:, sl].T / np.sqrt(hs)
            sc = np.where(mask, sc, -np.inf)
            p = np.exp(sc - sc.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            att[:, sl] = p @ v[:, sl]
        h = h + att @ W[(l, 15)].reshape(D, D).T
        n = rms(h, W[(l, 11)])
        u = n @ W[(l, 16)].reshape(4 * D, D).T
        u = u / (1.0 + np.exp(-u))
        h = h + u @ W[(l, 17)].reshape(D, 4 * D).T
    n = rms(h, W[(-1, 2)])
    lg = n @ W[(-1, 1)].reshape(V, D).T
    lg = lg - lg.max(axis=1, keepdims=True)
    lp = lg - np.log(np.exp(lg).sum(axis=1, keepdims=True))
    return -lp[np.arange(M), tgt].sum()


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("train") / "tiny.snai")
    modelgen.random_model(p, 37, 16, 12, 2, seed=11, std=0.3)
    return p


def test_oracle_gradients_match_finite_differences(tiny):
    o = O.Oracle(tiny, num_heads=2)
    rng = np.random.default_rng(5)
    M = 9
    x = rng.integers(0, 37, M).astype(np.int32)
    x[3] = x[7] = x[1]  # a repeated token: its embedding gradient sums positions
    x[5] = 99           # out of range: reads row 0
    y = rng.integers(0, 37, M).astype(np.int32)
    loss = o.train_grads(x, y)
    W = weights64(o)
    D, L, hs = o.dim, o.layers, o.head_size
    heads = 2
    base = loss64(W, x, y, D, L, heads, hs)
    assert abs(loss * M - base) <= 1e-4 * abs(base)
    eps = 1e-5
    checked = 0
    for key in list(W):
        g = o.tensor(key[0], key[1], "grad").astype(np.float64)
        idx = list(np.argsort(-np.abs(g))[:3]) + list(rng.integers(0, g.size, 3))
        for j in idx:
            Wp = dict(W)
            a = W[key].copy()
            a[j] += eps
            Wp[key] = a
            lp = loss64(Wp, x, y, D, L, heads, hs)
            a[j] -= 2 * eps
            lm = loss64(Wp, x, y, D, L, heads, hs)
            fd = (lp - lm) / (2 * eps)
            assert abs(fd - g[j]) <= 2e-3 * np.abs(g).max() + 2e-3 * abs(fd), (key, j, fd, g[j])
            checked += 1
    assert checked >= 6 * len(W)
    o.close()


def adam_f32(w, m, v, g, lr, t, scale, sparse, clip):
    """core/cortex.nim:145-160 and the clip factor of :255-258, element-wise
    in float32 with the reference's operation order."""
    f = np.float32
    w, m, v = w.copy(), m.copy(), v.copy()
    b1, b2 = f(0.9), f(0.999)
    b1t = f(1.0) - np.power(b1, f(t), dtype=np.float32)
    b2t = f(1.0) - np.power(b2, f(t), dtype=np.float32)
    gg = g * f(clip) if clip is not None else g.copy()
    grad = gg / f(scale)
    ok = ~(np.isnan(grad) | (grad > 9999) | (grad < -9999))
    if sparse:
        ok &= grad != 0
    m2 = b1 * m + (f(1.0) - b1) * grad
    v2 = b2 * v + (f(1.0) - b2) * grad * grad
    w2 = w - (f(lr) * (m2 / b1t)) / (np.sqrt(v2 / b2t) + f(1e-8))
    return np.where(ok, w2, w), np.where(ok, m2, m), np.where(ok, v2, v)


@pytest.mark.parametrize("clipped", [False, True])
def test_oracle_adam_and_clip_bit_exact(tiny, clipped):
    o = O.Oracle(tiny, num_heads=2)
    rng = np.random.default_rng(7)
    keys = [(-1, 0), (-1, 1), (-1, 2)] + [(l, t) for l in range(o.layers) for t in TYPES]
    G = {}
    for k in keys:
        n = o.tensor_size(*k)
        g = (rng.standard_normal(n) * (0.05 if clipped else 1e-3)).astype(np.float32)
        if k == (-1, 0):
            g[: n // 2] = 0  # embedding rows without gradient keep their moments
        G[k] = g
        o.set_tensor(k[0], k[1], g, "grad")
    W0 = {k: o.tensor(k[0], k[1]) for k in keys}
    total = np.float32(0)  # calcL2Sq per tensor (:218-226), summed in clipGlobalGradientNorm's order
    for k in keys[:3] + [(l, t) for l in range(o.layers) for t in (12, 13, 14, 15, 16, 17, 10, 11)]:
        part = np.float32(0)
        for val in G[k]:
            part = np.float32(part + np.float32(val * val))
        total = np.float32(total + part)
    gn = np.float32(np.sqrt(total))
    assert (gn > 1) == clipped
    clip = np.float32(np.float32(1.0) / gn) if clipped else None
    lr, scale = 0.01, 9.0
    o.train_apply(lr, scale)
    assert o.adam_steps == 1
    for k in keys:
        z = np.zeros_like(G[k])
        w, m, v = adam_f32(W0[k], z, z, G[k], lr, 1, scale, k == (-1, 0), clip)
        assert np.array_equal(o.tensor(k[0], k[1]), w), k
        assert np.array_equal(o.tensor(k[0], k[1], "m"), m), k
        assert np.array_equal(o.tensor(k[0], k[1], "v"), v), k
    o.close()


def test_oracle_train_step_zero_tokens_and_ctx_cut(tiny):
    o = O.Oracle(tiny, num_heads=2)
    assert o.train_step([], [], 0.1) == 0.0
    assert o.adam_steps == 0
    x = np.arange(20, dtype=np.int32) % 37
    loss = o.train_step(x, (x + 1) % 37, 0.01)  # 20 > ctx 12: the first 12 are used
    o2 = O.Oracle(tiny, num_heads=2)
    assert loss == o2.train_step(x[:12], ((x + 1) % 37)[:12], 0.01)
    assert o.adam_steps == 1
    o.close()
    o2.close()
