"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (snai_oracle.c).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference legs, never by the product (snai_b200/).  Parity unpinned: the
reference (Nim engine, PHP host) cannot be built here and ships no golden
vectors; see snai_oracle.c.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_c = ctypes
_vp = _c.c_void_p
_SIGS = {
    "oracle_init": (_vp, [_c.c_int] * 5),
    "oracle_load_stream": (_vp, [_c.c_char_p, _c.c_int]),
    "oracle_forward": (None, [_vp, _vp, _c.c_int, _vp]),
    "oracle_reset_cache": (None, [_vp]),
    "oracle_get_pos": (_c.c_int, [_vp]),
    "oracle_get_heads": (_c.c_int, [_vp]),
    "oracle_get_head_size": (_c.c_int, [_vp]),
    "oracle_get_vocab": (_c.c_int, [_vp]),
    "oracle_get_ctx": (_c.c_int, [_vp]),
    "oracle_get_dim": (_c.c_int, [_vp]),
    "oracle_get_layers": (_c.c_int, [_vp]),
    "oracle_free": (None, [_vp]),
    "oracle_load_layer": (None, [_vp, _c.c_int, _c.c_int, _vp, _c.c_int]),
    "oracle_extract_layer": (None, [_vp, _c.c_int, _c.c_int, _vp, _c.c_int]),
    "oracle_sample_a": (_c.c_int, [_vp, _c.c_int, _vp, _c.c_int, _c.c_double, _c.c_double, _c.c_float, _c.c_int]),
    "oracle_sample_b": (_c.c_int, [_vp, _c.c_int, _vp, _c.c_int, _c.c_double, _c.c_int, _c.c_double, _c.c_double,
                                   _c.c_float, _c.c_int, _vp]),
    "oracle_exp_contract": (None, [_vp, _vp, _c.c_long]),
    "oracle_exp_libm": (None, [_vp, _vp, _c.c_long]),
    "oracle_generate": (_c.c_double, [_vp, _c.c_int, _vp, _c.c_int, _c.c_int, _vp, _c.c_int, _c.c_double,
                                      _c.c_double, _c.c_int, _c.c_double, _c.c_int, _vp, _vp, _vp, _c.c_int]),
    "oracle_bench_decode": (_c.c_double, [_vp, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_double, _c.c_double,
                                          _c.c_int, _c.c_double, _c.c_uint, _c.c_int]),
    "oracle_batch_new": (_vp, [_vp, _c.c_int, _c.c_int, _c.c_uint]),
    "oracle_batch_free": (None, [_vp]),
    "oracle_batch_step": (_c.c_double, [_vp, _c.c_int, _c.c_double, _c.c_double, _c.c_int, _c.c_double,
                                        _c.c_int]),
    "oracle_train_step": (_c.c_float, [_vp, _vp, _vp, _c.c_int, _c.c_float]),
    "oracle_train_grads": (_c.c_float, [_vp, _vp, _vp, _c.c_int]),
    "oracle_train_apply": (None, [_vp, _c.c_float, _c.c_float]),
    "oracle_train_tensor_get": (None, [_vp, _c.c_int, _c.c_int, _c.c_int, _vp, _c.c_int]),
    "oracle_train_tensor_set": (None, [_vp, _c.c_int, _c.c_int, _c.c_int, _vp, _c.c_int]),
    "oracle_adam_t": (_c.c_int, [_vp]),
    "oracle_sample_rows": (_c.c_double, [_vp, _c.c_int, _c.c_int, _vp, _c.c_int, _vp, _c.c_int, _c.c_double,
                                         _c.c_double, _c.c_int, _c.c_double, _c.c_int, _vp, _c.c_int]),
}

_lib = None


def build():
    """Compiles liboracle.so from snai_oracle.c (make)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _p(a):
    return a.ctypes.data_as(_vp)


class Oracle:
    """One model + one sequence, the shape of the reference's CortexState."""

    def __init__(self, path=None, num_heads=1, shape=None):
        L = lib()
        if path is not None:
            self.h = L.oracle_load_stream(str(path).encode(), int(num_heads))
        else:
            self.h = L.oracle_init(*shape, int(num_heads))
        if not self.h:
            raise RuntimeError("oracle could not load the model")
        self.vocab = L.oracle_get_vocab(self.h)
        self.ctx = L.oracle_get_ctx(self.h)
        self.dim = L.oracle_get_dim(self.h)
        self.layers = L.oracle_get_layers(self.h)

    def close(self):
        if self.h:
            lib().oracle_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, logits=None):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.vocab, dtype=np.float32) if logits is None else logits
        lib().oracle_forward(self.h, _p(t), len(t), _p(out))
        return out

    def reset(self):
        lib().oracle_reset_cache(self.h)

    @property
    def pos(self):
        return lib().oracle_get_pos(self.h)

    @property
    def head_size(self):
        return lib().oracle_get_head_size(self.h)

    def generate(self, prompts, steps, uniforms, variant, temperature, rep, top_k=40, top_p=0.9, exp_mode=1,
                 forced=None, want_logits=False, nthreads=8):
        """src/snai_inference.php:113-215 loop over many sequences (threads)."""
        P = np.ascontiguousarray(prompts, dtype=np.int32)
        n, plen = P.shape
        U = np.ascontiguousarray(uniforms, dtype=np.float32).reshape(n, steps)
        ids = np.zeros((n, steps), dtype=np.int32)
        F = None if forced is None else np.ascontiguousarray(forced, dtype=np.int32).reshape(n, steps)
        lg = np.zeros((n, steps + 1, self.vocab), dtype=np.float32) if want_logits else None
        secs = lib().oracle_generate(self.h, n, _p(P), plen, steps, _p(U), variant, temperature, rep, top_k, top_p,
                                     exp_mode, None if F is None else _p(F), _p(ids), None if lg is None else _p(lg),
                                     nthreads)
        return ids, lg, secs

    # -- training (core/cortex.nim:565-822) ----------------------------------
    _WHICH = {"grad": 0, "m": 1, "v": 2}

    def tensor_size(self, layer, ttype):
        v, dim = self.vocab, self.dim
        f = 4 * dim
        return {0: v * dim, 1: v * dim, 2: dim, 10: dim, 11: dim, 12: dim * dim, 13: dim * dim, 14: dim * dim,
                15: dim * dim, 16: f * dim, 17: f * dim}[ttype]

    def train_step(self, inputs, targets, lr):
        a = np.ascontiguousarray(inputs, dtype=np.int32)
        b = np.ascontiguousarray(targets, dtype=np.int32)
        return float(lib().oracle_train_step(self.h, _p(a), _p(b), len(a), float(lr)))

    def train_grads(self, inputs, targets):
        a = np.ascontiguousarray(inputs, dtype=np.int32)
        b = np.ascontiguousarray(targets, dtype=np.int32)
        return float(lib().oracle_train_grads(self.h, _p(a), _p(b), len(a)))

    def train_apply(self, lr, scale):
        lib().oracle_train_apply(self.h, float(lr), float(scale))

    @property
    def adam_steps(self):
        return lib().oracle_adam_t(self.h)

    def tensor(self, layer, ttype, which="weight"):
        n = self.tensor_size(layer, ttype)
        out = np.zeros(n, dtype=np.float32)
        if which == "weight":
            lib().oracle_extract_layer(self.h, layer, ttype, _p(out), n)
        else:
            lib().oracle_train_tensor_get(self.h, self._WHICH[which], layer, ttype, _p(out), n)
        return out

    def set_tensor(self, layer, ttype, values, which="weight"):
        a = np.ascontiguousarray(values, dtype=np.float32)
        if which == "weight":
            lib().oracle_load_layer(self.h, layer, ttype, _p(a), a.size)
        else:
            lib().oracle_train_tensor_set(self.h, self._WHICH[which], layer, ttype, _p(a), a.size)

    def batch(self, nseq, start_pos, seed=1):
        """A persistent batch of sequences for step-by-step CPU timing."""
        return OracleBatch(self, nseq, start_pos, seed)

    def bench_decode(self, nseq, start_pos, steps, variant, temperature, rep, top_k, top_p, seed, nthreads):
        return lib().oracle_bench_decode(self.h, nseq, start_pos, steps, variant, temperature, rep, top_k, top_p,
                                         seed, nthreads)


class OracleBatch:
    def __init__(self, oracle, nseq, start_pos, seed):
        self.o = oracle  # keeps the model alive
        self.h = lib().oracle_batch_new(oracle.h, nseq, start_pos, seed)
        self.nseq = nseq

    def step(self, variant, temperature, rep, top_k=40, top_p=0.9, nthreads=1):
        """One decode step for every sequence; returns wall seconds."""
        return lib().oracle_batch_step(self.h, variant, temperature, rep, top_k, top_p, nthreads)

    def close(self):
        if self.h:
            lib().oracle_batch_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_a(logits, hist, temperature, rep, u, exp_mode=1):
    """src/snai_inference.php:151-195 on one row (the row is not modified)."""
    row = np.array(logits, dtype=np.float32, copy=True)
    h = np.ascontiguousarray(hist, dtype=np.int32)
    return lib().oracle_sample_a(_p(row), len(row), _p(h), len(h), temperature, rep, u, exp_mode)


def sample_b(logits, in_tokens, temperature, top_k, top_p, rep, u, exp_mode=1, want_order=False):
    """src/tensor_ffi_adapter.php:168-204 on one row."""
    row = np.ascontiguousarray(logits, dtype=np.float32)
    t = np.ascontiguousarray(in_tokens, dtype=np.int32)
    order = np.zeros(max(1, min(top_k, len(row))), dtype=np.int32) if want_order else None
    r = lib().oracle_sample_b(_p(row), len(row), _p(t), len(t), temperature, top_k, top_p, rep, u, exp_mode,
                              None if order is None else _p(order))
    return (r, order) if want_order else r


def sample_rows(logits, hist, uniforms, variant, temperature, rep, top_k=40, top_p=0.9, exp_mode=1, nthreads=8):
    """Samples every row of logits [R, V] with history hist [R, H]; returns
    (ids, rows per second)."""
    L = np.ascontiguousarray(logits, dtype=np.float32)
    R, V = L.shape
    H = np.ascontiguousarray(hist, dtype=np.int32).reshape(R, -1)
    U = np.ascontiguousarray(uniforms, dtype=np.float32)
    out = np.zeros(R, dtype=np.int32)
    rate = lib().oracle_sample_rows(_p(L), R, V, _p(H), H.shape[1], _p(U), variant, temperature, rep, top_k, top_p,
                                    exp_mode, _p(out), nthreads)
    return out, rate


def exp_contract(x):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    lib().oracle_exp_contract(_p(x), _p(y), len(x))
    return y


def exp_libm(x):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    lib().oracle_exp_libm(_p(x), _p(y), len(x))
    return y
