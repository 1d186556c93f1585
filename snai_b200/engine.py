"""Python face of libcortex.so: the reference's host-side callers, re-expressed.

`Cortex` wraps one engine state (many independent sequence slots on one GPU).
`SnaiCortexBridge` mirrors the PHP class of src/tensor_ffi_adapter.php:15-206
method for method, and `run_inference` the driver loop of
src/snai_inference.php:113-215.  Everything numeric happens in the library;
this module only moves arguments across the C ABI.
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import CortexError, SampleParams, check, load
from .modelgen import read_header

VARIANT_A = 0  # src/snai_inference.php sampler
VARIANT_B = 1  # src/tensor_ffi_adapter.php generate_next_token sampler


def sample_params(variant, temperature, rep_penalty, top_k=40, top_p=0.9, nan_guard=None):
    if nan_guard is None:
        nan_guard = 1 if variant == VARIANT_A else 0
    return SampleParams(int(variant), float(temperature), float(rep_penalty), int(top_k), float(top_p),
                        int(nan_guard))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Cortex:
    """One decode engine on one GPU with `max_seqs` sequence slots."""

    def __init__(self, path=None, num_heads=1, max_seqs=1, device=0, precision=_lib.PREC_FP32, shape=None):
        self.lib = load()
        if path is not None:
            h = self.lib.cortex_load_stream_ex(str(path).encode(), int(num_heads), int(max_seqs), int(device),
                                               int(precision))
        else:
            vocab, dim, ctx, layers = shape
            h = self.lib.cortex_init_ex(vocab, dim, ctx, layers, int(num_heads), int(max_seqs), int(device),
                                        int(precision))
        if not h:
            raise CortexError(f"could not create the engine: {_lib.last_error()}")
        self.h = h
        self.vocab = self.lib.get_vocab_size(h)
        self.ctx = self.lib.get_ctx_size(h)
        self.slots = self.lib.cortex_num_slots(h)
        self.head_size = self.lib.cortex_head_size(h)
        self.heads = self.lib.cortex_num_heads(h)
        self.device = device
        self.dim = read_header(path)["hidden_dim"] if path is not None else shape[1]

    def close(self):
        if self.h:
            self.lib.cortex_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- per-slot state -----------------------------------------------------
    def reset(self, slots=None):
        if slots is None:
            check(self.lib.cortex_seq_reset(self.h, None, 0), "cortex_seq_reset")
        else:
            s = np.ascontiguousarray(slots, dtype=np.int32)
            check(self.lib.cortex_seq_reset(self.h, _ptr(s), len(s)), "cortex_seq_reset")

    def pos(self, slot=0):
        return self.lib.cortex_seq_pos(self.h, int(slot))

    # -- host-memory calls ----------------------------------------------------
    def forward(self, tokens, slots=None, want_logits=True):
        """Feeds tokens [B, n] (one row per slot); returns logits [B, V] of each
        slot's last token (rows of slots cut off by ctx keep zeros)."""
        t = np.ascontiguousarray(np.atleast_2d(tokens), dtype=np.int32)
        B, n = t.shape
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        out = np.zeros((B, self.vocab), dtype=np.float32) if want_logits else None
        check(self.lib.cortex_forward_batch(self.h, _ptr(t), B, n, None if sl is None else _ptr(sl),
                                            None if out is None else _ptr(out), _lib.HOST_PTRS),
              "cortex_forward_batch")
        return out

    def decode(self, uniforms, params, slots=None):
        """One sample+feed step for each slot; returns the sampled ids [B]."""
        u = np.ascontiguousarray(uniforms, dtype=np.float32)
        B = len(u)
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        ids = np.zeros(B, dtype=np.int32)
        check(self.lib.cortex_decode_batch(self.h, None if sl is None else _ptr(sl), B, _ptr(u),
                                           ctypes.byref(params), _ptr(ids), _lib.HOST_PTRS),
              "cortex_decode_batch")
        return ids

    def decode_steps(self, uniforms, params, slots=None):
        """len(uniforms) sample+feed steps for each slot through the graph-
        replayed decode (uniforms [steps, B]); returns the ids [steps, B]."""
        u = np.ascontiguousarray(uniforms, dtype=np.float32)
        steps, B = u.shape
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        ids = np.zeros((steps, B), dtype=np.int32)
        check(self.lib.cortex_decode_steps(self.h, None if sl is None else _ptr(sl), B, steps, _ptr(u),
                                           ctypes.byref(params), _ptr(ids), _lib.HOST_PTRS),
              "cortex_decode_steps")
        return ids

    def decode_steps_dev(self, uniforms_dev, params, ids_dev, slots=None):
        """Device-pointer decode_steps: uniforms_dev [steps, B] float32,
        ids_dev [steps, B] int32 (torch tensors)."""
        steps, B = uniforms_dev.shape
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        check(self.lib.cortex_decode_steps(self.h, None if sl is None else _ptr(sl), B, steps,
                                           ctypes.c_void_p(uniforms_dev.data_ptr()), ctypes.byref(params),
                                           ctypes.c_void_p(ids_dev.data_ptr()), _lib.DEVICE_PTRS),
              "cortex_decode_steps")

    def logits(self, slots):
        s = np.ascontiguousarray(slots, dtype=np.int32)
        out = np.zeros((len(s), self.vocab), dtype=np.float32)
        check(self.lib.cortex_get_logits(self.h, _ptr(s), len(s), _ptr(out)), "cortex_get_logits")
        return out

    # -- device-memory calls (torch CUDA tensors as plain device buffers) ----
    def set_stream(self, stream_handle):
        check(self.lib.cortex_set_stream(self.h, ctypes.c_void_p(stream_handle)), "cortex_set_stream")

    def forward_dev(self, tokens_dev, batch, n_tok, slots=None):
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        check(self.lib.cortex_forward_batch(self.h, ctypes.c_void_p(tokens_dev.data_ptr()), batch, n_tok,
                                            None if sl is None else _ptr(sl), None, _lib.DEVICE_PTRS),
              "cortex_forward_batch")

    def decode_dev(self, uniforms_dev, params, ids_dev, slots=None):
        sl = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        check(self.lib.cortex_decode_batch(self.h, None if sl is None else _ptr(sl), int(uniforms_dev.numel()),
                                           ctypes.c_void_p(uniforms_dev.data_ptr()), ctypes.byref(params),
                                           ctypes.c_void_p(ids_dev.data_ptr()), _lib.DEVICE_PTRS),
              "cortex_decode_batch")

    def synchronize(self):
        check(self.lib.cortex_synchronize(self.h), "cortex_synchronize")

    @property
    def launches(self):
        return self.lib.cortex_kernel_launches(self.h)

    def rewind(self, pos, slots=None):
        s = None if slots is None else np.ascontiguousarray(slots, dtype=np.int32)
        n = self.slots if s is None else len(s)
        check(self.lib.cortex_seq_rewind(self.h, None if s is None else _ptr(s), n, int(pos)), "cortex_seq_rewind")

    PROFILE_KINDS = ("embed", "rmsnorm", "qkv", "attention", "wo", "up", "down", "logits", "sampler", "pass")

    def profile(self, on=True):
        check(self.lib.cortex_profile_enable(self.h, 1 if on else 0), "cortex_profile_enable")

    def profile_read(self):
        """{kind: (launches, ms, algorithmic bytes, flops)}"""
        out = {}
        for k, name in enumerate(self.PROFILE_KINDS):
            n, ms, by, fl = ctypes.c_longlong(), ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
            check(self.lib.cortex_profile_read(self.h, k, ctypes.byref(n), ctypes.byref(ms), ctypes.byref(by),
                                               ctypes.byref(fl)), "cortex_profile_read")
            out[name] = (n.value, ms.value, by.value, fl.value)
        return out


    # -- training (core/cortex.nim:565-822) ------------------------------------
    def _tensor_size(self, layer, ttype):
        d, v, f = self.dim, self.vocab, 4 * self.dim
        sizes = {0: v * d, 1: v * d, 2: d, 10: d, 11: d, 12: d * d, 13: d * d, 14: d * d, 15: d * d, 16: f * d,
                 17: f * d}
        return sizes[ttype]

    def train_step(self, inputs, targets, lr):
        """cortex_train_step: one step on the sequence (slot 0); the mean loss."""
        a = np.ascontiguousarray(inputs, dtype=np.int32)
        b = np.ascontiguousarray(targets, dtype=np.int32)
        return float(self.lib.cortex_train_step(self.h, _ptr(a), _ptr(b), len(a), float(lr)))

    def train_grads(self, inputs, targets):
        """Forward + backward only; gradients stay on the device; the mean loss."""
        a = np.ascontiguousarray(inputs, dtype=np.int32)
        b = np.ascontiguousarray(targets, dtype=np.int32)
        loss = ctypes.c_float(0.0)
        check(self.lib.cortex_train_grads(self.h, _ptr(a), _ptr(b), len(a), ctypes.byref(loss)), "cortex_train_grads")
        return float(loss.value)

    def train_apply(self, lr, scale):
        check(self.lib.cortex_train_apply(self.h, float(lr), float(scale)), "cortex_train_apply")
        self.synchronize()

    def train_info(self):
        steps, cf, gn, cl = ctypes.c_int(0), ctypes.c_float(0), ctypes.c_float(0), ctypes.c_int(0)
        rc = self.lib.cortex_train_info(self.h, ctypes.byref(steps), ctypes.byref(cf), ctypes.byref(gn),
                                        ctypes.byref(cl))
        return {"adam_steps": steps.value, "clip_factor": cf.value, "grad_norm": gn.value, "clipped": bool(cl.value),
                "ok": rc == 0}

    def tensor(self, layer, ttype, which="weight"):
        """A tensor by (layer, type code): which = weight, grad, m or v."""
        n = self._tensor_size(layer, ttype)
        out = np.zeros(n, dtype=np.float32)
        if which == "weight":
            self.lib.cortex_extract_layer(self.h, layer, ttype, _ptr(out), n)
        elif which == "grad":
            self.lib.cortex_extract_grad_layer(self.h, layer, ttype, _ptr(out), n)
        else:
            self.lib.cortex_extract_adam_layer(self.h, layer, ttype, which == "v", _ptr(out), n)
        return out

    def set_tensor(self, layer, ttype, values, which="weight"):
        a = np.ascontiguousarray(values, dtype=np.float32)
        if which == "weight":
            self.lib.cortex_load_layer(self.h, layer, ttype, _ptr(a), a.size)
        elif which == "grad":
            self.lib.cortex_load_grad_layer(self.h, layer, ttype, _ptr(a), a.size)
        else:
            self.lib.cortex_load_adam_layer(self.h, layer, ttype, which == "v", _ptr(a), a.size)


class CortexGroup:
    """Engines on several GPUs in one process (cortex_group_*): `total`
    sequences split into contiguous shards, one per listed device; one file
    read, weights fanned out by peer copies; calls gathered on the host."""

    def __init__(self, path, num_heads, total, devices, precision=_lib.PREC_FP32):
        self.lib = load()
        d = np.ascontiguousarray(devices, dtype=np.int32)
        h = self.lib.cortex_group_load(str(path).encode(), int(num_heads), int(total), _ptr(d), len(d),
                                       int(precision))
        if not h:
            raise CortexError(f"could not create the group: {_lib.last_error()}")
        self.h = h
        self.total = total
        self.size = self.lib.cortex_group_size(h)
        self.vocab = self.lib.get_vocab_size(self.lib.cortex_group_engine(h, 0))
        self.load_seconds = self.lib.cortex_group_load_seconds(h)

    def shard(self, i):
        a, n = ctypes.c_int(), ctypes.c_int()
        check(self.lib.cortex_group_shard(self.h, i, ctypes.byref(a), ctypes.byref(n)), "cortex_group_shard")
        return a.value, a.value + n.value

    def engine_state(self, i):
        return self.lib.cortex_group_engine(self.h, i)

    def forward(self, tokens, want_logits=True):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros((self.total, self.vocab), dtype=np.float32) if want_logits else None
        check(self.lib.cortex_group_forward(self.h, _ptr(t), t.shape[1], None if out is None else _ptr(out)),
              "cortex_group_forward")
        return out

    def decode_steps(self, uniforms, params):
        u = np.ascontiguousarray(uniforms, dtype=np.float32)
        ids = np.zeros(u.shape, dtype=np.int32)
        check(self.lib.cortex_group_decode_steps(self.h, u.shape[0], _ptr(u), ctypes.byref(params), _ptr(ids)),
              "cortex_group_decode_steps")
        return ids

    def average(self):
        """Federated average of the engines' weights (cortex_group_average)."""
        check(self.lib.cortex_group_average(self.h), "cortex_group_average")

    def close(self):
        if self.h:
            self.lib.cortex_group_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_device(logits_dev, uniforms_dev, params, hist_dev=None, hist_len_dev=None, out_dev=None, stream=0):
    """Stateless GPU sampler over device tensors (cortex_sample)."""
    lib = load()
    rows, vocab = logits_dev.shape
    ld = logits_dev.stride(0)
    hist_cols = 0 if hist_dev is None else hist_dev.shape[1]
    check(lib.cortex_sample(ctypes.c_void_p(logits_dev.data_ptr()), rows, vocab, ld,
                            None if hist_dev is None else ctypes.c_void_p(hist_dev.data_ptr()), hist_cols,
                            None if hist_len_dev is None else ctypes.c_void_p(hist_len_dev.data_ptr()),
                            ctypes.c_void_p(uniforms_dev.data_ptr()), ctypes.byref(params),
                            ctypes.c_void_p(out_dev.data_ptr()), ctypes.c_void_p(stream)), "cortex_sample")
    return out_dev


class SnaiCortexBridge:
    """src/tensor_ffi_adapter.php:15-206 over libcortex.so.

    `generate_next_token` takes the uniform draw `u` that replaces
    mt_rand()/mt_getrandmax() (:197) and samples on the GPU.
    """

    def __init__(self, filepath, num_heads=1):
        self.lib = load()
        header = read_header(filepath)  # :63-65
        if not header:
            raise CortexError("Fatal: could not read the model header")
        self.vocab_size = header["vocab_size"]
        self.hidden_dim = header["hidden_dim"]
        self.ctx_size = header["ctx_size"]
        self.num_layers = header["num_layers"]
        self.ffn_dim = header["ffn_dim"]
        self.num_heads = num_heads
        self.state_ptr = self.lib.cortex_load_stream(str(filepath).encode(), int(num_heads))  # :74
        if not self.state_ptr:
            raise CortexError(f"Fatal: the engine could not load the stream: {_lib.last_error()}")
        self.cached_c_logits = np.zeros(self.vocab_size, dtype=np.float32)  # :81

    def init_gpu(self):
        self.lib.cortex_init_gpu()

    def close(self):
        if self.state_ptr:
            self.lib.cortex_free(self.state_ptr)
            self.state_ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def extract_state(self):
        """:95-133: every tensor as little-endian fp32 bytes."""
        d, v = self.hidden_dim, self.vocab_size
        sizes = {0: v * d, 1: v * d, 2: d, 10: d, 11: d, 12: d * d, 13: d * d, 14: d * d, 15: d * d,
                 16: self.ffn_dim * d, 17: self.ffn_dim * d}
        gname = {0: "embeddings", 1: "w_out", 2: "rms_final"}
        lname = {10: "rms_att", 11: "rms_ffn", 12: "w_q", 13: "w_k", 14: "w_v", 15: "w_o", 16: "w_up",
                 17: "w_down"}
        state = {"magic": "SNAI_V4", "vocab_size": v, "hidden_dim": d, "ctx_size": self.ctx_size,
                 "num_layers": self.num_layers, "num_heads": self.num_heads,
                 "tensors": {"global": {}, "layers": []}}
        for t, name in gname.items():
            a = np.zeros(sizes[t], dtype=np.float32)
            self.lib.cortex_extract_layer(self.state_ptr, -1, t, _ptr(a), sizes[t])
            state["tensors"]["global"][name] = a.tobytes()
        for l in range(self.num_layers):
            layer = {}
            for t, name in lname.items():
                a = np.zeros(sizes[t], dtype=np.float32)
                self.lib.cortex_extract_layer(self.state_ptr, l, t, _ptr(a), sizes[t])
                layer[name] = a.tobytes()
            state["tensors"]["layers"].append(layer)
        return state

    def train_step(self, inputs, targets, lr):
        """:135-151: the last ctx tokens of the batch, one training step on the GPU."""
        n = min(len(inputs), self.ctx_size)
        if n == 0:
            return 0.0
        a = np.ascontiguousarray(inputs[-n:], dtype=np.int32)
        b = np.ascontiguousarray(targets[-n:], dtype=np.int32)
        return self.lib.cortex_train_step(self.state_ptr, _ptr(a), _ptr(b), n, float(lr))

    def generate_next_token(self, input_tokens, temp=0.7, top_k=40, top_p=0.9, rep_pen=1.15, u=0.5):
        """:153-205.  Feeds the whole window (no cache reset, as the PHP code)
        and samples the next id with the variant-B sampler on the GPU."""
        import torch

        toks = list(input_tokens)
        if len(toks) > self.ctx_size:
            toks = toks[-self.ctx_size:]
        c_in = np.ascontiguousarray(toks, dtype=np.int32)
        self.lib.cortex_forward(self.state_ptr, _ptr(c_in), len(c_in), _ptr(self.cached_c_logits))
        dev = torch.device("cuda")
        logits = torch.from_numpy(self.cached_c_logits).view(1, -1).to(dev)
        hist = torch.from_numpy(c_in).view(1, -1).to(dev)
        uni = torch.tensor([u], dtype=torch.float32, device=dev)
        out = torch.zeros(1, dtype=torch.int32, device=dev)
        sample_device(logits, uni, sample_params(VARIANT_B, temp, rep_pen, top_k, top_p), hist, None, out)
        return int(out.item())


def run_inference(path, prompt_ids, uniforms, temperature=0.25, rep_penalty=1.15, max_new_tokens=256,
                  stop_tokens=(2,), num_heads=None, precision=_lib.PREC_FP32, device=0):
    """src/snai_inference.php:113-215 on the GPU: reset, feed the prompt,
    then {sample, stop check, feed} per step.  heads default to max(1, d/64)
    (:55); the prompt is cut to the last ctx-max_new ids (:113-115).
    Returns (generated ids, stop reason)."""
    h = read_header(path)
    if h is None:
        raise CortexError("not a SNAI_V4 file")
    heads = num_heads if num_heads is not None else max(1, h["hidden_dim"] // 64)
    ctx = h["ctx_size"]
    toks = list(prompt_ids)
    if len(toks) > ctx - max_new_tokens:
        toks = toks[-(ctx - max_new_tokens):] if ctx - max_new_tokens > 0 else []
    eng = Cortex(path, num_heads=heads, max_seqs=1, device=device, precision=precision)
    try:
        eng.reset([0])
        eng.forward(np.asarray([toks], dtype=np.int32), want_logits=False)
        params = sample_params(VARIANT_A, temperature, rep_penalty, nan_guard=1)
        out = []
        for i in range(max_new_tokens):
            tok = int(eng.decode(np.asarray([uniforms[i]], dtype=np.float32), params, slots=[0])[0])
            if tok == -1:
                return out, "nan"
            if tok in stop_tokens:
                return out, "stop"
            out.append(tok)
            if len(toks) + i >= ctx - 1:
                return out, "ctx"
        return out, "max"
    finally:
        eng.close()


def merge_files(paths, out_path, device=0):
    """src/net2net_forge.php merge_models / src/train_cluster.php
    average_models_stream on the GPU (cortex_merge_files)."""
    lib = load()
    arr = (ctypes.c_char_p * len(paths))(*[str(p).encode() for p in paths])
    check(lib.cortex_merge_files(arr, len(paths), str(out_path).encode(), int(device)), "cortex_merge_files")
    return out_path


def upscale_file(in_path, out_path, target_dim, seed=4321, device=0):
    """src/net2net_forge.php upscale_model on the GPU (cortex_upscale_file)."""
    lib = load()
    check(lib.cortex_upscale_file(str(in_path).encode(), str(out_path).encode(), int(target_dim), int(seed),
                                  int(device)), "cortex_upscale_file")
    return out_path


def average_states(engines):
    """Federated average of the engines' weights in GPU memory
    (cortex_average_states): Cortex objects or raw state pointers."""
    lib = load()
    hs = [e.h if hasattr(e, "h") else e for e in engines]
    arr = (ctypes.c_void_p * len(hs))(*hs)
    check(lib.cortex_average_states(arr, len(hs)), "cortex_average_states")
