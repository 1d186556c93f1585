"""SNAI_V4 model files: header, layout, a seeded initializer and Net2Net upscale.

Format (src/tensor_io.php:15-59, core/cortex.nim:969-1044): 8-byte magic
"SNAI_V4\\0", then vocab, hidden, ffn, ctx, layers as little-endian u32, then
little-endian fp32 tensors in this order: embeddings [V,d], w_out [V,d],
rms_final [d], and per layer rms_att [d], rms_ffn [d], Wq, Wk, Wv, Wo [d,d],
W_up [ffn,d], W_down [d,ffn].

`random_model` restates src/init_base.php:77-100 (layout, unit RMSNorm
weights) with seeded N(0, std) weights instead of the unseeded uniform ones;
`upscale_model` restates the upscale of src/net2net_forge.php:108-214 with a
seeded noise generator.
"""
import os
import struct

import numpy as np

MAGIC = b"SNAI_V4\x00"
HEADER_SIZE = 28


def expected_size(vocab, dim, ffn, layers):
    """File size the inference host requires (src/snai_inference.php:64-70)."""
    size = 28 + vocab * dim * 4 * 2 + dim * 4
    layer = dim * 4 * 2 + dim * dim * 4 * 4 + ffn * dim * 4 * 2
    return size + layer * layers


def read_header(path):
    """src/tensor_io.php:22-59: None unless a full SNAI_V4 header is present."""
    try:
        with open(path, "rb") as f:
            data = f.read(HEADER_SIZE)
    except OSError:
        return None
    if len(data) < HEADER_SIZE or data[:8].rstrip(b"\x00") != b"SNAI_V4":
        return None
    vocab, hidden, ffn, ctx, layers = struct.unpack("<5I", data[8:28])
    return {"vocab_size": vocab, "hidden_dim": hidden, "ffn_dim": ffn, "ctx_size": ctx, "num_layers": layers}


def _write_header(f, vocab, dim, ffn, ctx, layers):
    f.write(MAGIC)
    f.write(struct.pack("<5I", vocab, dim, ffn, ctx, layers))


def tensor_shapes(vocab, dim, ffn, layers):
    """(name, shape) of every tensor in file order."""
    out = [("embeddings", (vocab, dim)), ("w_out", (vocab, dim)), ("rms_final", (dim,))]
    for l in range(layers):
        out += [(f"{l}.rms_att", (dim,)), (f"{l}.rms_ffn", (dim,)), (f"{l}.w_q", (dim, dim)),
                (f"{l}.w_k", (dim, dim)), (f"{l}.w_v", (dim, dim)), (f"{l}.w_o", (dim, dim)),
                (f"{l}.w_up", (ffn, dim)), (f"{l}.w_down", (dim, ffn))]
    return out


def random_model(path, vocab, dim, ctx, layers, seed=1234, std=0.02):
    """Writes a seeded model in the init_base layout: RMSNorm weights 1, every
    other tensor N(0, std) fp32 (src/init_base.php:77-100 with seeded values)."""
    ffn = 4 * dim
    rng = np.random.default_rng(seed)
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(path, "wb") as f:
        _write_header(f, vocab, dim, ffn, ctx, layers)
        for name, shape in tensor_shapes(vocab, dim, ffn, layers):
            if name.endswith("rms_final") or name.endswith("rms_att") or name.endswith("rms_ffn"):
                t = np.ones(shape, dtype="<f4")
            else:
                t = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype("<f4")
            f.write(t.tobytes())
    return path


def read_model(path):
    """Header dict and {name: fp32 array} of a SNAI_V4 file."""
    h = read_header(path)
    if h is None:
        raise ValueError(f"{path}: not a SNAI_V4 file")
    vocab, dim, ffn, layers = h["vocab_size"], h["hidden_dim"], h["ffn_dim"], h["num_layers"]
    out = {}
    with open(path, "rb") as f:
        f.seek(HEADER_SIZE)
        for name, shape in tensor_shapes(vocab, dim, ffn, layers):
            n = int(np.prod(shape))
            out[name] = np.frombuffer(f.read(4 * n), dtype="<f4").reshape(shape).copy()
    return h, out


NOISE_FACTOR = 0.005  # src/net2net_forge.php: NOISE_FACTOR


def upscale_model(in_path, out_path, target_dim, seed=4321):
    """src/net2net_forge.php:149-214.  dim -> target_dim, ffn -> 4*target_dim,
    ctx x2, layers x2.  Old entries are copied (times 0.01 for Wo and W_down of
    the new layers, which repeat layer l % old_layers); every new entry is
    uniform noise in [-0.005, 0.005] (seeded here, mt_rand there)."""
    h, t = read_model(in_path)
    vocab, old_dim, old_ffn, old_ctx, old_layers = (h["vocab_size"], h["hidden_dim"], h["ffn_dim"], h["ctx_size"],
                                                    h["num_layers"])
    if target_dim <= old_dim:
        raise ValueError("target_dim must be larger than the current dim")
    new_dim, new_ffn, new_ctx, new_layers = target_dim, 4 * target_dim, old_ctx * 2, old_layers * 2
    rng = np.random.default_rng(seed)

    def grow(old, new_shape, scale=1.0):
        # src/net2net_forge.php:108-147: row by row; old values * scale, noise elsewhere
        out = ((rng.random(new_shape) * 2.0 - 1.0) * NOISE_FACTOR).astype(np.float32)
        old2 = old.reshape(old.shape[0] if old.ndim == 2 else 1, -1)
        r, c = old2.shape
        dst = out.reshape(new_shape[0] if len(new_shape) == 2 else 1, -1)
        dst[:r, :c] = (old2.astype(np.float64) * scale).astype(np.float32)
        return out

    with open(out_path, "wb") as f:
        _write_header(f, vocab, new_dim, new_ffn, new_ctx, new_layers)
        f.write(grow(t["embeddings"], (vocab, new_dim)).astype("<f4").tobytes())
        f.write(grow(t["w_out"], (vocab, new_dim)).astype("<f4").tobytes())
        f.write(grow(t["rms_final"], (new_dim,)).astype("<f4").tobytes())
        for l in range(new_layers):
            src = l % old_layers
            out_scale = 0.01 if l >= old_layers else 1.0
            for key, shape, scale in [("rms_att", (new_dim,), 1.0), ("rms_ffn", (new_dim,), 1.0),
                                      ("w_q", (new_dim, new_dim), 1.0), ("w_k", (new_dim, new_dim), 1.0),
                                      ("w_v", (new_dim, new_dim), 1.0), ("w_o", (new_dim, new_dim), out_scale),
                                      ("w_up", (new_ffn, new_dim), 1.0), ("w_down", (new_dim, new_ffn), out_scale)]:
                f.write(grow(t[f"{src}.{key}"], shape, scale).astype("<f4").tobytes())
    return out_path
