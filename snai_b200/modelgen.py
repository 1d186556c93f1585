"""SNAI_V4 model files: header, layout, a seeded initializer and Net2Net upscale.

Format (src/tensor_io.php:15-59, core/cortex.nim:969-1044): 8-byte magic
"SNAI_V4\\0", then vocab, hidden, ffn, ctx, layers as little-endian u32, then
little-endian fp32 tensors in this order: embeddings [V,d], w_out [V,d],
rms_final [d], and per layer rms_att [d], rms_ffn [d], Wq, Wk, Wv, Wo [d,d],
W_up [ffn,d], W_down [d,ffn].

`random_model` restates src/init_base.php:77-100 (layout, unit RMSNorm
weights) with seeded N(0, std) weights instead of the unseeded uniform ones.
Net2Net upscaling and merging are library calls (cortex_upscale_file,
cortex_merge_files).
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
