"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference's model
merging and Net2Net upscaling, the checker of the library's GPU versions
(cortex_merge_files, cortex_upscale_file, cortex_average_states).

Imported by tests/ only.  Restates:
  src/net2net_forge.php:29-102   merge_models (and the same arithmetic of
                                 src/train_cluster.php:144-224
                                 average_models_stream): header of the first
                                 file; float j = fp32((sum_i double(x_i[j])) / n),
                                 summed in file order, missing floats 0.0
  src/net2net_forge.php:108-214  upscale_model: dim -> target, ffn -> 4 target,
                                 ctx x 2, layers x 2; old entries
                                 fp32(double(x) * scale) (scale 0.01 for Wo and
                                 W_down of the new layers, which repeat layer
                                 l % old_layers), new entries
                                 fp32(((u * 2) - 1) * 0.005)
The PHP code draws u from mt_rand(); the library (and this restatement) draw
it from SplitMix64 (Steele, Lea and Flood 2014) keyed by (seed, output tensor
index, element index), so a seeded upscale is reproducible.  Parity
unpinned: PHP is not available to run the reference itself.
"""
import struct

import numpy as np

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x):
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def uniform(seed, stream, n):
    """u in [0, 1) for elements 0..n-1 of output tensor `stream`."""
    j = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        inner = _splitmix64((np.uint64(stream) << np.uint64(40)) + j)
    z = _splitmix64(np.uint64(seed) ^ inner)
    return (z >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def merge(paths, out_path):
    """src/net2net_forge.php:29-102 on whole files (the PHP code streams them)."""
    data = [open(p, "rb").read() for p in paths]
    hdr = data[0][:28]
    for d, p in zip(data[1:], paths[1:]):
        if d[:28] != hdr:
            raise ValueError(f"{p}: header differs")
    nf = (len(data[0]) - 28) // 4
    s = np.zeros(nf, dtype=np.float64)
    for d in data:
        x = np.frombuffer(d[28:28 + 4 * ((len(d) - 28) // 4)], dtype="<f4").astype(np.float64)[:nf]
        s[:len(x)] += x  # in file order; past a shorter file's end it adds nothing (0.0)
    out = (s / float(len(paths))).astype("<f4")
    with open(out_path, "wb") as f:
        f.write(hdr)
        f.write(out.tobytes())
    return out_path


def upscale(in_path, out_path, target_dim, seed):
    """src/net2net_forge.php:149-214 with the seeded noise above."""
    raw = open(in_path, "rb").read()
    magic, (vocab, old_dim, old_ffn, old_ctx, old_layers) = raw[:8], struct.unpack("<5I", raw[8:28])
    if target_dim <= old_dim:
        raise ValueError("target_dim must be larger")
    new_dim, new_ffn, new_ctx, new_layers = target_dim, 4 * target_dim, old_ctx * 2, old_layers * 2
    layer_floats = 2 * old_dim + 4 * old_dim * old_dim + 2 * old_dim * old_ffn
    need = 2 * vocab * old_dim + old_dim + old_layers * layer_floats
    src = np.zeros(need, dtype=np.float32)
    got = np.frombuffer(raw[28:28 + 4 * need], dtype="<f4")
    src[:len(got)] = got
    stream = [0]

    def grow(off, orr, oc, nr, nc, scale):
        old = src[off:off + orr * oc].reshape(orr, oc).astype(np.float64)
        u = uniform(seed, stream[0], nr * nc).reshape(nr, nc)
        stream[0] += 1
        out = ((u * 2.0) - 1.0) * 0.005
        out[:orr, :oc] = old * scale
        return out.astype("<f4").tobytes()

    parts = [magic, struct.pack("<5I", vocab, new_dim, new_ffn, new_ctx, new_layers)]
    parts.append(grow(0, vocab, old_dim, vocab, new_dim, 1.0))
    parts.append(grow(vocab * old_dim, vocab, old_dim, vocab, new_dim, 1.0))
    parts.append(grow(2 * vocab * old_dim, 1, old_dim, 1, new_dim, 1.0))
    layer0 = 2 * vocab * old_dim + old_dim
    dd = old_dim * old_dim
    for l in range(new_layers):
        q = layer0 + (l % old_layers) * layer_floats
        os_ = 0.01 if l >= old_layers else 1.0
        parts += [grow(q, 1, old_dim, 1, new_dim, 1.0), grow(q + old_dim, 1, old_dim, 1, new_dim, 1.0),
                  grow(q + 2 * old_dim, old_dim, old_dim, new_dim, new_dim, 1.0),
                  grow(q + 2 * old_dim + dd, old_dim, old_dim, new_dim, new_dim, 1.0),
                  grow(q + 2 * old_dim + 2 * dd, old_dim, old_dim, new_dim, new_dim, 1.0),
                  grow(q + 2 * old_dim + 3 * dd, old_dim, old_dim, new_dim, new_dim, os_),
                  grow(q + 2 * old_dim + 4 * dd, old_ffn, old_dim, new_ffn, new_dim, 1.0),
                  grow(q + 2 * old_dim + 4 * dd + old_ffn * old_dim, old_dim, old_ffn, new_dim, new_ffn, os_)]
    with open(out_path, "wb") as f:
        f.write(b"".join(parts))
    return out_path
