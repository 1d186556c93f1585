"""Model merging, federated averaging and Net2Net upscaling.

CPU: the oracle's restatement (oracle/net2net.py) against known answers
derived from src/net2net_forge.php:29-214 and src/train_cluster.php:144-224.
GPU: the library's versions (cortex_merge_files, cortex_upscale_file,
cortex_average_states / cortex_group_average) against the oracle, byte for
byte."""
import os
import struct

import numpy as np
import pytest

from conftest import gpu_available, make_model
from oracle import net2net as N2


def _write(path, vocab, dim, ffn, ctx, layers, floats):
    with open(path, "wb") as f:
        f.write(b"SNAI_V4\x00" + struct.pack("<5I", vocab, dim, ffn, ctx, layers))
        f.write(np.asarray(floats, dtype="<f4").tobytes())


def test_merge_known_answers(tmp_path):
    a, b, c = (str(tmp_path / n) for n in ("a", "b", "c"))
    # fp32 values whose mean differs between a double sum and a float sum
    x = np.float32([1.0, 0.1, 16777216.0, -3.0, 1e-30])
    y = np.float32([2.0, 0.2, 1.0, 3.0, 1e-30])
    z = np.float32([4.0, 0.3, 1.0, 0.5, -2e-30])
    for p, v in ((a, x), (b, y), (c, z)):
        _write(p, 1, 5, 20, 4, 0, v)
    out = str(tmp_path / "m")
    N2.merge([a, b, c], out)
    got = np.frombuffer(open(out, "rb").read()[28:], dtype="<f4")
    want = ((x.astype(np.float64) + y + z) / 3.0).astype(np.float32)
    assert np.array_equal(got, want)
    assert got[2] == np.float32((16777216.0 + 2.0) / 3.0)  # the double sum keeps the +1 +1
    assert open(out, "rb").read()[:28] == open(a, "rb").read()[:28]


def test_merge_rejects_other_headers_and_pads_short_files(tmp_path):
    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    _write(a, 1, 4, 16, 4, 0, [1, 2, 3, 4])
    _write(b, 1, 8, 16, 4, 0, [1, 2, 3, 4])
    with pytest.raises(ValueError):
        N2.merge([a, b], str(tmp_path / "m"))
    _write(b, 1, 4, 16, 4, 0, [3, 4])  # shorter: its missing floats count as 0.0
    N2.merge([a, b], str(tmp_path / "m"))
    got = np.frombuffer(open(str(tmp_path / "m"), "rb").read()[28:], dtype="<f4")
    assert got.tolist() == [2.0, 3.0, 1.5, 2.0]


def test_upscale_structure(tmp_path, model_dir):
    """Shape rules and copied entries of upscale_model (src/net2net_forge.php:149-214)."""
    from snai_b200 import modelgen
    src = make_model(model_dir, "n2n_src.snai", 50, 8, 16, 2, seed=3, std=0.5)
    dst = str(tmp_path / "up.snai")
    N2.upscale(src, dst, 12, seed=7)
    h = modelgen.read_header(dst)
    assert (h["hidden_dim"], h["ffn_dim"], h["ctx_size"], h["num_layers"]) == (12, 48, 32, 4)
    assert os.path.getsize(dst) == modelgen.expected_size(50, 12, 48, 4)
    _, s = modelgen.read_model(src)
    _, t = modelgen.read_model(dst)
    assert np.array_equal(t["embeddings"][:, :8], s["embeddings"])
    new = t["embeddings"][:, 8:]
    assert np.all(np.abs(new) <= np.float32(0.005)) and np.abs(new).max() > 0.004
    for l in range(4):
        src_l = l % 2
        scale = 0.01 if l >= 2 else 1.0
        assert np.array_equal(t[f"{l}.w_q"][:8, :8], s[f"{src_l}.w_q"])
        want_o = (s[f"{src_l}.w_o"].astype(np.float64) * scale).astype(np.float32)
        assert np.array_equal(t[f"{l}.w_o"][:8, :8], want_o)
        want_d = (s[f"{src_l}.w_down"].astype(np.float64) * scale).astype(np.float32)
        assert np.array_equal(t[f"{l}.w_down"][:8, :32], want_d)
        assert np.array_equal(t[f"{l}.rms_att"][:8], s[f"{src_l}.rms_att"])
        assert np.all(np.abs(t[f"{l}.rms_att"][8:]) <= 0.005)  # new RMSNorm entries are noise, not 1
    # the same seed gives the same file, another seed other noise
    d2 = str(tmp_path / "up2.snai")
    N2.upscale(src, d2, 12, seed=7)
    assert open(d2, "rb").read() == open(dst, "rb").read()
    N2.upscale(src, d2, 12, seed=8)
    assert open(d2, "rb").read() != open(dst, "rb").read()
    with pytest.raises(ValueError):
        N2.upscale(src, d2, 8, seed=7)


def test_uniform_is_splitmix64():
    # SplitMix64 reference values (seed 0 state increments): the first
    # outputs of the generator seeded with 0 are 0xE220A8397B1DCDAF, ...
    v = N2._splitmix64(np.uint64(0))
    assert int(v) == 0xE220A8397B1DCDAF
    u = N2.uniform(1234, 3, 100000)
    assert u.min() >= 0.0 and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.01


gpu = pytest.mark.gpu
needs_gpu = pytest.mark.skipif(not gpu_available(), reason="needs a CUDA GPU")


@gpu
@needs_gpu
def test_gpu_merge_matches_oracle(tmp_path, model_dir, built):
    from snai_b200 import CortexError, merge_files
    paths = [make_model(model_dir, f"merge{i}.snai", 300, 64, 16, 2, seed=20 + i, std=0.3) for i in range(3)]
    merge_files(paths, str(tmp_path / "gpu.snai"))
    N2.merge(paths, str(tmp_path / "cpu.snai"))
    assert open(tmp_path / "gpu.snai", "rb").read() == open(tmp_path / "cpu.snai", "rb").read()
    other = make_model(model_dir, "merge_other.snai", 300, 32, 16, 2, seed=1)
    with pytest.raises(CortexError, match="header"):
        merge_files([paths[0], other], str(tmp_path / "bad.snai"))


@gpu
@needs_gpu
def test_gpu_upscale_matches_oracle(tmp_path, model_dir, built):
    from snai_b200 import Cortex, upscale_file
    src = make_model(model_dir, "n2n_drone.snai", 1000, 128, 64, 2, seed=5)
    upscale_file(src, str(tmp_path / "gpu.snai"), 256, seed=4321)
    N2.upscale(src, str(tmp_path / "cpu.snai"), 256, seed=4321)
    assert open(tmp_path / "gpu.snai", "rb").read() == open(tmp_path / "cpu.snai", "rb").read()
    e = Cortex(str(tmp_path / "gpu.snai"), num_heads=4)  # a loadable model: d 256, ctx 128, 4 layers
    assert e.ctx == 128
    e.close()


@gpu
@needs_gpu
def test_gpu_average_states_matches_oracle(tmp_path, model_dir, built):
    """Engines holding three different models (on every visible GPU, or all
    on device 0) end with the oracle's mean of the three files."""
    import torch

    from snai_b200 import PREC_BF16, Cortex, average_states, load
    from snai_b200 import modelgen
    paths = [make_model(model_dir, f"avg{i}.snai", 500, 128, 32, 2, seed=40 + i, std=0.3) for i in range(3)]
    n = torch.cuda.device_count()
    engines = [Cortex(p, num_heads=2, max_seqs=2, device=i % n, precision=PREC_BF16) for i, p in enumerate(paths)]
    average_states(engines)
    N2.merge(paths, str(tmp_path / "mean.snai"))
    _, want = modelgen.read_model(str(tmp_path / "mean.snai"))
    lib = load()
    import ctypes
    for e in engines:
        for (layer, typ, name) in ((-1, 0, "embeddings"), (-1, 1, "w_out"), (0, 13, "0.w_k"), (1, 17, "1.w_down")):
            a = np.zeros(want[name].size, dtype=np.float32)
            lib.cortex_extract_layer(e.h, layer, typ, a.ctypes.data_as(ctypes.c_void_p), a.size)
            assert np.array_equal(a.reshape(want[name].shape), want[name]), (e.device, name)
    # the averaged engines run the averaged model (bf16 copies repacked)
    toks = np.random.default_rng(1).integers(0, 500, (2, 6)).astype(np.int32)
    ref = Cortex(str(tmp_path / "mean.snai"), num_heads=2, max_seqs=2, precision=PREC_BF16)
    assert np.array_equal(engines[0].forward(toks), ref.forward(toks))
    ref.close()
    for e in engines:
        e.close()
