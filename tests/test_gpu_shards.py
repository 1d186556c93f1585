"""Shard invariance: splitting the sequences over several engines (as the
ranks of a multi-GPU run split them) gives the ids one engine gives for all
of them, bit for bit.  Sequences are independent (core/cortex.nim:487-563
keeps no state shared between them), so a row's logits, and hence its id,
must not depend on which other rows share its pass.  The engines here share
one GPU; each holds its own weights and KV cache, as a rank does."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import PREC_BF16, PREC_FP32, Cortex, VARIANT_A, VARIANT_B, sample_params  # noqa: E402
from snai_b200.shard import shard_range  # noqa: E402
from conftest import make_model  # noqa: E402


@pytest.mark.parametrize("prec,total,parts,variant", [
    (PREC_BF16, 512, 2, VARIANT_B),  # 512 rows vs 2 x 256 (CTA-pair GEMMs on both sides)
    (PREC_BF16, 1024, 4, VARIANT_A),
    (PREC_FP32, 48, 3, VARIANT_B),   # fp32 projections
])
def test_split_engines_match_one_engine(prec, total, parts, variant, model_dir, built):
    path = make_model(model_dir, "shard.snai", 4096, 256, 128, 2, seed=9)
    steps, plen = 6, 16
    rng = np.random.default_rng(total + parts)
    prompts = rng.integers(0, 4096, (total, plen)).astype(np.int32)
    U = rng.random((steps, total)).astype(np.float32)
    prm = sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9) if variant == VARIANT_B else sample_params(VARIANT_A, 0.8, 1.15)
    one = Cortex(path, num_heads=4, max_seqs=total, precision=prec)
    one.forward(prompts, want_logits=False)
    want = one.decode_steps(U, prm)
    one.close()
    got = np.zeros_like(want)
    for r in range(parts):
        a, b = shard_range(total, r, parts)
        e = Cortex(path, num_heads=4, max_seqs=b - a, precision=prec)
        e.forward(prompts[a:b], want_logits=False)
        got[:, a:b] = e.decode_steps(np.ascontiguousarray(U[:, a:b]), prm)
        e.close()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("prec,total,variant", [(PREC_BF16, 600, VARIANT_B), (PREC_FP32, 40, VARIANT_A)])
def test_group_matches_one_engine(prec, total, variant, model_dir, built):
    """cortex_group_*: one process, one engine per listed device (every
    visible GPU, or device 0 twice with one GPU), the model file read once
    and fanned out by peer copies: the same logits and ids as one engine,
    gathered into the caller's arrays."""
    from snai_b200 import CortexGroup
    path = make_model(model_dir, "shard.snai", 4096, 256, 128, 2, seed=9)
    n = torch.cuda.device_count()
    devices = list(range(n)) if n > 1 else [0, 0]
    steps, plen = 5, 12
    rng = np.random.default_rng(total)
    prompts = rng.integers(0, 4096, (total, plen)).astype(np.int32)
    U = rng.random((steps, total)).astype(np.float32)
    prm = sample_params(VARIANT_B, 0.7, 1.1, 40, 0.9) if variant == VARIANT_B else sample_params(VARIANT_A, 0.8, 1.15)
    one = Cortex(path, num_heads=4, max_seqs=total, precision=prec)
    want_lg = one.forward(prompts)
    want = one.decode_steps(U, prm)
    one.close()
    g = CortexGroup(path, 4, total, devices, precision=prec)
    assert g.size == len(devices) and g.load_seconds > 0
    assert [g.shard(i) for i in range(g.size)] == [shard_range(total, i, len(devices)) for i in range(g.size)]
    got_lg = g.forward(prompts)
    assert np.array_equal(got_lg, want_lg)
    assert np.array_equal(g.decode_steps(U, prm), want)
    g.close()
