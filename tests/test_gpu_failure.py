"""The failure path of a device-side wait, exercised without faulting the GPU.

Every wait of the library's kernels (TMA stages, MMA completion, epilogue
hand-offs) is bounded: when it expires the kernel records an error code in
the state's device error word, returns, and the host reports it from
cortex_synchronize.  cortex_selftest_wait_timeout queues a kernel whose
mbarrier wait can never complete (nothing arrives), with a 1 ms limit, so
this test sees that path end to end: the kernel returns, the error surfaces
once through cortex_synchronize / cortex_last_error, and the same state
then runs a forward pass normally."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from snai_b200 import Cortex, CortexError, load  # noqa: E402
from conftest import rel_err  # noqa: E402


def test_expired_wait_reports_and_context_survives(small_model, built):
    lib = load()
    e = Cortex(small_model, num_heads=2)
    assert lib.cortex_selftest_wait_timeout(e.h, 10) == -2  # limit below 1 us is refused
    for _ in range(2):
        assert lib.cortex_selftest_wait_timeout(e.h, 1_000_000) == 0
        rc = lib.cortex_synchronize(e.h)
        assert rc == -6, rc
        msg = lib.cortex_last_error().decode()
        assert "self-test" in msg and "expired" in msg, msg
        assert lib.cortex_synchronize(e.h) == 0  # reported once, then cleared
    # the kernel returned on its own: the context and the state still work
    rng = np.random.default_rng(3)
    toks = rng.integers(0, 1000, (1, 12)).astype(np.int32)
    got = e.forward(toks)[0]
    ref = O.Oracle(small_model, num_heads=2).forward(toks[0])
    assert rel_err(got, ref) < 2e-5
    # an expired wait is also reported by a call that waits for the GPU
    assert lib.cortex_selftest_wait_timeout(e.h, 1_000_000) == 0
    with pytest.raises(CortexError, match="self-test"):
        e.forward(toks[:, :1])
    assert lib.cortex_selftest_wait_timeout(None, 1_000_000) == -1
    e.close()


def test_wait_timeout_argument_checks(small_model, built):
    lib = load()
    e = Cortex(small_model, num_heads=2)
    assert lib.cortex_selftest_wait_timeout(e.h, 3_000_000_000) == -2
    assert "limit_ns" in lib.cortex_last_error().decode()
    assert lib.cortex_synchronize(e.h) == 0
    e.close()
