"""The bounded mbarrier wait that every kernel of the library uses, exercised
through ``g4_selftest_wait``: a wait that nothing completes must come back
after the 2 s bound with the device error recorded (never hang), a wait that
sees another warp's abort must return at once without overwriting the first
error, and a completed barrier must pass straight through."""

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib  # noqa: E402

DEV_TIMEOUT_TMA, DEV_TIMEOUT_PEER = 1, 3


def test_completed_barrier_passes():
    code, done, ms = _lib.selftest_wait(0)
    assert (code, done) == (0, True)
    assert ms < 100.0


def test_expired_wait_reports_and_returns():
    n0 = _lib.launch_counts()["selftest_wait"]
    code, done, ms = _lib.selftest_wait(1)
    assert _lib.launch_counts()["selftest_wait"] == n0 + 1
    assert (code, done) == (DEV_TIMEOUT_PEER, False)
    assert 1900.0 <= ms <= 4000.0, ms  # the 2 s bound, read from %globaltimer
    # the context is still usable afterwards
    x = torch.ones(1024, device="cuda")
    assert x.sum().item() == 1024.0


def test_abort_from_another_role_returns_promptly():
    code, done, ms = _lib.selftest_wait(2)
    assert (code, done) == (DEV_TIMEOUT_TMA, False)  # the first error is kept
    assert ms < 100.0
