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


@pytest.mark.parametrize("sq", [300, 1], ids=["attention", "short_window_decode"])
def test_each_call_clears_a_stale_device_error_word(sq):
    """A workspace whose error word still holds an earlier failed call's code
    reads 0 after a successful call: every call zeroes its header first (a
    one-CTA kernel that the call's first kernel overlaps), the attention
    kernels and the short-window decode alike."""
    import ctypes

    from parity_util import make_inputs

    from gemma4_fa4_kernels_b200 import ops

    q, k, v = make_inputs((1, sq, 4, 256), (1, 300, 2, 256), (1, 300, 2, 256), seed=5,
                          with_dout=False)
    out = torch.empty_like(q)
    lse = torch.empty(1, 4, sq, dtype=torch.float32, device="cuda")
    a = ops._build_args(q, k, v, out, lse, window=1024, vision_ids=None, document_ids=None,
                        cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=None,
                        max_seqlen_k=None)
    lib = _lib.load()
    ws = torch.zeros(max(lib.g4_attn_fwd_workspace_bytes(ctypes.byref(a)), 256),
                     dtype=torch.uint8, device="cuda")
    ws[:4].view(torch.int32).fill_(DEV_TIMEOUT_PEER)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.g4_attn_fwd(ctypes.byref(a), ctypes.c_void_p(stream)) == 0, _lib.last_error()
    code = ctypes.c_int(-1)
    assert lib.g4_read_device_error(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(code),
                                    ctypes.c_void_p(stream)) == 0
    assert code.value == 0
    assert torch.isfinite(out.float()).all()
