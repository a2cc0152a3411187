"""The allocation-free backward entry point, ``g4_attn_bwd_noalloc``.

Some callers cannot allocate device memory when they run the backward: a
runtime that plans every device buffer ahead of time and forbids cudaMalloc
during execution, or a plugin host that passes an op its tensors but no scratch
buffer.  For them the library keeps one static device scratch array (16 MiB per
GPU) and this entry point uses it instead of a caller workspace.

These tests call it through the C ABI and check that two calls in a row give
the same gradients as ``g4_attn_bwd`` with a caller workspace, within the
parity tolerance, with the array's device error word still 0 after each call,
and that a call whose minimum scratch exceeds the array is refused before any
launch.  The file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from parity_util import REL_L2_TOL, make_inputs, rel_l2

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib, ops  # noqa: E402


def _noalloc_bwd(q, k, v, out, lse, dout, window):
    lib = _lib.load()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    a = ops._build_args(q, k, v, out, lse, window=window, vision_ids=None, document_ids=None,
                        cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=None,
                        max_seqlen_k=None)
    a.dout = dout.data_ptr()
    a.do_stride = ops._strides3(dout, False)
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.dq_stride = ops._strides3(dq, False)
    a.dk_stride = ops._strides3(dk, False)
    a.dv_stride = ops._strides3(dv, False)
    a.workspace, a.workspace_bytes = None, 0  # ignored by this entry point
    rc = lib.g4_attn_bwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.G4_OK, _lib.last_error()
    return dq, dk, dv


@pytest.mark.parametrize("shape", [(1, 300, 8, 1, 512, 0), (2, 260, 4, 2, 256, 1024)],
                         ids=["global_d512", "local_d256"])
def test_noalloc_backward_matches_workspace_backward_twice(shape):
    b, s, hq, hkv, d, window = shape
    q, k, v, dout = make_inputs((b, s, hq, d), (b, s, hkv, d), (b, s, hkv, d), seed=77)
    out, lse = ops.attn_fwd(q, k, v, window=window)
    ref = ops.attn_bwd(q, k, v, out, lse, dout, window=window)
    lib = _lib.load()
    for _ in range(2):
        got = _noalloc_bwd(q, k, v, out, lse, dout, window)
        code = ctypes.c_int(-1)
        rc = lib.g4_attn_bwd_noalloc_device_error(ctypes.byref(code),
                                                  torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.G4_OK, _lib.last_error()
        assert code.value == 0
        for g, r in zip(got, ref):
            assert rel_l2(g.float().cpu().numpy(), r.float().cpu().numpy()) <= REL_L2_TOL


def test_noalloc_backward_refuses_oversized_scratch_before_launch():
    lib = _lib.load()
    a = _lib.G4AttnArgs()
    # 32 heads x 131072 tokens needs at least 32 MiB of scratch (the per-row
    # delta and log2 LSE): more than the array holds.
    tokens = 131072
    a.q, a.k, a.v, a.o, a.lse = 0x1000, 0x2000, 0x3000, 0x4000, 0x5000
    a.dout, a.dq, a.dk, a.dv = 0x6000, 0x7000, 0x8000, 0x9000
    for f, h in (("q_stride", 32), ("o_stride", 32), ("do_stride", 32), ("dq_stride", 32),
                 ("k_stride", 4), ("v_stride", 4), ("dk_stride", 4), ("dv_stride", 4)):
        getattr(a, f)[:] = [tokens * h * 512, h * 512, 512]
    a.lse_stride[:] = [32 * tokens, tokens]
    a.batch, a.seqlen_q, a.seqlen_k = 1, tokens, tokens
    a.num_q_heads, a.num_kv_heads, a.head_dim_qk, a.head_dim_v = 32, 4, 512, 512
    assert lib.g4_attn_bwd_min_workspace_bytes(ctypes.byref(a)) > _lib.NOALLOC_SCRATCH_BYTES
    rc = lib.g4_attn_bwd_noalloc(ctypes.byref(a), None)
    assert rc == _lib.G4_ERR_WORKSPACE
    assert "scratch" in _lib.last_error()
