"""The two ways the materialised backward launches dV and dK: one interleaved
launch when the dO and Q operands fit in half of the L2 together (small
problems), two launches otherwise.  The large case is checked against a
PyTorch fp32 attention on the GPU (the float64 oracle is too slow at 32 heads
x 2048 tokens x d512); both cases check which launches ran."""

import pytest
import torch

from parity_util import REL_L2_TOL, make_inputs, rel_l2

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib, ops  # noqa: E402


def _fp32_grads(q, k, v, dout):
    """Causal, scale 1.0, GQA by head repetition; BSHD in, BSHD gradients out."""
    qf, kf, vf = (t.detach().float().transpose(1, 2).requires_grad_(True) for t in (q, k, v))
    g = qf.shape[1] // kf.shape[1]
    kr, vr = kf.repeat_interleave(g, dim=1), vf.repeat_interleave(g, dim=1)
    s = qf @ kr.transpose(-1, -2)
    n = s.shape[-1]
    s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    o = torch.softmax(s, dim=-1) @ vr
    o.backward(dout.float().transpose(1, 2))
    return [t.grad.transpose(1, 2) for t in (qf, kf, vf)]


def _run(s, hq, hkv, d, seed):
    q, k, v, dout = make_inputs((1, s, hq, d), (1, s, hkv, d), (1, s, hkv, d), seed=seed)
    n0 = _lib.launch_counts()
    out, lse = ops.attn_fwd(q, k, v, window=0)
    grads = ops.attn_bwd(q, k, v, out, lse, dout, window=0)
    torch.cuda.synchronize()
    n1 = _lib.launch_counts()
    used = {k_: n1[k_] - n0[k_] for k_ in ("bwd_gemm_dv", "bwd_gemm_dk", "bwd_gemm_dvdk")}
    return (q, k, v, dout), grads, used


def test_large_problem_launches_dv_and_dk_separately():
    # 2048 tokens x 32 heads x (512 + 512) x 2 B = 128 MB of dO and Q: two launches
    ins, grads, used = _run(2048, 32, 4, 512, seed=41)
    assert used == {"bwd_gemm_dv": 1, "bwd_gemm_dk": 1, "bwd_gemm_dvdk": 0}
    ref = _fp32_grads(*ins)
    for name, got, r in zip(("dq", "dk", "dv"), grads, ref):
        err = rel_l2(got.float().cpu().numpy(), r.cpu().numpy())
        assert err < REL_L2_TOL, (name, err)


def test_small_problem_interleaves_dv_and_dk():
    ins, grads, used = _run(384, 8, 2, 512, seed=42)
    assert used == {"bwd_gemm_dv": 0, "bwd_gemm_dk": 0, "bwd_gemm_dvdk": 1}
    ref = _fp32_grads(*ins)
    for name, got, r in zip(("dq", "dk", "dv"), grads, ref):
        err = rel_l2(got.float().cpu().numpy(), r.cpu().numpy())
        assert err < REL_L2_TOL, (name, err)
