"""Maximum-size parity with an analytic oracle (the reference pins long
contexts the same way: Q = 0, constant V, EXP-0014).

With Q = 0 every visible score is 0, so every visible key gets weight 1:
  O = mean of the visible V rows = 0.25 exactly (V = 0.25),
  LSE = ln(number of visible keys),
  dS = P (dP - delta) = 0 (dP is the same for every key of a row and equals
  delta), so dQ = dK = 0 up to rounding, and
  dV[k] = sum over the query heads of the group and over the queries q that
  see k of dO[q] / (visible keys of q).
At these sizes the scratch of the materialised algorithms (two-pass forward,
P/dS backward) exceeds any workspace, so they run in bands; the global case
also runs once more on the compact kernels (single-kernel forward, recompute
backward)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
if not torch.cuda.is_available():  # pragma: no cover - CPU containers
    pytest.skip("needs a CUDA device", allow_module_level=True)

from gemma4_fa4_kernels_b200 import _lib, ops  # noqa: E402

BF = torch.bfloat16


def _operands(shape_q, shape_kv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.zeros(shape_q, dtype=BF, device="cuda")
    k = torch.randn(shape_kv, generator=g, device="cuda").to(BF)  # any K: Q = 0 ignores it
    v = torch.full(shape_kv, 0.25, dtype=BF, device="cuda")
    do = torch.randn(shape_q, generator=g, device="cuda").to(BF)
    return q, k, v, do


@pytest.mark.parametrize("algorithm", ["bands", "compact"])
def test_global_d512_maximum_length_forward_and_backward(algorithm):
    s, hq, hkv, d = 262144, 4, 1, 512
    q, k, v, do = _operands((1, s, hq, d), (1, s, hkv, d), seed=5)
    n0 = _lib.launch_counts()
    fwd_alg, bwd_alg = ("auto", "auto") if algorithm == "bands" else ("single", "recompute")
    out, lse = ops.attn_fwd(q, k, v, window=0, algorithm=fwd_alg)
    dq, dk, dv = ops.attn_bwd(q, k, v, out, lse, do, window=0, algorithm=bwd_alg)
    torch.cuda.synchronize()
    n1 = _lib.launch_counts()
    if algorithm == "bands":  # several bands of the two-pass forward and the P/dS backward
        assert n1["fwd_score"] - n0["fwd_score"] >= 2 and n1["attn_fwd"] == n0["attn_fwd"]
        assert n1["bwd_score"] - n0["bwd_score"] >= 4 and n1["bwd_dq"] == n0["bwd_dq"]
    else:
        assert n1["attn_fwd"] > n0["attn_fwd"]
        assert n1["bwd_dq"] > n0["bwd_dq"] and n1["bwd_dkv"] > n0["bwd_dkv"]
    assert torch.all(out == 0.25)
    cnt = torch.arange(1, s + 1, device="cuda", dtype=torch.float64)  # causal: q+1 keys
    ref_lse = torch.log(cnt)[None, None, :].expand(1, hq, s)
    assert (lse.double() - ref_lse).abs().max().item() < 1e-3
    # dV[k] = sum_h sum_{q >= k} dO[q, h] / (q + 1): a reverse cumulative sum
    w = do.double().sum(dim=2) / cnt[None, :, None]           # (1, s, d)
    ref_dv = torch.flip(torch.cumsum(torch.flip(w, [1]), dim=1), [1])[:, :, None, :]
    err = (dv.double() - ref_dv).norm() / ref_dv.norm()
    assert err.item() < 1e-2, err.item()
    scale = do.double().abs().max().item()
    assert dq.double().abs().max().item() < 1e-3 * scale
    assert dk.double().abs().max().item() < 1e-3 * scale


def test_local_d256_packed_long_segments_windowed_counts():
    cu = [0, 30000, 30001, 100000, 131072]
    t, hq, hkv, d, win = cu[-1], 8, 4, 256, 1024
    q, k, v, _ = _operands((t, hq, d), (t, hkv, d), seed=6)
    cuq = torch.tensor(cu, dtype=torch.int32, device="cuda")
    mx = max(b - a for a, b in zip(cu[:-1], cu[1:]))
    out, lse = ops.attn_fwd(q, k, v, window=win, cu_seqlens_q=cuq, cu_seqlens_k=cuq,
                            max_seqlen_q=mx, max_seqlen_k=mx)
    torch.cuda.synchronize()
    assert torch.all(out == 0.25)
    local = torch.cat([torch.arange(b - a, device="cuda") for a, b in zip(cu[:-1], cu[1:])])
    ref = torch.log(torch.clamp(local + 1, max=win).double())
    assert (lse.double() - ref[None, :]).abs().max().item() < 1e-3


def test_decode_against_a_maximum_length_cache():
    # one query token against a 262143-key static cache view (spare capacity kept)
    cap, sk, hq, hkv, d = 262144, 262143, 32, 4, 512
    g = torch.Generator(device="cuda").manual_seed(7)
    kc = torch.randn(1, hkv, cap, d, generator=g, device="cuda").to(BF)
    vc = torch.full((1, hkv, cap, d), 0.25, dtype=BF, device="cuda")
    q = torch.zeros(1, 1, hq, d, dtype=BF, device="cuda")
    n0 = _lib.launch_counts()["decode"]
    out, lse = ops.attn_fwd(q, kc[:, :, :sk].transpose(1, 2), vc[:, :, :sk].transpose(1, 2),
                            window=0)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["decode"] == n0 + 1
    assert torch.all(out == 0.25)
    assert abs(lse.double().max().item() - math.log(sk)) < 1e-3
    assert abs(lse.double().min().item() - math.log(sk)) < 1e-3
