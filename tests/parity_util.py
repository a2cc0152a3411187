"""Helpers shared by the GPU parity tests: seeded inputs and error metrics.

Inputs follow the BASELINE recipe: N(0,1) per element from a seeded CPU
generator, every head vector RMS-normalised to unit RMS, cast to BF16.  The
oracle always sees the BF16-rounded values (as float64), so the measured
error is the kernel's, not the input quantisation's.
"""

from __future__ import annotations

import numpy as np
import torch

# rel-L2 <= 1e-2 for O/dQ/dK/dV
# and |LSE| abs <= 1e-3 against the high-precision oracle.
REL_L2_TOL = 1e-2
LSE_ABS_TOL = 1e-3


def rms_unit(x: torch.Tensor) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + 1e-6)


def make_inputs(shape_q, shape_k, shape_v, *, seed, device="cuda", with_dout=True, dlse_shape=None):
    g = torch.Generator().manual_seed(seed)
    q = rms_unit(torch.randn(*shape_q, generator=g)).to(torch.bfloat16)
    k = rms_unit(torch.randn(*shape_k, generator=g)).to(torch.bfloat16)
    v = rms_unit(torch.randn(*shape_v, generator=g)).to(torch.bfloat16)
    out = [q.to(device), k.to(device), v.to(device)]
    if with_dout:
        do_shape = tuple(shape_q[:-1]) + (shape_v[-1],)
        out.append(torch.randn(*do_shape, generator=g).to(torch.bfloat16).to(device))
    if dlse_shape is not None:
        out.append(torch.randn(*dlse_shape, generator=g).to(device))
    return out


def bshd_to_bhsd_np(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().double().numpy().transpose(0, 2, 1, 3)


def bhsd_to_bshd(x: np.ndarray) -> np.ndarray:
    return x.transpose(0, 2, 1, 3)


def thd_np(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().double().numpy()


# Relative errors use max(||ref||, RMS_FLOOR * sqrt(n)) as denominator, so a
# reference that is exactly zero is judged against an absolute RMS floor
# instead of 0.  Example: dQ of a query that sees a single key is exactly 0;
# the kernel forms delta = rowsum(dO * O) (the flash-attention identity) and
# leaves an fp32 summation residual of ~1e-5 RMS there.  Gradients of these
# unit-RMS inputs are O(0.1-1), so the floor does not loosen normal cases.
RMS_FLOOR = 1e-2


def rel_l2(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = max(np.linalg.norm(ref.ravel()), RMS_FLOOR * np.sqrt(max(ref.size, 1)))
    return float(np.linalg.norm((got - ref).ravel()) / denom)


def lse_abs_err(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert np.array_equal(np.isneginf(got), np.isneginf(ref)), "masked-row pattern differs"
    fin = np.isfinite(ref)
    return float(np.abs(got[fin] - ref[fin]).max()) if fin.any() else 0.0


def eager_bf16_attention(q, k, v, allowed_bhqk, dout=None):
    """BF16 eager PyTorch attention (B,S,H,D inputs) with autograd, used as the
    precision yardstick: the north star requires the kernel's error to be no
    worse than twice this baseline's error against the same oracle."""
    qh = q.detach().transpose(1, 2).clone().requires_grad_(True)
    kh = k.detach().transpose(1, 2).clone().requires_grad_(True)
    vh = v.detach().transpose(1, 2).clone().requires_grad_(True)
    rep = qh.shape[1] // kh.shape[1]
    ke = kh.repeat_interleave(rep, dim=1)
    ve = vh.repeat_interleave(rep, dim=1)
    scores = qh @ ke.transpose(-1, -2)
    scores = scores.masked_fill(~allowed_bhqk, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    probs = torch.nan_to_num(probs, nan=0.0)
    out = probs @ ve
    grads = None
    if dout is not None:
        out.backward(dout.transpose(1, 2))
        grads = (qh.grad.transpose(1, 2), kh.grad.transpose(1, 2), vh.grad.transpose(1, 2))
    return out.transpose(1, 2), grads


def assert_close_to_oracle(name, got, ref, eager=None, tol=REL_L2_TOL):
    """rel-L2 <= tol against the oracle, and (if given) no worse than twice the
    BF16-eager error."""
    e = rel_l2(got, ref)
    assert e <= tol, f"{name}: rel-L2 {e:.3e} > {tol}"
    if eager is not None:
        # 2x the BF16-eager error, with a slack of 5e-3 (5e-5 RMS at the floor) for cases where
        # eager is exact by construction (e.g. one visible key, where autograd's
        # sum(P*dP) cancels exactly).
        e_eager = rel_l2(eager, ref)
        assert e <= 2.0 * e_eager + 5e-3, f"{name}: {e:.3e} > 2 x eager {e_eager:.3e}"
    return e
