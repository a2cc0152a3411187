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


def rel_l2(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = np.linalg.norm(ref.ravel())
    return float(np.linalg.norm((got - ref).ravel()) / max(denom, 1e-30))


def lse_abs_err(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert np.array_equal(np.isneginf(got), np.isneginf(ref)), "masked-row pattern differs"
    fin = np.isfinite(ref)
    return float(np.abs(got[fin] - ref[fin]).max()) if fin.any() else 0.0
