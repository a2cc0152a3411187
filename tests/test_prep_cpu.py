"""Fused Q/K/V preparation without a GPU: admission in the Python surface and
in the C ABI (every check runs before any launch), and the workspace query."""

import ctypes

import pytest
import torch

from gemma4_fa4_kernels_b200 import UnsupportedB200Path, _lib
from gemma4_fa4_kernels_b200 import prep


def _args(**over):
    a = _lib.G4PrepArgs()
    a.x, a.weight, a.cos, a.sin, a.rot, a.plain = 0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 0x60000
    a.x_stride[:] = [4096 * 4 * 512, 4 * 512, 512]
    a.rot_stride[:] = [4096 * 4 * 512, 4 * 512, 512]
    a.plain_stride[:] = [4096 * 4 * 512, 4 * 512, 512]
    a.cos_stride[:] = [0, 512]
    a.batch, a.seqlen, a.num_heads, a.head_dim, a.rotary_dim = 1, 4096, 4, 512, 512
    a.eps = 1e-6
    for key, value in over.items():
        setattr(a, key, value)
    return a


def _fwd(a):
    return _lib.load().g4_prep_fwd(ctypes.byref(a), None)


@pytest.mark.parametrize("over,code,needle", [
    (dict(x=None), _lib.G4_ERR_INVALID, "x is required"),
    (dict(x=0x10008), _lib.G4_ERR_INVALID, "16-byte aligned"),
    (dict(head_dim=128), _lib.G4_ERR_UNSUPPORTED, "head dimension"),
    (dict(rotary_dim=130), _lib.G4_ERR_UNSUPPORTED, "power of two"),
    (dict(rotary_dim=384), _lib.G4_ERR_UNSUPPORTED, "power of two"),
    (dict(rotary_dim=8), _lib.G4_ERR_UNSUPPORTED, "power of two"),
    (dict(rotary_dim=7), _lib.G4_ERR_INVALID, "even"),
    (dict(rotary_dim=1024), _lib.G4_ERR_INVALID, "even"),
    (dict(eps=0.0), _lib.G4_ERR_INVALID, "eps"),
    (dict(cos=None), _lib.G4_ERR_INVALID, "cos and sin"),
    (dict(rot=None, plain=None), _lib.G4_ERR_INVALID, "at least one"),
    (dict(plain=0x50000), _lib.G4_ERR_INVALID, "distinct"),
])
def test_malformed_prep_arguments_fail_before_launch(over, code, needle):
    assert _fwd(_args(**over)) == code
    assert needle in _lib.last_error()


def test_overlapping_output_rows_are_refused():
    a = _args()
    a.rot_stride[:] = [4096 * 4 * 512, 4 * 512, 256]  # heads overlap half a row
    assert _fwd(a) == _lib.G4_ERR_INVALID
    assert "overlap" in _lib.last_error()
    a = _args()
    a.x_stride[:] = [0, 0, 512]  # broadcast input rows are fine; outputs are checked
    a.rot_stride[:] = [0, 8, 512]
    assert _fwd(a) == _lib.G4_ERR_INVALID


def test_unaligned_strides_are_refused():
    a = _args()
    a.x_stride[1] = 4 * 512 + 4
    assert _fwd(a) == _lib.G4_ERR_INVALID
    assert "multiples of 8" in _lib.last_error()


def test_backward_requirements_and_workspace_query():
    lib = _lib.load()
    a = _args(rot=None, plain=None, drot=0x70000, dx=0x80000, dweight=0x90000)
    a.drot_stride[:] = a.x_stride[:]
    a.dx_stride[:] = a.x_stride[:]
    need = lib.g4_prep_bwd_workspace_bytes(ctypes.byref(a))
    # one FP32 partial row of the scale gradient per CTA, at most 8 CTAs per SM
    assert 512 * 4 <= need <= 148 * 8 * 512 * 4
    assert lib.g4_prep_bwd(ctypes.byref(a), None) == _lib.G4_ERR_WORKSPACE
    a.dweight = None
    assert lib.g4_prep_bwd_workspace_bytes(ctypes.byref(a)) == 0
    b = _args(rot=None, plain=None, dx=0x80000, dweight=0x90000, drot=None, dplain=0x70000)
    b.dplain_stride[:] = b.x_stride[:]
    b.dx_stride[:] = b.x_stride[:]
    assert lib.g4_prep_bwd(ctypes.byref(b), None) == _lib.G4_ERR_INVALID
    assert "dweight needs" in _lib.last_error()


def test_python_surface_checks_before_the_library():
    src = torch.zeros(1, 2, 3, 512, dtype=torch.bfloat16)
    w = torch.ones(512, dtype=torch.bfloat16)
    cos = torch.ones(1, 3, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="even integer"):
        prep.prepare_global_kv_from_projection_source(src, k_norm_weight=w, cos=cos, sin=cos,
                                                      partial_rotary_factor=0.3)
    with pytest.raises(UnsupportedB200Path, match="CUDA"):
        prep.prepare_global_kv_from_projection_source(src, k_norm_weight=w, cos=cos, sin=cos)
    with pytest.raises(UnsupportedB200Path, match="CUDA"):
        prep.prepare_value(src, layout="bhsd")
    with pytest.raises(ValueError, match="layout"):
        prep.prepare_value(src, layout="sbhd")
