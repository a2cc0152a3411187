"""The C-ABI library loads on a CPU-only host, exports every entry point its
header declares, and rejects malformed arguments before touching a device."""

import ctypes
import os
import re

import pytest

from gemma4_fa4_kernels_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gemma4_b200.h")


def _declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    assert _declared_symbols() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.g4_abi_version() == _lib.ABI_VERSION


def _args(**over):
    a = _lib.G4AttnArgs()
    a.q, a.k, a.v, a.o, a.lse = 0x1000, 0x2000, 0x3000, 0x4000, 0x5000
    for f in ("q_stride", "k_stride", "o_stride"):
        getattr(a, f)[:] = [2048 * 32 * 256, 32 * 256, 256]
    a.k_stride[:] = [2048 * 16 * 256, 16 * 256, 256]
    a.v_stride[:] = [2048 * 16 * 256, 16 * 256, 256]
    a.lse_stride[:] = [32 * 2048, 2048]
    a.batch, a.seqlen_q, a.seqlen_k = 1, 2048, 2048
    a.num_q_heads, a.num_kv_heads, a.head_dim_qk, a.head_dim_v = 32, 16, 256, 256
    a.window = 1024
    for key, value in over.items():
        setattr(a, key, value)
    return a


def _call(a):
    lib = _lib.load()
    return lib.g4_attn_fwd(ctypes.byref(a), None)


def test_workspace_queries_need_no_device():
    lib = _lib.load()
    a = _args()
    assert lib.g4_attn_fwd_workspace_bytes(ctypes.byref(a)) >= 256
    b = lib.g4_attn_bwd_workspace_bytes(ctypes.byref(a))
    # backward keeps two fp32 rows (delta, log2 LSE) per query head and token
    assert b >= 2 * 4 * 32 * 2048


@pytest.mark.parametrize("over,code,needle", [
    (dict(q=None), _lib.G4_ERR_INVALID, "required"),
    (dict(q=0x1001), _lib.G4_ERR_INVALID, "16-byte aligned"),
    (dict(v=0x2000), _lib.G4_ERR_INVALID, "distinct"),
    (dict(head_dim_qk=128, head_dim_v=128), _lib.G4_ERR_UNSUPPORTED, "head dims"),
    (dict(num_q_heads=30), _lib.G4_ERR_INVALID, "multiple of KV heads"),
    (dict(seqlen_q=4096), _lib.G4_ERR_UNSUPPORTED, "Sq <= Sk"),
    (dict(window=-1), _lib.G4_ERR_INVALID, "window"),
    (dict(workspace=0x3008, workspace_bytes=1 << 30), _lib.G4_ERR_INVALID, "workspace"),
])
def test_malformed_arguments_fail_before_launch(over, code, needle):
    assert _call(_args(**over)) == code
    assert needle in _lib.last_error()


def test_metadata_only_on_local_layers():
    a = _args(window=0, vision_ids=0x6000)
    assert _call(a) == _lib.G4_ERR_UNSUPPORTED


def test_strides_must_be_16_byte_multiples():
    a = _args()
    a.q_stride[1] = 32 * 256 + 4
    assert _call(a) == _lib.G4_ERR_INVALID
    assert "multiples of 8" in _lib.last_error()


def test_missing_workspace_is_reported():
    lib = _lib.load()
    a = _args()
    assert lib.g4_attn_fwd(ctypes.byref(a), None) == _lib.G4_ERR_WORKSPACE


def test_argument_blocks_are_cached_per_signature():
    """ops caches an argument block and its workspace sizes per call signature
    (shapes, strides, flags); each call gets a fresh copy whose pointers it
    writes, so a cached block never carries another call's pointers and a new
    signature builds (and sizes) its own block."""
    from gemma4_fa4_kernels_b200 import _lib, ops

    ops._SIG_CACHE.clear()
    builds, sizings = [], []

    def build_for(tag):
        def build():
            a = _lib.G4AttnArgs()
            a.batch, a.window = tag, 7
            a.q = 0x1000 * tag  # a pointer the caller must overwrite
            builds.append(tag)
            return a
        return build

    def sizes(a):
        sizings.append(a.batch)
        return (100 * a.batch, 10 * a.batch)

    a1, s1 = ops._cached_args(("k", 1), build_for(1), sizes)
    a1.q = 0xAAAA
    a2, s2 = ops._cached_args(("k", 1), build_for(1), sizes)
    a3, s3 = ops._cached_args(("k", 2), build_for(2), sizes)
    assert builds == [1, 2] and sizings == [1, 2]
    assert s1 == s2 == (100, 10) and s3 == (200, 20)
    assert a2.q == 0x1000 and a2.window == 7  # a fresh copy, not the first call's block
    assert a1 is not a2 and a3.batch == 2
    ops._SIG_CACHE.clear()
