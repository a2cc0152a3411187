"""ctypes binding of ``libgemma4_b200.so`` (C ABI: ``include/gemma4_b200.h``).

The library is loaded from the package directory.  There is no fallback: if it
is missing or fails to load, every operator raises ``LibraryUnavailable``.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libgemma4_b200.so")

ABI_VERSION = 2

G4_OK = 0
G4_ERR_INVALID = 1
G4_ERR_UNSUPPORTED = 2
G4_ERR_CUDA = 3
G4_ERR_DEVICE = 4
G4_ERR_WORKSPACE = 5

# Size of the static scratch array behind g4_attn_bwd_noalloc.
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024

# Every exported entry point declared in include/gemma4_b200.h.
EXPORTED_SYMBOLS = (
    "g4_abi_version",
    "g4_last_error",
    "g4_attn_fwd_workspace_bytes",
    "g4_attn_fwd_min_workspace_bytes",
    "g4_attn_fwd",
    "g4_attn_bwd_workspace_bytes",
    "g4_attn_bwd_min_workspace_bytes",
    "g4_attn_bwd",
    "g4_attn_bwd_noalloc",
    "g4_attn_bwd_noalloc_device_error",
    "g4_merge_attention_partial",
    "g4_cast_f32_bf16",
    "g4_add_f32",
    "g4_read_device_error",
    "g4_selftest_wait",
    "g4_tile_schedule_workspace_bytes",
    "g4_tile_schedule",
    "g4_build_mask",
    "g4_prep_bwd_workspace_bytes",
    "g4_prep_fwd",
    "g4_prep_bwd",
    "g4_kernel_count",
    "g4_kernel_name",
    "g4_launch_count",
    "g4_profile_enable",
    "g4_profile_reset",
    "g4_profile_read",
)


class LibraryUnavailable(RuntimeError):
    """The native library could not be loaded (build it with ``build.py``)."""


class G4AttnArgs(ctypes.Structure):
    """Mirror of ``g4_attn_args``."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("dout", ctypes.c_void_p),
        ("dlse", ctypes.c_void_p),
        ("dq", ctypes.c_void_p),
        ("dk", ctypes.c_void_p),
        ("dv", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 3),
        ("k_stride", ctypes.c_int64 * 3),
        ("v_stride", ctypes.c_int64 * 3),
        ("o_stride", ctypes.c_int64 * 3),
        ("do_stride", ctypes.c_int64 * 3),
        ("dq_stride", ctypes.c_int64 * 3),
        ("dk_stride", ctypes.c_int64 * 3),
        ("dv_stride", ctypes.c_int64 * 3),
        ("lse_stride", ctypes.c_int64 * 2),
        ("batch", ctypes.c_int32),
        ("seqlen_q", ctypes.c_int32),
        ("seqlen_k", ctypes.c_int32),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_k", ctypes.c_void_p),
        ("max_seqlen_q", ctypes.c_int32),
        ("max_seqlen_k", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim_qk", ctypes.c_int32),
        ("head_dim_v", ctypes.c_int32),
        ("window", ctypes.c_int32),
        ("vision_ids", ctypes.c_void_p),
        ("document_ids", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("causal_shift", ctypes.c_int32),
        ("grad_accumulate", ctypes.c_int32),
    ]


class G4MergeArgs(ctypes.Structure):
    """Mirror of ``g4_merge_args``."""

    _fields_ = [
        ("o_acc", ctypes.c_void_p),
        ("lse_acc", ctypes.c_void_p),
        ("o_part", ctypes.c_void_p),
        ("lse_part", ctypes.c_void_p),
        ("o_acc_stride", ctypes.c_int64 * 2),
        ("o_part_stride", ctypes.c_int64 * 2),
        ("lse_acc_stride", ctypes.c_int64 * 2),
        ("lse_part_stride", ctypes.c_int64 * 2),
        ("tokens", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
    ]


class G4PrepArgs(ctypes.Structure):
    """Mirror of ``g4_prep_args``."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("cos", ctypes.c_void_p),
        ("sin", ctypes.c_void_p),
        ("rot", ctypes.c_void_p),
        ("plain", ctypes.c_void_p),
        ("drot", ctypes.c_void_p),
        ("dplain", ctypes.c_void_p),
        ("dx", ctypes.c_void_p),
        ("dweight", ctypes.c_void_p),
        ("x_stride", ctypes.c_int64 * 3),
        ("rot_stride", ctypes.c_int64 * 3),
        ("plain_stride", ctypes.c_int64 * 3),
        ("drot_stride", ctypes.c_int64 * 3),
        ("dplain_stride", ctypes.c_int64 * 3),
        ("dx_stride", ctypes.c_int64 * 3),
        ("cos_stride", ctypes.c_int64 * 2),
        ("batch", ctypes.c_int32),
        ("seqlen", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("rotary_dim", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LibraryUnavailable(
                f"{LIB_PATH} is missing; run `python -m gemma4_fa4_kernels_b200.build`")
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as exc:
            raise LibraryUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
        P = ctypes.POINTER(G4AttnArgs)
        lib.g4_abi_version.restype = ctypes.c_int
        lib.g4_last_error.restype = ctypes.c_char_p
        for name in ("g4_attn_fwd_workspace_bytes", "g4_attn_fwd_min_workspace_bytes",
                     "g4_attn_bwd_workspace_bytes", "g4_attn_bwd_min_workspace_bytes"):
            fn = getattr(lib, name)
            fn.argtypes = [P]
            fn.restype = ctypes.c_size_t
        for name in ("g4_attn_fwd", "g4_attn_bwd", "g4_attn_bwd_noalloc"):
            fn = getattr(lib, name)
            fn.argtypes = [P, ctypes.c_void_p]
            fn.restype = ctypes.c_int
        lib.g4_merge_attention_partial.argtypes = [ctypes.POINTER(G4MergeArgs), ctypes.c_void_p]
        lib.g4_merge_attention_partial.restype = ctypes.c_int
        lib.g4_cast_f32_bf16.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_void_p]
        lib.g4_cast_f32_bf16.restype = ctypes.c_int
        lib.g4_add_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                   ctypes.c_void_p]
        lib.g4_add_f32.restype = ctypes.c_int
        lib.g4_read_device_error.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int),
                                             ctypes.c_void_p]
        lib.g4_read_device_error.restype = ctypes.c_int
        lib.g4_attn_bwd_noalloc_device_error.argtypes = [ctypes.POINTER(ctypes.c_int),
                                                         ctypes.c_void_p]
        lib.g4_attn_bwd_noalloc_device_error.restype = ctypes.c_int
        lib.g4_selftest_wait.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_double)]
        lib.g4_selftest_wait.restype = ctypes.c_int
        lib.g4_tile_schedule_workspace_bytes.argtypes = [P]
        lib.g4_tile_schedule_workspace_bytes.restype = ctypes.c_size_t
        lib.g4_tile_schedule.argtypes = [P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.c_void_p]
        lib.g4_tile_schedule.restype = ctypes.c_int
        lib.g4_build_mask.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p]
        lib.g4_build_mask.restype = ctypes.c_int
        PP = ctypes.POINTER(G4PrepArgs)
        lib.g4_prep_bwd_workspace_bytes.argtypes = [PP]
        lib.g4_prep_bwd_workspace_bytes.restype = ctypes.c_size_t
        for name in ("g4_prep_fwd", "g4_prep_bwd"):
            fn = getattr(lib, name)
            fn.argtypes = [PP, ctypes.c_void_p]
            fn.restype = ctypes.c_int
        lib.g4_kernel_count.restype = ctypes.c_int
        lib.g4_kernel_name.argtypes = [ctypes.c_int]
        lib.g4_kernel_name.restype = ctypes.c_char_p
        lib.g4_launch_count.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]
        lib.g4_launch_count.restype = ctypes.c_int
        lib.g4_profile_enable.argtypes = [ctypes.c_int]
        lib.g4_profile_enable.restype = ctypes.c_int
        lib.g4_profile_reset.restype = ctypes.c_int
        lib.g4_profile_read.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_longlong),
                                        ctypes.POINTER(ctypes.c_double)]
        lib.g4_profile_read.restype = ctypes.c_int
        if lib.g4_abi_version() != ABI_VERSION:
            raise LibraryUnavailable(
                f"ABI mismatch: library {lib.g4_abi_version()}, bindings {ABI_VERSION}")
        _lib = lib
        return lib


def last_error() -> str:
    return load().g4_last_error().decode(errors="replace")


def kernel_names() -> list[str]:
    lib = load()
    return [lib.g4_kernel_name(i).decode() for i in range(lib.g4_kernel_count())]


def launch_counts() -> dict[str, int]:
    """Launches per kernel issued by this process so far."""
    lib = load()
    out = {}
    for i, name in enumerate(kernel_names()):
        c = ctypes.c_longlong(0)
        lib.g4_launch_count(i, ctypes.byref(c))
        out[name] = int(c.value)
    return out


def selftest_wait(mode: int) -> tuple[int, bool, float]:
    """Run the bounded-wait self-test (``g4_selftest_wait``) on the current
    device: returns (device error code, wait completed, wait duration in ms)."""
    lib = load()
    code, done, ms = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_double(0.0)
    rc = lib.g4_selftest_wait(int(mode), ctypes.byref(code), ctypes.byref(done), ctypes.byref(ms))
    if rc != G4_OK:
        raise RuntimeError(f"g4_selftest_wait: {last_error()}")
    return int(code.value), bool(done.value), float(ms.value)


def profile_enable(enable: bool) -> None:
    load().g4_profile_enable(1 if enable else 0)


def profile_reset() -> None:
    load().g4_profile_reset()


def profile_read() -> dict[str, tuple[int, float]]:
    """Per kernel: (launches, summed device ms) since the last reset."""
    lib = load()
    out = {}
    for i, name in enumerate(kernel_names()):
        n, ms = ctypes.c_longlong(0), ctypes.c_double(0.0)
        rc = lib.g4_profile_read(i, ctypes.byref(n), ctypes.byref(ms))
        if rc != G4_OK:
            raise RuntimeError(f"g4_profile_read: {last_error()}")
        out[name] = (int(n.value), float(ms.value))
    return out
