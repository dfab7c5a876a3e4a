"""ctypes view of the C ABI in include/gdn_b200.h.

This is the thin host binding that replaces the reference's
``solution/cuda/binding.py`` (a torch cpp_extension JIT load, binding.py:20-31):
it loads the prebuilt ``lib/libgdn_b200.so`` and passes plain device pointers,
sizes and the current torch stream.  There is no CPU fallback: if the library
cannot be loaded the call raises.
"""
from __future__ import annotations

import ctypes
import threading

from . import _build

GDN_OK = 0
GDN_SEQLENS_INT32 = 0
GDN_SEQLENS_INT64 = 1
GDN_ERR_DEVICE_BAD_SEQLENS = 16
GDN_ERR_DEVICE_TIMEOUT = 32

# Every symbol include/gdn_b200.h declares.
EXPORTED_SYMBOLS = (
    "gdn_decode_launch",
    "gdn_prefill_workspace_size",
    "gdn_prefill_launch",
    "gdn_status_string",
    "gdn_read_device_status",
    "gdn_abi_version",
    "gdn_mma_selftest",
    "gdn_prefill_launch_noalloc",
    "gdn_decode_launch_host_staged",
    "gdn_decode_launch_tokens",
    "gdn_decode_launch_bf16_state",
    "gdn_decode_launch_heads",
    "gdn_prefill_launch_heads",
    "gdn_prefill_workspace_size_heads",
    "gdn_prefill_cp_workspace_size",
    "gdn_prefill_cp_summary_offset",
    "gdn_prefill_cp_launch",
)
ABI_VERSION = 9
PATH_AUTO, PATH_RECURRENT, PATH_CHUNKED, PATH_SEGMENTED = 0, 1, 2, 3
MMA_KIND_BF16, MMA_KIND_TF32, MMA_KIND_F16 = 1, 2, 3
MMA_A_MN, MMA_B_MN, MMA_D_LANE16, MMA_A_TMEM, MMA_NO_COMPLETION = 1, 2, 4, 8, 16


class GdnDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("state", ctypes.c_void_p),
        ("A_log", ctypes.c_void_p),
        ("a", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("new_state", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("scale", ctypes.c_float),
    ]


class GdnPrefillArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("state", ctypes.c_void_p),
        ("A_log", ctypes.c_void_p),
        ("a", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("cu_seqlens_dtype", ctypes.c_int32),
        ("path", ctypes.c_int32),
        ("total_tokens", ctypes.c_int64),
        ("num_seqs", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("output", ctypes.c_void_p),
        ("new_state", ctypes.c_void_p),
    ]


class GdnError(RuntimeError):
    """A gdn_status_t other than GDN_OK returned by the C ABI."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


_lib = None
_lock = threading.Lock()


def load(build_if_needed: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) the C-ABI library and declare its signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if build_if_needed:
            _build.build()
        if not _build.LIB_PATH.exists():
            raise RuntimeError(f"{_build.LIB_PATH} is missing; run __graft_entry__.build()")
        lib = ctypes.CDLL(str(_build.LIB_PATH))
        P = ctypes.c_void_p
        lib.gdn_decode_launch.argtypes = [ctypes.POINTER(GdnDecodeArgs), P]
        lib.gdn_decode_launch.restype = ctypes.c_int
        lib.gdn_decode_launch_host_staged.argtypes = [ctypes.POINTER(GdnDecodeArgs), ctypes.POINTER(GdnDecodeArgs),
                                                      ctypes.c_int, P]
        lib.gdn_decode_launch_host_staged.restype = ctypes.c_int
        lib.gdn_decode_launch_tokens.argtypes = [ctypes.POINTER(GdnDecodeArgs), ctypes.c_int64, P]
        lib.gdn_decode_launch_tokens.restype = ctypes.c_int
        lib.gdn_decode_launch_bf16_state.argtypes = [ctypes.POINTER(GdnDecodeArgs), P]
        lib.gdn_decode_launch_bf16_state.restype = ctypes.c_int
        lib.gdn_decode_launch_heads.argtypes = [ctypes.POINTER(GdnDecodeArgs), ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int64, ctypes.c_int32, P]
        lib.gdn_decode_launch_heads.restype = ctypes.c_int
        lib.gdn_prefill_launch_heads.argtypes = [ctypes.POINTER(GdnPrefillArgs), ctypes.c_int32, ctypes.c_int32, P,
                                                 ctypes.c_size_t, P]
        lib.gdn_prefill_launch_heads.restype = ctypes.c_int
        lib.gdn_prefill_workspace_size_heads.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
        lib.gdn_prefill_workspace_size_heads.restype = ctypes.c_size_t
        lib.gdn_prefill_cp_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32]
        lib.gdn_prefill_cp_workspace_size.restype = ctypes.c_size_t
        lib.gdn_prefill_cp_summary_offset.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.gdn_prefill_cp_summary_offset.restype = ctypes.c_size_t
        lib.gdn_prefill_cp_launch.argtypes = [ctypes.POINTER(GdnPrefillArgs), P, ctypes.c_size_t, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, P]
        lib.gdn_prefill_cp_launch.restype = ctypes.c_int
        lib.gdn_prefill_workspace_size.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.gdn_prefill_workspace_size.restype = ctypes.c_size_t
        lib.gdn_prefill_launch.argtypes = [ctypes.POINTER(GdnPrefillArgs), P, ctypes.c_size_t, P]
        lib.gdn_prefill_launch.restype = ctypes.c_int
        lib.gdn_status_string.argtypes = [ctypes.c_int]
        lib.gdn_status_string.restype = ctypes.c_char_p
        lib.gdn_read_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_int, P]
        lib.gdn_read_device_status.restype = ctypes.c_int
        lib.gdn_abi_version.argtypes = []
        lib.gdn_abi_version.restype = ctypes.c_int
        lib.gdn_mma_selftest.argtypes = [ctypes.c_int] * 5 + [P, P, P, P]
        lib.gdn_mma_selftest.restype = ctypes.c_int
        if lib.gdn_abi_version() != ABI_VERSION:
            raise RuntimeError("libgdn_b200.so ABI version mismatch; rebuild it")
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load(build_if_needed=False).gdn_status_string(int(status)).decode()
    except Exception:  # library not loadable: still give a readable message
        return f"status {status}"


def check(status: int, what: str) -> None:
    if status != GDN_OK:
        raise GdnError(status, what)


def read_device_status(stream_handle: int, clear: bool = True) -> int:
    out = ctypes.c_int(0)
    check(load().gdn_read_device_status(ctypes.byref(out), int(clear), ctypes.c_void_p(stream_handle)),
          "gdn_read_device_status")
    return out.value
