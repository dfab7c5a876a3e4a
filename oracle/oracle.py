"""Python front end of the CPU parity checker (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg /
reference arm may import this module.  The product path (the
``kachua-mlsys_b200`` package) never imports it and has no CPU fallback.

``decode`` and ``prefill`` mirror the reference's ``run(...)`` functions:

* decode  -> gdn_decode_qk4_v8_d128_k_last/solution/reference_torch_impl.py:12-72,
  returns ``(output fp32 [B,8,128], new_state fp32 [B,8,128,128])``;
* prefill -> gdn_prefill_qk4_v8_d128_k_last/solution/reference_torch_impl.py:17-92,
  returns ``(output bf16 [T,8,128], new_state fp32 [N,8,128,128])``.

Head counts come from the tensor shapes (q/k heads from ``q``, v heads from
``v``): 4 / 8 is the reference; other counts with the same grouping check the
head-count variants of the kernels.

The arithmetic lives in ``gdn_oracle.c`` (built into ``oracle/_build``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libgdn_oracle.so"
_lib = None


def build() -> Path:
    """Compile the C oracle with the committed Makefile (idempotent)."""
    src = _HERE / "gdn_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        P = ctypes.c_void_p
        lib.oracle_gdn_decode.argtypes = [P, P, P, P, P, P, P, P, ctypes.c_float,
                                          ctypes.c_int64, P, P, ctypes.c_int]
        lib.oracle_gdn_decode.restype = ctypes.c_int
        lib.oracle_gdn_prefill.argtypes = [P, P, P, P, P, P, P, P, P, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_float, P, P, ctypes.c_int]
        lib.oracle_gdn_prefill.restype = ctypes.c_int
        lib.oracle_gdn_decode_heads.argtypes = lib.oracle_gdn_decode.argtypes + [ctypes.c_int, ctypes.c_int]
        lib.oracle_gdn_decode_heads.restype = ctypes.c_int
        lib.oracle_gdn_prefill_heads.argtypes = lib.oracle_gdn_prefill.argtypes + [ctypes.c_int, ctypes.c_int]
        lib.oracle_gdn_prefill_heads.restype = ctypes.c_int
        _lib = lib
    return _lib


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def _cpu(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if t.dtype != dtype:
        raise TypeError(f"oracle expects {dtype}, got {t.dtype}")
    return t.detach().to("cpu").contiguous()


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def _scale(scale) -> float:
    return 0.0 if scale is None else float(scale)


def decode(q, k, v, state, A_log, a, dt_bias, b, scale=None, threads: int | None = None):
    """Reference decode step on the CPU; same arguments as the reference ``run``."""
    lib = _load()
    bf, f32 = torch.bfloat16, torch.float32
    q, k, v, a, b = (_cpu(x, bf) for x in (q, k, v, a, b))
    state, A_log, dt_bias = (_cpu(x, f32) for x in (state, A_log, dt_bias))
    B, hqk, hv = q.shape[0], q.shape[-2], v.shape[-2]  # 4 / 8 in the reference; others for the heads variants
    out = torch.empty((B, hv, 128), dtype=f32)
    new_state = torch.empty_like(state)
    rc = lib.oracle_gdn_decode_heads(_ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a),
                                     _ptr(dt_bias), _ptr(b), _scale(scale), B, _ptr(out),
                                     _ptr(new_state), threads or default_threads(), hqk, hv)
    assert rc == 0
    return out, new_state


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None,
            threads: int | None = None):
    """Reference varlen prefill on the CPU; ``state=None`` means zero initial state."""
    lib = _load()
    bf, f32 = torch.bfloat16, torch.float32
    q, k, v, a, b = (_cpu(x, bf) for x in (q, k, v, a, b))
    A_log, dt_bias = (_cpu(x, f32) for x in (A_log, dt_bias))
    cu = cu_seqlens.detach().to("cpu", torch.int64).contiguous()
    N = cu.numel() - 1
    T, hqk, hv = q.shape[0], q.shape[-2], v.shape[-2]
    st = None if state is None else _cpu(state, f32)
    out = torch.empty((T, hv, 128), dtype=bf)
    new_state = torch.empty((N, hv, 128, 128), dtype=f32)
    rc = lib.oracle_gdn_prefill_heads(_ptr(q), _ptr(k), _ptr(v),
                                      None if st is None else _ptr(st), _ptr(A_log), _ptr(a),
                                      _ptr(dt_bias), _ptr(b), _ptr(cu), N, T, _scale(scale),
                                      _ptr(out), _ptr(new_state), threads or default_threads(), hqk, hv)
    assert rc == 0
    return out, new_state
