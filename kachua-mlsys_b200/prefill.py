"""Prefill drop-in: ``launch_gdn`` for ``gdn_prefill_qk4_v8_d128_k_last``.

Same destination-passing signature as the reference plugin,
``launch_gdn(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output,
new_state)`` (gdn_prefill_qk4_v8_d128_k_last/solution/triton/kernel.py:56-57),
including its conveniences: ``state``/``output``/``new_state`` may be ``None``
(kernel.py:72-91; ``state=None`` is a zero initial state), ``scale`` None or 0
selects 1/sqrt(128) (kernel.py:69-70), and ``(output, new_state)`` is returned
(kernel.py:192, 252, 262).  The scratch space the reference allocated with
``torch.empty`` per call (kernel.py:136-168, 196-218) is one workspace buffer
here, sized by ``gdn_prefill_workspace_size``.

Semantics follow the reference oracle where the two reference files differ:
an empty sequence gets a zero ``new_state`` row (prefill
reference_torch_impl.py:53-55; the Triton kernel copied the input state).
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi

HQK, HV, D = 4, 8, 128


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check(t, name, dtype, shape, device) -> None:
    _need(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _need(t.device == device, f"{name} must be on {device}, got {t.device}")
    _need(t.is_contiguous(), f"{name} must be contiguous")
    _need(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state,
             check_seqlens: bool = False, require_cuda: bool = True) -> tuple[int, int]:
    """Checks every argument; returns ``(total_tokens, num_seqs)``.

    With ``check_seqlens`` the cu_seqlens values are copied to the host and
    checked (a device sync); otherwise the kernels check them on the device
    and report through ``device_status``.  ``require_cuda=False`` checks only
    shapes/dtypes/layout (host-side tests).
    """
    _need(isinstance(q, torch.Tensor) and q.dim() == 3, "q must be a [T, 4, 128] tensor")
    T = q.shape[0]
    HQK, HV = heads(q, v)
    dev = q.device
    _need(dev.type == "cuda" or not require_cuda, "q must be a CUDA tensor (there is no CPU path)")
    _need(isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.dim() == 1 and cu_seqlens.numel() >= 1,
          "cu_seqlens must be a 1-D tensor of N+1 offsets")
    _need(cu_seqlens.dtype in (torch.int32, torch.int64), "cu_seqlens must be int32 or int64")
    _need(cu_seqlens.device == dev, f"cu_seqlens must be on {dev}")
    _need(cu_seqlens.is_contiguous(), "cu_seqlens must be contiguous")
    N = cu_seqlens.numel() - 1
    _check(q, "q", torch.bfloat16, (T, HQK, D), dev)
    _check(k, "k", torch.bfloat16, (T, HQK, D), dev)
    _check(v, "v", torch.bfloat16, (T, HV, D), dev)
    if state is not None:
        _check(state, "state", torch.float32, (N, HV, D, D), dev)
        _need(N == 0 or state.data_ptr() != new_state.data_ptr(), "state must not alias new_state")
    _check(A_log, "A_log", torch.float32, (HV,), dev)
    _check(dt_bias, "dt_bias", torch.float32, (HV,), dev)
    _need(isinstance(a, torch.Tensor) and a.numel() == T * HV, f"a must be [T, {HV}]")
    _need(isinstance(b, torch.Tensor) and b.numel() == T * HV, f"b must be [T, {HV}]")
    _check(a, "a", torch.bfloat16, a.shape, dev)
    _check(b, "b", torch.bfloat16, b.shape, dev)
    _check(output, "output", torch.bfloat16, (T, HV, D), dev)
    _check(new_state, "new_state", torch.float32, (N, HV, D, D), dev)
    if check_seqlens:
        cu = cu_seqlens.to("cpu", torch.int64)
        _need(int(cu[0]) >= 0, "cu_seqlens[0] must be >= 0")
        _need(bool((cu[1:] >= cu[:-1]).all()), "cu_seqlens must be non-decreasing")
        _need(int(cu[-1]) <= T, f"cu_seqlens[-1]={int(cu[-1])} exceeds total tokens {T}")
    return T, N


def heads(q, v) -> tuple[int, int]:
    """(q/k heads, v heads) from the tensors: 4 / 8 in the reference."""
    hqk = q.shape[-2] if isinstance(q, torch.Tensor) and q.dim() >= 2 else HQK
    hv = v.shape[-2] if isinstance(v, torch.Tensor) and v.dim() >= 2 else HV
    _need(hqk >= 1 and hv >= hqk and hv % hqk == 0,
          f"v heads ({hv}) must be a multiple of q/k heads ({hqk})")
    return hqk, hv


def workspace_bytes(total_tokens: int, num_seqs: int) -> int:
    return int(_capi.load().gdn_prefill_workspace_size(int(total_tokens), int(num_seqs)))


def _ptr(t):
    return ctypes.c_void_p(None if t is None else t.data_ptr())


PATHS = {"auto": 0, "recurrent": 1, "chunked": 2, "segmented": 3}


def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, output=None,
               new_state=None, workspace: torch.Tensor | None = None, check_seqlens: bool = False,
               path: str = "auto"):
    """Varlen GDN prefill (destination-passing); returns ``(output, new_state)``.

    ``path`` selects the algorithm: ``"auto"`` (token-recurrent kernel for
    batches of short sequences, chunked tensor-core kernels otherwise),
    ``"recurrent"`` or ``"chunked"``.  ``workspace`` may be passed to reuse a
    device buffer of at least ``workspace_bytes(T, N)`` bytes.  Head counts
    other than 4 q/k / 8 v (q ``[T, HQK, 128]``, v ``[T, HV, 128]``) run the
    token-recurrent kernel.
    """
    _need(path in PATHS, f"path must be one of {sorted(PATHS)}")
    _need(isinstance(q, torch.Tensor), "q must be a torch.Tensor")
    if isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.device != q.device:
        cu_seqlens = cu_seqlens.to(q.device)
    N = cu_seqlens.numel() - 1
    hqk, hv = heads(q, v)
    _need((hqk, hv) == (HQK, HV) or path in ("auto", "recurrent"),
          "head counts other than 4 / 8 run the token-recurrent kernel only (path auto or recurrent)")
    if output is None:
        output = torch.empty((q.shape[0], hv, D), dtype=torch.bfloat16, device=q.device)
    if new_state is None:
        new_state = torch.empty((N, hv, D, D), dtype=torch.float32, device=q.device)
    T, N = validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, check_seqlens)
    lib = _capi.load()
    if (hqk, hv) != (HQK, HV):
        args = _capi.GdnPrefillArgs(
            _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
            _ptr(cu_seqlens),
            _capi.GDN_SEQLENS_INT64 if cu_seqlens.dtype == torch.int64 else _capi.GDN_SEQLENS_INT32,
            PATHS["recurrent"], T, N, 0.0 if scale is None else float(scale), _ptr(output), _ptr(new_state))
        with torch.cuda.device(q.device):
            stream = torch.cuda.current_stream(q.device).cuda_stream
            _capi.check(lib.gdn_prefill_launch_heads(ctypes.byref(args), hqk, hv, ctypes.c_void_p(stream)),
                        "gdn_prefill_launch_heads")
        return output, new_state
    need = int(lib.gdn_prefill_workspace_size(T, N))
    if need > 0 and (workspace is None or workspace.numel() * workspace.element_size() < need
                     or workspace.device != q.device):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    args = _capi.GdnPrefillArgs(
        _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
        _ptr(cu_seqlens),
        _capi.GDN_SEQLENS_INT64 if cu_seqlens.dtype == torch.int64 else _capi.GDN_SEQLENS_INT32,
        PATHS[path], T, N, 0.0 if scale is None else float(scale), _ptr(output), _ptr(new_state))
    ws_ptr = _ptr(workspace) if need > 0 else ctypes.c_void_p(None)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _capi.check(lib.gdn_prefill_launch(ctypes.byref(args), ws_ptr, need, ctypes.c_void_p(stream)),
                    "gdn_prefill_launch")
    return output, new_state


def device_status(device=None, clear: bool = True) -> int:
    """Synchronises and returns the device status word (GDN_ERR_DEVICE_* bits)."""
    device = torch.device("cuda") if device is None else torch.device(device)
    with torch.cuda.device(device):
        return _capi.read_device_status(torch.cuda.current_stream(device).cuda_stream, clear)
