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


def workspace_bytes(total_tokens: int, num_seqs: int, num_v_heads: int = HV) -> int:
    """Workspace bytes for ``launch_gdn`` (gdn_prefill_workspace_size[_heads])."""
    lib = _capi.load()
    if num_v_heads == HV:
        return int(lib.gdn_prefill_workspace_size(int(total_tokens), int(num_seqs)))
    return int(lib.gdn_prefill_workspace_size_heads(int(total_tokens), int(num_seqs), int(num_v_heads)))


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
    device buffer of at least ``workspace_bytes(T, N)`` bytes (other head
    counts: ``workspace_bytes(T, N, hv)``).  Head counts other than 4 q/k /
    8 v (q ``[T, HQK, 128]``, v ``[T, HV, 128]``, HV a multiple of HQK) take
    the same paths.
    """
    _need(path in PATHS, f"path must be one of {sorted(PATHS)}")
    _need(isinstance(q, torch.Tensor), "q must be a torch.Tensor")
    if isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.device != q.device:
        cu_seqlens = cu_seqlens.to(q.device)
    N = cu_seqlens.numel() - 1
    hqk, hv = heads(q, v)
    if output is None:
        output = torch.empty((q.shape[0], hv, D), dtype=torch.bfloat16, device=q.device)
    if new_state is None:
        new_state = torch.empty((N, hv, D, D), dtype=torch.float32, device=q.device)
    T, N = validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state, check_seqlens)
    lib = _capi.load()
    other_heads = (hqk, hv) != (HQK, HV)
    need = workspace_bytes(T, N, hv)
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
        if other_heads:
            _capi.check(lib.gdn_prefill_launch_heads(ctypes.byref(args), hqk, hv, ws_ptr, need,
                                                     ctypes.c_void_p(stream)), "gdn_prefill_launch_heads")
        else:
            _capi.check(lib.gdn_prefill_launch(ctypes.byref(args), ws_ptr, need, ctypes.c_void_p(stream)),
                        "gdn_prefill_launch")
    return output, new_state


def device_status(device=None, clear: bool = True) -> int:
    """Synchronises and returns the device status word (GDN_ERR_DEVICE_* bits)."""
    device = torch.device("cuda") if device is None else torch.device(device)
    with torch.cuda.device(device):
        return _capi.read_device_status(torch.cuda.current_stream(device).cuda_stream, clear)


# ------------------------------------------------------ context parallelism --
def cp_split(cu_seqlens, world: int) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Token ranges of a batch for ``world`` context-parallel ranks: every
    sequence's chunks (64 tokens) are split into ``world`` consecutive ranges
    of whole chunks (the last may be partial).  Returns, per rank, the global
    token indices it holds and its local cu_seqlens (int64, on the CPU).
    Every sequence needs at least ``world`` chunks' worth of tokens beyond the
    last rank's first token, i.e. ``64 * (world - 1) + 1`` tokens."""
    cu = [int(x) for x in torch.as_tensor(cu_seqlens).to("cpu", torch.int64)]
    out = []
    for r in range(world):
        idx, lens = [], []
        for s in range(len(cu) - 1):
            t0, t1 = cu[s], cu[s + 1]
            nch = (t1 - t0 + 63) // 64
            _need(t1 - t0 > 64 * (world - 1), f"sequence {s} ({t1 - t0} tokens) is too short for {world} ranks")
            c0, c1 = nch * r // world, nch * (r + 1) // world
            a, b = t0 + 64 * c0, min(t1, t0 + 64 * c1)
            _need(b > a, f"sequence {s} leaves rank {r} no tokens")
            idx.append(torch.arange(a, b))
            lens.append(b - a)
        loc = torch.zeros(len(lens) + 1, dtype=torch.int64)
        if lens:
            loc[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0)
        out.append((torch.cat(idx) if idx else torch.zeros(0, dtype=torch.int64), loc))
    return out


def cp_workspace_bytes(local_tokens: int, num_seqs: int, world: int) -> int:
    return int(_capi.load().gdn_prefill_cp_workspace_size(int(local_tokens), int(num_seqs), int(world)))


def cp_summary_region(workspace: torch.Tensor, local_tokens: int, num_seqs: int, world: int) -> torch.Tensor:
    """The uint8 view of the workspace that the ranks all-gather: world blocks
    of num_seqs x 8 x 98304 bytes (one carry summary per rank and unit)."""
    off = int(_capi.load().gdn_prefill_cp_summary_offset(int(local_tokens), int(num_seqs)))
    return workspace[off: off + world * num_seqs * HV * 98304]


def cp_launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, workspace,
              rank: int, world: int, phase: int) -> None:
    """One phase of the context-parallel prefill on this rank's local tokens
    (``gdn_prefill_cp_launch``); the caller all-gathers ``cp_summary_region``
    between phase 0 and phase 1."""
    T, N = validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state)
    lib = _capi.load()
    need = cp_workspace_bytes(T, N, world)
    _need(workspace.numel() * workspace.element_size() >= need and workspace.device == q.device,
          f"workspace must be >= {need} bytes on {q.device}")
    args = _capi.GdnPrefillArgs(
        _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
        _ptr(cu_seqlens),
        _capi.GDN_SEQLENS_INT64 if cu_seqlens.dtype == torch.int64 else _capi.GDN_SEQLENS_INT32,
        PATHS["chunked"], T, N, 0.0 if scale is None else float(scale), _ptr(output), _ptr(new_state))
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _capi.check(lib.gdn_prefill_cp_launch(ctypes.byref(args), _ptr(workspace), need, rank, world, phase,
                                              ctypes.c_void_p(stream)), "gdn_prefill_cp_launch")


def launch_gdn_context_parallel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, output=None,
                                new_state=None, group=None, workspace: torch.Tensor | None = None):
    """Prefill with every sequence split by token range over the ranks of a
    ``torch.distributed`` (NCCL) group, one GPU per rank: the tensors are this
    rank's tokens (ranges as ``cp_split`` makes them) with its local
    cu_seqlens; ``state`` is read on rank 0.  Returns ``(output, new_state)``:
    this rank's outputs, and the state after its range (on the last rank, the
    final state).  One all-gather of ``world x num_seqs x 768 KiB`` carries
    the ranks' carry summaries."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    N = cu_seqlens.numel() - 1
    if output is None:
        output = torch.empty((q.shape[0], HV, D), dtype=torch.bfloat16, device=q.device)
    if new_state is None:
        new_state = torch.empty((N, HV, D, D), dtype=torch.float32, device=q.device)
    need = cp_workspace_bytes(q.shape[0], N, world)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    cp_launch(q, k, v, state if rank == 0 else None, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
              workspace, rank, world, 0)
    region = cp_summary_region(workspace, q.shape[0], N, world)
    block = region.numel() // world
    dist.all_gather_into_tensor(region, region[rank * block:(rank + 1) * block], group=group)
    cp_launch(q, k, v, None, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state, workspace, rank, world, 1)
    return output, new_state
