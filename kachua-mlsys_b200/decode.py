"""Decode drop-in: ``launch_gdn`` for ``gdn_decode_qk4_v8_d128_k_last``.

Same destination-passing signature as the reference plugin,
``launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)``
(gdn_decode_qk4_v8_d128_k_last/solution/cuda/kernel.cu:982-994 and
solution/triton/kernel.py:27-28).  The work runs in the sm_100a decode kernel
behind ``gdn_decode_launch`` (include/gdn_b200.h) on the current torch stream.

Differences from the reference plugin, all stricter:
  * shapes, dtypes, devices and contiguity are checked and a ``ValueError``
    is raised before anything launches (the reference checked nothing);
  * ``scale`` is honoured (the reference CUDA kernel hard-coded 1/sqrt(128),
    kernel.cu:25,612-615); ``None`` or 0 selects 1/sqrt(128) as the oracle;
  * ``output`` / ``new_state`` may be ``None`` and are then allocated;
  * ``state`` may be the same tensor as ``new_state`` (in-place update).
"""
from __future__ import annotations

import ctypes

import torch

from . import _capi

HQK, HV, D = 4, 8, 128


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check(t: torch.Tensor, name: str, dtype: torch.dtype, numel: int, device) -> None:
    _need(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _need(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _need(t.device == device, f"{name} must be on {device}, got {t.device}")
    _need(t.is_contiguous(), f"{name} must be contiguous")
    _need(t.numel() == numel, f"{name} has {t.numel()} elements, expected {numel}")


def validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state, require_cuda: bool = True) -> int:
    """Checks every argument; returns the batch size B.

    q is ``[B, T, 4, 128]`` with T tokens per sequence (T = 1 for a plain
    decode step); k, v, a, b and output carry the same T.  Other head counts
    (q ``[B, T, HQK, 128]``, v ``[B, T, HV, 128]``, HV a multiple of HQK) are
    accepted for the head-count variant.
    ``require_cuda=False`` checks only shapes/dtypes/layout (host-side tests).
    """
    _need(isinstance(q, torch.Tensor) and q.dim() == 4, "q must be a [B, T, 4, 128] tensor")
    B, T = q.shape[0], q.shape[1]
    HQK, HV = heads(q, v)
    _need(T >= 1 and tuple(q.shape) == (B, T, HQK, D), f"q must be [B, T, 4, 128], got {tuple(q.shape)}")
    dev = q.device
    _need(dev.type == "cuda" or not require_cuda, "q must be a CUDA tensor (there is no CPU path)")
    _check(q, "q", torch.bfloat16, B * T * HQK * D, dev)
    _check(k, "k", torch.bfloat16, B * T * HQK * D, dev)
    _check(v, "v", torch.bfloat16, B * T * HV * D, dev)
    sdt = state.dtype if isinstance(state, torch.Tensor) else None
    _need(sdt in (torch.float32, torch.bfloat16), "state must be float32 (or bfloat16: the bf16-state variant)")
    _need(sdt == torch.float32 or T == 1, "a bf16 state takes one token per step")
    _check(state, "state", sdt, B * HV * D * D, dev)
    _check(A_log, "A_log", torch.float32, HV, dev)
    _check(a, "a", torch.bfloat16, B * T * HV, dev)
    _check(dt_bias, "dt_bias", torch.float32, HV, dev)
    _check(b, "b", torch.bfloat16, B * T * HV, dev)
    _check(output, "output", torch.bfloat16, B * T * HV * D, dev)
    _check(new_state, "new_state", sdt, B * HV * D * D, dev)
    _need(tuple(state.shape) == (B, HV, D, D), f"state must be [B, {HV}, 128, 128], got {tuple(state.shape)}")
    _need(tuple(new_state.shape) == (B, HV, D, D), f"new_state must be [B, {HV}, 128, 128]")
    return B


def heads(q, v) -> tuple[int, int]:
    """(q/k heads, v heads) from the tensors: 4 / 8 in the reference."""
    hqk = q.shape[-2] if isinstance(q, torch.Tensor) and q.dim() >= 2 else HQK
    hv = v.shape[-2] if isinstance(v, torch.Tensor) and v.dim() >= 2 else HV
    _need(hqk >= 1 and hv >= hqk and hv % hqk == 0,
          f"v heads ({hv}) must be a multiple of q/k heads ({hqk})")
    return hqk, hv


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale=None, output=None, new_state=None):
    """One GDN decode step (destination-passing); returns ``(output, new_state)``.

    ``output`` is bf16 ``[B, 8, 128]`` (``[B, 1, 8, 128]`` is accepted too);
    ``new_state`` is the fp32 k-last state after the step.  A bf16 ``state``
    (and ``new_state``) selects the bf16-state variant: the same step with
    the state stored in bf16, half the bytes to stream.  With T > 1 tokens
    per sequence (q ``[B, T, 4, 128]``: speculative or multi-token decode)
    the tokens are applied in order in one call, ``output`` is
    ``[B, T, 8, 128]`` and ``new_state`` the state after the last token.
    """
    _need(isinstance(q, torch.Tensor) and q.dim() == 4, "q must be a [B, T, 4, 128] tensor")
    T = q.shape[1]
    hqk, hv = heads(q, v)
    if output is None:
        shape = (q.shape[0], hv, D) if T == 1 else (q.shape[0], T, hv, D)
        output = torch.empty(shape, dtype=torch.bfloat16, device=q.device)
    if new_state is None:
        new_state = torch.empty_like(state)
    B = validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state)
    lib = _capi.load()
    args = _capi.GdnDecodeArgs(
        _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
        _ptr(output), _ptr(new_state), B, 0.0 if scale is None else float(scale))
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if (hqk, hv) != (HQK, HV):
            _capi.check(lib.gdn_decode_launch_heads(ctypes.byref(args), hqk, hv, T,
                                                    int(state.dtype == torch.bfloat16), ctypes.c_void_p(stream)),
                        "gdn_decode_launch_heads")
        elif state.dtype == torch.bfloat16:
            _capi.check(lib.gdn_decode_launch_bf16_state(ctypes.byref(args), ctypes.c_void_p(stream)),
                        "gdn_decode_launch_bf16_state")
        elif T == 1:
            _capi.check(lib.gdn_decode_launch(ctypes.byref(args), ctypes.c_void_p(stream)),
                        "gdn_decode_launch")
        else:
            _capi.check(lib.gdn_decode_launch_tokens(ctypes.byref(args), T, ctypes.c_void_p(stream)),
                        "gdn_decode_launch_tokens")
    return output, new_state


class PreparedLaunch:
    """A validated decode call that can be re-issued with ~one ctypes call.

    For serving loops that call the same buffers every step (and for CUDA
    graph capture): arguments are checked once here; ``__call__`` launches on
    the current stream of the tensors' device.  Every form ``launch_gdn``
    takes is accepted: T >= 1 tokens per sequence, an fp32 or (one token) a
    bf16 state, any supported head counts; all go through
    ``gdn_decode_launch_heads``, which routes the reference's 4 / 8 heads to
    the same kernels as ``gdn_decode_launch``.
    """

    def __init__(self, q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
        _need(isinstance(q, torch.Tensor) and q.dim() == 4, "q must be a [B, T, 4, 128] tensor")
        B = validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state)
        self.tokens = int(q.shape[1])
        self.hqk, self.hv = heads(q, v)
        self.bf16_state = int(state.dtype == torch.bfloat16)
        self._keep = (q, k, v, state, A_log, a, dt_bias, b, output, new_state)
        self.device = q.device
        self.lib = _capi.load()
        self.args = _capi.GdnDecodeArgs(
            _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
            _ptr(output), _ptr(new_state), B, 0.0 if scale is None else float(scale))
        self._ref = ctypes.byref(self.args)

    def __call__(self) -> None:
        if torch.cuda.current_device() != self.device.index:
            raise RuntimeError(f"PreparedLaunch for {self.device} called with cuda:"
                               f"{torch.cuda.current_device()} current")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = self.lib.gdn_decode_launch_heads(self._ref, self.hqk, self.hv, self.tokens, self.bf16_state,
                                              ctypes.c_void_p(stream))
        if rc:
            _capi.check(rc, "gdn_decode_launch_heads")


def kernel(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """Value-returning form of the reference binding (binding.py:34-51)."""
    return launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale)


class HostStager:
    """``launch_gdn`` for a state kept in HOST memory (offloaded between steps).

    Inputs and outputs are host tensors (pinned, or the copies do not
    overlap).  Each call is one ``gdn_decode_launch_host_staged``: the state
    is cut into ``slices`` whose host->device copy, decode kernel and
    device->host copy overlap on three streams, so a step costs about the
    bidirectional PCIe time of the state rather than the sum of both
    directions.  Device buffers for one batch size are allocated here once and
    reused by every call.
    """

    def __init__(self, batch: int, device, slices: int = 8):
        self.batch, self.device = batch, torch.device(device)
        self.slices = max(1, min(slices, 64, max(batch, 1)))
        dev = self.device
        self.q = torch.empty((batch, 1, HQK, D), dtype=torch.bfloat16, device=dev)
        self.k = torch.empty_like(self.q)
        self.v = torch.empty((batch, 1, HV, D), dtype=torch.bfloat16, device=dev)
        self.a = torch.empty((batch, 1, HV), dtype=torch.bfloat16, device=dev)
        self.b = torch.empty_like(self.a)
        self.state = torch.empty((batch, HV, D, D), dtype=torch.float32, device=dev)
        self.out = torch.empty((batch, HV, D), dtype=torch.bfloat16, device=dev)
        self.A_log = torch.empty(HV, dtype=torch.float32, device=dev)
        self.dt_bias = torch.empty(HV, dtype=torch.float32, device=dev)
        self.lib = _capi.load()
        self.dev_args = _capi.GdnDecodeArgs(
            _ptr(self.q), _ptr(self.k), _ptr(self.v), None, _ptr(self.A_log), _ptr(self.a), _ptr(self.dt_bias),
            _ptr(self.b), _ptr(self.out), _ptr(self.state), batch, 0.0)

    def bytes_per_step(self) -> tuple[int, int]:
        h2d = sum(t.numel() * t.element_size() for t in (self.q, self.k, self.v, self.a, self.b, self.state,
                                                        self.A_log, self.dt_bias))
        d2h = sum(t.numel() * t.element_size() for t in (self.out, self.state))
        return h2d, d2h

    def __call__(self, q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
        """All tensors on the host; writes output / new_state (may be ``state``)."""
        B = validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state, require_cuda=False)
        _need(B == self.batch, f"stager built for batch {self.batch}, got {B}")
        _need(q.shape[1] == 1, "HostStager is for one token per sequence")
        _need(heads(q, v) == (HQK, HV), "HostStager takes 4 q/k and 8 v heads")
        _need(state.dtype == torch.float32, "HostStager takes the fp32 state")
        _need(q.device.type == "cpu", "HostStager takes host tensors")
        host = _capi.GdnDecodeArgs(
            _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
            _ptr(output), _ptr(new_state), B, 0.0 if scale is None else float(scale))
        self.dev_args.batch = B
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _capi.check(self.lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(self.dev_args),
                                                               self.slices, ctypes.c_void_p(stream)),
                        "gdn_decode_launch_host_staged")
        return output, new_state
