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

    ``require_cuda=False`` checks only shapes/dtypes/layout (host-side tests).
    """
    _need(isinstance(q, torch.Tensor) and q.dim() == 4, "q must be a [B, 1, 4, 128] tensor")
    B = q.shape[0]
    _need(tuple(q.shape) == (B, 1, HQK, D), f"q must be [B, 1, 4, 128], got {tuple(q.shape)}")
    dev = q.device
    _need(dev.type == "cuda" or not require_cuda, "q must be a CUDA tensor (there is no CPU path)")
    _check(q, "q", torch.bfloat16, B * HQK * D, dev)
    _check(k, "k", torch.bfloat16, B * HQK * D, dev)
    _check(v, "v", torch.bfloat16, B * HV * D, dev)
    _check(state, "state", torch.float32, B * HV * D * D, dev)
    _check(A_log, "A_log", torch.float32, HV, dev)
    _check(a, "a", torch.bfloat16, B * HV, dev)
    _check(dt_bias, "dt_bias", torch.float32, HV, dev)
    _check(b, "b", torch.bfloat16, B * HV, dev)
    _check(output, "output", torch.bfloat16, B * HV * D, dev)
    _check(new_state, "new_state", torch.float32, B * HV * D * D, dev)
    _need(tuple(state.shape) == (B, HV, D, D), f"state must be [B, 8, 128, 128], got {tuple(state.shape)}")
    _need(tuple(new_state.shape) == (B, HV, D, D), "new_state must be [B, 8, 128, 128]")
    return B


def _ptr(t: torch.Tensor):
    return ctypes.c_void_p(t.data_ptr())


def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale=None, output=None, new_state=None):
    """One GDN decode step (destination-passing); returns ``(output, new_state)``.

    ``output`` is bf16 ``[B, 8, 128]`` (``[B, 1, 8, 128]`` is accepted too);
    ``new_state`` is the fp32 k-last state after the step.
    """
    _need(isinstance(q, torch.Tensor), "q must be a torch.Tensor")
    if output is None:
        output = torch.empty((q.shape[0], HV, D), dtype=torch.bfloat16, device=q.device)
    if new_state is None:
        new_state = torch.empty_like(state)
    B = validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state)
    lib = _capi.load()
    args = _capi.GdnDecodeArgs(
        _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(A_log), _ptr(a), _ptr(dt_bias), _ptr(b),
        _ptr(output), _ptr(new_state), B, 0.0 if scale is None else float(scale))
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _capi.check(lib.gdn_decode_launch(ctypes.byref(args), ctypes.c_void_p(stream)),
                    "gdn_decode_launch")
    return output, new_state


class PreparedLaunch:
    """A validated decode call that can be re-issued with ~one ctypes call.

    For serving loops that call the same buffers every step (and for CUDA
    graph capture): arguments are checked once here; ``__call__`` launches on
    the current stream of the tensors' device.
    """

    def __init__(self, q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
        B = validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state)
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
        rc = self.lib.gdn_decode_launch(self._ref, ctypes.c_void_p(stream))
        if rc:
            _capi.check(rc, "gdn_decode_launch")


def kernel(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """Value-returning form of the reference binding (binding.py:34-51)."""
    return launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale)


class HostStager:
    """``launch_gdn`` over HOST (pinned) tensors, copies pipelined with compute.

    The batch is cut into slices; slice i's host->device copy, slice i-1's
    kernel and slice i-2's device->host copy run on three streams at once, so
    a step costs about max(H2D, D2H) of PCIe time rather than their sum.
    Device buffers are allocated once per (batch, device) and reused.
    """

    def __init__(self, batch: int, device, slices: int = 8):
        self.batch, self.device = batch, torch.device(device)
        self.slices = max(1, min(slices, batch))
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
        self.streams = [torch.cuda.Stream(dev) for _ in range(3)]

    def bytes_per_step(self) -> tuple[int, int]:
        h2d = sum(t.numel() * t.element_size() for t in (self.q, self.k, self.v, self.a, self.b, self.state,
                                                        self.A_log, self.dt_bias))
        d2h = sum(t.numel() * t.element_size() for t in (self.out, self.state))
        return h2d, d2h

    def __call__(self, q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
        """All tensors on the host (pinned for overlap); writes output/new_state."""
        B = self.batch
        h2d, comp, d2h = self.streams
        cur = torch.cuda.current_stream(self.device)
        for s in self.streams:
            s.wait_stream(cur)
        with torch.cuda.stream(h2d):
            self.A_log.copy_(A_log, non_blocking=True)
            self.dt_bias.copy_(dt_bias, non_blocking=True)
        bounds = [B * i // self.slices for i in range(self.slices + 1)]
        ev_in, ev_done = [], []
        for i in range(self.slices):
            lo, hi = bounds[i], bounds[i + 1]
            with torch.cuda.stream(h2d):
                for dst, src in ((self.q, q), (self.k, k), (self.v, v), (self.a, a), (self.b, b),
                                 (self.state, state)):
                    dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d)
                ev_in.append(e)
            with torch.cuda.stream(comp):
                comp.wait_event(ev_in[i])
                launch_gdn(self.q[lo:hi], self.k[lo:hi], self.v[lo:hi], self.state[lo:hi], self.A_log,
                           self.a[lo:hi], self.dt_bias, self.b[lo:hi], scale, self.out[lo:hi],
                           self.state[lo:hi])
                e = torch.cuda.Event()
                e.record(comp)
                ev_done.append(e)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_done[i])
                output.view(B, HV, D)[lo:hi].copy_(self.out[lo:hi], non_blocking=True)
                new_state[lo:hi].copy_(self.state[lo:hi], non_blocking=True)
        for s in self.streams:
            cur.wait_stream(s)
        return output, new_state
