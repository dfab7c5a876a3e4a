"""gdn_prefill_launch_noalloc: the prefill entry point for callers that cannot
allocate device memory (a host that owns all device memory and offers no
allocator, or a step where cudaMalloc is not allowed, e.g. under stream
capture).  It must give the same results as gdn_prefill_launch with a
caller-provided workspace, on repeated calls that reuse its fixed scratch
array, and must refuse problems larger than that array.

Collected last on purpose (file name), so a stopping run has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

from tests.conftest import state_rel_err

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 32 << 20  # GDN_NOALLOC_SCRATCH_BYTES


def _lib(pkg):
    lib = pkg._capi.load()
    lib.gdn_prefill_launch_noalloc.argtypes = [ctypes.POINTER(pkg._capi.GdnPrefillArgs), ctypes.c_void_p]
    lib.gdn_prefill_launch_noalloc.restype = ctypes.c_int
    return lib


def _args(pkg, g, out, ns, path):
    C = pkg._capi
    P = lambda t: ctypes.c_void_p(None if t is None else t.data_ptr())  # noqa: E731
    return C.GdnPrefillArgs(
        P(g.q), P(g.k), P(g.v), P(g.state), P(g.A_log), P(g.a), P(g.dt_bias), P(g.b), P(g.cu_seqlens),
        C.GDN_SEQLENS_INT64, path, g.q.shape[0], g.cu_seqlens.numel() - 1, g.scale, P(out), P(ns))


def _noalloc(pkg, g, path):
    lib = _lib(pkg)
    T, N = g.q.shape[0], g.cu_seqlens.numel() - 1
    out = torch.full((T, 8, 128), float("nan"), dtype=torch.bfloat16, device=g.q.device)
    ns = torch.full((N, 8, 128, 128), float("nan"), device=g.q.device)
    args = _args(pkg, g, out, ns, path)
    rc = lib.gdn_prefill_launch_noalloc(ctypes.byref(args),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, pkg._capi.status_string(rc)
    torch.cuda.synchronize()
    return out, ns


@pytest.mark.parametrize("path", ["chunked", "auto"])
def test_noalloc_matches_workspace_entry_point(pkg, cuda_dev, path):
    code = pkg.prefill.PATHS[path]
    # two calls in a row with different shapes: the second reuses the scratch
    # array the first left behind
    for lengths, seed in (([300, 77, 0, 129], 61), ([64, 1, 700], 62)):
        g = pkg.inputs.make_prefill_inputs(lengths, seed=seed, with_state=True).to(cuda_dev)
        ref_out, ref_ns = pkg.prefill.launch_gdn(*g.args(), path=path)
        out, ns = _noalloc(pkg, g, code)
        assert pkg.prefill.device_status(cuda_dev) == 0
        torch.testing.assert_close(out.float(), ref_out.float(), atol=1e-2, rtol=1e-2)
        assert state_rel_err(ns, ref_ns) < 1e-3
        assert torch.isfinite(ns).all()


def test_noalloc_rejects_oversized_problem(pkg, cuda_dev):
    lib = _lib(pkg)
    T = 8192  # one sequence whose workspace exceeds the fixed array
    assert lib.gdn_prefill_workspace_size(T, 1) > NOALLOC_SCRATCH_BYTES
    g = pkg.inputs.make_prefill_inputs([T], seed=63, with_state=False).to(cuda_dev)
    out = torch.zeros((T, 8, 128), dtype=torch.bfloat16, device=cuda_dev)
    ns = torch.zeros((1, 8, 128, 128), device=cuda_dev)
    args = _args(pkg, g, out, ns, pkg.prefill.PATHS["chunked"])
    rc = lib.gdn_prefill_launch_noalloc(ctypes.byref(args), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 4  # GDN_ERR_WORKSPACE: nothing launched
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0 and torch.count_nonzero(ns) == 0
