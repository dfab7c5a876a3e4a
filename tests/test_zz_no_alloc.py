"""gdn_prefill_launch_noalloc: the prefill entry point for callers that cannot
allocate device memory (a host that owns all device memory and offers no
allocator, or a step where cudaMalloc is not allowed, e.g. under stream
capture).  It must give the same results as gdn_prefill_launch with a
caller-provided workspace, on repeated calls that reuse its fixed scratch
array, on every prefill path; it must accept every problem that runs on the
scratch-free token-recurrent kernel whatever its size, and refuse chunked
problems whose operand records do not fit the array.

Collected last on purpose (file name), so a stopping run has already run
every other test; it also passes alone in a fresh process.
"""
import ctypes
import re

import pytest
import torch

from tests.conftest import REPO, state_rel_err

pytestmark = pytest.mark.gpu


def _scratch_bytes() -> int:
    """GDN_NOALLOC_SCRATCH_BYTES as the header defines it."""
    text = (REPO / "include" / "gdn_b200.h").read_text()
    m = re.search(r"#define\s+GDN_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*<<\s*(\d+)\)", text)
    assert m, "GDN_NOALLOC_SCRATCH_BYTES not found in include/gdn_b200.h"
    return int(m.group(1)) << int(m.group(2))


NOALLOC_SCRATCH_BYTES = _scratch_bytes()
RECORD_BYTES = 8 * 96 * 1024  # operand records per 64-token chunk (8 v-heads)


def _min_workspace(T: int, N: int) -> int:
    """Lower bound of what the chunked paths need: the operand records."""
    return ((T + 63) // 64 + N) * RECORD_BYTES


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


def _check_pair(pkg, dev, lengths, seed, path):
    g = pkg.inputs.make_prefill_inputs(lengths, seed=seed, with_state=True).to(dev)
    ref_out, ref_ns = pkg.prefill.launch_gdn(*g.args(), path=path)
    out, ns = _noalloc(pkg, g, pkg.prefill.PATHS[path])
    assert pkg.prefill.device_status(dev) == 0
    torch.testing.assert_close(out.float(), ref_out.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, ref_ns) < 1e-3
    assert torch.isfinite(ns).all()


# (path, two problems run back to back: the second reuses the array the first left behind)
CASES = {
    "chunked": (([300, 77, 0, 129], 61), ([64, 1, 700], 62)),
    "auto": (([300, 77, 0, 129], 63), ([64, 1, 700], 64)),
    "segmented": (([1000], 65), ([700, 0, 450], 66)),
    "recurrent": (([40, 0, 17], 67), ([5, 9, 130], 68)),
}


@pytest.mark.parametrize("path", sorted(CASES))
def test_noalloc_matches_workspace_entry_point(pkg, cuda_dev, path):
    for lengths, seed in CASES[path]:
        _check_pair(pkg, cuda_dev, lengths, seed, path)


def test_noalloc_recurrent_has_no_size_limit(pkg, cuda_dev):
    """The token recurrence needs no scratch: problems far larger than the
    array run when the path is asked for, and when AUTO picks it (many short
    sequences, whose chunked records would not fit)."""
    assert _min_workspace(8192, 1) > NOALLOC_SCRATCH_BYTES
    _check_pair(pkg, cuda_dev, [8192], 70, "recurrent")
    lengths = [1] * 64  # AUTO: mean length 1 -> recurrent
    assert _min_workspace(64, 64) > NOALLOC_SCRATCH_BYTES
    _check_pair(pkg, cuda_dev, lengths, 71, "auto")
    _check_pair(pkg, cuda_dev, [3, 30, 12, 0] * 20, 72, "auto")


def test_noalloc_between_thresholds_runs_single_pass(pkg, cuda_dev):
    """One 2400-token sequence: its records fit the array, its records plus
    the segmented carry's summaries do not.  It is accepted and runs the
    single-pass carry, matching the segmented run of the workspace entry point."""
    lib = _lib(pkg)
    T = 2400
    assert _min_workspace(T, 1) < NOALLOC_SCRATCH_BYTES < lib.gdn_prefill_workspace_size(T, 1)
    _check_pair(pkg, cuda_dev, [T], 73, "auto")


def test_noalloc_rejects_oversized_problem(pkg, cuda_dev):
    lib = _lib(pkg)
    T = 8192  # one sequence whose chunked records exceed the fixed array
    assert _min_workspace(T, 1) > NOALLOC_SCRATCH_BYTES
    g = pkg.inputs.make_prefill_inputs([T], seed=74, with_state=False).to(cuda_dev)
    for path in ("chunked", "auto", "segmented"):
        out = torch.zeros((T, 8, 128), dtype=torch.bfloat16, device=cuda_dev)
        ns = torch.zeros((1, 8, 128, 128), device=cuda_dev)
        args = _args(pkg, g, out, ns, pkg.prefill.PATHS[path])
        rc = lib.gdn_prefill_launch_noalloc(ctypes.byref(args),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 4, path  # GDN_ERR_WORKSPACE: nothing launched
        torch.cuda.synchronize()
        assert torch.count_nonzero(out) == 0 and torch.count_nonzero(ns) == 0
