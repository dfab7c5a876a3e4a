"""The reference's own GPU kernels (installed unmodified in baseline/_ref by
baseline/install_ref.py) against the oracle, on the box the bench times them.

bench.py reports their speed beside this project's; these tests say what
those reference timings compute.  The reference decode CUDA extension
(kernel.cu::launch_gdn) matches the oracle.  The reference Triton prefill
(triton/kernel.py::launch_gdn) matches it on its direct path (gdn_prefill_kernel_v2:
short sequences, or few of them), within the reference harness's own
tolerance; on its split-WY path (one sequence of 1024+ tokens, or 2-15
sequences of ~240+) and flat-WY path (16+ sequences, 8192+ tokens) its
outputs and final states do not match the oracle with the Triton in this
image (3.6.0).  Those cases are expected failures, kept so that a fixed
reference shows up as XPASS.
"""
import sys

import pytest
import torch

from tests.conftest import REPO, state_rel_err

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(REPO / "baseline"))
import reference_gpu  # noqa: E402

sys.path.pop(0)

_why = reference_gpu.missing()
needs_ref = pytest.mark.skipif(_why is not None, reason=_why or "")


@needs_ref
@pytest.mark.parametrize("B", [1, 3, 8, 64])
def test_reference_decode_matches_oracle(pkg, orc, cuda_dev, B):
    ext = reference_gpu.decode_ext()
    inp = pkg.inputs.make_decode_inputs(B, seed=900 + B)
    ro, rs = orc.decode(*inp.args())
    g = inp.to(cuda_dev)
    out = torch.empty((B, 8, 128), dtype=torch.bfloat16, device=cuda_dev)
    ns = torch.empty_like(g.state)
    ext.launch_gdn(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, g.scale, out, ns)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(), ro.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, rs) < 1e-3


def _ref_prefill(pkg, orc, dev, lengths, seed):
    mod = reference_gpu.prefill_module()
    inp = pkg.inputs.make_prefill_inputs(lengths, seed=seed, with_state=True)
    ro, rs = orc.prefill(*inp.args())
    g = inp.to(dev)
    T, N = g.total_tokens, g.num_seqs
    out = torch.zeros((T, 8, 128), dtype=torch.bfloat16, device=dev)
    ns = torch.zeros((N, 8, 128, 128), device=dev)
    mod.launch_gdn(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, g.cu_seqlens, g.scale, out, ns)
    torch.cuda.synchronize()
    return out, ns, ro, rs


_BROKEN = pytest.mark.xfail(reason="reference Triton split-WY / flat-WY paths disagree with the oracle "
                                   "(Triton 3.6.0, B200)", strict=False)


@needs_ref
@pytest.mark.parametrize("lengths", [
    [64], [300], [300, 77, 129],
    pytest.param([1377], marks=_BROKEN, id="split_wy_1x1377"),
    pytest.param([512] * 4, marks=_BROKEN, id="split_wy_4x512"),
    pytest.param([512] * 16, marks=_BROKEN, id="flat_wy_16x512"),
])
def test_reference_prefill_vs_oracle(pkg, orc, cuda_dev, lengths):
    out, ns, ro, rs = _ref_prefill(pkg, orc, cuda_dev, lengths, seed=len(lengths) + 40)
    # the reference harness's tolerance (bench_fi_timing.py:241-242), state norm-wise
    torch.testing.assert_close(out.float().cpu(), ro.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, rs) < 1e-2
