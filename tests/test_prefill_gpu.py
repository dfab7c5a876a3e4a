"""Prefill parity against the CPU oracle (prefill reference_torch_impl.py:17-92).

Bars: bf16 output within atol/rtol 1e-2; fp32 final state within 1e-3
norm-wise relative error.  Edge cases follow the reference's documented
hazards: chunk-boundary lengths, empty sequences, state=None, int32
cu_seqlens, single tokens, and the two BASELINE prefill configs at full size.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.conftest import state_rel_err
from tests.golden.cases import CASES, build_inputs

pytestmark = pytest.mark.gpu

OUT_TOL = dict(atol=1e-2, rtol=1e-2)


@pytest.fixture(params=["recurrent", "chunked", "segmented"])
def path(request):
    """recurrent: token recurrence; chunked: chunked path with its own carry
    choice; segmented: chunked with the segmented (composed) carry forced."""
    return request.param


def _run(pkg, inp, dev, **kw):
    g = inp.to(dev)
    out, ns = pkg.prefill.launch_gdn(*g.args(), **kw)
    torch.cuda.synchronize()
    assert pkg.prefill.device_status(dev) == 0
    return out.cpu(), ns.cpu()


def _check(pkg, orc, inp, dev, **kw):
    ro, rs = orc.prefill(*inp.args())
    out, ns = _run(pkg, inp, dev, **kw)
    torch.testing.assert_close(out.float(), ro.float(), **OUT_TOL)
    assert state_rel_err(ns, rs) < 1e-3
    return out, ns, ro, rs


@pytest.mark.parametrize("lengths", [[1], [15], [16], [17], [63], [64], [65], [127], [128], [129],
                                     [200], [1, 1, 1], [64, 64], [5, 0, 70], [0], [0, 0, 3]])
def test_prefill_lengths(pkg, orc, cuda_dev, lengths, path):
    _check(pkg, orc, pkg.inputs.make_prefill_inputs(lengths, seed=sum(lengths) + 1, with_state=True),
           cuda_dev, path=path)


@pytest.mark.parametrize("lengths", [[33], [300, 7]])
def test_prefill_state_none(pkg, orc, cuda_dev, lengths, path):
    _check(pkg, orc, pkg.inputs.make_prefill_inputs(lengths, seed=41, with_state=False), cuda_dev, path=path)


def test_prefill_int32_cu_seqlens(pkg, orc, cuda_dev, path):
    inp = pkg.inputs.make_prefill_inputs([70, 3, 140], seed=42, with_state=True)
    ro, rs = orc.prefill(*inp.args())
    inp.cu_seqlens = inp.cu_seqlens.to(torch.int32)
    out, ns = _run(pkg, inp, cuda_dev, path=path)
    torch.testing.assert_close(out.float(), ro.float(), **OUT_TOL)
    assert state_rel_err(ns, rs) < 1e-3


def test_prefill_uncovered_tokens_zero(pkg, orc, cuda_dev, path):
    """Tokens past cu_seqlens[-1] get zero output, as the reference's torch.zeros."""
    inp = pkg.inputs.make_prefill_inputs([20, 30], seed=43, with_state=True)
    inp.cu_seqlens = torch.tensor([0, 20, 40], dtype=torch.int64)  # last 10 tokens uncovered
    ro, rs = orc.prefill(*inp.args())
    g = inp.to(cuda_dev)
    out = torch.full((50, 8, 128), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    pkg.prefill.launch_gdn(*g.args(), output=out, path=path)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out[40:]) == 0
    torch.testing.assert_close(out.float().cpu(), ro.float(), **OUT_TOL)


@pytest.mark.parametrize("name", ["prefill_varlen", "prefill_nostate"])
def test_prefill_matches_reference_vectors(pkg, cuda_dev, name, path):
    inp = build_inputs(CASES[name])
    z = np.load(Path(__file__).parent / "golden" / f"{name}.npz")
    out, ns = _run(pkg, inp, cuda_dev, path=path)
    ref_out = torch.from_numpy(z["output"]).view(torch.bfloat16).float()
    torch.testing.assert_close(out.float(), ref_out, **OUT_TOL)
    assert state_rel_err(ns, torch.from_numpy(z["new_state"])) < 1e-3


def test_decode_equals_prefill_t1(pkg, cuda_dev):
    """A batch of T=1 sequences through prefill equals one decode step."""
    d = pkg.inputs.make_decode_inputs(6, seed=44)
    g = d.to(cuda_dev)
    out_d, ns_d = pkg.decode.launch_gdn(*g.args())
    cu = torch.arange(7, dtype=torch.int64, device=cuda_dev)
    out_p, ns_p = pkg.prefill.launch_gdn(g.q[:, 0].contiguous(), g.k[:, 0].contiguous(),
                                         g.v[:, 0].contiguous(), g.state, g.A_log,
                                         g.a[:, 0].contiguous(), g.dt_bias, g.b[:, 0].contiguous(),
                                         cu, g.scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(out_p.float(), out_d.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns_p, ns_d) < 1e-5


def test_prefill_bad_seqlens_reported(pkg, cuda_dev, path):
    """cu_seqlens past T is caught on the device: status bit set, no fault."""
    inp = pkg.inputs.make_prefill_inputs([10, 10], seed=45, with_state=True)
    g = inp.to(cuda_dev)
    g.cu_seqlens = torch.tensor([0, 10, 25], dtype=torch.int64, device=cuda_dev)
    pkg.prefill.launch_gdn(*g.args(), path=path)
    assert pkg.prefill.device_status(cuda_dev) & 16
    assert pkg.prefill.device_status(cuda_dev) == 0  # cleared by the read


def test_prefill_config2(pkg, orc, cuda_dev, path):
    """one sequence of 4096 tokens, zero initial state."""
    _check(pkg, orc, pkg.inputs.config2(with_state=False), cuda_dev, path=path)


def test_prefill_config3(pkg, orc, cuda_dev, path):
    """32 ragged sequences (~33k tokens), non-zero state."""
    _check(pkg, orc, pkg.inputs.config3(), cuda_dev, path=path)


def test_prefill_deterministic(pkg, cuda_dev, path):
    inp = pkg.inputs.make_prefill_inputs([300, 77], seed=46, with_state=True)
    o1, s1 = _run(pkg, inp, cuda_dev, path=path)
    o2, s2 = _run(pkg, inp, cuda_dev, path=path)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


@pytest.mark.parametrize("lengths", [[1000], [2048, 700], [5, 3000, 0], [640, 64, 65, 1],
                                     [1100, 700, 1500, 2048, 1]])
def test_prefill_segmented_long(pkg, orc, cuda_dev, lengths):
    """The segmented carry (sequences split into composed segments) on long
    sequences, uneven segment splits and empty / one-chunk neighbours; with
    1-3 and 4 sequences it runs 4 and 3 segments per chain, with 5 none."""
    _check(pkg, orc, pkg.inputs.make_prefill_inputs(lengths, seed=sum(lengths) + 7, with_state=True),
           cuda_dev, path="segmented")


@pytest.mark.parametrize("lengths", [[4096], [2048] * 2, [2048] * 3, [1536] * 4, [1100] * 6])
def test_prefill_segmented_auto(pkg, orc, cuda_dev, lengths):
    """The automatic choice on long sequences: 1, 2, 3 and 4 of them take the
    segmented carry with 8, 6, 4 and 3 segments per chain on a 148-SM part,
    6 the single pass."""
    _check(pkg, orc, pkg.inputs.make_prefill_inputs(lengths, seed=len(lengths) + 50, with_state=True),
           cuda_dev, path="auto")


@pytest.mark.parametrize("hqk,hv", [(16, 32), (2, 4), (1, 2), (4, 4)])
@pytest.mark.parametrize("hpath", ["recurrent", "chunked", "auto"])
def test_prefill_other_head_counts(pkg, orc, cuda_dev, hqk, hv, hpath):
    """Head counts other than 4 / 8 (the contest's 16 / 32, other grouping
    ratios, one v-head per q/k head) on every path: the chunked tensor-core
    kernels take the counts at run time."""
    inp = pkg.inputs.make_prefill_inputs([33, 0, 70, 1, 130], seed=hv + hqk, with_state=True, hqk=hqk, hv=hv)
    _check(pkg, orc, inp, cuda_dev, path=hpath)


@pytest.mark.parametrize("lengths,hpath", [([2048], "chunked"), ([4096], "auto"), ([700, 1500, 64], "chunked")])
def test_prefill_qk16_v32_long(pkg, orc, cuda_dev, lengths, hpath):
    """The contest's 16 / 32 head layout on long sequences through the chunked
    tensor-core path (single pass, and the automatic choice)."""
    inp = pkg.inputs.make_prefill_inputs(lengths, seed=sum(lengths), with_state=True, hqk=16, hv=32)
    _check(pkg, orc, inp, cuda_dev, path=hpath)


def test_segmented_matches_single_pass(pkg, cuda_dev):
    """Segmented and single-pass carries agree closely on the same batch."""
    inp = pkg.inputs.make_prefill_inputs([1500, 900], seed=48, with_state=True)
    o_s, s_s = _run(pkg, inp, cuda_dev, path="segmented")
    o_c, s_c = _run(pkg, inp, cuda_dev, path="recurrent")
    torch.testing.assert_close(o_s.float(), o_c.float(), **OUT_TOL)
    assert state_rel_err(s_s, s_c) < 1e-3


def test_chunked_matches_recurrent(pkg, cuda_dev):
    """The two CUDA paths agree with each other on a multi-chunk varlen batch."""
    inp = pkg.inputs.make_prefill_inputs([257, 64, 130, 1], seed=47, with_state=True)
    o_r, s_r = _run(pkg, inp, cuda_dev, path="recurrent")
    o_c, s_c = _run(pkg, inp, cuda_dev, path="chunked")
    torch.testing.assert_close(o_c.float(), o_r.float(), **OUT_TOL)
    assert state_rel_err(s_c, s_r) < 1e-3
