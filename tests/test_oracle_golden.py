"""Pins the C oracle to the reference's own PyTorch implementations.

The golden vectors in tests/golden/*.npz were produced by running the
reference's reference_torch_impl.run (decode :12-72, prefill :17-92) on the
seeded inputs of tests/golden/cases.py (script: tests/golden/gen_golden.py).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.golden.cases import CASES, build_inputs, input_digest

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_vectors(name, orc):
    case = CASES[name]
    inp = build_inputs(case)
    z = np.load(GOLDEN / f"{name}.npz")
    assert bytes(z["digest"]).decode() == input_digest(inp), "input generator changed"
    ref_state = torch.from_numpy(z["new_state"])
    if case["kind"] == "decode":
        out, ns = orc.decode(*inp.args())
        ref_out = torch.from_numpy(z["output"])
        assert out.dtype == torch.float32 and out.shape == ref_out.shape
        # fp32 restatement vs fp32 torch: only summation order differs
        torch.testing.assert_close(out, ref_out, atol=1e-6, rtol=1e-5)
    else:
        out, ns = orc.prefill(*inp.args())
        ref_out = torch.from_numpy(z["output"]).view(torch.bfloat16)
        assert out.dtype == torch.bfloat16 and out.shape == ref_out.shape
        # bf16 rounding of fp32 values that differ in the last fp32 bits: <= 1 bf16
        # ulp, plus an absolute floor for outputs that are fp32 cancellation noise
        diff = (out.float() - ref_out.float()).abs()
        ulp = ref_out.float().abs() * 2.0 ** -7 + 1e-7
        assert bool((diff <= ulp).all())
        assert (diff > 0).float().mean() < 0.01
    assert ns.shape == ref_state.shape
    torch.testing.assert_close(ns, ref_state, atol=1e-6, rtol=1e-5)


def test_oracle_empty_sequence_zero_state(orc, pkg):
    inp = pkg.inputs.make_prefill_inputs([3, 0, 2], seed=9, with_state=True)
    _, ns = orc.prefill(*inp.args())
    assert torch.count_nonzero(ns[1]) == 0
    assert torch.count_nonzero(ns[0]) > 0


def test_oracle_decode_equals_prefill_t1(orc, pkg):
    """Both reference oracles share one step (decode :52-69 vs prefill :66-88)."""
    d = pkg.inputs.make_decode_inputs(3, seed=5)
    out_d, ns_d = orc.decode(*d.args())
    cu = torch.arange(4, dtype=torch.int64)
    out_p, ns_p = orc.prefill(d.q[:, 0], d.k[:, 0], d.v[:, 0], d.state, d.A_log, d.a[:, 0],
                              d.dt_bias, d.b[:, 0], cu, d.scale)
    torch.testing.assert_close(ns_p, ns_d, atol=0, rtol=0)
    torch.testing.assert_close(out_p.float(), out_d.to(torch.bfloat16).float(), atol=0, rtol=0)
