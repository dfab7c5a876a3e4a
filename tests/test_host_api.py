"""Host-side behaviour of the two launch_gdn drop-ins that needs no GPU:
argument checking (ValueError before any launch) and the input generators."""
import pytest
import torch


def test_decode_rejects_cpu_tensors(pkg):
    d = pkg.inputs.make_decode_inputs(2, seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.decode.launch_gdn(*d.args())


def test_prefill_rejects_cpu_tensors(pkg):
    p = pkg.inputs.make_prefill_inputs([3, 4], seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.prefill.launch_gdn(*p.args())


def test_decode_validate_shapes_and_dtypes(pkg):
    d = pkg.inputs.make_decode_inputs(2, seed=0)
    out = torch.empty(2, 8, 128, dtype=torch.bfloat16)
    ns = torch.empty_like(d.state)
    args = [d.q, d.k, d.v, d.state, d.A_log, d.a, d.dt_bias, d.b, out, ns]
    assert pkg.decode.validate(*args, require_cuda=False) == 2
    bad = list(args)
    bad[0] = d.q.float()
    with pytest.raises(ValueError, match="q must be"):
        pkg.decode.validate(*bad, require_cuda=False)
    bad = list(args)
    bad[3] = d.state.transpose(-1, -2)
    with pytest.raises(ValueError, match="contiguous"):
        pkg.decode.validate(*bad, require_cuda=False)
    bad = list(args)
    bad[8] = torch.empty(2, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="output"):
        pkg.decode.validate(*bad, require_cuda=False)


def test_decode_validate_multi_token(pkg):
    d = pkg.inputs.make_decode_inputs(2, seed=0, tokens=3)
    out = torch.empty(2, 3, 8, 128, dtype=torch.bfloat16)
    ns = torch.empty_like(d.state)
    args = [d.q, d.k, d.v, d.state, d.A_log, d.a, d.dt_bias, d.b, out, ns]
    assert pkg.decode.validate(*args, require_cuda=False) == 2
    bad = list(args)
    bad[8] = torch.empty(2, 8, 128, dtype=torch.bfloat16)  # one token's output for three tokens
    with pytest.raises(ValueError, match="output"):
        pkg.decode.validate(*bad, require_cuda=False)
    bad = list(args)
    bad[2] = d.v[:, :2].contiguous()
    with pytest.raises(ValueError, match="v has"):
        pkg.decode.validate(*bad, require_cuda=False)


def test_decode_validate_bf16_state(pkg):
    d = pkg.inputs.make_decode_inputs(2, seed=0)
    out = torch.empty(2, 8, 128, dtype=torch.bfloat16)
    s16 = d.state.to(torch.bfloat16)
    args = [d.q, d.k, d.v, s16, d.A_log, d.a, d.dt_bias, d.b, out, torch.empty_like(s16)]
    assert pkg.decode.validate(*args, require_cuda=False) == 2
    bad = list(args)
    bad[9] = torch.empty_like(d.state)  # fp32 new_state for a bf16 state
    with pytest.raises(ValueError, match="new_state"):
        pkg.decode.validate(*bad, require_cuda=False)
    m = pkg.inputs.make_decode_inputs(2, seed=0, tokens=2)
    with pytest.raises(ValueError, match="one token"):
        pkg.decode.validate(m.q, m.k, m.v, s16, m.A_log, m.a, m.dt_bias, m.b,
                            torch.empty(2, 2, 8, 128, dtype=torch.bfloat16), torch.empty_like(s16),
                            require_cuda=False)


def test_prefill_validate_seqlens(pkg):
    p = pkg.inputs.make_prefill_inputs([3, 4], seed=0)
    out = torch.empty(7, 8, 128, dtype=torch.bfloat16)
    ns = torch.empty(2, 8, 128, 128)
    args = [p.q, p.k, p.v, p.state, p.A_log, p.a, p.dt_bias, p.b, p.cu_seqlens, out, ns]
    assert pkg.prefill.validate(*args, check_seqlens=True, require_cuda=False) == (7, 2)
    bad = list(args)
    bad[8] = torch.tensor([0, 5, 4], dtype=torch.int64)
    with pytest.raises(ValueError, match="non-decreasing"):
        pkg.prefill.validate(*bad, check_seqlens=True, require_cuda=False)
    bad[8] = torch.tensor([0, 3, 9], dtype=torch.int64)
    with pytest.raises(ValueError, match="exceeds"):
        pkg.prefill.validate(*bad, check_seqlens=True, require_cuda=False)
    bad[8] = torch.tensor([0, 3, 7], dtype=torch.float32)
    with pytest.raises(ValueError, match="int32 or int64"):
        pkg.prefill.validate(*bad, require_cuda=False)
    bad = list(args)
    bad[10] = torch.empty(3, 8, 128, 128)
    with pytest.raises(ValueError, match="new_state"):
        pkg.prefill.validate(*bad, require_cuda=False)


def test_inputs_deterministic(pkg):
    a = pkg.inputs.make_decode_inputs(3, seed=4)
    b = pkg.inputs.make_decode_inputs(3, seed=4)
    for x, y in zip(a.args()[:-1], b.args()[:-1]):
        assert torch.equal(x, y)
    q = a.q.float()
    torch.testing.assert_close(q.norm(dim=-1), torch.ones(3, 1, 4), atol=1e-2, rtol=0)
    assert a.A_log.exp().min() >= 1.0 and a.A_log.exp().max() <= 16.0
    assert torch.count_nonzero(a.dt_bias) == 0


def test_config_shapes(pkg):
    c1 = pkg.inputs.config1()
    assert c1.state.shape == (256, 8, 128, 128)
    lens = pkg.inputs.config3_lengths()
    assert len(lens) == 32 and min(lens) >= 64 and max(lens) <= 2048
    c3 = pkg.inputs.make_prefill_inputs(lens[:2], seed=0)
    assert c3.cu_seqlens.tolist() == [0, lens[0], lens[0] + lens[1]]
