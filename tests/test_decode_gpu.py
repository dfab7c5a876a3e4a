"""Decode kernel parity against the CPU oracle (decode reference_torch_impl.py:12-72).

Bars (from the north star): bf16 output within atol/rtol 1e-2 of the oracle's
fp32 output; fp32 new state within 1e-3 norm-wise relative error
(max|got-ref| / max|ref|).
"""
import numpy as np
import pytest
import torch

from tests.conftest import state_rel_err
from tests.golden.cases import CASES, build_inputs

pytestmark = pytest.mark.gpu


def _run(pkg, inp, dev, **kw):
    g = inp.to(dev)
    out, ns = pkg.decode.launch_gdn(*g.args(), **kw)
    torch.cuda.synchronize()
    return out.cpu(), ns.cpu()


@pytest.mark.parametrize("batch", [1, 2, 3, 5, 8, 17, 64, 256])
def test_decode_matches_oracle(pkg, orc, cuda_dev, batch):
    inp = pkg.inputs.make_decode_inputs(batch, seed=100 + batch)
    ro, rs = orc.decode(*inp.args())
    out, ns = _run(pkg, inp, cuda_dev)
    assert out.dtype == torch.bfloat16 and out.shape == (batch, 8, 128)
    torch.testing.assert_close(out.float(), ro, atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, rs) < 1e-3
    # the streaming update is fp32 throughout: far inside the bar
    assert state_rel_err(ns, rs) < 1e-5


@pytest.mark.parametrize("name", ["decode_b2", "decode_b1_scale"])
def test_decode_matches_reference_vectors(pkg, cuda_dev, name):
    """GPU output against the vectors produced by the reference itself."""
    from pathlib import Path

    case = CASES[name]
    inp = build_inputs(case)
    z = np.load(Path(__file__).parent / "golden" / f"{name}.npz")
    out, ns = _run(pkg, inp, cuda_dev)
    torch.testing.assert_close(out.float(), torch.from_numpy(z["output"]), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, torch.from_numpy(z["new_state"])) < 1e-5


def test_decode_in_place(pkg, orc, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(33, seed=7)
    ro, rs = orc.decode(*inp.args())
    g = inp.to(cuda_dev)
    out = torch.empty(33, 1, 8, 128, dtype=torch.bfloat16, device=cuda_dev)  # [B,1,8,128] form
    pkg.decode.launch_gdn(g.q, g.k, g.v, g.state, g.A_log, g.a, g.dt_bias, g.b, g.scale, out, g.state)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.view(33, 8, 128).float().cpu(), ro, atol=1e-2, rtol=1e-2)
    assert state_rel_err(g.state, rs) < 1e-5


@pytest.mark.parametrize("scale", [None, 0.0, 0.05, -0.3])
def test_decode_scale(pkg, orc, cuda_dev, scale):
    inp = pkg.inputs.make_decode_inputs(4, seed=3)
    inp.scale = scale
    ro, rs = orc.decode(*inp.args())
    out, ns = _run(pkg, inp, cuda_dev)
    torch.testing.assert_close(out.float(), ro, atol=1e-2, rtol=1e-2)


def test_decode_deterministic(pkg, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(40, seed=8)
    o1, s1 = _run(pkg, inp, cuda_dev)
    o2, s2 = _run(pkg, inp, cuda_dev)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_decode_empty_batch(pkg, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(0, seed=0)
    out, ns = _run(pkg, inp, cuda_dev)
    assert out.shape == (0, 8, 128) and ns.shape == (0, 8, 128, 128)


def test_decode_large_values_finite(pkg, orc, cuda_dev):
    """Extreme gates: softplus threshold (a > 20) and saturated beta."""
    inp = pkg.inputs.make_decode_inputs(6, seed=21)
    inp.a = (inp.a.float() * 30).to(torch.bfloat16)
    inp.b = (inp.b.float() * 30).to(torch.bfloat16)
    ro, rs = orc.decode(*inp.args())
    out, ns = _run(pkg, inp, cuda_dev)
    assert torch.isfinite(out.float()).all() and torch.isfinite(ns).all()
    torch.testing.assert_close(out.float(), ro, atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns, rs) < 1e-3


@pytest.mark.parametrize("batch,tokens", [(3, 2), (5, 4), (16, 8), (1, 17), (64, 3)])
def test_decode_multi_token_matches_oracle(pkg, orc, cuda_dev, batch, tokens):
    """T tokens per sequence in one call equal the oracle's token recurrence
    over T-token sequences (the prefill oracle with uniform lengths)."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=batch * 31 + tokens, tokens=tokens)
    cu = torch.arange(0, (batch + 1) * tokens, tokens, dtype=torch.int64)
    flat = lambda t: t.reshape(batch * tokens, *t.shape[2:])  # noqa: E731
    ro, rs = orc.prefill(flat(inp.q), flat(inp.k), flat(inp.v), inp.state, inp.A_log, flat(inp.a),
                         inp.dt_bias, flat(inp.b), cu, inp.scale)
    g = inp.to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(*g.args())
    torch.cuda.synchronize()
    assert tuple(out.shape) == (batch, tokens, 8, 128)
    torch.testing.assert_close(out.cpu().float().reshape(batch * tokens, 8, 128), ro.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns.cpu(), rs) < 1e-3


def test_decode_multi_token_matches_steps_and_in_place(pkg, cuda_dev):
    """One T-token call agrees with T single-token calls, also with the state
    updated in place."""
    batch, tokens = 9, 5
    g = pkg.inputs.make_decode_inputs(batch, seed=3, tokens=tokens).to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(*g.args())
    s = g.state.clone()
    for t in range(tokens):
        sl = lambda x: x[:, t:t + 1].contiguous()  # noqa: E731
        o_t, s = pkg.decode.launch_gdn(sl(g.q), sl(g.k), sl(g.v), s, g.A_log, sl(g.a), g.dt_bias, sl(g.b),
                                       g.scale)
        torch.testing.assert_close(out[:, t].float(), o_t.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns.cpu(), s.cpu()) < 1e-5
    inplace = g.state.clone()
    out2, ns2 = pkg.decode.launch_gdn(g.q, g.k, g.v, inplace, g.A_log, g.a, g.dt_bias, g.b, g.scale,
                                      new_state=inplace)
    torch.cuda.synchronize()
    assert torch.equal(out2, out) and torch.equal(inplace, ns)


@pytest.mark.parametrize("batch", [1, 8, 17, 64, 300])
def test_decode_bf16_state(pkg, orc, cuda_dev, batch):
    """The bf16-state variant equals the oracle run on the bf16 state (read
    as fp32), its new state within bf16 rounding (norm-wise 2^-8), also in
    place."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=batch + 11)
    s16 = inp.state.to(torch.bfloat16)
    ro, rs = orc.decode(inp.q, inp.k, inp.v, s16.float(), inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale)
    g = inp.to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(g.q, g.k, g.v, s16.to(cuda_dev), g.A_log, g.a, g.dt_bias, g.b, g.scale)
    torch.cuda.synchronize()
    assert ns.dtype == torch.bfloat16
    torch.testing.assert_close(out.cpu().float(), ro.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns.cpu().float(), rs) < 2 ** -8
    st = s16.to(cuda_dev)
    out2, _ = pkg.decode.launch_gdn(g.q, g.k, g.v, st, g.A_log, g.a, g.dt_bias, g.b, g.scale, new_state=st)
    torch.cuda.synchronize()
    assert torch.equal(out2, out) and torch.equal(st, ns)


@pytest.mark.parametrize("hqk,hv", [(16, 32), (2, 8), (8, 8), (1, 4)])
@pytest.mark.parametrize("tokens", [1, 3])
def test_decode_other_head_counts(pkg, orc, cuda_dev, hqk, hv, tokens):
    """Head counts other than 4 / 8 (e.g. the contest's 16 / 32), one and
    three tokens per step, against the oracle with the same grouping."""
    batch = 6
    inp = pkg.inputs.make_decode_inputs(batch, seed=hqk * 100 + hv + tokens, tokens=tokens, hqk=hqk, hv=hv)
    cu = torch.arange(0, (batch + 1) * tokens, tokens, dtype=torch.int64)
    flat = lambda t: t.reshape(batch * tokens, *t.shape[2:])  # noqa: E731
    ro, rs = orc.prefill(flat(inp.q), flat(inp.k), flat(inp.v), inp.state, inp.A_log, flat(inp.a),
                         inp.dt_bias, flat(inp.b), cu, inp.scale)
    g = inp.to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(*g.args())
    torch.cuda.synchronize()
    assert pkg.prefill.device_status(cuda_dev) == 0
    torch.testing.assert_close(out.cpu().float().reshape(batch * tokens, hv, 128), ro.float(), atol=1e-2,
                               rtol=1e-2)
    assert state_rel_err(ns.cpu(), rs) < 1e-3


def test_decode_other_head_counts_bf16_state(pkg, orc, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(5, seed=9, hqk=16, hv=32)
    s16 = inp.state.to(torch.bfloat16)
    ro, rs = orc.decode(inp.q, inp.k, inp.v, s16.float(), inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale)
    g = inp.to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(g.q, g.k, g.v, s16.to(cuda_dev), g.A_log, g.a, g.dt_bias, g.b, g.scale)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu().float(), ro.float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ns.cpu().float(), rs) < 2 ** -8


@pytest.mark.parametrize("batch,tokens,hqk,hv,bf16", [
    (256, 1, 4, 8, False), (12, 1, 4, 8, False), (64, 3, 4, 8, False), (40, 1, 4, 8, True), (6, 2, 16, 32, False),
    (5, 1, 16, 32, True),
])
def test_prepared_launch_every_form(pkg, cuda_dev, batch, tokens, hqk, hv, bf16):
    """PreparedLaunch (the bench's back-to-back step, one ctypes call per
    launch) computes exactly what launch_gdn computes, for every decode form."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=batch + tokens, tokens=tokens, hqk=hqk, hv=hv).to(cuda_dev)
    st = inp.state.to(torch.bfloat16) if bf16 else inp.state
    ref_out, ref_ns = pkg.decode.launch_gdn(inp.q, inp.k, inp.v, st, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale)
    out, ns = torch.empty_like(ref_out), torch.empty_like(ref_ns)
    launch = pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, st, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                                       out, ns)
    launch()
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)


def test_prepared_launch_rejects_bf16_state_with_tokens(pkg, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(2, seed=1, tokens=2).to(cuda_dev)
    s16 = inp.state.to(torch.bfloat16)
    out = torch.empty((2, 2, 8, 128), dtype=torch.bfloat16, device=cuda_dev)
    with pytest.raises(ValueError):
        pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, s16, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, out,
                                  torch.empty_like(s16))


def test_decode_steps_back_to_back_with_copies_between(pkg, cuda_dev):
    """Decode kernels launch as programmatic dependents of the previous kernel
    in the stream.  Consecutive steps (each reading the state the previous one
    wrote) and steps whose token inputs were just copied up from pinned host
    memory in the same stream, with no synchronisation in between, give the
    bits of the same steps run one at a time."""
    B, steps = 64, 6
    inps = [pkg.inputs.make_decode_inputs(B, seed=300 + i) for i in range(steps)]
    h_tok = [[t.pin_memory() for t in (x.q, x.k, x.v, x.a, x.b)] for x in inps]
    d_tok = [torch.empty_like(t, device=cuda_dev) for t in h_tok[0]]
    A_log, dt_bias = inps[0].A_log.to(cuda_dev), inps[0].dt_bias.to(cuda_dev)
    state0 = inps[0].state.to(cuda_dev)
    # one at a time
    ref_outs, st = [], state0
    for i in range(steps):
        q, k, v, a, b = (t.to(cuda_dev) for t in h_tok[i])
        out, st = pkg.decode.launch_gdn(q, k, v, st, A_log, a, dt_bias, b, inps[0].scale)
        torch.cuda.synchronize()
        ref_outs.append(out.clone())
    ref_state = st.clone()
    # back to back: copy up, decode, next copy, next decode ... one sync at the end
    outs = [torch.empty_like(ref_outs[0]) for _ in range(steps)]
    states = [state0, torch.empty_like(state0), torch.empty_like(state0)]
    for i in range(steps):
        for d, h in zip(d_tok, h_tok[i]):
            d.copy_(h, non_blocking=True)
        pkg.decode.launch_gdn(d_tok[0], d_tok[1], d_tok[2], states[i % 3], A_log, d_tok[3], dt_bias, d_tok[4],
                              inps[0].scale, output=outs[i], new_state=states[(i + 1) % 3])
    torch.cuda.synchronize()
    for i in range(steps):
        assert torch.equal(outs[i], ref_outs[i]), i
    assert torch.equal(states[steps % 3], ref_state)


@pytest.mark.parametrize("batch,slices", [(256, 16), (37, 8), (3, 16)])
def test_host_stager_matches_device_call(pkg, cuda_dev, batch, slices):
    """HostStager (pinned host tensors in and out, state sliced over three
    streams) gives the same bits as one device-side launch_gdn; the same
    stager called twice (the second time with the result as the new input)
    stays equal."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=batch + 5)
    st = pkg.decode.HostStager(batch, cuda_dev, slices=slices)
    h = [t.pin_memory() for t in (inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b)]
    state = h[3]
    for _ in range(2):
        out = torch.empty((batch, 8, 128), dtype=torch.bfloat16).pin_memory()
        ns = torch.empty_like(state).pin_memory()
        st(h[0], h[1], h[2], state, h[4], h[5], h[6], h[7], inp.scale, out, ns)
        torch.cuda.synchronize()
        g = [t.to(cuda_dev) for t in (h[0], h[1], h[2], state, h[4], h[5], h[6], h[7])]
        ref_out, ref_ns = pkg.decode.launch_gdn(*g[:8], scale=inp.scale)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out.cpu()) and torch.equal(ns, ref_ns.cpu())
        state = ns


def test_host_stager_in_place(pkg, cuda_dev):
    """The host state may be updated in place (new_state is state)."""
    batch = 20
    inp = pkg.inputs.make_decode_inputs(batch, seed=77)
    st = pkg.decode.HostStager(batch, cuda_dev, slices=6)
    h = [t.pin_memory() for t in (inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b)]
    g = [t.to(cuda_dev) for t in h]
    ref_out, ref_ns = pkg.decode.launch_gdn(*g, scale=inp.scale)
    out = torch.empty((batch, 8, 128), dtype=torch.bfloat16).pin_memory()
    st(h[0], h[1], h[2], h[3], h[4], h[5], h[6], h[7], inp.scale, out, h[3])
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out.cpu()) and torch.equal(h[3], ref_ns.cpu())
