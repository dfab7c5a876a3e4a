"""BASELINE config 4 at its stated size, sharded by sequence over emulated ranks.

(a) decode of B = 4096 sequences (2 GiB of fp32 state) and (b) prefill of 64
sequences x 8192 tokens (524,288 tokens, non-zero initial state), both with
the config-0/2 input distributions.  For W in {2, 4, 8} the problem is split
the way the multi-GPU bench splits it (contiguous decode slices; LPT prefill
shards), every shard runs on cuda:0 one after another (the ranks' kernels
never wait on one another, so no cross-rank synchronisation is emulated),
and the merged result must be BITWISE equal to the unsharded run: the kernels
are deterministic and sequences independent.  One seeded sequence per shard
(W = 8) is also checked against the CPU oracle.
"""
import pytest
import torch

from tests.conftest import state_rel_err

pytestmark = pytest.mark.gpu

WORLDS = (2, 4, 8)


@pytest.fixture(scope="module")
def decode4a(pkg, cuda_dev):
    inp = pkg.inputs.make_decode_inputs(4096, seed=4)
    g = inp.to(cuda_dev)
    out, ns = pkg.decode.launch_gdn(*g.args())
    torch.cuda.synchronize()
    yield inp, g, out, ns
    del g, out, ns
    torch.cuda.empty_cache()


def test_config4a_decode_shards_bitwise(pkg, cuda_dev, decode4a):
    _, g, ref_out, ref_ns = decode4a
    B = g.q.shape[0]
    for W in WORLDS:
        out, ns = torch.empty_like(ref_out), torch.empty_like(ref_ns)
        for r in range(W):
            lo, hi = pkg.shard.decode_slice(B, W, r)
            s = pkg.shard.shard_decode_inputs(g, W, r)
            pkg.decode.launch_gdn(*s.args(), output=out[lo:hi], new_state=ns[lo:hi])
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), W
        assert torch.equal(ns, ref_ns), W


def test_config4a_one_sequence_per_shard_vs_oracle(pkg, orc, decode4a):
    inp, _, ref_out, ref_ns = decode4a
    B = inp.q.shape[0]
    for r in range(8):
        lo, _ = pkg.shard.decode_slice(B, 8, r)
        s = slice(lo, lo + 1)
        ro, rs = orc.decode(inp.q[s], inp.k[s], inp.v[s], inp.state[s], inp.A_log, inp.a[s], inp.dt_bias,
                            inp.b[s], inp.scale)
        torch.testing.assert_close(ref_out[s].float().cpu(), ro.float(), atol=1e-2, rtol=1e-2)
        assert state_rel_err(ref_ns[s], rs) < 1e-3


@pytest.fixture(scope="module")
def prefill4b(pkg, cuda_dev):
    inp = pkg.inputs.make_prefill_inputs([8192] * 64, seed=5, with_state=True)
    g = inp.to(cuda_dev)
    out, ns = pkg.prefill.launch_gdn(*g.args())
    torch.cuda.synchronize()
    yield inp, g, out, ns
    del g, out, ns
    torch.cuda.empty_cache()


def test_config4b_prefill_shards_bitwise(pkg, cuda_dev, prefill4b):
    inp, g, ref_out, ref_ns = prefill4b
    for W in WORLDS:
        shards = pkg.shard.plan_prefill_shards(inp.cu_seqlens, W)
        outs, states = [], []
        for sh in shards:
            part = pkg.shard.shard_prefill_inputs(g, sh)
            part.cu_seqlens = part.cu_seqlens.to(cuda_dev)
            o, s = pkg.prefill.launch_gdn(*part.args())
            outs.append(o)
            states.append(s)
        out, ns = pkg.shard.merge_prefill(shards, outs, states, inp.total_tokens, inp.num_seqs)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), W
        assert torch.equal(ns, ref_ns), W
        del outs, states, out, ns


def test_config4b_one_sequence_per_shard_vs_oracle(pkg, orc, prefill4b):
    inp, _, ref_out, ref_ns = prefill4b
    cu = inp.cu_seqlens
    for sh in pkg.shard.plan_prefill_shards(cu, 8):
        s = sh.seqs[len(sh.seqs) // 2]
        t0, t1 = int(cu[s]), int(cu[s + 1])
        one = pkg.inputs.PrefillInputs(inp.q[t0:t1], inp.k[t0:t1], inp.v[t0:t1], inp.state[s:s + 1], inp.A_log,
                                       inp.a[t0:t1], inp.dt_bias, inp.b[t0:t1],
                                       torch.tensor([0, t1 - t0], dtype=torch.int64), scale=inp.scale)
        ro, rs = orc.prefill(*one.args())
        torch.testing.assert_close(ref_out[t0:t1].float().cpu(), ro.float(), atol=1e-2, rtol=1e-2)
        assert state_rel_err(ref_ns[s:s + 1], rs) < 1e-3
