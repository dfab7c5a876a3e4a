"""Sharded results equal the unsharded run bit for bit (config 4's check).

Ranks are emulated one after another on cuda:0 (no cross-rank waits), which
exercises the same plan / pack / merge code the multi-GPU bench uses.  The
kernels are deterministic and per-sequence independent; shards keep the same
kernel dispatch as the whole batch (chunked path, one carry CTA per sequence
and v-head).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4])
def test_prefill_shards_bitwise(pkg, cuda_dev, world):
    inp = pkg.inputs.make_prefill_inputs([200] * 20, seed=81, with_state=True)
    ref_out, ref_ns = pkg.prefill.launch_gdn(*inp.to(cuda_dev).args())
    shards = pkg.shard.plan_prefill_shards(inp.cu_seqlens, world)
    outs, states = [], []
    for sh in shards:
        g = pkg.shard.shard_prefill_inputs(inp, sh).to(cuda_dev)
        o, s = pkg.prefill.launch_gdn(*g.args())
        outs.append(o)
        states.append(s)
    out, ns = pkg.shard.merge_prefill(shards, outs, states, inp.total_tokens, inp.num_seqs)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)


@pytest.mark.parametrize("world", [2, 8])
def test_decode_shards_bitwise(pkg, cuda_dev, world):
    inp = pkg.inputs.make_decode_inputs(64, seed=82)
    ref_out, ref_ns = pkg.decode.launch_gdn(*inp.to(cuda_dev).args())
    outs, states = [], []
    for r in range(world):
        g = pkg.shard.shard_decode_inputs(inp, world, r).to(cuda_dev)
        o, s = pkg.decode.launch_gdn(*g.args())
        outs.append(o)
        states.append(s)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(outs), ref_out) and torch.equal(torch.cat(states), ref_ns)


def test_prefill_shard_one_sequence_vs_oracle(pkg, orc, cuda_dev):
    """One sequence of a sharded config-4-shaped batch against the CPU oracle."""
    inp = pkg.inputs.make_prefill_inputs([1024] * 8, seed=83, with_state=True)
    sh = pkg.shard.plan_prefill_shards(inp.cu_seqlens, 8)[3]
    part = pkg.shard.shard_prefill_inputs(inp, sh)
    out, ns = pkg.prefill.launch_gdn(*part.to(cuda_dev).args())
    ro, rs = orc.prefill(*part.args())
    torch.testing.assert_close(out.float().cpu(), ro.float(), atol=1e-2, rtol=1e-2)
    err = (ns.cpu() - rs).abs().max() / rs.abs().max()
    assert err < 1e-3
