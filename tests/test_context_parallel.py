"""Context-parallel prefill (one batch of long sequences split by token range
over ranks).  The host-side split runs on the CPU; the kernels run with the
ranks emulated one after another on one GPU (the all-gather done by copies),
and for real over NCCL when two GPUs are present."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from tests.conftest import state_rel_err

REPO = Path(__file__).resolve().parents[1]


def test_cp_split_covers_every_token(pkg):
    cu = torch.tensor([0, 1000, 1000 + 129, 1000 + 129 + 4096], dtype=torch.int64)
    for world in (1, 2, 3):
        parts = pkg.prefill.cp_split(cu, world)
        got = torch.sort(torch.cat([idx for idx, _ in parts])).values
        assert torch.equal(got, torch.arange(int(cu[-1])))
        for r, (idx, loc) in enumerate(parts):
            assert loc.numel() == 4 and int(loc[-1]) == idx.numel()
            lens = (loc[1:] - loc[:-1]).tolist()
            assert all(x >= 1 for x in lens)
            starts = idx[loc[:-1]] - cu[:-1]  # each range starts on a chunk boundary of its sequence
            assert bool((starts % 64 == 0).all())
    with pytest.raises(ValueError, match="too short"):
        pkg.prefill.cp_split(torch.tensor([0, 100], dtype=torch.int64), 3)


@pytest.mark.parametrize("num_seqs,world", [(1, 1), (1, 2), (1, 8), (2, 2), (3, 4), (20, 2), (1, 64)])
def test_cp_summary_region_layout(pkg, num_seqs, world):
    """The all-gathered region (world blocks of one 98304-byte slot per unit)
    sits at an offset every rank computes alike, followed by the rank's own
    1 to 8 segment slots per unit (one wave of pass A)."""
    for local_tokens in (1, 5000, 70000):
        need = pkg.prefill.cp_workspace_bytes(local_tokens, num_seqs, world)
        off = int(pkg._capi.load().gdn_prefill_cp_summary_offset(local_tokens, num_seqs))
        units = num_seqs * 8
        gathered = world * units * 98304
        assert 0 < off and off + gathered < need and (need - off - gathered) % (units * 98304) == 0
        segs = (need - off - gathered) // (units * 98304)
        assert 1 <= segs <= 8 and (2 * units * segs <= 148 or segs == 1)


def _local(inp, idx, loc, dev):
    pick = lambda t: t[idx].contiguous().to(dev)  # noqa: E731
    return (pick(inp.q), pick(inp.k), pick(inp.v), inp.A_log.to(dev), pick(inp.a), inp.dt_bias.to(dev),
            pick(inp.b), loc.to(dev))


@pytest.mark.gpu
@pytest.mark.parametrize("world,lengths", [
    (2, [1000, 2048, 300]), (3, [5000]), (4, [700, 1500, 260, 4096]),
    (2, [130]),            # rank 0 holds one chunk: 7 of its 8 segments are empty (identity summaries)
    (8, [9000]),           # 8 ranks x 8 segments of 2-3 chunks
    (2, [40000]),          # 8 segments of ~39 chunks per rank
    (3, [3000] * 10),      # one segment per rank: pass A writes the rank summaries itself
])
def test_cp_emulated_matches_single_gpu(pkg, cuda_dev, world, lengths):
    inp = pkg.inputs.make_prefill_inputs(lengths, seed=world * 17 + len(lengths), with_state=True)
    ref_out, ref_ns = pkg.prefill.launch_gdn(*inp.to(cuda_dev).args())
    parts = pkg.prefill.cp_split(inp.cu_seqlens, world)
    N = len(lengths)
    ranks = []
    for r, (idx, loc) in enumerate(parts):
        q, k, v, A_log, a, dt_bias, b, cu = _local(inp, idx, loc, cuda_dev)
        out = torch.empty((q.shape[0], 8, 128), dtype=torch.bfloat16, device=cuda_dev)
        ns = torch.empty((N, 8, 128, 128), device=cuda_dev)
        ws = torch.empty(pkg.prefill.cp_workspace_bytes(q.shape[0], N, world), dtype=torch.uint8, device=cuda_dev)
        st = inp.state.to(cuda_dev) if r == 0 else None
        pkg.prefill.cp_launch(q, k, v, st, A_log, a, dt_bias, b, cu, inp.scale, out, ns, ws, r, world, 0)
        ranks.append((q, k, v, A_log, a, dt_bias, b, cu, out, ns, ws))
    regions = [pkg.prefill.cp_summary_region(rk[10], rk[0].shape[0], N, world) for rk in ranks]
    block = regions[0].numel() // world
    for dst in regions:  # the all-gather
        for r, src in enumerate(regions):
            dst[r * block:(r + 1) * block].copy_(src[r * block:(r + 1) * block])
    for r, (q, k, v, A_log, a, dt_bias, b, cu, out, ns, ws) in enumerate(ranks):
        pkg.prefill.cp_launch(q, k, v, None, A_log, a, dt_bias, b, cu, inp.scale, out, ns, ws, r, world, 1)
    torch.cuda.synchronize()
    assert pkg.prefill.device_status(cuda_dev) == 0
    for r, (idx, _) in enumerate(parts):
        torch.testing.assert_close(ranks[r][8].float(), ref_out[idx.to(cuda_dev)].float(), atol=1e-2, rtol=1e-2)
    assert state_rel_err(ranks[-1][9].cpu(), ref_ns.cpu()) < 1e-3


@pytest.mark.gpu
def test_cp_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, PYTHONPATH=str(REPO))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29617", str(REPO / "tests" / "_cp_worker.py")]
    res = subprocess.run(cmd, env=env, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "CP OK" in res.stdout
