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


def _range_summary(inp, s, t0, t1):
    """The affine carry map of tokens [t0, t1) of sequence s, per v-head, in
    float64: S -> S T + Z on the k-last state, where each token applies
    S -> g S (I - beta k k^T) + beta v k^T (oracle prefill: decay, then the
    delta-rule update).  Returns (T, Z), each [8, 128, 128]."""
    import math

    A_log, dt_bias = inp.A_log.double(), inp.dt_bias.double()
    T = torch.eye(128, dtype=torch.float64).repeat(8, 1, 1)
    Z = torch.zeros(8, 128, 128, dtype=torch.float64)
    for t in range(t0, t1):
        for h in range(8):
            x = float(inp.a[t, h]) + float(dt_bias[h])
            sp = x if x > 20 else math.log1p(math.exp(x))
            g = math.exp(-math.exp(float(A_log[h])) * sp)
            beta = 1.0 / (1.0 + math.exp(-float(inp.b[t, h])))
            kk = inp.k[t, h // 2].double()
            for M, add in ((T[h], None), (Z[h], inp.v[t, h].double())):
                M.copy_(g * (M - beta * torch.outer(M @ kk, kk)))
                if add is not None:
                    M.add_(beta * torch.outer(add, kk))
    return T, Z


def _gloo_cp_worker(rank, world, port, q):
    """One context-parallel rank on the CPU: summary of its ranges, all-gather
    over gloo, composition into its start states, the oracle over its tokens."""
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import __graft_entry__
    from oracle import oracle

    pkg = __graft_entry__.load_package()
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        lengths = [150, 200]
        inp = pkg.inputs.make_prefill_inputs(lengths, seed=91, with_state=True)
        cu = [int(x) for x in inp.cu_seqlens]
        parts = pkg.prefill.cp_split(inp.cu_seqlens, world)
        idx, loc = parts[rank]
        mine = torch.stack([torch.stack(_range_summary(inp, s, int(idx[loc[s]]), int(idx[loc[s + 1] - 1]) + 1))
                            for s in range(len(lengths))])  # [N, 2, 8, 128, 128]
        got = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)
        start = inp.state.double().clone()  # composition of ranks 0 .. rank-1 onto the initial state
        for r in range(rank):
            start = start @ got[r][:, 0] + got[r][:, 1]
        pick = lambda t: t[idx]  # noqa: E731
        out, ns = oracle.prefill(pick(inp.q), pick(inp.k), pick(inp.v), start.float(), inp.A_log, pick(inp.a),
                                 inp.dt_bias, pick(inp.b), loc, inp.scale, threads=1)
        ref_out, ref_ns = oracle.prefill(*inp.args(), threads=1)
        err_o = (out.float() - ref_out[idx].float()).abs().max().item()
        ok = err_o < 1e-2
        if rank == world - 1:
            ok = ok and state_rel_err(ns, ref_ns) < 1e-3
        q.put(("ok", rank, ok, err_o, cu))
    except Exception as e:  # reported to the test through the queue
        q.put(("error", rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_cp_protocol_gloo_world2():
    """The context-parallel decomposition over two gloo ranks on the CPU: per
    rank affine summaries, an all-gather, composed start states, and each
    rank's tokens run from its start state match one run over the whole
    batch (outputs 1e-2, final state 1e-3)."""
    import multiprocessing as mp
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_cp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert all(r[0] == "ok" and r[2] for r in res), res


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
], ids=["w2-ragged3", "w3-5000", "w4-ragged4", "w2-130", "w8-9000", "w2-40000", "w3-10x3000"])
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
