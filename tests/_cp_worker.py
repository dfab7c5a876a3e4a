"""Worker for tests/test_context_parallel.py: one process per GPU, NCCL.

Every rank builds the same seeded batch, takes its token ranges, runs the
context-parallel prefill, and checks its outputs (and, on the last rank, the
final state) against a single-GPU prefill of the whole batch on its own GPU.
"""
import datetime
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import __graft_entry__  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    pkg = __graft_entry__.load_package()
    ok = True
    for lengths in ([3000, 1024], [8192]):
        inp = pkg.inputs.make_prefill_inputs(lengths, seed=len(lengths) * 7, with_state=True)
        ref_out, ref_ns = pkg.prefill.launch_gdn(*inp.to(dev).args())
        idx, loc = pkg.prefill.cp_split(inp.cu_seqlens, world)[rank]
        pick = lambda t: t[idx].contiguous().to(dev)  # noqa: E731
        out, ns = pkg.prefill.launch_gdn_context_parallel(
            pick(inp.q), pick(inp.k), pick(inp.v), inp.state.to(dev), inp.A_log.to(dev), pick(inp.a),
            inp.dt_bias.to(dev), pick(inp.b), loc.to(dev), inp.scale)
        torch.cuda.synchronize()
        err_o = (out.float() - ref_out[idx.to(dev)].float()).abs().max().item()
        ok = ok and err_o < 1e-2 and pkg.prefill.device_status(dev) == 0
        if rank == world - 1:
            rel = ((ns - ref_ns).abs().max() / ref_ns.abs().max()).item()
            ok = ok and rel < 1e-3
            print(f"rank {rank} lengths {lengths}: out err {err_o:.2e}, state rel {rel:.2e}", flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and int(flag.item()) == 1:
        print("CP OK", flush=True)
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
