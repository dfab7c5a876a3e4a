"""Sequence sharding of the GDN paths across GPUs, and the final gather.

Sequences never interact (the oracle loops over them independently: decode
reference_torch_impl.py:52-69, prefill :51-90), so both paths partition by
sequence with no collective in the data path:

* decode: contiguous batch slices, rank r owns rows [B*r/W, B*(r+1)/W);
* prefill: longest-processing-time assignment by token count (longest
  sequence first to the least-loaded rank, ties to the lower rank), each
  rank's sequences packed contiguously with a rebased cu_seqlens and an index
  map back to the global order.

After the step each rank owns its slice of outputs and states; ``gather_*``
brings them to rank 0 (point-to-point sends; over NCCL these ride NVLink) and
restores the global order.  The plan functions are pure host code.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .inputs import DecodeInputs, PrefillInputs

HV, D = 8, 128


# ------------------------------------------------------------------ decode --
def decode_slice(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of a decode batch owned by ``rank``."""
    return batch * rank // world, batch * (rank + 1) // world


def shard_decode_inputs(inp: DecodeInputs, world: int, rank: int) -> DecodeInputs:
    lo, hi = decode_slice(inp.q.shape[0], world, rank)
    return DecodeInputs(inp.q[lo:hi], inp.k[lo:hi], inp.v[lo:hi], inp.state[lo:hi], inp.A_log,
                        inp.a[lo:hi], inp.dt_bias, inp.b[lo:hi], scale=inp.scale)


# ----------------------------------------------------------------- prefill --
@dataclass
class PrefillShard:
    rank: int
    seqs: list[int]          # global sequence indices, in local order
    token_index: torch.Tensor  # int64 [T_local]: global token of each local token
    cu_seqlens: torch.Tensor   # int64 [len(seqs)+1], rebased

    @property
    def tokens(self) -> int:
        return int(self.token_index.numel())


def plan_prefill(lengths, world: int) -> list[list[int]]:
    """LPT assignment of sequences to ranks by token count.

    Returns, per rank, the assigned global sequence indices in increasing
    order (so a rank's packed layout follows the global order).
    """
    load = [0] * world
    owned: list[list[int]] = [[] for _ in range(world)]
    order = sorted(range(len(lengths)), key=lambda s: (-int(lengths[s]), s))
    for s in order:
        r = min(range(world), key=lambda i: (load[i], i))
        owned[r].append(s)
        load[r] += int(lengths[s])
    return [sorted(o) for o in owned]


def make_prefill_shard(cu_seqlens: torch.Tensor, seqs: list[int], rank: int) -> PrefillShard:
    cu = cu_seqlens.to("cpu", torch.int64)
    pieces, lens = [], []
    for s in seqs:
        t0, t1 = int(cu[s]), int(cu[s + 1])
        pieces.append(torch.arange(t0, t1, dtype=torch.int64))
        lens.append(t1 - t0)
    tok = torch.cat(pieces) if pieces else torch.zeros(0, dtype=torch.int64)
    local_cu = torch.zeros(len(seqs) + 1, dtype=torch.int64)
    if lens:
        local_cu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0)
    return PrefillShard(rank, list(seqs), tok, local_cu)


def plan_prefill_shards(cu_seqlens: torch.Tensor, world: int) -> list[PrefillShard]:
    cu = cu_seqlens.to("cpu", torch.int64)
    lengths = (cu[1:] - cu[:-1]).tolist()
    return [make_prefill_shard(cu, seqs, r) for r, seqs in enumerate(plan_prefill(lengths, world))]


def shard_prefill_inputs(inp: PrefillInputs, shard: PrefillShard) -> PrefillInputs:
    """The packed inputs of one shard, on the device of ``inp`` (host tensors
    are then copied to the rank's GPU; device tensors are gathered in place)."""
    ti = shard.token_index.to(inp.q.device)
    sidx = torch.tensor(shard.seqs, dtype=torch.int64, device=inp.q.device)
    state = None if inp.state is None else inp.state.index_select(0, sidx)
    return PrefillInputs(inp.q.index_select(0, ti), inp.k.index_select(0, ti), inp.v.index_select(0, ti),
                         state, inp.A_log, inp.a.index_select(0, ti), inp.dt_bias,
                         inp.b.index_select(0, ti), shard.cu_seqlens.clone(), scale=inp.scale)


def merge_prefill(shards: list[PrefillShard], outputs, states, total_tokens: int, num_seqs: int):
    """Scatter per-shard (output, new_state) back to global order (rank 0)."""
    dev = outputs[0].device
    out = torch.zeros((total_tokens, HV, D), dtype=torch.bfloat16, device=dev)
    ns = torch.zeros((num_seqs, HV, D, D), dtype=torch.float32, device=dev)
    for sh, o, s in zip(shards, outputs, states):
        if sh.tokens:
            out.index_copy_(0, sh.token_index.to(dev), o.to(dev))
        if sh.seqs:
            ns.index_copy_(0, torch.tensor(sh.seqs, dtype=torch.int64, device=dev), s.to(dev))
    return out, ns


# ------------------------------------------------------------------ gather --
def gather_to_rank0(tensors: list[torch.Tensor], shapes_per_rank: list[list[tuple]], rank: int,
                    world: int, group=None):
    """Point-to-point gather of each rank's tensors to rank 0.

    ``shapes_per_rank[r]`` lists the shapes rank r contributes (known to every
    rank from the shared plan, so no size exchange is needed).  Returns, on
    rank 0, a list over ranks of the received tensor lists; elsewhere None.

    Rank 0 posts the receives from every peer at once and the peers their
    sends, as one batch (``batch_isend_irecv``: one NCCL group), so the
    transfers from all peers run concurrently over NVLink into rank 0 rather
    than one peer and one tensor at a time.  Empty tensors are skipped on both
    sides (their shapes are known everywhere).  The call returns once this
    rank's transfers are complete on its current stream.
    """
    import torch.distributed as dist

    ops = []
    got = None
    if rank != 0:
        for t in tensors:
            if t.numel():
                ops.append(dist.P2POp(dist.isend, t.contiguous(), 0, group))
    else:
        got = [list(tensors)]
        for r in range(1, world):
            recv = []
            for shp, like in zip(shapes_per_rank[r], tensors):
                buf = torch.empty(shp, dtype=like.dtype, device=like.device)
                if buf.numel():
                    ops.append(dist.P2POp(dist.irecv, buf, r, group))
                recv.append(buf)
            got.append(recv)
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return got
