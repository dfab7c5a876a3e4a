"""Seeded synthetic GDN inputs (stand-ins for the missing contest dataset).

Every tensor is drawn on the CPU from ``torch.Generator().manual_seed(seed)``
in a fixed order, so a given (shape, seed) gives identical bytes on any host
and for any GPU count; callers copy to devices afterwards.

Distributions (the five BASELINE configs):
  q, k  ~ N(0,1), L2-normalised per head along d, then bf16
  v     ~ N(0,1) bf16;  a, b ~ N(0,1) bf16
  A_log = log U[1,16] fp32 [8];  dt_bias = 0 fp32 [8]
  state ~ N(0, 0.02) fp32, k-last [.., 8, 128(V), 128(K)]
  scale = 1/sqrt(128)
Shapes follow the reference definitions: decode q/k [B,1,4,128], v [B,1,8,128],
a/b [B,1,8] (decode reference_torch_impl.py:24-27); prefill q/k [T,4,128],
v [T,8,128], a/b [T,8], cu_seqlens [N+1] (prefill reference_torch_impl.py:18-23).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

NUM_QK_HEADS = 4
NUM_V_HEADS = 8
HEAD_DIM = 128
DEFAULT_SCALE = 1.0 / math.sqrt(HEAD_DIM)


def _qk(gen: torch.Generator, shape) -> torch.Tensor:
    x = torch.randn(shape, generator=gen, dtype=torch.float32)
    x = x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    return x.to(torch.bfloat16)


def _gate_params(gen: torch.Generator, hv: int = NUM_V_HEADS):
    A_log = torch.log(torch.empty(hv, dtype=torch.float32).uniform_(1.0, 16.0, generator=gen))
    dt_bias = torch.zeros(hv, dtype=torch.float32)
    return A_log, dt_bias


@dataclass
class DecodeInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: torch.Tensor
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    scale: float = DEFAULT_SCALE

    def args(self):
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias, self.b,
                self.scale)

    def to(self, device) -> "DecodeInputs":
        return DecodeInputs(*(t.to(device) for t in self.args()[:-1]), scale=self.scale)


@dataclass
class PrefillInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: torch.Tensor | None
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    cu_seqlens: torch.Tensor
    scale: float = DEFAULT_SCALE

    def args(self):
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias, self.b,
                self.cu_seqlens, self.scale)

    def to(self, device) -> "PrefillInputs":
        vals = [None if t is None else t.to(device) for t in self.args()[:-1]]
        return PrefillInputs(*vals, scale=self.scale)

    @property
    def num_seqs(self) -> int:
        return self.cu_seqlens.numel() - 1

    @property
    def total_tokens(self) -> int:
        return self.q.shape[0]


def make_decode_inputs(batch: int, seed: int = 0, tokens: int = 1, hqk: int = NUM_QK_HEADS,
                       hv: int = NUM_V_HEADS) -> DecodeInputs:
    """Decode config 0/1/4a inputs: ``batch`` sequences, ``tokens`` tokens each
    (1 for a plain decode step; more for speculative / multi-token decode);
    ``hqk`` / ``hv`` head counts (4 / 8 in the reference)."""
    gen = torch.Generator().manual_seed(seed)
    q = _qk(gen, (batch, tokens, hqk, HEAD_DIM))
    k = _qk(gen, (batch, tokens, hqk, HEAD_DIM))
    v = torch.randn((batch, tokens, hv, HEAD_DIM), generator=gen).to(torch.bfloat16)
    a = torch.randn((batch, tokens, hv), generator=gen).to(torch.bfloat16)
    b = torch.randn((batch, tokens, hv), generator=gen).to(torch.bfloat16)
    A_log, dt_bias = _gate_params(gen, hv)
    state = torch.randn((batch, hv, HEAD_DIM, HEAD_DIM), generator=gen) * 0.02
    return DecodeInputs(q, k, v, state, A_log, a, dt_bias, b)


def cu_seqlens_from_lengths(lengths) -> torch.Tensor:
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int64)
    if len(lengths):
        cu[1:] = torch.cumsum(torch.as_tensor(list(lengths), dtype=torch.int64), 0)
    return cu


def varlen_lengths(num_seqs: int, lo: int, hi: int, seed: int) -> list[int]:
    """Config 3 lengths: uniform integers in [lo, hi] drawn from the seed."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (num_seqs,), generator=gen).tolist()


def make_prefill_inputs(lengths, seed: int = 0, with_state: bool = True, hqk: int = NUM_QK_HEADS,
                        hv: int = NUM_V_HEADS) -> PrefillInputs:
    """Prefill inputs for sequences of the given lengths, packed via cu_seqlens;
    ``hqk`` / ``hv`` head counts (4 / 8 in the reference)."""
    gen = torch.Generator().manual_seed(seed)
    T = int(sum(lengths))
    N = len(lengths)
    q = _qk(gen, (T, hqk, HEAD_DIM))
    k = _qk(gen, (T, hqk, HEAD_DIM))
    v = torch.randn((T, hv, HEAD_DIM), generator=gen).to(torch.bfloat16)
    a = torch.randn((T, hv), generator=gen).to(torch.bfloat16)
    b = torch.randn((T, hv), generator=gen).to(torch.bfloat16)
    A_log, dt_bias = _gate_params(gen, hv)
    state = None
    if with_state:
        state = torch.randn((N, hv, HEAD_DIM, HEAD_DIM), generator=gen) * 0.02
    return PrefillInputs(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens_from_lengths(lengths))


# The BASELINE configs, by number.
def config0() -> DecodeInputs:
    return make_decode_inputs(8, seed=0)


def config1() -> DecodeInputs:
    return make_decode_inputs(256, seed=0)


def config2(with_state: bool = False) -> PrefillInputs:
    return make_prefill_inputs([4096], seed=0, with_state=with_state)


def config3_lengths(seed: int = 0) -> list[int]:
    return varlen_lengths(32, 64, 2048, seed)


def config3() -> PrefillInputs:
    return make_prefill_inputs(config3_lengths(0), seed=0, with_state=True)
