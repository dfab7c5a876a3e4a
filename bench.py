"""Benchmark of the B200 GDN kernels (one JSON line on rank 0).

Headline (value): GDN decode on BASELINE config 1 -- B=256 sequences per GPU,
one token each, fp32 k-last state [256, 8, 128, 128] -- reported as the
state-stream HBM throughput in GB/s summed over GPUs (weak scaling: every GPU
owns its own 256 sequences; sequences are independent, so there is no
collective in the timed region).  Per-step microseconds are in
``ms_per_step``/``decode_us_per_step``; ``roofline`` relates the step to the
measured copy peak, ``e2e`` times it through the public API with the state in
pinned host memory.

Ride-alongs in the same line: prefill configs 2 and 3 and the 16 / 32-head
layout (one GPU), each with its roofline; ``config4a`` / ``config4b``, BASELINE
config 4 as written (the fixed global problem split over the N ranks, with
and without the final gather to rank 0); for N > 1 the context-parallel
prefill of one 131072-token sequence split by token range over the N GPUs;
on one GPU the reference's own decode and prefill kernels timed beside these
(``reference_gpu``) and the CPU baselines (``cpu_baseline``: the C port;
``cpu_reference_torch``: the reference's PyTorch code).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

Timing: W untimed warm-up steps, then exactly K steps between a barrier and
a device synchronize, timed with CUDA events on the launching stream; the
reported time is the max over ranks.  Decode steps run back to back over three
rotating 128 MiB state buffers (inputs larger than L2, each step pays for its
own write-backs).  Other legs are timed call by call with an L2 flush (a
256 MiB read) before each, outside the events.  ``--impl reference`` times the
reference's own algorithm on the host CPU (the oracle port in oracle/, all
host threads).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
import __graft_entry__  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DECODE_BATCH = 256
STATE_BYTES_PER_SEQ = 8 * 128 * 128 * 4
# algorithmic bytes of one decode step per sequence: state read + write,
# q, k, v, a, b, output (bf16), plus A_log/dt_bias once per launch
DECODE_BYTES_PER_SEQ = 2 * STATE_BYTES_PER_SEQ + 1024 + 1024 + 2048 + 16 + 16 + 2048
DECODE_BYTES_FIXED = 64
# prefill algorithmic bytes per token (q, k, v, a, b read; output written) and
# the fixed chunked-WY FLOP count per token at C = 64 over 8 v-heads
PREFILL_BYTES_PER_TOKEN = 1024 + 1024 + 2048 + 16 + 16 + 2048
PREFILL_FLOPS_PER_TOKEN = 1452715.0
# ncu DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one prefill
# call, summed over its kernels (table, prepare, carry), per leg, from one
# capture of this file's own --workload prefill2 / prefill3 runs
# (profiles/prefill_call_traffic_config2_config3.md); legs without a capture
# report None
PREFILL_NCU_TRAFFIC = {"config2": 28218112, "config3": 1075082752}
L2_FLUSH_BYTES = 256 << 20
SLEEP_CYCLES = 200_000  # ~100 us GPU spin before each timed step (outside the events)
# dram__bytes_read.sum + dram__bytes_write.sum per gdn_decode_kernel launch at
# B=256 in steady state: the mean over launches 21-23 of this file's own
# back-to-back decode loop under ncu --cache-control none (profiles/)
DECODE_NCU_TRAFFIC = 265698133


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {k: d[k] for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def max_over_ranks(x: float, ws: int, device) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws: int):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def flush_l2(buf: torch.Tensor) -> None:
    """Evicts L2 by READING a 256 MiB buffer: the L2 ends up full of clean lines,
    so the next timed kernel neither hits its inputs in L2 nor pays for writing
    back someone else's dirty lines (a write-based flush would charge the
    timed kernel ~126 MB of write-backs)."""
    torch.sum(buf, dtype=torch.float32)


def per_call_ms(times: list[float]) -> float:
    """The per-call device time of a leg: the mean of the middle 80 % of its
    per-call event times.  CUDA event timestamps on the B200 advance in steps
    of about 2 us (short calls time as 6.14, 8.16, 10.18 us ...), so the median
    of a short call is one of two or three grid values; the calls start at
    random against that grid, and the mean of many of them estimates the
    duration to a fraction of a step."""
    t = sorted(times)
    cut = len(t) // 10
    t = t[cut:len(t) - cut] if len(t) > 2 * cut else t
    return sum(t) / len(t)


def time_steps(step, steps: int, warmup: int, ws: int, device, flush: torch.Tensor | None):
    """Runs warmup+steps calls of ``step``; returns (per-step device ms list, wall s)."""
    for _ in range(warmup):
        if flush is not None:
            flush_l2(flush)
        step()
    torch.cuda.synchronize(device)
    barrier(ws)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = time.perf_counter()
    for i in range(steps):
        if flush is not None:
            flush_l2(flush)  # outside the timed events
        # keep the GPU busy while the host enqueues the step, so the start event
        # is not timing host-side launch latency
        torch.cuda._sleep(SLEEP_CYCLES)
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - t0
    barrier(ws)
    return [s.elapsed_time(e) for s, e in evs], wall


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def cpu_decode_baseline(pkg, budget_s: float):
    """The reference algorithm (oracle port, C + OpenMP) on the host, decode B=256."""
    from oracle import oracle

    inp = pkg.inputs.make_decode_inputs(DECODE_BATCH, seed=0)
    threads = cpu_threads()
    oracle.decode(*inp.args(), threads=threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.decode(*inp.args(), threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 200:
            break
    sec = el / n
    return {"value": DECODE_BATCH * STATE_BYTES_PER_SEQ * 2 / sec / 1e9, "unit": "GB/s",
            "us_per_step": sec * 1e6, "cores": threads, "kind": "port",
            "sample": f"{n} full decode steps of config 1 (B=256) through oracle/gdn_oracle.c"}


def cpu_torch_reference(pkg, budget_s: float):
    """The reference's own PyTorch implementation (reference_torch_impl.run,
    unmodified, from baseline/_ref) on the host CPU with every host thread:
    decode config 0 (B = 8) and one config-1 step (B = 256), and prefill of 8
    sequences x 512 tokens -- bounded samples of about ``budget_s`` each."""
    sys.path.insert(0, str(REPO / "baseline"))
    import reference_gpu as rg

    if rg.missing():
        return {"unavailable": rg.missing()}
    threads = cpu_threads()
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        dec = rg.torch_reference("gdn_decode_qk4_v8_d128_k_last")
        pre = rg.torch_reference("gdn_prefill_qk4_v8_d128_k_last")
        res = {"cores": threads, "kind": "reference (reference_torch_impl.run, PyTorch on the host CPU)"}
        for B in (8, DECODE_BATCH):
            inp = pkg.inputs.make_decode_inputs(B, seed=B)
            dec(*inp.args())  # warm
            n, t0 = 0, time.perf_counter()
            while True:
                dec(*inp.args())
                n += 1
                el = time.perf_counter() - t0
                if el >= budget_s / 2 or n >= 50:
                    break
            res[f"decode_B{B}"] = {"ms_per_step": round(el / n * 1e3, 2), "steps": n,
                                   "state_gbs": round(B * STATE_BYTES_PER_SEQ * 2 / (el / n) / 1e9, 3)}
        inp = pkg.inputs.make_prefill_inputs([512] * 8, seed=0, with_state=True)
        n, t0 = 0, time.perf_counter()
        while True:
            pre(*inp.args())
            n += 1
            el = time.perf_counter() - t0
            if el >= budget_s or n >= 20:
                break
        res["prefill_8x512"] = {"tokens_per_s": round(n * inp.total_tokens / el, 1), "calls": n}
        return res
    finally:
        torch.set_num_threads(prev)


def cpu_prefill_baseline(pkg, budget_s: float):
    from oracle import oracle

    threads = cpu_threads()
    inp = pkg.inputs.make_prefill_inputs([512] * 8, seed=0, with_state=True)
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.prefill(*inp.args(), threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 50:
            break
    return {"tokens_per_s": n * inp.total_tokens / el, "cores": threads, "kind": "port",
            "sample": f"{n} x prefill of 8 sequences x 512 tokens through oracle/gdn_oracle.c"}


def bench_prefill(pkg, device, lengths, seed, steps, warmup, ws, flush, peaks, with_state=True,
                  traffic=None, hqk=4, hv=8):
    inp = pkg.inputs.make_prefill_inputs(lengths, seed=seed, with_state=with_state, hqk=hqk, hv=hv).to(device)
    T, N = inp.total_tokens, inp.num_seqs
    out = torch.empty((T, hv, 128), dtype=torch.bfloat16, device=device)
    ns = torch.empty((N, hv, 128, 128), dtype=torch.float32, device=device)
    ws_bytes = pkg.prefill.workspace_bytes(T, N, hv)
    wsb = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)

    def step():
        pkg.prefill.launch_gdn(*inp.args(), output=out, new_state=ns, workspace=wsb)

    times, _ = time_steps(step, steps, warmup, ws, device, flush)
    ms = max_over_ranks(per_call_ms(times), ws, device)
    # per token: q, k (hqk heads) and v, a, b, output (hv heads); states hv x 64 KiB per sequence
    per_tok = 2 * hqk * 256 + hv * (256 + 2 + 2 + 256)
    bytes_ = per_tok * T + (hv // 8) * STATE_BYTES_PER_SEQ * N * (2 if with_state else 1)
    flops = PREFILL_FLOPS_PER_TOKEN * (hv / 8) * T
    res = {"tokens": T, "seqs": N, "ms": ms, "tokens_per_s": T * ws / (ms * 1e-3),
           "algo_bytes": bytes_, "algo_flops": flops,
           "hbm_gbs": bytes_ / (ms * 1e-3) / 1e9, "tflops": flops / (ms * 1e-3) / 1e12,
           "roofline": prefill_roofline(bytes_, flops, ms, peaks, traffic)}
    if (hqk, hv) != (4, 8):
        res["heads"] = [hqk, hv]
    return res


def prefill_roofline(algo_bytes: float, algo_flops: float, ms: float, peaks: dict, traffic=None) -> dict:
    """Roofline of one prefill call: the bound is whichever of the HBM floor
    (algorithmic bytes / measured copy bandwidth) and the tensor floor
    (algorithmic FLOPs / measured bf16 burst GEMM rate) is longer; both
    fractions are given.  ``traffic``: ncu DRAM bytes of one call (summed over
    its kernels), or None where no capture covers the leg."""
    t_hbm = algo_bytes / (peaks["hbm_gbs"] * 1e9)
    t_tc = algo_flops / (peaks["bf16_tflops"] * 1e12)
    hbm_gbs = algo_bytes / (ms * 1e-3) / 1e9
    tflops = algo_flops / (ms * 1e-3) / 1e12
    if t_hbm >= t_tc:
        r = {"bound": "hbm", "achieved": round(hbm_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
             "frac": round(hbm_gbs / peaks["hbm_gbs"], 4)}
    else:
        r = {"bound": "tensor", "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
             "frac": round(tflops / peaks["bf16_tflops"], 4)}
    r.update({"hbm_frac": round(hbm_gbs / peaks["hbm_gbs"], 4),
              "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
              "floor_us": round(max(t_hbm, t_tc) * 1e6, 2), "traffic": traffic,
              "algo": "bytes = 6176 x tokens + 512 KiB x seqs x (1 + initial state); "
                      "flops = 1,452,715 x tokens (chunked WY at C = 64, 8 v-heads)"})
    return r


def bench_prefill_cp(pkg, device, rank, ws, lengths, steps, warmup, flush, peaks):
    """Context-parallel prefill (N > 1): the SAME batch split by token range
    over the ranks (strong scaling), timed per call as max over ranks and
    compared with one GPU running the whole batch."""
    full = pkg.inputs.make_prefill_inputs(lengths, seed=7, with_state=True)
    idx, loc = pkg.prefill.cp_split(full.cu_seqlens, ws)[rank]
    pick = lambda t: t[idx].contiguous().to(device)  # noqa: E731
    q, k, v, a, b = pick(full.q), pick(full.k), pick(full.v), pick(full.a), pick(full.b)
    st, A_log, dt_bias, cu = (full.state.to(device), full.A_log.to(device), full.dt_bias.to(device),
                              loc.to(device))
    N = len(lengths)
    out = torch.empty((q.shape[0], 8, 128), dtype=torch.bfloat16, device=device)
    ns = torch.empty((N, 8, 128, 128), dtype=torch.float32, device=device)
    wsb = torch.empty(pkg.prefill.cp_workspace_bytes(q.shape[0], N, ws), dtype=torch.uint8, device=device)

    def step():
        pkg.prefill.launch_gdn_context_parallel(q, k, v, st, A_log, a, dt_bias, b, cu, full.scale, out, ns,
                                                workspace=wsb)

    times, _ = time_steps(step, steps, warmup, ws, device, flush)
    ms = max_over_ranks(per_call_ms(times), ws, device)
    del q, k, v, a, b, out, wsb
    one = bench_prefill(pkg, device, lengths, 7, steps, warmup, ws, flush, peaks)  # every rank: all of it
    T = int(full.cu_seqlens[-1])
    return {"lengths": lengths, "tokens": T, "ms": ms, "tokens_per_s": T / (ms * 1e-3),
            "one_gpu_ms": one["ms"], "speedup_vs_one_gpu": one["ms"] / ms,
            "scaling": "strong (one batch over all ranks)"}


def bench_decode_small(pkg, device, flush, batches=(1, 8, 16, 32, 64), steps=60):
    """Per-call device time (per_call_ms, L2 flushed, us) of one decode step at the
    small batch sizes the reference's published decode numbers cover (B <= 64),
    where the step is latency- rather than bandwidth-bound."""
    res = {}
    for B in batches:
        inp = pkg.inputs.make_decode_inputs(B, seed=B).to(device)
        out = torch.empty((B, 8, 128), dtype=torch.bfloat16, device=device)
        ns = torch.empty_like(inp.state)
        launch = pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b,
                                           inp.scale, out, ns)
        times, _ = time_steps(launch, steps, 3, 1, device, flush)
        res[str(B)] = round(per_call_ms(times) * 1e3, 2)
    return res


def rotating_states(state: torch.Tensor) -> list[torch.Tensor]:
    """Three state buffers for back-to-back steps (step i reads buffer i % 3
    and writes (i + 1) % 3): every step reads a state that misses L2 and pays
    for its own write-backs, as in the config-1 leg."""
    return [state, torch.empty_like(state), torch.empty_like(state)]


def bench_decode_tokens(pkg, device, flush, batch=256, tokens=(2, 4, 8), steps=20):
    """Multi-token (speculative) decode at config 1's batch: T tokens per
    sequence in one call; the state is read and written once per call, so the
    state-stream GB/s stays near the single-token step's.  Per call with the
    L2 flushed, and back to back over rotating state buffers (the config-1
    leg's steady state)."""
    res = {}
    for T in tokens:
        inp = pkg.inputs.make_decode_inputs(batch, seed=T, tokens=T).to(device)
        out = torch.empty((batch, T, 8, 128), dtype=torch.bfloat16, device=device)
        st = rotating_states(inp.state)
        launches = [pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, st[i], inp.A_log, inp.a, inp.dt_bias, inp.b,
                                              inp.scale, out, st[(i + 1) % 3]) for i in range(3)]
        it = [0]

        def step():
            launches[it[0] % 3]()
            it[0] += 1

        times, _ = time_steps(step, steps, 3, 1, device, flush)
        ms = per_call_ms(times)
        bb, _ = time_back_to_back(step, 30, 6, 1, device)
        res[str(T)] = {"us_per_call": round(ms * 1e3, 2), "us_per_token": round(ms * 1e3 / T, 2),
                       "state_gbs": round(batch * STATE_BYTES_PER_SEQ * 2 / (ms * 1e-3) / 1e9, 1),
                       "us_per_call_back_to_back": round(bb * 1e3, 2),
                       "state_gbs_back_to_back": round(batch * STATE_BYTES_PER_SEQ * 2 / (bb * 1e-3) / 1e9, 1)}
    return res


def bench_decode_bf16(pkg, device, flush, batch=256, steps=20):
    """Config 1's step with the state stored in bf16 (half the state stream)."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=7).to(device)
    st = rotating_states(inp.state.to(torch.bfloat16))
    out = torch.empty((batch, 8, 128), dtype=torch.bfloat16, device=device)
    launches = [pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, st[i], inp.A_log, inp.a, inp.dt_bias, inp.b,
                                          inp.scale, out, st[(i + 1) % 3]) for i in range(3)]
    it = [0]

    def step():
        launches[it[0] % 3]()
        it[0] += 1

    times, _ = time_steps(step, steps, 3, 1, device, flush)
    ms = per_call_ms(times)
    bb, _ = time_back_to_back(step, 30, 6, 1, device)
    return {"batch": batch, "us_per_step": round(ms * 1e3, 2),
            "state_gbs": round(batch * STATE_BYTES_PER_SEQ / (ms * 1e-3) / 1e9, 1),
            "us_per_step_back_to_back": round(bb * 1e3, 2),
            "state_gbs_back_to_back": round(batch * STATE_BYTES_PER_SEQ / (bb * 1e-3) / 1e9, 1),
            "note": "state bytes = 2 x B x 256 KiB (bf16), read and written once; device time, per call with "
                    "the L2 flushed, and back to back over three rotating state buffers"}


def bench_decode_heads(pkg, device, flush, batch=64, hqk=16, hv=32, steps=20):
    """The contest's other head layout (16 q/k, 32 v heads): one step of
    ``batch`` sequences (2 MiB of fp32 state each)."""
    inp = pkg.inputs.make_decode_inputs(batch, seed=3, hqk=hqk, hv=hv).to(device)
    out = torch.empty((batch, hv, 128), dtype=torch.bfloat16, device=device)
    ns = torch.empty_like(inp.state)

    def step():
        pkg.decode.launch_gdn(*inp.args(), output=out, new_state=ns)

    times, _ = time_steps(step, steps, 3, 1, device, flush)
    ms = per_call_ms(times)
    state_bytes = 2 * inp.state.numel() * 4
    return {"batch": batch, "heads": [hqk, hv], "us_per_step": round(ms * 1e3, 2),
            "state_gbs": round(state_bytes / (ms * 1e-3) / 1e9, 1)}


def device_decode_inputs(pkg, batch: int, seed: int, device):
    """Config-0 distributions drawn directly on the GPU (fast at 2 GiB of
    state; the timing does not depend on the values)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def qk(shape):
        x = torch.randn(shape, generator=g, device=device)
        return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)

    q, k = qk((batch, 1, 4, 128)), qk((batch, 1, 4, 128))
    v = torch.randn((batch, 1, 8, 128), generator=g, device=device).to(torch.bfloat16)
    a = torch.randn((batch, 1, 8), generator=g, device=device).to(torch.bfloat16)
    b = torch.randn((batch, 1, 8), generator=g, device=device).to(torch.bfloat16)
    A_log = torch.log(torch.empty(8, device=device).uniform_(1.0, 16.0, generator=g))
    dt_bias = torch.zeros(8, device=device)
    state = torch.randn((batch, 8, 128, 128), generator=g, device=device) * 0.02
    return pkg.inputs.DecodeInputs(q, k, v, state, A_log, a, dt_bias, b)


def device_prefill_inputs(pkg, lengths, seed: int, device, with_state=True):
    """Config-2 distributions for packed sequences, drawn on the GPU."""
    g = torch.Generator(device=device).manual_seed(seed)
    T, N = int(sum(lengths)), len(lengths)

    def qk(shape):
        x = torch.randn(shape, generator=g, device=device)
        return (x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)).to(torch.bfloat16)

    q, k = qk((T, 4, 128)), qk((T, 4, 128))
    v = torch.randn((T, 8, 128), generator=g, device=device).to(torch.bfloat16)
    a = torch.randn((T, 8), generator=g, device=device).to(torch.bfloat16)
    b = torch.randn((T, 8), generator=g, device=device).to(torch.bfloat16)
    A_log = torch.log(torch.empty(8, device=device).uniform_(1.0, 16.0, generator=g))
    dt_bias = torch.zeros(8, device=device)
    state = torch.randn((N, 8, 128, 128), generator=g, device=device) * 0.02 if with_state else None
    cu = pkg.inputs.cu_seqlens_from_lengths(lengths).to(device)
    return pkg.inputs.PrefillInputs(q, k, v, state, A_log, a, dt_bias, b, cu)


def time_gather_median(pkg, tensors, shapes, ws, device, reps=3):
    """The final gather of every rank's outputs and states to rank 0 (NCCL
    point-to-point, every peer's transfers concurrent), device time of the
    median of ``reps`` gathers, max over ranks."""
    rank = int(os.environ.get("RANK", "0"))
    if ws == 1:
        return {"gather_ms": 0.0, "gather_bytes": 0}
    stream = torch.cuda.current_stream(device)
    pkg.shard.gather_to_rank0(tensors, shapes, rank, ws)  # warm the P2P paths
    torch.cuda.synchronize(device)
    times = []
    for _ in range(reps):
        barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        got = pkg.shard.gather_to_rank0(tensors, shapes, rank, ws)
        e1.record(stream)
        torch.cuda.synchronize(device)
        del got
        times.append(e0.elapsed_time(e1))
    ms = max_over_ranks(sorted(times)[len(times) // 2], ws, device)
    moved = sum(math.prod(s) * t.element_size() for r in range(1, ws) for s, t in zip(shapes[r], tensors))
    return {"gather_ms": ms, "gather_bytes": moved, "gather_gbs_into_rank0": moved / (ms * 1e-3) / 1e9}


def bench_config4a(pkg, device, rank, ws, steps, warmup, peaks):
    """BASELINE config 4a: decode of B = 4096 sequences (2 GiB of fp32 state)
    split by sequence over the ranks -- the FIXED global problem (strong
    scaling).  Steps run back to back over two state buffers (read one, write
    the other; each rank's slice is larger than L2 up to N = 8), max over
    ranks; then the gather of outputs and states to rank 0."""
    B = 4096
    lo, hi = pkg.shard.decode_slice(B, ws, rank)
    inp = device_decode_inputs(pkg, hi - lo, 4000 + rank, device)
    out = torch.empty((hi - lo, 8, 128), dtype=torch.bfloat16, device=device)
    st = [inp.state, torch.empty_like(inp.state)]
    launches = [pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, st[i], inp.A_log, inp.a, inp.dt_bias, inp.b,
                                          inp.scale, out, st[1 - i]) for i in range(2)]
    it = [0]

    def step():
        launches[it[0] % 2]()
        it[0] += 1

    ms_local, _ = time_back_to_back(step, steps, warmup, ws, device)
    ms = max_over_ranks(ms_local, ws, device)
    shapes = [[(pkg.shard.decode_slice(B, ws, r)[1] - pkg.shard.decode_slice(B, ws, r)[0], 8, 128),
               (pkg.shard.decode_slice(B, ws, r)[1] - pkg.shard.decode_slice(B, ws, r)[0], 8, 128, 128)]
              for r in range(ws)]
    gat = time_gather_median(pkg, [out, st[it[0] % 2]], shapes, ws, device)
    state_bytes = 2 * B * STATE_BYTES_PER_SEQ
    algo_local = DECODE_BYTES_PER_SEQ * (hi - lo) + DECODE_BYTES_FIXED
    achieved = algo_local / (ms_local * 1e-3) / 1e9
    res = {"batch": B, "per_rank": hi - lo, "ms": ms, "us_per_step": round(ms * 1e3, 2),
           "state_gbs": state_bytes / (ms * 1e-3) / 1e9,
           "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": round(achieved / peaks["hbm_gbs"], 4), "per": "rank (rank-local step time)"},
           **gat}
    res["ms_with_gather"] = ms + res["gather_ms"]
    res["state_gbs_with_gather"] = state_bytes / (res["ms_with_gather"] * 1e-3) / 1e9
    return res


def bench_config4b(pkg, device, rank, ws, steps, warmup, flush, peaks):
    """BASELINE config 4b: prefill of 64 sequences x 8192 tokens (524,288
    tokens) split by sequence over the ranks (LPT plan) -- the FIXED global
    problem (strong scaling).  Per-call device time with the L2 flushed
    before each call, per_call_ms, max over ranks; then the gather of outputs and
    states to rank 0."""
    lengths = [8192] * 64
    plan = pkg.shard.plan_prefill(lengths, ws)
    mine = [lengths[s] for s in plan[rank]]
    res = {"seqs": 64, "tokens": sum(lengths), "per_rank_seqs": len(mine)}
    if mine:
        inp = device_prefill_inputs(pkg, mine, 5000 + rank, device)
        T, N = inp.total_tokens, inp.num_seqs
        out = torch.empty((T, 8, 128), dtype=torch.bfloat16, device=device)
        ns = torch.empty((N, 8, 128, 128), dtype=torch.float32, device=device)
        wsb = torch.empty(max(pkg.prefill.workspace_bytes(T, N), 1), dtype=torch.uint8, device=device)

        def step():
            pkg.prefill.launch_gdn(*inp.args(), output=out, new_state=ns, workspace=wsb)
    else:  # more ranks than sequences: this rank idles but joins every collective
        out = torch.empty((0, 8, 128), dtype=torch.bfloat16, device=device)
        ns = torch.empty((0, 8, 128, 128), dtype=torch.float32, device=device)

        def step():
            pass
    times, _ = time_steps(step, steps, warmup, ws, device, flush)
    ms_local = per_call_ms(times)
    ms = max_over_ranks(ms_local, ws, device)
    shapes = [[(sum(lengths[s] for s in plan[r]), 8, 128), (len(plan[r]), 8, 128, 128)] for r in range(ws)]
    gat = time_gather_median(pkg, [out, ns], shapes, ws, device)
    T_all = sum(lengths)
    tok_local = sum(mine)
    flops = PREFILL_FLOPS_PER_TOKEN * tok_local
    bytes_ = PREFILL_BYTES_PER_TOKEN * tok_local + STATE_BYTES_PER_SEQ * len(mine) * 2
    roof = prefill_roofline(bytes_, flops, ms_local, peaks, PREFILL_NCU_TRAFFIC.get("config4b_rank8x8192")
                            if len(mine) == 8 else None) if mine else None
    if roof:
        roof["per"] = "rank (its shard's bytes and FLOPs over its own call time)"
    res.update({"ms": ms, "tokens_per_s": T_all / (ms * 1e-3), "roofline": roof, **gat})
    res["ms_with_gather"] = ms + res["gather_ms"]
    res["tokens_per_s_with_gather"] = T_all / (res["ms_with_gather"] * 1e-3)
    return res


def split_total(total: int, parts: int, seed: int) -> list[int]:
    """``parts`` positive lengths summing to ``total`` (seeded random cut points):
    the published prefill shapes give only T and N."""
    gen = torch.Generator().manual_seed(seed)
    cuts = sorted(torch.randperm(total - 1, generator=gen)[: parts - 1].add(1).tolist())
    edges = [0] + cuts + [total]
    return [edges[i + 1] - edges[i] for i in range(parts)]


# Prefill shapes timed against the reference's Triton kernel
# and 3, a config-4b shard, and the reference's published shapes (T, N) from
# its experiment log (lengths within a batch are not published: seeded split).
REF_PREFILL_SHAPES = {
    "config2_T4096_N1": ([4096], False),
    "config3_32seq": (None, True),
    "pub_T1377_N1": ([1377], True),
    "pub_T2107_N1": ([2107], True),
    "pub_T5709_N2": (split_total(5709, 2, 5709), True),
    "pub_T8192_N34": (split_total(8192, 34, 8192), True),
    "config4b_shard_8x8192": ([8192] * 8, True),
}
REF_DECODE_BATCHES = (1, 8, 16, 32, 64, 256)


def agreement(ro, rns, out, ns) -> dict:
    """How the reference kernel's output and state compare with this project's
    (which the GPU tests hold to the oracle): max abs output difference, the
    norm-wise state difference, and whether both are within the reference
    harness's own tolerance (allclose atol = rtol = 1e-2, bench_fi_timing.py:241-242)."""
    od = float((ro.float() - out.float()).abs().max())
    sd = float((rns - ns).abs().max() / ns.abs().max().clamp_min(1e-30))
    ok = bool(torch.allclose(ro.float(), out.float(), atol=1e-2, rtol=1e-2)) and sd <= 1e-2
    return {"out_max_abs_diff": od, "state_rel_diff": sd, "ref_within_tolerance": ok}


def bench_reference_gpu(pkg, device, flush, steps=20, prefill=True):
    """The reference's own GPU kernels beside this project's, same box, same
    run, same timing (per-call CUDA events, L2 flushed by a 256 MiB read
    before every call, per_call_ms): the reference decode extension
    (``kernel.cu::launch_gdn``) at the contest's batch sizes and config 1, and
    the reference Triton prefill (``kernel.py::launch_gdn``) on configs 2/3 and
    its published shapes.  Each reference output is compared with this
    project's output for the same inputs (this project's is oracle-checked by
    the GPU tests)."""
    sys.path.insert(0, str(REPO / "baseline"))
    import reference_gpu as rg

    why = rg.missing()
    if why:
        return {"unavailable": why}
    res = {"how": "per-call device time (CUDA events, mean of the middle 80 % of the calls), L2 flushed "
                  "before each call; "
                  "ratio = reference time / this project's time (>1: this project is faster)"}
    dec = {}
    ext = rg.decode_ext()
    for B in REF_DECODE_BATCHES:
        inp = pkg.inputs.make_decode_inputs(B, seed=500 + B).to(device)
        out, ns = torch.empty((B, 8, 128), dtype=torch.bfloat16, device=device), torch.empty_like(inp.state)
        ro, rns = torch.empty_like(out), torch.empty_like(inp.state)
        ours = pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b,
                                         inp.scale, out, ns)

        def ref():
            ext.launch_gdn(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale, ro, rns)

        t_ref, _ = time_steps(ref, 3 * steps, 3, 1, device, flush)  # short calls: more samples
        t_our, _ = time_steps(ours, 3 * steps, 3, 1, device, flush)
        mr, mo = per_call_ms(t_ref) * 1e3, per_call_ms(t_our) * 1e3
        dec[str(B)] = {"ref_us": round(mr, 2), "ours_us": round(mo, 2), "ratio": round(mr / mo, 3),
                       **agreement(ro, rns, out, ns)}
    res["decode_vs_reference_cuda"] = dec
    if not prefill:
        return res
    pre = {}
    try:
        mod = rg.prefill_module()
    except Exception as e:  # noqa: BLE001  (reported in the line, not fatal)
        res["prefill_vs_reference_triton"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        return res
    for name, (lengths, with_state) in REF_PREFILL_SHAPES.items():
        lengths = lengths if lengths is not None else pkg.inputs.config3_lengths(0)
        inp = pkg.inputs.make_prefill_inputs(lengths, seed=len(lengths) * 7 + 1, with_state=with_state).to(device)
        T, N = inp.total_tokens, inp.num_seqs
        out = torch.empty((T, 8, 128), dtype=torch.bfloat16, device=device)
        ns = torch.empty((N, 8, 128, 128), dtype=torch.float32, device=device)
        ro, rns = torch.empty_like(out), torch.empty_like(ns)
        wsb = torch.empty(max(pkg.prefill.workspace_bytes(T, N), 1), dtype=torch.uint8, device=device)

        def ours():
            pkg.prefill.launch_gdn(*inp.args(), output=out, new_state=ns, workspace=wsb)

        def ref():
            mod.launch_gdn(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.cu_seqlens,
                           inp.scale, ro, rns)

        try:
            t_ref, _ = time_steps(ref, steps, 3, 1, device, flush)
        except Exception as e:  # noqa: BLE001
            pre[name] = {"tokens": T, "seqs": N, "error": f"{type(e).__name__}: {str(e)[:200]}"}
            continue
        t_our, _ = time_steps(ours, steps, 3, 1, device, flush)
        mr, mo = per_call_ms(t_ref) * 1e3, per_call_ms(t_our) * 1e3
        pre[name] = {"tokens": T, "seqs": N, "ref_us": round(mr, 1), "ours_us": round(mo, 1),
                     "ref_mtok_s": round(T / mr, 2), "ours_mtok_s": round(T / mo, 2), "ratio": round(mr / mo, 3),
                     **agreement(ro, rns, out, ns)}
    res["prefill_vs_reference_triton"] = pre
    return res


def soak(step, seconds: float, device, flush):
    """Untimed repeats of ``step`` so the clock sampler sees the GPU under this load."""
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for _ in range(20):
            if flush is not None:
                flush_l2(flush)
            step()
        torch.cuda.synchronize(device)


def time_back_to_back(step, steps: int, warmup: int, ws: int, device):
    """K steps issued back to back between one event pair (steady state)."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(ws)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(SLEEP_CYCLES)  # the queue fills while the GPU spins
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - t0
    barrier(ws)
    return e0.elapsed_time(e1) / steps, wall


def bench_decode(pkg, args, device, ws, rank, flush, peaks, peaks_kind):
    """Config 1 decode, steady state: three rotating 128 MiB state buffers (step
    i reads buffer i%3 and writes (i+1)%3), so every state read misses L2 and
    every step pays for its own write-backs; K steps back to back."""
    B = DECODE_BATCH
    inp = pkg.inputs.make_decode_inputs(B, seed=1000 + rank).to(device)
    out = torch.empty((B, 8, 128), dtype=torch.bfloat16, device=device)
    st = [inp.state, torch.empty_like(inp.state), torch.empty_like(inp.state)]
    launches = [pkg.decode.PreparedLaunch(inp.q, inp.k, inp.v, st[i], inp.A_log, inp.a, inp.dt_bias,
                                          inp.b, inp.scale, out, st[(i + 1) % 3]) for i in range(3)]
    it = [0]

    def step():
        launches[it[0] % 3]()
        it[0] += 1

    with ClockSampler(device.index) as clk:
        if args.soak > 0:
            soak(step, args.soak, device, None)
        ms_local, wall = time_back_to_back(step, args.steps, args.warmup, ws, device)
    ms = max_over_ranks(ms_local, ws, device)
    state_bytes = B * STATE_BYTES_PER_SEQ * 2
    algo_bytes = DECODE_BYTES_PER_SEQ * B + DECODE_BYTES_FIXED
    res = {
        "ms": ms, "ms_local": ms_local, "wall": wall, "clocks": clk.summary(),
        "value": ws * state_bytes / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "achieved": round(algo_bytes / (ms_local * 1e-3) / 1e9, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(algo_bytes / (ms_local * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "peak_source": ("measured: MEASURED_PEAKS.json hbm_gbs" if peaks_kind == "measured"
                                     else "fallback 6650 GB/s"),
                     "traffic": DECODE_NCU_TRAFFIC, "algo_bytes_per_launch": algo_bytes,
                     "kernel": "gdn_decode_kernel<4>",
                     "traffic_source": "ncu dram bytes read + write, steady state: mean of launches 21-23 of "
                                       "--workload decode (profiles/gdn_decode_kernel_B256.md)"},
    }
    if not args.skip_e2e:
        stager = pkg.decode.HostStager(B, device)
        h_in = [t.cpu().pin_memory() for t in (inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a,
                                                inp.dt_bias, inp.b)]
        h_out = torch.empty((B, 8, 128), dtype=torch.bfloat16).pin_memory()
        h_ns = torch.empty_like(h_in[3]).pin_memory()

        def e2e_step():
            q, k, v, s_, A_log, a, dtb, b = h_in
            stager(q, k, v, s_, A_log, a, dtb, b, inp.scale, h_out, h_ns)

        e2e_steps = max(3, min(args.steps, 10))
        e2e_times, _ = time_steps(e2e_step, e2e_steps, 3, ws, device, None)
        e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), ws, device)
        h2d, d2h = stager.bytes_per_step()
        res["e2e"] = {"value": round(ws * state_bytes / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
                      "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": d2h,
                      "api": "decode.HostStager -> gdn_decode_launch_host_staged (pinned host buffers; state sliced, H2D / kernel / D2H overlapped on three streams; PCIe copies timed)"}

        # The serving form: the state stays on the device between steps; each
        # step copies its token inputs (q, k, v, a, b) up from pinned host
        # memory and its output back down.
        h_tok = [t.cpu().pin_memory() for t in (inp.q, inp.k, inp.v, inp.a, inp.b)]
        d_tok = [torch.empty_like(t, device=device) for t in h_tok]
        states = [inp.state.clone(), torch.empty_like(inp.state)]
        d_out = torch.empty((B, 8, 128), dtype=torch.bfloat16, device=device)
        it = [0]

        def resident_step():
            for d, h in zip(d_tok, h_tok):
                d.copy_(h, non_blocking=True)
            i = it[0] % 2
            it[0] += 1
            pkg.decode.launch_gdn(d_tok[0], d_tok[1], d_tok[2], states[i], inp.A_log, d_tok[3], inp.dt_bias,
                                  d_tok[4], inp.scale, output=d_out, new_state=states[1 - i])
            h_out.copy_(d_out, non_blocking=True)

        r_times, _ = time_steps(resident_step, e2e_steps, 3, ws, device, None)
        r_ms = max_over_ranks(sum(r_times) / len(r_times), ws, device)
        res["e2e_state_resident"] = {
            "value": round(ws * state_bytes / (r_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(r_ms, 4),
            "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in h_tok),
            "d2h_bytes_per_step": h_out.numel() * h_out.element_size(),
            "api": "decode.launch_gdn with the state resident on the device; token inputs up and the output down "
                   "over PCIe every step (timed)"}
    return res


def run_ours(args):
    ws, rank, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
    pkg = __graft_entry__.load_package()
    peaks, peaks_kind = load_peaks()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    wl = args.workload
    line = {}
    if wl in ("all", "decode"):
        d = bench_decode(pkg, args, device, ws, rank, flush, peaks, peaks_kind)
        line = {
            "metric": "gdn decode state-stream HBM GB/s (config 1: B=256 per GPU, fp32 k-last state)",
            "value": round(d["value"], 2),
            "unit": "GB/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(d["ms"], 5),
            "decode_us_per_step": round(d["ms"] * 1e3, 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp32 state / bf16 io",
            "data": "synthetic (seeded; BASELINE config 1 distributions)",
            "config": {"workload": "config1_decode_B256_per_gpu", "batch_per_gpu": DECODE_BATCH,
                       "global_batch": DECODE_BATCH * ws, "seq_len": 1,
                       "parallelism": f"sequence-shard x{ws}",
                       "l2": "inputs larger than L2: 3 rotating 128 MiB state buffers, steps back to back"},
            "gpu_launches": args.steps,  # one decode kernel per timed step
            "roofline": d["roofline"],
            "clocks": d["clocks"],
            "wall_s_timed_region": round(d["wall"], 4),
        }
        if "e2e" in d:
            line["e2e"] = d["e2e"]
            line["e2e_state_resident"] = d["e2e_state_resident"]
        if ws == 1:
            line["decode_small_batch_us"] = bench_decode_small(pkg, device, flush)
            line["decode_multi_token"] = bench_decode_tokens(pkg, device, flush)
            line["decode_bf16_state"] = bench_decode_bf16(pkg, device, flush)
            line["decode_qk16_v32"] = bench_decode_heads(pkg, device, flush)
    pf = {}
    psteps = max(3, args.steps // 2)
    if ws == 1:
        if wl in ("all", "prefill2"):
            pf["config2_T4096_N1"] = bench_prefill(pkg, device, [4096], 0, psteps, args.warmup, ws, flush, peaks,
                                                   with_state=False, traffic=PREFILL_NCU_TRAFFIC.get("config2"))
        if wl in ("all", "prefill3"):
            pf["config3_32seq"] = bench_prefill(pkg, device, pkg.inputs.config3_lengths(0), 0, psteps,
                                                args.warmup, ws, flush, peaks, traffic=PREFILL_NCU_TRAFFIC.get("config3"))
        if wl == "prefill4b_shard":  # one rank's share of config 4b at N = 8, alone (for per-kernel captures)
            pf["config4b_shard_8x8192"] = bench_prefill(pkg, device, [8192] * 8, 5, psteps, args.warmup, ws, flush,
                                                        peaks)
        if wl in ("all", "prefill_heads"):
            # the contest's other head layout (16 q/k, 32 v heads) on config 2's and config 3's shapes
            pf["qk16_v32_T4096_N1"] = bench_prefill(pkg, device, [4096], 0, psteps, args.warmup, ws, flush, peaks,
                                                    with_state=False, hqk=16, hv=32)
            pf["qk16_v32_config3_lengths"] = bench_prefill(pkg, device, pkg.inputs.config3_lengths(0), 0, psteps,
                                                           args.warmup, ws, flush, peaks, hqk=16, hv=32)
    if wl in ("all", "prefill_cp") and ws > 1:
        try:  # a ride-along: an error (the same on every rank) is reported, not fatal to the line
            pf["context_parallel_1x131072"] = bench_prefill_cp(pkg, device, rank, ws, [131072], 5,
                                                               min(args.warmup, 3), flush, peaks)
        except (ValueError, RuntimeError) as e:
            pf["context_parallel_1x131072"] = {"error": str(e)[:300]}
    if pf:
        line["prefill"] = pf
        # flat summary of the legs: tokens/s and the roofline fraction of its bound
        line["prefill_tokens_per_s"] = {k: round(v["tokens_per_s"], 1) for k, v in pf.items() if "tokens_per_s" in v}
        line["prefill_roofline_frac"] = {k: v["roofline"]["frac"] for k, v in pf.items() if v.get("roofline")}
    if wl in ("all", "config4"):
        # BASELINE config 4 as written: the fixed global problem split over the N ranks
        line["config4a"] = bench_config4a(pkg, device, rank, ws, args.steps, args.warmup, peaks)
        torch.cuda.empty_cache()
        line["config4b"] = bench_config4b(pkg, device, rank, ws, max(3, args.steps // 2), min(args.warmup, 3),
                                          flush, peaks)
        torch.cuda.empty_cache()
    if ws == 1 and wl in ("all", "reference_gpu", "reference_gpu_decode") and not args.skip_ref_gpu:
        try:  # a ride-along: an error is reported in the line, not fatal to it
            line["reference_gpu"] = bench_reference_gpu(pkg, device, flush,
                                                         prefill=wl != "reference_gpu_decode")
        except Exception as e:  # noqa: BLE001
            line["reference_gpu"] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
    if rank == 0 and ws == 1 and not args.skip_cpu and wl == "all":
        line["cpu_baseline"] = cpu_decode_baseline(pkg, args.cpu_budget)
        line["cpu_baseline_prefill"] = cpu_prefill_baseline(pkg, args.cpu_budget)
        try:  # the reference's own PyTorch code on the host CPU (ride-along; the C port is the baseline proper)
            line["cpu_reference_torch"] = cpu_torch_reference(pkg, args.cpu_budget)
        except Exception as e:  # noqa: BLE001
            line["cpu_reference_torch"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference(args):
    """The reference's own algorithm on the host CPU (oracle port), rank 0 only."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    pkg = __graft_entry__.load_package()
    from oracle import oracle

    threads = cpu_threads()
    B = DECODE_BATCH
    inp = pkg.inputs.make_decode_inputs(B, seed=1000)
    for _ in range(max(1, min(args.warmup, 3))):
        oracle.decode(*inp.args(), threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.decode(*inp.args(), threads=threads)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    value = B * STATE_BYTES_PER_SEQ * 2 / sec / 1e9
    line = {
        "impl": "reference",
        "metric": "gdn decode state-stream HBM GB/s (config 1: B=256 per GPU, fp32 k-last state)",
        "value": round(value, 4), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; BASELINE config 1 distributions)",
        "config": {"workload": "config1_decode_B256_per_gpu", "batch_per_gpu": B, "global_batch": B,
                   "seq_len": 1, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full decode steps of config 1 (B=256) through "
                                   "oracle/gdn_oracle.c (restatement of reference_torch_impl.py)"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds per CPU-baseline sample")
    ap.add_argument("--workload", default="all",
                    choices=["all", "decode", "prefill2", "prefill3", "prefill_heads", "prefill4b_shard", "config4",
                             "prefill_cp", "reference_gpu", "reference_gpu_decode"],
                    help="all = the JSON line the driver reads; the others time one workload")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline (profiling runs)")
    ap.add_argument("--skip-e2e", action="store_true", help="omit the host-buffer e2e leg")
    ap.add_argument("--skip-ref-gpu", action="store_true",
                    help="omit the reference's own GPU kernels (baseline/_ref) timed beside ours")
    ap.add_argument("--soak", type=float, default=1.0,
                    help="seconds of untimed steps under the clock sampler before timing")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
