"""A FlashInfer-Bench style runner for packed solutions (``solution.json``).

The reference times its plugins on the contest's trace set with
``scripts/bench_fi_timing.py``: it finds a definition record
(``definitions/**/<name>.json``) and the definition's workload records
(``workloads/**/<name>.jsonl``, one ``{"workload": {...}}`` per line), builds
the call arguments from a workload (axes resolve the definition's named
shapes; inputs are ``random``, ``scalar`` or ``safetensors`` entries,
``:194-246``), runs the solution once and checks every output against a
reference with ``allclose(atol = rtol = 1e-2)`` (``:265-312``), then times it
with a cold L2 (``bench_gpu_time(cold_l2_cache=True)``, ``:342-346``).

This module does the same for a packed solution of this project (or any
solution record of the same form): ``load_solution`` unpacks its sources
(``pack_solution.unpack``) and imports its entry point; outputs are
allocated from the definition's ``outputs`` section and passed
destination-style, as the harness calls ``launch_gdn``.  The reference
computation is a caller-supplied function of the inputs, or the
definition's own ``reference`` source when it carries one.  Timing uses CUDA
events around each call with a 256 MiB read between calls to evict L2.

The contest dataset is absent here; ``write_trace_set`` writes definition
and workload records of the same form, with seeded inputs (BASELINE
distributions) stored as safetensors files.

    python kachua-mlsys_b200/fib/runner.py --trace-set DIR --solution solution.json [--workload-idx -1]
"""
from __future__ import annotations

import importlib.util
import json
import statistics
import sys
import tempfile
from pathlib import Path
from typing import Callable

import torch

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "int8": torch.int8,
          "int16": torch.int16, "int32": torch.int32, "int64": torch.int64, "bool": torch.bool}
DTYPE_NAMES = {v: k for k, v in DTYPES.items()}
ATOL = RTOL = 1e-2
DECODE, PREFILL = "gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last"


# ------------------------------------------------------------ trace set -----
def is_trace_root(path: Path) -> bool:
    return (path / "definitions").is_dir() and (path / "workloads").is_dir()


def resolve_trace_set(path) -> Path:
    """The trace-set root: ``path`` itself or its first child holding
    ``definitions/`` and ``workloads/``."""
    root = Path(path).expanduser()
    if not root.exists():
        raise FileNotFoundError(f"trace set path does not exist: {root}")
    if is_trace_root(root):
        return root
    for child in sorted(root.iterdir()):
        if child.is_dir() and is_trace_root(child):
            return child
    raise FileNotFoundError(f"no definitions/ and workloads/ under {root} or one level below")


def _find(root: Path, sub: str, pattern: str) -> Path:
    hits = sorted(root.joinpath(sub).rglob(pattern))
    if not hits:
        raise FileNotFoundError(f"{pattern} not found under {root / sub}")
    return hits[0]


def load_definition(root: Path, name: str) -> dict:
    return json.loads(_find(root, "definitions", f"{name}.json").read_text())


def load_workloads(root: Path, name: str) -> list[dict]:
    with open(_find(root, "workloads", f"{name}.jsonl"), encoding="utf-8") as f:
        return [json.loads(line)["workload"] for line in f if line.strip()]


def resolve_shape(shape, axes_def: dict, axes: dict):
    """Named dimensions -> sizes (workload axes first, then const axes)."""
    if shape is None:
        return None
    out = []
    for dim in shape:
        if isinstance(dim, int):
            out.append(dim)
        elif dim in axes:
            out.append(int(axes[dim]))
        elif axes_def.get(dim, {}).get("type") == "const" and "value" in axes_def[dim]:
            out.append(int(axes_def[dim]["value"]))
        else:
            raise KeyError(f"cannot resolve dimension {dim!r}")
    return out


def workload_inputs(root: Path, definition: dict, workload: dict, device) -> dict:
    """The call's inputs by name, in the definition's order: tensors on
    ``device``, scalars as Python numbers, absent optional inputs as None."""
    from safetensors.torch import load_file

    axes_def, axes = definition["axes"], workload.get("axes", {})
    gen = torch.Generator(device="cpu").manual_seed(int(workload.get("seed", 0)))
    cache: dict = {}
    args = {}
    for name, spec in definition["inputs"].items():
        w = workload["inputs"].get(name)
        if w is None:
            args[name] = None
            continue
        kind = w["type"]
        if kind == "scalar":
            args[name] = w["value"]
            continue
        dtype = DTYPES[spec["dtype"]]
        shape = resolve_shape(spec["shape"], axes_def, axes)
        if kind == "safetensors":
            path = Path(w["path"])
            path = path if path.is_absolute() else root / path
            if path not in cache:
                cache[path] = load_file(str(path))
            t = cache[path][w["tensor_key"]]
            if shape is not None and list(t.shape) != shape:
                raise ValueError(f"{name}: stored shape {list(t.shape)} != definition shape {shape}")
            args[name] = t.to(device=device, dtype=dtype)
        elif kind == "random":
            if dtype.is_floating_point:
                t = torch.randn(shape, generator=gen).to(dtype)
            else:
                t = torch.randint(-16, 16, shape, generator=gen).to(dtype)
            args[name] = t.to(device)
        else:
            raise ValueError(f"unsupported workload input type {kind!r}")
    return args


def allocate_outputs(definition: dict, workload: dict, device) -> dict:
    """Destination tensors for the definition's outputs (shapes from the workload's axes)."""
    outs = {}
    for name, spec in definition["outputs"].items():
        shape = resolve_shape(spec["shape"], definition["axes"], workload.get("axes", {}))
        outs[name] = torch.empty(shape, dtype=DTYPES[spec["dtype"]], device=device)
    return outs


# ------------------------------------------------------------- solutions ----
def load_solution(solution, work_dir=None) -> tuple[dict, Callable]:
    """(solution record, entry function) of a solution record or JSON file:
    its sources are written under ``work_dir`` (a temporary directory when
    None) and its entry point ``<file>::<function>`` imported."""
    if not isinstance(solution, dict):
        solution = json.loads(Path(solution).read_text())
    pkg_dir = Path(__file__).resolve().parents[1]
    spec = importlib.util.spec_from_file_location("gdn_runner_pack_solution", pkg_dir / "pack_solution.py")
    packer = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(packer)
    dest = Path(work_dir) if work_dir is not None else Path(tempfile.mkdtemp(prefix="gdn_solution_"))
    entry_file = packer.unpack(solution, dest)
    entry_fn = solution["spec"]["entry_point"].split("::", 1)[1]
    mspec = importlib.util.spec_from_file_location(f"gdn_solution_{abs(hash(str(entry_file)))}", entry_file)
    mod = importlib.util.module_from_spec(mspec)
    sys.modules[mspec.name] = mod
    mspec.loader.exec_module(mod)
    return solution, getattr(mod, entry_fn)


def definition_reference(definition: dict) -> Callable | None:
    """The definition's own ``reference`` function (its ``run``, or its only
    function), if the record carries source code."""
    src = definition.get("reference")
    if not src:
        return None
    scope: dict = {}
    exec(compile(src, f"<reference of {definition.get('name')}>", "exec"), scope)  # noqa: S102
    if callable(scope.get("run")):
        return scope["run"]
    fns = [v for k, v in scope.items() if callable(v) and getattr(v, "__module__", None) is None and
           not k.startswith("__")]
    return fns[-1] if fns else None


# ----------------------------------------------------------------- runs -----
def check_outputs(outputs: dict, expected, atol=ATOL, rtol=RTOL) -> dict:
    """Per output: max abs / rel error and allclose(atol, rtol) against ``expected``
    (a tuple in the definition's output order, or a dict by name)."""
    names = list(outputs)
    if isinstance(expected, torch.Tensor):
        expected = (expected,)
    if not isinstance(expected, dict):
        if len(expected) != len(names):
            raise ValueError(f"reference returned {len(expected)} outputs, the definition has {len(names)}")
        expected = dict(zip(names, expected))
    per, ok_all, ma, mr = {}, True, 0.0, 0.0
    for n in names:
        got = outputs[n].detach().float().cpu()
        ref = expected[n].detach().float().cpu().reshape(got.shape)
        err = (got - ref).abs()
        max_abs = float(err.max()) if err.numel() else 0.0
        max_rel = float((err / ref.abs().clamp_min(1e-12)).max()) if err.numel() else 0.0
        ok = bool(torch.allclose(got, ref, atol=atol, rtol=rtol))
        per[n] = {"max_abs_error": max_abs, "max_rel_error": max_rel, "within_tolerance": ok}
        ok_all, ma, mr = ok_all and ok, max(ma, max_abs), max(mr, max_rel)
    return {"max_abs_error": ma, "max_rel_error": mr, "within_tolerance": ok_all, "atol": atol, "rtol": rtol,
            "per_output": per}


def time_cold_l2(fn: Callable, iters: int = 20, warmup: int = 3, flush_bytes: int = 256 << 20) -> list[float]:
    """Device time (us) of each of ``iters`` calls, CUDA events on the current
    stream, with L2 evicted (a read of ``flush_bytes``) before every call."""
    flush = torch.empty(flush_bytes // 4, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in evs:
        torch.sum(flush)
        torch.cuda._sleep(100_000)  # the host enqueues the call while the GPU is busy
        e0.record(stream)
        fn()
        e1.record(stream)
    torch.cuda.synchronize()
    return [e0.elapsed_time(e1) * 1e3 for e0, e1 in evs]


def run_workload(root: Path, definition: dict, workload: dict, entry: Callable, reference: Callable | None,
                 device="cuda", iters: int = 20) -> dict:
    """One workload: call the entry once and check it, then time it cold."""
    inputs = workload_inputs(root, definition, workload, device)
    outputs = allocate_outputs(definition, workload, device)
    call = list(inputs.values()) + list(outputs.values())
    entry(*call)
    torch.cuda.synchronize()
    result = {"definition": definition["name"], "uuid": workload.get("uuid"), "axes": workload.get("axes", {})}
    if reference is not None:
        host = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in inputs.items()}
        result["correctness"] = check_outputs(outputs, reference(**host))
    times = time_cold_l2(lambda: entry(*call), iters=iters)
    result.update({"median_us": statistics.median(times), "mean_us": statistics.mean(times), "min_us": min(times),
                   "max_us": max(times), "iters": len(times), "timing": "cuda events, L2 evicted before each call"})
    return result


def run(trace_set, solution, workload_idx: int = -1, reference: Callable | None = None, work_dir=None,
        iters: int = 20) -> list[dict]:
    """Every workload (``workload_idx`` < 0) or one of the solution's
    definition; ``reference`` defaults to the definition's own reference code."""
    root = resolve_trace_set(trace_set)
    sol, entry = load_solution(solution, work_dir)
    definition = load_definition(root, sol["definition"])
    ref = reference if reference is not None else definition_reference(definition)
    wls = load_workloads(root, sol["definition"])
    picked = wls if workload_idx < 0 else [wls[workload_idx]]
    return [dict(run_workload(root, definition, w, entry, ref, iters=iters), solution=sol["name"]) for w in picked]


# -------------------------------------------------- synthetic trace set -----
def _axis(kind: str, value: int | None = None, description: str = "") -> dict:
    d = {"type": kind}
    if value is not None:
        d["value"] = value
    if description:
        d["description"] = description
    return d


def definition_record(name: str) -> dict:
    """The definition record of one of the two GDN definitions (the fields
    and dimension names of the FlashInfer trace templates for GDN decode and
    prefill: axes, inputs, outputs, k-last state)."""
    heads = {"num_q_heads": _axis("const", 4), "num_k_heads": _axis("const", 4),
             "num_v_heads": _axis("const", 8), "head_size": _axis("const", 128)}
    t = lambda shape, dtype, **kw: dict({"shape": shape, "dtype": dtype}, **kw)  # noqa: E731
    if name == DECODE:
        axes = {"batch_size": _axis("var", description="sequences decoded together"),
                "seq_len": _axis("const", 1), **heads}
        tok = ["batch_size", "seq_len"]
        inputs = {"q": t(tok + ["num_q_heads", "head_size"], "bfloat16"),
                  "k": t(tok + ["num_k_heads", "head_size"], "bfloat16"),
                  "v": t(tok + ["num_v_heads", "head_size"], "bfloat16"),
                  "state": t(["batch_size", "num_v_heads", "head_size", "head_size"], "float32", optional=True),
                  "A_log": t(["num_v_heads"], "float32"), "a": t(tok + ["num_v_heads"], "bfloat16"),
                  "dt_bias": t(["num_v_heads"], "float32"), "b": t(tok + ["num_v_heads"], "bfloat16"),
                  "scale": t(None, "float32", optional=True)}
        outputs = {"output": t(tok + ["num_v_heads", "head_size"], "bfloat16"),
                   "new_state": t(["batch_size", "num_v_heads", "head_size", "head_size"], "float32")}
    elif name == PREFILL:
        axes = {"total_seq_len": _axis("var"), "num_seqs": _axis("var"), **heads, "len_cu_seqlens": _axis("var")}
        inputs = {"q": t(["total_seq_len", "num_q_heads", "head_size"], "bfloat16"),
                  "k": t(["total_seq_len", "num_k_heads", "head_size"], "bfloat16"),
                  "v": t(["total_seq_len", "num_v_heads", "head_size"], "bfloat16"),
                  "state": t(["num_seqs", "num_v_heads", "head_size", "head_size"], "float32", optional=True),
                  "A_log": t(["num_v_heads"], "float32"), "a": t(["total_seq_len", "num_v_heads"], "bfloat16"),
                  "dt_bias": t(["num_v_heads"], "float32"), "b": t(["total_seq_len", "num_v_heads"], "bfloat16"),
                  "cu_seqlens": t(["len_cu_seqlens"], "int64"), "scale": t(None, "float32", optional=True)}
        outputs = {"output": t(["total_seq_len", "num_v_heads", "head_size"], "bfloat16"),
                   "new_state": t(["num_seqs", "num_v_heads", "head_size", "head_size"], "float32")}
    else:
        raise ValueError(f"unknown definition {name!r}")
    return {"name": name, "op_type": "gdn", "axes": axes, "inputs": inputs, "outputs": outputs,
            "tags": ["stage:decode" if name == DECODE else "stage:prefill", "synthetic"]}


def write_trace_set(root, decode_batches=(1, 8, 64), prefill_lengths=([4096], [300, 77, 0, 129]), seed=0) -> Path:
    """Writes a trace set of the dataset's form under ``root``: the two
    definitions, and one workload per decode batch size and per prefill length
    list, their tensors drawn from this package's seeded inputs (BASELINE
    distributions) and stored as safetensors."""
    from safetensors.torch import save_file

    pkg_dir = Path(__file__).resolve().parents[1]
    inputs_mod = sys.modules.get("gdn_runner_inputs")
    if inputs_mod is None:
        spec = importlib.util.spec_from_file_location("gdn_runner_inputs", pkg_dir / "inputs.py")
        inputs_mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = inputs_mod  # dataclasses resolve their module by name
        spec.loader.exec_module(inputs_mod)
    root = Path(root)
    for sub in ("definitions/gdn", "workloads/gdn", "blob/workloads/gdn"):
        (root / sub).mkdir(parents=True, exist_ok=True)
    for name in (DECODE, PREFILL):
        (root / "definitions/gdn" / f"{name}.json").write_text(json.dumps(definition_record(name), indent=2))

    def entry(path, key):
        return {"type": "safetensors", "path": str(path.relative_to(root)), "tensor_key": key}

    lines = []
    for i, B in enumerate(decode_batches):
        inp = inputs_mod.make_decode_inputs(B, seed=seed + i)
        path = root / "blob/workloads/gdn" / f"decode_{i}.safetensors"
        names = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")
        save_file({n: getattr(inp, n).contiguous() for n in names}, str(path))
        wl = {"uuid": f"synthetic-decode-{i}", "axes": {"batch_size": B},
              "inputs": {**{n: entry(path, n) for n in names}, "scale": {"type": "scalar", "value": inp.scale}}}
        lines.append(json.dumps({"definition": DECODE, "workload": wl}))
    (root / "workloads/gdn" / f"{DECODE}.jsonl").write_text("\n".join(lines) + "\n")

    lines = []
    for i, lengths in enumerate(prefill_lengths):
        inp = inputs_mod.make_prefill_inputs(lengths, seed=seed + 100 + i, with_state=True)
        path = root / "blob/workloads/gdn" / f"prefill_{i}.safetensors"
        names = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")
        save_file({n: getattr(inp, n).contiguous() for n in names}, str(path))
        wl = {"uuid": f"synthetic-prefill-{i}",
              "axes": {"total_seq_len": inp.total_tokens, "num_seqs": inp.num_seqs,
                       "len_cu_seqlens": inp.num_seqs + 1},
              "inputs": {**{n: entry(path, n) for n in names}, "scale": {"type": "scalar", "value": inp.scale}}}
        lines.append(json.dumps({"definition": PREFILL, "workload": wl}))
    (root / "workloads/gdn" / f"{PREFILL}.jsonl").write_text("\n".join(lines) + "\n")
    return root


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="Run a packed GDN solution over a FlashInfer-Bench style trace set")
    ap.add_argument("--trace-set", required=True, help="trace-set root (definitions/, workloads/)")
    ap.add_argument("--solution", required=True, help="solution.json")
    ap.add_argument("--workload-idx", type=int, default=-1, help="one workload index, or -1 for all")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    for r in run(args.trace_set, args.solution, args.workload_idx, iters=args.iters):
        c = r.get("correctness")
        tag = "unchecked" if c is None else ("OK" if c["within_tolerance"] else "OUT-OF-TOL")
        print(f"{r['solution']} {r['uuid']} {r['axes']}: median {r['median_us']:.2f} us [{tag}]")
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    sys.exit(main())
