"""Pack the B200 kernels as a FlashInfer-Bench solution (``solution.json``).

The reference packs each plugin from its ``config.toml`` with
``flashinfer_bench.agents.pack_solution_from_files`` (``scripts/pack_solution.py:34-84``):
a Solution with ``name``, ``definition``, ``author``, a build spec
(``language``, ``target_hardware = ["cuda"]``, ``entry_point``, optional
``binding``) and the source files as ``{path, content}`` records.  That
library is not a dependency here, so this module writes the same record as
plain JSON.  The solution's files:

* ``kernel.py`` -- the entry module (``kernel.py::launch_gdn``), made from
  ``fib/kernel_template.py`` and the definition's ``launch_gdn``;
* ``kachua_mlsys_b200/`` -- this package's Python modules and CUDA sources
  (``lib/`` is built from them on the first call);
* ``include/gdn_b200.h`` -- the C ABI header the sources include.

    python kachua-mlsys_b200/pack_solution.py gdn_prefill_qk4_v8_d128_k_last -o solution.json

``unpack`` writes a solution's sources into a directory (what a harness does
before it imports the entry point).
"""
from __future__ import annotations

import argparse
import json
import sys
import tomllib
from pathlib import Path

PKG = Path(__file__).resolve().parent
FIB = PKG / "fib"
INCLUDE = PKG.parent / "include"
PACKED_PKG = "kachua_mlsys_b200"  # the package directory's name inside a solution
MODULES = ("__init__.py", "_build.py", "_capi.py", "decode.py", "prefill.py", "inputs.py", "shard.py")
DEFINITIONS = ("gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last")


def load_config(definition: str) -> dict:
    path = FIB / f"{definition}.toml"
    if not path.exists():
        raise ValueError(f"no solution config for {definition!r} (known: {', '.join(DEFINITIONS)})")
    with open(path, "rb") as f:
        return tomllib.load(f)


def entry_source(definition: str) -> str:
    """The entry module: the template with the definition's launch_gdn."""
    build = load_config(definition)["build"]
    text = (FIB / "kernel_template.py").read_text().replace("@@DEFINITION@@", definition)
    marker = "# @@LAUNCH_GDN@@\n"
    if marker not in text:
        raise RuntimeError("kernel_template.py lost its launch_gdn marker")
    return text.replace(marker, (FIB / build["entry_function"]).read_text())


def solution_files(definition: str) -> list[tuple[str, str]]:
    """(relative path, text) of every file of the solution."""
    files = [("kernel.py", entry_source(definition))]
    files += [(f"{PACKED_PKG}/{m}", (PKG / m).read_text()) for m in MODULES]
    csrc = sorted(list((PKG / "csrc").glob("*.cu")) + list((PKG / "csrc").glob("*.cuh")))
    files += [(f"{PACKED_PKG}/csrc/{p.name}", p.read_text()) for p in csrc]
    files += [(f"include/{p.name}", p.read_text()) for p in sorted(INCLUDE.glob("*.h"))]
    return files


def pack(definition: str, output: Path | None = None) -> dict:
    """The Solution record for ``definition``; written as JSON to ``output`` if given."""
    cfg = load_config(definition)
    sol, build = cfg["solution"], cfg["build"]
    if sol["definition"] != definition:
        raise ValueError(f"{definition}.toml names definition {sol['definition']!r}")
    spec = {"language": build["language"], "target_hardware": ["cuda"], "entry_point": build["entry_point"]}
    if build.get("binding"):
        spec["binding"] = build["binding"]
    solution = {
        "name": sol["name"],
        "definition": definition,
        "author": sol["author"],
        "description": "Gated Delta Network kernels for B200 (sm_100a): hand-written CUDA behind a C ABI, "
                       "compiled with nvcc on first use.",
        "spec": spec,
        "sources": [{"path": p, "content": c} for p, c in solution_files(definition)],
    }
    if output is not None:
        Path(output).write_text(json.dumps(solution, indent=2))
    return solution


def unpack(solution: dict, dest: Path) -> Path:
    """Writes the solution's sources under ``dest``; returns the entry file's path."""
    dest = Path(dest).resolve()
    for src in solution["sources"]:
        rel = Path(src["path"])
        if rel.is_absolute() or ".." in rel.parts:
            raise ValueError(f"unsafe source path {src['path']!r}")
        out = dest / rel
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(src["content"])
    return dest / solution["spec"]["entry_point"].split("::")[0]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Pack a FlashInfer-Bench solution.json for the B200 GDN kernels")
    ap.add_argument("definition", choices=DEFINITIONS)
    ap.add_argument("-o", "--output", type=Path, default=Path("solution.json"))
    args = ap.parse_args(argv)
    sol = pack(args.definition, args.output)
    print(f"Solution packed: {args.output}\n  Name: {sol['name']}\n  Definition: {sol['definition']}\n"
          f"  Language: {sol['spec']['language']}\n  Files: {len(sol['sources'])}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
