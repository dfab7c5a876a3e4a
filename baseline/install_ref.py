"""Installs the UNMODIFIED reference GPU solutions into ``baseline/_ref/``.

The reference (romitjain/kachua-mlsys) is not a Python package -- ``pip install
--target baseline/_ref <reference>`` stops with "Neither 'setup.py' nor
'pyproject.toml' found" -- so this recipe does what its harness does instead:

* copies the two solution directories, byte for byte, to
  ``baseline/_ref/gdn_decode_qk4_v8_d128_k_last/solution`` and
  ``baseline/_ref/gdn_prefill_qk4_v8_d128_k_last/solution``;
* builds the decode CUDA extension from the copied ``solution/cuda/kernel.cu``
  exactly as ``solution/cuda/binding.py:20-31`` does (``torch.utils.cpp_extension
  .load``, name ``kachua_gdn_cuda_ext``, ``extra_cuda_cflags=["-O3"]``), into
  ``baseline/_ref/build_decode`` for sm_100 (``TORCH_CUDA_ARCH_LIST=10.0``: this
  container has no GPU to detect the architecture from).

The Triton prefill (``solution/triton/kernel.py::launch_gdn``) needs no build:
Triton compiles it on the GPU at its first call.  ``baseline/_ref`` is
git-ignored (it is the reference's code, not this project's) and travels to the
GPU box with the rest of the tree; nothing on the box reads the original
checkout.

    python baseline/install_ref.py [--src <reference checkout>]
"""
from __future__ import annotations

import argparse
import filecmp
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "_ref"
DEFS = ("gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last")
DECODE_EXT = "kachua_gdn_cuda_ext"


def copy_solutions(src: Path) -> None:
    for d in DEFS:
        s, t = src / d / "solution", DEST / d / "solution"
        if t.exists() and not filecmp.dircmp(s, t).diff_files:
            continue
        if t.exists():
            shutil.rmtree(t)
        shutil.copytree(s, t, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        cfg = src / d / "config.toml"
        if cfg.exists():
            shutil.copy2(cfg, DEST / d / "config.toml")


def build_decode() -> Path:
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    kernel = DEST / DEFS[0] / "solution" / "cuda" / "kernel.cu"
    build = DEST / "build_decode"
    build.mkdir(parents=True, exist_ok=True)
    load(name=DECODE_EXT, sources=[str(kernel)], extra_cuda_cflags=["-O3"], with_cuda=True,
         build_directory=str(build), verbose=False)
    so = next(build.glob(f"{DECODE_EXT}*.so"))
    return so


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("GDN_REFERENCE_SRC", "/root/reference"))
    args = ap.parse_args()
    src = Path(args.src)
    if not (src / DEFS[0]).is_dir():
        print(f"reference checkout not found at {src}; nothing installed", file=sys.stderr)
        return 1
    DEST.mkdir(parents=True, exist_ok=True)
    copy_solutions(src)
    so = build_decode()
    print(f"installed {DEST} (decode extension {so.name})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
