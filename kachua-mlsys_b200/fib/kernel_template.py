"""FlashInfer-Bench entry point for @@DEFINITION@@ (packed by
kachua-mlsys_b200/pack_solution.py).

The B200 kernels are the package packed beside this file
(``kachua_mlsys_b200/``).  It is imported by path under a module name of its
own, and its C-ABI library is compiled on the first call (nvcc, sm_100a)
into ``kachua_mlsys_b200/lib/``, then reused while the sources are unchanged.
The harness hands over torch tensors (``binding = torch``) or DLPack-capable
tensors (tvm_ffi, which the reference's Triton plugin converts with
``torch.from_dlpack``, prefill ``kernel.py:58-66``); both become torch views
of the same memory, so the destination-passing outputs are written in place.
"""
from __future__ import annotations

import hashlib
import importlib.util
import sys
from pathlib import Path

import torch

_PKG_DIR = Path(__file__).resolve().parent / "kachua_mlsys_b200"
# a module name per unpacked copy, so that two copies never alias
_NAME = "kachua_mlsys_b200_" + hashlib.sha1(str(_PKG_DIR).encode()).hexdigest()[:12]


def package():
    mod = sys.modules.get(_NAME)
    if mod is None:
        spec = importlib.util.spec_from_file_location(_NAME, _PKG_DIR / "__init__.py",
                                                      submodule_search_locations=[str(_PKG_DIR)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[_NAME] = mod
        spec.loader.exec_module(mod)
    return mod


def _tensor(x):
    return x if x is None or isinstance(x, torch.Tensor) else torch.from_dlpack(x)


def _scale(x):
    return None if x is None else float(x)


# @@LAUNCH_GDN@@


try:  # the reference registers its entry as this tvm_ffi global (prefill kernel.py:28,55-56)
    from tvm_ffi import register_global_func

    register_global_func("flashinfer.kernel", launch_gdn, override=True)
except Exception:  # tvm_ffi absent or refusing: the module attribute is still the entry point
    pass
