"""FlashInfer-Bench entry module for ``gdn_decode_qk4_v8_d128_k_last`` on B200.

Drop-in for the reference solution's ``launch_gdn`` (gdn_decode_qk4_v8_d128_k_last/solution/cuda/kernel.cu:982-994 (torch binding) and solution/triton/kernel.py:27-28):
same name, same destination-passing arguments.  Tensors may arrive as torch
tensors or as DLPack-capable handles (tvm_ffi); the call goes to the sm_100a
library through its C ABI.  The function is also registered as the tvm_ffi
global ``flashinfer.kernel`` when tvm_ffi is importable, as the reference did.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import torch

_PKG_DIR = Path(__file__).resolve().parents[4]
_PKG_NAME = "kachua_mlsys_b200"


def _package():
    mod = sys.modules.get(_PKG_NAME)
    if mod is not None and hasattr(mod, "decode"):
        return mod
    spec = importlib.util.spec_from_file_location(_PKG_NAME, _PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(_PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[_PKG_NAME] = mod
    spec.loader.exec_module(mod)
    return mod


def _tensor(x):
    if x is None or isinstance(x, torch.Tensor) or isinstance(x, (int, float)):
        return x
    return torch.from_dlpack(x)


def launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    pkg = _package()
    q, k, v, state, A_log, a, dt_bias, b = (_tensor(t) for t in (q, k, v, state, A_log, a, dt_bias, b))
    output, new_state = _tensor(output), _tensor(new_state)
    return pkg.decode.launch_gdn(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)


try:  # the reference registered its entry under this tvm_ffi name
    from tvm_ffi import register_global_func

    register_global_func("flashinfer.kernel", launch_gdn, override=True)
except Exception:  # tvm_ffi absent or name already bound: the module entry still works
    pass
