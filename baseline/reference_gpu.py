"""The reference's own kernels and PyTorch code, loaded from ``baseline/_ref`` for timing.

``install_ref.py`` puts the unmodified reference solutions there.  This module
only loads them, the way the reference's harness does:

* decode: the torch extension built from ``solution/cuda/kernel.cu``
  (``binding.py:20-31``); its ``launch_gdn(q, k, v, state, A_log, a, dt_bias,
  b, scale, out, new_state)`` (``kernel.cu:982-994``) is the entry point the
  decode ``config.toml`` names (``kernel.cu::launch_gdn``, binding torch);
* prefill: ``solution/triton/kernel.py`` imported as a module; its
  ``launch_gdn(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
  output, new_state)`` (``kernel.py:56-262``) takes torch tensors directly
  (``torch.from_dlpack`` of a torch tensor is the tensor itself).

Nothing here is on the product path: ``bench.py`` times these beside this
project's kernels, and a GPU test checks their outputs against the oracle.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"
DECODE_EXT = "kachua_gdn_cuda_ext"
_cache: dict = {}


def missing() -> str | None:
    """None when both reference kernels are installed, else why not."""
    if not (REF / "gdn_prefill_qk4_v8_d128_k_last" / "solution" / "triton" / "kernel.py").exists():
        return "baseline/_ref not installed (python baseline/install_ref.py)"
    if not list((REF / "build_decode").glob(f"{DECODE_EXT}*.so")):
        return "reference decode extension not built (python baseline/install_ref.py)"
    return None


def decode_ext():
    """The reference decode torch extension (module with ``launch_gdn``)."""
    if "decode" not in _cache:
        import torch  # noqa: F401  (libtorch must be loaded before the extension)

        so = next((REF / "build_decode").glob(f"{DECODE_EXT}*.so"))
        spec = importlib.util.spec_from_file_location(DECODE_EXT, so)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _cache["decode"] = mod
    return _cache["decode"]


def prefill_module():
    """The reference Triton prefill module (with ``launch_gdn``)."""
    if "prefill" not in _cache:
        import tvm_ffi

        path = REF / "gdn_prefill_qk4_v8_d128_k_last" / "solution" / "triton" / "kernel.py"
        name = "kachua_ref_triton_prefill"
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod  # triton resolves kernel globals through the module
        # The module registers its entry point under the tvm_ffi global name
        # "flashinfer.kernel" at import; another solution loaded in this
        # process (this project's packed one) may hold that name already, so
        # the registration is allowed to replace it while the module loads.
        orig = tvm_ffi.register_global_func
        tvm_ffi.register_global_func = lambda func_name, f=None, override=False: orig(func_name, f, True)
        try:
            spec.loader.exec_module(mod)
        finally:
            tvm_ffi.register_global_func = orig
        _cache["prefill"] = mod
    return _cache["prefill"]


def torch_reference(definition: str):
    """``run`` of the reference's own PyTorch implementation of ``definition``
    (``solution/reference_torch_impl.py``, decode ``:12``, prefill ``:17``):
    the reference's CPU algorithm, timed on the host cores beside the GPU kernels."""
    key = "torch_" + definition
    if key not in _cache:
        path = REF / definition / "solution" / "reference_torch_impl.py"
        name = f"kachua_ref_torch_{definition}"
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        _cache[key] = mod.run
    return _cache[key]
