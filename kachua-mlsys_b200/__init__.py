"""B200 (sm_100a) Gated Delta Network kernels behind the reference's plugin API.

The directory name contains a hyphen, so it is imported under the module
name ``kachua_mlsys_b200`` with :func:`load_package` in ``__graft_entry__``
(or any ``importlib`` path import).

Public surface (drop-ins for the two reference plugins of
romitjain/kachua-mlsys):

* ``decode.launch_gdn``  -- gdn_decode_qk4_v8_d128_k_last
* ``prefill.launch_gdn`` -- gdn_prefill_qk4_v8_d128_k_last
* ``inputs``             -- seeded synthetic inputs of the benchmark configs
* ``shard``              -- sequence sharding across GPUs and the final gather
"""
from . import _build, _capi, decode, inputs, prefill, shard  # noqa: F401

__all__ = ["decode", "prefill", "inputs", "build"]


def build(force: bool = False, verbose: bool = False):
    """Compile lib/libgdn_b200.so for sm_100a (no-op when up to date)."""
    return _build.build(force=force, verbose=verbose)
