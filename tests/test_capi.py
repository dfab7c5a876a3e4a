"""The C-ABI library loads, exports what include/gdn_b200.h declares, and
rejects bad arguments on the host (no GPU needed: validation precedes any
device call)."""
import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "include" / "gdn_b200.h"


def _declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(gdn_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_expected(pkg):
    assert set(_declared_functions()) == set(pkg._capi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._capi.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.gdn_abi_version() == pkg._capi.ABI_VERSION


def test_status_strings(pkg):
    lib = pkg._capi.load()
    for code in (0, 1, 2, 3, 4, 5, 6, 7, 16, 32):
        s = lib.gdn_status_string(code).decode()
        assert s and s != "unknown status"
    assert lib.gdn_status_string(999).decode() == "unknown status"


def test_decode_host_validation(pkg):
    lib = pkg._capi.load()
    C = pkg._capi
    assert lib.gdn_decode_launch(None, None) == 1  # NULL args
    args = C.GdnDecodeArgs()
    args.batch = -1
    assert lib.gdn_decode_launch(ctypes.byref(args), None) == 2
    args.batch = 0
    assert lib.gdn_decode_launch(ctypes.byref(args), None) == 0  # empty batch: no-op
    args.batch = 4
    assert lib.gdn_decode_launch(ctypes.byref(args), None) == 1  # NULL pointers
    for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "output", "new_state"):
        setattr(args, f, 0x1000)
    args.state = 0x1008  # not 16-byte aligned
    assert lib.gdn_decode_launch(ctypes.byref(args), None) == 3


def test_decode_tokens_validation(pkg):
    lib = pkg._capi.load()
    C = pkg._capi
    args = C.GdnDecodeArgs()
    assert lib.gdn_decode_launch_tokens(None, 2, None) == 1
    args.batch = 4
    assert lib.gdn_decode_launch_tokens(ctypes.byref(args), 0, None) == 2
    assert lib.gdn_decode_launch_tokens(ctypes.byref(args), 3, None) == 1  # NULL pointers
    for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "output", "new_state"):
        setattr(args, f, 0x1000)
    args.q = 0x1002  # q, k need 8-byte alignment
    assert lib.gdn_decode_launch_tokens(ctypes.byref(args), 3, None) == 3
    args.batch = 0
    assert lib.gdn_decode_launch_tokens(ctypes.byref(args), 3, None) == 0


def test_heads_validation(pkg):
    lib = pkg._capi.load()
    C = pkg._capi
    d, p = C.GdnDecodeArgs(), C.GdnPrefillArgs()
    d.batch = 2
    assert lib.gdn_decode_launch_heads(None, 16, 32, 1, 0, None) == 1
    assert lib.gdn_decode_launch_heads(ctypes.byref(d), 3, 8, 1, 0, None) == 2   # 8 not a multiple of 3
    assert lib.gdn_decode_launch_heads(ctypes.byref(d), 16, 32, 2, 1, None) == 2  # bf16 state: one token
    assert lib.gdn_decode_launch_heads(ctypes.byref(d), 16, 32, 1, 0, None) == 1  # NULL pointers
    assert lib.gdn_prefill_launch_heads(ctypes.byref(p), 0, 8, None, 0, None) == 2
    p.total_tokens, p.num_seqs = 16, 1
    p.cu_seqlens_dtype = C.GDN_SEQLENS_INT64
    assert lib.gdn_prefill_launch_heads(ctypes.byref(p), 16, 32, None, 0, None) == 1
    # the chunked paths size their workspace by the v-head count
    assert lib.gdn_prefill_workspace_size_heads(4096, 1, 32) > 3 * lib.gdn_prefill_workspace_size(4096, 1)
    assert lib.gdn_prefill_workspace_size_heads(4096, 1, 8) == lib.gdn_prefill_workspace_size(4096, 1)
    assert lib.gdn_prefill_workspace_size_heads(-1, 1, 8) == 0 and lib.gdn_prefill_workspace_size_heads(1, 1, 0) == 0


def test_decode_host_staged_validation(pkg):
    lib = pkg._capi.load()
    C = pkg._capi
    host, dev = C.GdnDecodeArgs(), C.GdnDecodeArgs()
    assert lib.gdn_decode_launch_host_staged(None, ctypes.byref(dev), 8, None) == 1
    host.batch, dev.batch = 4, 3  # batch mismatch
    assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), 8, None) == 2
    dev.batch = 4
    for slices in (0, 65):
        assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), slices, None) == 2
    assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), 8, None) == 1  # NULLs
    for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "output", "new_state"):
        setattr(host, f, 0x1000)
        setattr(dev, f, 0x3000)
    dev.state = 0x4000  # the device state buffer is dev->new_state, updated in place
    assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), 8, None) == 2
    dev.state = None
    dev.new_state = 0x3008  # not 16-byte aligned
    assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), 8, None) == 3
    host.batch = dev.batch = 0
    assert lib.gdn_decode_launch_host_staged(ctypes.byref(host), ctypes.byref(dev), 8, None) == 0


def test_prefill_host_validation(pkg):
    lib = pkg._capi.load()
    C = pkg._capi
    a = C.GdnPrefillArgs()
    a.total_tokens, a.num_seqs = -1, 1
    assert lib.gdn_prefill_launch(ctypes.byref(a), None, 0, None) == 2
    a.total_tokens, a.num_seqs = 16, 1
    a.cu_seqlens_dtype = 7
    assert lib.gdn_prefill_launch(ctypes.byref(a), None, 0, None) == 6
    a.cu_seqlens_dtype = C.GDN_SEQLENS_INT64
    assert lib.gdn_prefill_launch(ctypes.byref(a), None, 0, None) == 1
    for f in ("q", "k", "v", "A_log", "a", "dt_bias", "b", "cu_seqlens", "output", "new_state"):
        setattr(a, f, 0x2000)
    a.q = 0x2008  # bf16 tiles need 16-byte alignment
    assert lib.gdn_prefill_launch(ctypes.byref(a), None, 0, None) == 3
    a.q = 0x2000
    a.state = 0x2000  # aliases new_state
    assert lib.gdn_prefill_launch(ctypes.byref(a), None, 0, None) == 2


def test_workspace_size_monotone(pkg):
    lib = pkg._capi.load()
    sizes = [lib.gdn_prefill_workspace_size(t, n) for t, n in ((0, 1), (64, 1), (4096, 1), (33000, 32))]
    assert sizes == sorted(sizes)
    assert lib.gdn_prefill_workspace_size(-1, 1) == 0
    for s in sizes:
        assert s % 256 == 0


def test_build_is_fresh(pkg):
    assert pkg._build.is_fresh(), "libgdn_b200.so is stale relative to csrc/"
