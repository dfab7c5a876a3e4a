"""FlashInfer-Bench packaging: solution.json records, unpacking, and the
packed entry points (the reference packs each plugin with
scripts/pack_solution.py:34-84 from its config.toml)."""
import importlib.util
import inspect
import json
import shutil

import pytest
import torch

from tests.conftest import REPO

DECODE, PREFILL = "gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last"
# the reference plugins' entry signatures (decode kernel.cu:982-994, prefill kernel.py:56-57)
SIGNATURES = {
    DECODE: ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale", "output", "new_state"],
    PREFILL: ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale", "output", "new_state"],
}


@pytest.fixture(scope="module")
def packer(pkg):
    spec = importlib.util.spec_from_file_location("gdn_pack_solution", REPO / "kachua-mlsys_b200" / "pack_solution.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _import_entry(path):
    spec = importlib.util.spec_from_file_location(f"gdn_entry_{abs(hash(str(path)))}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _DLPackOnly:
    """A tensor seen only through the DLPack protocol (as tvm_ffi hands them over)."""

    def __init__(self, t):
        self._t = t

    def __dlpack__(self, *args, **kwargs):
        return self._t.__dlpack__(*args, **kwargs)

    def __dlpack_device__(self):
        return self._t.__dlpack_device__()


@pytest.mark.parametrize("definition", [DECODE, PREFILL])
def test_pack_record(packer, definition, tmp_path):
    out = tmp_path / "solution.json"
    sol = packer.pack(definition, out)
    assert json.loads(out.read_text()) == sol
    assert sol["definition"] == definition and sol["name"] and sol["author"]
    assert sol["spec"] == {"language": "triton", "target_hardware": ["cuda"], "entry_point": "kernel.py::launch_gdn"}
    paths = [s["path"] for s in sol["sources"]]
    assert len(paths) == len(set(paths)) and paths[0] == "kernel.py"
    csrc = sorted(p.name for p in (REPO / "kachua-mlsys_b200" / "csrc").iterdir() if p.suffix in (".cu", ".cuh"))
    assert sorted(p.split("/")[-1] for p in paths if p.startswith("kachua_mlsys_b200/csrc/")) == csrc
    assert "include/gdn_b200.h" in paths
    assert not any(p.startswith(("oracle", "tests", "_work")) or p.endswith(".so") for p in paths)
    for s in sol["sources"][1:]:  # byte-identical to the repository's files
        rel = s["path"].replace("kachua_mlsys_b200/", "kachua-mlsys_b200/", 1)
        assert (REPO / rel).read_text() == s["content"], s["path"]


def test_pack_rejects_unknown_definition(packer):
    with pytest.raises(ValueError, match="no solution config"):
        packer.pack("gdn_decode_qk16_v32_d128_k_last")


def test_unpack_rejects_unsafe_paths(packer, tmp_path):
    with pytest.raises(ValueError, match="unsafe"):
        packer.unpack({"sources": [{"path": "../x.py", "content": ""}],
                       "spec": {"entry_point": "kernel.py::launch_gdn"}}, tmp_path)


@pytest.mark.parametrize("definition", [DECODE, PREFILL])
def test_unpacked_entry_imports_and_validates(packer, pkg, definition, tmp_path):
    """The unpacked entry module imports its own packed copy of the package
    (no GPU, nothing built) and rejects CPU tensors before any launch."""
    entry = packer.unpack(packer.pack(definition), tmp_path)
    mod = _import_entry(entry)
    assert list(inspect.signature(mod.launch_gdn).parameters) == SIGNATURES[definition]
    assert str(tmp_path.resolve()) in mod.package().__file__
    inp = (pkg.inputs.make_decode_inputs(2, seed=0) if definition == DECODE
           else pkg.inputs.make_prefill_inputs([70], seed=0, with_state=True))
    args = [_DLPackOnly(t) if isinstance(t, torch.Tensor) else t for t in inp.args()]  # the tvm_ffi route
    with pytest.raises(ValueError, match="CUDA tensor"):
        mod.launch_gdn(*args, None, None)
    assert not (tmp_path / "kachua_mlsys_b200" / "lib").exists()  # nothing was compiled


def test_entry_registers_tvm_ffi_global(packer, pkg, tmp_path):
    """Like the reference, the entry is also the tvm_ffi global
    ``flashinfer.kernel``; a call through it reaches the same validation."""
    tvm_ffi = pytest.importorskip("tvm_ffi")
    _import_entry(packer.unpack(packer.pack(PREFILL), tmp_path))
    fn = tvm_ffi.get_global_func("flashinfer.kernel")
    inp = pkg.inputs.make_prefill_inputs([70], seed=0, with_state=True)
    with pytest.raises(Exception, match="CUDA tensor"):
        fn(*inp.args()[:-1], 0.0, None, None)


def test_cli_writes_solution(packer, tmp_path, capsys):
    out = tmp_path / "s.json"
    assert packer.main([PREFILL, "-o", str(out)]) == 0
    assert json.loads(out.read_text())["definition"] == PREFILL
    assert "Solution packed" in capsys.readouterr().out


def _unpacked_with_library(packer, pkg, definition, dest):
    """Unpacks a solution and seeds its lib/ with the in-tree library: the
    packed CUDA sources are byte-identical (test_pack_record), so the copy is
    what its first call would compile; the stamp is the copy's own digest."""
    entry = packer.unpack(packer.pack(definition), dest)
    mod = _import_entry(entry)
    packed = mod.package()
    lib_dir = dest / "kachua_mlsys_b200" / "lib"
    lib_dir.mkdir(exist_ok=True)
    shutil.copy2(pkg._build.LIB_PATH, lib_dir / "libgdn_b200.so")
    (lib_dir / "libgdn_b200.so.stamp").write_text(packed._build.source_digest())
    assert packed._build.is_fresh()
    return mod


@pytest.mark.gpu
def test_packed_decode_matches_package(packer, pkg, cuda_dev, tmp_path):
    mod = _unpacked_with_library(packer, pkg, DECODE, tmp_path)
    inp = pkg.inputs.make_decode_inputs(16, seed=5).to(cuda_dev)
    ref_out, ref_ns = pkg.decode.launch_gdn(*inp.args())
    out = torch.empty_like(ref_out)
    ns = torch.empty_like(ref_ns)
    a = list(inp.args())  # q k v state A_log a dt_bias b scale
    mod.launch_gdn(*[_DLPackOnly(t) if isinstance(t, torch.Tensor) else t for t in a], _DLPackOnly(out),
                   _DLPackOnly(ns))
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)
    assert "kachua_mlsys_b200/lib" in str(mod.package()._build.LIB_PATH)


@pytest.mark.gpu
def test_packed_prefill_matches_package(packer, pkg, cuda_dev, tmp_path):
    mod = _unpacked_with_library(packer, pkg, PREFILL, tmp_path)
    inp = pkg.inputs.make_prefill_inputs([300, 1, 2048], seed=6, with_state=True).to(cuda_dev)
    ref_out, ref_ns = pkg.prefill.launch_gdn(*inp.args())
    out, ns = mod.launch_gdn(*inp.args())  # output / new_state allocated by the entry (None)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)
