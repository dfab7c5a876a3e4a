"""The FlashInfer-Bench style runner (kachua-mlsys_b200/fib/runner.py): trace
set records of the dataset's form, argument building from a workload,
per-output checks, and both packed solutions run over a synthetic trace set
and checked against the CPU oracle (the reference runner's flow,
scripts/bench_fi_timing.py:194-312)."""
import importlib.util
import json
import shutil

import pytest
import torch

from tests.conftest import REPO

DECODE, PREFILL = "gdn_decode_qk4_v8_d128_k_last", "gdn_prefill_qk4_v8_d128_k_last"


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def runner():
    return _load("gdn_fib_runner", REPO / "kachua-mlsys_b200" / "fib" / "runner.py")


@pytest.fixture(scope="module")
def packer():
    return _load("gdn_pack_solution_r", REPO / "kachua-mlsys_b200" / "pack_solution.py")


def test_trace_set_records_and_inputs(runner, pkg, tmp_path):
    root = runner.write_trace_set(tmp_path / "traces" / "set", decode_batches=(3,), prefill_lengths=([17, 0, 70],))
    assert runner.resolve_trace_set(tmp_path / "traces") == root  # found one level below
    d = runner.load_definition(root, DECODE)
    assert d["axes"]["num_v_heads"] == {"type": "const", "value": 8}
    (wl,) = runner.load_workloads(root, DECODE)
    args = runner.workload_inputs(root, d, wl, "cpu")
    assert list(args) == ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale"]
    ref = pkg.inputs.make_decode_inputs(3, seed=0)
    for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b"):
        assert torch.equal(args[n], getattr(ref, n)), n
    outs = runner.allocate_outputs(d, wl, "cpu")
    assert outs["output"].shape == (3, 1, 8, 128) and outs["output"].dtype == torch.bfloat16
    assert outs["new_state"].shape == (3, 8, 128, 128)
    p = runner.load_definition(root, PREFILL)
    (wl,) = runner.load_workloads(root, PREFILL)
    args = runner.workload_inputs(root, p, wl, "cpu")
    assert args["cu_seqlens"].tolist() == [0, 17, 17, 87] and args["q"].shape == (87, 4, 128)
    assert runner.resolve_shape(["num_seqs", "num_v_heads"], p["axes"], wl["axes"]) == [3, 8]
    with pytest.raises(KeyError):
        runner.resolve_shape(["nope"], p["axes"], wl["axes"])


def test_random_and_scalar_inputs(runner, tmp_path):
    root = runner.write_trace_set(tmp_path, decode_batches=(2,), prefill_lengths=([5],))
    d = runner.load_definition(root, DECODE)
    wl = {"axes": {"batch_size": 2}, "seed": 3,
          "inputs": {"q": {"type": "random"}, "scale": {"type": "scalar", "value": 0.5}}}
    args = runner.workload_inputs(root, d, wl, "cpu")
    assert args["q"].shape == (2, 1, 4, 128) and args["q"].dtype == torch.bfloat16
    assert args["scale"] == 0.5 and args["state"] is None


def test_check_outputs_flags_a_planted_error(runner):
    good = torch.randn(4, 8)
    res = runner.check_outputs({"output": good.clone(), "new_state": good.clone()}, (good, good))
    assert res["within_tolerance"] and res["max_abs_error"] == 0.0
    bad = good.clone()
    bad[1, 2] += 0.5  # planted in the expected values
    res = runner.check_outputs({"output": good.clone(), "new_state": good.clone()}, {"output": good,
                                                                                     "new_state": bad})
    assert not res["within_tolerance"]
    assert res["per_output"]["output"]["within_tolerance"] and not res["per_output"]["new_state"]["within_tolerance"]
    with pytest.raises(ValueError):
        runner.check_outputs({"output": good}, (good, good))


def _seed_library(pkg, packer, definition, dest):
    """Unpacks the solution and seeds its lib/ with the in-tree library (the
    packed sources are byte-identical, so this is what its first call would
    compile), keeping nvcc out of the test."""
    packer.unpack(packer.pack(definition), dest)
    lib = dest / "kachua_mlsys_b200" / "lib"
    lib.mkdir(exist_ok=True)
    shutil.copy2(pkg._build.LIB_PATH, lib / "libgdn_b200.so")
    (lib / "libgdn_b200.so.stamp").write_text(pkg._build.source_digest())


@pytest.mark.gpu
@pytest.mark.parametrize("definition", [DECODE, PREFILL])
def test_packed_solutions_through_runner_vs_oracle(runner, packer, pkg, orc, cuda_dev, definition, tmp_path):
    root = runner.write_trace_set(tmp_path / "traces", decode_batches=(1, 8, 64),
                                  prefill_lengths=([4096], [300, 77, 0, 129], [64] * 40))
    sol_path = tmp_path / "solution.json"
    packer.pack(definition, sol_path)
    work = tmp_path / "solution"
    _seed_library(pkg, packer, definition, work)
    ref = orc.decode if definition == DECODE else orc.prefill
    results = runner.run(root, sol_path, reference=ref, work_dir=work, iters=5)
    assert len(results) == 3
    for r in results:
        c = r["correctness"]
        assert c["within_tolerance"], json.dumps(r)
        assert set(c["per_output"]) == {"output", "new_state"}
        assert 0 < r["median_us"] < 1e5
    assert pkg.prefill.device_status(cuda_dev) == 0
