"""The FlashInfer-Bench drop-in modules load and keep the reference's entry
signatures (decode kernel.cu:982-994 / triton/kernel.py:27; prefill
triton/kernel.py:56)."""
import importlib.util
import inspect
import tomllib
from pathlib import Path

import pytest

SOL = Path(__file__).resolve().parents[1] / "kachua-mlsys_b200" / "solutions"
EXPECTED = {
    "gdn_decode_qk4_v8_d128_k_last":
        ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale", "output", "new_state"],
    "gdn_prefill_qk4_v8_d128_k_last":
        ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale", "output", "new_state"],
}


@pytest.mark.parametrize("definition", sorted(EXPECTED))
def test_solution_entry(definition):
    cfg = tomllib.loads((SOL / definition / "config.toml").read_text())
    assert cfg["solution"]["definition"] == definition
    fname, func = cfg["build"]["entry_point"].split("::")
    path = SOL / definition / "solution" / "b200" / fname
    spec = importlib.util.spec_from_file_location(f"sol_{definition}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    fn = getattr(mod, func)
    assert list(inspect.signature(fn).parameters) == EXPECTED[definition]
