"""Golden-vector cases: seeded inputs whose reference outputs live in *.npz.

The inputs are rebuilt from the seed by ``kachua-mlsys_b200/inputs.py``; the
stored digest guards against a silent change of the generator.
"""
from __future__ import annotations

import hashlib
import importlib.util
import sys
from pathlib import Path

_REPO = Path(__file__).resolve().parents[2]


def _inputs_module():
    name = "kachua_mlsys_b200.inputs"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, _REPO / "kachua-mlsys_b200" / "inputs.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


CASES = {
    # decode, default scale (None -> 1/sqrt(128)), two sequences
    "decode_b2": {"kind": "decode", "batch": 2, "seed": 1, "scale": None},
    # decode with an explicit, non-default scale
    "decode_b1_scale": {"kind": "decode", "batch": 1, "seed": 2, "scale": 0.05},
    # varlen prefill: ragged lengths, an empty sequence, a chunk-crossing one
    "prefill_varlen": {"kind": "prefill", "lengths": [5, 0, 70], "seed": 3, "state": True},
    # prefill with state=None (zero initial state)
    "prefill_nostate": {"kind": "prefill", "lengths": [17], "seed": 4, "state": False},
}


def build_inputs(case):
    inp_mod = _inputs_module()
    if case["kind"] == "decode":
        inp = inp_mod.make_decode_inputs(case["batch"], seed=case["seed"])
    else:
        inp = inp_mod.make_prefill_inputs(case["lengths"], seed=case["seed"],
                                          with_state=case["state"])
    inp.scale = case["scale"] if "scale" in case else inp.scale
    return inp


def input_digest(inp) -> str:
    h = hashlib.sha1()
    for t in inp.args():
        if t is None:
            h.update(b"none")
        elif hasattr(t, "numpy"):
            h.update(t.contiguous().view(-1).view(__import__("torch").uint8).numpy().tobytes())
        else:
            h.update(repr(t).encode())
    return h.hexdigest()
