"""Generate the golden vectors that pin the C oracle to the reference.

Run manually in a container that has the reference checkout (read-only):

    python tests/golden/gen_golden.py --reference /path/to/kachua-mlsys

It imports the reference's own PyTorch implementations

  gdn_decode_qk4_v8_d128_k_last/solution/reference_torch_impl.py  (run, :12-72)
  gdn_prefill_qk4_v8_d128_k_last/solution/reference_torch_impl.py (run, :17-92)

runs them on seeded synthetic inputs from ``kachua-mlsys_b200/inputs.py`` and
stores inputs (as a seed + a checksum) and the reference outputs in
``tests/golden/*.npz``.  Nothing at test time reads the reference checkout.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from tests.golden.cases import CASES, build_inputs, input_digest  # noqa: E402


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    args = ap.parse_args()
    ref = Path(args.reference)
    dec = _load(ref / "gdn_decode_qk4_v8_d128_k_last/solution/reference_torch_impl.py", "ref_dec")
    pre = _load(ref / "gdn_prefill_qk4_v8_d128_k_last/solution/reference_torch_impl.py", "ref_pre")
    torch.set_num_threads(8)
    for name, case in CASES.items():
        inp = build_inputs(case)
        if case["kind"] == "decode":
            out, ns = dec.run(*inp.args())
        else:
            out, ns = pre.run(*inp.args())
        np.savez_compressed(
            Path(__file__).parent / f"{name}.npz",
            digest=np.frombuffer(input_digest(inp).encode(), dtype=np.uint8),
            output=out.float().numpy() if out.dtype != torch.bfloat16 else out.view(torch.int16).numpy(),
            output_is_bf16=np.array(out.dtype == torch.bfloat16),
            new_state=ns.numpy(),
        )
        print(name, tuple(out.shape), tuple(ns.shape), hashlib.sha1(ns.numpy().tobytes()).hexdigest()[:12])


if __name__ == "__main__":
    main()
