"""Generate the committed golden fixtures in this directory. Run from the repository root:

    python tests/golden/make_golden.py --reference PATH_TO_REFERENCE_CHECKOUT

Outputs
  tiny_seed0.npz             the tiny config (G=4, M_total=1024, 64x128, lens [256,0,512,256])
                             as produced by ggemm_asm_b200.inputs, with the oracle's bf16 output
                             bits and the plain-C restatement's float64 output
  reference_group_lens.json  group sizes from the REFERENCE harness's own generator
                             (ggemm-asm bench.py:205-212, make_group_lens), obtained by importing
                             the reference bench.py (its .cuda() call is redirected to the CPU).
                             Only this generation step reads the reference; tests never do.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from ggemm_asm_b200 import inputs  # noqa: E402
from oracle import vark_oracle as vo  # noqa: E402


def make_tiny():
    p = inputs.make_problem("tiny", seed=0)
    ref = vo.wgrad_torch(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    exact = vo.wgrad_c_f64(p.lhs, p.rhs, p.lhs_scale, p.rhs_scale, p.group_offs)
    np.savez_compressed(HERE / "tiny_seed0.npz",
                        lhs_u8=p.lhs.view(torch.uint8).numpy(),
                        rhs_u8=p.rhs.view(torch.uint8).numpy(),
                        lhs_scale=p.lhs_scale.numpy(), rhs_scale=p.rhs_scale.numpy(),
                        group_offs=p.offs, out_bf16_bits=ref.view(torch.uint16).numpy(),
                        out_f64=exact)


def make_reference_lens(ref_root: Path):
    spec = importlib.util.spec_from_file_location("ggemm_asm_reference_bench", ref_root / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    orig_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self  # no GPU here: keep the tensor on the CPU
    try:
        cases = []
        for E, M, seed in [(32, 131072, 42), (128, 1048576, 42), (4, 1024, 42), (32, 131072, 7)]:
            lens = mod.make_group_lens(E, M, seed=seed)
            offs = mod.make_group_offs(lens)
            cases.append({"E": E, "M_total": M, "seed": seed, "lens": lens.tolist(),
                          "offs_last": int(offs[-1])})
    finally:
        torch.Tensor.cuda = orig_cuda
    (HERE / "reference_group_lens.json").write_text(json.dumps(
        {"source": "ggemm-asm bench.py:205-218 make_group_lens/make_group_offs", "cases": cases},
        indent=1) + "\n")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference repository")
    args = ap.parse_args()
    make_tiny()
    if Path(args.reference, "bench.py").exists():
        make_reference_lens(Path(args.reference))
    else:
        print("reference not present: reference_group_lens.json left unchanged")
    print("golden fixtures written to", HERE)
