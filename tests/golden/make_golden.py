"""Generate golden vectors from the reference's own oracle function — run here, once.

Extracts ``naive_self_attention`` from the reference's test.py (test.py:8-15)
with ``ast`` and runs it unchanged except for one token: the causal mask
tensor is created on the inputs' device instead of the literal "cuda"
(test.py:10), so the function runs on the CPU. Inputs follow test.py's
recipe (fp16 N(0, 0.5^2) clamped to +-0.1, cast to e4m3, test.py:30-37) and
also plain N(0,1) e4m3 values; the function sees them dequantised to fp16
(test.py:39-41). Inputs (e4m3 codes, keyed by case), outputs and scales (keyed by case and
scale) are saved to
``tests/golden/naive_attention_cases.npz``.

The generated file is committed; this script needs the reference checkout
and is not run by the tests. Usage: python tests/golden/make_golden.py REFERENCE_ROOT
(or set FA8_REFERENCE_ROOT).
"""
from __future__ import annotations

import ast
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_naive(ref_root: str):
    src = (Path(ref_root) / "test.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef)
              and n.name == "naive_self_attention")
    code = ast.get_source_segment(src, fn).replace('device="cuda"', "device=q.device")
    ns = {"torch": torch}
    exec(compile(code, "reference_test_py_naive_self_attention", "exec"), ns)
    return ns["naive_self_attention"]


def main(ref_root):
    naive = load_naive(ref_root)
    g = torch.Generator().manual_seed(42)
    cases = {}
    specs = [("clamped_s128_d64", 128, 64, "clamped"), ("normal_s128_d64", 128, 64, "normal"),
             ("normal_s256_d128", 256, 128, "normal")]
    for name, S, D, dist in specs:
        shape = (1, 2, S, D)
        def draw():
            if dist == "clamped":
                x = torch.empty(shape, dtype=torch.float16).normal_(0.0, 0.5, generator=g)
                x = x.clamp(-0.1, 0.1)
            else:
                x = torch.randn(shape, generator=g).to(torch.float16)
            return x.to(torch.float8_e4m3fn)
        q, k, v = draw(), draw(), draw()
        cases[name + "_q"] = q.view(torch.uint8).numpy()
        cases[name + "_k"] = k.view(torch.uint8).numpy()
        cases[name + "_v"] = v.view(torch.uint8).numpy()
        for scale_name, scale in (("sqrt_d", 1.0 / math.sqrt(D)), ("sqrt_s", 1.0 / math.sqrt(S))):
            out = naive(q.to(torch.float16), k.to(torch.float16), v.to(torch.float16), scale)
            key = f"{name}_{scale_name}"
            cases[key + "_scale"] = np.float32(scale)
            cases[key + "_out"] = out.numpy()
    np.savez_compressed(HERE / "naive_attention_cases.npz", **cases)
    print(sorted(cases))


if __name__ == "__main__":
    import os
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FA8_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set FA8_REFERENCE_ROOT)")
    main(root)
