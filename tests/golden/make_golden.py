"""Generates tests/golden/torch_helper_golden.json from the reference's OWN
PyTorch restatement of its op library.

The reference's pytorch backend (src/backend/pytorch/runtime.rs:114-155)
emits a fixed set of Python helper functions (`tysor_linear`, `tysor_silu`,
`tysor_softmax`, `tysor_rms_norm`, `tysor_cross_entropy`, `tysor_rope`,
`tysor_causal_mask`, `tysor_repeat_kv`, `tysor_flatten_heads`,
`tysor_embedding`, `tysor_dropout`, pattern initialisers) into every script it
runs.  This script reads those string literals from the reference source,
executes them with this container's CPU torch, and records their outputs on
small seeded inputs.  The committed JSON is the golden set the oracle is
checked against (tests/test_oracle_golden.py); nothing at test time reads the
reference tree.

Run from the repository root with the reference checkout's path:

    python tests/golden/make_golden.py <path to the tysor reference checkout>
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np
import torch

HELPERS = os.path.join("src", "backend", "pytorch", "runtime.rs")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "torch_helper_golden.json")


def extract_helpers(path: str) -> str:
    src = open(path).read()
    start = src.index('out.push_str("import torch')
    stop = src.index('out.push_str("def build_parameters')
    chunk = src[start:stop]
    lits = re.findall(r'"((?:[^"\\]|\\.)*)"', chunk)
    code = "".join(lits)
    # Rust string escapes used in these literals.
    code = code.replace("\\n", "\n").replace("\\'", "'").replace('\\"', '"').replace("\\\\", "\\")
    return code


def seeded(shape, seed, lo=-1.0, hi=1.0):
    rng = np.random.default_rng(seed)
    return rng.uniform(lo, hi, size=shape).astype(np.float32)


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the tysor reference checkout>")
    ref = os.path.join(sys.argv[1], HELPERS)
    ns: dict = {}
    exec(compile(extract_helpers(ref), ref, "exec"), ns)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    cases = []

    def add(name, op, inputs, args, out):
        cases.append({
            "name": name, "op": op,
            "inputs": {k: {"shape": list(v.shape), "data": [float(x) for x in v.reshape(-1)]}
                       for k, v in inputs.items()},
            "args": args,
            "out": {"shape": list(out.shape), "data": [float(x) for x in out.reshape(-1).tolist()]},
        })

    # pattern initialisers
    for (i, o) in [(3, 4), (16, 3)]:
        add(f"linear_weight_{i}x{o}", "linear_weight", {}, {"in": i, "out": o},
            ns["tysor_init_linear_weight"](i, o).numpy())
        add(f"linear_bias_{o}", "linear_bias", {}, {"out": o}, ns["tysor_init_linear_bias"](o).numpy())
    add("embedding_weight_32x8", "embedding_weight", {}, {"num": 32, "dim": 8},
        ns["tysor_init_embedding_weight"](32, 8).numpy())

    for seed, (r, w) in enumerate([(2, 3), (4, 17), (8, 64), (3, 257)]):
        x = seeded((r, w), 100 + seed, -3, 3)
        add(f"silu_{r}x{w}", "silu", {"x": x}, {}, ns["tysor_silu"](T(x)).numpy())
        add(f"softmax_{r}x{w}", "softmax", {"x": x}, {}, ns["tysor_softmax"](T(x)).numpy())
        add(f"rms_norm_{r}x{w}", "rms_norm", {"x": x}, {"hidden": w},
            ns["tysor_rms_norm"](T(x), w).numpy())
        add(f"dropout_{r}x{w}", "dropout", {"x": x}, {"p": 0.25},
            ns["tysor_dropout"](T(x), 0.25).numpy())
        t = np.abs(seeded((r, w), 200 + seed, 0, 1))
        t = (t / t.sum(axis=1, keepdims=True)).astype(np.float32)
        add(f"cross_entropy_{r}x{w}", "cross_entropy", {"logits": x, "target": t}, {},
            ns["tysor_cross_entropy"](T(x), T(t)).numpy())

    for seed, (m, k, n) in enumerate([(2, 3, 4), (5, 7, 3), (16, 32, 8)]):
        x = seeded((m, k), 300 + seed)
        w = seeded((k, n), 400 + seed)
        b = seeded((n,), 500 + seed)
        add(f"linear_{m}x{k}x{n}", "linear", {"x": x, "w": w, "b": b}, {},
            ns["tysor_linear"](T(x), T(w), T(b)).numpy())
        add(f"linear_nobias_{m}x{k}x{n}", "linear", {"x": x, "w": w}, {},
            ns["tysor_linear"](T(x), T(w)).numpy())

    for seed, shape in enumerate([(1, 2, 4), (2, 3, 5, 8), (1, 4, 16, 16)]):
        x = seeded(shape, 600 + seed, -2, 2)
        add(f"rope_{'x'.join(map(str, shape))}", "rope", {"x": x},
            {"head_dim": shape[-1], "theta": 10000.0},
            ns["tysor_rope"](T(x), shape[-1], 10000.0).numpy())
        add(f"causal_mask_{'x'.join(map(str, shape))}", "causal_mask", {"x": x}, {},
            ns["tysor_causal_mask"](T(x)).numpy())
        add(f"flatten_heads_{'x'.join(map(str, shape))}", "flatten_heads", {"x": x}, {},
            ns["tysor_flatten_heads"](T(x)).numpy())
        add(f"repeat_kv_{'x'.join(map(str, shape))}", "repeat_kv", {"x": x}, {"repeats": 3},
            ns["tysor_repeat_kv"](T(x), 3).numpy())

    emb = ns["tysor_init_embedding_weight"](32, 8).numpy()
    idx = np.array([0.0, 5.0, 31.0, 7.9, 16.0], dtype=np.float32)
    add("embedding_pattern_32x8", "embedding", {"idx": idx, "weight": emb}, {},
        ns["tysor_embedding"](T(idx), T(emb)).numpy())

    with open(OUT, "w") as f:
        json.dump({"source": "src/backend/pytorch/runtime.rs:114-155 helper functions, run with torch "
                             + torch.__version__ + " on CPU",
                   "cases": cases}, f)
    print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    sys.exit(main())
