"""Data-parallel test cases shared by tests/test_gpu_dp.py and the per-rank
worker (tests/dp_worker.py): one rank's share of a seeded batch.

* `mlp`: the two-layer MLP at full size, x and target [8192, 1024], rows
  sharded evenly (tysor_b200.dist.shard_rows), mean squared error over the
  global batch.
* `lm`: a 2-layer llama_lm (d 128, 4/2 heads, ffn 192, vocab 512) on
  4 sequences of 64 tokens, split evenly at world sizes 2 and 4.

world == 1 gives the full batch, whose gradient the ranks' summed
gradients must equal.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tysor_b200.dist import shard_rows  # noqa: E402
from tysor_b200.programs import llama_lm, mlp_train, random_parameters  # noqa: E402

MLP = dict(rows=8192, d_in=1024, d_hidden=4096)
LM = dict(layers=2, batch=4, seq=64, d_model=128, n_heads=4, n_kv_heads=2, hidden=192, vocab=512)


def case(workload, rank, world):
    """(graph, shapes, inputs, parameters) of `rank`'s shard."""
    if workload == "mlp":
        rows, d_in, d_h = MLP["rows"], MLP["d_in"], MLP["d_hidden"]
        g = mlp_train(d_in, d_h, d_in, lr=0.0, iterations=1, loss_scale=1.0 / (rows * d_in))
        lo, hi = shard_rows(rows, rank, world)
        x = np.random.default_rng(0).standard_normal((rows, d_in), dtype=np.float32)
        t = np.random.default_rng(1).standard_normal((rows, d_in), dtype=np.float32)
        inputs = {"x": np.ascontiguousarray(x[lo:hi]), "target": np.ascontiguousarray(t[lo:hi])}
        shapes = {"x": [hi - lo, d_in], "target": [hi - lo, d_in]}
        return g, shapes, inputs, random_parameters(g, 1234)
    if workload == "lm":
        lo, hi = shard_rows(LM["batch"], rank, world)
        cfg = dict(LM, batch=hi - lo)
        g = llama_lm(**cfg, lr=0.0, iterations=1)
        seqs = np.random.default_rng(11).integers(0, LM["vocab"], (LM["batch"], LM["seq"] + 1))[lo:hi]
        inputs = {"ids": np.ascontiguousarray(seqs[:, :-1]).astype(np.float32).reshape(-1),
                  "labels": np.ascontiguousarray(seqs[:, 1:]).astype(np.float32).reshape(-1)}
        t = (hi - lo) * LM["seq"]
        return g, {"ids": [t], "labels": [t]}, inputs, random_parameters(g, 4)
    raise ValueError(workload)
