"""The stacked-block language model (`llama_lm`: embedding, decoder blocks,
final RMSNorm, tied output projection, next-token cross entropy against
labels) on the device against the oracle at a reduced size.  Bars: loss
rel 1e-5; parameter gradients Frobenius rel 1e-4; losses over 3 SGD steps
rel 1e-4 (the tracking bar for training)."""
import numpy as np
import pytest

import local as L
from tysor_b200.graph import GraphBuilder
from tysor_b200.programs import llama_lm, random_parameters

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, batch=2, seq=64, d_model=128, n_heads=4, n_kv_heads=2, hidden=192, vocab=512)


def frob(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def lm_case(lr):
    g = llama_lm(**CFG, lr=lr, iterations=3)
    t = CFG["batch"] * CFG["seq"]
    seq = np.random.default_rng(11).integers(0, CFG["vocab"], t + 1)
    inputs = {"ids": seq[:-1].astype(np.float32), "labels": seq[1:].astype(np.float32)}
    params = random_parameters(g, seed=4)
    return g, {"ids": [t], "labels": [t]}, inputs, params


def to_oracle(params):
    return {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}


def test_tied_logits_and_embedding_gradients(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    num, dim, rows = 300, 64, 96
    b = GraphBuilder()
    ids, labels = b.param("ids"), b.param("labels")
    emb = b.let("emb", b.ctor("Embedding", num, dim))
    x = b.let("x", b.apply(emb, ids))
    logits = b.let("logits", b.call("tied_logits", x, emb))
    b.ret(b.let("loss", b.call("cross_entropy", logits, labels)))
    b.train(objective="loss", lr=0.0)
    g = b.build()
    rng = np.random.default_rng(2)
    inputs = {"ids": rng.integers(0, num, rows).astype(np.float32),
              "labels": rng.integers(0, num, rows).astype(np.float32)}
    params = random_parameters(g, seed=7, std=0.5)
    shapes = {"ids": [rows], "labels": [rows]}
    values, grads, _ = L.train_step_grads(g, shapes, inputs=inputs, parameters=to_oracle(params))
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=inputs, parameters=params)
    ex.train(1, 0.0)
    lid = g.named["logits"]
    assert frob(ex.value(lid).data, values[lid][1].data) < 1e-5
    name = f"embedding_{g.named['emb']}_weight"
    assert frob(ex.parameter_grad(name), grads[name].data) < 1e-5
    ex.close()


def test_lm_gradients_match_the_oracle(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    g, shapes, inputs, params = lm_case(0.0)
    L.set_threads(16)
    values, grads, _ = L.train_step_grads(g, shapes, inputs=inputs, parameters=to_oracle(params))
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=inputs, parameters=params)
    losses = ex.train(1, 0.0)
    oid = g.objective_id()
    want = float(values[oid][1].data.astype(np.float64).sum())
    assert abs(losses[0] - want) <= 1e-5 * abs(want), (losses, want)
    assert len(grads) == len(params)
    for name, gt in grads.items():
        got = ex.parameter_grad(name)
        assert np.isfinite(got).all(), name
        assert frob(got, gt.data) < 1e-4, name
    ex.close()


def test_lm_training_tracks_the_oracle(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    g, shapes, inputs, params = lm_case(0.01)
    L.set_threads(16)
    want, wparams = L.train(g, shapes, inputs=inputs, parameters=to_oracle(params))
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=inputs, parameters=params)
    got = ex.train()
    assert len(got) == 3
    for a, b in zip(got, want):
        assert abs(a - b) <= 1e-4 * abs(b), (got, want)
    assert want[-1] < want[0]
    for name, t in wparams.items():
        assert frob(ex.parameter(name), t.data) < 1e-5, name
    ex.close()
