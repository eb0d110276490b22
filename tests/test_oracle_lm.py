"""The oracle's tied output projection (`tied_logits`, an extension with no
reference counterpart) against a float64 NumPy restatement, and a small
`llama_lm` training run on the oracle (losses finite and decreasing, as the
reference's harness requires of train fixtures, run_tests.rs:525-530)."""
import numpy as np

import local as L
from tysor_b200.graph import GraphBuilder
from tysor_b200.programs import llama_lm, random_parameters


def _softmax64(z):
    z = z - z.max(axis=1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=1, keepdims=True)


def test_tied_logits_forward_and_gradients():
    num, dim, rows = 37, 12, 9
    b = GraphBuilder()
    ids, labels = b.param("ids"), b.param("labels")
    emb = b.let("emb", b.ctor("Embedding", num, dim))
    x = b.let("x", b.apply(emb, ids))
    logits = b.let("logits", b.call("tied_logits", x, emb))
    b.ret(b.let("loss", b.call("cross_entropy", logits, labels)))
    b.train(objective="loss", lr=0.0)
    g = b.build()
    rng = np.random.default_rng(0)
    idv = rng.integers(0, num, rows)
    lab = rng.integers(0, num, rows)
    table = rng.standard_normal((num, dim)).astype(np.float32)
    name = f"embedding_{g.named['emb']}_weight"
    params = {name: L.Tensor([num, dim], table.reshape(-1).copy())}
    values, grads, _ = L.train_step_grads(g, {"ids": [rows], "labels": [rows]},
                                          inputs={"ids": idv.astype(np.float32), "labels": lab.astype(np.float32)},
                                          parameters=params)
    e64 = table.astype(np.float64)
    x64 = e64[idv]
    z = x64 @ e64.T
    got_logits = values[g.named["logits"]][1].data.reshape(rows, num)
    np.testing.assert_allclose(got_logits, z, rtol=1e-5, atol=1e-5)
    # cross_entropy backward is softmax - onehot (layers.rs:479-488)
    G = _softmax64(z)
    G[np.arange(rows), lab] -= 1.0
    dX = G @ e64
    dE = G.T @ x64
    np.add.at(dE, idv, dX)  # embedding backward: scatter-add of the rows' gradients
    got = grads[name].data.reshape(num, dim)
    assert np.linalg.norm(got - dE) / np.linalg.norm(dE) < 1e-5


def test_tied_logits_rejects_a_non_embedding_callee():
    b = GraphBuilder()
    x = b.param("x")
    lin = b.let("lin", b.ctor("linear", 4, 4, False))
    b.ret(b.call("tied_logits", x, lin))
    g = b.build()
    try:
        L.run_forward(g, {"x": [2, 4]})
    except L.OracleError as e:
        assert "Embedding constructor" in str(e)
    else:
        raise AssertionError("expected an error")


def test_small_lm_trains_on_the_oracle():
    cfg = dict(layers=2, batch=1, seq=16, d_model=32, n_heads=4, n_kv_heads=2, hidden=48, vocab=64)
    g = llama_lm(**cfg, lr=0.01, iterations=4)
    rng = np.random.default_rng(1)
    t = cfg["batch"] * cfg["seq"]
    seq = rng.integers(0, cfg["vocab"], t + 1)
    inputs = {"ids": seq[:-1].astype(np.float32), "labels": seq[1:].astype(np.float32)}
    init = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in random_parameters(g, 3).items()}
    losses, params = L.train(g, {"ids": [t], "labels": [t]}, inputs=inputs, parameters=init)
    assert len(losses) == 4 and np.isfinite(losses).all()
    assert all(b < a for a, b in zip(losses, losses[1:])), losses
    emb = [k for k in params if k.startswith("embedding_")]
    assert len(emb) == 1 and params[emb[0]].shape == [cfg["vocab"], cfg["d_model"]]
