"""The Llama-style decoder block (batched matmul, transpose, RoPE, repeat_kv,
causal mask, Softmax, RMSNorm gain, SwiGLU) forward + backward + SGD on the
device against the oracle, at a reduced size that still runs every matmul
on the tcgen05 path.  Bars: forward output Frobenius rel 1e-5; parameter
gradients rel 1e-4 (a dozen chained strict matmuls and row reductions);
losses over 3 SGD steps rel 1e-4."""
import numpy as np
import pytest

import local as L
from tysor_b200.programs import llama_block

pytestmark = pytest.mark.gpu

CFG = dict(batch=2, seq=64, d_model=256, n_heads=4, n_kv_heads=2, hidden=384, eps=1e-6, lr=1e-4)


def frob(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def params_for(g, seed=5):
    rng = np.random.default_rng(seed)
    consts = {n.output: n.const for n in g.nodes if n.kind == "const"}
    out = {}
    for n in g.nodes:
        if n.kind == "ctor" and n.op == "linear":
            i, o = consts[n.inputs[0]], consts[n.inputs[1]]
            out[f"linear_{n.output}_weight"] = (0.05 * rng.standard_normal((i, o))).astype(np.float32)
        elif n.kind == "ctor" and n.op == "RMSNorm":
            h = consts[n.inputs[0]]
            out[f"rmsnorm_{n.output}_gain"] = (1 + 0.02 * rng.standard_normal(h)).astype(np.float32)
    return out


def test_block_forward_backward_and_sgd(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    g = llama_block(**CFG)
    T = CFG["batch"] * CFG["seq"]
    shapes = {"x": [T, CFG["d_model"]]}
    x = np.random.default_rng(1).standard_normal((T, CFG["d_model"])).astype(np.float32)
    params = params_for(g)
    oparams = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}

    values, grads, _ = L.train_step_grads(g, shapes, inputs={"x": x}, parameters=oparams)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": x}, parameters=params)
    losses = ex.train(1, 0.0)  # lr 0: parameters stay, gradients are kept
    out_id = g.outputs[0]
    assert frob(ex.value(out_id).data, values[out_id][1].data) < 1e-5
    for name, gt in grads.items():
        assert frob(ex.parameter_grad(name), gt.data) < 1e-4, name
    assert abs(losses[0] - L.tensor_sum(values[out_id][1])) <= 1e-4 * abs(L.tensor_sum(values[out_id][1])) + 1e-2
    ex.close()

    want_losses, want_params = L.train(g, shapes, inputs={"x": x}, parameters=oparams, lr=CFG["lr"], iterations=3)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": x}, parameters=params)
    got = ex.train(3, CFG["lr"])
    # The loss is a sum of ~N(0,1) outputs that mostly cancel (sum ~ 3 over
    # 32768 terms of magnitude ~1), so its error is judged against the size
    # of the terms: rel 1e-5 of sum(|out|).
    scale = float(np.abs(values[out_id][1].data).sum())
    for a, b in zip(got, want_losses):
        assert abs(a - b) <= 1e-5 * scale, (got, want_losses, scale)
    for name, t in want_params.items():
        assert frob(ex.parameter(name), t.data) < 1e-5, name
    ex.close()


@pytest.mark.parametrize("shape", [[2, 3, 64, 32], [1, 2, 1024, 32], [1, 2, 2048, 32]])
def test_attention_core_with_fused_scale_and_masked_softmax(cuda_ctx, shape):
    """softmax(causal_mask(scale(q . k^T, c))) . v, training semantics: the
    executor folds the scale into the GEMM's alpha and runs mask+softmax as
    one kernel (forward and backward); values and the gradients reaching q,
    k and v must match the op-by-op oracle.  Row widths that are multiples
    of 1024 take the register-resident softmax (one or two warps per row
    at widths 1024 and 2048)."""
    from tysor_b200.graph import GraphBuilder
    from tysor_b200.runtime import CudaGraphExecutor
    b = GraphBuilder()
    q, k, v = b.param("q"), b.param("k"), b.param("v")
    kt = b.call("transpose", k, 2, 3)
    s = b.call("scale", b.call("matmul", q, kt), 0.17)
    p = b.let("p", b.apply(b.ctor("Softmax"), b.call("causal_mask", s)))
    out = b.let("out", b.call("matmul", p, v))
    b.ret(out)
    b.train(objective="out", lr=0.0)
    g = b.build()
    rng = np.random.default_rng(3)
    ins = {n: rng.standard_normal(shape).astype(np.float32) for n in ("q", "k", "v")}
    shapes = {n: shape for n in ins}
    vgrads = {}
    values, _, _ = L.train_step_grads(g, shapes, inputs=ins, value_grads=vgrads)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins)
    ex.train(1, 0.0)
    assert frob(ex.value(g.named["p"]).data, values[g.named["p"]][1].data) < 1e-5
    assert frob(ex.value(out).data, values[out][1].data) < 1e-5
    for name in ("q", "k", "v"):
        vid = g.named[name]
        assert frob(ex.value_grad(vid).data, vgrads[vid].data) < 1e-5, name
    ex.close()


def test_block_medium_uses_transposed_operand_copies(cuda_ctx):
    """A size at which the executor transposes the M/N-contiguous operands of
    the weight-gradient and attention matmuls before the GEMM (operand
    elements x 2000 <= GEMM FLOPs): gradients and the updated parameters must
    still match the oracle, and nothing may be NaN."""
    from tysor_b200.runtime import CudaGraphExecutor
    cfg = dict(batch=1, seq=512, d_model=512, n_heads=4, n_kv_heads=2, hidden=1024, eps=1e-6, lr=1e-5)
    g = llama_block(**cfg)
    T = cfg["seq"]
    shapes = {"x": [T, cfg["d_model"]]}
    x = np.random.default_rng(2).standard_normal((T, cfg["d_model"])).astype(np.float32)
    params = params_for(g, seed=9)
    oparams = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
    L.set_threads(16)
    values, grads, _ = L.train_step_grads(g, shapes, inputs={"x": x}, parameters=oparams)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": x}, parameters=params)
    losses = ex.train(1, 0.0)
    assert np.isfinite(losses).all()
    out_id = g.outputs[0]
    assert frob(ex.value(out_id).data, values[out_id][1].data) < 1e-5
    for name, gt in grads.items():
        got = ex.parameter_grad(name)
        assert np.isfinite(got).all(), name
        assert frob(got, gt.data) < 1e-4, name
    ex.close()


def test_traced_step_reports_every_item_and_matches_a_plain_step(cuda_ctx):
    """tysor_cuda_graph_train_traced runs the same step op by op: every item
    has a forward/backward/update label and a device time, and the gradients
    it leaves equal the oracle's."""
    from tysor_b200.runtime import CudaGraphExecutor
    g = llama_block(**CFG)
    T = CFG["batch"] * CFG["seq"]
    shapes = {"x": [T, CFG["d_model"]]}
    x = np.random.default_rng(1).standard_normal((T, CFG["d_model"])).astype(np.float32)
    params = params_for(g)
    oparams = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
    _, grads, _ = L.train_step_grads(g, shapes, inputs={"x": x}, parameters=oparams)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": x}, parameters=params)
    items = ex.train_traced(0.0)
    assert len(items) > 20
    assert all(lab.split(" ")[0] in ("fwd", "bwd", "update") for lab, _ in items), items[:5]
    assert all(ms >= 0.0 for _, ms in items)
    assert any(lab.startswith("fwd apply linear") for lab, _ in items)
    for name, gt in grads.items():
        assert frob(ex.parameter_grad(name), gt.data) < 1e-4, name
    ex.close()


@pytest.mark.parametrize("seq", [200, 256, 1024, 2048])
def test_fused_causal_attention_rows_whose_masked_entries_keep_probability(cuda_ctx, seq):
    """The causal GEMMs skip masked entries as exact zeros, which they are
    unless a row's visible scores all lie below about -9896: then every
    masked entry keeps probability exp(-1e4 - max) / d (here 1 / #masked).
    Such rows are computed as the reference computes them: the softmax
    records each row's masked probability and fix-ups after P.V and after
    dV add the skipped terms.  Head 0 has ordinary scores.  In head 1 every
    key is the constant 60 and the first half of the queries the constant
    -60 (scores -19584: those rows leak, their visible entries get
    probability 0 and every masked one 1 / #masked), the second half
    ordinary (each row's scores equal across keys); constant operands keep
    the scores exact, so the check is not swamped by the conditioning of
    softmax at scores of -2e4.  Probabilities, output and the gradients
    reaching q, k and v against the op-by-op oracle.  (At 200 tokens the
    GEMMs take 128-row tiles, at 256 and more 256-row pair tiles.)"""
    from tysor_b200.graph import GraphBuilder
    from tysor_b200.runtime import CudaGraphExecutor
    b = GraphBuilder()
    q, k, v = b.param("q"), b.param("k"), b.param("v")
    s = b.call("scale", b.call("matmul", q, b.call("transpose", k, 2, 3)), 0.17)
    p = b.let("p", b.apply(b.ctor("Softmax"), b.call("causal_mask", s)))
    out = b.let("out", b.call("matmul", p, v))
    b.ret(out)
    b.train(objective="out", lr=0.0)
    g = b.build()
    shape = [1, 2, seq, 32]
    rng = np.random.default_rng(seq)
    ins = {n: rng.standard_normal(shape).astype(np.float32) for n in ("q", "k", "v")}
    ins["k"][0, 1] = 60.0
    ins["q"][0, 1, : seq // 2] = -60.0
    shapes = {n: shape for n in ins}
    vgrads = {}
    L.set_threads(16)
    values, _, _ = L.train_step_grads(g, shapes, inputs=ins, value_grads=vgrads)
    want_p = values[g.named["p"]][1].data.reshape(shape[:2] + [seq, seq])
    assert want_p[0, 1, 0, 1] > 0.0  # the second head's rows do leak
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins)
    ex.train(1, 0.0)
    assert frob(ex.value(g.named["p"]).data, values[g.named["p"]][1].data) < 1e-5
    assert frob(ex.value(out).data, values[out][1].data) < 1e-5
    for name in ("q", "k", "v"):
        vid = g.named[name]
        assert frob(ex.value_grad(vid).data, vgrads[vid].data) < 1e-5, name
    ex.close()


def test_weight_gradients_with_split_k(cuda_ctx):
    """Weight gradients with few output tiles and a long K (8192 rows into a
    256 x 256 weight) take the split-K path (parts summed in a fixed order);
    the second use of the same weight accumulates into the first's
    gradient.  Gradients against the oracle at rel 1e-5."""
    from tysor_b200.graph import GraphBuilder
    from tysor_b200.runtime import CudaGraphExecutor
    rows, d = 8192, 256
    b = GraphBuilder()
    x1, x2 = b.param("x1"), b.param("x2")
    lin = b.let("lin", b.ctor("linear", d, d, False))
    h = b.binary("*", b.apply(lin, x1), b.apply(lin, x2))
    b.ret(b.let("out", h))
    b.train(objective="out", lr=0.0)
    g = b.build()
    rng = np.random.default_rng(21)
    ins = {"x1": rng.standard_normal((rows, d)).astype(np.float32),
           "x2": rng.standard_normal((rows, d)).astype(np.float32)}
    shapes = {k: [rows, d] for k in ins}
    params = {f"linear_{g.named['lin']}_weight": (0.05 * rng.standard_normal((d, d))).astype(np.float32)}
    oparams = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
    L.set_threads(16)
    _, grads, _ = L.train_step_grads(g, shapes, inputs=ins, parameters=oparams)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    ex.train(1, 0.0)
    for name, gt in grads.items():
        assert frob(ex.parameter_grad(name), gt.data) < 1e-5, name
    ex.close()


def test_gradient_buffers_handed_to_inputs(cuda_ctx):
    """Training hands a node's gradient buffer to one input instead of
    copying it (a view's input, one operand of '+' or '-'); later
    contributions then add into that buffer.  A graph where the same value
    reaches the objective through a view, both operands of '+', and '-':
    parameter gradients and updated parameters against the oracle."""
    from tysor_b200.graph import GraphBuilder
    from tysor_b200.runtime import CudaGraphExecutor
    b = GraphBuilder()
    x = b.param("x")
    l1 = b.let("l1", b.ctor("linear", 64, 64, False))
    a = b.let("a", b.apply(l1, x))
    v = b.call("reshape", b.call("reshape", a, 8, 16, 64), 128, 64)
    c = b.binary("+", a, v)
    d = b.binary("-", c, b.binary("+", a, a))
    e = b.binary("+", d, c)
    b.ret(b.let("loss", b.binary("*", e, e)))
    b.train(objective="loss", lr=1e-3, iterations=1)
    g = b.build()
    shapes = {"x": [128, 64]}
    xv = np.random.default_rng(4).standard_normal((128, 64)).astype(np.float32)
    params = params_for(g, seed=6)
    oparams = {k: L.Tensor(list(p.shape), p.reshape(-1).copy()) for k, p in params.items()}
    _, grads, _ = L.train_step_grads(g, shapes, inputs={"x": xv}, parameters=oparams)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": xv}, parameters=params)
    ex.train(1, 0.0)
    for name, gt in grads.items():
        assert frob(ex.parameter_grad(name), gt.data) < 1e-5, name
    ex.close()
