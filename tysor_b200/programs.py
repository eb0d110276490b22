"""Lowered graphs of tysor programs.

Two groups:

* `FIXTURES`: the reference's hot-path test fixtures (tests/*.ty allowlisted
  for the native backend in src/bin/run_tests.rs:34-66), lowered by hand with
  `GraphBuilder` in the order the reference front end lowers them, together
  with the `--shape` arguments the harness passes (run_tests.rs:229-267).
* Workloads named by their sizes: the matmul+relu program at 2048^2, the
  two-layer MLP trainer, and the Llama-style decoder block, which needs the
  extensions (batched matmul, `transpose`, `RMSNorm` gain) the reference
  cannot express.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List

import numpy as np

from .graph import Graph, GraphBuilder


@dataclass
class Fixture:
    name: str
    build: Callable[[], Graph]
    shapes: Dict[str, List[int]]
    modes: List[str] = field(default_factory=list)   # run | backward | train


# ---- reference fixtures ----------------------------------------------------

# Every allowlisted fixture declares its parameters `tensor[float16]`; the
# string is carried into the printed results (computation stays f32).
FIXTURE_DTYPE = "float16"


def _model_matmul_relu() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x, w = b.param("x"), b.param("w")
    y = b.let("y", b.call("matmul", x, w))
    z = b.let("z", b.call("relu", y))
    b.ret(z)
    return b.build()


def _run_activation_layers() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    sm = b.ctor("Softmax")
    si = b.ctor("SiLU")
    b.ret(b.apply(sm, b.apply(si, x)))
    return b.build()


def _run_binary_ops() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x, y = b.param("x"), b.param("y")
    s = b.let("sum", b.binary("+", x, y))
    d = b.let("diff", b.binary("-", s, y))
    sc = b.let("scaled", b.binary("*", d, 2.0))
    sh = b.let("shifted", b.binary("+", 1.0, sc))
    b.ret(b.binary("/", sh, 2.0))
    return b.build()


def _run_cross_entropy() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    lg, t = b.param("logits"), b.param("target")
    b.ret(b.call("cross_entropy", lg, t))
    return b.build()


def _run_dropout() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    drop = b.let("drop", b.ctor("Dropout", 0.25))
    b.ret(b.apply(drop, x))
    return b.build()


def _run_linear_bias() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    proj = b.let("proj", b.ctor("linear", 3, 2, True))
    b.ret(b.apply(proj, x))
    return b.build()


def _transformer(b: GraphBuilder, idx, mask: bool):
    tok = b.let("tok", b.ctor("Embedding", 32, 8))
    out_proj = b.let("out_proj", b.ctor("linear", 16, 3, False))
    x = b.let("x", b.apply(tok, idx))
    x = b.let("x", b.call("rms_norm", x, 8))
    x = b.let("x", b.call("reshape", x, 1, 2, 4))
    x = b.let("x", b.call("rope", x, 4, 10000.0))
    x = b.let("x", b.call("repeat_kv", x, 2))
    if mask:
        x = b.let("x", b.call("causal_mask", x))
    x = b.let("x", b.call("flatten_heads", x))
    return b.let("logits", b.apply(out_proj, x))


def _run_transformer_mask() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    idx = b.param("idx")
    b.ret(_transformer(b, idx, True))
    return b.build()


def _run_rms_norm() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    b.ret(b.call("rms_norm", x, 3))
    return b.build()


def _run_scale_builtin() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    y = b.let("y", b.call("scale", x, 2.0))
    z = b.let("z", b.call("relu", y))
    b.ret(b.call("scale", z, 0.5))
    return b.build()


def _run_two_layer_mlp() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    hidden = b.let("hidden", b.ctor("linear", 3, 4))
    out = b.let("out", b.ctor("linear", 4, 2, False))
    b.ret(b.apply(out, b.call("relu", b.apply(hidden, x))))
    return b.build()


def _backward_basic_ops() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x, y, w = b.param("x"), b.param("y"), b.param("w")
    prod = b.let("prod", b.binary("*", x, y))
    logits = b.let("logits", b.call("matmul", prod, w))
    loss = b.let("loss", b.call("relu", b.call("scale", logits, 0.5)))
    b.ret(loss)
    b.train(objective="loss", lr=0.1)
    return b.build()


def _backward_cross_entropy() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    lg, t = b.param("logits"), b.param("target")
    b.ret(b.let("loss", b.call("cross_entropy", lg, t)))
    b.train(objective="loss", lr=0.1)
    return b.build()


def _backward_dropout() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    drop = b.let("drop", b.ctor("Dropout", 0.25))
    b.ret(b.let("y", b.apply(drop, x)))
    b.train(objective="y", lr=0.1)
    return b.build()


def _backward_linear(bias: bool) -> Callable[[], Graph]:
    def build() -> Graph:
        b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
        x = b.param("x")
        proj = b.let("proj", b.ctor("linear", 3, 2, bias))
        b.ret(b.let("y", b.apply(proj, x)))
        b.train(objective="y", lr=0.1)
        return b.build()
    return build


def _backward_rms_norm() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x = b.param("x")
    b.ret(b.let("y", b.call("rms_norm", x, 3)))
    b.train(objective="y", lr=0.1)
    return b.build()


def _backward_act(op: str) -> Callable[[], Graph]:
    def build() -> Graph:
        b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
        x = b.param("x")
        b.ret(b.let("y", b.apply(b.ctor(op), x)))
        b.train(objective="y", lr=0.1)
        return b.build()
    return build


def _train_linear_ce(bias: bool, iterations: int) -> Callable[[], Graph]:
    def build() -> Graph:
        b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
        x, t = b.param("x"), b.param("target")
        proj = b.let("proj", b.ctor("linear", 3, 3, bias))
        logits = b.let("logits", b.apply(proj, x))
        b.ret(b.let("loss", b.call("cross_entropy", logits, t)))
        b.train(objective="loss", lr=0.05, iterations=iterations)
        return b.build()
    return build


def _train_dropout() -> Graph:
    b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
    x, t = b.param("x"), b.param("target")
    proj = b.let("proj", b.ctor("linear", 3, 3, False))
    drop = b.let("drop", b.ctor("Dropout", 0.25))
    logits = b.let("logits", b.apply(drop, b.apply(proj, x)))
    b.ret(b.let("loss", b.call("cross_entropy", logits, t)))
    b.train(objective="loss", lr=0.05, iterations=3)
    return b.build()


def _train_transformer(mask: bool) -> Callable[[], Graph]:
    def build() -> Graph:
        b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
        idx, t = b.param("idx"), b.param("target")
        logits = _transformer(b, idx, mask)
        b.ret(b.let("loss", b.call("cross_entropy", logits, t)))
        b.train(objective="loss", lr=0.1, iterations=3)
        return b.build()
    return build


def _train_mlp(act: str) -> Callable[[], Graph]:
    def build() -> Graph:
        b = GraphBuilder(param_dtype=FIXTURE_DTYPE)
        x, t = b.param("x"), b.param("target")
        hidden = b.let("hidden", b.ctor("linear", 3, 4, False))
        out = b.let("out", b.ctor("linear", 4, 3, False))
        if act == "relu":
            h = b.call("relu", b.apply(hidden, x))
        else:
            si = b.ctor("SiLU")
            h = b.apply(si, b.apply(hidden, x))
        logits = b.let("logits", b.apply(out, h))
        b.ret(b.let("loss", b.call("cross_entropy", logits, t)))
        b.train(objective="loss", lr=0.05, iterations=3)
        return b.build()
    return build


_X23 = {"x": [2, 3]}
_XT23 = {"x": [2, 3], "target": [2, 3]}
_IDX = {"idx": [1], "target": [1, 3]}

FIXTURES: Dict[str, Fixture] = {f.name: f for f in [
    Fixture("test_model_matmul_relu.ty", _model_matmul_relu, {"x": [2, 3], "w": [3, 4]}, ["run"]),
    Fixture("test_run_activation_layers.ty", _run_activation_layers, _X23, ["run"]),
    Fixture("test_run_binary_ops.ty", _run_binary_ops, {"x": [2, 3], "y": [2, 3]}, ["run"]),
    Fixture("test_run_cross_entropy.ty", _run_cross_entropy, {"logits": [2, 3], "target": [2, 3]}, ["run"]),
    Fixture("test_run_dropout.ty", _run_dropout, _X23, ["run"]),
    Fixture("test_run_linear_bias.ty", _run_linear_bias, _X23, ["run"]),
    Fixture("test_run_pytorch_transformer_mask.ty", _run_transformer_mask, {"idx": [1]}, ["run"]),
    Fixture("test_run_rms_norm.ty", _run_rms_norm, _X23, ["run"]),
    Fixture("test_run_scale_builtin.ty", _run_scale_builtin, _X23, ["run"]),
    Fixture("test_run_two_layer_mlp.ty", _run_two_layer_mlp, _X23, ["run"]),
    Fixture("test_backward_basic_ops.ty", _backward_basic_ops,
            {"x": [2, 3], "y": [2, 3], "w": [3, 2]}, ["backward"]),
    Fixture("test_backward_cross_entropy.ty", _backward_cross_entropy,
            {"logits": [2, 3], "target": [2, 3]}, ["backward"]),
    Fixture("test_backward_dropout.ty", _backward_dropout, _X23, ["backward"]),
    Fixture("test_backward_linear_bias.ty", _backward_linear(True), _X23, ["backward"]),
    Fixture("test_backward_linear_layer.ty", _backward_linear(False), _X23, ["backward"]),
    Fixture("test_backward_rms_norm.ty", _backward_rms_norm, _X23, ["backward"]),
    Fixture("test_backward_silu_layer.ty", _backward_act("SiLU"), _X23, ["backward"]),
    Fixture("test_backward_softmax_layer.ty", _backward_act("Softmax"), _X23, ["backward"]),
    Fixture("test_train_backend_single.ty", _train_linear_ce(False, 2), _XT23, ["train"]),
    Fixture("test_train_dropout.ty", _train_dropout, _XT23, ["train"]),
    Fixture("test_train_linear_bias.ty", _train_linear_ce(True, 3), _XT23, ["train"]),
    Fixture("test_train_pytorch_transformer.ty", _train_transformer(False), _IDX, ["train"]),
    Fixture("test_train_pytorch_transformer_mask.ty", _train_transformer(True), _IDX, ["train"]),
    Fixture("test_train_small_mlp.ty", _train_mlp("relu"), _XT23, ["train"]),
    Fixture("test_train_silu_mlp.ty", _train_mlp("silu"), _XT23, ["train"]),
]}


# ---- workloads ---------------------------------------------------------------

def matmul_relu() -> Graph:
    """y = relu(x @ w): the test_model_matmul_relu program, run at any --shape."""
    return _model_matmul_relu()


def mlp_train(d_in: int = 1024, d_hidden: int = 4096, d_out: int = 1024, lr: float = 1e-3,
              iterations: int = 100, loss_scale: float = None) -> Graph:
    """Linear(d_in->d_hidden)+bias, ReLU, Linear(d_hidden->d_out)+bias, squared
    error summed over all elements (the reference has no MSE op; the loss is
    `d = y - target; d * d`, summed by the trainer, executor.rs:810).  With
    `loss_scale` = 1 / (elements of the global batch) the squared errors are
    scaled before the trainer sums them, which makes the objective the mean
    squared error."""
    b = GraphBuilder()
    x, t = b.param("x"), b.param("target")
    l1 = b.let("l1", b.ctor("linear", d_in, d_hidden, True))
    l2 = b.let("l2", b.ctor("linear", d_hidden, d_out, True))
    y = b.let("y", b.apply(l2, b.call("relu", b.apply(l1, x))))
    d = b.let("d", b.binary("-", y, t))
    sq = b.binary("*", d, d)
    if loss_scale is not None:
        sq = b.call("scale", sq, float(loss_scale))
    b.ret(b.let("loss", sq))
    b.train(objective="loss", lr=lr, iterations=iterations)
    return b.build()


def llama_block(batch: int = 8, seq: int = 2048, d_model: int = 2048, n_heads: int = 16,
                n_kv_heads: int = 4, hidden: int = 5632, theta: float = 10000.0,
                eps: float = 1e-6, lr: float = 1e-3, mse_target: bool = False) -> Graph:
    """Llama-style decoder block (the structure of examples/llama.ty's
    DecoderBlock with GroupedQueryAttention and SwiGLU), written with the
    batched-matmul / transpose / RMSNorm extensions:

        h   = x + o_proj(attn(RMSNorm(x)))
        out = h + down(SiLU(gate(RMSNorm(h))) * up(RMSNorm(h)))

    x is [batch*seq, d_model].  Attention: q/k/v projections, reshape to
    [B, S, H, hd], transpose to [B, H, S, hd], RoPE on q and k, repeat_kv on
    k and v, scores = q @ k^T scaled by 1/sqrt(hd), causal_mask, Softmax,
    @ v, transpose back and flatten.  The objective is the block output (its
    gradient seed is all ones, as for any objective, executor.rs:579), or with
    `mse_target` the squared error against a `target` input,
    `d = out - target; loss = d * d` (summed by the trainer), which keeps a
    training run bounded."""
    b = GraphBuilder("block")
    x = b.param("x")
    target = b.param("target") if mse_target else None
    out = b.let("out", decoder_block(b, x, batch, seq, d_model, n_heads, n_kv_heads, hidden, theta, eps))
    if target is not None:
        d = b.let("d", b.binary("-", out, target))
        b.ret(b.let("loss", b.binary("*", d, d)))
        b.train(objective="loss", lr=lr, iterations=1)
    else:
        b.ret(out)
        b.train(objective="out", lr=lr, iterations=1)
    return b.build()


def decoder_block(b: GraphBuilder, x, batch: int, seq: int, d_model: int, n_heads: int, n_kv_heads: int,
                  hidden: int, theta: float, eps: float, prefix: str = ""):
    """Appends one decoder block to `b` and returns its output value (see
    llama_block); `prefix` keeps the named values of stacked blocks apart."""
    hd = d_model // n_heads
    rep = n_heads // n_kv_heads
    P = prefix
    n1 = b.let(P + "attn_norm", b.ctor("RMSNorm", d_model, eps))
    qp = b.let(P + "q_proj", b.ctor("linear", d_model, n_heads * hd, False))
    kp = b.let(P + "k_proj", b.ctor("linear", d_model, n_kv_heads * hd, False))
    vp = b.let(P + "v_proj", b.ctor("linear", d_model, n_kv_heads * hd, False))
    op = b.let(P + "o_proj", b.ctor("linear", n_heads * hd, d_model, False))
    n2 = b.let(P + "ffn_norm", b.ctor("RMSNorm", d_model, eps))
    gp = b.let(P + "gate_proj", b.ctor("linear", d_model, hidden, False))
    up = b.let(P + "up_proj", b.ctor("linear", d_model, hidden, False))
    dp = b.let(P + "down_proj", b.ctor("linear", hidden, d_model, False))
    act = b.let(P + "act", b.ctor("SiLU"))
    sm = b.let(P + "softmax", b.ctor("Softmax"))

    hn = b.let(P + "hn", b.apply(n1, x))

    def heads(t, nh):
        t = b.call("reshape", t, batch, seq, nh, hd)
        return b.call("transpose", t, 1, 2)

    q = b.let(P + "q", b.call("rope", heads(b.apply(qp, hn), n_heads), hd, theta))
    k = b.let(P + "k", b.call("rope", heads(b.apply(kp, hn), n_kv_heads), hd, theta))
    v = b.let(P + "v", heads(b.apply(vp, hn), n_kv_heads))
    k = b.let(P + "k", b.call("repeat_kv", k, rep))
    v = b.let(P + "v", b.call("repeat_kv", v, rep))
    kt = b.call("transpose", k, 2, 3)
    scores = b.call("scale", b.call("matmul", q, kt), 1.0 / (hd ** 0.5))
    probs = b.let(P + "probs", b.apply(sm, b.call("causal_mask", scores)))
    ctx = b.call("matmul", probs, v)
    ctx = b.call("reshape", b.call("transpose", ctx, 1, 2), batch * seq, n_heads * hd)
    h = b.let(P + "h", b.binary("+", x, b.apply(op, ctx)))

    hn2 = b.let(P + "hn2", b.apply(n2, h))
    gate = b.apply(act, b.apply(gp, hn2))
    ff = b.binary("*", gate, b.apply(up, hn2))
    return b.binary("+", h, b.apply(dp, ff))


def llama_lm(layers: int = 4, batch: int = 8, seq: int = 2048, d_model: int = 2048, n_heads: int = 16,
             n_kv_heads: int = 4, hidden: int = 5632, vocab: int = 32000, theta: float = 10000.0,
             eps: float = 1e-6, lr: float = 1e-3, iterations: int = 50) -> Graph:
    """Llama-style language model for next-token training:

        x      = Embedding(vocab, d_model)(ids)          ids: [batch*seq] token ids
        x      = decoder_block(x)  (x layers)
        logits = tied_logits(RMSNorm(x), embedding)      [batch*seq, vocab]
        loss   = cross_entropy(logits, labels)           labels: [batch*seq] ids

    The output projection is tied to the embedding table (the `tied_logits`
    extension); `labels` holds the next token of every position, and the
    trainer sums the per-row losses (executor.rs:810)."""
    b = GraphBuilder("lm")
    ids, labels = b.param("ids"), b.param("labels")
    emb = b.let("embed", b.ctor("Embedding", vocab, d_model))
    x = b.let("x0", b.apply(emb, ids))
    for i in range(layers):
        x = b.let(f"x{i + 1}", decoder_block(b, x, batch, seq, d_model, n_heads, n_kv_heads, hidden, theta, eps,
                                             prefix=f"l{i}_"))
    norm = b.let("final_norm", b.ctor("RMSNorm", d_model, eps))
    logits = b.let("logits", b.call("tied_logits", b.apply(norm, x), emb))
    b.ret(b.let("loss", b.call("cross_entropy", logits, labels)))
    b.train(objective="loss", lr=lr, iterations=iterations)
    return b.build()


def llama_lm_flops(layers: int, batch: int, seq: int, d_model: int, n_heads: int, n_kv_heads: int,
                   hidden: int, vocab: int) -> float:
    """Forward + backward FLOPs of one llama_lm step as executed (attention
    over the full materialised score matrix; 3x the forward FLOPs)."""
    t = batch * seq
    head = 2.0 * t * d_model * vocab
    return 3.0 * (layers * llama_block_flops(batch, seq, d_model, n_heads, n_kv_heads, hidden) / 3.0 + head)


def llama_block_flops(batch: int, seq: int, d_model: int, n_heads: int, n_kv_heads: int,
                      hidden: int) -> float:
    """Matmul FLOPs of one forward+backward of `llama_block` (backward = input
    and weight gradients of every projection, both operand gradients of both
    attention matmuls)."""
    t = batch * seq
    hd = d_model // n_heads
    kv = n_kv_heads * hd
    proj = 2 * t * d_model * (d_model + 2 * kv + d_model) + 2 * t * d_model * hidden * 3
    attn = 2 * 2 * batch * n_heads * seq * seq * hd
    return 3.0 * (proj + attn)


def random_parameters(graph: Graph, seed: int = 1234, std: float = 0.02) -> Dict[str, np.ndarray]:
    """Seeded initial values for every trainable parameter a graph's
    constructors create under the train executor's names
    (training/executor.rs:152-221): linear weights [in, out] and embedding
    tables [num, dim] N(0, std), linear biases 0, RMSNorm gains N(1, std).
    Constructors are visited in graph order, so a seed fixes every value."""
    rng = np.random.default_rng(seed)
    consts = {n.output: n.const for n in graph.nodes if n.kind == "const"}
    params: Dict[str, np.ndarray] = {}
    for n in graph.nodes:
        if n.kind != "ctor":
            continue
        if n.op == "linear":
            args = [consts[i] for i in n.inputs]
            if len(args) < 2 or isinstance(args[1], bool):
                raise ValueError("random_parameters needs linear(in, out[, bias]) constructors")
            i, o = int(args[0]), int(args[1])
            params[f"linear_{n.output}_weight"] = (std * rng.standard_normal((i, o))).astype(np.float32)
            if len(args) > 2 and bool(args[2]):
                params[f"linear_{n.output}_bias"] = np.zeros(o, np.float32)
        elif n.op == "Embedding":
            num, dim = int(consts[n.inputs[0]]), int(consts[n.inputs[1]])
            params[f"embedding_{n.output}_weight"] = (std * rng.standard_normal((num, dim))).astype(np.float32)
        elif n.op == "RMSNorm":
            h = int(consts[n.inputs[0]])
            params[f"rmsnorm_{n.output}_gain"] = (1.0 + std * rng.standard_normal(h)).astype(np.float32)
    return params
