"""Front-end extensions for `examples/llama.ty`-style programs
(tysor_b200/frontend.py): user-layer inlining, `scale(x, d, h)`,
`config.head_dim`, conditional expressions and optional inputs, tuple
returns, integer folding of compile-time arithmetic in arguments.

The end-to-end checks take the programs in examples/ -- the Llama decoder
block written with these extensions (user layers, a derived head_dim, the
three-argument scale, an optional target) and a 2-layer LM with
`DecoderBlock()[n_layers]` -- and run them through the oracle next to the
hand-lowered `programs.llama_block` / `programs.llama_lm`: with parameters
drawn in constructor order, the output and every gradient are bit-identical
(the same operations on the same values)."""
import os
import sys

import numpy as np
import pytest

import local as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tysor_b200.frontend import TysorSyntaxError, lower  # noqa: E402
from tysor_b200.programs import llama_block, random_parameters  # noqa: E402


def structure(g):
    """Nodes without value names: (kind, op / binop, constant, inputs)."""
    return [(n.kind, n.binop if n.kind == "binary" else n.op, repr(n.const), list(n.inputs)) for n in g.nodes]


def test_inlined_layer_equals_the_written_out_body():
    inlined = """
layer Norm(t: tensor, width: int): tensor:
  n = RMSNorm(width, 0.00001)
  return n(t)

layer model(x: tensor): tensor:
  proj = linear(8, 8, false)
  return x -> Norm(8) -> proj()
"""
    flat = """
layer model(x: tensor): tensor:
  proj = linear(8, 8, false)
  n = RMSNorm(8, 0.00001)
  return proj(n(x))
"""
    a, b = lower(inlined), lower(flat)
    # The stage order puts the projection's constructor first in both.
    assert structure(a) == structure(b)
    assert a.outputs == b.outputs


def test_each_call_makes_its_own_parameters():
    src = """
layer Proj(t: tensor): tensor:
  p = linear(4, 4, true)
  return p(t)

layer model(x: tensor): tensor:
  return x -> Proj() -> relu() -> Proj()
"""
    g = lower(src)
    ctors = [n for n in g.nodes if n.kind == "ctor"]
    assert [c.op for c in ctors] == ["linear", "linear"]
    names = set(random_parameters(g, 1))
    assert len(names) == 4  # two weights, two biases


def test_scale_of_a_width_over_heads():
    src = """
config c:
  hidden_dim : int = 2048
  n_heads    : int = 16

layer model(x: tensor): tensor:
  return x -> scale(c.hidden_dim, c.n_heads)
"""
    g = lower(src)
    consts = [n.const for n in g.nodes if n.kind == "const"]
    assert consts == [1.0 / (128.0 ** 0.5)]
    assert [n.op for n in g.nodes if n.kind in ("primitive", "call")] == ["scale"]


def test_config_head_dim_is_derived_unless_declared():
    base = """
config llama_config:
  hidden_dim : int = 512
  n_heads    : int = 8{extra}

layer model(x: tensor): tensor:
  return reshape(x, 2, config.head_dim)
"""
    g = lower(base.format(extra=""))
    assert [n.const for n in g.nodes if n.kind == "const"] == [2, 64]
    g = lower(base.format(extra="\n  head_dim   : int = 32"))
    assert [n.const for n in g.nodes if n.kind == "const"] == [2, 32]
    with pytest.raises(TysorSyntaxError, match="not a multiple"):
        lower(base.replace("n_heads    : int = 8", "n_heads    : int = 7").format(extra=""))


def test_conditionals_optional_inputs_and_tuple_returns():
    src = """
config c:
  use_relu : bool = true
  depth    : int = 3

layer model(x: tensor, target=None): (tensor, tensor):
  y = relu(x) if c.use_relu else x
  z = scale(y, 2.0) if c.depth > 2 else y
  loss = z - target if target else None
  return z, loss
"""
    full = lower(src)
    assert [v.name for v in full.values if v.is_parameter] == ["x", "target"]
    assert len(full.outputs) == 2
    assert [n.op for n in full.nodes if n.kind in ("primitive", "call")] == ["relu", "scale"]
    bare = lower(src, inputs=["x"])
    assert [v.name for v in bare.values if v.is_parameter] == ["x"]
    assert len(bare.outputs) == 1 and not any(n.kind == "binary" for n in bare.nodes)


def test_integer_arithmetic_in_arguments_folds():
    src = """
config c:
  n_heads    : int = 16
  n_kv_heads : int = 4

layer model(x: tensor): tensor:
  return repeat_kv(x, c.n_heads / c.n_kv_heads)
"""
    g = lower(src)
    assert [n.const for n in g.nodes if n.kind == "const"] == [4]
    assert not any(n.kind == "binary" for n in g.nodes)


EXAMPLES = os.path.join(ROOT, "examples")
with open(os.path.join(EXAMPLES, "llama_block.ty")) as _f:
    LLAMA_STYLE = _f.read()

CFG = dict(batch=2, seq=64, d_model=256, n_heads=4, n_kv_heads=2, hidden=384, eps=1e-6, lr=1e-4)


def by_ctor_order(g, params):
    """Parameter arrays in constructor order (names carry graph ids)."""
    order = []
    for n in g.nodes:
        if n.kind == "ctor":
            order += sorted(k for k in params if k.split("_")[1] == str(n.output))
    return [params[k] for k in order], order


@pytest.mark.parametrize("with_target", [True, False])
def test_llama_style_program_matches_the_hand_lowered_block(with_target):
    t = CFG["batch"] * CFG["seq"]
    g = lower(LLAMA_STYLE, inputs=["x", "target"] if with_target else ["x"])
    want = llama_block(**CFG, mse_target=with_target)
    shapes = {"x": [t, CFG["d_model"]]}
    rng = np.random.default_rng(3)
    ins = {"x": rng.standard_normal(t * CFG["d_model"]).astype(np.float32)}
    if with_target:
        shapes["target"] = [t, CFG["d_model"]]
        ins["target"] = rng.standard_normal(t * CFG["d_model"]).astype(np.float32)
    pg, pw = random_parameters(g, 9), random_parameters(want, 9)
    arrays_g, names_g = by_ctor_order(g, pg)
    arrays_w, names_w = by_ctor_order(want, pw)
    assert [a.shape for a in arrays_g] == [a.shape for a in arrays_w]

    def run(graph, params):
        ps = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
        values, grads, _ = L.train_step_grads(graph, shapes, inputs=ins, parameters=ps)
        return values[graph.objective_id()][1].data, grads

    out_g, grads_g = run(g, pg)
    out_w, grads_w = run(want, pw)
    np.testing.assert_array_equal(out_g, out_w)
    for ng, nw in zip(names_g, names_w):
        np.testing.assert_array_equal(grads_g[ng].data, grads_w[nw].data, err_msg=nw)


def test_repeated_stages_and_binary_stages():
    """`f()[n]` applies a stage n times (a local layer instance keeps its
    parameters, a constructor or user layer makes new ones each time), and a
    stage that is an expression applies its calls to the piped value
    (frontend_ir.rs:730-786)."""
    src = """
layer Proj(t: tensor): tensor:
  p = linear(8, 8, false)
  return p(t)

layer shared(x: tensor): tensor:
  p = linear(8, 8, false)
  return x -> p()[3]

layer fresh(x: tensor): tensor:
  return x -> Proj()[3] -> relu()[2] * 2.0

layer model(x: tensor): tensor:
  return x -> relu() - 1.0
"""
    g = lower(src, "shared")
    assert [n.kind for n in g.nodes].count("ctor") == 1 and [n.kind for n in g.nodes].count("apply") == 3
    g = lower(src, "fresh")
    kinds = [(n.kind, n.op or n.binop) for n in g.nodes]
    assert [k for k in kinds if k[0] == "ctor"] == [("ctor", "linear")] * 3
    assert [k for k in kinds if k[0] == "primitive"] == [("primitive", "relu")] * 2 and kinds[-1] == ("binary", "*")
    g = lower(src)
    assert [(n.kind, n.op or n.binop) for n in g.nodes][-1] == ("binary", "-")
    with pytest.raises(TysorSyntaxError, match="non-negative integer"):
        lower("layer model(x: tensor): tensor:\n  return x -> relu()[1.5]\n")


def test_reference_repetition_fixture_lowers():
    """The reference's own repetition fixture (tests/test_arrow_constructor_repeat.ty), each layer."""
    here = os.path.dirname(os.path.abspath(__file__))
    for cand in (os.environ.get("TYSOR_REFERENCE_DIR"), os.path.join(os.path.dirname(here), "..", "reference")):
        path = cand and os.path.join(cand, "tests", "test_arrow_constructor_repeat.ty")
        if path and os.path.isfile(path):
            break
    else:
        pytest.skip("no reference checkout here")
    src = open(path).read()
    kinds = lambda g: [(n.kind, n.op or n.binop) for n in g.nodes if n.kind != "const"]  # noqa: E731
    assert kinds(lower(src, "ProjectDirect")) == [("ctor", "linear"), ("apply", "+")]
    assert kinds(lower(src, "RepeatRelu")) == [("primitive", "relu"), ("primitive", "relu"), ("binary", "*")]
    assert kinds(lower(src, "RepeatLocal")) == [("ctor", "linear"), ("apply", "+"), ("apply", "+")]


with open(os.path.join(EXAMPLES, "llama_lm.ty")) as _f:
    LM_STYLE = _f.read()


def test_repeated_user_layer_lm_matches_the_hand_lowered_lm():
    """`DecoderBlock()[n_layers]` (llama.ty's repetition) with the tied head
    lowers to the computation of `programs.llama_lm`: loss and every
    gradient bit-identical in the oracle."""
    from tysor_b200.programs import llama_lm
    g = lower(LM_STYLE)
    want = llama_lm(layers=2, batch=2, seq=64, d_model=256, n_heads=4, n_kv_heads=2, hidden=384, vocab=512,
                    eps=1e-6)
    t = 128
    seqs = np.random.default_rng(5).integers(0, 512, (2, 65))
    ins = {"ids": seqs[:, :-1].astype(np.float32).reshape(-1), "labels": seqs[:, 1:].astype(np.float32).reshape(-1)}
    shapes = {"ids": [t], "labels": [t]}
    pg, pw = random_parameters(g, 4), random_parameters(want, 4)
    arrays_g, names_g = by_ctor_order(g, pg)
    arrays_w, names_w = by_ctor_order(want, pw)
    assert [a.shape for a in arrays_g] == [a.shape for a in arrays_w] and len(names_g) == 20

    def run(graph, params):
        ps = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
        values, grads, _ = L.train_step_grads(graph, shapes, inputs=ins, parameters=ps)
        return values[graph.outputs[0]][1].data, grads

    out_g, grads_g = run(g, pg)
    out_w, grads_w = run(want, pw)
    np.testing.assert_array_equal(out_g, out_w)
    for ng, nw in zip(names_g, names_w):
        np.testing.assert_array_equal(grads_g[ng].data, grads_w[nw].data, err_msg=nw)


def test_pipeline_continuation_lines():
    """A line starting with `->` continues the pipeline above it (the layout
    of examples/llama.ty's attention)."""
    one = "layer model(x: tensor): tensor:\n  y = x -> relu() -> scale(2.0) -> relu()\n  return y\n"
    split = ("layer model(x: tensor): tensor:\n  y = x -> relu()\n        -> scale(2.0)\n"
             "        -> relu()\n  return y\n")
    assert structure(lower(one)) == structure(lower(split))


def test_reference_llama_example_lowers():
    """The reference's examples/llama.ty lowers: its 32 DecoderBlocks inlined
    (`DecoderBlock()[n_layers]`), its own RMSNorm layer shadowing the library
    constructor, `config.head_dim`, the three-argument `scale`, `reshape(heads:
    n)` with the name dropped, and `loss` present only when `targets` is an
    input.  (Running it is another matter: its `q * k` is an elementwise
    product under the reference's `*`.)"""
    import collections
    here = os.path.dirname(os.path.abspath(__file__))
    for cand in (os.environ.get("TYSOR_REFERENCE_DIR"), os.path.join(os.path.dirname(here), "..", "reference")):
        path = cand and os.path.join(cand, "examples", "llama.ty")
        if path and os.path.isfile(path):
            break
    else:
        pytest.skip("no reference checkout here")
    src = open(path).read()
    full = lower(src, inputs=["idx", "targets"])
    ctors = collections.Counter(n.op for n in full.nodes if n.kind == "ctor")
    calls = collections.Counter(n.op for n in full.nodes if n.kind == "call")
    assert ctors == {"linear": 32 * 7 + 1, "Dropout": 33, "Embedding": 1, "Softmax": 32, "SiLU": 32}
    assert calls["rms_norm"] == 65 and calls["causal_mask"] == 32 and calls["cross_entropy"] == 1
    assert len(full.outputs) == 2
    logits_only = lower(src, inputs=["idx"])
    assert len(logits_only.outputs) == 1 and "cross_entropy" not in {n.op for n in logits_only.nodes}


def test_unary_minus_is_zero_minus_its_operand():
    """`-e` lowers as the binary `0 - e` (the reference's unary minus,
    compiler/frontend_ir.rs:606-615); a negative number stays a literal, and
    the oracle runs the result."""
    neg = "layer model(x: tensor, w: tensor): tensor:\n  return -(x + w) * -w\n"
    sub = "layer model(x: tensor, w: tensor): tensor:\n  return (0 - (x + w)) * (0 - w)\n"
    assert structure(lower(neg)) == structure(lower(sub))
    lit = lower("layer model(x: tensor): tensor:\n  return scale(x, -0.5)\n")
    assert [n.kind for n in lit.nodes] == ["const", "primitive"] and lit.nodes[0].const == -0.5
    twice = lower("layer model(x: tensor): tensor:\n  return --x\n")
    assert [n.binop for n in twice.nodes if n.kind == "binary"] == ["-", "-"]
    out, _ = L.run_forward(lower(neg), {"x": [2, 3], "w": [2, 3]})
    x = L.synthetic([2, 3]).data
    np.testing.assert_array_equal(out.data, -(x + x) * -x)


def test_logical_conditions():
    """Conditions take `!`, `&&` and `||` over compile-time values and input
    names, with the reference's precedence (`||` below `&&` below the
    comparisons, `!` binding tightest: compiler/parser.rs:351-361, 402-409)
    and its constant rules (frontend_ir.rs:1286-1300)."""
    src = """
config c:
  use_relu : bool = true
  depth    : int = 3

layer model(x: tensor, target=None): (tensor, tensor):
  y = relu(x) if !c.use_relu || c.depth > 2 && c.depth < 4 else x
  z = scale(y, 2.0) if !(c.depth == 3) else y
  loss = z - target if target && c.use_relu else None
  flat = z if !target else relu(z)
  return flat, loss
"""
    full = lower(src)
    assert [n.op for n in full.nodes if n.kind in ("primitive", "call")] == ["relu", "relu"]
    assert len(full.outputs) == 2 and any(n.kind == "binary" for n in full.nodes)
    bare = lower(src, inputs=["x"])
    assert [n.op for n in bare.nodes if n.kind in ("primitive", "call")] == ["relu"]
    assert len(bare.outputs) == 1 and not any(n.kind == "binary" for n in bare.nodes)
    with pytest.raises(TysorSyntaxError, match="must be known while lowering"):
        lower("layer model(x: tensor): tensor:\n  return x if x > 1 && true else x\n")


def test_type_annotations_with_dims_and_typed_assignments():
    """`tensor[dtype, dims...]` keeps its dtype whatever the dims hold
    (brackets included), and `name : type = value` assigns the value."""
    annotated = lower("layer model(x: tensor[float16, Dims[:2]], w: tensor[float16]): tensor[float16, Dims[:2]]:\n"
                      "  k : int32 = 2\n  y : tensor[float16, Dims[:2]] = scale(x, k)\n  return y + w\n")
    plain = lower("layer model(x: tensor[float16], w: tensor[float16]): tensor[float16]:\n"
                  "  k = 2\n  y = scale(x, k)\n  return y + w\n")
    assert structure(annotated) == structure(plain)
    assert [(v.name, v.dtype) for v in annotated.values if v.is_parameter] == [("x", "float16"), ("w", "float16")]
    with pytest.raises(TysorSyntaxError, match="unclosed"):
        lower("layer model(x: tensor[float16, Dims[:2]): tensor:\n  return x\n")


def test_train_block_variants_and_field_rules():
    """Tuple-valued train fields make one run per element with scalars
    broadcast; the executor trains the first run (training/executor.rs:132-138).
    A bare name is its own value (`optimizer = sgd`), `learning_rate` is `lr`,
    and the reference's declaration checks hold (semantic_analyzer.rs:808-850)."""
    base = "layer model(x: tensor): tensor:\n  return relu(x)\n\ntrain model:\n"
    g = lower(base + "  optimizer = (sgd, adam)\n  lr = (1e-4, 5e-4)\n  objective = x\n  iteration = 5\n")
    assert (g.optimizer, g.lr, g.iterations, g.objective) == ("sgd", 1e-4, 5, "x")
    g = lower(base + "  optimizer = sgd\n  learning_rate = 2\n  iteration = 3\n  objective = x\n"
                     "  scheduler = cosine(warmup: 100)\n")
    assert (g.optimizer, g.lr, g.iterations) == ("sgd", 2.0, 3)
    g = lower(base + "  lr = 1e-3, 2e-3\n  iteration = 2.0\n")
    assert (g.optimizer, g.lr, g.iterations) == ("sgd", 1e-3, 1)  # a float iteration count is not an int
    for body, msg in [("  lr = 1e-4, 5e-4, 1e-3\n  iteration = (2, 3)\n", "must have the same length"),
                      ("  lr = ()\n", "cannot use an empty tuple"),
                      ("  subtrain = 1\n", "'subtrain' is no longer supported"),
                      ("  lr = 1\n  lr = 2\n", "Duplicate field 'lr'"),
                      ("  epochs = (1, 2)\n", "'epochs' does not support tuple variants")]:
        with pytest.raises(TysorSyntaxError, match=msg):
            lower(base + body)


def test_train_objective_must_name_a_model_symbol():
    """The objective is a bare name among `layer model`'s parameters,
    assigned names and mentioned names (semantic_analyzer.rs:850-893)."""
    model = "layer model(x: tensor, t: tensor): tensor:\n  y = relu(x)\n  loss = cross_entropy(y, t)\n  return loss\n"
    assert lower(model + "\ntrain model:\n  objective = loss\n").objective == "loss"
    assert lower(model + "\ntrain model:\n  objective = (loss, y)\n").objective == "loss"
    for obj, msg in [('"loss"', "must reference a named tensor root"), ("relu(x)", "must reference a named"),
                     ("missing", "unknown model root 'missing'")]:
        with pytest.raises(TysorSyntaxError, match=msg):
            lower(model + f"\ntrain model:\n  objective = {obj}\n")


def test_train_run_needs_layer_model_and_train_model():
    """A train run exists only for `layer model` with a `train model:` block
    (frontend_ir.rs:458-465); --train without one is an error
    (training/executor.rs:132-138)."""
    layer = "layer model(x: tensor): tensor:\n  return relu(x)\n"
    block = "\ntrain model:\n  lr = 0.5\n  iteration = 2\n"
    assert lower(layer + block).train_run and lower(layer + block).lr == 0.5
    assert not lower(layer).train_run
    other = "layer other(x: tensor): tensor:\n  return relu(x)\n\ntrain other:\n  lr = 0.5\n"
    assert not lower(other, entry="other").train_run
    as_fn = "fn model(x: tensor): tensor:\n  return relu(x)\n" + block
    assert not lower(as_fn).train_run
    for name in ("llama_block.ty", "llama_lm.ty"):  # their usage lines run --train
        with open(os.path.join(ROOT, "examples", name)) as fh:
            assert lower(fh.read()).train_run, name
