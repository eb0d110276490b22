"""The `.ty` front end (tysor_b200/frontend.py) and the CLI's argument
handling, on the CPU.

* Every allowlisted reference fixture lowers to exactly the graph written
  by hand in tysor_b200/programs.py (values with their ids, names and dtype
  strings, nodes, outputs, train settings) -- when a reference checkout is
  available (TYSOR_REFERENCE_DIR or ../reference).
* Programs written here: pipelines, binary operators and constants,
  constructors, config fields, train blocks, keyword arguments (kept in
  their written position, as the reference's builder does), and the errors
  for what the front end does not lower (recursion, unknown names, None
  where a value is needed).
* `python -m tysor_b200` rejects bad command lines with exit code 2 and the
  reference's messages, and reports a program error with exit code 1.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tysor_b200.frontend import TysorSyntaxError, lower  # noqa: E402
from tysor_b200.programs import FIXTURES, mlp_train  # noqa: E402


def signature(g):
    return ([(v.id, v.kind, v.is_parameter, v.name, v.dtype) for v in g.values],
            [(n.kind, n.output, n.op, n.binop if n.kind == "binary" else "", repr(n.const), list(n.inputs))
             for n in g.nodes],
            list(g.outputs), g.objective, g.lr, g.iterations, g.optimizer)


def reference_tests_dir():
    for cand in (os.environ.get("TYSOR_REFERENCE_DIR"), os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "tests")):
            return os.path.join(cand, "tests")
    return None


@pytest.mark.parametrize("name", sorted(FIXTURES))
def test_reference_fixture_lowers_to_the_hand_lowered_graph(name):
    tests = reference_tests_dir()
    if tests is None:
        pytest.skip("no reference checkout here")
    with open(os.path.join(tests, name)) as f:
        got = lower(f.read())
    assert signature(got) == signature(FIXTURES[name].build())


MLP_SRC = """
# the two-layer MLP trainer, squared error summed by the trainer
layer model(x: tensor, target: tensor): tensor:
  l1 = linear(8, 16, true)
  l2 = linear(16, 8, true)
  y = x -> l1() -> relu() -> l2()
  d = y - target
  loss = d * d
  return loss

train model:
  optimizer = "sgd"
  lr = 0.001
  iteration = 4
  objective = loss
"""


def test_a_program_lowers_like_the_builder():
    """The MLP above is mlp_train(8, 16, 8) written in the DSL: same graph."""
    got = lower(MLP_SRC)
    want = mlp_train(8, 16, 8, lr=0.001, iterations=4)
    assert signature(got) == signature(want)


def test_config_fields_constants_and_constructor_stages():
    src = """
config dims:
  hidden : int = 6
  p      : float = 0.5

layer model(x: tensor[float16]): tensor[float16]:
  proj = linear(dims.hidden, 4)
  y = x -> proj() -> SiLU() -> Dropout(dims.p)
  return 2.0 * y - 1.0
"""
    g = lower(src)
    kinds = [(n.kind, n.binop if n.kind == "binary" else n.op, n.const) for n in g.nodes]
    # constants in argument order, the constructor stage before its input
    assert kinds[:3] == [("const", "", 6), ("const", "", 4), ("ctor", "linear", None)]
    assert [k for k in kinds if k[0] == "ctor"] == [("ctor", "linear", None), ("ctor", "Dropout", None),
                                                    ("ctor", "SiLU", None)]
    assert g.values[0].dtype == "float16"
    assert g.value_dtypes()[g.outputs[0]] == "float16"


@pytest.mark.parametrize("src,msg", [
    ("layer helper(x: tensor): tensor:\n  return helper(x)\n\n"
     "layer model(x: tensor): tensor:\n  return helper(x)\n", "recursive call"),
    ("layer model(x: tensor): tensor:\n  return x if x2 else x\n", "must be known while lowering"),
    ("layer model(x: tensor): tensor:\n  y = None\n  return x + y\n", "'y' is None here"),
    ("layer model(x: tensor): tensor:\n  return x + None\n", "None is not a graph value"),
    ("config a:\n  n : int = 1\nconfig b:\n  n : int = 2\n\n"
     "layer model(x: tensor): tensor:\n  return scale(x, config.n)\n", "exactly one config block"),
    ("layer model(x: tensor): tensor:\n  return relu(z)\n", "unknown name"),
    ("layer model(x: tensor): tensor:\n  y = x\n", "no return"),
    ("layer other(x: tensor): tensor:\n  return x\n", "Entry function 'model' not found"),
    ("layer model(x: tensor): tensor:\n  return x & 2\n", "unexpected character"),
    ("layer model(x: tensor): tensor:\n  return x ! 2\n", "expected 'nl', got '!'"),
    ("layer model(x: tensor): tensor:\n  return !x\n", "not a graph value"),
    ("layer model(x: tensor): tensor:\n  return relu(x > 1)\n", "not a graph value"),
])
def test_what_the_front_end_does_not_lower_is_an_error(src, msg):
    with pytest.raises(TysorSyntaxError, match=msg):
        lower(src)


def run_cli(*args):
    return subprocess.run([sys.executable, "-m", "tysor_b200", *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=120)


def test_cli_rejects_bad_command_lines(tmp_path):
    prog = tmp_path / "m.ty"
    prog.write_text(MLP_SRC)
    for args, msg in [((), "missing input path"),
                      ((str(prog), "--bogus"), "unknown option: --bogus"),
                      ((str(prog), "--shape", "x=2y3"), "invalid dimension '2y3' in shape 'x=2y3'"),
                      ((str(prog), "--backend", "local"), "backend 'local' is not part of this build"),
                      ((str(prog), "--backend", "tpu"), "unsupported backend 'tpu'"),
                      ((str(prog), "--ir", "--run"), "option --ir belongs to the reference compiler")]:
        res = run_cli(*args)
        assert res.returncode == 2, (args, res.stderr)
        assert msg in res.stderr and "usage:" in res.stderr, (args, res.stderr)


def test_cli_reports_a_bad_program(tmp_path):
    prog = tmp_path / "bad.ty"
    prog.write_text("layer model(x: tensor): tensor:\n  return relu(z)\n")
    res = run_cli(str(prog), "--run", "--shape", "x=2x3")
    assert res.returncode == 1 and "unknown name" in res.stderr


def test_keyword_arguments_keep_their_position():
    """The reference's builder lowers a call's arguments in written order and
    drops their names (ir/builder.rs:119-123)."""
    named = lower("layer model(x: tensor): tensor:\n  return repeat_kv(x, times: 2)\n")
    plain = lower("layer model(x: tensor): tensor:\n  return repeat_kv(x, 2)\n")
    assert signature(named) == signature(plain)
