"""`python -m tysor_b200 <file.ty> --run/--backward/--train --backend cuda`:
programs written in the DSL, read by the front end, run on the device, and
printed as the reference prints them; the printed numbers (4 decimals for
tensors, 6 for losses) are compared with the oracle's values for the same
lowered graph, and the dtype strings with the annotations' propagation."""
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import local as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
from tysor_b200.frontend import lower  # noqa: E402

pytestmark = pytest.mark.gpu

MLP = """
layer model(x: tensor[float16], target: tensor[float16]): tensor[float16]:
  l1 = linear(8, 16, true)
  l2 = linear(16, 8, false)
  y = x -> l1() -> SiLU() -> l2()
  d = y - target
  loss = d * d
  return loss

train model:
  optimizer = "sgd"
  lr = 0.0001
  iteration = 5
  objective = loss
"""

ATTN = """
layer model(idx: tensor[float16]): tensor[float16]:
  tok = Embedding(32, 8)
  out_proj = linear(16, 3, false)
  x = tok(idx)
  x = rms_norm(x, 8)
  x = reshape(x, 1, 2, 4)
  x = rope(x, 4, 10000.0)
  x = repeat_kv(x, 2)
  x = causal_mask(x)
  x = flatten_heads(x)
  return x -> out_proj()
"""

TENSOR = re.compile(r"(?:(\w+):\n)?shape=\[([^\]]*)\] dtype=(\S+)\nvalues=\[([^\]]*)\]")


def cli(tmp_path, src, *args):
    prog = tmp_path / "prog.ty"
    prog.write_text(src)
    res = subprocess.run([sys.executable, "-m", "tysor_b200", str(prog), "--backend", "cuda", *args], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    return res.stdout


def tensors(text):
    out = []
    for name, shape, dtype, vals in TENSOR.findall(text):
        out.append((name, [int(s) for s in shape.split(",") if s.strip()], dtype,
                    np.array([float(v) for v in vals.split(",") if v.strip()])))
    return out


def test_run_prints_the_reference_section(tmp_path):
    text = cli(tmp_path, ATTN, "--run", "--shape", "idx=1")
    assert "--- Execution Output ---" in text
    [(_, shape, dtype, vals)] = tensors(text)
    want, _ = L.run_forward(lower(ATTN), {"idx": [1]})
    assert shape == want.shape and dtype == want.dtype == "float32"  # an Embedding's output
    np.testing.assert_allclose(vals, want.data, atol=1.5e-4)


def test_backward_prints_every_parameter_gradient(tmp_path):
    text = cli(tmp_path, MLP, "--backward", "--shape", "x=4x8", "--shape", "target=4x8")
    assert "--- Gradient Output ---" in text
    got = tensors(text)
    want = L.backward_report(lower(MLP), {"x": [4, 8], "target": [4, 8]})
    assert [g[0] for g in got] == [n for n, _ in want] == ["x_grad", "target_grad"]
    for (name, shape, dtype, vals), (_, w) in zip(got, want):
        assert shape == w.shape and dtype == w.dtype == "float16", name
        np.testing.assert_allclose(vals, w.data, atol=1.5e-4, rtol=1e-4, err_msg=name)


def test_train_prints_the_loss_of_every_step(tmp_path):
    text = cli(tmp_path, MLP, "--train", "--shape", "x=4x8", "--shape", "target=4x8")
    assert "--- Training Output ---" in text and "backend=cuda" in text
    steps = re.findall(r"step=(\d+) loss=([-0-9.e+]+) params=(\d+)", text)
    want, params = L.train(lower(MLP), {"x": [4, 8], "target": [4, 8]})
    assert [int(s) for s, _, _ in steps] == [1, 2, 3, 4, 5]
    assert all(int(p) == len(params) == 3 for _, _, p in steps)
    got = np.array([float(v) for _, v, _ in steps])
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6)
    assert got[-1] < got[0]


def test_llama_style_program_trains_on_the_device(tmp_path):
    """The Llama decoder block written with user layers, a derived head_dim,
    the three-argument scale and an optional target (the front end's
    extensions), trained through the CLI; the optional target is an input
    only when it gets a --shape."""
    from test_frontend_ext import LLAMA_STYLE
    shapes = {"x": [128, 256], "target": [128, 256]}
    text = cli(tmp_path, LLAMA_STYLE, "--train", "--shape", "x=128x256", "--shape", "target=128x256")
    steps = re.findall(r"step=(\d+) loss=([-0-9.e+]+) params=(\d+)", text)
    want, params = L.train(lower(LLAMA_STYLE, inputs=list(shapes)), shapes)
    assert len(steps) == 1 and int(steps[0][2]) == len(params) == 9
    np.testing.assert_allclose(float(steps[0][1]), want[0], rtol=1e-4)
    text = cli(tmp_path, LLAMA_STYLE, "--run", "--shape", "x=128x256")
    [(_, shape, _, _)] = tensors(text)
    assert shape == [128, 256]
