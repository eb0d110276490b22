"""The oracle against the reference's own PyTorch helper functions
(tests/golden/torch_helper_golden.json, made by tests/golden/make_golden.py)
and against hand-computed known answers."""
import json
import math
import os

import numpy as np
import pytest

import local as L

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "torch_helper_golden.json")
with open(GOLDEN) as f:
    CASES = json.load(f)["cases"]


def _t(d):
    return L.Tensor(list(d["shape"]), np.asarray(d["data"], dtype=np.float32))


def _run(case):
    op, ins, args = case["op"], {k: _t(v) for k, v in case["inputs"].items()}, case["args"]
    if op == "linear_weight":
        return L.linear_weight(args["in"], args["out"])
    if op == "linear_bias":
        return L.linear_bias(args["out"])
    if op == "embedding_weight":
        return L.embedding_weight(args["num"], args["dim"])
    if op == "silu":
        return L.silu(ins["x"])
    if op == "softmax":
        return L.softmax(ins["x"])
    if op == "rms_norm":
        return L.rms_norm(ins["x"], args["hidden"])
    if op == "dropout":
        return L.dropout(ins["x"], args["p"])
    if op == "cross_entropy":
        return L.cross_entropy(ins["logits"], ins["target"])
    if op == "linear":
        return L.linear_with_parameters(ins["x"], ins["w"], ins.get("b"))
    if op == "rope":
        return L.rope(ins["x"], args["head_dim"], args["theta"])
    if op == "causal_mask":
        return L.causal_mask(ins["x"])
    if op == "flatten_heads":
        return L.flatten_heads(ins["x"])
    if op == "repeat_kv":
        return L.repeat_kv(ins["x"], args["repeats"])
    if op == "embedding":
        w = ins["weight"]
        return L.embedding(ins["idx"], w, w.shape[0], w.shape[1])
    raise AssertionError(op)


# Copies, gathers, masks and pattern initialisers must match bit for bit;
# reductions and transcendentals differ only in summation order / libm.
EXACT = {"linear_weight", "linear_bias", "embedding_weight", "causal_mask", "flatten_heads",
         "repeat_kv", "embedding", "dropout"}


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_torch_helpers(case):
    got = _run(case)
    want = np.asarray(case["out"]["data"], dtype=np.float32)
    assert list(got.shape) == list(case["out"]["shape"])
    if case["op"] in EXACT:
        np.testing.assert_array_equal(got.data, want)
    else:
        err = np.linalg.norm(got.data.astype(np.float64) - want) / max(np.linalg.norm(want), 1e-30)
        assert err < 1e-6, err


def test_rms_norm_known_answer():
    # test_run_rms_norm.ty with x=2x3: row 0 = [0.125, 0.25, 0.375]
    x = L.synthetic([2, 3])
    y = L.rms_norm(x, 3)
    ms = (0.125 ** 2 + 0.25 ** 2 + 0.375 ** 2) / 3
    s = 1 / math.sqrt(ms + 1e-5)
    np.testing.assert_allclose(y.data[:3], [0.125 * s, 0.25 * s, 0.375 * s], rtol=1e-6)


def test_matmul_known_answer():
    # test_model_matmul_relu.ty with x=2x3, w=3x4: exact small dyadic rationals.
    x = L.synthetic([2, 3])
    w = L.synthetic([3, 4])
    y = L.matmul(x, w)
    xe = np.array([(i % 17 + 1) / 8 for i in range(6)]).reshape(2, 3)
    we = np.array([(i % 17 + 1) / 8 for i in range(12)]).reshape(3, 4)
    np.testing.assert_array_equal(y.data, (xe @ we).reshape(-1).astype(np.float32))


def test_matmul_sequential_order_bit_exact():
    # The oracle must equal a literal i-j-k loop (tensor.rs:179-188), bit for bit.
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (7, 33)).astype(np.float32)
    b = rng.uniform(-1, 1, (33, 5)).astype(np.float32)
    ref = np.zeros((7, 5), dtype=np.float32)
    for i in range(7):
        for j in range(5):
            acc = np.float32(0)
            for k in range(33):
                acc = np.float32(acc + np.float32(a[i, k] * b[k, j]))
            ref[i, j] = acc
    got = L.matmul(L.Tensor([7, 33], a.reshape(-1).copy()), L.Tensor([33, 5], b.reshape(-1).copy()))
    np.testing.assert_array_equal(got.data, ref.reshape(-1))


def test_sgd_and_sum_bit_exact():
    rng = np.random.default_rng(1)
    p = rng.standard_normal(1000).astype(np.float32)
    g = rng.standard_normal(1000).astype(np.float32)
    want = (p - np.float32(0.05) * g).astype(np.float32)
    pt = L.Tensor([1000], p.copy())
    L.sgd(pt, L.Tensor([1000], g), 0.05)
    np.testing.assert_array_equal(pt.data, want)
    acc = np.float32(0)
    for v in p:
        acc = np.float32(acc + v)
    assert L.tensor_sum(L.Tensor([1000], p)) == acc


def test_embedding_out_of_range_is_an_error():
    w = L.embedding_weight(4, 2)
    with pytest.raises(L.OracleError):
        L.embedding(L.Tensor([1], np.array([4.0], np.float32)), w, 4, 2)
    with pytest.raises(L.OracleError):
        L.embedding(L.Tensor([1], np.array([-1.0], np.float32)), w, 4, 2)


def test_embedding_backward_skips_out_of_range():
    g = L.Tensor([3, 2], np.arange(6, dtype=np.float32))
    idx = L.Tensor([3], np.array([1.0, 9.0, 1.0], np.float32))
    wg = L.embedding_backward(g, idx, 4, 2)
    np.testing.assert_array_equal(wg.data, [0, 0, 0 + 4, 1 + 5, 0, 0, 0, 0])
