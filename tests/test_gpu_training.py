"""Training on the device tracks the oracle (the reference's local trainer,
executor.rs:764-816) step by step: every loss of a 100-step run within rel
1e-4 (the tracking bar for training), and the final parameters close to the
oracle's f64 twin."""
import numpy as np
import pytest

import local as L
from tysor_b200.programs import llama_lm, mlp_train, random_parameters

pytestmark = pytest.mark.gpu


def frob(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_oracle(params, dt=np.float32):
    return {k: L.Tensor(list(v.shape), np.asarray(v, dt).reshape(-1).copy()) for k, v in params.items()}


def rel_errors(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return np.abs(got - want) / np.abs(want)


def test_mlp_100_steps_track_the_oracle(cuda_ctx):
    """The two-layer MLP configuration at a reduced size: x, target
    [256, 64] N(0,1), 64 -> 256 -> 64 with bias and ReLU, mean squared
    error, SGD lr 0.05 (lr 1e-3 on this mean barely moves it in 100 steps),
    100 steps."""
    from tysor_b200.runtime import CudaGraphExecutor
    rows, d_in, d_h = 256, 64, 256
    g = mlp_train(d_in, d_h, d_in, lr=0.05, iterations=100, loss_scale=1.0 / (rows * d_in))
    rng = np.random.default_rng(0)
    ins = {"x": rng.standard_normal((rows, d_in), dtype=np.float32),
           "target": rng.standard_normal((rows, d_in), dtype=np.float32)}
    shapes = {"x": [rows, d_in], "target": [rows, d_in]}
    params = random_parameters(g, seed=1, std=0.1)
    L.set_threads(16)
    want, wparams = L.train(g, shapes, inputs=ins, parameters=to_oracle(params))
    with L.precision(64):
        _, wparams64 = L.train(g, shapes, inputs={k: v.astype(np.float64) for k, v in ins.items()},
                               parameters=to_oracle(params, np.float64))
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    got = ex.train()
    assert len(got) == 100
    rel = rel_errors(got, want)
    assert rel.max() <= 1e-4, (rel.max(), int(rel.argmax()))
    assert want[-1] < want[0]
    # Final parameters against the oracle's f64 twin: within 1e-5, or no
    # further from it than the f32 oracle.  The biases start at zero, so
    # they are sums of 100 cancelling bias gradients: the gradient bar of
    # the default accumulation chunk (3e-5) applies to them.
    for name, t in wparams.items():
        got_p = ex.parameter(name)
        err_dev, err_ref = frob(got_p, wparams64[name].data), frob(t.data, wparams64[name].data)
        bar = 3e-5 if name.endswith("_bias") else 1e-5
        assert err_dev < bar or err_dev <= err_ref, (name, err_dev, err_ref)
        assert frob(got_p, t.data) < 1e-4, name
    ex.close()


def test_lm_20_steps_track_the_oracle(cuda_ctx):
    """A 2-layer llama_lm (d 128, 4/2 heads, ffn 192, vocab 512, 2 x 64
    tokens) for 20 SGD steps at lr 1e-3: every loss within rel 1e-4."""
    from tysor_b200.runtime import CudaGraphExecutor
    cfg = dict(layers=2, batch=2, seq=64, d_model=128, n_heads=4, n_kv_heads=2, hidden=192, vocab=512)
    g = llama_lm(**cfg, lr=1e-3, iterations=20)
    t = cfg["batch"] * cfg["seq"]
    seq = np.random.default_rng(5).integers(0, cfg["vocab"], t + 1)
    ins = {"ids": seq[:-1].astype(np.float32), "labels": seq[1:].astype(np.float32)}
    shapes = {"ids": [t], "labels": [t]}
    params = random_parameters(g, seed=6)
    L.set_threads(16)
    want, _ = L.train(g, shapes, inputs=ins, parameters=to_oracle(params))
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    got = ex.train()
    rel = rel_errors(got, want)
    assert rel.max() <= 1e-4, (rel.max(), int(rel.argmax()))
    assert want[-1] < want[0]
    ex.close()
