"""Parity at the benchmarked sizes: the workloads `bench.py` times, with its
own seeded inputs and parameters, on the device against the oracle.

* Llama block at full dimensions, one sequence: S 2048, d_model 2048,
  16 query / 4 KV heads (head_dim 128), SwiGLU 5632, RMSNorm eps 1e-6,
  squared error against a seeded target (bench.py's `block` workload with
  batch 1): forward output, loss, every parameter gradient, and the
  parameters after one SGD step.  This runs the kernel forms of the
  benchmark on their real operands: the persistent pair GEMM at K 2048 and
  5632, the causal score/probability GEMMs, the fused softmax backward in
  the dP GEMM's epilogue, the residual epilogue and split-K weight
  gradients.
* Two-layer MLP at full size ([8192, 1024] -> 4096 -> 1024, bias, ReLU, mean
  squared error, SGD lr 1e-3) for 3 steps.
* The 4-layer LM (full block dimensions, vocab 32000, tied head, next-token
  cross entropy) on one sequence of 256 tokens for 2 steps.

Bars (the accuracy contract: strict matmul and fp32 ops rel 1e-5, training
losses rel 1e-4): forward values and parameters Frobenius rel 1e-5; losses
rel 1e-4; parameter gradients Frobenius rel GRAD_BAR.  Every measured error
is printed (run with -s) so the margin is visible.
"""
import os
import sys

import numpy as np
import pytest

import local as L
from tysor_b200.programs import random_parameters

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402  (the workloads' seeded inputs)

pytestmark = pytest.mark.gpu

GRAD_BAR = 1e-5


def frob(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_oracle(params):
    return {k: L.Tensor(list(v.shape), np.ascontiguousarray(v, np.float32).reshape(-1).copy())
            for k, v in params.items()}


def report(title, errs):
    worst = max(errs.items(), key=lambda kv: kv[1])
    print(f"\n{title}: worst {worst[0]} {worst[1]:.3e}")
    for k, v in sorted(errs.items()):
        print(f"  {k}: {v:.3e}")


def test_block_full_dims_one_sequence(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    wl = bench.Block()
    seq = 2048
    g = wl.graph(1, batch=1, seq=seq)
    shapes = wl.shapes(1, tokens=seq)
    ins = wl.inputs(0, 1, tokens=seq)
    params = random_parameters(g, 1234)
    L.set_threads(os.cpu_count() or 1)
    values, grads, _ = L.train_step_grads(g, shapes, inputs=ins, parameters=to_oracle(params))
    want_params = to_oracle(params)
    L.apply_sgd(want_params, grads, wl.lr)

    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    losses = ex.train(1, wl.lr)
    errs = {}
    out_id = g.named["out"]
    errs["value out"] = frob(ex.value(out_id).data, values[out_id][1].data)
    loss_id = g.objective_id()
    want_loss = L.tensor_sum(values[loss_id][1])
    errs["loss"] = abs(losses[0] - want_loss) / abs(want_loss)
    assert len(grads) == len(params)
    for name, gt in grads.items():
        got = ex.parameter_grad(name)
        assert np.isfinite(got).all(), name
        errs["grad " + name] = frob(got, gt.data)
    for name, t in want_params.items():
        errs["param " + name] = frob(ex.parameter(name), t.data)
    ex.close()
    report("block 1 x 2048, full dims", errs)
    assert errs["value out"] < 1e-5
    assert errs["loss"] < 1e-4
    for k, v in errs.items():
        if k.startswith("grad "):
            assert v < GRAD_BAR, (k, v)
        if k.startswith("param "):
            assert v < 1e-5, (k, v)


def test_mlp_full_size_three_steps(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    wl = bench.Mlp()
    g = wl.graph(1)
    shapes = wl.shapes(1)
    ins = wl.inputs(0, 1)
    params = random_parameters(g, 1234)
    L.set_threads(os.cpu_count() or 1)
    want, wparams = L.train(g, shapes, inputs=ins, parameters=to_oracle(params), lr=wl.lr, iterations=3)
    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    got = ex.train(3, wl.lr)
    errs = {f"loss {i}": abs(a - b) / abs(b) for i, (a, b) in enumerate(zip(got, want))}
    for name, t in wparams.items():
        errs["param " + name] = frob(ex.parameter(name), t.data)
    ex.close()
    report("mlp [8192,1024]->4096->1024, 3 steps", errs)
    for k, v in errs.items():
        assert v < (1e-4 if k.startswith("loss") else 1e-5), (k, v)


def test_lm_4_layers_vocab_32000_two_steps(cuda_ctx):
    from tysor_b200.runtime import CudaGraphExecutor
    wl = bench.Lm()
    seq = 256
    g = wl.graph(1, batch=1, seq=seq)
    lr = wl.base_lr / seq
    shapes = wl.shapes(1, tokens=seq)
    ins = wl.inputs(0, 1, tokens=seq)
    params = random_parameters(g, 1234)
    L.set_threads(os.cpu_count() or 1)
    # Step 1 with its gradients, then step 2 from the updated parameters.
    values, grads, _ = L.train_step_grads(g, shapes, inputs=ins, parameters=to_oracle(params))
    oid = g.objective_id()
    want_losses = [L.tensor_sum(values[oid][1])]
    p1 = to_oracle(params)
    L.apply_sgd(p1, grads, lr)
    more, p2 = L.train(g, shapes, inputs=ins, parameters=p1, lr=lr, iterations=1)
    want_losses += more

    ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs=ins, parameters=params)
    got = ex.train(1, lr)
    errs = {}
    for name, gt in grads.items():
        errs["grad " + name] = frob(ex.parameter_grad(name), gt.data)
    got += ex.train(1, lr)
    errs.update({f"loss {i}": abs(a - b) / abs(b) for i, (a, b) in enumerate(zip(got, want_losses))})
    for name, t in p2.items():
        errs["param " + name] = frob(ex.parameter(name), t.data)
    ex.close()
    report("lm 4 layers, vocab 32000, 1 x 256 tokens, 2 steps", errs)
    for k, v in errs.items():
        bar = 1e-4 if k.startswith("loss") else (GRAD_BAR if k.startswith("grad") else 1e-5)
        assert v < bar, (k, v)
