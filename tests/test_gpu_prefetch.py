"""Prefetched inputs (tysor_cuda_graph_prefetch_input): values queued from
pinned host memory on the copy stream are taken by the following train
calls in order, and training on them gives exactly the losses and
parameters of uploading each value right before its step -- also when the
steps are enqueued without waiting (tysor_cuda_graph_train_enqueue), the
host running ahead of the device, and each loss is read back on the
stream."""
import numpy as np
import pytest
import torch

from tysor_b200 import native
from tysor_b200.programs import mlp_train, random_parameters

pytestmark = pytest.mark.gpu

ROWS, D_IN, D_H = 512, 128, 256


def batches(n):
    rng = np.random.default_rng(11)
    return [{"x": rng.standard_normal((ROWS, D_IN), dtype=np.float32),
             "target": rng.standard_normal((ROWS, D_IN), dtype=np.float32)} for _ in range(n)]


def make(ctx, first):
    from tysor_b200.runtime import CudaGraphExecutor
    g = mlp_train(D_IN, D_H, D_IN, lr=0.01, iterations=1, loss_scale=1.0 / (ROWS * D_IN))
    ex = CudaGraphExecutor(ctx, g, {"x": [ROWS, D_IN], "target": [ROWS, D_IN]}, inputs=first,
                           parameters=random_parameters(g, 5))
    return g, ex


def reference_run(ctx, data):
    """Upload each batch, then step (synchronously)."""
    g, ex = make(ctx, data[0])
    ex.train(1, 0.0)  # plans the buffers (lr 0: parameters unchanged)
    want = []
    for b in data:
        for name, arr in b.items():
            ex.upload_input(name, arr)
        want += ex.train(1, 0.01)
    want_p = {n: ex.parameter(n) for n in random_parameters(g, 5)}
    ex.close()
    return want, want_p


def test_enqueued_prefetched_steps_match_synchronous_steps(cuda_ctx):
    data = batches(6)
    want, want_p = reference_run(cuda_ctx, data)
    g, ex = make(cuda_ctx, data[0])
    ex.train(1, 0.0)
    pinned = [{k: torch.from_numpy(v).pin_memory() for k, v in b.items()} for b in data]
    losses = torch.zeros(len(data), dtype=torch.float32).pin_memory()
    host = losses.numpy()
    for name, t in pinned[0].items():
        ex.prefetch_input(name, t.numpy())
    for i in range(len(data)):
        if i + 1 < len(data):
            for name, t in pinned[i + 1].items():
                ex.prefetch_input(name, t.numpy())
        ex.train_enqueue(1, 0.01, host[i:i + 1])  # returns at once
    cuda_ctx.synchronize()
    assert [float(v) for v in host] == want
    for n, w in want_p.items():
        np.testing.assert_array_equal(ex.parameter(n), w)
    ex.close()


def test_prefetched_steps_match_uploaded_steps(cuda_ctx):
    data = batches(5)
    # Reference run: upload each batch, then step.
    g, ex = make(cuda_ctx, data[0])
    ex.train(1, 0.0)  # plans the buffers (lr 0: parameters unchanged)
    want = []
    for b in data:
        for name, arr in b.items():
            ex.upload_input(name, arr)
        want += ex.train(1, 0.01)
    names = list(random_parameters(g, 5))
    want_p = {n: ex.parameter(n) for n in names}
    ex.close()

    # Prefetched run from pinned host memory, one step ahead.
    g, ex = make(cuda_ctx, data[0])
    ex.train(1, 0.0)
    pinned = [{k: torch.from_numpy(v).pin_memory() for k, v in b.items()} for b in data]
    got = []
    for name, t in pinned[0].items():
        ex.prefetch_input(name, t.numpy())
    for i in range(len(data)):
        if i + 1 < len(data):
            for name, t in pinned[i + 1].items():
                ex.prefetch_input(name, t.numpy())
        got += ex.train(1, 0.01)
    assert got == want
    for n in names:
        np.testing.assert_array_equal(ex.parameter(n), want_p[n])
    ex.close()


def test_prefetch_queue_holds_two_values(cuda_ctx):
    data = batches(3)
    g, ex = make(cuda_ctx, data[0])
    ex.train(1, 0.0)
    ex.prefetch_input("x", data[1]["x"])
    ex.prefetch_input("x", data[2]["x"])
    with pytest.raises(native.NativeError, match="two prefetched values"):
        ex.prefetch_input("x", data[0]["x"])
    with pytest.raises(native.NativeError, match="holds"):
        ex.prefetch_input("target", data[0]["target"][:5])
    ex.train(2, 0.0)  # takes one queued value (the call's first step); one stays queued
    ex.prefetch_input("x", data[0]["x"])
    ex.close()


def test_replanning_forgets_uploaded_inputs(cuda_ctx):
    """An input written by upload_input lives in the planned buffers; a
    re-plan (here: a new matmul mode) makes new buffers, so the next step
    must take the input from its host copy again, not read a buffer nothing
    wrote."""
    data = batches(2)
    g, ex = make(cuda_ctx, data[0])
    ex.train(1, 0.0)
    for name, arr in data[1].items():
        ex.upload_input(name, arr)
    cuda_ctx.set_matmul_mode("exact")
    try:
        got = ex.train(1, 0.0)  # re-planned: the constructor's inputs (data[0])
    finally:
        cuda_ctx.set_matmul_mode("strict")
    ex.close()
    cuda_ctx.set_matmul_mode("exact")
    try:
        _, fresh = make(cuda_ctx, data[0])
        want = fresh.train(1, 0.0)
        fresh.close()
    finally:
        cuda_ctx.set_matmul_mode("strict")
    assert got == want
