"""The library's own data-parallel path: the NCCL communicator of a context
(tysor_cuda_nccl_get_unique_id / tysor_cuda_comm_init) and the train step's
gradient all-reduce (tysor_cuda_graph_enable_allreduce).

* One rank: a communicator over a single GPU makes the all-reduce an
  identity, so a step with it enabled must give bit-identical gradients,
  loss and parameters to a step without it, and tysor_cuda_allreduce_sum on
  a buffer must leave it unchanged.
* Two and four ranks (needs that many GPUs): each rank trains on its share
  of the batch with the all-reduce on; the summed gradients must equal the
  one-rank full-batch gradient (Frobenius rel 1e-5: only the fp32 summation
  order differs), and the summed loss the full-batch loss.  Run under torch.distributed.run
  with a gloo group for the id exchange and a bounded process lifetime.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from dp_cases import case  # noqa: E402

pytestmark = pytest.mark.gpu


def frob(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def full_batch(workload, device=0):
    from tysor_b200.runtime import CudaContext, CudaGraphExecutor
    g, shapes, inputs, params = case(workload, 0, 1)
    with CudaContext(device) as ctx:
        ex = CudaGraphExecutor(ctx, g, shapes, inputs=inputs, parameters=params)
        losses = ex.train(1, 0.0)
        grads = {n: ex.parameter_grad(n) for n in ex.parameter_names()}
        ex.close()
    return losses, grads


def test_one_rank_communicator_is_an_identity():
    from tysor_b200 import native
    from tysor_b200.runtime import CudaContext, CudaGraphExecutor, DeviceBuffer
    lib = native.lib()
    g, shapes, inputs, params = case("lm", 0, 1)
    want_losses, want_grads = full_batch("lm")
    with CudaContext(0) as ctx:
        uid = np.zeros(128, np.uint8)
        native.check(lib.tysor_cuda_nccl_get_unique_id(uid.ctypes.data_as(native.U8P)), "unique id")
        native.check(lib.tysor_cuda_comm_init(ctx.handle, 1, 0, uid.ctypes.data_as(native.U8P), 30000), "comm_init")
        try:
            x = np.random.default_rng(3).standard_normal(100003).astype(np.float32)
            buf = DeviceBuffer.from_array(ctx, x)
            native.check(lib.tysor_cuda_allreduce_sum(ctx.handle, buf.handle, x.size), "allreduce")
            np.testing.assert_array_equal(buf.read(), x)
            buf.free()
            ex = CudaGraphExecutor(ctx, g, shapes, inputs=inputs, parameters=params)
            ex.enable_allreduce(True)
            for _ in range(2):  # the eager first step, then the captured graph's replay
                losses = ex.train(1, 0.0)
                assert losses == want_losses
                for name, w in want_grads.items():
                    np.testing.assert_array_equal(ex.parameter_grad(name), w, err_msg=name)
            ex.close()
        finally:
            native.check(lib.tysor_cuda_comm_free(ctx.handle), "comm_free")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("workload", ["mlp", "lm"])
def test_ranks_sum_to_the_full_batch_gradient(workload, world, tmp_path):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / f"{workload}.npz"
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           os.path.join(HERE, "dp_worker.py"), "--workload", workload, "--out", str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    got = np.load(out)
    want_losses, want_grads = full_batch(workload)
    assert abs(float(got["loss"][0]) - want_losses[0]) <= 1e-5 * abs(want_losses[0])
    errs = {name: frob(got[name], w) for name, w in want_grads.items()}
    print(f"\n{workload} {world}-rank vs 1-rank gradients:", {k: f"{v:.2e}" for k, v in errs.items()})
    for name, e in errs.items():
        assert e < 1e-5, (name, e)
