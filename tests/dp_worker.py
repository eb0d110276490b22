"""One rank of the data-parallel check in tests/test_gpu_dp.py (launched by
torch.distributed.run, one process per GPU).

Each rank takes its share of the batch (rows of the MLP, sequences of the
LM), creates a context on its GPU, joins the library's NCCL communicator
(the unique id travels over a gloo process group with a short timeout),
enables the step's gradient all-reduce and runs one train step at lr 0.
Rank 0 saves the all-reduced parameter gradients and loss to --out; every
rank reports its own result line so a failure names the rank.
"""
import argparse
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--workload", choices=["mlp", "lm"], required=True)
    p.add_argument("--out", required=True)
    args = p.parse_args()
    import torch
    import torch.distributed as dist

    from tysor_b200 import dist as tdist
    from tysor_b200.runtime import CudaContext, CudaGraphExecutor
    from dp_cases import case

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(local)
    g, shapes, inputs, params = case(args.workload, rank, world)
    ctx = CudaContext(local)
    try:
        tdist.init_comm(ctx, dist, timeout_ms=60000)
        ex = CudaGraphExecutor(ctx, g, shapes, inputs=inputs, parameters=params)
        ex.enable_allreduce(True)
        losses = ex.train(1, 0.0)
        grads = {name: ex.parameter_grad(name) for name in ex.parameter_names()}
        ex.close()
        tdist.check_peers(dist)
        if rank == 0:
            np.savez(args.out, loss=np.array(losses, np.float64), **grads)
        print(f"rank {rank}/{world}: ok, loss {losses[0]!r}", flush=True)
    finally:
        from tysor_b200 import native
        native.lib().tysor_cuda_comm_free(ctx.handle)
        ctx.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
