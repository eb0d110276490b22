"""Host-side plumbing of batch-sharded data parallelism.

The reference has no multi-device code.  Training here shards the batch
(rows / sequences) across ranks, one process per GPU; each rank runs the
whole step on its shard and the parameter gradients plus the loss are
summed with one NCCL all-reduce inside libtysor_cuda
(`tysor_cuda_graph_enable_allreduce`).  Sum, not mean: the reference loss is a
sum over the objective (training/executor.rs:810), so the sum of per-shard
gradients is the full-batch gradient.

torch.distributed is used only to exchange the NCCL unique id and to take
the max of per-rank timings; it can run on gloo (tests, CPU) or nccl.
"""
from __future__ import annotations

from typing import Tuple

import numpy as np


def shard_rows(total: int, rank: int, world: int, unit: int = 1) -> Tuple[int, int]:
    """[start, stop) of rank's share of `total` rows, in whole units of `unit`
    rows (a sequence), as even as possible; earlier ranks take the remainder."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("invalid rank / world size")
    if total % unit:
        raise ValueError("rows must be a whole number of units")
    units = total // unit
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start * unit, stop * unit


def broadcast_unique_id(uid: bytes, dist, src: int = 0) -> bytes:
    """Sends rank `src`'s 128-byte NCCL id to every rank (any backend)."""
    obj = [uid if dist.get_rank() == src else None]
    dist.broadcast_object_list(obj, src=src)
    out = obj[0]
    if not isinstance(out, (bytes, bytearray)) or len(out) != 128:
        raise RuntimeError("bad NCCL unique id received")
    return bytes(out)


def init_comm(ctx, dist, timeout_ms: int = 60000) -> None:
    """Creates the context's NCCL communicator over the ranks of `dist`."""
    from . import native
    lib = native.lib()
    rank, world = dist.get_rank(), dist.get_world_size()
    uid = np.zeros(128, np.uint8)
    if rank == 0:
        native.check(lib.tysor_cuda_nccl_get_unique_id(uid.ctypes.data_as(native.U8P)), "nccl_get_unique_id")
    got = broadcast_unique_id(uid.tobytes(), dist)
    uid = np.frombuffer(got, dtype=np.uint8).copy()
    native.check(lib.tysor_cuda_comm_init(ctx.handle, world, rank, uid.ctypes.data_as(native.U8P), timeout_ms),
                 "comm_init")


def check_peers(dist, timeout_s: float = 10.0) -> None:
    """Between steps: every rank must answer within `timeout_s`, else a
    RuntimeError names the ranks that did not (gloo's monitored barrier;
    other backends use a plain barrier bounded by the group timeout)."""
    import datetime
    if dist.get_backend() == "gloo":
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=timeout_s), wait_all_ranks=True)
    else:
        dist.barrier()


def max_over_ranks(value: float, dist, device=None) -> float:
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
