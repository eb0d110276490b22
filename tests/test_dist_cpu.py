"""Host-side data-parallel logic on CPU with world_size-2 gloo process groups:
batch sharding, NCCL-id exchange, the sum-of-shards = full-batch gradient
identity that makes the all-reduce exact, and detection of a rank that
leaves (the survivor gets an error, it does not hang)."""
import datetime
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _grad_worker(rank, world, port, q):
    try:
        dist = _setup(rank, world, port, 30)
        import torch
        import local as L
        from tysor_b200.dist import broadcast_unique_id, shard_rows
        from tysor_b200.programs import mlp_train

        uid = broadcast_unique_id(bytes(range(128)) if rank == 0 else b"", dist)
        assert uid == bytes(range(128))

        g = mlp_train(d_in=16, d_hidden=32, d_out=16)
        rng = np.random.default_rng(0)
        x = rng.standard_normal((8, 16)).astype(np.float32)
        t = rng.standard_normal((8, 16)).astype(np.float32)
        params = {}
        prng = np.random.default_rng(1)
        for name, shape in (("linear_4_weight", [16, 32]), ("linear_4_bias", [32]),
                            ("linear_8_weight", [32, 16]), ("linear_8_bias", [16])):
            params[name] = L.Tensor(shape, (0.1 * prng.standard_normal(int(np.prod(shape)))).astype(np.float32))
        a, b = shard_rows(8, rank, world)
        shapes = {"x": [b - a, 16], "target": [b - a, 16]}
        _, grads, _ = L.train_step_grads(g, shapes, inputs={"x": x[a:b], "target": t[a:b]}, parameters=params)
        summed = {}
        for name in sorted(grads):
            ten = torch.from_numpy(grads[name].data.copy())
            dist.all_reduce(ten)
            summed[name] = ten.numpy()
        if rank == 0:
            _, full, _ = L.train_step_grads(g, {"x": [8, 16], "target": [8, 16]}, inputs={"x": x, "target": t},
                                            parameters=params)
            for name, want in full.items():
                err = np.linalg.norm(summed[name] - want.data) / np.linalg.norm(want.data)
                assert err < 1e-5, (name, err)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def _failure_worker(rank, world, port, q):
    try:
        dist = _setup(rank, world, port, 20)
        from tysor_b200.dist import check_peers
        check_peers(dist, 10)  # step 0: both ranks present
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()
            os._exit(0)  # leaves between steps
        try:
            check_peers(dist, 3)  # step 1: rank 1 is gone
            q.put((rank, "no error"))
        except Exception as e:
            q.put((rank, "error: " + str(e).splitlines()[0][:120]))
    except Exception as e:
        q.put((rank, "setup " + repr(e)))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, msg = q.get(timeout=timeout)
        out[r] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_shard_rows():
    from tysor_b200.dist import shard_rows
    assert [shard_rows(16384, r, 4, unit=2048) for r in range(4)] == [(0, 4096), (4096, 8192), (8192, 12288),
                                                                      (12288, 16384)]
    assert [shard_rows(10, r, 3) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    with pytest.raises(ValueError):
        shard_rows(10, 3, 3)


def test_two_ranks_sum_of_shard_gradients_is_the_full_gradient():
    out = _run(_grad_worker)
    assert out == {0: "ok", 1: "ok"}, out


def test_a_rank_that_leaves_is_reported_not_waited_for():
    out = _run(_failure_worker)
    assert out[1] == "left"
    assert out[0].startswith("error"), out
