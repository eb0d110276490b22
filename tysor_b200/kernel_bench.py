"""Micro-benchmark of single kernels through the C ABI (used for the ncu
captures summarised under profiles/).

    python -m tysor_b200.kernel_bench matmul --m 4096 --n 5632 --k 2048 [--mode strict]
        [--ta] [--tb] [--reps 10]
    python -m tysor_b200.kernel_bench rowop --op softmax --rows 65536 --width 4096

Prints one JSON line with the average time per call (CUDA events on the
library's stream) and the achieved FLOP/s or GB/s.
"""
from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    import torch

    from . import native
    from .runtime import CudaContext, DeviceBuffer

    p = argparse.ArgumentParser()
    p.add_argument("kind", choices=["matmul", "rowop"])
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=5632)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--ta", action="store_true")
    p.add_argument("--tb", action="store_true")
    p.add_argument("--mode", default="strict", choices=["strict", "fast", "exact"])
    p.add_argument("--op", default="softmax", choices=["softmax", "rms_norm", "silu", "cross_entropy_labels"])
    p.add_argument("--rows", type=int, default=65536)
    p.add_argument("--width", type=int, default=4096)
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args()

    ctx = CudaContext(0, matmul=a.mode)
    lib = native.lib()
    stream = torch.cuda.ExternalStream(lib.tysor_cuda_context_stream(ctx.handle))
    rng = np.random.default_rng(0)
    if a.kind == "matmul":
        m, n, k = a.m, a.n, a.k
        A = DeviceBuffer.from_array(ctx, rng.uniform(-1, 1, m * k).astype(np.float32))
        B = DeviceBuffer.from_array(ctx, rng.uniform(-1, 1, k * n).astype(np.float32))
        C = DeviceBuffer.zeros(ctx, m * n)
        lda = m if a.ta else k
        ldb = k if a.tb else n

        def call():
            native.check(lib.tysor_cuda_dispatch_matmul_ex(ctx.handle, 1, m, n, k, A.handle, a.ta, lda, 0, B.handle,
                                                           a.tb, ldb, 0, C.handle, n, 0, None, 1.0, False, False))
        work, unit = 2.0 * m * n * k, "TFLOP/s"
    else:
        rows, w = a.rows, a.width
        X = DeviceBuffer.from_array(ctx, rng.standard_normal(rows * w, dtype=np.float32))
        O = DeviceBuffer.zeros(ctx, rows * w)
        lab = DeviceBuffer.from_array(ctx, rng.integers(0, w, rows).astype(np.float32))

        def call():
            if a.op == "softmax":
                ok = lib.tysor_cuda_dispatch_softmax(ctx.handle, X.handle, O.handle, rows, w)
            elif a.op == "rms_norm":
                ok = lib.tysor_cuda_dispatch_rms_norm(ctx.handle, X.handle, O.handle, rows, w)
            elif a.op == "silu":
                ok = lib.tysor_cuda_dispatch_unary(ctx.handle, 2, X.handle, O.handle, rows * w, 0.0)
            else:
                ok = lib.tysor_cuda_dispatch_cross_entropy_labels(ctx.handle, X.handle, lab.handle, O.handle, rows, w)
            native.check(ok)
        work = 8.0 * rows * w if a.op != "cross_entropy_labels" else 4.0 * rows * w
        unit = "GB/s"
    for _ in range(a.warmup):
        call()
    ctx.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(a.reps):
        call()
    e.record(stream)
    ctx.synchronize()
    e.synchronize()
    ms = s.elapsed_time(e) / a.reps
    rate = work / (ms / 1000.0) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"kind": a.kind, "args": vars(a), "ms": round(ms, 4), unit: round(rate, 1)}))
    ctx.close()


if __name__ == "__main__":
    main()
