"""Micro-benchmark of single kernels through the C ABI (used for the ncu
captures summarised under profiles/).

    python kernel_bench.py matmul --m 4096 --n 5632 --k 2048 [--mode strict]
        [--ta] [--tb] [--reps 10]
    python kernel_bench.py rowop --op softmax --rows 65536 --width 4096
    python kernel_bench.py sweep [--div 1] [--reps 20] [--warmup 3]
    python kernel_bench.py block [--batch 1] [--reps 2] [--mode strict16]

Prints one JSON line with the average time per call (CUDA events on the
library's stream) and the achieved FLOP/s or GB/s.  `sweep` prints one line
per op of the norm/activation/loss sweep (x [65536, 4096] ~N(0,1), gain
~N(1,0.02), eps 1e-6; logits [8192, 32000] ~N(0,2), labels U[0, 32000))
and of the matmul+relu program (x, w [2048, 2048] U[-1,1]), each with its
algorithmic bytes (or FLOPs) and the fraction of the measured peak.  `--div
d` divides the row counts by d (for profiler captures of a smaller case).
All inputs are larger than L2 (126 MB), so back-to-back calls read HBM.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main() -> None:
    import torch

    from tysor_b200 import native
    from tysor_b200.runtime import CudaContext, DeviceBuffer

    p = argparse.ArgumentParser()
    p.add_argument("kind", choices=["matmul", "rowop", "sweep", "block"])
    p.add_argument("--batch", type=int, default=1, help="block: sequences of 2048 tokens")
    p.add_argument("--div", type=int, default=1)
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=5632)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--ta", action="store_true")
    p.add_argument("--tb", action="store_true")
    p.add_argument("--mode", default="strict", choices=["strict", "fast", "exact", "strict16"])
    p.add_argument("--op", default="softmax", choices=["softmax", "rms_norm", "silu", "cross_entropy_labels"])
    p.add_argument("--rows", type=int, default=65536)
    p.add_argument("--width", type=int, default=4096)
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args()

    ctx = CudaContext(0, matmul=a.mode)
    lib = native.lib()
    stream = torch.cuda.ExternalStream(lib.tysor_cuda_context_stream(ctx.handle))
    if a.kind == "sweep":
        sweep(ctx, lib, stream, a)
        ctx.close()
        return
    if a.kind == "block":
        # `reps` train steps of bench.py's Llama block (d 2048, 16/4 heads, ffn
        # 5632) on `batch` sequences of 2048 tokens: a small case of the
        # benchmarked step for profiler captures (batch 1 holds ~5 GB).
        import bench
        from tysor_b200.programs import random_parameters
        from tysor_b200.runtime import CudaGraphExecutor
        wl = bench.Block()
        tokens = a.batch * wl.seq
        g = wl.graph(1, batch=a.batch, seq=wl.seq)
        ex = CudaGraphExecutor(ctx, g, wl.shapes(1, tokens=tokens), inputs=wl.inputs(0, 1, tokens=tokens),
                               parameters=random_parameters(g, 1234))
        print(json.dumps({"kind": "block", "batch": a.batch, "mode": a.mode, "losses": ex.train(a.reps, wl.lr)}))
        ex.close()
        ctx.close()
        return
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


def time_calls(ctx, stream, call, reps: int, warmup: int) -> float:
    """Average milliseconds per call, CUDA events on the library's stream."""
    import torch
    for _ in range(warmup):
        call()
    ctx.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        call()
    e.record(stream)
    ctx.synchronize()
    e.synchronize()
    return s.elapsed_time(e) / max(reps, 1)


def measured_peaks():
    import os
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]), "tf32_tflops": float(pk["bf16_tflops"]) / 2.0}, "measured"
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "tf32_tflops": 1590.0 / 2.0}, "fallback"


def sweep(ctx, lib, stream, a) -> None:
    """The norm/activation/loss op sweep and matmul+relu at their full sizes
    (rows divided by --div)."""
    from tysor_b200 import native
    from tysor_b200.runtime import DeviceBuffer
    peaks, src = measured_peaks()
    rng = np.random.default_rng(0)
    rows, width = 65536 // a.div, 4096
    n = rows * width
    x = DeviceBuffer.from_array(ctx, rng.standard_normal(n, dtype=np.float32))
    dy = DeviceBuffer.from_array(ctx, rng.standard_normal(n, dtype=np.float32))
    out = DeviceBuffer.zeros(ctx, n)
    gain = DeviceBuffer.from_array(ctx, (1 + 0.02 * rng.standard_normal(width)).astype(np.float32))
    dgain = DeviceBuffer.zeros(ctx, width)
    ok = native.check
    h = ctx.handle
    f4 = 4.0 * n
    ops = [
        ("rms_norm", "x[%d,%d] -> y (eps 1e-5, no gain)" % (rows, width), 2 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_rms_norm(h, x.handle, out.handle, rows, width))),
        ("rms_norm_gain", "x, g -> y (eps 1e-6)", 2 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_rms_norm_gain(h, x.handle, gain.handle, out.handle, rows, width, 1e-6))),
        ("rms_norm_gain_backward", "x, dy -> dx, dgain", 3 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_rms_norm_gain_backward(h, x.handle, gain.handle, dy.handle, out.handle,
                                                                   dgain.handle, rows, width, 1e-6, False))),
        ("silu", "x -> y", 2 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_unary(h, 2, x.handle, out.handle, n, 0.0))),
        ("silu_backward", "x, dy -> dx", 3 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_silu_backward(h, x.handle, dy.handle, out.handle, n, False))),
        ("softmax", "x -> y", 2 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_softmax(h, x.handle, out.handle, rows, width))),
        ("softmax_backward", "y, dy -> dx (diagonal term)", 3 * f4,
         lambda: ok(lib.tysor_cuda_dispatch_softmax_backward(h, x.handle, dy.handle, out.handle, n, False))),
    ]
    lines = [run_op(ctx, stream, name, desc, nbytes, call, a, peaks, src) for name, desc, nbytes, call in ops]
    for buf in (x, dy, out, gain, dgain):
        buf.free()

    crows, classes = 8192 // a.div, 32000
    cn = crows * classes
    logits = DeviceBuffer.from_array(ctx, (2.0 * rng.standard_normal(cn, dtype=np.float32)))
    labels_np = rng.integers(0, classes, crows)
    labels = DeviceBuffer.from_array(ctx, labels_np.astype(np.float32))
    onehot = np.zeros(cn, np.float32)
    onehot[np.arange(crows) * classes + labels_np] = 1.0
    target = DeviceBuffer.from_array(ctx, onehot)
    del onehot
    loss = DeviceBuffer.zeros(ctx, crows)
    grad = DeviceBuffer.zeros(ctx, cn)
    c4 = 4.0 * cn
    ops = [
        ("cross_entropy_labels", "logits[%d,%d], labels -> loss" % (crows, classes), c4,
         lambda: ok(lib.tysor_cuda_dispatch_cross_entropy_labels(h, logits.handle, labels.handle, loss.handle,
                                                                 crows, classes))),
        ("cross_entropy_labels_backward", "logits, labels -> dlogits", 2 * c4,
         lambda: ok(lib.tysor_cuda_dispatch_cross_entropy_labels_backward(h, logits.handle, labels.handle,
                                                                          grad.handle, crows, classes, False))),
        ("cross_entropy", "logits, dense target -> loss (reference path)", 2 * c4,
         lambda: ok(lib.tysor_cuda_dispatch_cross_entropy(h, logits.handle, target.handle, loss.handle,
                                                          crows, classes))),
        ("cross_entropy_backward", "logits, dense target -> dlogits", 3 * c4,
         lambda: ok(lib.tysor_cuda_dispatch_cross_entropy_backward(h, logits.handle, target.handle, grad.handle,
                                                                   crows, classes, False))),
    ]
    lines += [run_op(ctx, stream, name, desc, nbytes, call, a, peaks, src) for name, desc, nbytes, call in ops]
    for buf in (logits, labels, target, loss, grad):
        buf.free()

    m = 2048
    xm = DeviceBuffer.from_array(ctx, np.random.default_rng(0).uniform(-1, 1, m * m).astype(np.float32))
    wm = DeviceBuffer.from_array(ctx, np.random.default_rng(1).uniform(-1, 1, m * m).astype(np.float32))
    ym = DeviceBuffer.zeros(ctx, m * m)
    ms = time_calls(ctx, stream, lambda: ok(lib.tysor_cuda_dispatch_matmul_ex(
        h, 1, m, m, m, xm.handle, False, m, 0, wm.handle, False, m, 0, ym.handle, m, 0, None, 1.0, False, True)),
        a.reps, a.warmup)
    flops = 2.0 * m ** 3
    tf = flops / (ms / 1e3) / 1e12
    # strict16 issues its three products at the fp16 (= bf16) tensor rate; the others at tf32's.
    peak = 2.0 * peaks["tf32_tflops"] if a.mode == "strict16" else peaks["tf32_tflops"]
    mmas = 1 if a.mode == "fast" else 3
    engine = {"strict": "strict 3xTF32", "strict16": "strict16 (split-fp16, packing included)", "fast": "fast 1xTF32",
              "exact": "exact (CUDA cores)"}[a.mode]
    lines.append({"op": "matmul_relu", "shape": f"x, w [2048, 2048] {engine}", "ms": round(ms, 4),
                  "TFLOP/s": round(tf, 1), "peak": peak, "frac": round(tf / peak, 4),
                  "pipe_frac": round(mmas * tf / peak, 4), "peak_source": src})
    for buf in (xm, wm, ym):
        buf.free()
    for line in lines:
        print(json.dumps(line), flush=True)


def run_op(ctx, stream, name, desc, nbytes, call, a, peaks, src) -> dict:
    ms = time_calls(ctx, stream, call, a.reps, a.warmup)
    gbs = nbytes / (ms / 1e3) / 1e9
    return {"op": name, "shape": desc, "bytes": nbytes, "ms": round(ms, 4), "GB/s": round(gbs, 1),
            "peak": peaks["hbm_gbs"], "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": src}


if __name__ == "__main__":
    main()
