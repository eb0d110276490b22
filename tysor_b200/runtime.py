"""Host-side runtime of the CUDA backend: the Python mirror of the
reference's backend entry points, driving libtysor_cuda.so.

  run_cuda_module      <- run_metal_module / run_local_forward_module
                          (src/backend/metal/runtime.rs:434-451,
                           src/runtime/interpreter.rs:24-54)
  backward_cuda_module <- run_backward_module (src/training/backward.rs:382-399)
  train_cuda_module    <- run_train_module (src/training/executor.rs:764-816)

Each returns the values and also formats them exactly as the reference
prints them (tensor.rs:36-69, backward.rs:385-397, executor.rs:794-814), so
a harness can diff the text.  There is no fallback path: every tensor
operation runs in libtysor_cuda on an sm_100 device.
"""
from __future__ import annotations

import collections
import ctypes
import json
import os
import re
import weakref
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import native
from .graph import Graph
from .native import check, fptr

MATMUL_MODES = {"strict": 0, "fast": 1, "exact": 2, "strict16": 3}


class CudaContext:
    """A device, its stream and scratch (tysor_cuda_context_new).

    Buffers and graph executors made on a context must be released before
    it; `close()` releases any that are still open."""

    def __init__(self, device: int = 0, matmul: Optional[str] = None):
        """`matmul`: strict (3xTF32), strict16, fast or exact; by default
        $TYSOR_CUDA_MATMUL, else strict."""
        mode = matmul or os.environ.get("TYSOR_CUDA_MATMUL", "strict")
        if mode not in MATMUL_MODES:
            raise ValueError(f"matmul mode {mode!r}: expected one of {', '.join(MATMUL_MODES)}")
        self._lib = native.lib()
        self.handle = self._lib.tysor_cuda_context_new(int(device))
        check(self.handle, "tysor_cuda_context_new")
        self.device = device
        self._children = weakref.WeakSet()
        self.set_matmul_mode(mode)

    def _adopt(self, child) -> None:
        self._children.add(child)

    def set_matmul_accumulation(self, kblocks: int) -> None:
        """k-blocks (16 elements of K) per tensor-memory accumulation chunk;
        0 = the default (8).  Shorter is more accurate and slower."""
        check(native.lib().tysor_cuda_set_matmul_accumulation(self.handle, int(kblocks)), "set_matmul_accumulation")

    def set_matmul_mode(self, mode: str) -> None:
        check(self._lib.tysor_cuda_set_matmul_mode(self.handle, MATMUL_MODES[mode]), "set_matmul_mode")

    def synchronize(self) -> None:
        check(self._lib.tysor_cuda_synchronize(self.handle), "synchronize")

    def close(self) -> None:
        if self.handle:
            for child in list(self._children):
                child.close()
            self._lib.tysor_cuda_context_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class DeviceBuffer:
    """An fp32 device buffer (tysor_cuda_buffer_*)."""

    def __init__(self, ctx: CudaContext, handle, count: int):
        self.ctx = ctx
        self.handle = handle
        self.count = count
        ctx._adopt(self)

    @classmethod
    def from_array(cls, ctx: CudaContext, arr) -> "DeviceBuffer":
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        h = native.lib().tysor_cuda_buffer_new_with_data(ctx.handle, fptr(a), a.size)
        check(h, "buffer_new_with_data")
        return cls(ctx, h, a.size)

    @classmethod
    def zeros(cls, ctx: CudaContext, count: int) -> "DeviceBuffer":
        h = native.lib().tysor_cuda_buffer_new_zeroed(ctx.handle, int(count))
        check(h, "buffer_new_zeroed")
        return cls(ctx, h, int(count))

    def read(self, count: Optional[int] = None) -> np.ndarray:
        n = self.count if count is None else count
        out = np.empty(n, dtype=np.float32)
        check(native.lib().tysor_cuda_buffer_read(self.handle, fptr(out), n), "buffer_read")
        return out

    def write(self, arr) -> None:
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        check(native.lib().tysor_cuda_buffer_write(self.handle, fptr(a), a.size), "buffer_write")

    def free(self) -> None:
        if self.handle and self.ctx.handle:
            native.lib().tysor_cuda_buffer_free(self.handle)
        self.handle = None

    close = free

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


@dataclass
class HostTensor:
    shape: List[int]
    data: np.ndarray
    dtype: str = "float32"


def _format_value(v: float) -> str:
    """Rust's `{:.4}` for an f32 (tensor.rs:63-66): correctly rounded fixed
    point, `inf` / `-inf`, and `NaN` for every NaN."""
    v = float(v)
    return "NaN" if v != v else f"{v:.4f}"


def format_tensor(t: HostTensor) -> str:
    """tensor.rs:48-69 print_tensor_body."""
    vals = ", ".join(_format_value(v) for v in t.data)
    return f"shape=[{', '.join(str(d) for d in t.shape)}] dtype={t.dtype}\nvalues=[{vals}]"


class CudaGraphExecutor:
    """The device-resident executor for one lowered graph."""

    def __init__(self, ctx: CudaContext, graph: Graph, shapes: Dict[str, Sequence[int]],
                 inputs: Optional[Dict[str, np.ndarray]] = None,
                 parameters: Optional[Dict[str, np.ndarray]] = None):
        self.ctx = ctx
        self.graph = graph
        self._lib = native.lib()
        self.handle = self._lib.tysor_cuda_graph_new(ctx.handle, graph.to_text().encode())
        check(self.handle, "graph_new")
        # dtype strings carried with the values (computation is f32);
        # gradients carry the objective's (the ones seed's, backward.rs:178).
        self._dtypes = graph.value_dtypes()
        self._grad_dtype = self._dtypes.get(graph.objective_id(), "float32") if graph.outputs else "float32"
        # host arrays of queued prefetches (at most two wait per input, one
        # more may still be copying)
        self._prefetched: Dict[str, collections.deque] = {}
        ctx._adopt(self)
        for name, dims in shapes.items():
            self.set_shape(name, dims)
        for name, arr in (inputs or {}).items():
            self.set_input(name, arr)
        for name, arr in (parameters or {}).items():
            self.set_parameter(name, arr)

    def set_shape(self, name: str, dims: Sequence[int]) -> None:
        d = (ctypes.c_int64 * len(dims))(*[int(x) for x in dims])
        check(self._lib.tysor_cuda_graph_set_shape(self.handle, name.encode(), d, len(dims)), "set_shape")

    def set_input(self, name: str, arr) -> None:
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        check(self._lib.tysor_cuda_graph_set_input(self.handle, name.encode(), fptr(a), a.size), "set_input")

    def set_parameter(self, name: str, arr) -> None:
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        check(self._lib.tysor_cuda_graph_set_parameter(self.handle, name.encode(), fptr(a), a.size),
              "set_parameter")

    def set_capture(self, enable: bool) -> None:
        check(self._lib.tysor_cuda_graph_set_capture(self.handle, bool(enable)), "set_capture")

    def set_loss_order(self, order: str) -> None:
        """"tree" (default) or "sequential" (the reference's f32 tensor_sum order)."""
        codes = {"tree": 0, "sequential": 1}
        if order not in codes:
            raise ValueError("loss order is 'tree' or 'sequential'")
        check(self._lib.tysor_cuda_graph_set_loss_order(self.handle, codes[order]), "set_loss_order")

    def enable_allreduce(self, enable: bool = True) -> None:
        check(self._lib.tysor_cuda_graph_enable_allreduce(self.handle, bool(enable)), "enable_allreduce")

    # --- execution -----------------------------------------------------------
    def run(self) -> HostTensor:
        check(self._lib.tysor_cuda_graph_run(self.handle), "run")
        if not self.graph.outputs:
            raise native.NativeError("Entry function did not return a value")
        if len(self.graph.outputs) != 1:
            raise native.NativeError("Runtime interpreter currently supports a single return value")
        return self.value(self.graph.outputs[0])

    def backward(self) -> List[Tuple[str, HostTensor]]:
        """backward.rs:382-399: gradient of every graph parameter (zeros if none)."""
        check(self._lib.tysor_cuda_graph_backward(self.handle), "backward")
        out = []
        for v in self.graph.parameters():
            g = self.value_grad(v.id)
            if g is None:
                t = self.value(v.id)
                g = HostTensor(t.shape, np.zeros_like(t.data), t.dtype)
            out.append((f"{v.name}_grad", g))
        return out

    def train(self, iterations: Optional[int] = None, lr: Optional[float] = None) -> List[float]:
        it = self.graph.iterations if iterations is None else int(iterations)
        rate = self.graph.lr if lr is None else float(lr)
        if self.graph.optimizer != "sgd":
            raise native.NativeError("Train executor currently supports only optimizer='sgd'")
        losses = np.zeros(max(it, 1), dtype=np.float32)
        check(self._lib.tysor_cuda_graph_train(self.handle, it, rate, fptr(losses)), "train")
        return [float(x) for x in losses[:it]]

    def train_enqueue(self, iterations: int, lr: float, host_losses: Optional[np.ndarray] = None) -> None:
        """Enqueues `iterations` train steps without waiting; step i's loss is
        copied to host_losses[i] (a float32 array, pinned for an asynchronous
        copy) on the stream.  The values are valid after ctx.synchronize(),
        which also reports errors.  Keep host_losses alive until then."""
        ptr = None
        if host_losses is not None:
            if host_losses.dtype != np.float32 or not host_losses.flags["C_CONTIGUOUS"] or host_losses.size < iterations:
                raise ValueError("host_losses must be a contiguous float32 array of at least `iterations` values")
            ptr = fptr(host_losses)
        check(self._lib.tysor_cuda_graph_train_enqueue(self.handle, int(iterations), float(lr), ptr), "train_enqueue")

    def train_traced(self, lr: Optional[float] = None) -> List[Tuple[str, float]]:
        """One train step launched op by op; returns (label, device ms) for
        each planned step item, in forward, backward, update order."""
        rate = self.graph.lr if lr is None else float(lr)
        n = ctypes.c_int(0)
        check(self._lib.tysor_cuda_graph_train_traced(self.handle, rate, None, 0, ctypes.byref(n)), "train_traced")
        ms = np.zeros(max(n.value, 1), dtype=np.float32)
        check(self._lib.tysor_cuda_graph_train_traced(self.handle, rate, fptr(ms), ms.size, ctypes.byref(n)),
              "train_traced")
        labels = [(self._lib.tysor_cuda_graph_trace_label(self.handle, i) or b"").decode() for i in range(n.value)]
        return list(zip(labels, [float(v) for v in ms[:n.value]]))

    # --- results -------------------------------------------------------------
    def shape(self, value_id: int) -> List[int]:
        r = self._lib.tysor_cuda_graph_value_rank(self.handle, int(value_id))
        check(r >= 0, "value_rank")
        d = (ctypes.c_int64 * max(r, 1))()
        check(self._lib.tysor_cuda_graph_value_shape(self.handle, int(value_id), d), "value_shape")
        return [int(d[i]) for i in range(r)]

    def value(self, value_id: int) -> HostTensor:
        s = self.shape(value_id)
        out = np.empty(int(np.prod(s, dtype=np.int64)), dtype=np.float32)
        check(self._lib.tysor_cuda_graph_read_value(self.handle, int(value_id), fptr(out), out.size), "read_value")
        return HostTensor(s, out, self._dtypes.get(int(value_id), "float32"))

    def value_grad(self, value_id: int) -> Optional[HostTensor]:
        s = self.shape(value_id)
        out = np.empty(int(np.prod(s, dtype=np.int64)), dtype=np.float32)
        if not self._lib.tysor_cuda_graph_read_value_grad(self.handle, int(value_id), fptr(out), out.size):
            return None
        return HostTensor(s, out, self._grad_dtype)

    def parameter_names(self) -> List[str]:
        n = self._lib.tysor_cuda_graph_num_parameters(self.handle)
        check(n >= 0, "num_parameters")
        return [self._lib.tysor_cuda_graph_parameter_name(self.handle, i).decode() for i in range(n)]

    def parameter(self, name: str) -> np.ndarray:
        n = self._lib.tysor_cuda_graph_parameter_count(self.handle, name.encode())
        out = np.empty(n, dtype=np.float32)
        check(self._lib.tysor_cuda_graph_read_parameter(self.handle, name.encode(), fptr(out), n), "read_parameter")
        return out

    def parameter_grad(self, name: str) -> np.ndarray:
        n = self._lib.tysor_cuda_graph_parameter_count(self.handle, name.encode())
        out = np.empty(n, dtype=np.float32)
        check(self._lib.tysor_cuda_graph_read_parameter_grad(self.handle, name.encode(), fptr(out), n),
              "read_parameter_grad")
        return out

    def parameters(self) -> Dict[str, np.ndarray]:
        return {n: self.parameter(n) for n in self.parameter_names()}

    def launch_count(self) -> int:
        return int(self._lib.tysor_cuda_graph_launch_count(self.handle))

    def close(self) -> None:
        if self.handle and self.ctx.handle:
            self._lib.tysor_cuda_graph_free(self.handle)
        self.handle = None

    def upload_input(self, name: str, arr) -> None:
        """Host -> device copy of a graph input, enqueued on the stream (pinned
        host memory makes it asynchronous); the graph must have run once."""
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        check(self._lib.tysor_cuda_graph_upload_input(self.handle, name.encode(), fptr(a), a.size), "upload_input")

    def prefetch_input(self, name: str, arr) -> None:
        """Queues the next value of a graph input: host -> device on the
        library's copy stream (overlapping kernels already queued), taken by
        the next run / backward / train call; at most two may wait.  Pinned
        host memory makes the copy asynchronous: keep the array unchanged
        until that call returns (this object holds a reference until then)."""
        a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32).reshape(-1))
        check(self._lib.tysor_cuda_graph_prefetch_input(self.handle, name.encode(), fptr(a), a.size),
              "prefetch_input")
        self._prefetched.setdefault(name, collections.deque(maxlen=3)).append(a)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- reference-shaped entry points --------------------------------------------------

DUMP_ENV = "TYSOR_DUMP_DIR"


def dump_tensor(name: str, t: HostTensor, directory: Optional[str] = None) -> Optional[str]:
    """Binary side channel next to the text output: when `directory` (or the
    TYSOR_DUMP_DIR environment variable) is set, writes `<name>.f32` (the
    values, little-endian f32, row-major) and `<name>.json` (shape, dtype)
    there, so results can be compared at full precision instead of through
    the 4-decimal text of print_tensor.  Returns the .f32 path, or None."""
    d = directory or os.environ.get(DUMP_ENV)
    if not d:
        return None
    os.makedirs(d, exist_ok=True)
    safe = re.sub(r"[^A-Za-z0-9_.-]", "_", name)
    path = os.path.join(d, safe + ".f32")
    np.ascontiguousarray(np.asarray(t.data, dtype=np.float32).reshape(-1)).astype("<f4").tofile(path)
    with open(os.path.join(d, safe + ".json"), "w") as f:
        json.dump({"name": name, "shape": [int(x) for x in t.shape], "dtype": t.dtype}, f)
    return path


def read_dump(name: str, directory: str) -> HostTensor:
    """Reads back a tensor written by dump_tensor."""
    safe = re.sub(r"[^A-Za-z0-9_.-]", "_", name)
    with open(os.path.join(directory, safe + ".json")) as f:
        meta = json.load(f)
    data = np.fromfile(os.path.join(directory, safe + ".f32"), dtype="<f4").astype(np.float32)
    return HostTensor(list(meta["shape"]), data, meta["dtype"])


def run_cuda_module(ctx: CudaContext, graph: Graph, shapes, inputs=None, echo: bool = True) -> HostTensor:
    ex = CudaGraphExecutor(ctx, graph, shapes, inputs)
    try:
        out = ex.run()
    finally:
        ex.close()
    dump_tensor("output", out)
    if echo:
        print("\n--- Execution Output ---")
        print(format_tensor(out))
        print("------------------------")
    return out


def backward_cuda_module(ctx: CudaContext, graph: Graph, shapes, inputs=None, echo: bool = True):
    ex = CudaGraphExecutor(ctx, graph, shapes, inputs)
    try:
        grads = ex.backward()
    finally:
        ex.close()
    for name, t in grads:
        dump_tensor(f"{name}_grad", t)
    if echo:
        print("\n--- Gradient Output ---")
        for name, t in grads:
            print(f"{name}:")
            print(format_tensor(t))
        print("-----------------------")
    return grads


def train_cuda_module(ctx: CudaContext, graph: Graph, shapes, inputs=None, parameters=None,
                      echo: bool = True):
    ex = CudaGraphExecutor(ctx, graph, shapes, inputs, parameters)
    try:
        losses = ex.train()
        params = ex.parameters()
    finally:
        ex.close()
    dump_tensor("losses", HostTensor([len(losses)], np.asarray(losses, np.float32)))
    for name, t in params.items():
        flat = np.asarray(t, np.float32).reshape(-1)
        dump_tensor(f"param_{name}", HostTensor([int(flat.size)], flat))
    if echo:
        print("\n--- Training Output ---")
        print("backend=cuda")
        for i, loss in enumerate(losses):
            print(f"step={i + 1} loss={loss:.6f} params={len(params)}")
        print("-----------------------")
    return losses, params
