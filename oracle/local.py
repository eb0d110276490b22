"""CPU oracle: a Python restatement of the reference `local` backend's three
executors, calling the C op library in tysor_local.c for all tensor math.

TEST INFRASTRUCTURE ONLY.  The product package (tysor_b200/) never imports
this module; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
use it as the checker.

  run_forward         <- src/runtime/graph_executor.rs:96-356   (--run)
  compute_value_grads <- src/training/backward.rs:145-380       (--backward)
  train               <- src/training/executor.rs:252-816       (--train)

Extensions with no reference counterpart (batched matmul, `transpose`,
`RMSNorm` with gain, cross_entropy against class labels) are restated here
too, so the CUDA backend has a CPU check for them; where the reference would
raise for such a program, it still raises unless the program uses one of
the extensions.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libtysor_oracle.so")
# The f64 twin of the C library (tysor_local.c built with TL_F64): the same
# algorithm in double precision, used only to measure errors against a
# nearly exact answer (precision(64)).
_LIB64_PATH = os.path.join(_HERE, "libtysor_oracle64.so")
_libs: Dict[int, ctypes.CDLL] = {}
_bits = 32

OPS = {"+": 0, "-": 1, "*": 2, "/": 3}


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    """The C op library of the current precision (f32 unless precision(64))."""
    if _bits not in _libs:
        path = _LIB64_PATH if _bits == 64 else _LIB_PATH
        if not os.path.exists(path):
            build()
        _lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I = ctypes.c_int64
        D = ctypes.c_double
        F = ctypes.c_float
        sig = {
            "tl_set_threads": (None, [ctypes.c_int]),
            "tl_synthetic": (None, [P, I]),
            "tl_linear_weight_init": (None, [P, I]),
            "tl_linear_bias_init": (None, [P, I]),
            "tl_embedding_weight_init": (None, [P, I]),
            "tl_backward_fake_weight": (None, [P, I]),
            "tl_binary_tt": (None, [ctypes.c_int, P, P, P, I]),
            "tl_binary_ts": (None, [ctypes.c_int, P, D, P, I]),
            "tl_binary_st": (None, [ctypes.c_int, D, P, P, I]),
            "tl_negate": (None, [P, P, I]),
            "tl_add_in_place": (None, [P, P, I]),
            "tl_relu": (None, [P, P, I]),
            "tl_relu_backward": (None, [P, P, P, I]),
            "tl_silu": (None, [P, P, I]),
            "tl_silu_backward": (None, [P, P, P, I]),
            "tl_dropout": (ctypes.c_int, [P, D, P, I]),
            "tl_matmul": (None, [P, P, P, I, I, I]),
            "tl_transpose2d": (None, [P, P, I, I]),
            "tl_bias_add": (None, [P, P, I, I]),
            "tl_softmax": (None, [P, P, I, I]),
            "tl_softmax_backward": (None, [P, P, P, I]),
            "tl_rms_norm": (None, [P, P, I, I]),
            "tl_rms_norm_gain": (None, [P, P, P, I, I, F]),
            "tl_rms_norm_gain_backward": (None, [P, P, P, P, P, I, I, F]),
            "tl_cross_entropy": (None, [P, P, P, I, I]),
            "tl_cross_entropy_backward": (None, [P, P, P, I, I]),
            "tl_cross_entropy_labels": (ctypes.c_int, [P, P, P, I, I]),
            "tl_cross_entropy_labels_backward": (ctypes.c_int, [P, P, P, I, I]),
            "tl_embedding": (ctypes.c_int, [P, P, P, I, I, I]),
            "tl_embedding_backward": (None, [P, P, P, I, I, I]),
            "tl_repeat_kv": (None, [P, P, I, I, I, I]),
            "tl_repeat_kv_backward": (None, [P, P, I, I, I, I]),
            "tl_causal_mask": (None, [P, P, I, I, I]),
            "tl_causal_mask_backward": (None, [P, P, I, I, I]),
            "tl_rope": (None, [P, P, I, I, I, D]),
            "tl_rope_backward": (None, [P, P, I, I, I, D]),
            "tl_transpose": (None, [P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
            "tl_bias_grad": (None, [P, P, I, I]),
            "tl_sgd": (None, [P, P, D, I]),
            "tl_sum": (D, [P, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib.tl_set_threads(_threads)
        _libs[_bits] = _lib
    return _libs[_bits]


_threads = 1


def set_threads(n: int) -> None:
    global _threads
    _threads = int(n)
    for handle in _libs.values():
        handle.tl_set_threads(_threads)


def _dt():
    """numpy dtype of tensor data at the current precision."""
    return np.float64 if _bits == 64 else np.float32


class precision:
    """`with precision(64):` runs the oracle in f64 (the same loops in double;
    tensors hold float64 data) -- an error-budget reference, not the
    reference's own arithmetic."""

    def __init__(self, bits: int):
        if bits not in (32, 64):
            raise ValueError("precision is 32 or 64 bits")
        self.bits = bits

    def __enter__(self):
        global _bits
        self._saved, _bits = _bits, self.bits
        return self

    def __exit__(self, *exc):
        global _bits
        _bits = self._saved


def _p(a: np.ndarray):
    assert a.dtype == _dt() and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return max(n, 1)


@dataclass
class Tensor:
    """runtime/tensor.rs:3-18 SimpleTensor: shape + flat f32 data (+ dtype string)."""
    shape: List[int]
    data: np.ndarray
    dtype: str = "float32"

    def clone(self) -> "Tensor":
        return Tensor(list(self.shape), self.data.copy(), self.dtype)


def _new(shape, dtype="float32") -> Tensor:
    return Tensor(list(shape), np.zeros(_numel(shape), dtype=_dt()), dtype)


class OracleError(RuntimeError):
    pass


# ---- op library (tensor.rs / layers.rs) -----------------------------------

def synthetic(shape, dtype="float32") -> Tensor:
    t = _new(shape, dtype)
    lib().tl_synthetic(_p(t.data), t.data.size)
    return t


def linear_weight(i, o, dtype="float32") -> Tensor:
    t = _new([i, o], dtype)
    lib().tl_linear_weight_init(_p(t.data), t.data.size)
    return t


def linear_bias(o, dtype="float32") -> Tensor:
    t = _new([o], dtype)
    lib().tl_linear_bias_init(_p(t.data), t.data.size)
    return t


def embedding_weight(n, d, dtype="float32") -> Tensor:
    t = _new([n, d], dtype)
    lib().tl_embedding_weight_init(_p(t.data), t.data.size)
    return t


def backward_fake_weight(i, o, dtype="float32") -> Tensor:
    t = _new([i, o], dtype)
    lib().tl_backward_fake_weight(_p(t.data), t.data.size)
    return t


def ones_gain(n) -> Tensor:
    return Tensor([n], np.ones(n, dtype=_dt()))


def binary_tt(op, a: Tensor, b: Tensor) -> Tensor:
    if a.shape != b.shape:
        raise OracleError("tensor shape mismatch")
    out = _new(a.shape, a.dtype)
    lib().tl_binary_tt(OPS[op], _p(a.data), _p(b.data), _p(out.data), out.data.size)
    return out


def binary_ts(op, a: Tensor, s: float) -> Tensor:
    out = _new(a.shape, a.dtype)
    lib().tl_binary_ts(OPS[op], _p(a.data), float(s), _p(out.data), out.data.size)
    return out


def binary_st(op, s: float, b: Tensor) -> Tensor:
    out = _new(b.shape, b.dtype)
    lib().tl_binary_st(OPS[op], float(s), _p(b.data), _p(out.data), out.data.size)
    return out


def negate(a: Tensor) -> Tensor:
    out = _new(a.shape, a.dtype)
    lib().tl_negate(_p(a.data), _p(out.data), out.data.size)
    return out


def add_in_place(dst: Tensor, src: Tensor) -> None:
    if dst.shape != src.shape:
        raise OracleError("tensor shape mismatch")
    lib().tl_add_in_place(_p(dst.data), _p(src.data), dst.data.size)


def relu(a: Tensor) -> Tensor:
    out = _new(a.shape, a.dtype)
    lib().tl_relu(_p(a.data), _p(out.data), out.data.size)
    return out


def relu_backward(out_act: Tensor, grad: Tensor) -> Tensor:
    if out_act.shape != grad.shape:
        raise OracleError("tensor shape mismatch")
    out = _new(grad.shape, grad.dtype)
    lib().tl_relu_backward(_p(out_act.data), _p(grad.data), _p(out.data), out.data.size)
    return out


def silu(a: Tensor) -> Tensor:
    out = _new(a.shape, a.dtype)
    lib().tl_silu(_p(a.data), _p(out.data), out.data.size)
    return out


def silu_backward(x: Tensor, grad: Tensor) -> Tensor:
    if x.shape != grad.shape:
        raise OracleError("backward_silu shape mismatch")
    out = _new(x.shape, x.dtype)
    lib().tl_silu_backward(_p(x.data), _p(grad.data), _p(out.data), out.data.size)
    return out


def dropout(a: Tensor, p: float) -> Tensor:
    out = _new(a.shape, a.dtype)
    if lib().tl_dropout(_p(a.data), float(p), _p(out.data), out.data.size) != 0:
        raise OracleError("dropout probability must be in [0, 1)")
    return out


def _batch_dims(a: Tensor, b: Tensor):
    if len(a.shape) < 2 or len(b.shape) < 2:
        raise OracleError("matmul currently requires rank-2 tensors")
    if len(a.shape) != len(b.shape) or a.shape[:-2] != b.shape[:-2]:
        raise OracleError("matmul currently requires rank-2 tensors")
    return a.shape[:-2]


def matmul(a: Tensor, b: Tensor) -> Tensor:
    """tensor.rs:163-194 for rank 2; rank >= 3 with equal leading dims is the
    batched extension (one rank-2 product per leading index)."""
    if len(a.shape) == 2 and len(b.shape) == 2:
        batch: List[int] = []
    else:
        batch = _batch_dims(a, b)
    m, k = a.shape[-2], a.shape[-1]
    k2, n = b.shape[-2], b.shape[-1]
    if k != k2:
        raise OracleError(f"matmul inner dimension mismatch: lhs={a.shape} rhs={b.shape}")
    nb = _numel(batch) if batch else 1
    out = _new(list(batch) + [m, n], a.dtype)
    av = a.data.reshape(nb, m * k)
    bv = b.data.reshape(nb, k * n)
    ov = out.data.reshape(nb, m * n)
    for i in range(nb):
        ai = np.ascontiguousarray(av[i])
        bi = np.ascontiguousarray(bv[i])
        oi = np.zeros(m * n, dtype=_dt())
        lib().tl_matmul(_p(ai), _p(bi), _p(oi), m, k, n)
        ov[i] = oi
    return out


def transpose_last2(t: Tensor) -> Tensor:
    """tensor.rs:196-213 transpose_2d (applied per leading index for the
    batched extension)."""
    r, c = t.shape[-2], t.shape[-1]
    lead = t.shape[:-2]
    nb = _numel(lead) if lead else 1
    out = _new(list(lead) + [c, r], t.dtype)
    src = t.data.reshape(nb, r * c)
    dst = out.data.reshape(nb, r * c)
    for i in range(nb):
        si = np.ascontiguousarray(src[i])
        di = np.zeros(r * c, dtype=_dt())
        lib().tl_transpose2d(_p(si), _p(di), r, c)
        dst[i] = di
    return out


def transpose(t: Tensor, a: int, b: int) -> Tensor:
    rank = len(t.shape)
    a = a + rank if a < 0 else a
    b = b + rank if b < 0 else b
    if not (0 <= a < rank and 0 <= b < rank):
        raise OracleError("transpose axis out of range")
    dims = (ctypes.c_int64 * rank)(*t.shape)
    shape = list(t.shape)
    shape[a], shape[b] = shape[b], shape[a]
    out = _new(shape, t.dtype)
    lib().tl_transpose(_p(t.data), _p(out.data), dims, rank, a, b)
    return out


def linear_with_parameters(x: Tensor, w: Tensor, b: Optional[Tensor]) -> Tensor:
    """layers.rs:102-117."""
    out = matmul(x, w)
    if b is not None:
        if len(b.shape) != 1 or b.shape[0] != out.shape[1]:
            raise OracleError("linear bias shape mismatch")
        lib().tl_bias_add(_p(out.data), _p(b.data), out.shape[0], out.shape[1])
    return out


def softmax(x: Tensor) -> Tensor:
    if not x.shape:
        raise OracleError("softmax requires a tensor with at least one dimension")
    w = x.shape[-1]
    if w == 0 or x.data.size % w != 0:
        raise OracleError("softmax requires the last dimension to divide the data length")
    out = _new(x.shape, x.dtype)
    lib().tl_softmax(_p(x.data), _p(out.data), x.data.size // w, w)
    return out


def softmax_backward(y: Tensor, grad: Tensor) -> Tensor:
    if y.shape != grad.shape:
        raise OracleError("backward_softmax shape mismatch")
    out = _new(y.shape, y.dtype)
    lib().tl_softmax_backward(_p(y.data), _p(grad.data), _p(out.data), out.data.size)
    return out


def rms_norm(x: Tensor, hidden: int) -> Tensor:
    if not x.shape or x.shape[-1] != hidden:
        raise OracleError(f"rms_norm hidden size mismatch: expected {hidden}, got {x.shape}")
    out = _new(x.shape, x.dtype)
    lib().tl_rms_norm(_p(x.data), _p(out.data), x.data.size // hidden, hidden)
    return out


def rms_norm_gain(x: Tensor, g: Tensor, eps: float) -> Tensor:
    h = x.shape[-1]
    if g.shape != [h]:
        raise OracleError("RMSNorm gain shape mismatch")
    out = _new(x.shape, x.dtype)
    lib().tl_rms_norm_gain(_p(x.data), _p(g.data), _p(out.data), x.data.size // h, h, eps)
    return out


def rms_norm_gain_backward(x: Tensor, g: Tensor, dy: Tensor, eps: float):
    h = x.shape[-1]
    dx = _new(x.shape, x.dtype)
    dg = _new([h], x.dtype)
    lib().tl_rms_norm_gain_backward(_p(x.data), _p(g.data), _p(dy.data), _p(dx.data), _p(dg.data),
                                    x.data.size // h, h, eps)
    return dx, dg


def _ce_is_labels(logits: Tensor, target: Tensor) -> bool:
    rows = logits.data.size // max(logits.shape[-1], 1)
    return target.shape != logits.shape and target.data.size == rows


def cross_entropy(logits: Tensor, target: Tensor) -> Tensor:
    """layers.rs:301-324 (dense target); class-label target is the extension."""
    w = logits.shape[-1] if logits.shape else 1
    rows = logits.data.size // max(w, 1)
    out = _new([rows, 1], logits.dtype)
    if _ce_is_labels(logits, target):
        if lib().tl_cross_entropy_labels(_p(logits.data), _p(target.data), _p(out.data), rows, w):
            raise OracleError("cross_entropy label out of range")
        return out
    if logits.shape != target.shape:
        raise OracleError("cross_entropy requires logits and target to have identical shapes")
    lib().tl_cross_entropy(_p(logits.data), _p(target.data), _p(out.data), rows, w)
    return out


def cross_entropy_backward(logits: Tensor, target: Tensor) -> Tensor:
    w = logits.shape[-1]
    rows = logits.data.size // w
    out = _new(logits.shape, logits.dtype)
    if _ce_is_labels(logits, target):
        if lib().tl_cross_entropy_labels_backward(_p(logits.data), _p(target.data), _p(out.data),
                                                  rows, w):
            raise OracleError("cross_entropy label out of range")
        return out
    if logits.shape != target.shape:
        raise OracleError("backward_cross_entropy_logits shape mismatch")
    lib().tl_cross_entropy_backward(_p(logits.data), _p(target.data), _p(out.data), rows, w)
    return out


def embedding(idx: Tensor, w: Tensor, num: int, dim: int) -> Tensor:
    if w.shape != [num, dim]:
        raise OracleError("embedding weight shape mismatch")
    out = _new(list(idx.shape) + [dim], w.dtype)
    if lib().tl_embedding(_p(idx.data), _p(w.data), _p(out.data), idx.data.size, num, dim):
        raise OracleError("Embedding index out of range")
    return out


def embedding_backward(grad: Tensor, idx: Tensor, num: int, dim: int) -> Tensor:
    out = _new([num, dim], grad.dtype)
    lib().tl_embedding_backward(_p(grad.data), _p(idx.data), _p(out.data), idx.data.size, num, dim)
    return out


def reshape(x: Tensor, shape: List[int]) -> Tensor:
    """layers.rs:162-171."""
    if x.data.size != int(np.prod(shape, dtype=np.int64)):
        raise OracleError("reshape requires matching element counts")
    return Tensor(list(shape), x.data.copy(), x.dtype)


def repeat_kv(x: Tensor, repeats: int) -> Tensor:
    if repeats <= 0:
        raise OracleError("repeat_kv repeats must be positive")
    if len(x.shape) < 2:
        raise OracleError("repeat_kv expects rank >= 2")
    shape = list(x.shape)
    shape[1] *= repeats
    inner = _numel(x.shape[2:]) if len(x.shape) > 2 else 1
    out = _new(shape, x.dtype)
    lib().tl_repeat_kv(_p(x.data), _p(out.data), x.shape[0], x.shape[1], inner, repeats)
    return out


def repeat_kv_backward(grad: Tensor, x: Tensor, repeats: int) -> Tensor:
    if repeats <= 0:
        raise OracleError("repeat_kv backward requires repeats > 0")
    if len(x.shape) < 2 or len(grad.shape) != len(x.shape):
        raise OracleError("repeat_kv backward expects matching ranks >= 2")
    inner = _numel(x.shape[2:]) if len(x.shape) > 2 else 1
    out = _new(x.shape, grad.dtype)
    lib().tl_repeat_kv_backward(_p(grad.data), _p(out.data), x.shape[0], x.shape[1], inner, repeats)
    return out


def flatten_heads(x: Tensor) -> Tensor:
    if len(x.shape) < 3:
        return x.clone()
    return Tensor(list(x.shape[:-2]) + [x.shape[-2] * x.shape[-1]], x.data.copy(), x.dtype)


def _mask_dims(t: Tensor):
    q, k = t.shape[-2], t.shape[-1]
    return t.data.size // max(q * k, 1), q, k


def causal_mask(x: Tensor) -> Tensor:
    if len(x.shape) < 2:
        raise OracleError("causal_mask expects rank >= 2")
    o, q, k = _mask_dims(x)
    out = _new(x.shape, x.dtype)
    lib().tl_causal_mask(_p(x.data), _p(out.data), o, q, k)
    return out


def causal_mask_backward(grad: Tensor) -> Tensor:
    if len(grad.shape) < 2:
        raise OracleError("causal_mask backward expects rank >= 2")
    o, q, k = _mask_dims(grad)
    out = _new(grad.shape, grad.dtype)
    lib().tl_causal_mask_backward(_p(grad.data), _p(out.data), o, q, k)
    return out


def _rope_dims(t: Tensor, head_dim: int, what: str):
    if not t.shape or t.shape[-1] != head_dim:
        raise OracleError(f"{what} head_dim mismatch")
    if head_dim % 2 != 0:
        raise OracleError("rope requires an even head_dim" if what == "rope"
                          else "rope backward requires even head_dim")
    seq = t.shape[-2] if len(t.shape) >= 2 else t.shape[0]
    outer = t.data.size // (seq * head_dim)
    return outer, seq


def rope(x: Tensor, head_dim: int, theta: float) -> Tensor:
    outer, seq = _rope_dims(x, head_dim, "rope")
    out = _new(x.shape, x.dtype)
    lib().tl_rope(_p(x.data), _p(out.data), outer, seq, head_dim, float(theta))
    return out


def rope_backward(grad: Tensor, head_dim: int, theta: float) -> Tensor:
    outer, seq = _rope_dims(grad, head_dim, "rope backward")
    out = _new(grad.shape, grad.dtype)
    lib().tl_rope_backward(_p(grad.data), _p(out.data), outer, seq, head_dim, float(theta))
    return out


def bias_grad(grad: Tensor) -> Tensor:
    if len(grad.shape) != 2:
        raise OracleError("backward_linear_bias currently requires rank-2 gradients")
    out = _new([grad.shape[1]], grad.dtype)
    lib().tl_bias_grad(_p(grad.data), _p(out.data), grad.shape[0], grad.shape[1])
    return out


def linear_input_grad(grad: Tensor, w: Tensor) -> Tensor:
    """layers.rs:521-523 backward_linear_input = g . W^T."""
    return matmul(grad, transpose_last2(w))


def linear_weight_grad(grad: Tensor, x: Tensor) -> Tensor:
    """layers.rs:525-527 backward_linear_weight = X^T . g."""
    return matmul(transpose_last2(x), grad)


def sgd(p: Tensor, g: Tensor, lr: float) -> None:
    lib().tl_sgd(_p(p.data), _p(g.data), float(lr), p.data.size)


def tensor_sum(t: Tensor) -> float:
    return float(lib().tl_sum(_p(t.data), t.data.size))


# ---- runtime values --------------------------------------------------------

@dataclass
class Closure:
    kind: str                       # linear | embedding | act | rmsnorm
    op: str = ""
    in_features: Optional[int] = None
    out_features: int = 0
    with_bias: bool = True
    num: int = 0
    dim: int = 0
    probability: float = 0.0
    eps: float = 1e-5
    hidden: int = 0
    ctor_id: int = -1


def _num(v) -> float:
    tag, x = v
    if tag == "int":
        return float(x)
    if tag == "float":
        return float(x)
    if tag == "bool":
        return 1.0 if x else 0.0
    raise OracleError("Graph executor expected scalar value")


def _int(v) -> int:
    tag, x = v
    if tag != "int":
        raise OracleError("Graph executor expected integer value")
    return int(x)


def _bool(v) -> bool:
    tag, x = v
    if tag != "bool":
        raise OracleError("Graph executor expected bool value")
    return bool(x)


def _tensor(v) -> Tensor:
    if v is None or v[0] != "tensor":
        raise OracleError("Graph executor expected tensor value")
    return v[1]


def _const_value(node):
    c = node.const
    if isinstance(c, bool):
        return ("bool", c)
    if isinstance(c, int):
        return ("int", c)
    return ("float", float(c))


def _build_ctor(graph, node, values) -> Closure:
    """graph_executor.rs:163-223 and training/executor.rs:152-221."""
    ins = node.inputs
    op = node.op
    if op == "linear":
        cl = Closure("linear", ctor_id=node.output)
        if len(ins) == 1:
            cl.out_features = _int(values[ins[0]])
            return cl
        if len(ins) == 2 and values[ins[1]][0] == "bool":
            cl.out_features = _int(values[ins[0]])
            cl.with_bias = _bool(values[ins[1]])
            return cl
        cl.in_features = _int(values[ins[0]])
        cl.out_features = _int(values[ins[1]])
        if len(ins) == 3:
            cl.with_bias = _bool(values[ins[2]])
        return cl
    if op in ("SiLU", "Softmax"):
        return Closure("act", op=op)
    if op == "Embedding":
        return Closure("embedding", num=_int(values[ins[0]]), dim=_int(values[ins[1]]),
                       ctor_id=node.output)
    if op == "Dropout":
        return Closure("act", op="Dropout", probability=_num(values[ins[0]]))
    if op == "RMSNorm":
        eps = _num(values[ins[1]]) if len(ins) > 1 else 1e-5
        return Closure("rmsnorm", hidden=_int(values[ins[0]]), eps=eps, ctor_id=node.output)
    raise OracleError(f"Unsupported library constructor '{op}'")


def linear_weight_name(i):
    return f"linear_{i}_weight"


def linear_bias_name(i):
    return f"linear_{i}_bias"


def embedding_weight_name(i):
    return f"embedding_{i}_weight"


def rmsnorm_gain_name(i):
    return f"rmsnorm_{i}_gain"


def _binary_forward(node, values):
    lhs, rhs = values[node.inputs[0]], values[node.inputs[1]]
    op = node.binop
    if lhs[0] == "tensor" and rhs[0] == "tensor":
        return ("tensor", binary_tt(op, lhs[1], rhs[1]))
    if lhs[0] == "tensor":
        return ("tensor", binary_ts(op, lhs[1], _num(rhs)))
    if rhs[0] == "tensor":
        return ("tensor", binary_st(op, _num(lhs), rhs[1]))
    a, b = _num(lhs), _num(rhs)
    return ("float", {"+": a + b, "-": a - b, "*": a * b, "/": a / b if b != 0 else float("inf")}[op])


def _library_call_forward(node, values):
    op = node.op
    ins = node.inputs
    if op == "rms_norm":
        return rms_norm(_tensor(values[ins[0]]), _int(values[ins[1]]))
    if op == "cross_entropy":
        return cross_entropy(_tensor(values[ins[0]]), _tensor(values[ins[1]]))
    if op == "reshape":
        return reshape(_tensor(values[ins[0]]), [_int(values[i]) for i in ins[1:]])
    if op == "repeat_kv":
        return repeat_kv(_tensor(values[ins[0]]), _int(values[ins[1]]))
    if op == "flatten_heads":
        return flatten_heads(_tensor(values[ins[0]]))
    if op == "causal_mask":
        return causal_mask(_tensor(values[ins[0]]))
    if op == "rope":
        return rope(_tensor(values[ins[0]]), _int(values[ins[1]]), _num(values[ins[2]]))
    if op == "transpose":
        return transpose(_tensor(values[ins[0]]), _int(values[ins[1]]), _int(values[ins[2]]))
    raise OracleError(f"Unsupported library graph call '{op}'")


def _primitive_forward(node, values):
    op = node.op
    ins = node.inputs
    if op == "matmul":
        return matmul(_tensor(values[ins[0]]), _tensor(values[ins[1]]))
    if op == "relu":
        return relu(_tensor(values[ins[0]]))
    if op == "scale":
        return binary_ts("*", _tensor(values[ins[0]]), _num(values[ins[1]]))
    raise OracleError(f"Unsupported primitive graph op '{op}'")


def _input_tensor(value, shapes, inputs):
    """graph_executor.rs:80-93: the parameter's --shape, pattern data (or the
    given input values) and its annotated dtype string (float32 if none)."""
    dtype = getattr(value, "dtype", "") or "float32"
    if inputs is not None and value.name in inputs:
        arr = np.ascontiguousarray(np.asarray(inputs[value.name], dtype=_dt()).reshape(-1))
        shape = shapes.get(value.name, [arr.size])
        if _numel(shape) != arr.size:
            raise OracleError(f"input '{value.name}' has {arr.size} values, shape {shape}")
        return Tensor(list(shape), arr.copy(), dtype)
    if value.name not in shapes:
        raise OracleError(f"Missing --shape for tensor parameter '{value.name}'")
    return synthetic(shapes[value.name], dtype)


def _forward(graph, shapes, inputs, parameters: Optional[Dict[str, Tensor]]):
    """One forward walk.  parameters=None is the --run/--backward semantics
    (pattern weights created per apply, graph_executor.rs:225-247); a dict is
    the train semantics (lazy named parameters, training/executor.rs:223-250,
    386-421)."""
    values: Dict[int, tuple] = {}
    for v in graph.values:
        if v.is_parameter:
            values[v.id] = ("tensor", _input_tensor(v, shapes, inputs))
    for node in graph.nodes:
        if node.kind == "const":
            val = _const_value(node)
        elif node.kind == "binary":
            val = _binary_forward(node, values)
        elif node.kind == "primitive":
            val = ("tensor", _primitive_forward(node, values))
        elif node.kind == "call" and node.op == "tied_logits":
            val = ("tensor", _tied_logits_forward(node, values, parameters))
        elif node.kind == "call":
            val = ("tensor", _library_call_forward(node, values))
        elif node.kind == "ctor":
            val = ("closure", _build_ctor(graph, node, values))
        elif node.kind == "apply":
            callee = values.get(node.inputs[0])
            x = _tensor(values.get(node.inputs[1]))
            if callee is None or callee[0] != "closure":
                raise OracleError("Unsupported graph apply operation")
            val = ("tensor", _apply_forward(callee[1], x, parameters))
        else:
            raise OracleError(f"unknown node kind {node.kind}")
        values[node.output] = val
    return values


def _tied_weight(cl: "Closure", parameters) -> Tensor:
    """The embedding table an Embedding constructor owns: the named train
    parameter (created on first use, as apply does) or the constant
    pattern of --run."""
    if parameters is None:
        return embedding_weight(cl.num, cl.dim)
    name = embedding_weight_name(cl.ctor_id)
    if name not in parameters:
        parameters[name] = embedding_weight(cl.num, cl.dim)
    return parameters[name]


def _tied_logits_forward(node, values, parameters) -> Tensor:
    """Extension (no reference counterpart): `tied_logits(h, emb)` is the
    tied output projection h . E^T with E the [num, dim] table of the
    Embedding constructor `emb`."""
    x = _tensor(values[node.inputs[0]])
    callee = values.get(node.inputs[1])
    if callee is None or callee[0] != "closure" or callee[1].kind != "embedding":
        raise OracleError("tied_logits expects an Embedding constructor as its second argument")
    cl = callee[1]
    if len(x.shape) != 2 or x.shape[1] != cl.dim:
        raise OracleError(f"tied_logits expects [rows, {cl.dim}] input, got {x.shape}")
    return matmul(x, transpose_last2(_tied_weight(cl, parameters)))


def _apply_forward(cl: Closure, x: Tensor, parameters):
    if cl.kind == "linear":
        if parameters is None:
            # layers.rs:77-100 apply_linear: pattern weights, rank-2 input.
            if len(x.shape) != 2:
                raise OracleError("linear currently requires rank-2 input tensors")
            inf = cl.in_features if cl.in_features is not None else x.shape[1]
            if x.shape[1] != inf:
                raise OracleError(f"linear expected input feature size {inf}, got {x.shape[1]}")
            w = linear_weight(inf, cl.out_features)
            b = linear_bias(cl.out_features) if cl.with_bias else None
            return linear_with_parameters(x, w, b)
        wname = linear_weight_name(cl.ctor_id)
        inf = cl.in_features if cl.in_features is not None else x.shape[1]
        if wname not in parameters:
            parameters[wname] = linear_weight(inf, cl.out_features)
        b = None
        if cl.with_bias:
            bname = linear_bias_name(cl.ctor_id)
            if bname not in parameters:
                parameters[bname] = linear_bias(cl.out_features)
            b = parameters[bname]
        return linear_with_parameters(x, parameters[wname], b)
    if cl.kind == "embedding":
        if parameters is None:
            w = embedding_weight(cl.num, cl.dim)
        else:
            name = embedding_weight_name(cl.ctor_id)
            if name not in parameters:
                parameters[name] = embedding_weight(cl.num, cl.dim)
            w = parameters[name]
        return embedding(x, w, cl.num, cl.dim)
    if cl.kind == "rmsnorm":
        if not x.shape or x.shape[-1] != cl.hidden:
            raise OracleError(f"rms_norm hidden size mismatch: expected {cl.hidden}, got {x.shape}")
        if parameters is None:
            g = ones_gain(cl.hidden)
        else:
            name = rmsnorm_gain_name(cl.ctor_id)
            if name not in parameters:
                parameters[name] = ones_gain(cl.hidden)
            g = parameters[name]
        return rms_norm_gain(x, g, cl.eps)
    if cl.kind == "act":
        if cl.op == "SiLU":
            return silu(x)
        if cl.op == "Softmax":
            return softmax(x)
        if cl.op == "Dropout":
            return dropout(x, cl.probability)
    raise OracleError("Unsupported graph apply operation")


# ---- --run ------------------------------------------------------------------

def run_forward(graph, shapes, inputs=None):
    """graph_executor.rs:249-356 + interpreter.rs:24-54: returns (output tensor, values)."""
    values = _forward(graph, shapes, inputs, None)
    if not graph.outputs:
        raise OracleError("Entry function did not return a value")
    if len(graph.outputs) != 1:
        raise OracleError("Runtime interpreter currently supports a single return value")
    out = values.get(graph.outputs[0])
    if out is None or out[0] != "tensor":
        raise OracleError("Runtime interpreter only supports tensor returns")
    return out[1], values


# ---- --backward ---------------------------------------------------------------

def _acc(grads: Dict, key, g: Tensor) -> None:
    if key in grads:
        add_in_place(grads[key], g)
    else:
        grads[key] = g.clone()


def compute_value_gradients(graph, shapes, inputs=None):
    """training/backward.rs:145-380.  Returns (values, grads by value id)."""
    values = _forward(graph, shapes, inputs, None)
    oid = graph.objective_id()
    obj = _tensor(values.get(oid))
    grads: Dict[int, Tensor] = {}
    _acc(grads, oid, Tensor(list(obj.shape), np.ones(obj.data.size, dtype=_dt()), obj.dtype))
    for node in reversed(graph.nodes):
        if node.output not in grads:
            continue
        g = grads[node.output].clone()
        if node.kind in ("const", "ctor"):
            continue
        if node.kind == "apply":
            if len(node.inputs) != 2:
                raise OracleError("Graph backward currently supports only single-input apply nodes")
            callee = graph.producer(node.inputs[0])
            if callee is None:
                raise OracleError("Graph backward could not resolve apply callee producer")
            x = _tensor(values.get(node.inputs[1]))
            cl = values[node.inputs[0]][1]
            if callee.op == "linear":
                inf = cl.in_features if cl.in_features is not None else (x.shape[1] if len(x.shape) > 1 else 0)
                w = backward_fake_weight(inf, cl.out_features)
                _acc(grads, node.inputs[1], matmul(g, transpose_last2(w)))
            elif callee.op == "SiLU":
                _acc(grads, node.inputs[1], silu_backward(x, g))
            elif callee.op == "Softmax":
                _acc(grads, node.inputs[1], softmax_backward(_tensor(values[node.output]), g))
            elif callee.op == "Dropout":
                _acc(grads, node.inputs[1], dropout(g, cl.probability))
            elif callee.op == "RMSNorm":
                dx, _ = rms_norm_gain_backward(x, ones_gain(cl.hidden), g, cl.eps)
                _acc(grads, node.inputs[1], dx)
            else:
                raise OracleError("Graph backward does not support this library apply yet")
        elif node.kind == "binary":
            lhs, rhs = values[node.inputs[0]], values[node.inputs[1]]
            op = node.binop
            if lhs[0] == "tensor" and rhs[0] == "tensor":
                if op == "+":
                    _acc(grads, node.inputs[0], g)
                    _acc(grads, node.inputs[1], g)
                elif op == "-":
                    _acc(grads, node.inputs[0], g)
                    _acc(grads, node.inputs[1], negate(g))
                elif op == "*":
                    _acc(grads, node.inputs[0], binary_tt("*", g, rhs[1]))
                    _acc(grads, node.inputs[1], binary_tt("*", g, lhs[1]))
                elif op == "/":
                    rhs_sq = binary_tt("*", rhs[1], rhs[1])
                    num = binary_tt("*", g, lhs[1])
                    _acc(grads, node.inputs[0], binary_tt("/", g, rhs[1]))
                    _acc(grads, node.inputs[1], negate(binary_tt("/", num, rhs_sq)))
            elif lhs[0] == "tensor":
                if op in ("+", "-"):
                    _acc(grads, node.inputs[0], g)
                else:
                    _acc(grads, node.inputs[0], binary_ts(op, g, _num(rhs)))
            elif rhs[0] == "tensor":
                if op == "+":
                    _acc(grads, node.inputs[1], g)
                elif op == "-":
                    _acc(grads, node.inputs[1], negate(g))
                elif op == "*":
                    _acc(grads, node.inputs[1], binary_ts("*", g, _num(lhs)))
                else:
                    raise OracleError("Backward for scalar/tensor division is not implemented yet")
        elif node.kind == "primitive":
            if node.op == "matmul":
                a = _tensor(values[node.inputs[0]])
                b = _tensor(values[node.inputs[1]])
                _acc(grads, node.inputs[0], matmul(g, transpose_last2(b)))
                _acc(grads, node.inputs[1], matmul(transpose_last2(a), g))
            elif node.op == "relu":
                _acc(grads, node.inputs[0], relu_backward(_tensor(values[node.output]), g))
            elif node.op == "scale":
                _acc(grads, node.inputs[0], binary_ts("*", g, _num(values[node.inputs[1]])))
            else:
                raise OracleError(f"Unsupported primitive op '{node.op}' in graph backward")
        elif node.kind == "call":
            if node.op == "rms_norm":
                x = _tensor(values[node.inputs[0]])
                if x.shape != g.shape:
                    raise OracleError("backward_rms_norm_input shape mismatch")
                _acc(grads, node.inputs[0], g)
            elif node.op == "cross_entropy":
                logits = _tensor(values[node.inputs[0]])
                target = _tensor(values[node.inputs[1]])
                _acc(grads, node.inputs[0], cross_entropy_backward(logits, target))
                _acc(grads, node.inputs[1], _new(target.shape, target.dtype))
            elif node.op == "transpose":
                _acc(grads, node.inputs[0],
                     transpose(g, _int(values[node.inputs[1]]), _int(values[node.inputs[2]])))
            else:
                raise OracleError(f"Unsupported library op '{node.op}' in graph backward")
    return values, grads


def backward_report(graph, shapes, inputs=None) -> List[Tuple[str, Tensor]]:
    """backward.rs:382-399: (name_grad, tensor) for each graph parameter."""
    values, grads = compute_value_gradients(graph, shapes, inputs)
    out = []
    for v in graph.values:
        if not v.is_parameter:
            continue
        if v.id in grads:
            out.append((f"{v.name}_grad", grads[v.id]))
        elif v.id in values:
            t = _tensor(values[v.id])
            out.append((f"{v.name}_grad", _new(t.shape, t.dtype)))
    return out


# ---- --train ------------------------------------------------------------------

def compute_parameter_gradients(graph, values, oid, parameters, value_grads=None) -> Dict[str, Tensor]:
    """training/executor.rs:563-743.  If `value_grads` is a dict it receives
    the per-value gradients of the walk as well."""
    obj = _tensor(values.get(oid))
    vgrads: Dict[int, Tensor] = {oid: Tensor(list(obj.shape), np.ones(obj.data.size, _dt()), obj.dtype)}
    pgrads: Dict[str, Tensor] = {}
    for node in reversed(graph.nodes):
        if node.output not in vgrads:
            continue
        g = vgrads[node.output].clone()
        k = node.kind
        if k in ("const", "ctor"):
            continue
        if k == "binary":
            lhs, rhs = values[node.inputs[0]], values[node.inputs[1]]
            op = node.binop
            if lhs[0] == "tensor" and rhs[0] == "tensor":
                if op == "+":
                    _acc(vgrads, node.inputs[0], g)
                    _acc(vgrads, node.inputs[1], g)
                elif op == "-":
                    _acc(vgrads, node.inputs[0], g)
                    _acc(vgrads, node.inputs[1], negate(g))
                elif op == "*":
                    _acc(vgrads, node.inputs[0], binary_tt("*", g, rhs[1]))
                    _acc(vgrads, node.inputs[1], binary_tt("*", g, lhs[1]))
                elif op == "/":
                    _acc(vgrads, node.inputs[0], binary_tt("/", g, rhs[1]))
            elif lhs[0] == "tensor":
                if op in ("+", "-"):
                    _acc(vgrads, node.inputs[0], g)
                else:
                    _acc(vgrads, node.inputs[0], binary_ts(op, g, _num(rhs)))
            elif rhs[0] == "tensor":
                if op == "+":
                    _acc(vgrads, node.inputs[1], g)
                elif op == "-":
                    _acc(vgrads, node.inputs[1], negate(g))
                elif op == "*":
                    _acc(vgrads, node.inputs[1], binary_ts("*", g, _num(lhs)))
        elif k == "primitive":
            if node.op == "matmul":
                a = _tensor(values[node.inputs[0]])
                b = _tensor(values[node.inputs[1]])
                _acc(vgrads, node.inputs[0], matmul(g, transpose_last2(b)))
                _acc(vgrads, node.inputs[1], matmul(transpose_last2(a), g))
            elif node.op == "relu":
                _acc(vgrads, node.inputs[0], relu_backward(_tensor(values[node.output]), g))
            elif node.op == "scale":
                _acc(vgrads, node.inputs[0], binary_ts("*", g, _num(values[node.inputs[1]])))
            else:
                raise OracleError("Unsupported primitive op in train backward")
        elif k == "call":
            op = node.op
            x = values.get(node.inputs[0])
            if op == "rms_norm":
                if _tensor(x).shape != g.shape:
                    raise OracleError("backward_rms_norm_input shape mismatch")
                _acc(vgrads, node.inputs[0], g)
            elif op == "cross_entropy":
                _acc(vgrads, node.inputs[0],
                     cross_entropy_backward(_tensor(x), _tensor(values[node.inputs[1]])))
            elif op in ("reshape", "flatten_heads"):
                xt = _tensor(x)
                if g.data.size != xt.data.size:
                    raise OracleError("reshape backward requires matching element counts")
                _acc(vgrads, node.inputs[0], Tensor(list(xt.shape), g.data.copy(), g.dtype))
            elif op == "repeat_kv":
                _acc(vgrads, node.inputs[0],
                     repeat_kv_backward(g, _tensor(x), _int(values[node.inputs[1]])))
            elif op == "causal_mask":
                _acc(vgrads, node.inputs[0], causal_mask_backward(g))
            elif op == "rope":
                _acc(vgrads, node.inputs[0],
                     rope_backward(g, _int(values[node.inputs[1]]), _num(values[node.inputs[2]])))
            elif op == "transpose":
                _acc(vgrads, node.inputs[0],
                     transpose(g, _int(values[node.inputs[1]]), _int(values[node.inputs[2]])))
            elif op == "tied_logits":
                cl = values[node.inputs[1]][1]
                w = _tied_weight(cl, parameters)
                _acc(vgrads, node.inputs[0], matmul(g, w))
                _acc(pgrads, embedding_weight_name(cl.ctor_id), matmul(transpose_last2(g), _tensor(x)))
        elif k == "apply":
            cl = values[node.inputs[0]][1]
            x = _tensor(values.get(node.inputs[1]))
            if cl.kind == "linear":
                wname = linear_weight_name(cl.ctor_id)
                if wname in parameters:
                    w = parameters[wname]
                else:
                    inf = cl.in_features if cl.in_features is not None else x.shape[1]
                    w = linear_weight(inf, cl.out_features)
                _acc(vgrads, node.inputs[1], linear_input_grad(g, w))
                _acc(pgrads, wname, linear_weight_grad(g, x))
                if cl.with_bias:
                    _acc(pgrads, linear_bias_name(cl.ctor_id), bias_grad(g))
            elif cl.kind == "embedding":
                _acc(pgrads, embedding_weight_name(cl.ctor_id),
                     embedding_backward(g, x, cl.num, cl.dim))
            elif cl.kind == "rmsnorm":
                name = rmsnorm_gain_name(cl.ctor_id)
                gain = parameters[name] if name in parameters else ones_gain(cl.hidden)
                dx, dg = rms_norm_gain_backward(x, gain, g, cl.eps)
                _acc(vgrads, node.inputs[1], dx)
                _acc(pgrads, name, dg)
            elif cl.kind == "act":
                if cl.op == "SiLU":
                    _acc(vgrads, node.inputs[1], silu_backward(x, g))
                elif cl.op == "Softmax":
                    _acc(vgrads, node.inputs[1], softmax_backward(_tensor(values[node.output]), g))
                elif cl.op == "Dropout":
                    _acc(vgrads, node.inputs[1], dropout(g, cl.probability))
                else:
                    raise OracleError("Unsupported activation in train backward")
            else:
                raise OracleError("Unsupported apply in train backward")
    if value_grads is not None:
        value_grads.update(vgrads)
    return pgrads


def apply_sgd(parameters: Dict[str, Tensor], grads: Dict[str, Tensor], lr: float) -> None:
    """training/executor.rs:745-762 (BTreeMap order: sorted names)."""
    for name in sorted(grads):
        if name not in parameters:
            continue
        p = parameters[name]
        if p.shape != grads[name].shape:
            raise OracleError(f"Parameter gradient shape mismatch for '{name}'")
        sgd(p, grads[name], lr)


def train(graph, shapes, inputs=None, parameters: Optional[Dict[str, Tensor]] = None,
          lr: Optional[float] = None, iterations: Optional[int] = None):
    """training/executor.rs:764-816.  Returns (losses, parameters)."""
    if graph.optimizer != "sgd":
        raise OracleError("Train executor currently supports only optimizer='sgd'")
    lr = graph.lr if lr is None else lr
    iterations = graph.iterations if iterations is None else iterations
    oid = graph.objective_id()
    params: Dict[str, Tensor] = {} if parameters is None else {k: v.clone() for k, v in parameters.items()}
    losses = []
    for _ in range(iterations):
        values = _forward(graph, shapes, inputs, params)
        grads = compute_parameter_gradients(graph, values, oid, params)
        losses.append(tensor_sum(_tensor(values[oid])))
        apply_sgd(params, grads, lr)
    return losses, params


def train_step_grads(graph, shapes, inputs=None, parameters=None, value_grads=None):
    """One forward + parameter-gradient pass without the update (used to
    check the device backward in isolation).  Returns (values, grads, params);
    `value_grads`, if a dict, receives the per-value gradients."""
    params: Dict[str, Tensor] = {} if parameters is None else {k: v.clone() for k, v in parameters.items()}
    oid = graph.objective_id()
    values = _forward(graph, shapes, inputs, params)
    grads = compute_parameter_gradients(graph, values, oid, params, value_grads)
    return values, grads, params


# ---- text output (tensor.rs:36-69, executor.rs:794-814) -------------------------

def format_tensor(t: Tensor) -> str:
    """tensor.rs:48-69 print_tensor_body; Rust's `{:.4}` prints every NaN as
    `NaN` and infinities as `inf` / `-inf`."""
    vals = ", ".join("NaN" if float(v) != float(v) else f"{float(v):.4f}" for v in t.data)
    return f"shape=[{', '.join(str(d) for d in t.shape)}] dtype={t.dtype}\nvalues=[{vals}]"
