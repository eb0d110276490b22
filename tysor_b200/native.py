"""ctypes binding of libtysor_cuda.so (include/tysor_cuda.h).

This is the Python mirror of the reference's Rust FFI block
(src/backend/metal/native.rs:14-136): one declaration per exported C
function, plus `check()` which turns a false/NULL return into an exception
carrying tysor_cuda_last_error(), the way native.rs:148-157 does.

There is no fallback: if the library is missing or no sm_100 device is
present, loading or context creation raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_bool, c_char_p, c_double, c_float, c_int, c_int64, c_size_t, c_uint8, c_uint32, c_uint64, c_void_p

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtysor_cuda.so")

V = c_void_p
U32 = c_uint32
U64 = c_uint64
FP = POINTER(c_float)
I64P = POINTER(c_int64)
U8P = POINTER(c_uint8)

SIGNATURES = {
    "tysor_cuda_last_error": (c_char_p, []),
    "tysor_cuda_context_new": (V, [c_int]),
    "tysor_cuda_context_free": (None, [V]),
    "tysor_cuda_synchronize": (c_bool, [V]),
    "tysor_cuda_set_matmul_mode": (c_bool, [V, c_int]),
    "tysor_cuda_context_stream": (V, [V]),
    "tysor_cuda_probe_wait_timeout": (c_bool, [V, c_int64]),
    "tysor_cuda_set_matmul_accumulation": (c_bool, [V, c_int]),
    "tysor_cuda_buffer_new_with_data": (V, [V, FP, c_size_t]),
    "tysor_cuda_buffer_new_zeroed": (V, [V, c_size_t]),
    "tysor_cuda_buffer_free": (None, [V]),
    "tysor_cuda_buffer_read": (c_bool, [V, FP, c_size_t]),
    "tysor_cuda_buffer_write": (c_bool, [V, FP, c_size_t]),
    "tysor_cuda_buffer_view": (V, [V, c_size_t, c_size_t]),
    "tysor_cuda_buffer_count": (c_size_t, [V]),
    "tysor_cuda_dispatch_matmul": (c_bool, [V, V, V, V, U32, U32, U32]),
    "tysor_cuda_dispatch_unary": (c_bool, [V, c_int, V, V, U32, c_float]),
    "tysor_cuda_dispatch_binary_tt": (c_bool, [V, c_int, V, V, V, U32]),
    "tysor_cuda_dispatch_binary_ts": (c_bool, [V, c_int, V, V, U32, c_double]),
    "tysor_cuda_dispatch_binary_st": (c_bool, [V, c_int, V, V, U32, c_double]),
    "tysor_cuda_dispatch_rms_norm": (c_bool, [V, V, V, U32, U32]),
    "tysor_cuda_dispatch_softmax": (c_bool, [V, V, V, U32, U32]),
    "tysor_cuda_dispatch_cross_entropy": (c_bool, [V, V, V, V, U32, U32]),
    "tysor_cuda_dispatch_linear": (c_bool, [V, V, V, V, V, U32, U32, U32, c_bool]),
    "tysor_cuda_dispatch_embedding": (c_bool, [V, V, V, V, U32, U32, U32]),
    "tysor_cuda_dispatch_repeat_kv": (c_bool, [V, V, V, U32, U32, U32, U32]),
    "tysor_cuda_dispatch_causal_mask": (c_bool, [V, V, V, U32, U32, U32]),
    "tysor_cuda_dispatch_rope": (c_bool, [V, V, V, U32, U32, U32, c_double]),
    "tysor_cuda_dispatch_matmul_ex": (c_bool, [V, U32, U32, U32, U32, V, c_bool, U64, U64, V, c_bool, U64,
                                               U64, V, U64, U64, V, c_float, c_bool, c_bool]),
    "tysor_cuda_dispatch_relu_backward": (c_bool, [V, V, V, V, U64, c_bool]),
    "tysor_cuda_dispatch_silu_backward": (c_bool, [V, V, V, V, U64, c_bool]),
    "tysor_cuda_dispatch_softmax_backward": (c_bool, [V, V, V, V, U64, c_bool]),
    "tysor_cuda_dispatch_cross_entropy_backward": (c_bool, [V, V, V, V, U32, U32, c_bool]),
    "tysor_cuda_dispatch_rope_backward": (c_bool, [V, V, V, U32, U32, U32, c_double, c_bool]),
    "tysor_cuda_dispatch_repeat_kv_backward": (c_bool, [V, V, V, U32, U32, U32, U32, c_bool]),
    "tysor_cuda_dispatch_causal_mask_backward": (c_bool, [V, V, V, U32, U32, U32, c_bool]),
    "tysor_cuda_dispatch_embedding_backward": (c_bool, [V, V, V, V, U32, U32, U32, c_bool]),
    "tysor_cuda_dispatch_bias_grad": (c_bool, [V, V, V, U32, U32, c_bool]),
    "tysor_cuda_dispatch_add_inplace": (c_bool, [V, V, V, U64]),
    "tysor_cuda_dispatch_sgd_update": (c_bool, [V, V, V, U64, c_double]),
    "tysor_cuda_dispatch_reduce_sum": (c_bool, [V, V, V, U64]),
    "tysor_cuda_dispatch_rms_norm_gain": (c_bool, [V, V, V, V, U32, U32, c_float]),
    "tysor_cuda_dispatch_rms_norm_gain_backward": (c_bool, [V, V, V, V, V, V, U32, U32, c_float, c_bool]),
    "tysor_cuda_dispatch_cross_entropy_labels": (c_bool, [V, V, V, V, U32, U32]),
    "tysor_cuda_dispatch_cross_entropy_labels_backward": (c_bool, [V, V, V, V, U32, U32, c_bool]),
    "tysor_cuda_dispatch_transpose": (c_bool, [V, V, V, I64P, c_int, c_int, c_int]),
    "tysor_cuda_graph_new": (V, [V, c_char_p]),
    "tysor_cuda_graph_free": (None, [V]),
    "tysor_cuda_graph_set_shape": (c_bool, [V, c_char_p, I64P, c_int]),
    "tysor_cuda_graph_set_input": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_set_parameter": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_upload_input": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_prefetch_input": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_run": (c_bool, [V]),
    "tysor_cuda_graph_backward": (c_bool, [V]),
    "tysor_cuda_graph_train": (c_bool, [V, c_int, c_double, FP]),
    "tysor_cuda_graph_train_enqueue": (c_bool, [V, c_int, c_double, FP]),
    "tysor_cuda_graph_train_traced": (c_bool, [V, c_double, FP, c_int, POINTER(c_int)]),
    "tysor_cuda_graph_trace_label": (c_char_p, [V, c_int]),
    "tysor_cuda_graph_value_rank": (c_int, [V, c_int]),
    "tysor_cuda_graph_value_shape": (c_bool, [V, c_int, I64P]),
    "tysor_cuda_graph_read_value": (c_bool, [V, c_int, FP, c_size_t]),
    "tysor_cuda_graph_read_value_grad": (c_bool, [V, c_int, FP, c_size_t]),
    "tysor_cuda_graph_num_parameters": (c_int, [V]),
    "tysor_cuda_graph_parameter_name": (c_char_p, [V, c_int]),
    "tysor_cuda_graph_parameter_count": (c_size_t, [V, c_char_p]),
    "tysor_cuda_graph_read_parameter": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_read_parameter_grad": (c_bool, [V, c_char_p, FP, c_size_t]),
    "tysor_cuda_graph_launch_count": (c_int64, [V]),
    "tysor_cuda_graph_set_capture": (c_bool, [V, c_bool]),
    "tysor_cuda_graph_set_loss_order": (c_bool, [V, c_int]),
    "tysor_cuda_matmul_noalloc": (c_bool, [V, U32, U32, U32, V, V, V]),
    "tysor_cuda_matmul_noalloc_status": (c_bool, [V]),
    "tysor_cuda_nccl_get_unique_id": (c_bool, [U8P]),
    "tysor_cuda_comm_init": (c_bool, [V, c_int, c_int, U8P, c_int]),
    "tysor_cuda_comm_free": (c_bool, [V]),
    "tysor_cuda_allreduce_sum": (c_bool, [V, V, U64]),
    "tysor_cuda_graph_enable_allreduce": (c_bool, [V, c_bool]),
}

_lib = None


class NativeError(RuntimeError):
    """An error reported by libtysor_cuda (tysor_cuda_last_error)."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeError(f"{LIB_PATH} is not built; run `python -m tysor_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().tysor_cuda_last_error()
    return msg.decode() if msg else "unknown tysor_cuda error"


def check(ok, what: str = ""):
    if not ok:
        raise NativeError(f"{what}: {last_error()}" if what else last_error())
    return ok


def fptr(arr):
    """float* of a C-contiguous float32 numpy array."""
    import numpy as np
    assert arr.dtype == np.float32 and arr.flags["C_CONTIGUOUS"]
    return arr.ctypes.data_as(FP)
