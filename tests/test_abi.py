"""The C ABI library loads without a GPU and exports every function that
include/tysor_cuda.h declares; the ctypes table covers the same set."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tysor_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tysor_cuda_\w+)\s*\(", text)))


def test_header_declares_the_metal_bridge_surface():
    names = declared_functions()
    # native.rs:14-136 binds these 16 Metal entry points; each has a CUDA twin.
    metal = ["last_error", "context_new", "context_free", "buffer_new_with_data", "buffer_new_zeroed",
             "buffer_free", "buffer_read", "dispatch_matmul", "dispatch_unary", "dispatch_binary_tt",
             "dispatch_binary_ts", "dispatch_binary_st", "dispatch_rms_norm", "dispatch_softmax",
             "dispatch_cross_entropy", "dispatch_linear", "dispatch_embedding", "dispatch_repeat_kv",
             "dispatch_causal_mask", "dispatch_rope"]
    for m in metal:
        assert "tysor_cuda_" + m in names


def test_library_exports_every_declared_symbol():
    from tysor_b200 import build, native
    if not os.path.exists(native.LIB_PATH):
        build.build()
    lib = ctypes.CDLL(native.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from tysor_b200 import native
    assert sorted(native.SIGNATURES) == declared_functions()


def test_no_gpu_means_a_loud_error():
    """Without a device, context creation fails with a message; nothing
    silently falls back to the CPU."""
    import torch
    if torch.cuda.is_available():
        return
    from tysor_b200 import native
    lib = native.lib()
    assert lib.tysor_cuda_context_new(0) is None
    assert native.last_error()
