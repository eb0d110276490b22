"""tcgen05 matmul through the C ABI against the oracle's sequential f32
matmul (runtime/tensor.rs:163-194).

Tolerances (Frobenius-relative): strict 3xTF32 1e-5, fast 1xTF32 2e-3;
the CUDA-core path (exact mode, and shapes that break TMA alignment) must be
bit-identical to the oracle."""
import numpy as np
import pytest

import local as L

pytestmark = pytest.mark.gpu


def frob(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_mm(a, b):
    m, k = a.shape
    n = b.shape[1]
    t = L.matmul(L.Tensor([m, k], np.ascontiguousarray(a, np.float32).reshape(-1)),
                 L.Tensor([k, n], np.ascontiguousarray(b, np.float32).reshape(-1)))
    return t.data.reshape(m, n)


def run_ex(ctx, a_stored, ta, b_stored, tb, m, n, k, batch=1, bias=None, alpha=1.0, acc=None, relu=False):
    from tysor_b200 import native
    from tysor_b200.runtime import DeviceBuffer
    lib = native.lib()
    A = DeviceBuffer.from_array(ctx, a_stored)
    B = DeviceBuffer.from_array(ctx, b_stored)
    C = DeviceBuffer.from_array(ctx, acc) if acc is not None else DeviceBuffer.zeros(ctx, batch * m * n)
    Bi = DeviceBuffer.from_array(ctx, bias) if bias is not None else None
    lda = a_stored.shape[-1]
    ldb = b_stored.shape[-1]
    sa = a_stored.shape[-2] * lda if batch > 1 else 0
    sb = b_stored.shape[-2] * ldb if batch > 1 else 0
    ok = lib.tysor_cuda_dispatch_matmul_ex(ctx.handle, batch, m, n, k, A.handle, ta, lda, sa, B.handle, tb, ldb, sb,
                                           C.handle, n, m * n if batch > 1 else 0,
                                           Bi.handle if Bi else None, alpha, acc is not None, relu)
    native.check(ok, "matmul_ex")
    out = C.read().reshape(batch, m, n) if batch > 1 else C.read().reshape(m, n)
    for buf in (A, B, C, Bi):
        if buf:
            buf.free()
    return out


SHAPES = [(128, 256, 64), (300, 200, 72), (257, 130, 36), (64, 48, 16), (1000, 1000, 1000)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
def test_strict_matmul_layouts(cuda_ctx, m, n, k, ta, tb):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    want = oracle_mm(a, b)
    got = run_ex(cuda_ctx, np.ascontiguousarray(a.T) if ta else a, ta,
                 np.ascontiguousarray(b.T) if tb else b, tb, m, n, k)
    assert frob(got, want) < 1e-5


def test_matmul_relu_2048_strict(cuda_ctx):
    """The matmul+relu program at x, w fp32 [2048, 2048], U[-1, 1]."""
    from tysor_b200.runtime import DeviceBuffer
    from tysor_b200 import native
    rng0, rng1 = np.random.default_rng(0), np.random.default_rng(1)
    x = rng0.uniform(-1, 1, (2048, 2048)).astype(np.float32)
    w = rng1.uniform(-1, 1, (2048, 2048)).astype(np.float32)
    L.set_threads(8)
    want = np.maximum(oracle_mm(x, w), 0)
    got = run_ex(cuda_ctx, x, False, w, False, 2048, 2048, 2048, relu=True)
    assert frob(got, want) < 1e-5


def test_fast_mode_tolerance(cuda_ctx):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (512, 1024)).astype(np.float32)
    b = rng.uniform(-1, 1, (1024, 384)).astype(np.float32)
    want = oracle_mm(a, b)
    cuda_ctx.set_matmul_mode("fast")
    try:
        got = run_ex(cuda_ctx, a, False, b, False, 512, 384, 1024)
    finally:
        cuda_ctx.set_matmul_mode("strict")
    err = frob(got, want)
    assert 1e-7 < err < 2e-3


def test_exact_mode_is_bit_exact(cuda_ctx):
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (70, 50)).astype(np.float32)
    b = rng.uniform(-1, 1, (50, 33)).astype(np.float32)
    cuda_ctx.set_matmul_mode("exact")
    try:
        got = run_ex(cuda_ctx, a, False, b, False, 70, 33, 50)
    finally:
        cuda_ctx.set_matmul_mode("strict")
    np.testing.assert_array_equal(got, oracle_mm(a, b))


def test_unaligned_shapes_use_exact_path(cuda_ctx):
    rng = np.random.default_rng(7)
    a = rng.uniform(-1, 1, (5, 3)).astype(np.float32)
    b = rng.uniform(-1, 1, (3, 7)).astype(np.float32)
    got = run_ex(cuda_ctx, a, False, b, False, 5, 7, 3)
    np.testing.assert_array_equal(got, oracle_mm(a, b))


def test_batched_and_epilogue(cuda_ctx):
    rng = np.random.default_rng(8)
    bt, m, n, k = 3, 130, 96, 64
    a = rng.uniform(-1, 1, (bt, m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (bt, k, n)).astype(np.float32)
    c0 = rng.uniform(-1, 1, (bt, m, n)).astype(np.float32)
    got = run_ex(cuda_ctx, a, False, b, False, m, n, k, batch=bt, alpha=0.5, acc=c0)
    for i in range(bt):
        prod = oracle_mm(a[i], b[i])
        want = c0[i] + prod * np.float32(0.5)
        assert frob(got[i], want) < 1e-5


def test_bias_epilogue(cuda_ctx):
    rng = np.random.default_rng(9)
    a = rng.uniform(-1, 1, (200, 96)).astype(np.float32)
    b = rng.uniform(-1, 1, (96, 300)).astype(np.float32)
    bias = rng.uniform(-1, 1, 300).astype(np.float32)
    got = run_ex(cuda_ctx, a, False, b, False, 200, 300, 96, bias=bias)
    assert frob(got, oracle_mm(a, b) + bias) < 1e-5


def test_dispatch_matmul_metal_signature(cuda_ctx):
    """tysor_cuda_dispatch_matmul has the Metal bridge's argument order."""
    from tysor_b200 import native
    from tysor_b200.runtime import DeviceBuffer
    x = L.synthetic([2, 3]).data.reshape(2, 3)
    w = L.synthetic([3, 4]).data.reshape(3, 4)
    X, W, O = DeviceBuffer.from_array(cuda_ctx, x), DeviceBuffer.from_array(cuda_ctx, w), DeviceBuffer.zeros(cuda_ctx, 8)
    native.check(native.lib().tysor_cuda_dispatch_matmul(cuda_ctx.handle, X.handle, W.handle, O.handle, 2, 4, 3))
    np.testing.assert_array_equal(O.read().reshape(2, 4), oracle_mm(x, w))


def test_one_sm_kernel_when_the_pair_form_is_off():
    """The 1-SM (cta_group::1) form, selected with TYSOR_CUDA_GEMM_2SM=0
    (the cluster-pair form is the default for 256-column tiles), against the
    oracle for both operand layouts; run in a child process because the
    switch is read at load time."""
    import os
    import subprocess
    import sys
    code = r'''
import sys, numpy as np
sys.path[:0] = [".", "oracle"]
import local as L
from tysor_b200 import native
from tysor_b200.runtime import CudaContext, DeviceBuffer
ctx = CudaContext(0)
lib = native.lib()
rng = np.random.default_rng(4)
for (m, n, k, ta, tb) in [(512, 512, 256, False, False), (640, 768, 96, False, True), (300, 520, 64, True, False)]:
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    A = DeviceBuffer.from_array(ctx, np.ascontiguousarray(a.T) if ta else a)
    B = DeviceBuffer.from_array(ctx, np.ascontiguousarray(b.T) if tb else b)
    C = DeviceBuffer.zeros(ctx, m * n)
    native.check(lib.tysor_cuda_dispatch_matmul_ex(ctx.handle, 1, m, n, k, A.handle, ta, m if ta else k, 0,
                 B.handle, tb, k if tb else n, 0, C.handle, n, 0, None, 1.0, False, False))
    got = C.read().reshape(m, n).astype(np.float64)
    want = L.matmul(L.Tensor([m, k], a.reshape(-1).copy()), L.Tensor([k, n], b.reshape(-1).copy())).data.reshape(m, n)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 1e-5, (m, n, k, ta, tb, err)
print("ok")
'''
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, TYSOR_CUDA_GEMM_2SM="0")
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("ta,tb", [(False, True), (True, False), (False, False)])
def test_persistent_pair_kernel_many_tiles_per_cluster(cuda_ctx, ta, tb):
    """Shapes with several 256-row tiles per resident cluster (the persistent
    schedule), both B tile widths (N > 128 and N <= 128, the latter with B's
    parts stacked, including N not a multiple of 32), batched, with the
    accumulate / alpha / bias epilogue."""
    rng = np.random.default_rng(11)
    for (bt, m, n, k) in [(3, 1024, 1000, 200), (2, 2048, 128, 336), (2, 520, 100, 88), (2, 768, 40, 64)]:
        a = rng.uniform(-1, 1, (bt, m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (bt, k, n)).astype(np.float32)
        c0 = rng.uniform(-1, 1, (bt, m, n)).astype(np.float32)
        a_st = np.ascontiguousarray(a.transpose(0, 2, 1)) if ta else a
        b_st = np.ascontiguousarray(b.transpose(0, 2, 1)) if tb else b
        got = run_ex(cuda_ctx, a_st, ta, b_st, tb, m, n, k, batch=bt, alpha=0.75, acc=c0)
        for i in range(bt):
            want = c0[i] + oracle_mm(a[i], b[i]) * np.float32(0.75)
            assert frob(got[i], want) < 1e-5, (bt, m, n, k, i)


@pytest.mark.parametrize("switch", ["TYSOR_CUDA_GEMM_CONV_A", "TYSOR_CUDA_GEMM_STACK_B", "TYSOR_CUDA_GEMM_PERSISTENT"])
def test_gemm_form_opt_outs(switch):
    """Each opt-out (A's low part from a split pass instead of shared memory;
    B's parts in three MMAs instead of stacked; the non-persistent pair
    kernel) against the oracle on N > 128 and N <= 128 shapes, in a child
    process because the switches are read at load time."""
    import os
    import subprocess
    import sys
    code = r'''
import sys, numpy as np
sys.path[:0] = [".", "oracle"]
import local as L
from tysor_b200 import native
from tysor_b200.runtime import CudaContext, DeviceBuffer
ctx = CudaContext(0)
lib = native.lib()
rng = np.random.default_rng(5)
for (m, n, k, ta, tb) in [(1024, 512, 256, False, True), (768, 128, 320, True, False), (512, 72, 96, False, False)]:
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    A = DeviceBuffer.from_array(ctx, np.ascontiguousarray(a.T) if ta else a)
    B = DeviceBuffer.from_array(ctx, np.ascontiguousarray(b.T) if tb else b)
    C = DeviceBuffer.zeros(ctx, m * n)
    native.check(lib.tysor_cuda_dispatch_matmul_ex(ctx.handle, 1, m, n, k, A.handle, ta, m if ta else k, 0,
                 B.handle, tb, k if tb else n, 0, C.handle, n, 0, None, 1.0, False, False))
    got = C.read().reshape(m, n).astype(np.float64)
    want = L.matmul(L.Tensor([m, k], a.reshape(-1).copy()), L.Tensor([k, n], b.reshape(-1).copy())).data.reshape(m, n)
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 1e-5, (m, n, k, ta, tb, err)
print("ok")
'''
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, **{switch: "0"})
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
