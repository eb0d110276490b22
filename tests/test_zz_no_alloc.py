"""tysor_cuda_matmul_noalloc: the strict matmul for callers that cannot
allocate device memory -- a host framework that has reserved the GPU's
memory for its own pool, or a path where cudaMalloc's implicit device
synchronisation is not allowed.

The caller provides A, B and C; the entry point takes its scratch from a
fixed 32 MiB array inside the library.  This file is collected last so that
a run that stops at the first failure has already run every other test, and
it passes both alone in a fresh process and after the rest of the suite.

Checks, each against the oracle's matmul (the sequential fp32 loop of
tensor.rs:163-194) at the strict-matmul tolerance (Frobenius rel 1e-5):
  * two calls in a row of different shapes, each equal to the oracle and to
    the existing entry point (tysor_cuda_dispatch_matmul), so the second is
    not disturbed by what the first left in the shared scratch;
  * M < 256, where A's low part is split into the fixed array (the larger
    shapes build it in shared memory instead);
  * a call whose operands fill the array exactly is accepted, one beyond it
    is rejected with a clear error;
  * tysor_cuda_matmul_noalloc_status reports no recorded kernel error after
    the calls.
"""
import numpy as np
import pytest

import local as L

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 8 * 1024 * 1024


def frob(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_matmul(a, b):
    L.set_threads(16)
    out = L.matmul(L.Tensor(list(a.shape), a.reshape(-1).copy()), L.Tensor(list(b.shape), b.reshape(-1).copy()))
    return out.data.reshape(a.shape[0], b.shape[1])


def existing_entry_point(ctx, a, b):
    from tysor_b200 import native
    from tysor_b200.runtime import DeviceBuffer
    m, k = a.shape
    n = b.shape[1]
    A, B, C = DeviceBuffer.from_array(ctx, a), DeviceBuffer.from_array(ctx, b), DeviceBuffer.zeros(ctx, m * n)
    native.check(native.lib().tysor_cuda_dispatch_matmul(ctx.handle, A.handle, B.handle, C.handle, m, n, k))
    out = C.read().reshape(m, n)
    for buf in (A, B, C):
        buf.free()
    return out


def noalloc_matmul(a, b):
    """Inputs and output in memory the caller owns (here: torch tensors);
    the status query then waits for the stream and reports kernel errors."""
    import torch
    from tysor_b200 import native
    m, k = a.shape
    n = b.shape[1]
    ta = torch.from_numpy(a).cuda()
    tb = torch.from_numpy(b).cuda()
    tc = torch.full((m, n), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ok = native.lib().tysor_cuda_matmul_noalloc(stream, m, n, k, ta.data_ptr(), tb.data_ptr(), tc.data_ptr())
    native.check(ok, "matmul_noalloc")
    native.check(native.lib().tysor_cuda_matmul_noalloc_status(stream), "matmul_noalloc_status")
    return tc.cpu().numpy()


def operands(rng, m, n, k):
    return rng.uniform(-1, 1, (m, k)).astype(np.float32), rng.uniform(-1, 1, (k, n)).astype(np.float32)


def test_noalloc_matches_the_oracle_and_the_existing_entry_point_twice(cuda_ctx):
    rng = np.random.default_rng(11)
    # The second shape differs in size and finds the first call's data in
    # the scratch; the third has M < 256 and splits A into the array.
    for m, n, k in [(512, 768, 1024), (300, 200, 72), (100, 384, 512)]:
        a, b = operands(rng, m, n, k)
        want = oracle_matmul(a, b)
        got = noalloc_matmul(a, b)
        assert np.isfinite(got).all()
        assert frob(got, want) < 1e-5, (m, n, k)
        assert frob(got, existing_entry_point(cuda_ctx, a, b)) < 1e-5, (m, n, k)


def test_noalloc_accepts_operands_that_fill_the_scratch_exactly(cuda_ctx):
    # A (128 x 2048) + B (2048 x 3968) = 262,144 + 8,126,464 = 8,388,608.
    m, n, k = 128, 3968, 2048
    assert m * k + k * n == SCRATCH_FLOATS
    a, b = operands(np.random.default_rng(12), m, n, k)
    for _ in range(2):
        assert frob(noalloc_matmul(a, b), oracle_matmul(a, b)) < 1e-5


def test_noalloc_rejects_operands_beyond_the_fixed_scratch(cuda_ctx):
    import torch
    from tysor_b200 import native
    for m, n, k in [(128, 3972, 2048), (4096, 4096, 2048)]:  # 8,396,800 and 16.8M elements
        ta = torch.zeros((m, k), device="cuda")
        tb = torch.zeros((k, n), device="cuda")
        tc = torch.zeros((m, n), device="cuda")
        ok = native.lib().tysor_cuda_matmul_noalloc(torch.cuda.current_stream().cuda_stream, m, n, k,
                                                   ta.data_ptr(), tb.data_ptr(), tc.data_ptr())
        assert not ok
        assert "scratch holds at most" in native.last_error()
    assert native.lib().tysor_cuda_matmul_noalloc_status(torch.cuda.current_stream().cuda_stream)
