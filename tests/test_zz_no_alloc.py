"""tysor_cuda_matmul_noalloc: the strict matmul for callers that cannot
allocate device memory (a host framework that owns the GPU's memory pool,
or a path where cudaMalloc's device synchronisation is not allowed).

The caller provides A, B and C; the entry point takes its scratch from a
fixed array inside the library.  This file is collected last so that a run
that stops at the first failure has already run every other test, and it
passes both alone in a fresh process and after the rest of the suite.  The
result of two calls in a row must equal the existing entry point's
(tysor_cuda_dispatch_matmul) within the strict-matmul tolerance (Frobenius
rel 1e-5), and the second call must not be disturbed by what the first left
in the shared scratch."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def frob(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def reference_matmul(ctx, a, b):
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
    """Inputs and output in memory the caller owns (here: torch tensors)."""
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
    torch.cuda.synchronize()
    return tc.cpu().numpy()


def test_noalloc_matches_the_existing_entry_point_twice(cuda_ctx):
    rng = np.random.default_rng(11)
    shapes = [(512, 768, 1024), (300, 200, 72)]  # the second differs in size and leaves
    for m, n, k in shapes:                       # the first call's data in the scratch
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        want = reference_matmul(cuda_ctx, a, b)
        got = noalloc_matmul(a, b)
        assert np.isfinite(got).all()
        assert frob(got, want) < 1e-5


def test_noalloc_rejects_operands_beyond_the_fixed_scratch(cuda_ctx):
    import torch
    from tysor_b200 import native
    m, n, k = 4096, 4096, 2048  # A + B = 16.8M elements > 8.4M
    ta = torch.zeros((m, k), device="cuda")
    tb = torch.zeros((k, n), device="cuda")
    tc = torch.zeros((m, n), device="cuda")
    ok = native.lib().tysor_cuda_matmul_noalloc(torch.cuda.current_stream().cuda_stream, m, n, k,
                                               ta.data_ptr(), tb.data_ptr(), tc.data_ptr())
    assert not ok
    assert "scratch holds at most" in native.last_error()
