"""Per-op parity of the bandwidth-bound kernels, through the C ABI, against
the oracle (runtime/tensor.rs, runtime/layers.rs).

Bars: copies, gathers, masks, rotations, updates and exact elementwise
arithmetic are bit-exact; ops with expf/logf or row sums are within
rel 1e-5 (per element, relative to max(|want|, 1)).  The norm / activation /
loss sweep runs at the full sizes: x [65536, 4096], logits [8192, 32000]."""
import ctypes

import numpy as np
import pytest

import local as L

pytestmark = pytest.mark.gpu


def T(shape, arr):
    return L.Tensor(list(shape), np.ascontiguousarray(arr, np.float32).reshape(-1))


def close(got, want, rtol=1e-5):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    err = np.abs(got - want) / np.maximum(np.abs(want), 1.0)
    assert float(err.max(initial=0.0)) <= rtol, float(err.max())


def close_sums(got, want, l1, rtol=1e-5):
    """Sums that cancel are judged against the size of their terms: the
    device (tree order) and the oracle (row order) both round within
    n * 2^-24 * sum|terms|; the bar is rtol * sum|terms| per output."""
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    l1 = np.asarray(l1, np.float64).reshape(-1)
    err = np.abs(got - want) / np.maximum(l1, 1e-30)
    assert float(err.max(initial=0.0)) <= rtol, float(err.max())


@pytest.fixture
def dev(cuda_ctx):
    from tysor_b200 import native
    from tysor_b200.runtime import DeviceBuffer

    class D:
        lib = native.lib()
        ctx = cuda_ctx
        h = cuda_ctx.handle

        @staticmethod
        def buf(a):
            return DeviceBuffer.from_array(cuda_ctx, a)

        @staticmethod
        def zeros(n):
            return DeviceBuffer.zeros(cuda_ctx, n)

        @staticmethod
        def ok(v):
            native.check(v)

    return D


def rnd(shape, seed, lo=-2.0, hi=2.0):
    return np.random.default_rng(seed).uniform(lo, hi, shape).astype(np.float32)


@pytest.mark.parametrize("op,fn", [(1, L.relu), (2, L.silu)])
def test_unary(dev, op, fn):
    x = rnd(10007, 1)
    X, O = dev.buf(x), dev.zeros(x.size)
    dev.ok(dev.lib.tysor_cuda_dispatch_unary(dev.h, op, X.handle, O.handle, x.size, 0.0))
    want = fn(T([x.size], x)).data
    if op == 1:
        np.testing.assert_array_equal(O.read(), want)
    else:
        close(O.read(), want, 1e-6)


@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_binary(dev, op):
    a, b = rnd(4099, 2), rnd(4099, 3, 0.5, 2.0)
    A, B, O = dev.buf(a), dev.buf(b), dev.zeros(a.size)
    sym = "+-*/"[op]
    dev.ok(dev.lib.tysor_cuda_dispatch_binary_tt(dev.h, op, A.handle, B.handle, O.handle, a.size))
    np.testing.assert_array_equal(O.read(), L.binary_tt(sym, T([a.size], a), T([b.size], b)).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_binary_ts(dev.h, op, A.handle, O.handle, a.size, 0.3))
    np.testing.assert_array_equal(O.read(), L.binary_ts(sym, T([a.size], a), 0.3).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_binary_st(dev.h, op, B.handle, O.handle, b.size, 1.7))
    np.testing.assert_array_equal(O.read(), L.binary_st(sym, 1.7, T([b.size], b)).data)


def test_rope_bit_exact(dev):
    shape = (2, 3, 64, 128)
    x = rnd(shape, 4)
    X, O, G = dev.buf(x), dev.zeros(x.size), dev.zeros(x.size)
    outer, seq, half = 6, 64, 64
    dev.ok(dev.lib.tysor_cuda_dispatch_rope(dev.h, X.handle, O.handle, outer, seq, half, 10000.0))
    np.testing.assert_array_equal(O.read(), L.rope(T(shape, x), 128, 10000.0).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_rope_backward(dev.h, X.handle, G.handle, outer, seq, half, 10000.0, False))
    np.testing.assert_array_equal(G.read(), L.rope_backward(T(shape, x), 128, 10000.0).data)


def test_repeat_kv_and_backward_bit_exact(dev):
    shape = (2, 4, 33, 8)
    x = rnd(shape, 5)
    X, O = dev.buf(x), dev.zeros(x.size * 4)
    dev.ok(dev.lib.tysor_cuda_dispatch_repeat_kv(dev.h, X.handle, O.handle, 2, 16, 33 * 8, 4))
    want = L.repeat_kv(T(shape, x), 4)
    np.testing.assert_array_equal(O.read(), want.data)
    g = rnd(want.shape, 6)
    Gb, D = dev.buf(g), dev.zeros(x.size)
    dev.ok(dev.lib.tysor_cuda_dispatch_repeat_kv_backward(dev.h, Gb.handle, D.handle, 2, 4, 33 * 8, 4, False))
    np.testing.assert_array_equal(D.read(), L.repeat_kv_backward(T(want.shape, g), T(shape, x), 4).data)


def test_causal_mask_and_backward_bit_exact(dev):
    shape = (3, 2, 37, 37)
    x = rnd(shape, 7)
    X, O, G = dev.buf(x), dev.zeros(x.size), dev.zeros(x.size)
    dev.ok(dev.lib.tysor_cuda_dispatch_causal_mask(dev.h, X.handle, O.handle, 6, 37, 37))
    np.testing.assert_array_equal(O.read(), L.causal_mask(T(shape, x)).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_causal_mask_backward(dev.h, X.handle, G.handle, 6, 37, 37, False))
    np.testing.assert_array_equal(G.read(), L.causal_mask_backward(T(shape, x)).data)


def test_embedding_forward_backward_bit_exact(dev):
    num, dim = 1000, 96
    w = rnd((num, dim), 8)
    idx = np.random.default_rng(9).integers(0, num, 777).astype(np.float32)
    idx[:50] = 17.0  # collisions: many tokens on one row
    W, I, O = dev.buf(w), dev.buf(idx), dev.zeros(idx.size * dim)
    dev.ok(dev.lib.tysor_cuda_dispatch_embedding(dev.h, I.handle, W.handle, O.handle, idx.size, dim, num))
    np.testing.assert_array_equal(O.read(), L.embedding(T([idx.size], idx), T([num, dim], w), num, dim).data)
    g = rnd((idx.size, dim), 10)
    Gb, WG = dev.buf(g), dev.zeros(num * dim)
    dev.ok(dev.lib.tysor_cuda_dispatch_embedding_backward(dev.h, Gb.handle, I.handle, WG.handle, idx.size, dim, num, False))
    want = L.embedding_backward(T([idx.size, dim], g), T([idx.size], idx), num, dim)
    np.testing.assert_array_equal(WG.read(), want.data)


def test_embedding_out_of_range_is_an_error(dev):
    from tysor_b200 import native
    w = rnd((4, 8), 11)
    idx = np.array([1.0, 4.0], np.float32)
    W, I, O = dev.buf(w), dev.buf(idx), dev.zeros(16)
    dev.ok(dev.lib.tysor_cuda_dispatch_embedding(dev.h, I.handle, W.handle, O.handle, 2, 8, 4))
    with pytest.raises(native.NativeError, match="out of range"):
        O.read()
    dev.ctx.synchronize()  # the error word was cleared


def test_sgd_bit_exact(dev):
    p, g = rnd(100003, 12), rnd(100003, 13)
    P, Gb = dev.buf(p), dev.buf(g)
    dev.ok(dev.lib.tysor_cuda_dispatch_sgd_update(dev.h, P.handle, Gb.handle, p.size, 1e-3))
    want = T([p.size], p)
    L.sgd(want, T([g.size], g), 1e-3)
    np.testing.assert_array_equal(P.read(), want.data)


def test_transpose_bit_exact(dev):
    shape = (2, 5, 3, 16)
    x = rnd(shape, 14)
    X, O = dev.buf(x), dev.zeros(x.size)
    dims = (ctypes.c_int64 * 4)(*shape)
    dev.ok(dev.lib.tysor_cuda_dispatch_transpose(dev.h, X.handle, O.handle, dims, 4, 1, 2))
    np.testing.assert_array_equal(O.read(), L.transpose(T(shape, x), 1, 2).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_transpose(dev.h, X.handle, O.handle, dims, 4, 2, 3))
    np.testing.assert_array_equal(O.read(), L.transpose(T(shape, x), 2, 3).data)


@pytest.mark.parametrize("shape,a,b", [((2, 3, 5, 4, 64), 1, 2), ((2, 3, 5, 4, 64), 1, 3), ((2, 3, 5, 4, 64), 0, 3),
                                       ((8, 16, 64, 128), 1, 2), ((3, 7, 9, 40), 0, 2)])
def test_transpose_of_whole_runs_bit_exact(dev, shape, a, b):
    """Swaps whose trailing axes form runs of >= 32 elements move the runs
    whole (one warp per run); every element still lands where the oracle
    puts it."""
    x = rnd(shape, 18)
    X, O = dev.buf(x), dev.zeros(x.size)
    dims = (ctypes.c_int64 * len(shape))(*shape)
    dev.ok(dev.lib.tysor_cuda_dispatch_transpose(dev.h, X.handle, O.handle, dims, len(shape), a, b))
    np.testing.assert_array_equal(O.read(), L.transpose(T(shape, x), a, b).data)
    np.testing.assert_array_equal(O.read().reshape(np.swapaxes(x, a, b).shape), np.swapaxes(x, a, b))


def test_bias_grad_and_reduce_sum(dev):
    g = rnd((3001, 77), 15)
    Gb, DB, S = dev.buf(g), dev.zeros(77), dev.zeros(1)
    dev.ok(dev.lib.tysor_cuda_dispatch_bias_grad(dev.h, Gb.handle, DB.handle, 3001, 77, False))
    close_sums(DB.read(), L.bias_grad(T(g.shape, g)).data, np.abs(g).sum(axis=0))
    dev.ok(dev.lib.tysor_cuda_dispatch_reduce_sum(dev.h, Gb.handle, S.handle, g.size))
    close_sums(S.read(), [L.tensor_sum(T([g.size], g))], [np.abs(g).sum()])


def test_activation_backwards(dev):
    x, g = rnd(5000, 16), rnd(5000, 17)
    X, Gb, D = dev.buf(x), dev.buf(g), dev.zeros(x.size)
    y = L.relu(T([x.size], x))
    Y = dev.buf(y.data)
    dev.ok(dev.lib.tysor_cuda_dispatch_relu_backward(dev.h, Y.handle, Gb.handle, D.handle, x.size, False))
    np.testing.assert_array_equal(D.read(), L.relu_backward(y, T([g.size], g)).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_silu_backward(dev.h, X.handle, Gb.handle, D.handle, x.size, False))
    close(D.read(), L.silu_backward(T([x.size], x), T([g.size], g)).data, 1e-6)
    sm = np.abs(x) / 3
    SM = dev.buf(sm)
    dev.ok(dev.lib.tysor_cuda_dispatch_softmax_backward(dev.h, SM.handle, Gb.handle, D.handle, x.size, False))
    np.testing.assert_array_equal(D.read(), L.softmax_backward(T([x.size], sm), T([g.size], g)).data)


@pytest.mark.parametrize("rows,width", [(5, 3), (33, 257), (300, 1024), (300, 2048), (65536, 4096)])
def test_rms_norm_softmax_silu_sweep(dev, rows, width):
    """rms_norm (reference semantics and the gain/eps extension), softmax and
    SiLU at x ~ N(0,1); the largest case is the [65536, 4096] sweep shape."""
    L.set_threads(16)
    rng = np.random.default_rng(rows)
    x = rng.standard_normal((rows, width), dtype=np.float32)
    gain = (1 + 0.02 * rng.standard_normal(width)).astype(np.float32)
    X, O = dev.buf(x), dev.zeros(x.size)
    xt = T(x.shape, x)
    dev.ok(dev.lib.tysor_cuda_dispatch_rms_norm(dev.h, X.handle, O.handle, rows, width))
    close(O.read(), L.rms_norm(xt, width).data)
    Gn = dev.buf(gain)
    dev.ok(dev.lib.tysor_cuda_dispatch_rms_norm_gain(dev.h, X.handle, Gn.handle, O.handle, rows, width, 1e-6))
    close(O.read(), L.rms_norm_gain(xt, T([width], gain), 1e-6).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_softmax(dev.h, X.handle, O.handle, rows, width))
    close(O.read(), L.softmax(xt).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_unary(dev.h, 2, X.handle, O.handle, x.size, 0.0))
    close(O.read(), L.silu(xt).data, 1e-6)
    # backward of the gain extension: dx = dy * g, dg = column sums
    dy = rng.standard_normal((rows, width), dtype=np.float32)
    DY, DX, DG = dev.buf(dy), dev.zeros(x.size), dev.zeros(width)
    dev.ok(dev.lib.tysor_cuda_dispatch_rms_norm_gain_backward(dev.h, X.handle, Gn.handle, DY.handle, DX.handle,
                                                              DG.handle, rows, width, 1e-6, False))
    wdx, wdg = L.rms_norm_gain_backward(xt, T([width], gain), T(dy.shape, dy), 1e-6)
    np.testing.assert_array_equal(DX.read(), wdx.data)
    scale = 1.0 / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-6)
    close_sums(DG.read(), wdg.data, np.abs(dy * x * scale).sum(axis=0))


@pytest.mark.parametrize("rows,width", [(2, 3), (17, 1000), (8192, 32000)])
def test_cross_entropy_sweep(dev, rows, width):
    """Dense-target CE (reference) and class-label CE (extension), forward
    and backward; the largest case is logits [8192, 32000] ~ N(0, 2), for
    both forms."""
    L.set_threads(16)
    rng = np.random.default_rng(width)
    logits = (2.0 * rng.standard_normal((rows, width))).astype(np.float32)
    labels = rng.integers(0, width, rows).astype(np.float32)
    LG, LB, O, G = dev.buf(logits), dev.buf(labels), dev.zeros(rows), dev.zeros(logits.size)
    lt = T(logits.shape, logits)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy_labels(dev.h, LG.handle, LB.handle, O.handle, rows, width))
    close(O.read(), L.cross_entropy(lt, T([rows], labels)).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy_labels_backward(dev.h, LG.handle, LB.handle, G.handle, rows,
                                                                     width, False))
    close(G.read(), L.cross_entropy_backward(lt, T([rows], labels)).data)
    # Dense target (the reference's own form, layers.rs:301-324): a general
    # non-negative target at the small sizes; at [8192, 32000] the one-hot
    # rows of the labels, as the config's parity path feeds it.
    if rows * width <= 17 * 1000:
        target = np.abs(rng.standard_normal((rows, width))).astype(np.float32)
    else:
        target = np.zeros((rows, width), np.float32)
        target[np.arange(rows), labels.astype(np.int64)] = 1.0
    TG = dev.buf(target)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy(dev.h, LG.handle, TG.handle, O.handle, rows, width))
    close(O.read(), L.cross_entropy(lt, T(target.shape, target)).data)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy_backward(dev.h, LG.handle, TG.handle, G.handle, rows, width,
                                                              False))
    close(G.read(), L.cross_entropy_backward(lt, T(target.shape, target)).data)


@pytest.mark.parametrize("rows,width", [(33, 4096), (3, 40000)])
def test_cross_entropy_backward_accumulates(dev, rows, width):
    """The backward kernels add into an existing gradient when asked
    (labels and dense targets, a power-of-two and a wide row)."""
    rng = np.random.default_rng(rows + width)
    logits = (2.0 * rng.standard_normal((rows, width))).astype(np.float32)
    labels = rng.integers(0, width, rows).astype(np.float32)
    target = np.abs(rng.standard_normal((rows, width))).astype(np.float32)
    old = rng.standard_normal((rows, width)).astype(np.float32)
    lt = T(logits.shape, logits)
    LG, LB, TG = dev.buf(logits), dev.buf(labels), dev.buf(target)
    G = dev.buf(old)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy_labels_backward(dev.h, LG.handle, LB.handle, G.handle, rows,
                                                                     width, True))
    close(G.read(), old.reshape(-1) + L.cross_entropy_backward(lt, T([rows], labels)).data)
    G = dev.buf(old)
    dev.ok(dev.lib.tysor_cuda_dispatch_cross_entropy_backward(dev.h, LG.handle, TG.handle, G.handle, rows, width,
                                                              True))
    close(G.read(), old.reshape(-1) + L.cross_entropy_backward(lt, T(target.shape, target)).data)


def test_pipeline_wait_gives_up_and_reports(dev):
    """The tensor-core pipelines' mbarrier wait is bounded: a wait on a
    barrier that nothing arrives at gives up after its cycle limit and
    records an error that the host reads as a failure.  The context stays
    usable afterwards (a matmul then runs and matches the oracle)."""
    from tysor_b200 import native
    assert not dev.lib.tysor_cuda_probe_wait_timeout(dev.h, 20000)
    assert "wait timed out" in native.last_error()
    assert not dev.lib.tysor_cuda_probe_wait_timeout(dev.h, 0)  # limit outside [1, 4e9]
    assert "limit" in native.last_error()
    a, b = rnd((256, 64), 30), rnd((64, 128), 31)
    A, B, C = dev.buf(a), dev.buf(b), dev.zeros(256 * 128)
    dev.ok(dev.lib.tysor_cuda_dispatch_matmul(dev.h, A.handle, B.handle, C.handle, 256, 128, 64))
    want = L.matmul(T(a.shape, a), T(b.shape, b)).data
    got = C.read()
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-5
