"""Matmul mode 3 ("strict16"): the three products of strict mode over fp16
halves of the operands, each operand row scaled by a power of two
(launch_pack16), on the tensor core's fp16 rate.

* Every operand layout, ragged K, M and N, against the oracle's sequential
  f32 matmul (runtime/tensor.rs:163-194) within the strict bar (Frobenius
  1e-5), and no further from the float64 product than 3xTF32 is (within a
  factor of 2).
* Rows of A and columns of B spread over 24 decades: each output element
  within 1e-6 of the float64 product, relative to its own |A|.|B| scale
  (the per-row scales keep fp16's 5-bit exponent out of the way).
* The epilogue (alpha, bias, relu, accumulate into C) as strict mode has it.
* GEMMs the mode does not cover (M < 256, N <= 128, batched) run 3xTF32:
  bit-identical to strict mode.
"""
import numpy as np
import pytest

import local as L

from test_gpu_gemm import frob, oracle_mm, run_ex

pytestmark = pytest.mark.gpu


def stored(x, trans):
    return np.ascontiguousarray(x.T if trans else x)


def mm(ctx, mode, a, b, ta, tb, **kw):
    ctx.set_matmul_mode(mode)
    try:
        m, k = a.shape
        n = b.shape[1]
        return run_ex(ctx, stored(a, ta), ta, stored(b, tb), tb, m, n, k, **kw)
    finally:
        ctx.set_matmul_mode("strict")


SHAPES = [(256, 136, 8), (512, 384, 1000), (300, 520, 72), (1000, 1000, 1000), (257, 259, 33), (768, 2048, 2048)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
def test_strict16_layouts(cuda_ctx, m, n, k, ta, tb):
    rng = np.random.default_rng(m * 5 + n * 7 + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    got = mm(cuda_ctx, "strict16", a, b, ta, tb)
    tf32 = mm(cuda_ctx, "strict", a, b, ta, tb)
    e16, e32 = frob(got, exact), frob(tf32, exact)
    print(f"\n{m}x{n}x{k} ta={ta} tb={tb}: strict16 vs f64 {e16:.2e}, 3xTF32 vs f64 {e32:.2e}")
    assert frob(got, oracle_mm(a, b)) < 1e-5
    assert e16 <= 2 * e32 + 1e-8


def test_strict16_rows_over_24_decades(cuda_ctx):
    m, n, k = 512, 384, 640
    rng = np.random.default_rng(7)
    ra = 10.0 ** rng.uniform(-12, 12, (m, 1))
    cb = 10.0 ** rng.uniform(-12, 12, (1, n))
    a = (rng.uniform(-1, 1, (m, k)) * ra).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) * cb).astype(np.float32)
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    exact = a64 @ b64
    scale = np.abs(a64) @ np.abs(b64)
    for ta, tb in [(False, True), (True, False)]:
        got = mm(cuda_ctx, "strict16", a, b, ta, tb)
        err = float(np.max(np.abs(got - exact) / scale))
        print(f"\nta={ta} tb={tb}: max |dev - f64| / (|A|.|B|) = {err:.2e}")
        assert err < 1e-6


def test_strict16_zero_rows_and_columns(cuda_ctx):
    m, n, k = 300, 260, 96
    rng = np.random.default_rng(3)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    a[::7] = 0.0
    b[:, ::5] = 0.0
    got = mm(cuda_ctx, "strict16", a, b, False, True)
    assert np.all(got[::7] == 0.0) and np.all(got[:, ::5] == 0.0)
    assert frob(got, oracle_mm(a, b)) < 1e-5


@pytest.mark.parametrize("relu", [False, True])
def test_strict16_epilogue(cuda_ctx, relu):
    m, n, k = 512, 520, 264
    rng = np.random.default_rng(11)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    c0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    got = mm(cuda_ctx, "strict16", a, b, False, False, bias=bias, alpha=0.5, relu=relu)
    want = oracle_mm(a, b).astype(np.float64) * 0.5 + bias
    if relu:
        want = np.maximum(want, 0.0)
    assert frob(got, want) < 1e-5
    got = mm(cuda_ctx, "strict16", a, b, False, True, acc=c0.reshape(-1).copy())
    assert frob(got, c0.astype(np.float64) + oracle_mm(a, b)) < 1e-5


@pytest.mark.parametrize("m,n,k,batch", [(128, 512, 256, 1), (512, 128, 256, 1), (256, 384, 128, 2)])
def test_uncovered_shapes_run_strict(cuda_ctx, m, n, k, batch):
    rng = np.random.default_rng(m + n + k + batch)
    a = rng.uniform(-1, 1, (batch, m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, k, n)).astype(np.float32)
    if batch == 1:
        a, b = a[0], b[0]
    outs = []
    for mode in ("strict", "strict16"):
        cuda_ctx.set_matmul_mode(mode)
        try:
            outs.append(run_ex(cuda_ctx, a, False, b, False, m, n, k, batch=batch))
        finally:
            cuda_ctx.set_matmul_mode("strict")
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.parametrize("ta,tb", [(True, False), (False, True)])
def test_strict16_odd_row_pitch(cuda_ctx, ta, tb):
    """Operands stored with a row pitch one element longer than the matrix
    (not a multiple of 4): the packing kernels fall back to scalar loads."""
    m, n, k = 260, 300, 200
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)

    def padded(x):
        out = np.zeros((x.shape[0], x.shape[1] + 1), np.float32)
        out[:, :-1] = x
        return out
    a_st = padded(a.T if ta else a)
    b_st = padded(b.T if tb else b)
    cuda_ctx.set_matmul_mode("strict16")
    try:
        got = run_ex(cuda_ctx, a_st, ta, b_st, tb, m, n, k)
    finally:
        cuda_ctx.set_matmul_mode("strict")
    assert frob(got, oracle_mm(a, b)) < 1e-5


def test_strict16_block_step_against_the_oracle(cuda_ctx):
    """A decoder block whose linear layers the split-fp16 engine covers (512
    tokens, d 256): forward output and every parameter gradient against the
    oracle, with both packings of each activation and gradient (row-wise for
    one GEMM, column-wise for the weight gradient's)."""
    from test_gpu_block import frob as bfrob, params_for
    from tysor_b200.programs import llama_block
    from tysor_b200.runtime import CudaGraphExecutor
    cfg = dict(batch=2, seq=256, d_model=256, n_heads=4, n_kv_heads=2, hidden=384, eps=1e-6, lr=1e-4)
    g = llama_block(**cfg)
    t = cfg["batch"] * cfg["seq"]
    shapes = {"x": [t, cfg["d_model"]]}
    x = np.random.default_rng(2).standard_normal((t, cfg["d_model"])).astype(np.float32)
    params = params_for(g)
    oparams = {k: L.Tensor(list(v.shape), v.reshape(-1).copy()) for k, v in params.items()}
    values, grads, _ = L.train_step_grads(g, shapes, inputs={"x": x}, parameters=oparams)
    out_id = g.outputs[0]
    cuda_ctx.set_matmul_mode("strict16")
    try:
        ex = CudaGraphExecutor(cuda_ctx, g, shapes, inputs={"x": x}, parameters=params)
        ex.train(1, 0.0)
        errs = {"out": bfrob(ex.value(out_id).data, values[out_id][1].data)}
        for name, gt in grads.items():
            errs[name] = bfrob(ex.parameter_grad(name), gt.data)
        ex.close()
    finally:
        cuda_ctx.set_matmul_mode("strict")
    print("\nstrict16 block vs oracle:", {k: f"{v:.1e}" for k, v in errs.items()})
    assert errs.pop("out") < 1e-5
    for name, e in errs.items():
        assert e < 1e-4, name
