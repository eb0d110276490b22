// Bandwidth-bound kernels (see ops.cuh).  This file is compiled with
// --fmad=false: every product and sum is rounded separately, so elementwise
// results equal the reference's f32 arithmetic bit for bit wherever the
// operation itself is exact (copies, masks, rotations with host-computed
// cos/sin, gathers, updates), and differ only by libm-level ulps in
// expf/logf or by summation order in row reductions.
#include <math.h>

#include "ops.cuh"

namespace tysor {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ bool aligned16(const void* p) { return (((uintptr_t)p) & 15) == 0; }

// x - tf32(x): the low part a strict 3xTF32 GEMM multiplies separately.
__device__ __forceinline__ float lo_part(float x) { return tf32_lo(x); }

// The probability every masked entry of a causal softmax row keeps: the
// masked scores all read -1e4, so each is exp(-1e4 - max) / d, the value the
// row stores there.  It is 0 unless the row's visible scores all lie below
// about -9896 (then exp(-1e4 - max) does not underflow); a row with nothing
// masked (qi = width - 1) has none.
__device__ __forceinline__ float masked_leak(int qi, int width, bool masked_zero, float m, float d) {
  return (qi < width - 1 && !masked_zero) ? expf(-1.0e4f - m) / d : 0.0f;
}
__device__ __forceinline__ float4 lo_part4(float4 v) {
  return make_float4(lo_part(v.x), lo_part(v.y), lo_part(v.z), lo_part(v.w));
}

// f32 -> i64 with Rust `as` semantics (truncation, saturation, NaN -> 0).
__device__ __forceinline__ long long rust_f32_to_i64(float v) {
  if (isnan(v)) return 0;
  if (v >= 9.2233720368547758e18f) return LLONG_MAX;
  if (v <= -9.2233720368547758e18f) return LLONG_MIN;
  return (long long)v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reductions; every thread gets the result.  `red` has >= 33 floats.
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = threadIdx.x < nw ? red[threadIdx.x] : 0.0f;
  if (w == 0) {
    t = warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = threadIdx.x < nw ? red[threadIdx.x] : -INFINITY;
  if (w == 0) {
    t = warp_max(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float apply_binary(int op, float a, float b) {
  switch (op) {
    case kAdd: return a + b;
    case kSub: return a - b;
    case kMul: return a * b;
    default: return a / b;
  }
}

__device__ __forceinline__ float apply_unary(int op, float x, float p) {
  switch (op) {
    case kUnaryRelu: return fmaxf(x, 0.0f);
    case kUnarySilu: return x / (1.0f + expf(-x));
    case kUnaryScale: return x * p;
    case kUnaryNeg: return -x;
    default: return x;
  }
}

// ---- elementwise ------------------------------------------------------------

__global__ void pattern_kernel(float* out, int64_t n, int mod, float add, float div) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = ((float)(i % mod) + add) / div;
}

__global__ void fill_kernel(float* out, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = v;
}

// Generic elementwise driver.  out[i] = op(in_0[i], ..., in_{N-1}[i]), or
// out[i] + op(...) with `acc` (the reference's add_in_place order).  When
// every pointer is 16-byte aligned each thread moves kUnroll float4 per
// input per iteration, all loads issued before the first use, so enough
// bytes are in flight to keep HBM busy; ragged tails and unaligned views
// take the scalar loop.  `out` may alias an input at the same index.
constexpr int kUnroll = 4;

template <int N>
struct In {
  const float* p[N > 0 ? N : 1];
};

template <int N, typename Op>
__device__ __forceinline__ float4 ew_apply4(Op op, const float4 (&a)[N > 0 ? N : 1], float4 o, int acc) {
  float s[N > 0 ? N : 1];
  float4 r;
#pragma unroll
  for (int k = 0; k < N; ++k) s[k] = a[k].x;
  r.x = op(s);
#pragma unroll
  for (int k = 0; k < N; ++k) s[k] = a[k].y;
  r.y = op(s);
#pragma unroll
  for (int k = 0; k < N; ++k) s[k] = a[k].z;
  r.z = op(s);
#pragma unroll
  for (int k = 0; k < N; ++k) s[k] = a[k].w;
  r.w = op(s);
  if (acc) r = make_float4(o.x + r.x, o.y + r.y, o.z + r.z, o.w + r.w);
  return r;
}

template <int N, typename Op>
__device__ __forceinline__ void ew_run(In<N> in, float* out, int64_t n, int acc, Op op) {
  bool vec = aligned16(out);
#pragma unroll
  for (int k = 0; k < N; ++k) vec = vec && aligned16(in.p[k]);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n >> 2;
    int64_t i = t0;
    for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
      float4 a[kUnroll][N > 0 ? N : 1];
      float4 o[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
        for (int k = 0; k < N; ++k) a[u][k] = ((const float4*)in.p[k])[i + u * stride];
        o[u] = acc ? ((const float4*)out)[i + u * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) ((float4*)out)[i + u * stride] = ew_apply4<N>(op, a[u], o[u], acc);
    }
    for (; i < n4; i += stride) {
      float4 a[N > 0 ? N : 1];
#pragma unroll
      for (int k = 0; k < N; ++k) a[k] = ((const float4*)in.p[k])[i];
      const float4 o = acc ? ((const float4*)out)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      ((float4*)out)[i] = ew_apply4<N>(op, a, o, acc);
    }
    done = n4 << 2;
  }
  for (int64_t e = done + t0; e < n; e += stride) {
    float s[N > 0 ? N : 1];
#pragma unroll
    for (int k = 0; k < N; ++k) s[k] = in.p[k][e];
    const float v = op(s);
    out[e] = acc ? out[e] + v : v;
  }
}

// The op is a template argument so the per-element body has no branch.
template <int OP>
__global__ void unary_kernel(const float* x, float* out, int64_t n, float p) {
  ew_run<1>(In<1>{{x}}, out, n, 0, [=](const float (&a)[1]) { return apply_unary(OP, a[0], p); });
}

// Gradient of x * x from g, as the '*' backward's two contributions give it
// to a fresh buffer: t = g * x stored, then t added: t + t.
__global__ void square_backward_kernel(const float* g, const float* x, float* out, int64_t n) {
  ew_run<2>(In<2>{{g, x}}, out, n, 0, [=](const float (&v)[2]) {
    const float t = v[0] * v[1];
    return t + t;
  });
}

__global__ void binary_tt_kernel(int op, const float* a, const float* b, float* out, int64_t n) {
  ew_run<2>(In<2>{{a, b}}, out, n, 0, [=](const float (&v)[2]) { return apply_binary(op, v[0], v[1]); });
}

__global__ void binary_ts_kernel(int op, const float* a, float s, float* out, int64_t n,
                                 int scalar_first) {
  ew_run<1>(In<1>{{a}}, out, n, 0, [=](const float (&v)[1]) {
    return scalar_first ? apply_binary(op, s, v[0]) : apply_binary(op, v[0], s);
  });
}

__global__ void add_inplace_kernel(float* dst, const float* src, int64_t n) {
  ew_run<1>(In<1>{{src}}, dst, n, 1, [=](const float (&v)[1]) { return v[0]; });
}

__global__ void binary_acc_kernel(int op, const float* a, const float* b, float s, int mode,
                                  float* dst, int64_t n) {
  // mode 0: op(a[i], b[i]); 1: op(a[i], s); 2: op(s, a[i])
  if (mode == 0)
    ew_run<2>(In<2>{{a, b}}, dst, n, 1, [=](const float (&v)[2]) { return apply_binary(op, v[0], v[1]); });
  else
    ew_run<1>(In<1>{{a}}, dst, n, 1, [=](const float (&v)[1]) {
      return mode == 1 ? apply_binary(op, v[0], s) : apply_binary(op, s, v[0]);
    });
}

__global__ void div_rhs_grad_kernel(const float* g, const float* l, const float* r, float* dst,
                                    int64_t n, int accumulate) {
  ew_run<3>(In<3>{{g, l, r}}, dst, n, accumulate, [=](const float (&v)[3]) {
    const float num = v[0] * v[1];
    const float den = v[2] * v[2];
    return -(num / den);
  });
}

__global__ void relu_backward_kernel(const float* y, const float* g, float* dx, int64_t n, int acc) {
  ew_run<2>(In<2>{{y, g}}, dx, n, acc, [=](const float (&v)[2]) { return v[1] * (v[0] > 0.0f ? 1.0f : 0.0f); });
}

__global__ void silu_backward_kernel(const float* x, const float* g, float* dx, int64_t n, int acc) {
  ew_run<2>(In<2>{{x, g}}, dx, n, acc, [=](const float (&a)[2]) {
    const float v = a[0];
    const float s = 1.0f / (1.0f + expf(-v));
    float t = v * s;
    t = t * (1.0f - s);
    return a[1] * (s + t);
  });
}

// h = silu(x) * u in one pass (SwiGLU's product): silu as unary_kernel
// computes it, then the product, so h is bit-identical to the two-kernel
// form; silu(x) is never stored.
__global__ void silu_mul_kernel(const float* x, const float* u, float* h, int64_t n) {
  ew_run<2>(In<2>{{x, u}}, h, n, 0, [=](const float (&a)[2]) {
    const float s = apply_unary(kUnarySilu, a[0], 0.0f);
    return s * a[1];
  });
}

// Backward of h = silu(x) * u from dh: du (+)= dh * silu(x) and
// dx (+)= silu_backward(x, dh * u), each element computed exactly as the
// '*' backward and silu_backward_kernel compute it; inputs read once, the
// activation's gradient never stored.
__device__ __forceinline__ void silu_mul_grad(float x, float u, float dh, float* dx, float* du) {
  const float s = apply_unary(kUnarySilu, x, 0.0f);
  *du = dh * s;
  const float ds = dh * u;
  const float sg = 1.0f / (1.0f + expf(-x));
  float t = x * sg;
  t = t * (1.0f - sg);
  *dx = ds * (sg + t);
}

__global__ void silu_mul_backward_kernel(const float* __restrict__ x, const float* __restrict__ u,
                                         const float* __restrict__ dh, float* __restrict__ dx,
                                         float* __restrict__ du, int64_t n, int acc_x, int acc_u) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (aligned16(x) && aligned16(u) && aligned16(dh) && aligned16(dx) && aligned16(du)) {
    const int64_t n4 = n >> 2;
    int64_t i = t0;
    for (; i + stride < n4; i += 2 * stride) {
      float4 a[2], b[2], c[2], ox[2], ou[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        a[k] = ((const float4*)x)[i + k * stride];
        b[k] = ((const float4*)u)[i + k * stride];
        c[k] = ((const float4*)dh)[i + k * stride];
        ox[k] = acc_x ? ((const float4*)dx)[i + k * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
        ou[k] = acc_u ? ((const float4*)du)[i + k * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float4 rx, ru;
        silu_mul_grad(a[k].x, b[k].x, c[k].x, &rx.x, &ru.x);
        silu_mul_grad(a[k].y, b[k].y, c[k].y, &rx.y, &ru.y);
        silu_mul_grad(a[k].z, b[k].z, c[k].z, &rx.z, &ru.z);
        silu_mul_grad(a[k].w, b[k].w, c[k].w, &rx.w, &ru.w);
        if (acc_x) rx = make_float4(ox[k].x + rx.x, ox[k].y + rx.y, ox[k].z + rx.z, ox[k].w + rx.w);
        if (acc_u) ru = make_float4(ou[k].x + ru.x, ou[k].y + ru.y, ou[k].z + ru.z, ou[k].w + ru.w);
        ((float4*)dx)[i + k * stride] = rx;
        ((float4*)du)[i + k * stride] = ru;
      }
    }
    for (; i < n4; i += stride) {
      const float4 a = ((const float4*)x)[i], b = ((const float4*)u)[i], c = ((const float4*)dh)[i];
      float4 rx, ru;
      silu_mul_grad(a.x, b.x, c.x, &rx.x, &ru.x);
      silu_mul_grad(a.y, b.y, c.y, &rx.y, &ru.y);
      silu_mul_grad(a.z, b.z, c.z, &rx.z, &ru.z);
      silu_mul_grad(a.w, b.w, c.w, &rx.w, &ru.w);
      if (acc_x) {
        const float4 o = ((const float4*)dx)[i];
        rx = make_float4(o.x + rx.x, o.y + rx.y, o.z + rx.z, o.w + rx.w);
      }
      if (acc_u) {
        const float4 o = ((const float4*)du)[i];
        ru = make_float4(o.x + ru.x, o.y + ru.y, o.z + ru.z, o.w + ru.w);
      }
      ((float4*)dx)[i] = rx;
      ((float4*)du)[i] = ru;
    }
    done = n4 << 2;
  }
  for (int64_t e = done + t0; e < n; e += stride) {
    float rx, ru;
    silu_mul_grad(x[e], u[e], dh[e], &rx, &ru);
    dx[e] = acc_x ? dx[e] + rx : rx;
    du[e] = acc_u ? du[e] + ru : ru;
  }
}

__global__ void softmax_backward_kernel(const float* y, const float* g, float* dx, int64_t n,
                                        int acc) {
  ew_run<2>(In<2>{{y, g}}, dx, n, acc, [=](const float (&a)[2]) {
    const float t = a[0] * (1.0f - a[0]);
    return t * a[1];
  });
}

__global__ void sgd_kernel(float* p, const float* g, float lr, int64_t n) {
  ew_run<2>(In<2>{{p, g}}, p, n, 0, [=](const float (&a)[2]) { return a[0] - lr * a[1]; });
}

// ---- row reductions -------------------------------------------------------------

// One block per row (grid-stride over rows).  Sum of squares, then
// y = x * (1 / sqrt(ms + eps)) (* g).
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                float* __restrict__ out, int64_t rows, int width, float eps) {
  __shared__ float red[33];
  const bool vec = (width & 3) == 0 && aligned16(x) && aligned16(out) && (g == nullptr || aligned16(g));
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * width;
    float* yr = out + r * width;
    float acc = 0.0f;
    if (vec) {
      for (int j = threadIdx.x; j < width / 4; j += blockDim.x) {
        float4 v = ((const float4*)xr)[j];
        acc += v.x * v.x;
        acc += v.y * v.y;
        acc += v.z * v.z;
        acc += v.w * v.w;
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) acc += xr[j] * xr[j];
    }
    const float ms = block_sum(acc, red) / (float)width;
    const float scale = 1.0f / sqrtf(ms + eps);
    if (vec) {
      for (int j = threadIdx.x; j < width / 4; j += blockDim.x) {
        float4 v = ((const float4*)xr)[j];
        v.x = v.x * scale;
        v.y = v.y * scale;
        v.z = v.z * scale;
        v.w = v.w * scale;
        if (g) {
          float4 w = ((const float4*)g)[j];
          v.x = v.x * w.x;
          v.y = v.y * w.y;
          v.z = v.z * w.z;
          v.w = v.w * w.w;
        }
        ((float4*)yr)[j] = v;
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) {
        float v = xr[j] * scale;
        yr[j] = g ? v * g[j] : v;
      }
    }
  }
}

// dx = dy * g; partial[block][j] = sum over the block's rows of dy * x * scale.
__global__ void rms_gain_backward_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                         const float* __restrict__ dy, float* __restrict__ dx,
                                         float* __restrict__ partial, int64_t rows, int width,
                                         float eps, int acc_dx, int rows_per_block) {
  __shared__ float red[33];
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  // Each thread owns columns j = threadIdx.x + k*blockDim.x; partial sums are
  // kept in the output row of this block, updated in row order.
  float* prow = partial + (int64_t)blockIdx.x * width;
  for (int j = threadIdx.x; j < width; j += blockDim.x) prow[j] = 0.0f;
  for (int64_t r = r0; r < r1; ++r) {
    const float* xr = x + r * width;
    float acc = 0.0f;
    for (int j = threadIdx.x; j < width; j += blockDim.x) acc += xr[j] * xr[j];
    const float ms = block_sum(acc, red) / (float)width;
    const float scale = 1.0f / sqrtf(ms + eps);
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float d = dy[r * width + j];
      const float v = d * g[j];
      dx[r * width + j] = acc_dx ? dx[r * width + j] + v : v;
      const float nrm = xr[j] * scale;
      prow[j] = prow[j] + d * nrm;
    }
  }
}

// Register-resident form for widths of 1024 * VPT: 256 threads, each
// owning VPT float4 columns.  The gain and the block's partial column sums
// stay in registers; x and dy are read once per row.
template <int VPT>
__global__ void __launch_bounds__(256) rms_gain_backward_reg_kernel(
    const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ dy,
    float* __restrict__ dx, float* __restrict__ partial, int64_t rows, float eps, int acc_dx,
    int rows_per_block) {
  __shared__ float red[33];
  constexpr int kWidth = 1024 * VPT;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  float4 gv[VPT], pv[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    gv[i] = ((const float4*)g)[threadIdx.x + i * 256];
    pv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int64_t r = r0; r < r1; ++r) {
    const float4* xr = (const float4*)(x + r * kWidth);
    const float4* dr = (const float4*)(dy + r * kWidth);
    float4* or_ = (float4*)(dx + r * kWidth);
    float4 xv[VPT], dv[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      xv[i] = xr[threadIdx.x + i * 256];
      dv[i] = dr[threadIdx.x + i * 256];
    }
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      acc += xv[i].x * xv[i].x;
      acc += xv[i].y * xv[i].y;
      acc += xv[i].z * xv[i].z;
      acc += xv[i].w * xv[i].w;
    }
    const float ms = block_sum(acc, red) / (float)kWidth;
    const float scale = 1.0f / sqrtf(ms + eps);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float4 v = make_float4(dv[i].x * gv[i].x, dv[i].y * gv[i].y, dv[i].z * gv[i].z, dv[i].w * gv[i].w);
      if (acc_dx) {
        const float4 o = or_[threadIdx.x + i * 256];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      or_[threadIdx.x + i * 256] = v;
      pv[i].x = pv[i].x + dv[i].x * (xv[i].x * scale);
      pv[i].y = pv[i].y + dv[i].y * (xv[i].y * scale);
      pv[i].z = pv[i].z + dv[i].z * (xv[i].z * scale);
      pv[i].w = pv[i].w + dv[i].w * (xv[i].w * scale);
    }
  }
  float4* prow = (float4*)(partial + (int64_t)blockIdx.x * kWidth);
#pragma unroll
  for (int i = 0; i < VPT; ++i) prow[threadIdx.x + i * 256] = pv[i];
}

// out[j] (+)= sum_b partial[b][j], b in order; eight partial rows are
// loaded ahead of their (ordered) additions.
__global__ void sum_partials_kernel(const float* partial, float* out, int nblocks, int width,
                                    int accumulate) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < width; j += gridDim.x * blockDim.x) {
    float acc = 0.0f;
    int b = 0;
    for (; b + 8 <= nblocks; b += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = partial[(int64_t)(b + u) * width + j];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = acc + v[u];
    }
    for (; b < nblocks; ++b) acc = acc + partial[(int64_t)b * width + j];
    out[j] = accumulate ? out[j] + acc : acc;
  }
}

__device__ __forceinline__ void row_max_sum(const float* xr, int width, float* red, float* m_out,
                                            float* denom_out) {
  float m = -INFINITY;
  for (int j = threadIdx.x; j < width; j += blockDim.x) m = fmaxf(m, xr[j]);
  m = block_max(m, red);
  float s = 0.0f;
  for (int j = threadIdx.x; j < width; j += blockDim.x) s += expf(xr[j] - m);
  s = block_sum(s, red);
  *m_out = m;
  *denom_out = fmaxf(s, 1.1920928955078125e-7f);  // max(sum, f32::EPSILON)
}

__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t rows,
                               int width) {
  __shared__ float red[33];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = x + r * width;
    float m, d;
    row_max_sum(xr, width, red, &m, &d);
    float* yr = out + r * width;
    for (int j = threadIdx.x; j < width; j += blockDim.x) yr[j] = expf(xr[j] - m) / d;
  }
}

// Register-resident row softmax for widths of 1024 * VPT: each of 256
// threads keeps VPT float4 of its row, so the row is read from HBM once and
// written once (registers capped so five blocks share an SM, four at VPT 8).  With `masked`, row r's entries with col > r % q read as
// -1e4 (causal_mask fused in front).  Same arithmetic as softmax_kernel.
template <int VPT>
__global__ void __launch_bounds__(256, VPT >= 8 ? 4 : 5) softmax_reg_kernel(const float* __restrict__ x,
                                                          float* __restrict__ out, int64_t rows,
                                                          int q, int masked, float* __restrict__ leak,
                                                          float* __restrict__ lo, int skip_zero) {
  __shared__ float red[33];
  constexpr int kWidth = 1024 * VPT;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int qi = masked ? (int)(r % q) : kWidth;
    const float4* xr = (const float4*)(x + r * kWidth);
    float4 v[VPT];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = threadIdx.x + i * 256;
      const int c = 4 * j;
      // Fully masked float4 groups are not read: their value is -1e4 whatever x holds.
      float4 t = c > qi ? make_float4(-1.0e4f, -1.0e4f, -1.0e4f, -1.0e4f) : xr[j];
      if (c + 0 > qi) t.x = -1.0e4f;
      if (c + 1 > qi) t.y = -1.0e4f;
      if (c + 2 > qi) t.z = -1.0e4f;
      if (c + 3 > qi) t.w = -1.0e4f;
      v[i] = t;
      m = fmaxf(fmaxf(fmaxf(m, t.x), fmaxf(t.y, t.z)), t.w);
    }
    m = block_max(m, red);
    const bool masked_zero = expf(-1.0e4f - m) == 0.0f;  // the row's masked entries underflow to 0
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      // Wholly masked groups are exact zeros when exp(-1e4 - max) underflows:
      // their exp, sum terms (+0) and divisions are skipped.
      if (masked_zero && 4 * (threadIdx.x + i * 256) > qi) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      v[i].x = expf(v[i].x - m);
      v[i].y = expf(v[i].y - m);
      v[i].z = expf(v[i].z - m);
      v[i].w = expf(v[i].w - m);
      s += v[i].x;
      s += v[i].y;
      s += v[i].z;
      s += v[i].w;
    }
    const float d = fmaxf(block_sum(s, red), 1.1920928955078125e-7f);
    if (leak != nullptr && threadIdx.x == 0) leak[r] = masked_leak(qi, kWidth, masked_zero, m, d);
    float4* yr = (float4*)(out + r * kWidth);
    float4* lr = lo ? (float4*)(lo + r * kWidth) : nullptr;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float4 t = v[i];
      if (masked_zero && 4 * (threadIdx.x + i * 256) > qi) {
        // Exact zeros: not stored at all into buffers that hold zeros there.
        if (!skip_zero) {
          yr[threadIdx.x + i * 256] = t;
          if (lr) lr[threadIdx.x + i * 256] = t;
        }
        continue;
      }
      t.x = t.x / d;
      t.y = t.y / d;
      t.z = t.z / d;
      t.w = t.w / d;
      yr[threadIdx.x + i * 256] = t;
      if (lr) lr[threadIdx.x + i * 256] = lo_part4(t);
    }
  }
}

// WPR warps per row for rows of 128 * NPL * WPR values (NPL float4 per
// lane; at most 64 registers, so four blocks share an SM): the row stays in
// registers and both reductions are warp shuffles,
// joined across the row's warps through shared memory under a named barrier
// of the row's 32 * WPR threads (no block-wide barrier).  A block of 8 warps
// has 8 / WPR rows in flight.  Same arithmetic and options as
// softmax_reg_kernel.
template <int NPL, int WPR>
__global__ void __launch_bounds__(256, 4) softmax_warp_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                           int64_t rows, int q, int masked, float* __restrict__ leak,
                                                           float* __restrict__ lo, int skip_zero) {
  constexpr int kWidth = 128 * NPL * WPR;
  constexpr int kRowsPerBlock = 8 / WPR;
  __shared__ float red[kRowsPerBlock][2][WPR];
  const int lane = threadIdx.x & 31;
  const int grp = (threadIdx.x >> 5) / WPR;  // the row slot of this warp
  const int wr = (threadIdx.x >> 5) % WPR;   // this warp's part of the row
  const int t = 32 * wr + lane;              // thread index within the row
  for (int64_t r = (int64_t)blockIdx.x * kRowsPerBlock + grp; r < rows; r += (int64_t)gridDim.x * kRowsPerBlock) {
    const int qi = masked ? (int)(r % q) : kWidth;
    const float4* xr = (const float4*)(x + r * kWidth);
    float4 v[NPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int c = 4 * (t + 32 * WPR * i);
      float4 u = c > qi ? make_float4(-1.0e4f, -1.0e4f, -1.0e4f, -1.0e4f) : xr[t + 32 * WPR * i];
      if (c + 1 > qi) u.y = -1.0e4f;
      if (c + 2 > qi) u.z = -1.0e4f;
      if (c + 3 > qi) u.w = -1.0e4f;
      v[i] = u;
      m = fmaxf(fmaxf(fmaxf(m, u.x), fmaxf(u.y, u.z)), u.w);
    }
    m = warp_max(m);
    if constexpr (WPR > 1) {
      if (lane == 0) red[grp][0][wr] = m;
      asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * WPR) : "memory");
      m = red[grp][0][0];
#pragma unroll
      for (int w = 1; w < WPR; ++w) m = fmaxf(m, red[grp][0][w]);
    }
    const bool masked_zero = expf(-1.0e4f - m) == 0.0f;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      if (masked_zero && 4 * (t + 32 * WPR * i) > qi) {
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        continue;
      }
      v[i].x = expf(v[i].x - m);
      v[i].y = expf(v[i].y - m);
      v[i].z = expf(v[i].z - m);
      v[i].w = expf(v[i].w - m);
      s += v[i].x;
      s += v[i].y;
      s += v[i].z;
      s += v[i].w;
    }
    s = warp_sum(s);
    if constexpr (WPR > 1) {
      // Slot 1 is free: every thread of the row read slot 1 of the previous
      // row before it arrived at this row's first barrier.
      if (lane == 0) red[grp][1][wr] = s;
      asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "r"(32 * WPR) : "memory");
      s = red[grp][1][0];
#pragma unroll
      for (int w = 1; w < WPR; ++w) s += red[grp][1][w];
    }
    const float d = fmaxf(s, 1.1920928955078125e-7f);
    if (leak != nullptr && t == 0) leak[r] = masked_leak(qi, kWidth, masked_zero, m, d);
    float4* yr = (float4*)(out + r * kWidth);
    float4* lr = lo ? (float4*)(lo + r * kWidth) : nullptr;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int j = t + 32 * WPR * i;
      float4 u = v[i];
      if (masked_zero && 4 * j > qi) {
        if (!skip_zero) {
          yr[j] = u;
          if (lr) lr[j] = u;
        }
        continue;
      }
      u.x = u.x / d;
      u.y = u.y / d;
      u.z = u.z / d;
      u.w = u.w / d;
      yr[j] = u;
      if (lr) lr[j] = lo_part4(u);
    }
  }
}

// Row r of [outer*q] rows of width k; row index within its q x k block is
// r % q.  Values with col > row read as -1e4.
__global__ void masked_softmax_kernel(const float* __restrict__ x, float* __restrict__ out,
                                      int64_t rows, int q, int width, float* __restrict__ leak,
                                      float* __restrict__ lo) {
  __shared__ float red[33];
  const bool vec = (width & 3) == 0 && aligned16(x) && aligned16(out);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int qi = (int)(r % q);
    const float* xr = x + r * width;
    float* yr = out + r * width;
    float m = -INFINITY;
    if (vec) {
      for (int j = threadIdx.x; j < width / 4; j += blockDim.x) {
        const float4 v = ((const float4*)xr)[j];
        const int c = 4 * j;
        m = fmaxf(m, c + 0 > qi ? -1.0e4f : v.x);
        m = fmaxf(m, c + 1 > qi ? -1.0e4f : v.y);
        m = fmaxf(m, c + 2 > qi ? -1.0e4f : v.z);
        m = fmaxf(m, c + 3 > qi ? -1.0e4f : v.w);
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) m = fmaxf(m, j > qi ? -1.0e4f : xr[j]);
    }
    m = block_max(m, red);
    float s = 0.0f;
    if (vec) {
      for (int j = threadIdx.x; j < width / 4; j += blockDim.x) {
        const float4 v = ((const float4*)xr)[j];
        const int c = 4 * j;
        s += expf((c + 0 > qi ? -1.0e4f : v.x) - m);
        s += expf((c + 1 > qi ? -1.0e4f : v.y) - m);
        s += expf((c + 2 > qi ? -1.0e4f : v.z) - m);
        s += expf((c + 3 > qi ? -1.0e4f : v.w) - m);
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) s += expf((j > qi ? -1.0e4f : xr[j]) - m);
    }
    const float d = fmaxf(block_sum(s, red), 1.1920928955078125e-7f);
    if (leak != nullptr && threadIdx.x == 0) leak[r] = masked_leak(qi, width, expf(-1.0e4f - m) == 0.0f, m, d);
    if (vec) {
      for (int j = threadIdx.x; j < width / 4; j += blockDim.x) {
        const float4 v = ((const float4*)xr)[j];
        const int c = 4 * j;
        float4 o;
        o.x = expf((c + 0 > qi ? -1.0e4f : v.x) - m) / d;
        o.y = expf((c + 1 > qi ? -1.0e4f : v.y) - m) / d;
        o.z = expf((c + 2 > qi ? -1.0e4f : v.z) - m) / d;
        o.w = expf((c + 3 > qi ? -1.0e4f : v.w) - m) / d;
        ((float4*)yr)[j] = o;
        if (lo) ((float4*)(lo + r * width))[j] = lo_part4(o);
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) {
        const float p = expf((j > qi ? -1.0e4f : xr[j]) - m) / d;
        yr[j] = p;
        if (lo) lo[r * width + j] = lo_part(p);
      }
    }
  }
}

// Row-wise form of masked_softmax_backward_kernel for k % 4 == 0 and 16-byte
// aligned buffers: one warp per row (grid-stride over rows), so the causal
// bound qi = r % q is computed once per row and the lanes walk only the
// float4 groups that hold data (col <= qi), plus the zero groups above the
// diagonal when they must be stored.  Same arithmetic per element.
__global__ void __launch_bounds__(256) masked_softmax_backward_rows_kernel(
    const float4* __restrict__ y, const float4* __restrict__ g, float4* __restrict__ dx, int64_t rows,
    int64_t q, int k4, int accumulate, float4* __restrict__ lo, int skip_zero) {
  const int lane = threadIdx.x & 31;
  const bool store_zero = !(skip_zero || (accumulate && lo == nullptr));
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int qi = (int)(r % q);
    const int data_end = min(k4, (qi >> 2) + 1);  // groups holding a col <= qi
    const int end = store_zero ? k4 : data_end;
    const int64_t base = r * k4;
    for (int j0 = 0; j0 < end; j0 += 32 * 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + 32 * u + lane;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < data_end) {
          const float4 yv = y[base + j], gv = g[base + j];
          const int col = 4 * j;
          v[u].x = (yv.x * (1.0f - yv.x)) * gv.x;
          v[u].y = col + 1 > qi ? 0.0f : (yv.y * (1.0f - yv.y)) * gv.y;
          v[u].z = col + 2 > qi ? 0.0f : (yv.z * (1.0f - yv.z)) * gv.z;
          v[u].w = col + 3 > qi ? 0.0f : (yv.w * (1.0f - yv.w)) * gv.w;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = j0 + 32 * u + lane;
        if (j >= end) continue;
        float4 t = v[u];
        if (accumulate) {
          const float4 o = dx[base + j];
          t = make_float4(o.x + t.x, o.y + t.y, o.z + t.z, o.w + t.w);
        }
        dx[base + j] = t;
        if (lo) lo[base + j] = lo_part4(t);
      }
    }
  }
}

__global__ void masked_softmax_backward_kernel(const float* __restrict__ y, const float* __restrict__ g,
                                               float* __restrict__ dx, int64_t n, int64_t q, int64_t k,
                                               int accumulate, float* __restrict__ lo, int skip_zero) {
  const bool vec = (k & 3) == 0 && aligned16(y) && aligned16(g) && aligned16(dx) && (lo == nullptr || aligned16(lo));
  if (vec) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i << 2;
      const int64_t col = e % k, row = (e / k) % q;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col <= row) {  // groups wholly above the diagonal read nothing
        const float4 yv = ((const float4*)y)[i], gv = ((const float4*)g)[i];
        v.x = (yv.x * (1.0f - yv.x)) * gv.x;
        v.y = col + 1 > row ? 0.0f : (yv.y * (1.0f - yv.y)) * gv.y;
        v.z = col + 2 > row ? 0.0f : (yv.z * (1.0f - yv.z)) * gv.z;
        v.w = col + 3 > row ? 0.0f : (yv.w * (1.0f - yv.w)) * gv.w;
      } else if (skip_zero || (accumulate && lo == nullptr)) {
        continue;  // the buffers already hold zero there, or this adds zero
      }
      if (accumulate) {
        const float4 o = ((float4*)dx)[i];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      ((float4*)dx)[i] = v;
      if (lo) ((float4*)lo)[i] = lo_part4(v);
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t col = i % k, row = (i / k) % q;
      const float v = col > row ? 0.0f : (y[i] * (1.0f - y[i])) * g[i];
      const float r = accumulate ? dx[i] + v : v;
      dx[i] = r;
      if (lo) lo[i] = lo_part(r);
    }
  }
}

// Row statistics in one read of the row: m = max_j x_j and
// d = max(sum_j exp(x_j - m), f32::EPSILON), kept per thread as a running
// (max, sum) pair rescaled when the max grows, then merged across the
// block.  kCeUnroll float4 per thread are in flight per iteration.
constexpr int kCeUnroll = 4;
constexpr int kCeGradUnroll = 2;  // the gradient pass holds x, t and the old gradient per float4

__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;  // both empty
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

__device__ __forceinline__ void ms_add4(float& m, float& s, float4 v) {
  const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
  if (mx > m) {
    s = s * expf(m - mx);
    m = mx;
  }
  s += expf(v.x - m);
  s += expf(v.y - m);
  s += expf(v.z - m);
  s += expf(v.w - m);
}

// The block's (max, sum of exp(x - max)) from each thread's pair; every
// thread gets (m, max(d, f32::EPSILON)).  `red` holds >= 66 floats.
__device__ void block_ms(float m, float s, float* red, float* m_out, float* d_out) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    ms_merge(m, s, m2, s2);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (lane == 0) {
    red[w] = m;
    red[32 + w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = lane < nw ? red[lane] : -INFINITY;
    s = lane < nw ? red[32 + lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      ms_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      red[64] = m;
      red[65] = s;
    }
  }
  __syncthreads();
  *m_out = red[64];
  *d_out = fmaxf(red[65], 1.1920928955078125e-7f);  // max(sum, f32::EPSILON)
}

// `red` holds >= 66 floats.  Every thread gets (m, d).
__device__ void row_stats(const float* __restrict__ xr, int width, bool vec, float* red, float* m_out,
                          float* d_out) {
  float m = -INFINITY, s = 0.0f;
  if (vec) {
    const float4* x4 = (const float4*)xr;
    const int n4 = width >> 2;
    int j = threadIdx.x;
    for (; j + (kCeUnroll - 1) * (int)blockDim.x < n4; j += kCeUnroll * blockDim.x) {
      float4 v[kCeUnroll];
#pragma unroll
      for (int u = 0; u < kCeUnroll; ++u) v[u] = x4[j + u * blockDim.x];
#pragma unroll
      for (int u = 0; u < kCeUnroll; ++u) ms_add4(m, s, v[u]);
    }
    for (; j < n4; j += blockDim.x) ms_add4(m, s, x4[j]);
  } else {
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float v = xr[j];
      if (v > m) {
        s = s * expf(m - v);
        m = v;
      }
      s += expf(v - m);
    }
  }
  block_ms(m, s, red, m_out, d_out);
}

// loss[r] = -sum_j t_j * ln(max(p_j, 1e-6)), p = softmax(x_r)  (layers.rs:301-324)
__global__ void __launch_bounds__(512, 2) cross_entropy_kernel(const float* __restrict__ logits,
                                     const float* __restrict__ target, float* __restrict__ loss,
                                     int64_t rows, int width) {
  __shared__ float red[66];
  const bool vec = (width & 3) == 0 && aligned16(logits) && aligned16(target);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    const float* tr = target + r * width;
    float m, d;
    row_stats(xr, width, vec, red, &m, &d);
    // ln(max(p, 1e-6)) with ln p = (x - m) - ln d: one subtraction per
    // element instead of exp, divide and log (ln is monotonic, so the clamp
    // moves to the log side).
    const float logd = logf(d), lclamp = logf(1e-6f);
    float acc = 0.0f;
    if (vec) {
      const int n4 = width >> 2;
      int j = threadIdx.x;
      for (; j + (kCeUnroll - 1) * (int)blockDim.x < n4; j += kCeUnroll * blockDim.x) {
        float4 x[kCeUnroll], t[kCeUnroll];
#pragma unroll
        for (int u = 0; u < kCeUnroll; ++u) {
          x[u] = ((const float4*)xr)[j + u * blockDim.x];
          t[u] = ((const float4*)tr)[j + u * blockDim.x];
        }
#pragma unroll
        for (int u = 0; u < kCeUnroll; ++u) {
          acc += t[u].x * fmaxf((x[u].x - m) - logd, lclamp);
          acc += t[u].y * fmaxf((x[u].y - m) - logd, lclamp);
          acc += t[u].z * fmaxf((x[u].z - m) - logd, lclamp);
          acc += t[u].w * fmaxf((x[u].w - m) - logd, lclamp);
        }
      }
      for (; j < n4; j += blockDim.x) {
        const float4 x = ((const float4*)xr)[j], t = ((const float4*)tr)[j];
        acc += t.x * fmaxf((x.x - m) - logd, lclamp);
        acc += t.y * fmaxf((x.y - m) - logd, lclamp);
        acc += t.z * fmaxf((x.z - m) - logd, lclamp);
        acc += t.w * fmaxf((x.w - m) - logd, lclamp);
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x)
        acc += tr[j] * fmaxf((xr[j] - m) - logd, lclamp);
    }
    acc = block_sum(acc, red);
    if (threadIdx.x == 0) loss[r] = 0.0f - acc;
  }
}

// Writes softmax(x_r) - t_r into grad_r (or adds it), where t_r is the dense
// target row or, with labels, the one-hot row of label `lab`.  The row was
// just read by row_stats, so x comes from L2 here; kCeUnroll float4 per
// thread are loaded ahead of their use.
// softmax - target with the row's 1/d precomputed (within one rounding of
// exp(x - m) / d).
__device__ __forceinline__ float4 ce_grad4(float4 x, float4 t, float m, float inv_d) {
  return make_float4(expf(x.x - m) * inv_d - t.x, expf(x.y - m) * inv_d - t.y, expf(x.z - m) * inv_d - t.z,
                     expf(x.w - m) * inv_d - t.w);
}

__device__ __forceinline__ float4 onehot4(int c, long long lab) {
  return make_float4(c == lab ? 1.0f : 0.0f, c + 1 == lab ? 1.0f : 0.0f, c + 2 == lab ? 1.0f : 0.0f,
                     c + 3 == lab ? 1.0f : 0.0f);
}

__device__ __forceinline__ void ce_grad_row(const float* __restrict__ xr, const float* __restrict__ tr,
                                            long long lab, float* __restrict__ gr, int width, bool vec,
                                            float m, float d, int accumulate) {
  const float inv_d = 1.0f / d;
  if (vec) {
    const int n4 = width >> 2;
    const float4* x4 = (const float4*)xr;
    const float4* t4 = (const float4*)tr;
    float4* g4 = (float4*)gr;
    int j = threadIdx.x;
    for (; j + (kCeGradUnroll - 1) * (int)blockDim.x < n4; j += kCeGradUnroll * blockDim.x) {
      float4 x[kCeGradUnroll], t[kCeGradUnroll], o[kCeGradUnroll];
#pragma unroll
      for (int u = 0; u < kCeGradUnroll; ++u) {
        const int jj = j + u * blockDim.x;
        x[u] = x4[jj];
        t[u] = tr ? t4[jj] : onehot4(4 * jj, lab);
        o[u] = accumulate ? g4[jj] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kCeGradUnroll; ++u) {
        float4 v = ce_grad4(x[u], t[u], m, inv_d);
        if (accumulate) v = make_float4(o[u].x + v.x, o[u].y + v.y, o[u].z + v.z, o[u].w + v.w);
        g4[j + u * blockDim.x] = v;
      }
    }
    for (; j < n4; j += blockDim.x) {
      float4 v = ce_grad4(x4[j], tr ? t4[j] : onehot4(4 * j, lab), m, inv_d);
      if (accumulate) {
        const float4 o = g4[j];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      g4[j] = v;
    }
  } else {
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float t = tr ? tr[j] : (j == lab ? 1.0f : 0.0f);
      const float v = expf(xr[j] - m) / d - t;
      gr[j] = accumulate ? gr[j] + v : v;
    }
  }
}

__global__ void __launch_bounds__(512, 3) cross_entropy_backward_kernel(const float* __restrict__ logits,
                                              const float* __restrict__ target,
                                              float* __restrict__ grad, int64_t rows, int width,
                                              int accumulate) {
  __shared__ float red[66];
  const bool vec = (width & 3) == 0 && aligned16(logits) && aligned16(target) && aligned16(grad);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float m, d;
    row_stats(logits + r * width, width, vec, red, &m, &d);
    ce_grad_row(logits + r * width, target + r * width, -1, grad + r * width, width, vec, m, d, accumulate);
  }
}

__global__ void __launch_bounds__(512, 4) cross_entropy_labels_kernel(const float* __restrict__ logits,
                                            const float* __restrict__ labels,
                                            float* __restrict__ loss, int64_t rows, int width,
                                            int* err) {
  __shared__ float red[66];
  const bool vec = (width & 3) == 0 && aligned16(logits);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    float m, d;
    row_stats(xr, width, vec, red, &m, &d);
    if (threadIdx.x == 0) {
      const long long lab = rust_f32_to_i64(labels[r]);
      if (lab < 0 || lab >= width) {
        atomicCAS(err, 0, (int)kErrIndexRange);
        loss[r] = NAN;
      } else {
        const float p = fmaxf(expf(xr[lab] - m) / d, 1e-6f);
        loss[r] = 0.0f - 1.0f * logf(p);
      }
    }
  }
}

__global__ void __launch_bounds__(512, 3) cross_entropy_labels_backward_kernel(const float* __restrict__ logits,
                                                     const float* __restrict__ labels,
                                                     float* __restrict__ grad, int64_t rows,
                                                     int width, int accumulate, int* err) {
  __shared__ float red[66];
  const bool vec = (width & 3) == 0 && aligned16(logits) && aligned16(grad);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const long long lab = rust_f32_to_i64(labels[r]);
    if (lab < 0 || lab >= width) {
      if (threadIdx.x == 0) atomicCAS(err, 0, (int)kErrIndexRange);
      continue;
    }
    float m, d;
    row_stats(logits + r * width, width, vec, red, &m, &d);
    ce_grad_row(logits + r * width, nullptr, lab, grad + r * width, width, vec, m, d, accumulate);
  }
}

// ---- gathers, copies, masks, rotations --------------------------------------------

__global__ void embedding_kernel(const float* __restrict__ idx, const float* __restrict__ w,
                                 float* __restrict__ out, int64_t count, int64_t num, int64_t dim,
                                 int* err) {
  const bool vec = (dim & 3) == 0 && aligned16(w) && aligned16(out);
  for (int64_t t = blockIdx.x; t < count; t += gridDim.x) {
    const long long r = rust_f32_to_i64(idx[t]);
    if (r < 0 || r >= num) {
      if (threadIdx.x == 0) atomicCAS(err, 0, (int)kErrIndexRange);
      continue;
    }
    const float* src = w + r * dim;
    float* dst = out + t * dim;
    if (vec) {
      for (int64_t j = threadIdx.x; j < dim / 4; j += blockDim.x)
        ((float4*)dst)[j] = ((const float4*)src)[j];
    } else {
      for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) dst[j] = src[j];
    }
  }
}

__global__ void emb_count_kernel(const float* idx, int64_t count, int64_t num, int* counts) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < count;
       t += (int64_t)gridDim.x * blockDim.x) {
    const long long r = rust_f32_to_i64(idx[t]);
    if (r >= 0 && r < num) atomicAdd(&counts[r], 1);
  }
}

// Single-block exclusive scan of counts -> offsets (and cursor = offsets).
__global__ void emb_scan_kernel(const int* counts, int* offsets, int* cursor, int64_t num) {
  __shared__ int buf[1024];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < num; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const int v = i < num ? counts[i] : 0;
    buf[threadIdx.x] = v;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
      int add = threadIdx.x >= o ? buf[threadIdx.x - o] : 0;
      __syncthreads();
      buf[threadIdx.x] += add;
      __syncthreads();
    }
    if (i < num) {
      const int excl = carry + buf[threadIdx.x] - v;
      offsets[i] = excl;
      cursor[i] = excl;
    }
    __syncthreads();
    if (threadIdx.x == 1023) carry += buf[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) offsets[num] = carry;
}

__global__ void emb_scatter_kernel(const float* idx, int64_t count, int64_t num, int* cursor,
                                   int* list) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < count;
       t += (int64_t)gridDim.x * blockDim.x) {
    const long long r = rust_f32_to_i64(idx[t]);
    if (r >= 0 && r < num) list[atomicAdd(&cursor[r], 1)] = (int)t;
  }
}

// Sorts each row's token list ascending (lists are short: insertion sort).
__global__ void emb_sort_kernel(const int* offsets, int* list, int64_t num) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < num;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int b = offsets[r], e = offsets[r + 1];
    for (int i = b + 1; i < e; ++i) {
      const int key = list[i];
      int j = i - 1;
      while (j >= b && list[j] > key) {
        list[j + 1] = list[j];
        --j;
      }
      list[j + 1] = key;
    }
  }
}

__global__ void emb_accumulate_kernel(const float* __restrict__ grad, const int* offsets,
                                      const int* list, float* __restrict__ wgrad, int64_t num,
                                      int64_t dim, int accumulate) {
  for (int64_t r = blockIdx.x; r < num; r += gridDim.x) {
    const int b = offsets[r], e = offsets[r + 1];
    for (int64_t j = threadIdx.x; j < dim; j += blockDim.x) {
      float acc = 0.0f;
      for (int i = b; i < e; ++i) acc = acc + grad[(int64_t)list[i] * dim + j];
      float* dst = wgrad + r * dim + j;
      *dst = accumulate ? *dst + acc : acc;
    }
  }
}

// out[o][h][e] = x[o][h / repeats][e] over rows of `inner` values.  seq > 0:
// x is stored [outer][seq][heads][inner / seq] instead (the layout before a
// transpose(1, 2), folded here), so row h of out gathers its positions from
// x's head h / repeats.
__device__ __forceinline__ int64_t kv_src(int64_t o, int64_t kvh, int64_t e, int64_t heads, int64_t inner,
                                          int64_t seq) {
  if (seq == 0) return (o * heads + kvh) * inner + e;
  const int64_t hd = inner / seq, p = e / hd, d = e - p * hd;
  return ((o * seq + p) * heads + kvh) * hd + d;
}

__global__ void repeat_kv_kernel(const float* __restrict__ x, float* __restrict__ out,
                                 int64_t outer, int64_t heads, int64_t inner, int64_t repeats, int64_t seq) {
  const int64_t out_heads = heads * repeats;
  const int64_t n = outer * out_heads * inner;
  const bool vec = (inner & 3) == 0 && (seq == 0 || ((inner / seq) & 3) == 0) && aligned16(x) && aligned16(out);
  if (vec) {
    const int64_t inner4 = inner >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i % inner4, row = i / inner4;
      const int64_t o = row / out_heads, dh = row % out_heads;
      ((float4*)out)[i] = *(const float4*)(x + kv_src(o, dh / repeats, 4 * e, heads, inner, seq));
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i % inner, row = i / inner;
      const int64_t o = row / out_heads, dh = row % out_heads;
      out[i] = x[kv_src(o, dh / repeats, e, heads, inner, seq)];
    }
  }
}

// dx[o][h][e] (+)= sum over r in order of g[o][h * repeats + r][e]; with
// seq > 0, dx is stored [outer][seq][heads][inner / seq].  Four values per
// thread when the rows allow float4 accesses.
__global__ void repeat_kv_backward_kernel(const float* __restrict__ g, float* __restrict__ dx,
                                          int64_t outer, int64_t heads, int64_t inner,
                                          int64_t repeats, int accumulate, int64_t seq) {
  const int64_t n = outer * heads * inner;
  const int64_t out_heads = heads * repeats;
  const bool vec = (inner & 3) == 0 && (seq == 0 || ((inner / seq) & 3) == 0) && aligned16(g) && aligned16(dx);
  if (vec) {
    const int64_t inner4 = inner >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i % inner4, row = i / inner4;
      const int64_t o = row / heads, h = row % heads;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int64_t r = 0; r < repeats; ++r) {
        const float4 v = ((const float4*)g)[(o * out_heads + h * repeats + r) * inner4 + e];
        acc = make_float4(acc.x + v.x, acc.y + v.y, acc.z + v.z, acc.w + v.w);
      }
      float4* d = (float4*)(dx + kv_src(o, h, 4 * e, heads, inner, seq));
      if (accumulate) {
        const float4 p = *d;
        acc = make_float4(p.x + acc.x, p.y + acc.y, p.z + acc.z, p.w + acc.w);
      }
      *d = acc;
    }
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i % inner, row = i / inner;
    const int64_t o = row / heads, h = row % heads;
    float acc = 0.0f;
    for (int64_t r = 0; r < repeats; ++r) acc = acc + g[(o * out_heads + h * repeats + r) * inner + e];
    float* d = dx + kv_src(o, h, e, heads, inner, seq);
    *d = accumulate ? *d + acc : acc;
  }
}

__global__ void causal_mask_kernel(const float* __restrict__ x, float* __restrict__ out,
                                   int64_t n, int64_t q, int64_t k, float fill, int backward,
                                   int accumulate) {
  const bool vec = (k & 3) == 0 && aligned16(x) && aligned16(out);
  if (vec) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i << 2;
      const int64_t col = e % k, row = (e / k) % q;
      float4 v = ((const float4*)x)[i];
      if (col + 0 > row) v.x = fill;
      if (col + 1 > row) v.y = fill;
      if (col + 2 > row) v.z = fill;
      if (col + 3 > row) v.w = fill;
      if (accumulate) {
        float4 o = ((float4*)out)[i];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      ((float4*)out)[i] = v;
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t col = i % k, row = (i / k) % q;
      const float v = col > row ? fill : x[i];
      out[i] = accumulate ? out[i] + v : v;
    }
  }
  (void)backward;
}

// Row `rp` (= o * seq + p, o = b * H + h) of a [B, H, seq, hd] tensor, as
// a row of the same tensor stored [B, seq, H, hd] when hs = H (the layout
// before transpose(1, 2)), or unchanged when hs = 0.
__device__ __forceinline__ int64_t head_row(int64_t rp, int64_t seq, int64_t hs) {
  if (hs == 0) return rp;
  const int64_t o = rp / seq, p = rp - o * seq;
  const int64_t b = o / hs, h = o - b * hs;
  return (b * seq + p) * hs + h;
}

// RoPE over rows of hd = 2 * half (rotate-half pairs f, f + half at
// position p = row % seq).  in_hs / out_hs: the input / output is stored
// [B, seq, H, hd] (head_row), which folds a transpose(1, 2) beside it.  Four
// pairs per thread with float4 accesses when half % 4 == 0 and the buffers
// are 16-byte aligned; the same products and sums per element either way.
__device__ __forceinline__ void rope_pair(float a, float b, float2 cs, int backward, float* y1, float* y2) {
  if (!backward) {
    const float t1 = a * cs.x, t2 = b * cs.y;
    const float t3 = a * cs.y, t4 = b * cs.x;
    *y1 = t1 - t2;
    *y2 = t3 + t4;
  } else {
    const float t1 = a * cs.x, t2 = b * cs.y;
    const float t3 = (-a) * cs.y, t4 = b * cs.x;
    *y1 = t1 + t2;
    *y2 = t3 + t4;
  }
}

__global__ void rope_kernel(const float* __restrict__ x, float* __restrict__ out,
                            const float2* __restrict__ table, int64_t outer, int64_t seq,
                            int64_t half, int backward, int accumulate, int64_t in_hs, int64_t out_hs) {
  const int64_t hd = 2 * half;
  if ((half & 3) == 0 && aligned16(x) && aligned16(out) && aligned16(table)) {
    const int64_t q4 = half >> 2;
    const int64_t n = outer * seq * q4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t f = 4 * (i % q4), rp = i / q4;
      const int64_t p = rp % seq;
      const float4 c01 = *(const float4*)(table + p * half + f);
      const float4 c23 = *(const float4*)(table + p * half + f + 2);
      const int64_t ib = head_row(rp, seq, in_hs) * hd, ob = head_row(rp, seq, out_hs) * hd;
      const float4 a = *(const float4*)(x + ib + f), b = *(const float4*)(x + ib + half + f);
      float4 y1, y2;
      rope_pair(a.x, b.x, make_float2(c01.x, c01.y), backward, &y1.x, &y2.x);
      rope_pair(a.y, b.y, make_float2(c01.z, c01.w), backward, &y1.y, &y2.y);
      rope_pair(a.z, b.z, make_float2(c23.x, c23.y), backward, &y1.z, &y2.z);
      rope_pair(a.w, b.w, make_float2(c23.z, c23.w), backward, &y1.w, &y2.w);
      float4* o1 = (float4*)(out + ob + f);
      float4* o2 = (float4*)(out + ob + half + f);
      if (accumulate) {
        const float4 p1 = *o1, p2 = *o2;
        y1 = make_float4(p1.x + y1.x, p1.y + y1.y, p1.z + y1.z, p1.w + y1.w);
        y2 = make_float4(p2.x + y2.x, p2.y + y2.y, p2.z + y2.z, p2.w + y2.w);
      }
      *o1 = y1;
      *o2 = y2;
    }
    return;
  }
  const int64_t n = outer * seq * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = i % half, rp = i / half;  // rp = o*seq + p
    const int64_t p = rp % seq;
    const float2 cs = table[p * half + f];
    const int64_t ib = head_row(rp, seq, in_hs) * hd, ob = head_row(rp, seq, out_hs) * hd;
    float y1, y2;
    rope_pair(x[ib + f], x[ib + half + f], cs, backward, &y1, &y2);
    if (accumulate) {
      out[ob + f] = out[ob + f] + y1;
      out[ob + half + f] = out[ob + half + f] + y2;
    } else {
      out[ob + f] = y1;
      out[ob + half + f] = y2;
    }
  }
}

struct Dims8 {
  int64_t d[8];
};

// General axis swap: each output element reads its source.  When the
// innermost axis is untouched, whole inner runs of `inner` elements move
// together (4-wide when aligned).
__global__ void transpose_kernel(const float* __restrict__ x, float* __restrict__ out,
                                 Dims8 out_dims, Dims8 in_strides, int rank, int a, int b,
                                 int64_t n, int64_t inner, int accumulate) {
  const bool vec = (inner & 3) == 0 && aligned16(x) && aligned16(out) && inner > 1;
  const int64_t w = vec ? 4 : 1;
  for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * w; i < n;
       i += (int64_t)gridDim.x * blockDim.x * w) {
    int64_t rem = i, src = 0;
    for (int d = rank - 1; d >= 0; --d) {
      const int64_t c = rem % out_dims.d[d];
      rem /= out_dims.d[d];
      const int sd = d == a ? b : (d == b ? a : d);
      src += c * in_strides.d[sd];
    }
    if (vec) {
      float4 v = *(const float4*)(x + src);
      if (accumulate) {
        float4 o = *(float4*)(out + i);
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      *(float4*)(out + i) = v;
    } else {
      out[i] = accumulate ? out[i] + x[src] : x[src];
    }
  }
}

// The same axis swap when the axes after the later swapped one hold a run
// of T4 float4 (16-byte aligned): x is [P][A][Mid][B][run], out is
// [P][B][Mid][A][run].  One warp per run: the run's source is found once
// (three divisions per run, not per element) and its lanes copy it.
__global__ void transpose_runs_kernel(const float4* __restrict__ x, float4* __restrict__ out, int64_t A,
                                      int64_t mid, int64_t B, int64_t runs, int t4, int accumulate) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < runs; r += warps) {
    // r = ((p * B + j) * mid + m) * A + i over the output.
    int64_t q = r;
    const int64_t i = q % A;
    q /= A;
    const int64_t m = q % mid;
    q /= mid;
    const int64_t j = q % B;
    const int64_t p = q / B;
    const int64_t src = ((p * A + i) * mid + m) * B + j;
    const float4* xs = x + src * t4;
    float4* os = out + r * t4;
    for (int k = lane; k < t4; k += 32) {
      float4 v = xs[k];
      if (accumulate) {
        const float4 o = os[k];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      os[k] = v;
    }
  }
}

// partial[c][j] = sum of grad rows [c*rpc, (c+1)*rpc) in column j, rows in order.
__global__ void colsum_partial_kernel(const float* __restrict__ g, float* __restrict__ partial,
                                      int64_t rows, int64_t width, int64_t rows_per_chunk) {
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t c = blockIdx.y;
  if (j >= width) return;
  const int64_t r0 = c * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  float acc = 0.0f;
  for (int64_t r = r0; r < r1; ++r) acc = acc + g[r * width + j];
  partial[c * width + j] = acc;
}

__global__ void reduce_partial_kernel(const float* __restrict__ x, float* __restrict__ partial,
                                      int64_t n) {
  __shared__ float red[33];
  float acc = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    acc += x[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

__global__ void reduce_final_kernel(const float* __restrict__ partial, float* out, int n) {
  __shared__ float red[33];
  float acc = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) out[0] = acc;
}

// The reference's tensor_sum (training/executor.rs:109-111): one f32
// accumulator adding x[0], x[1], ... in index order from 0.0, so the result
// rounds exactly as the reference's loss does.  One thread walks the whole
// tensor (each add waits for the previous one); it reads four float4 ahead
// of the adds so the loads overlap the chain.  Opt-in: a tree sum is
// typically closer to the exact sum, this one reproduces the reference.
__global__ void sequential_sum_kernel(const float* __restrict__ x, float* out, int64_t n) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float acc = 0.0f;
  int64_t i = 0;
  if ((((uintptr_t)x) & 15) == 0) {
    const float4* v = reinterpret_cast<const float4*>(x);
    const int64_t nv = n / 4;
    int64_t j = 0;
    for (; j + 4 <= nv; j += 4) {
      const float4 a = v[j], b = v[j + 1], c = v[j + 2], d = v[j + 3];
      acc = acc + a.x; acc = acc + a.y; acc = acc + a.z; acc = acc + a.w;
      acc = acc + b.x; acc = acc + b.y; acc = acc + b.z; acc = acc + b.w;
      acc = acc + c.x; acc = acc + c.y; acc = acc + c.z; acc = acc + c.w;
      acc = acc + d.x; acc = acc + d.y; acc = acc + d.z; acc = acc + d.w;
    }
    for (; j < nv; ++j) {
      const float4 a = v[j];
      acc = acc + a.x; acc = acc + a.y; acc = acc + a.z; acc = acc + a.w;
    }
    i = nv * 4;
  }
  for (; i < n; ++i) acc = acc + x[i];
  out[0] = acc;
}

int row_threads(int64_t width) {
  if (width >= 8192) return 1024;
  if (width >= 2048) return 512;
  if (width >= 256) return 256;
  return 128;
}

int row_blocks(int64_t rows) { return (int)(rows < 148 * 64 ? (rows < 1 ? 1 : rows) : 148 * 64); }

bool aligned16_host(const void* p) { return (((uintptr_t)p) & 15) == 0; }

// Loss rows: 512 threads with kCeUnroll float4 in flight each keep enough
// bytes outstanding while letting 4 rows share an SM.
int ce_threads(int64_t width) { return width >= 2048 ? 512 : row_threads(width); }

void check_launch() {
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace

void launch_pattern(float* out, int64_t n, int mod, float add, float div, cudaStream_t st) {
  if (n <= 0) return;
  pattern_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(out, n, mod, add, div);
  check_launch();
}

void launch_fill(float* out, int64_t n, float value, cudaStream_t st) {
  if (n <= 0) return;
  fill_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(out, n, value);
  check_launch();
}

void launch_unary(int op, const float* x, float* out, int64_t n, float param, cudaStream_t st) {
  if (n <= 0) return;
  const int blocks = elementwise_blocks((n + 3) / 4, kThreads);
  switch (op) {
    case kUnaryRelu: unary_kernel<kUnaryRelu><<<blocks, kThreads, 0, st>>>(x, out, n, param); break;
    case kUnarySilu: unary_kernel<kUnarySilu><<<blocks, kThreads, 0, st>>>(x, out, n, param); break;
    case kUnaryScale: unary_kernel<kUnaryScale><<<blocks, kThreads, 0, st>>>(x, out, n, param); break;
    case kUnaryNeg: unary_kernel<kUnaryNeg><<<blocks, kThreads, 0, st>>>(x, out, n, param); break;
    default: unary_kernel<-1><<<blocks, kThreads, 0, st>>>(x, out, n, param); break;
  }
  check_launch();
}

void launch_square_backward(const float* g, const float* x, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  square_backward_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(g, x, out, n);
  check_launch();
}

void launch_binary_tt(int op, const float* a, const float* b, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  binary_tt_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(op, a, b, out, n);
  check_launch();
}

void launch_binary_ts(int op, const float* a, float s, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  binary_ts_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(op, a, s, out, n, 0);
  check_launch();
}

void launch_binary_st(int op, float s, const float* b, float* out, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  binary_ts_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(op, b, s, out, n, 1);
  check_launch();
}

void launch_add_inplace(float* dst, const float* src, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  add_inplace_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(dst, src, n);
  check_launch();
}

void launch_binary_tt_acc(int op, const float* a, const float* b, float* dst, int64_t n,
                          cudaStream_t st) {
  if (n <= 0) return;
  binary_acc_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(op, a, b, 0.0f, 0, dst, n);
  check_launch();
}

void launch_binary_ts_acc(int op, const float* a, float s, float* dst, int64_t n, int scalar_first,
                          cudaStream_t st) {
  if (n <= 0) return;
  binary_acc_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(
      op, a, nullptr, s, scalar_first ? 2 : 1, dst, n);
  check_launch();
}

void launch_div_rhs_grad(const float* g, const float* lhs, const float* rhs, float* dst, int64_t n,
                         int accumulate, cudaStream_t st) {
  if (n <= 0) return;
  div_rhs_grad_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(g, lhs, rhs, dst, n,
                                                                            accumulate);
  check_launch();
}

void launch_relu_backward(const float* y, const float* g, float* dx, int64_t n, int acc,
                          cudaStream_t st) {
  if (n <= 0) return;
  relu_backward_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(y, g, dx, n, acc);
  check_launch();
}

void launch_silu_mul(const float* x, const float* u, float* h, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  silu_mul_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(x, u, h, n);
  check_launch();
}

void launch_silu_mul_backward(const float* x, const float* u, const float* dh, float* dx, float* du, int64_t n,
                              int acc_x, int acc_u, cudaStream_t st) {
  if (n <= 0) return;
  silu_mul_backward_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(x, u, dh, dx, du, n, acc_x, acc_u);
  check_launch();
}

void launch_silu_backward(const float* x, const float* g, float* dx, int64_t n, int acc,
                          cudaStream_t st) {
  if (n <= 0) return;
  silu_backward_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(x, g, dx, n, acc);
  check_launch();
}

void launch_softmax_backward(const float* y, const float* g, float* dx, int64_t n, int acc,
                             cudaStream_t st) {
  if (n <= 0) return;
  softmax_backward_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(y, g, dx, n, acc);
  check_launch();
}

void launch_rms_norm(const float* x, float* out, int64_t rows, int64_t width, cudaStream_t st) {
  if (rows <= 0) return;
  rms_norm_kernel<<<row_blocks(rows), row_threads(width / 4), 0, st>>>(x, nullptr, out, rows,
                                                                        (int)width, 1e-5f);
  check_launch();
}

void launch_rms_norm_gain(const float* x, const float* g, float* out, int64_t rows, int64_t width,
                          float eps, cudaStream_t st) {
  if (rows <= 0) return;
  rms_norm_kernel<<<row_blocks(rows), row_threads(width / 4), 0, st>>>(x, g, out, rows,
                                                                        (int)width, eps);
  check_launch();
}

static int64_t rms_gain_rows_per_block(int64_t rows) {
  int64_t rpb = ceil_div(rows, 148 * 2);
  return rpb < 1 ? 1 : rpb;
}

int64_t rms_gain_partial_elems(int64_t rows, int64_t width) {
  return ceil_div(rows, rms_gain_rows_per_block(rows)) * width;
}

void launch_rms_norm_gain_backward(const float* x, const float* g, const float* dy, float* dx,
                                   float* dg, float* partial, int64_t rows, int64_t width,
                                   float eps, int acc_dx, int acc_dg, cudaStream_t st) {
  if (rows <= 0) return;
  const int64_t rpb = rms_gain_rows_per_block(rows);
  const int nb = (int)ceil_div(rows, rpb);
  const bool reg = width % 1024 == 0 && width / 1024 <= 8 && ((width / 1024) & (width / 1024 - 1)) == 0 &&
                   aligned16_host(x) && aligned16_host(g) && aligned16_host(dy) && aligned16_host(dx) &&
                   aligned16_host(partial);
  if (reg) {
    switch (width / 1024) {
      case 1: rms_gain_backward_reg_kernel<1><<<nb, 256, 0, st>>>(x, g, dy, dx, partial, rows, eps, acc_dx, (int)rpb); break;
      case 2: rms_gain_backward_reg_kernel<2><<<nb, 256, 0, st>>>(x, g, dy, dx, partial, rows, eps, acc_dx, (int)rpb); break;
      case 4: rms_gain_backward_reg_kernel<4><<<nb, 256, 0, st>>>(x, g, dy, dx, partial, rows, eps, acc_dx, (int)rpb); break;
      default: rms_gain_backward_reg_kernel<8><<<nb, 256, 0, st>>>(x, g, dy, dx, partial, rows, eps, acc_dx, (int)rpb); break;
    }
  } else {
    rms_gain_backward_kernel<<<nb, row_threads(width), 0, st>>>(x, g, dy, dx, partial, rows,
                                                                (int)width, eps, acc_dx, (int)rpb);
  }
  check_launch();
  sum_partials_kernel<<<(int)ceil_div(width, 128), 128, 0, st>>>(partial, dg, nb, (int)width, acc_dg);
  check_launch();
}

// Launches the register-resident form when the width allows; false if not.
bool softmax_reg(const float* x, float* out, int64_t rows, int64_t width, int64_t q, int masked,
                 float* leak, float* lo, int skip_zero, cudaStream_t st);

void launch_softmax(const float* x, float* out, int64_t rows, int64_t width, cudaStream_t st) {
  if (rows <= 0) return;
  if (softmax_reg(x, out, rows, width, 1, 0, nullptr, nullptr, 0, st)) return;
  softmax_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(x, out, rows, (int)width);
  check_launch();
}

bool softmax_reg(const float* x, float* out, int64_t rows, int64_t width, int64_t q, int masked,
                 float* leak, float* lo, int skip_zero, cudaStream_t st) {
  if (width % 1024 != 0 || !aligned16_host(x) || !aligned16_host(out) || (lo && !aligned16_host(lo))) return false;
  if (width == 1024 || width == 2048) {
    const int wpr = (int)(width / 1024);
    const int64_t want = (rows * wpr + 7) / 8;
    const int wblocks = (int)(want < 148 * 16 ? want : 148 * 16);
    // Two warps per 2048-wide row measured faster than one warp holding 16
    // float4 per lane (128 registers, half the resident warps) or four warps.
    if (width == 1024) softmax_warp_kernel<8, 1><<<wblocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero);
    else softmax_warp_kernel<8, 2><<<wblocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero);
    check_launch();
    return true;
  }
  const int blocks = row_blocks(rows);
  switch (width / 1024) {
    case 1: softmax_reg_kernel<1><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero); break;
    case 2: softmax_reg_kernel<2><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero); break;
    case 4: softmax_reg_kernel<4><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero); break;
    case 8: softmax_reg_kernel<8><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked, leak, lo, skip_zero); break;
    default: return false;
  }
  check_launch();
  return true;
}

// Causal attention rows whose masked entries keep a probability (leak[r] =
// c_r != 0, see masked_leak) lose terms where the causal GEMMs skip masked
// entries as zeros; these kernels add them back, one block per batch item
// (head).  A head none of whose rows leaks returns after reading its rows'
// leak values.
//
// mode 2, after O = P.V with GemmEpilogue::tri 2: row r was contracted over
// keys k < kend(r) = the end of its tile of tile_rows rows (rounded up to
// 16); the keys after that are all masked for r, each with probability c_r,
// so o[r] += c_r * sum_{k >= kend(r)} v[k].
// mode 3, after dV = P^T.dO with tri 3: output row j (a key) was contracted
// over queries from the start of its tile; the queries before it all mask
// key j, each with its own c_q, so dv[j] += sum_{q < start(j)} c_q * dO[q].
// `x` is the GEMM's B operand (v or dO; x_trans: stored [n, k]); `out` its
// output, rows = the GEMM's M, `kn` its K, `n` its N.
__global__ void causal_leak_fix_kernel(int mode, const float* __restrict__ leak, int lrows,
                                       const float* __restrict__ x, int x_trans, int64_t x_ld, int64_t x_bs,
                                       float* __restrict__ out, int64_t o_ld, int64_t o_bs, int rows, int kn, int n,
                                       int tile_rows) {
  const int b = blockIdx.x;
  const float* lk = leak + (int64_t)b * lrows;
  int any = 0;
  for (int r = threadIdx.x; r < lrows; r += blockDim.x) any |= lk[r] != 0.0f;
  if (!__syncthreads_or(any)) return;
  const float* xb = x + (int64_t)b * x_bs;
  float* ob = out + (int64_t)b * o_bs;
  auto xv = [&](int k, int d) { return x_trans ? xb[(int64_t)d * x_ld + k] : xb[(int64_t)k * x_ld + d]; };
  for (int d = threadIdx.x; d < n; d += blockDim.x) {
    if (mode == 2) {
      // Tiles from the last: the suffix sum over keys grows as kend falls.
      float acc = 0.0f;
      int kk = kn;
      const int last = ((rows - 1) / tile_rows) * tile_rows;
      for (int t0 = last; t0 >= 0; t0 -= tile_rows) {
        int kend = ((t0 + tile_rows + 15) / 16) * 16;
        if (kend > kn) kend = kn;
        while (kk > kend) acc = acc + xv(--kk, d);
        const int t1 = t0 + tile_rows < rows ? t0 + tile_rows : rows;
        for (int r = t0; r < t1; ++r) {
          const float c = lk[r];
          if (c != 0.0f) ob[(int64_t)r * o_ld + d] = ob[(int64_t)r * o_ld + d] + c * acc;
        }
      }
    } else {
      // Tiles from the first: the prefix sum over queries grows with start.
      float acc = 0.0f;
      int qq = 0;
      for (int t0 = 0; t0 < rows; t0 += tile_rows) {
        for (; qq < t0 && qq < kn; ++qq) {
          const float c = lk[qq];
          if (c != 0.0f) acc = acc + c * xv(qq, d);
        }
        if (acc == 0.0f) continue;
        const int t1 = t0 + tile_rows < rows ? t0 + tile_rows : rows;
        for (int j = t0; j < t1; ++j) ob[(int64_t)j * o_ld + d] = ob[(int64_t)j * o_ld + d] + acc;
      }
    }
  }
}

void launch_causal_leak_fix(int mode, const float* leak, int64_t lrows, const float* x, bool x_trans, int64_t x_ld,
                            int64_t x_bs, float* out, int64_t o_ld, int64_t o_bs, int batch, int64_t rows, int64_t kn,
                            int64_t n, int tile_rows, cudaStream_t st) {
  if (batch <= 0 || rows <= 0 || n <= 0 || tile_rows <= 0) return;
  if (mode != 2 && mode != 3) throw CudaError("causal leak fix: mode is 2 or 3");
  if (rows > INT32_MAX || kn > INT32_MAX || n > INT32_MAX || lrows > INT32_MAX) throw CudaError("causal leak fix: too large");
  causal_leak_fix_kernel<<<batch, 128, 0, st>>>(mode, leak, (int)lrows, x, x_trans ? 1 : 0, x_ld, x_bs, out, o_ld,
                                                 o_bs, (int)rows, (int)kn, (int)n, tile_rows);
  check_launch();
}

void launch_masked_softmax(const float* x, float* out, int64_t outer, int64_t q, int64_t k,
                           float* leak, float* lo, int skip_zero, cudaStream_t st) {
  const int64_t rows = outer * q;
  if (rows <= 0) return;
  if (softmax_reg(x, out, rows, k, q, 1, leak, lo, skip_zero, st)) return;
  masked_softmax_kernel<<<row_blocks(rows), row_threads(k / 4), 0, st>>>(x, out, rows, (int)q, (int)k, leak, lo);
  check_launch();
}

void launch_masked_softmax_backward(const float* y, const float* g, float* dx, int64_t outer,
                                    int64_t q, int64_t k, int accumulate, float* lo, int skip_zero,
                                    cudaStream_t st) {
  const int64_t n = outer * q * k;
  if (n <= 0) return;
  if (k % 4 == 0 && k / 4 <= INT32_MAX && aligned16_host(y) && aligned16_host(g) && aligned16_host(dx) &&
      (lo == nullptr || aligned16_host(lo))) {
    const int64_t rows = outer * q;
    const int64_t want = (rows + 7) / 8;
    const int blocks = (int)(want < 148 * 16 ? want : 148 * 16);
    masked_softmax_backward_rows_kernel<<<blocks, 256, 0, st>>>(
        (const float4*)y, (const float4*)g, (float4*)dx, rows, q, (int)(k / 4), accumulate, (float4*)lo,
        skip_zero);
    check_launch();
    return;
  }
  masked_softmax_backward_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      y, g, dx, n, q, k, accumulate, lo, skip_zero);
  check_launch();
}

void launch_cross_entropy(const float* logits, const float* target, float* loss, int64_t rows,
                          int64_t width, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_kernel<<<row_blocks(rows), ce_threads(width), 0, st>>>(logits, target, loss, rows,
                                                                        (int)width);
  check_launch();
}

void launch_cross_entropy_backward(const float* logits, const float* target, float* grad,
                                   int64_t rows, int64_t width, int accumulate, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_backward_kernel<<<row_blocks(rows), ce_threads(width), 0, st>>>(
      logits, target, grad, rows, (int)width, accumulate);
  check_launch();
}

void launch_cross_entropy_labels(const float* logits, const float* labels, float* loss,
                                 int64_t rows, int64_t width, int* err, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_labels_kernel<<<row_blocks(rows), ce_threads(width), 0, st>>>(
      logits, labels, loss, rows, (int)width, err);
  check_launch();
}

void launch_cross_entropy_labels_backward(const float* logits, const float* labels, float* grad,
                                          int64_t rows, int64_t width, int accumulate, int* err,
                                          cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_labels_backward_kernel<<<row_blocks(rows), ce_threads(width), 0, st>>>(
      logits, labels, grad, rows, (int)width, accumulate, err);
  check_launch();
}

void launch_embedding(const float* idx, const float* weight, float* out, int64_t count,
                      int64_t num, int64_t dim, int* err, cudaStream_t st) {
  if (count <= 0) return;
  embedding_kernel<<<row_blocks(count), dim >= 1024 ? 256 : 128, 0, st>>>(idx, weight, out, count,
                                                                          num, dim, err);
  check_launch();
}

size_t embedding_backward_work_bytes(int64_t count, int64_t num) {
  return sizeof(int) * (size_t)(3 * num + 1 + (count > 0 ? count : 1));
}

void launch_embedding_backward(const float* grad, const float* idx, float* wgrad, int64_t count,
                               int64_t num, int64_t dim, void* work, int accumulate,
                               cudaStream_t st) {
  if (num <= 0) return;
  int* counts = (int*)work;
  int* offsets = counts + num;    // num + 1 entries
  int* cursor = offsets + num + 1;
  int* list = cursor + num;
  TYSOR_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * (size_t)num, st));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (count > 0) {
    emb_count_kernel<<<elementwise_blocks(count, kThreads), kThreads, 0, st>>>(idx, count, num, counts);
    check_launch();
  }
  emb_scan_kernel<<<1, 1024, 0, st>>>(counts, offsets, cursor, num);
  check_launch();
  if (count > 0) {
    emb_scatter_kernel<<<elementwise_blocks(count, kThreads), kThreads, 0, st>>>(idx, count, num,
                                                                                cursor, list);
    check_launch();
    emb_sort_kernel<<<elementwise_blocks(num, kThreads), kThreads, 0, st>>>(offsets, list, num);
    check_launch();
  }
  emb_accumulate_kernel<<<row_blocks(num), dim >= 1024 ? 256 : 128, 0, st>>>(
      grad, offsets, list, wgrad, num, dim, accumulate);
  check_launch();
}

void launch_repeat_kv(const float* x, float* out, int64_t outer, int64_t heads, int64_t inner,
                      int64_t repeats, cudaStream_t st, int64_t seq) {
  const int64_t n = outer * heads * repeats * inner;
  if (n <= 0) return;
  repeat_kv_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      x, out, outer, heads, inner, repeats, seq);
  check_launch();
}

void launch_repeat_kv_backward(const float* g, float* dx, int64_t outer, int64_t heads,
                               int64_t inner, int64_t repeats, int accumulate, cudaStream_t st, int64_t seq) {
  const int64_t n = outer * heads * inner;
  if (n <= 0) return;
  repeat_kv_backward_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      g, dx, outer, heads, inner, repeats, accumulate, seq);
  check_launch();
}

void launch_causal_mask(const float* x, float* out, int64_t outer, int64_t q, int64_t k,
                        cudaStream_t st) {
  const int64_t n = outer * q * k;
  if (n <= 0) return;
  causal_mask_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      x, out, n, q, k, -1.0e4f, 0, 0);
  check_launch();
}

void launch_causal_mask_backward(const float* g, float* dx, int64_t outer, int64_t q, int64_t k,
                                 int accumulate, cudaStream_t st) {
  const int64_t n = outer * q * k;
  if (n <= 0) return;
  causal_mask_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      g, dx, n, q, k, 0.0f, 1, accumulate);
  check_launch();
}

void launch_rope(const float* x, float* out, const float2* table, int64_t outer, int64_t seq,
                 int64_t half, cudaStream_t st, int64_t in_hs) {
  const int64_t n = outer * seq * half;
  if (n <= 0) return;
  rope_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(x, out, table, outer, seq,
                                                                    half, 0, 0, in_hs, 0);
  check_launch();
}

void launch_rope_backward(const float* g, float* dx, const float2* table, int64_t outer,
                          int64_t seq, int64_t half, int accumulate, cudaStream_t st, int64_t out_hs) {
  const int64_t n = outer * seq * half;
  if (n <= 0) return;
  rope_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(g, dx, table, outer, seq, half,
                                                                    1, accumulate, 0, out_hs);
  check_launch();
}

void launch_transpose(const float* x, float* out, const int64_t* dims, int rank, int a, int b,
                      int accumulate, cudaStream_t st) {
  if (rank < 1 || rank > 8) throw CudaError("transpose supports rank 1..8");
  Dims8 od{}, is{};
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= dims[i];
  if (n <= 0) return;
  is.d[rank - 1] = 1;
  for (int i = rank - 2; i >= 0; --i) is.d[i] = is.d[i + 1] * dims[i + 1];
  for (int i = 0; i < rank; ++i) od.d[i] = dims[i];
  od.d[a] = dims[b];
  od.d[b] = dims[a];
  const int hi = a > b ? a : b, lo = a < b ? a : b;
  int64_t inner = 1;
  for (int i = hi + 1; i < rank; ++i) inner *= dims[i];
  if (lo != hi && inner % 4 == 0 && inner / 4 >= 8 && inner / 4 <= INT32_MAX && aligned16_host(x) &&
      aligned16_host(out)) {
    int64_t mid = 1;
    for (int i = lo + 1; i < hi; ++i) mid *= dims[i];
    const int64_t runs = n / inner;
    transpose_runs_kernel<<<elementwise_blocks(runs * 32, kThreads), kThreads, 0, st>>>(
        (const float4*)x, (float4*)out, dims[lo], mid, dims[hi], runs, (int)(inner / 4), accumulate);
  } else {
    transpose_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
        x, out, od, is, rank, a, b, n, inner, accumulate);
  }
  check_launch();
}

static int64_t colsum_rows_per_chunk(int64_t rows) {
  int64_t r = ceil_div(rows, 64);
  return r < 1 ? 1 : r;
}

int64_t colsum_partial_elems(int64_t rows, int64_t width) {
  return ceil_div(rows, colsum_rows_per_chunk(rows)) * width;
}

void launch_colsum(const float* g, float* out, float* partial, int64_t rows, int64_t width,
                   int accumulate, cudaStream_t st) {
  if (width <= 0) return;
  if (rows <= 0) {
    if (!accumulate) launch_fill(out, width, 0.0f, st);
    return;
  }
  const int64_t rpc = colsum_rows_per_chunk(rows);
  const int64_t chunks = ceil_div(rows, rpc);
  colsum_partial_kernel<<<dim3((unsigned)ceil_div(width, 256), (unsigned)chunks), 256, 0, st>>>(
      g, partial, rows, width, rpc);
  check_launch();
  sum_partials_kernel<<<(int)ceil_div(width, 128), 128, 0, st>>>(partial, out, (int)chunks,
                                                                  (int)width, accumulate);
  check_launch();
}

void launch_reduce_sum(const float* x, float* out, float* partial, int64_t n, cudaStream_t st) {
  int blocks = (int)(ceil_div(n, 1024) < 1024 ? ceil_div(n, 1024) : 1024);
  if (blocks < 1) blocks = 1;
  reduce_partial_kernel<<<blocks, 256, 0, st>>>(x, partial, n);
  check_launch();
  reduce_final_kernel<<<1, 1024, 0, st>>>(partial, out, blocks);
  check_launch();
}

void launch_sequential_sum(const float* x, float* out, int64_t n, cudaStream_t st) {
  sequential_sum_kernel<<<1, 32, 0, st>>>(x, out, n);
  check_launch();
}

void launch_sgd(float* p, const float* g, float lr, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  sgd_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(p, g, lr, n);
  check_launch();
}

}  // namespace tysor
