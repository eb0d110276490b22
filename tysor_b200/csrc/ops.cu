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

// Generic elementwise driver: F(i) computes element i; vectorised 4-wide
// when every pointer involved is 16-byte aligned.
template <typename F4, typename F1>
__device__ __forceinline__ void ew_loop(int64_t n, bool vec, F4 f4, F1 f1) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = n >> 2;
    for (int64_t i = t0; i < n4; i += stride) f4(i);
    done = n4 << 2;
  }
  for (int64_t i = done + t0; i < n; i += stride) f1(i);
}

__global__ void unary_kernel(int op, const float* __restrict__ x, float* __restrict__ out,
                             int64_t n, float p) {
  const bool vec = aligned16(x) && aligned16(out);
  ew_loop(
      n, vec,
      [&](int64_t i) {
        float4 v = ((const float4*)x)[i];
        v.x = apply_unary(op, v.x, p);
        v.y = apply_unary(op, v.y, p);
        v.z = apply_unary(op, v.z, p);
        v.w = apply_unary(op, v.w, p);
        ((float4*)out)[i] = v;
      },
      [&](int64_t i) { out[i] = apply_unary(op, x[i], p); });
}

__global__ void binary_tt_kernel(int op, const float* a, const float* b, float* out, int64_t n) {
  const bool vec = aligned16(a) && aligned16(b) && aligned16(out);
  ew_loop(
      n, vec,
      [&](int64_t i) {
        float4 u = ((const float4*)a)[i], v = ((const float4*)b)[i];
        ((float4*)out)[i] = make_float4(apply_binary(op, u.x, v.x), apply_binary(op, u.y, v.y),
                                        apply_binary(op, u.z, v.z), apply_binary(op, u.w, v.w));
      },
      [&](int64_t i) { out[i] = apply_binary(op, a[i], b[i]); });
}

__global__ void binary_ts_kernel(int op, const float* a, float s, float* out, int64_t n,
                                 int scalar_first) {
  const bool vec = aligned16(a) && aligned16(out);
  ew_loop(
      n, vec,
      [&](int64_t i) {
        float4 u = ((const float4*)a)[i];
        if (scalar_first)
          u = make_float4(apply_binary(op, s, u.x), apply_binary(op, s, u.y),
                          apply_binary(op, s, u.z), apply_binary(op, s, u.w));
        else
          u = make_float4(apply_binary(op, u.x, s), apply_binary(op, u.y, s),
                          apply_binary(op, u.z, s), apply_binary(op, u.w, s));
        ((float4*)out)[i] = u;
      },
      [&](int64_t i) {
        out[i] = scalar_first ? apply_binary(op, s, a[i]) : apply_binary(op, a[i], s);
      });
}

__global__ void add_inplace_kernel(float* dst, const float* src, int64_t n) {
  const bool vec = aligned16(dst) && aligned16(src);
  ew_loop(
      n, vec,
      [&](int64_t i) {
        float4 d = ((float4*)dst)[i], s = ((const float4*)src)[i];
        ((float4*)dst)[i] = make_float4(d.x + s.x, d.y + s.y, d.z + s.z, d.w + s.w);
      },
      [&](int64_t i) { dst[i] = dst[i] + src[i]; });
}

__global__ void binary_acc_kernel(int op, const float* a, const float* b, float s, int mode,
                                  float* dst, int64_t n) {
  // mode 0: op(a[i], b[i]); 1: op(a[i], s); 2: op(s, a[i])
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = mode == 0 ? apply_binary(op, a[i], b[i])
                              : (mode == 1 ? apply_binary(op, a[i], s) : apply_binary(op, s, a[i]));
    dst[i] = dst[i] + v;
  }
}

__global__ void div_rhs_grad_kernel(const float* g, const float* l, const float* r, float* dst,
                                    int64_t n, int accumulate) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float num = g[i] * l[i];
    const float den = r[i] * r[i];
    const float v = -(num / den);
    dst[i] = accumulate ? dst[i] + v : v;
  }
}

__device__ __forceinline__ void store_acc(float* dx, int64_t i, float v, int accumulate) {
  dx[i] = accumulate ? dx[i] + v : v;
}

__global__ void relu_backward_kernel(const float* y, const float* g, float* dx, int64_t n, int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_acc(dx, i, g[i] * (y[i] > 0.0f ? 1.0f : 0.0f), acc);
}

__global__ void silu_backward_kernel(const float* x, const float* g, float* dx, int64_t n, int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float s = 1.0f / (1.0f + expf(-v));
    float t = v * s;
    t = t * (1.0f - s);
    store_acc(dx, i, g[i] * (s + t), acc);
  }
}

__global__ void softmax_backward_kernel(const float* y, const float* g, float* dx, int64_t n,
                                        int acc) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float t = y[i] * (1.0f - y[i]);
    store_acc(dx, i, t * g[i], acc);
  }
}

__global__ void sgd_kernel(float* p, const float* g, float lr, int64_t n) {
  const bool vec = aligned16(p) && aligned16(g);
  ew_loop(
      n, vec,
      [&](int64_t i) {
        float4 w = ((float4*)p)[i], d = ((const float4*)g)[i];
        w.x = w.x - lr * d.x;
        w.y = w.y - lr * d.y;
        w.z = w.z - lr * d.z;
        w.w = w.w - lr * d.w;
        ((float4*)p)[i] = w;
      },
      [&](int64_t i) { p[i] = p[i] - lr * g[i]; });
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

// out[j] (+)= sum_b partial[b][j], b in order.
__global__ void sum_partials_kernel(const float* partial, float* out, int nblocks, int width,
                                    int accumulate) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < width; j += gridDim.x * blockDim.x) {
    float acc = 0.0f;
    for (int b = 0; b < nblocks; ++b) acc = acc + partial[(int64_t)b * width + j];
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
// written once.  With `masked`, row r's entries with col > r % q read as
// -1e4 (causal_mask fused in front).  Same arithmetic as softmax_kernel.
template <int VPT>
__global__ void __launch_bounds__(256) softmax_reg_kernel(const float* __restrict__ x,
                                                          float* __restrict__ out, int64_t rows,
                                                          int q, int masked) {
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
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
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
    float4* yr = (float4*)(out + r * kWidth);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float4 t = v[i];
      t.x = t.x / d;
      t.y = t.y / d;
      t.z = t.z / d;
      t.w = t.w / d;
      yr[threadIdx.x + i * 256] = t;
    }
  }
}

// Row r of [outer*q] rows of width k; row index within its q x k block is
// r % q.  Values with col > row read as -1e4.
__global__ void masked_softmax_kernel(const float* __restrict__ x, float* __restrict__ out,
                                      int64_t rows, int q, int width) {
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
      }
    } else {
      for (int j = threadIdx.x; j < width; j += blockDim.x) yr[j] = expf((j > qi ? -1.0e4f : xr[j]) - m) / d;
    }
  }
}

__global__ void masked_softmax_backward_kernel(const float* __restrict__ y, const float* __restrict__ g,
                                               float* __restrict__ dx, int64_t n, int64_t q, int64_t k,
                                               int accumulate) {
  const bool vec = (k & 3) == 0 && aligned16(y) && aligned16(g) && aligned16(dx);
  if (vec) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i << 2;
      const int64_t col = e % k, row = (e / k) % q;
      const float4 yv = ((const float4*)y)[i], gv = ((const float4*)g)[i];
      float4 v;
      v.x = col + 0 > row ? 0.0f : (yv.x * (1.0f - yv.x)) * gv.x;
      v.y = col + 1 > row ? 0.0f : (yv.y * (1.0f - yv.y)) * gv.y;
      v.z = col + 2 > row ? 0.0f : (yv.z * (1.0f - yv.z)) * gv.z;
      v.w = col + 3 > row ? 0.0f : (yv.w * (1.0f - yv.w)) * gv.w;
      if (accumulate) {
        const float4 o = ((float4*)dx)[i];
        v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
      }
      ((float4*)dx)[i] = v;
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t col = i % k, row = (i / k) % q;
      const float v = col > row ? 0.0f : (y[i] * (1.0f - y[i])) * g[i];
      dx[i] = accumulate ? dx[i] + v : v;
    }
  }
}

__global__ void cross_entropy_kernel(const float* __restrict__ logits,
                                     const float* __restrict__ target, float* __restrict__ loss,
                                     int64_t rows, int width) {
  __shared__ float red[33];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    const float* tr = target + r * width;
    float m, d;
    row_max_sum(xr, width, red, &m, &d);
    float acc = 0.0f;
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float p = fmaxf(expf(xr[j] - m) / d, 1e-6f);
      acc += tr[j] * logf(p);
    }
    acc = block_sum(acc, red);
    if (threadIdx.x == 0) loss[r] = 0.0f - acc;
  }
}

__global__ void cross_entropy_backward_kernel(const float* __restrict__ logits,
                                              const float* __restrict__ target,
                                              float* __restrict__ grad, int64_t rows, int width,
                                              int accumulate) {
  __shared__ float red[33];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    float m, d;
    row_max_sum(xr, width, red, &m, &d);
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      const float v = expf(xr[j] - m) / d - target[r * width + j];
      grad[r * width + j] = accumulate ? grad[r * width + j] + v : v;
    }
  }
}

__global__ void cross_entropy_labels_kernel(const float* __restrict__ logits,
                                            const float* __restrict__ labels,
                                            float* __restrict__ loss, int64_t rows, int width,
                                            int* err) {
  __shared__ float red[33];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    float m, d;
    row_max_sum(xr, width, red, &m, &d);
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

__global__ void cross_entropy_labels_backward_kernel(const float* __restrict__ logits,
                                                     const float* __restrict__ labels,
                                                     float* __restrict__ grad, int64_t rows,
                                                     int width, int accumulate, int* err) {
  __shared__ float red[33];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* xr = logits + r * width;
    float m, d;
    row_max_sum(xr, width, red, &m, &d);
    const long long lab = rust_f32_to_i64(labels[r]);
    if (lab < 0 || lab >= width) {
      if (threadIdx.x == 0) atomicCAS(err, 0, (int)kErrIndexRange);
      continue;
    }
    for (int j = threadIdx.x; j < width; j += blockDim.x) {
      float v = expf(xr[j] - m) / d;
      if (j == lab) v = v - 1.0f;
      grad[r * width + j] = accumulate ? grad[r * width + j] + v : v;
    }
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

__global__ void repeat_kv_kernel(const float* __restrict__ x, float* __restrict__ out,
                                 int64_t outer, int64_t heads, int64_t inner, int64_t repeats) {
  const int64_t out_heads = heads * repeats;
  const int64_t n = outer * out_heads * inner;
  const bool vec = (inner & 3) == 0 && aligned16(x) && aligned16(out);
  if (vec) {
    const int64_t inner4 = inner >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n >> 2);
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i % inner4, row = i / inner4;
      const int64_t o = row / out_heads, dh = row % out_heads;
      ((float4*)out)[i] = ((const float4*)x)[(o * heads + dh / repeats) * inner4 + e];
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t e = i % inner, row = i / inner;
      const int64_t o = row / out_heads, dh = row % out_heads;
      out[i] = x[(o * heads + dh / repeats) * inner + e];
    }
  }
}

__global__ void repeat_kv_backward_kernel(const float* __restrict__ g, float* __restrict__ dx,
                                          int64_t outer, int64_t heads, int64_t inner,
                                          int64_t repeats, int accumulate) {
  const int64_t n = outer * heads * inner;
  const int64_t out_heads = heads * repeats;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i % inner, row = i / inner;
    const int64_t o = row / heads, h = row % heads;
    float acc = 0.0f;
    for (int64_t r = 0; r < repeats; ++r) acc = acc + g[(o * out_heads + h * repeats + r) * inner + e];
    dx[i] = accumulate ? dx[i] + acc : acc;
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

__global__ void rope_kernel(const float* __restrict__ x, float* __restrict__ out,
                            const float2* __restrict__ table, int64_t outer, int64_t seq,
                            int64_t half, int backward, int accumulate) {
  const int64_t n = outer * seq * half;
  const int64_t hd = 2 * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t f = i % half, rp = i / half;  // rp = o*seq + p
    const int64_t p = rp % seq;
    const float2 cs = table[p * half + f];
    const int64_t base = rp * hd;
    const float a = x[base + f], b = x[base + half + f];
    float y1, y2;
    if (!backward) {
      const float t1 = a * cs.x, t2 = b * cs.y;
      const float t3 = a * cs.y, t4 = b * cs.x;
      y1 = t1 - t2;
      y2 = t3 + t4;
    } else {
      const float t1 = a * cs.x, t2 = b * cs.y;
      const float t3 = (-a) * cs.y, t4 = b * cs.x;
      y1 = t1 + t2;
      y2 = t3 + t4;
    }
    if (accumulate) {
      out[base + f] = out[base + f] + y1;
      out[base + half + f] = out[base + half + f] + y2;
    } else {
      out[base + f] = y1;
      out[base + half + f] = y2;
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

int row_threads(int64_t width) {
  if (width >= 8192) return 1024;
  if (width >= 2048) return 512;
  if (width >= 256) return 256;
  return 128;
}

int row_blocks(int64_t rows) { return (int)(rows < 148 * 64 ? (rows < 1 ? 1 : rows) : 148 * 64); }

bool aligned16_host(const void* p) { return (((uintptr_t)p) & 15) == 0; }

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
  unary_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(op, x, out, n, param);
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
  int64_t rpb = ceil_div(rows, 148 * 4);
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
  rms_gain_backward_kernel<<<nb, row_threads(width), 0, st>>>(x, g, dy, dx, partial, rows,
                                                              (int)width, eps, acc_dx, (int)rpb);
  check_launch();
  sum_partials_kernel<<<(int)ceil_div(width, 256), 256, 0, st>>>(partial, dg, nb, (int)width, acc_dg);
  check_launch();
}

// Launches the register-resident form when the width allows; false if not.
bool softmax_reg(const float* x, float* out, int64_t rows, int64_t width, int64_t q, int masked,
                 cudaStream_t st);

void launch_softmax(const float* x, float* out, int64_t rows, int64_t width, cudaStream_t st) {
  if (rows <= 0) return;
  if (softmax_reg(x, out, rows, width, 1, 0, st)) return;
  softmax_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(x, out, rows, (int)width);
  check_launch();
}

bool softmax_reg(const float* x, float* out, int64_t rows, int64_t width, int64_t q, int masked,
                 cudaStream_t st) {
  if (width % 1024 != 0 || !aligned16_host(x) || !aligned16_host(out)) return false;
  const int blocks = row_blocks(rows);
  switch (width / 1024) {
    case 1: softmax_reg_kernel<1><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked); break;
    case 2: softmax_reg_kernel<2><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked); break;
    case 4: softmax_reg_kernel<4><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked); break;
    case 8: softmax_reg_kernel<8><<<blocks, 256, 0, st>>>(x, out, rows, (int)q, masked); break;
    default: return false;
  }
  check_launch();
  return true;
}

void launch_masked_softmax(const float* x, float* out, int64_t outer, int64_t q, int64_t k,
                           cudaStream_t st) {
  const int64_t rows = outer * q;
  if (rows <= 0) return;
  if (softmax_reg(x, out, rows, k, q, 1, st)) return;
  masked_softmax_kernel<<<row_blocks(rows), row_threads(k / 4), 0, st>>>(x, out, rows, (int)q, (int)k);
  check_launch();
}

void launch_masked_softmax_backward(const float* y, const float* g, float* dx, int64_t outer,
                                    int64_t q, int64_t k, int accumulate, cudaStream_t st) {
  const int64_t n = outer * q * k;
  if (n <= 0) return;
  masked_softmax_backward_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      y, g, dx, n, q, k, accumulate);
  check_launch();
}

void launch_cross_entropy(const float* logits, const float* target, float* loss, int64_t rows,
                          int64_t width, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(logits, target, loss, rows,
                                                                        (int)width);
  check_launch();
}

void launch_cross_entropy_backward(const float* logits, const float* target, float* grad,
                                   int64_t rows, int64_t width, int accumulate, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_backward_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(
      logits, target, grad, rows, (int)width, accumulate);
  check_launch();
}

void launch_cross_entropy_labels(const float* logits, const float* labels, float* loss,
                                 int64_t rows, int64_t width, int* err, cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_labels_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(
      logits, labels, loss, rows, (int)width, err);
  check_launch();
}

void launch_cross_entropy_labels_backward(const float* logits, const float* labels, float* grad,
                                          int64_t rows, int64_t width, int accumulate, int* err,
                                          cudaStream_t st) {
  if (rows <= 0) return;
  cross_entropy_labels_backward_kernel<<<row_blocks(rows), row_threads(width), 0, st>>>(
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
                      int64_t repeats, cudaStream_t st) {
  const int64_t n = outer * heads * repeats * inner;
  if (n <= 0) return;
  repeat_kv_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      x, out, outer, heads, inner, repeats);
  check_launch();
}

void launch_repeat_kv_backward(const float* g, float* dx, int64_t outer, int64_t heads,
                               int64_t inner, int64_t repeats, int accumulate, cudaStream_t st) {
  const int64_t n = outer * heads * inner;
  if (n <= 0) return;
  repeat_kv_backward_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(
      g, dx, outer, heads, inner, repeats, accumulate);
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
                 int64_t half, cudaStream_t st) {
  const int64_t n = outer * seq * half;
  if (n <= 0) return;
  rope_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(x, out, table, outer, seq,
                                                                    half, 0, 0);
  check_launch();
}

void launch_rope_backward(const float* g, float* dx, const float2* table, int64_t outer,
                          int64_t seq, int64_t half, int accumulate, cudaStream_t st) {
  const int64_t n = outer * seq * half;
  if (n <= 0) return;
  rope_kernel<<<elementwise_blocks(n, kThreads), kThreads, 0, st>>>(g, dx, table, outer, seq, half,
                                                                    1, accumulate);
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
  const int hi = a > b ? a : b;
  int64_t inner = 1;
  for (int i = hi + 1; i < rank; ++i) inner *= dims[i];
  transpose_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(
      x, out, od, is, rank, a, b, n, inner, accumulate);
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
  sum_partials_kernel<<<(int)ceil_div(width, 256), 256, 0, st>>>(partial, out, (int)chunks,
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

void launch_sgd(float* p, const float* g, float lr, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  sgd_kernel<<<elementwise_blocks((n + 3) / 4, kThreads), kThreads, 0, st>>>(p, g, lr, n);
  check_launch();
}

}  // namespace tysor
