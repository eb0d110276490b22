/*
 * CPU oracle: a C restatement of the reference `local` backend's op library.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library (tysor_b200/)
 * links, loads or calls this file; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg use it, and only as the checker.
 *
 * Every function follows the reference loop order and f32 rounding steps so
 * that its results are bit-identical to the Rust code it restates:
 *   - each product and each sum is rounded to f32 separately (the build uses
 *     -ffp-contract=off so no fused multiply-add is formed);
 *   - reductions run sequentially in index order starting from 0.0f;
 *   - transcendental calls are the C library's expf/logf/powf/cosf/sinf, the
 *     same libm entry points Rust's f32 methods call on Linux.
 * The only deliberate departure is the loop NESTING of matmul (i-k-j instead
 * of i-j-k, and rows split across POSIX threads): every output element still
 * accumulates its k products in increasing k order from 0.0f, so the values
 * are identical while the loop runs at memory speed.
 *
 * Built twice (oracle/Makefile): libtysor_oracle.so in f32, the restatement
 * itself, and libtysor_oracle64.so with TL_F64 defined, which runs the same
 * loops, constants and order in f64.  The f64 twin is not the reference's
 * arithmetic; tests use it as a nearly exact answer, to measure how far the
 * f32 oracle and the CUDA backend each land from it on large inputs.
 *
 * Reference files cited as path:line within the tysor project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#include <pthread.h>

#define TL_OK 0
#define TL_ERR_SHAPE 1
#define TL_ERR_INDEX 2
#define TL_ERR_ARG 3

enum { TL_ADD = 0, TL_SUB = 1, TL_MUL = 2, TL_DIV = 3 };

#ifdef TL_F64
typedef double real;
#define R_EXP exp
#define R_LOG log
#define R_SQRT sqrt
#define R_POW pow
#define R_COS cos
#define R_SIN sin
#define R_MAX fmax
#else
typedef float real;
#define R_EXP expf
#define R_LOG logf
#define R_SQRT sqrtf
#define R_POW powf
#define R_COS cosf
#define R_SIN sinf
#define R_MAX fmaxf
#endif

static int g_threads = 1;

void tl_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

int tl_get_threads(void) { return g_threads; }

/* ---- pattern tensors --------------------------------------------------- */

/* runtime/tensor.rs:24-34  make_synthetic_tensor: ((i % 17) + 1) / 8 */
void tl_synthetic(real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = (real)((i % 17) + 1) / 8.0f;
}

/* runtime/layers.rs:39-51  make_linear_weight: ((i % 13) + 1) / 16 */
void tl_linear_weight_init(real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = ((real)(i % 13) + 1.0f) / 16.0f;
}

/* runtime/layers.rs:53-63  make_linear_bias: ((i % 7) + 1) / 32 */
void tl_linear_bias_init(real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = ((real)(i % 7) + 1.0f) / 32.0f;
}

/* runtime/layers.rs:65-75  make_embedding_weight: ((i % 17) + 1) / 8 */
void tl_embedding_weight_init(real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = ((real)(i % 17) + 1.0f) / 8.0f;
}

/* training/backward.rs:225-235  fake linear weight of --backward: ((i % 11) - 5) / 16 */
void tl_backward_fake_weight(real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = ((real)(i % 11) - 5.0f) / 16.0f;
}

/* ---- elementwise ------------------------------------------------------- */

static inline real apply_op(int op, real a, real b) {
  switch (op) {
    case TL_ADD: return a + b;
    case TL_SUB: return a - b;
    case TL_MUL: return a * b;
    default: return a / b;
  }
}

/* runtime/tensor.rs:105-125 elementwise_binary */
void tl_binary_tt(int op, const real* a, const real* b, real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = apply_op(op, a[i], b[i]);
}

/* runtime/tensor.rs:127-140 tensor_scalar_binary (scalar narrowed f64 -> f32) */
void tl_binary_ts(int op, const real* a, double s, real* out, int64_t n) {
  real r = (real)s;
  for (int64_t i = 0; i < n; ++i) out[i] = apply_op(op, a[i], r);
}

/* runtime/tensor.rs:142-155 scalar_tensor_binary */
void tl_binary_st(int op, double s, const real* b, real* out, int64_t n) {
  real l = (real)s;
  for (int64_t i = 0; i < n; ++i) out[i] = apply_op(op, l, b[i]);
}

/* runtime/tensor.rs:86-92 negate */
void tl_negate(const real* a, real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = -a[i];
}

/* runtime/tensor.rs:94-103 add_in_place */
void tl_add_in_place(real* dst, const real* src, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] += src[i];
}

/* runtime/tensor.rs:215-221 apply_relu: value.max(0.0) */
void tl_relu(const real* a, real* out, int64_t n) {
  /* fmaxf has f32::max's NaN rule: the non-NaN operand wins. */
  for (int64_t i = 0; i < n; ++i) out[i] = R_MAX(a[i], 0.0f);
}

/* training/executor.rs:644-652 relu backward: grad * (out > 0 ? 1 : 0) */
void tl_relu_backward(const real* out_act, const real* grad, real* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dx[i] = grad[i] * (out_act[i] > 0.0f ? 1.0f : 0.0f);
}

/* runtime/tensor.rs:223-233 apply_silu: x / (1 + exp(-x)) */
void tl_silu(const real* a, real* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    real v = a[i];
    out[i] = v / (1.0f + R_EXP(-v));
  }
}

/* runtime/layers.rs:330-348 backward_silu */
void tl_silu_backward(const real* x, const real* grad, real* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    real v = x[i];
    real s = 1.0f / (1.0f + R_EXP(-v));
    real t = v * s;
    t = t * (1.0f - s);
    dx[i] = grad[i] * (s + t);
  }
}

/* runtime/layers.rs:119-129 apply_dropout (deterministic keep scale) */
int tl_dropout(const real* a, double p, real* out, int64_t n) {
  if (!(p >= 0.0 && p < 1.0)) return TL_ERR_ARG;
  real keep = (real)(1.0 - p);
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] * keep;
  return TL_OK;
}

/* ---- matmul ------------------------------------------------------------ */

/* runtime/tensor.rs:163-194 matmul (rank 2): out[r,c] = sum_k lhs[r,k]*rhs[k,c],
 * accumulated from 0.0f in increasing k.  Loop nest i-k-j, same per-element
 * sequence of roundings; rows are split across threads. */
typedef struct {
  const real *a, *b;
  real* c;
  int64_t r0, r1, k, n;
} mm_job;

static void mm_rows(const real* a, const real* b, real* c, int64_t r0, int64_t r1, int64_t k,
                    int64_t n) {
  for (int64_t i = r0; i < r1; ++i) {
    real* crow = c + i * n;
    for (int64_t j = 0; j < n; ++j) crow[j] = 0.0f;
    const real* arow = a + i * k;
    for (int64_t kk = 0; kk < k; ++kk) {
      const real av = arow[kk];
      const real* brow = b + kk * n;
      for (int64_t j = 0; j < n; ++j) {
        real prod = av * brow[j];
        crow[j] = crow[j] + prod;
      }
    }
  }
}

static void* mm_worker(void* arg) {
  mm_job* j = (mm_job*)arg;
  mm_rows(j->a, j->b, j->c, j->r0, j->r1, j->k, j->n);
  return NULL;
}

void tl_matmul(const real* a, const real* b, real* c, int64_t m, int64_t k, int64_t n) {
  int nt = g_threads;
  if (nt > m) nt = (int)m;
  if (nt <= 1 || m * n * k < 262144) {
    mm_rows(a, b, c, 0, m, k, n);
    return;
  }
  pthread_t tid[256];
  mm_job jobs[256];
  int64_t per = (m + nt - 1) / nt;
  int launched = 0;
  for (int t = 0; t < nt; ++t) {
    int64_t r0 = t * per, r1 = r0 + per > m ? m : r0 + per;
    if (r0 >= r1) break;
    jobs[t] = (mm_job){a, b, c, r0, r1, k, n};
    if (pthread_create(&tid[t], NULL, mm_worker, &jobs[t]) != 0) {
      mm_rows(a, b, c, r0, r1, k, n);
      tid[t] = 0;
    }
    launched = t + 1;
  }
  for (int t = 0; t < launched; ++t)
    if (tid[t]) pthread_join(tid[t], NULL);
}

/* runtime/tensor.rs:196-213 transpose_2d */
void tl_transpose2d(const real* a, real* out, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) out[c * rows + r] = a[r * cols + c];
}

/* runtime/layers.rs:102-117 apply_linear_with_parameters bias loop */
void tl_bias_add(real* out, const real* bias, int64_t batch, int64_t width) {
  for (int64_t r = 0; r < batch; ++r)
    for (int64_t c = 0; c < width; ++c) out[r * width + c] += bias[c];
}

/* ---- row reductions ---------------------------------------------------- */

/* runtime/tensor.rs:235-260 apply_softmax over the last axis */
void tl_softmax(const real* x, real* out, int64_t rows, int64_t width) {
  for (int64_t r = 0; r < rows; ++r) {
    const real* row = x + r * width;
    real* o = out + r * width;
    real mx = -INFINITY;
    for (int64_t j = 0; j < width; ++j) mx = R_MAX(mx, row[j]);
    real sum = 0.0f;
    for (int64_t j = 0; j < width; ++j) {
      real e = R_EXP(row[j] - mx);
      o[j] = e;
      sum = sum + e;
    }
    real denom = R_MAX(sum, FLT_EPSILON);
    for (int64_t j = 0; j < width; ++j) o[j] = o[j] / denom;
  }
}

/* runtime/layers.rs:350-364 backward_softmax (diagonal term only) */
void tl_softmax_backward(const real* y, const real* grad, real* dx, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    real t = y[i] * (1.0f - y[i]);
    dx[i] = t * grad[i];
  }
}

/* runtime/layers.rs:275-299 apply_rms_norm (no gain, eps 1e-5) */
void tl_rms_norm(const real* x, real* out, int64_t rows, int64_t width) {
  for (int64_t r = 0; r < rows; ++r) {
    const real* row = x + r * width;
    real acc = 0.0f;
    for (int64_t j = 0; j < width; ++j) acc = acc + row[j] * row[j];
    real ms = acc / (real)width;
    real scale = 1.0f / R_SQRT(ms + 1e-5f);
    for (int64_t j = 0; j < width; ++j) out[r * width + j] = row[j] * scale;
  }
}

/* Extension (no reference counterpart): RMSNorm with a learned gain and a
 * configurable eps: y = (x * rsqrt(mean(x^2) + eps)) * g.  The normalisation
 * part rounds exactly like tl_rms_norm. */
void tl_rms_norm_gain(const real* x, const real* g, real* out, int64_t rows, int64_t width,
                      float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const real* row = x + r * width;
    real acc = 0.0f;
    for (int64_t j = 0; j < width; ++j) acc = acc + row[j] * row[j];
    real ms = acc / (real)width;
    real scale = 1.0f / R_SQRT(ms + eps);
    for (int64_t j = 0; j < width; ++j) {
      real v = row[j] * scale;
      out[r * width + j] = v * g[j];
    }
  }
}

/* Extension backward, following the reference rule that the normalisation
 * passes the gradient through unchanged (layers.rs:366-371):
 *   dx = dy * g;   dg[j] = sum_r dy[r,j] * (x[r,j] * scale_r)  (rows in order). */
void tl_rms_norm_gain_backward(const real* x, const real* g, const real* dy, real* dx,
                               real* dg, int64_t rows, int64_t width, float eps) {
  for (int64_t j = 0; j < width; ++j) dg[j] = 0.0f;
  for (int64_t r = 0; r < rows; ++r) {
    const real* row = x + r * width;
    real acc = 0.0f;
    for (int64_t j = 0; j < width; ++j) acc = acc + row[j] * row[j];
    real ms = acc / (real)width;
    real scale = 1.0f / R_SQRT(ms + eps);
    for (int64_t j = 0; j < width; ++j) {
      real d = dy[r * width + j];
      dx[r * width + j] = d * g[j];
      real nrm = row[j] * scale;
      dg[j] = dg[j] + d * nrm;
    }
  }
}

/* runtime/layers.rs:301-324 apply_cross_entropy with a dense target:
 * loss[r] = -sum_j t[r,j] * ln(max(softmax[r,j], 1e-6)). */
void tl_cross_entropy(const real* logits, const real* target, real* loss, int64_t rows,
                      int64_t width) {
  real* probs = (real*)malloc(sizeof(real) * (size_t)width);
  for (int64_t r = 0; r < rows; ++r) {
    tl_softmax(logits + r * width, probs, 1, width);
    real acc = 0.0f;
    const real* t = target + r * width;
    for (int64_t j = 0; j < width; ++j) {
      real p = R_MAX(probs[j], 1e-6f);
      acc = acc - t[j] * R_LOG(p);
    }
    loss[r] = acc;
  }
  free(probs);
}

/* runtime/layers.rs:479-488 backward_cross_entropy_logits: softmax - target */
void tl_cross_entropy_backward(const real* logits, const real* target, real* grad, int64_t rows,
                               int64_t width) {
  tl_softmax(logits, grad, rows, width);
  int64_t n = rows * width;
  for (int64_t i = 0; i < n; ++i) grad[i] = grad[i] - target[i];
}

/* f32 -> i64 conversion with Rust `as` semantics (saturating, NaN -> 0). */
static inline int64_t rust_f32_to_i64(real v) {
  if (isnan(v)) return 0;
  if (v >= 9.2233720368547758e18f) return INT64_MAX;
  if (v <= -9.2233720368547758e18f) return INT64_MIN;
  return (int64_t)v;
}

/* Extension: cross entropy against integer class labels stored as f32 (the
 * reference has no integer tensor type; ids below 2^24 are exact in f32).
 * loss[r] = -ln(max(softmax[r, label_r], 1e-6)); a label outside
 * [0, width) is an error, like an out-of-range embedding index. */
int tl_cross_entropy_labels(const real* logits, const real* labels, real* loss, int64_t rows,
                            int64_t width) {
  real* probs = (real*)malloc(sizeof(real) * (size_t)width);
  int rc = TL_OK;
  for (int64_t r = 0; r < rows; ++r) {
    int64_t lab = rust_f32_to_i64(labels[r]);
    if (lab < 0 || lab >= width) { rc = TL_ERR_INDEX; break; }
    tl_softmax(logits + r * width, probs, 1, width);
    real p = R_MAX(probs[lab], 1e-6f);
    real acc = 0.0f;
    acc = acc - 1.0f * R_LOG(p);
    loss[r] = acc;
  }
  free(probs);
  return rc;
}

/* Extension backward: softmax - onehot(label). */
int tl_cross_entropy_labels_backward(const real* logits, const real* labels, real* grad,
                                     int64_t rows, int64_t width) {
  tl_softmax(logits, grad, rows, width);
  for (int64_t r = 0; r < rows; ++r) {
    int64_t lab = rust_f32_to_i64(labels[r]);
    if (lab < 0 || lab >= width) return TL_ERR_INDEX;
    grad[r * width + lab] = grad[r * width + lab] - 1.0f;
  }
  return TL_OK;
}

/* ---- gathers, copies, masks, rotations --------------------------------- */

/* runtime/layers.rs:131-160 apply_embedding_with_parameters */
int tl_embedding(const real* idx, const real* weight, real* out, int64_t count,
                 int64_t num_embeddings, int64_t dim) {
  for (int64_t i = 0; i < count; ++i) {
    int64_t index = rust_f32_to_i64(idx[i]);
    if (index < 0 || index >= num_embeddings) return TL_ERR_INDEX;
    memcpy(out + i * dim, weight + index * dim, sizeof(real) * (size_t)dim);
  }
  return TL_OK;
}

/* runtime/layers.rs:497-519 backward_embedding_weight: scatter-add in index
 * order, skipping out-of-range indices. */
void tl_embedding_backward(const real* grad, const real* idx, real* wgrad, int64_t count,
                           int64_t num_embeddings, int64_t dim) {
  memset(wgrad, 0, sizeof(real) * (size_t)(num_embeddings * dim));
  for (int64_t i = 0; i < count; ++i) {
    int64_t index = rust_f32_to_i64(idx[i]);
    if (index < 0 || index >= num_embeddings) continue;
    for (int64_t d = 0; d < dim; ++d) wgrad[index * dim + d] += grad[i * dim + d];
  }
}

/* runtime/layers.rs:173-201 apply_repeat_kv along dim 1 */
void tl_repeat_kv(const real* in, real* out, int64_t outer, int64_t heads, int64_t inner,
                  int64_t repeats) {
  int64_t out_heads = heads * repeats;
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t h = 0; h < heads; ++h) {
      const real* src = in + (o * heads + h) * inner;
      for (int64_t r = 0; r < repeats; ++r)
        memcpy(out + (o * out_heads + h * repeats + r) * inner, src, sizeof(real) * (size_t)inner);
    }
}

/* runtime/layers.rs:388-416 backward_repeat_kv_input: sum over repeats in order */
void tl_repeat_kv_backward(const real* grad, real* dx, int64_t outer, int64_t heads, int64_t inner,
                           int64_t repeats) {
  int64_t out_heads = heads * repeats;
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t h = 0; h < heads; ++h) {
      real* dst = dx + (o * heads + h) * inner;
      for (int64_t i = 0; i < inner; ++i) dst[i] = 0.0f;
      for (int64_t r = 0; r < repeats; ++r) {
        const real* g = grad + (o * out_heads + h * repeats + r) * inner;
        for (int64_t i = 0; i < inner; ++i) dst[i] += g[i];
      }
    }
}

/* runtime/layers.rs:217-236 apply_causal_mask: col > row -> -1e4 */
void tl_causal_mask(const real* in, real* out, int64_t outer, int64_t q, int64_t k) {
  int64_t n = outer * q * k;
  if (out != in) memcpy(out, in, sizeof(real) * (size_t)n);
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t r = 0; r < q; ++r)
      for (int64_t c = r + 1; c < k; ++c) out[o * q * k + r * k + c] = -1.0e4f;
}

/* runtime/layers.rs:418-436 backward_causal_mask_input: zero the upper triangle */
void tl_causal_mask_backward(const real* grad, real* dx, int64_t outer, int64_t q, int64_t k) {
  int64_t n = outer * q * k;
  if (dx != grad) memcpy(dx, grad, sizeof(real) * (size_t)n);
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t r = 0; r < q; ++r)
      for (int64_t c = r + 1; c < k; ++c) dx[o * q * k + r * k + c] = 0.0f;
}

static void rope_inv_freq(real* inv_freq, int64_t half, double theta) {
  for (int64_t i = 0; i < half; ++i)
    inv_freq[i] = R_POW((real)theta, -(real)i / (real)half);
}

/* runtime/layers.rs:238-273 apply_rope (half-split rotation, pos along dim -2) */
void tl_rope(const real* in, real* out, int64_t outer, int64_t seq, int64_t head_dim,
             double theta) {
  int64_t half = head_dim / 2;
  real* inv = (real*)malloc(sizeof(real) * (size_t)(half > 0 ? half : 1));
  rope_inv_freq(inv, half, theta);
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t p = 0; p < seq; ++p) {
      int64_t base = (o * seq + p) * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        real ang = (real)p * inv[i];
        real c = R_COS(ang), s = R_SIN(ang);
        real x1 = in[base + i], x2 = in[base + half + i];
        real a = x1 * c, b = x2 * s;
        real d = x1 * s, e = x2 * c;
        out[base + i] = a - b;
        out[base + half + i] = d + e;
      }
    }
  free(inv);
}

/* runtime/layers.rs:438-477 backward_rope_input (inverse rotation) */
void tl_rope_backward(const real* grad, real* dx, int64_t outer, int64_t seq, int64_t head_dim,
                      double theta) {
  int64_t half = head_dim / 2;
  real* inv = (real*)malloc(sizeof(real) * (size_t)(half > 0 ? half : 1));
  rope_inv_freq(inv, half, theta);
  for (int64_t o = 0; o < outer; ++o)
    for (int64_t p = 0; p < seq; ++p) {
      int64_t base = (o * seq + p) * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        real ang = (real)p * inv[i];
        real c = R_COS(ang), s = R_SIN(ang);
        real g1 = grad[base + i], g2 = grad[base + half + i];
        real a = g1 * c, b = g2 * s;
        real d = (-g1) * s, e = g2 * c;
        dx[base + i] = a + b;
        dx[base + half + i] = d + e;
      }
    }
  free(inv);
}

/* Extension: swap two axes of a row-major tensor (materialised copy).
 * dims has `rank` entries; the output has dims[a] and dims[b] exchanged. */
void tl_transpose(const real* in, real* out, const int64_t* dims, int rank, int a, int b) {
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) n *= dims[i];
  int64_t in_stride[16], out_dims[16], out_stride[16];
  in_stride[rank - 1] = 1;
  for (int i = rank - 2; i >= 0; --i) in_stride[i] = in_stride[i + 1] * dims[i + 1];
  for (int i = 0; i < rank; ++i) out_dims[i] = dims[i];
  out_dims[a] = dims[b];
  out_dims[b] = dims[a];
  out_stride[rank - 1] = 1;
  for (int i = rank - 2; i >= 0; --i) out_stride[i] = out_stride[i + 1] * out_dims[i + 1];
  for (int64_t o = 0; o < n; ++o) {
    int64_t rem = o, src = 0;
    for (int i = 0; i < rank; ++i) {
      int64_t ci = rem / out_stride[i];
      rem -= ci * out_stride[i];
      int si = (i == a) ? b : (i == b) ? a : i;
      src += ci * in_stride[si];
    }
    out[o] = in[src];
  }
}

/* runtime/layers.rs:529-549 backward_linear_bias: column sums, rows in order */
void tl_bias_grad(const real* grad, real* db, int64_t batch, int64_t width) {
  for (int64_t c = 0; c < width; ++c) db[c] = 0.0f;
  for (int64_t r = 0; r < batch; ++r)
    for (int64_t c = 0; c < width; ++c) db[c] += grad[r * width + c];
}

/* training/executor.rs:745-762 apply_sgd: p -= (lr as f32) * g */
void tl_sgd(real* p, const real* g, double lr, int64_t n) {
  real l = (real)lr;
  for (int64_t i = 0; i < n; ++i) {
    real step = l * g[i];
    p[i] = p[i] - step;
  }
}

/* training/executor.rs:109-111 tensor_sum (sequential f32) */
double tl_sum(const real* a, int64_t n) {
  real acc = 0.0f;
  for (int64_t i = 0; i < n; ++i) acc = acc + a[i];
  return (double)acc;
}
