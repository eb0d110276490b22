// Bandwidth-bound kernels of the tysor CUDA backend: elementwise, row
// reductions, gathers, masks, rotations, updates.  All fp32.  Each launcher
// enqueues on `st` and returns immediately; kernels that can meet an invalid
// index record it in the device error word `err` instead of trapping.
#pragma once

#include "common.cuh"

namespace tysor {

enum UnaryOp : int {
  kUnaryCopy = 0,
  kUnaryRelu = 1,
  kUnarySilu = 2,
  kUnaryScale = 3,  // x * param
  kUnaryNeg = 4,
};

enum BinaryOp : int { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3 };

// Pattern fills of the reference initialisers: out[i] = ((i % mod) + add) / div.
void launch_pattern(float* out, int64_t n, int mod, float add, float div, cudaStream_t st);
void launch_fill(float* out, int64_t n, float value, cudaStream_t st);

void launch_unary(int op, const float* x, float* out, int64_t n, float param, cudaStream_t st);
// out = t + t with t = g * x: the gradient of x * x into a fresh buffer.
void launch_square_backward(const float* g, const float* x, float* out, int64_t n, cudaStream_t st);
void launch_binary_tt(int op, const float* a, const float* b, float* out, int64_t n,
                      cudaStream_t st);
void launch_binary_ts(int op, const float* a, float s, float* out, int64_t n, cudaStream_t st);
void launch_binary_st(int op, float s, const float* b, float* out, int64_t n, cudaStream_t st);
// dst = dst + src (gradient accumulation, tensor.rs:94-103 order).
void launch_add_inplace(float* dst, const float* src, int64_t n, cudaStream_t st);
// dst = dst + op(a, b)  /  dst = dst + op(a, s) (or op(s, a) when scalar_first):
// the product is rounded first, then added, as the reference computes a
// gradient term and then accumulates it.
void launch_binary_tt_acc(int op, const float* a, const float* b, float* dst, int64_t n,
                          cudaStream_t st);
void launch_binary_ts_acc(int op, const float* a, float s, float* dst, int64_t n,
                          int scalar_first, cudaStream_t st);
// Gradient of the divisor of a tensor/tensor division (backward.rs:285-294):
// v = -((g * lhs) / (rhs * rhs)); dst = accumulate ? dst + v : v.
void launch_div_rhs_grad(const float* g, const float* lhs, const float* rhs, float* dst, int64_t n,
                         int accumulate, cudaStream_t st);

// Backward helpers.  `accumulate` adds the result into dx instead of storing.
void launch_relu_backward(const float* out_act, const float* grad, float* dx, int64_t n,
                          int accumulate, cudaStream_t st);
// h = silu(x) * u (SwiGLU's product, bit-identical to silu then '*').
void launch_silu_mul(const float* x, const float* u, float* h, int64_t n, cudaStream_t st);
// Its backward from dh: du (+)= dh * silu(x), dx (+)= silu'(x) rule of
// launch_silu_backward applied to dh * u.
void launch_silu_mul_backward(const float* x, const float* u, const float* dh, float* dx, float* du, int64_t n,
                              int acc_x, int acc_u, cudaStream_t st);
void launch_silu_backward(const float* x, const float* grad, float* dx, int64_t n, int accumulate,
                          cudaStream_t st);
void launch_softmax_backward(const float* y, const float* grad, float* dx, int64_t n,
                             int accumulate, cudaStream_t st);

void launch_rms_norm(const float* x, float* out, int64_t rows, int64_t width, cudaStream_t st);
void launch_rms_norm_gain(const float* x, const float* g, float* out, int64_t rows, int64_t width,
                          float eps, cudaStream_t st);
// dx (+)= dy * g;  dg = column sums of dy * x * rsqrt(mean(x^2)+eps).
// `partial` needs rms_gain_partial_elems(rows, width) floats of scratch.
int64_t rms_gain_partial_elems(int64_t rows, int64_t width);
void launch_rms_norm_gain_backward(const float* x, const float* g, const float* dy, float* dx,
                                   float* dg, float* partial, int64_t rows, int64_t width,
                                   float eps, int accumulate_dx, int accumulate_dg,
                                   cudaStream_t st);

void launch_softmax(const float* x, float* out, int64_t rows, int64_t width, cudaStream_t st);
// Softmax of causal_mask(x) over [outer][q][k] in one pass: entries with
// col > row take the mask's -1e4 (layers.rs:217-236), then the row softmax
// (tensor.rs:235-260) — the same arithmetic as the two ops in sequence.
// With `leak` ([outer * q]), writes each row's masked-entry probability
// exp(-1e4 - max) / d, which is 0 unless the row's visible scores all lie
// below about -9896 (and 0 for a row with nothing masked): causal GEMMs that
// skip masked entries as zeros add those terms back with
// launch_causal_leak_fix.  With `lo`, also writes each probability's low
// part (tf32_lo, the operand split a strict GEMM consuming them needs).
// With `skip_zero`, wholly masked groups (exact zeros) are not stored: for
// buffers known to hold zeros there already.
void launch_masked_softmax(const float* x, float* out, int64_t outer, int64_t q, int64_t k,
                           float* leak, float* lo, int skip_zero, cudaStream_t st);
// After a causal GEMM that skipped masked entries as zeros (mode 2: O = P.V,
// GemmEpilogue::tri 2; mode 3: dV = P^T.dO, tri 3; tile_rows as
// gemm_causal_tile_rows reports for it), adds back the terms of rows whose
// masked entries keep probability leak[row] (see launch_masked_softmax).
// x: the GEMM's B operand (V or dO) with its layout; out: its output; rows,
// kn, n: its M, K, N; lrows: the softmax rows per batch item.  A batch item
// without such a row costs one read of its leak values.
void launch_causal_leak_fix(int mode, const float* leak, int64_t lrows, const float* x, bool x_trans, int64_t x_ld,
                            int64_t x_bs, float* out, int64_t o_ld, int64_t o_bs, int batch, int64_t rows, int64_t kn,
                            int64_t n, int tile_rows, cudaStream_t st);
// Backward of Softmax(causal_mask(x)) with the reference rules: the
// diagonal softmax term y(1-y)g (layers.rs:350-364), then the mask zeroes
// col > row (layers.rs:418-436): dx (+)= col > row ? 0 : y(1-y)g.
void launch_masked_softmax_backward(const float* y, const float* g, float* dx, int64_t outer,
                                    int64_t q, int64_t k, int accumulate, float* lo, int skip_zero,
                                    cudaStream_t st);
void launch_cross_entropy(const float* logits, const float* target, float* loss, int64_t rows,
                          int64_t width, cudaStream_t st);
void launch_cross_entropy_backward(const float* logits, const float* target, float* grad,
                                   int64_t rows, int64_t width, int accumulate, cudaStream_t st);
void launch_cross_entropy_labels(const float* logits, const float* labels, float* loss,
                                 int64_t rows, int64_t width, int* err, cudaStream_t st);
void launch_cross_entropy_labels_backward(const float* logits, const float* labels, float* grad,
                                          int64_t rows, int64_t width, int accumulate, int* err,
                                          cudaStream_t st);

void launch_embedding(const float* idx, const float* weight, float* out, int64_t count,
                      int64_t num, int64_t dim, int* err, cudaStream_t st);
// Deterministic scatter-add: every weight row sums its tokens' gradient rows
// in increasing token order (layers.rs:497-519), skipping out-of-range ids.
// `work` needs embedding_backward_work_bytes(count, num) bytes.
size_t embedding_backward_work_bytes(int64_t count, int64_t num);
void launch_embedding_backward(const float* grad, const float* idx, float* wgrad, int64_t count,
                               int64_t num, int64_t dim, void* work, int accumulate,
                               cudaStream_t st);

// seq > 0: x (forward) / dx (backward) is stored [outer][seq][heads][inner /
// seq], the layout before transpose(1, 2) (the transpose is folded here).
void launch_repeat_kv(const float* x, float* out, int64_t outer, int64_t heads, int64_t inner,
                      int64_t repeats, cudaStream_t st, int64_t seq = 0);
void launch_repeat_kv_backward(const float* grad, float* dx, int64_t outer, int64_t heads,
                               int64_t inner, int64_t repeats, int accumulate, cudaStream_t st,
                               int64_t seq = 0);
void launch_causal_mask(const float* x, float* out, int64_t outer, int64_t q, int64_t k,
                        cudaStream_t st);
void launch_causal_mask_backward(const float* grad, float* dx, int64_t outer, int64_t q, int64_t k,
                                 int accumulate, cudaStream_t st);
// `table` holds seq x half (cos, sin) pairs computed on the host.
// in_hs / out_hs = H > 0: the input (forward) / output (backward) is stored
// [B][seq][H][hd] while rows run over [B][H][seq] (a transpose(1, 2) folded
// here).
void launch_rope(const float* x, float* out, const float2* table, int64_t outer, int64_t seq,
                 int64_t half, cudaStream_t st, int64_t in_hs = 0);
void launch_rope_backward(const float* grad, float* dx, const float2* table, int64_t outer,
                          int64_t seq, int64_t half, int accumulate, cudaStream_t st, int64_t out_hs = 0);
// Exchange axes a < b of a row-major tensor of rank <= 8.
void launch_transpose(const float* x, float* out, const int64_t* dims, int rank, int a, int b,
                      int accumulate, cudaStream_t st);

// Column sums of a [rows, width] gradient (bias gradient); `partial` needs
// colsum_partial_elems(rows, width) floats.
int64_t colsum_partial_elems(int64_t rows, int64_t width);
void launch_colsum(const float* grad, float* out, float* partial, int64_t rows, int64_t width,
                   int accumulate, cudaStream_t st);
// Sum of all elements into out[0]; `partial` needs 1024 floats.
void launch_reduce_sum(const float* x, float* out, float* partial, int64_t n, cudaStream_t st);
// out[0] = x[0] + x[1] + ... in index order with one f32 accumulator (the
// reference's tensor_sum rounding; one thread, so slow on large tensors).
void launch_sequential_sum(const float* x, float* out, int64_t n, cudaStream_t st);

// p = p - (lr * g), each product and difference rounded separately.
void launch_sgd(float* p, const float* g, float lr, int64_t n, cudaStream_t st);

}  // namespace tysor
