// The C ABI of libtysor_cuda.so: context, buffers, per-op dispatch
// (include/tysor_cuda.h).  Every entry point catches C++ exceptions and
// reports them through tysor_cuda_last_error(), the convention of the
// reference's Metal bridge (native/metal_bridge.mm:14-16, 72-97).
#include <math.h>
#include <string.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/tysor_cuda.h"
#include "context.cuh"
#include "ops.cuh"

namespace tysor {

std::atomic<int64_t> g_launches{0};

static thread_local std::string t_last_error;

void set_last_error(const std::string& msg) { t_last_error = msg; }
const char* last_error_cstr() { return t_last_error.c_str(); }

const char* device_error_message(int code) {
  switch (code) {
    case kErrIndexRange: return "Embedding index out of range";
    case kErrBarrierTimeout: return "a tensor-core pipeline wait timed out";
    case kErrTmemAlloc: return "tensor memory allocation failed";
    default: return "unknown device error";
  }
}

void* Context::ensure_scratch(size_t bytes) {
  if (bytes <= scratch_bytes) return scratch;
  TYSOR_CUDA(cudaStreamSynchronize(stream));
  if (scratch) TYSOR_CUDA(cudaFree(scratch));
  scratch = nullptr;
  size_t want = bytes + bytes / 4 + 4096;
  TYSOR_CUDA(cudaMalloc(&scratch, want));
  scratch_bytes = want;
  return scratch;
}

const float2* Context::rope_table(int64_t seq, int64_t half, double theta) {
  uint64_t bits;
  std::memcpy(&bits, &theta, sizeof bits);
  auto key = std::make_tuple(seq, half, bits);
  auto it = rope_tables.find(key);
  if (it != rope_tables.end()) return it->second;
  // Angles and their cos/sin are computed on the host with the C library in
  // f32, as layers.rs:254-262 computes them; the kernels then apply the
  // rotation with separately rounded products.
  std::vector<float> inv((size_t)(half > 0 ? half : 1));
  for (int64_t i = 0; i < half; ++i) inv[i] = powf((float)theta, -(float)i / (float)half);
  std::vector<float2> tab((size_t)(seq * half > 0 ? seq * half : 1));
  for (int64_t p = 0; p < seq; ++p)
    for (int64_t i = 0; i < half; ++i) {
      volatile float ang = (float)p * inv[i];
      tab[p * half + i] = make_float2(cosf(ang), sinf(ang));
    }
  float2* d = nullptr;
  TYSOR_CUDA(cudaMalloc(&d, sizeof(float2) * tab.size()));
  TYSOR_CUDA(cudaMemcpy(d, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice));
  rope_tables[key] = d;
  return d;
}

void Context::sync_and_check() {
  TYSOR_CUDA(cudaStreamSynchronize(stream));
  int code = 0;
  TYSOR_CUDA(cudaMemcpy(&code, d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    int zero = 0;
    TYSOR_CUDA(cudaMemcpy(d_err, &zero, sizeof(int), cudaMemcpyHostToDevice));
    throw CudaError(device_error_message(code));
  }
}

}  // namespace tysor

using namespace tysor;

namespace {

template <typename F>
bool guarded(F&& f) {
  try {
    f();
    return true;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return false;
  } catch (...) {
    set_last_error("unknown error");
    return false;
  }
}

Context* ctx_of(void* p) {
  if (!p) throw CudaError("null context");
  Context* c = static_cast<Context*>(p);
  TYSOR_CUDA(cudaSetDevice(c->device));
  return c;
}

Buffer* buf_of(void* p) {
  if (!p) throw CudaError("null buffer");
  return static_cast<Buffer*>(p);
}

float* ptr_of(void* p, size_t need, const char* what) {
  Buffer* b = buf_of(p);
  if (b->count < need)
    throw CudaError(std::string(what) + " buffer holds " + std::to_string(b->count) +
                    " elements, " + std::to_string(need) + " needed");
  return b->ptr;
}

GemmScratch gemm_scratch(Context* c, int batch, int64_t M, int64_t N, int64_t K,
                         const GemmOperand& A, const GemmOperand& Bm, int mode) {
  int64_t na = 0, nb = 0;
  gemm_scratch_need(batch, M, N, K, A, Bm, mode, &na, &nb);
  GemmScratch s{nullptr, nullptr, 0, 0};
  if (na + nb == 0) return s;
  const int64_t na_pad = (na + 63) & ~(int64_t)63;
  float* base = (float*)c->ensure_scratch(sizeof(float) * (size_t)(na_pad + nb + 64));
  s.a_lo = base;
  s.b_lo = base + na_pad;
  s.a_elems = na;
  s.b_elems = nb;
  return s;
}

void run_gemm(Context* c, int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A,
              const GemmOperand& Bm, const GemmOutput& out, const GemmEpilogue& ep_in) {
  GemmEpilogue ep = ep_in;
  ep.chunk_kb = c->accum_chunk_kb;
  const int mode =
      gemm_effective_mode(c->matmul_mode, batch, M, N, K, ep.tri, ep.smx_p != nullptr, out.ld, out.batch_stride);
  GemmScratch s = gemm_scratch(c, batch, M, N, K, A, Bm, mode);
  gemm_launch(batch, M, N, K, A, Bm, out, ep, mode, s, c->d_err, c->stream);
}

float* scratch_floats(Context* c, int64_t n) {
  return (float*)c->ensure_scratch(sizeof(float) * (size_t)(n > 0 ? n : 1));
}

}  // namespace

extern "C" {

const char* tysor_cuda_last_error(void) { return last_error_cstr(); }

void* tysor_cuda_context_new(int device) {
  Context* out = nullptr;
  guarded([&] {
    int n = 0;
    TYSOR_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n)
      throw CudaError("CUDA device " + std::to_string(device) + " not present (" +
                      std::to_string(n) + " visible)");
    cudaDeviceProp prop;
    TYSOR_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw CudaError(std::string("tysor_cuda is built for sm_100a; device is ") + prop.name);
    TYSOR_CUDA(cudaSetDevice(device));
    auto* c = new Context();
    c->device = device;
    TYSOR_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    TYSOR_CUDA(cudaMalloc(&c->d_err, 16));
    TYSOR_CUDA(cudaMemset(c->d_err, 0, 16));
    out = c;
  });
  return out;
}

void tysor_cuda_context_free(void* context) {
  if (!context) return;
  guarded([&] {
    Context* c = static_cast<Context*>(context);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& kv : c->rope_tables) cudaFree(kv.second);
    if (c->scratch) cudaFree(c->scratch);
    if (c->d_err) cudaFree(c->d_err);
    if (c->comm) tysor_cuda_comm_free(c);
    cudaStreamDestroy(c->stream);
    delete c;
  });
}

bool tysor_cuda_synchronize(void* context) {
  return guarded([&] { ctx_of(context)->sync_and_check(); });
}

bool tysor_cuda_set_matmul_accumulation(void* context, int kblocks) {
  return guarded([&] {
    if (kblocks < 0 || kblocks > 64) throw CudaError("accumulation chunk must be 0 (default) or 1..64 k-blocks");
    ctx_of(context)->accum_chunk_kb = kblocks;
  });
}

bool tysor_cuda_probe_wait_timeout(void* context, int64_t limit_cycles) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_wait_timeout_probe(c->d_err, (long long)limit_cycles, c->stream);
    c->sync_and_check();
  });
}

void* tysor_cuda_context_stream(void* context) {
  void* out = nullptr;
  guarded([&] { out = (void*)ctx_of(context)->stream; });
  return out;
}

bool tysor_cuda_set_matmul_mode(void* context, int mode) {
  return guarded([&] {
    if (mode < 0 || mode > 3)
      throw CudaError("matmul mode must be 0 (strict), 1 (fast), 2 (exact) or 3 (strict16)");
    ctx_of(context)->matmul_mode = mode;
  });
}

void* tysor_cuda_buffer_new_zeroed(void* context, size_t count) {
  Buffer* out = nullptr;
  guarded([&] {
    Context* c = ctx_of(context);
    auto* b = new Buffer();
    b->ctx = c;
    b->count = count;
    b->owned = true;
    TYSOR_CUDA(cudaMalloc(&b->ptr, sizeof(float) * (count ? count : 1)));
    TYSOR_CUDA(cudaMemsetAsync(b->ptr, 0, sizeof(float) * (count ? count : 1), c->stream));
    out = b;
  });
  return out;
}

void* tysor_cuda_buffer_new_with_data(void* context, const float* data, size_t count) {
  void* b = tysor_cuda_buffer_new_zeroed(context, count);
  if (!b) return nullptr;
  if (!tysor_cuda_buffer_write(b, data, count)) {
    tysor_cuda_buffer_free(b);
    return nullptr;
  }
  return b;
}

void tysor_cuda_buffer_free(void* buffer) {
  if (!buffer) return;
  Buffer* b = static_cast<Buffer*>(buffer);
  if (b->owned && b->ptr) {
    cudaSetDevice(b->ctx->device);
    cudaStreamSynchronize(b->ctx->stream);
    cudaFree(b->ptr);
  }
  delete b;
}

bool tysor_cuda_buffer_read(void* buffer, float* out_data, size_t count) {
  return guarded([&] {
    Buffer* b = buf_of(buffer);
    if (count > b->count) throw CudaError("buffer read past the end");
    ctx_of(b->ctx)->sync_and_check();
    TYSOR_CUDA(cudaMemcpy(out_data, b->ptr, sizeof(float) * count, cudaMemcpyDeviceToHost));
  });
}

bool tysor_cuda_buffer_write(void* buffer, const float* data, size_t count) {
  return guarded([&] {
    Buffer* b = buf_of(buffer);
    if (count > b->count) throw CudaError("buffer write past the end");
    Context* c = ctx_of(b->ctx);
    TYSOR_CUDA(cudaMemcpyAsync(b->ptr, data, sizeof(float) * count, cudaMemcpyHostToDevice, c->stream));
    TYSOR_CUDA(cudaStreamSynchronize(c->stream));
  });
}

void* tysor_cuda_buffer_view(void* base, size_t offset, size_t count) {
  Buffer* out = nullptr;
  guarded([&] {
    Buffer* b = buf_of(base);
    if (offset + count > b->count) throw CudaError("view outside its base buffer");
    auto* v = new Buffer();
    v->ctx = b->ctx;
    v->ptr = b->ptr + offset;
    v->count = count;
    v->owned = false;
    out = v;
  });
  return out;
}

size_t tysor_cuda_buffer_count(void* buffer) { return buffer ? buf_of(buffer)->count : 0; }

// ---- forward dispatch --------------------------------------------------------

bool tysor_cuda_dispatch_matmul(void* context, void* lhs, void* rhs, void* out, uint32_t m,
                                uint32_t n, uint32_t k) {
  return tysor_cuda_dispatch_linear(context, lhs, rhs, nullptr, out, m, n, k, false);
}

bool tysor_cuda_dispatch_linear(void* context, void* input, void* weight, void* bias, void* out,
                                uint32_t m, uint32_t n, uint32_t k, bool with_bias) {
  return guarded([&] {
    Context* c = ctx_of(context);
    GemmOperand A{ptr_of(input, (size_t)m * k, "lhs"), false, (int64_t)k, 0};
    GemmOperand Bm{ptr_of(weight, (size_t)k * n, "rhs"), false, (int64_t)n, 0};
    GemmOutput O{ptr_of(out, (size_t)m * n, "out"), (int64_t)n, 0};
    GemmEpilogue ep{with_bias ? ptr_of(bias, n, "bias") : nullptr, 1.0f, 0, 0};
    run_gemm(c, 1, m, n, k, A, Bm, O, ep);
  });
}

bool tysor_cuda_dispatch_matmul_ex(void* context, uint32_t batch, uint32_t m, uint32_t n,
                                   uint32_t k, void* a, bool trans_a, uint64_t lda,
                                   uint64_t stride_a, void* b, bool trans_b, uint64_t ldb,
                                   uint64_t stride_b, void* cbuf, uint64_t ldc, uint64_t stride_c,
                                   void* bias, float alpha, bool accumulate, bool relu) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (batch == 0) return;
    const uint64_t a_rows = trans_a ? k : m, a_cols = trans_a ? m : k;
    const uint64_t b_rows = trans_b ? n : k, b_cols = trans_b ? k : n;
    if (lda < a_cols || ldb < b_cols || ldc < n) throw CudaError("matmul_ex: leading dimension too small");
    const size_t a_need = (batch - 1) * stride_a + (a_rows ? (a_rows - 1) * lda + a_cols : 0);
    const size_t b_need = (batch - 1) * stride_b + (b_rows ? (b_rows - 1) * ldb + b_cols : 0);
    const size_t c_need = (batch - 1) * stride_c + (m ? (m - 1) * ldc + n : 0);
    GemmOperand A{ptr_of(a, a_need, "a"), trans_a, (int64_t)lda, (int64_t)stride_a};
    GemmOperand Bm{ptr_of(b, b_need, "b"), trans_b, (int64_t)ldb, (int64_t)stride_b};
    GemmOutput O{ptr_of(cbuf, c_need, "c"), (int64_t)ldc, (int64_t)stride_c};
    GemmEpilogue ep{bias ? ptr_of(bias, n, "bias") : nullptr, alpha, accumulate ? 1 : 0, relu ? 1 : 0};
    run_gemm(c, (int)batch, m, n, k, A, Bm, O, ep);
  });
}

bool tysor_cuda_dispatch_unary(void* context, int op, void* input, void* out, uint32_t count,
                               float param) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (op < 0 || op > 3) throw CudaError("unknown unary op");
    launch_unary(op, ptr_of(input, count, "input"), ptr_of(out, count, "out"), count, param, c->stream);
  });
}

bool tysor_cuda_dispatch_binary_tt(void* context, int op, void* lhs, void* rhs, void* out,
                                   uint32_t count) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (op < 0 || op > 3) throw CudaError("unsupported tensor binary op");
    launch_binary_tt(op, ptr_of(lhs, count, "lhs"), ptr_of(rhs, count, "rhs"), ptr_of(out, count, "out"),
                     count, c->stream);
  });
}

bool tysor_cuda_dispatch_binary_ts(void* context, int op, void* input, void* out, uint32_t count,
                                   double scalar) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (op < 0 || op > 3) throw CudaError("unsupported tensor binary op");
    launch_binary_ts(op, ptr_of(input, count, "input"), (float)scalar, ptr_of(out, count, "out"), count,
                     c->stream);
  });
}

bool tysor_cuda_dispatch_binary_st(void* context, int op, void* input, void* out, uint32_t count,
                                   double scalar) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (op < 0 || op > 3) throw CudaError("unsupported tensor binary op");
    launch_binary_st(op, (float)scalar, ptr_of(input, count, "input"), ptr_of(out, count, "out"), count,
                     c->stream);
  });
}

bool tysor_cuda_dispatch_rms_norm(void* context, void* input, void* out, uint32_t rows,
                                  uint32_t width) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_rms_norm(ptr_of(input, n, "input"), ptr_of(out, n, "out"), rows, width, c->stream);
  });
}

bool tysor_cuda_dispatch_softmax(void* context, void* input, void* out, uint32_t rows,
                                 uint32_t width) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_softmax(ptr_of(input, n, "input"), ptr_of(out, n, "out"), rows, width, c->stream);
  });
}

bool tysor_cuda_dispatch_cross_entropy(void* context, void* logits, void* target, void* out,
                                       uint32_t rows, uint32_t width) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_cross_entropy(ptr_of(logits, n, "logits"), ptr_of(target, n, "target"), ptr_of(out, rows, "out"),
                         rows, width, c->stream);
  });
}

bool tysor_cuda_dispatch_embedding(void* context, void* indices, void* weight, void* out,
                                   uint32_t index_count, uint32_t embedding_dim,
                                   uint32_t num_embeddings) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_embedding(ptr_of(indices, index_count, "indices"),
                     ptr_of(weight, (size_t)num_embeddings * embedding_dim, "weight"),
                     ptr_of(out, (size_t)index_count * embedding_dim, "out"), index_count,
                     num_embeddings, embedding_dim, c->d_err, c->stream);
  });
}

bool tysor_cuda_dispatch_repeat_kv(void* context, void* input, void* out, uint32_t outer,
                                   uint32_t out_heads, uint32_t inner, uint32_t repeats) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (repeats == 0 || out_heads % repeats != 0) throw CudaError("repeat_kv repeats must divide the output heads");
    const uint32_t heads = out_heads / repeats;
    launch_repeat_kv(ptr_of(input, (size_t)outer * heads * inner, "input"),
                     ptr_of(out, (size_t)outer * out_heads * inner, "out"), outer, heads, inner, repeats,
                     c->stream);
  });
}

bool tysor_cuda_dispatch_causal_mask(void* context, void* input, void* out, uint32_t outer,
                                     uint32_t q, uint32_t k) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)outer * q * k;
    launch_causal_mask(ptr_of(input, n, "input"), ptr_of(out, n, "out"), outer, q, k, c->stream);
  });
}

bool tysor_cuda_dispatch_rope(void* context, void* input, void* out, uint32_t outer,
                              uint32_t seq_len, uint32_t half_dim, double theta) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)outer * seq_len * half_dim * 2;
    const float2* tab = c->rope_table(seq_len, half_dim, theta);
    launch_rope(ptr_of(input, n, "input"), ptr_of(out, n, "out"), tab, outer, seq_len, half_dim, c->stream);
  });
}

// ---- backward and update -------------------------------------------------------------

bool tysor_cuda_dispatch_relu_backward(void* context, void* out_act, void* grad, void* dx,
                                       uint64_t count, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_relu_backward(ptr_of(out_act, count, "out"), ptr_of(grad, count, "grad"), ptr_of(dx, count, "dx"),
                         count, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_silu_backward(void* context, void* input, void* grad, void* dx,
                                       uint64_t count, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_silu_backward(ptr_of(input, count, "input"), ptr_of(grad, count, "grad"), ptr_of(dx, count, "dx"),
                         count, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_softmax_backward(void* context, void* output, void* grad, void* dx,
                                          uint64_t count, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_softmax_backward(ptr_of(output, count, "output"), ptr_of(grad, count, "grad"),
                            ptr_of(dx, count, "dx"), count, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_cross_entropy_backward(void* context, void* logits, void* target,
                                                void* grad, uint32_t rows, uint32_t width,
                                                bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_cross_entropy_backward(ptr_of(logits, n, "logits"), ptr_of(target, n, "target"),
                                  ptr_of(grad, n, "grad"), rows, width, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_rope_backward(void* context, void* grad, void* dx, uint32_t outer,
                                       uint32_t seq_len, uint32_t half_dim, double theta,
                                       bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)outer * seq_len * half_dim * 2;
    const float2* tab = c->rope_table(seq_len, half_dim, theta);
    launch_rope_backward(ptr_of(grad, n, "grad"), ptr_of(dx, n, "dx"), tab, outer, seq_len, half_dim,
                         accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_repeat_kv_backward(void* context, void* grad, void* dx, uint32_t outer,
                                            uint32_t heads, uint32_t inner, uint32_t repeats,
                                            bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (repeats == 0) throw CudaError("repeat_kv backward requires repeats > 0");
    launch_repeat_kv_backward(ptr_of(grad, (size_t)outer * heads * repeats * inner, "grad"),
                              ptr_of(dx, (size_t)outer * heads * inner, "dx"), outer, heads, inner,
                              repeats, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_causal_mask_backward(void* context, void* grad, void* dx, uint32_t outer,
                                              uint32_t q, uint32_t k, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)outer * q * k;
    launch_causal_mask_backward(ptr_of(grad, n, "grad"), ptr_of(dx, n, "dx"), outer, q, k, accumulate,
                                c->stream);
  });
}

bool tysor_cuda_dispatch_embedding_backward(void* context, void* grad, void* indices,
                                            void* weight_grad, uint32_t index_count,
                                            uint32_t embedding_dim, uint32_t num_embeddings,
                                            bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    void* work = c->ensure_scratch(embedding_backward_work_bytes(index_count, num_embeddings));
    launch_embedding_backward(ptr_of(grad, (size_t)index_count * embedding_dim, "grad"),
                              ptr_of(indices, index_count, "indices"),
                              ptr_of(weight_grad, (size_t)num_embeddings * embedding_dim, "weight_grad"),
                              index_count, num_embeddings, embedding_dim, work, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_bias_grad(void* context, void* grad, void* bias_grad, uint32_t rows,
                                   uint32_t width, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    float* partial = scratch_floats(c, colsum_partial_elems(rows, width));
    launch_colsum(ptr_of(grad, (size_t)rows * width, "grad"), ptr_of(bias_grad, width, "bias_grad"), partial,
                  rows, width, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_add_inplace(void* context, void* dst, void* src, uint64_t count) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_add_inplace(ptr_of(dst, count, "dst"), ptr_of(src, count, "src"), count, c->stream);
  });
}

bool tysor_cuda_dispatch_sgd_update(void* context, void* param, void* grad, uint64_t count,
                                    double lr) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_sgd(ptr_of(param, count, "param"), ptr_of(grad, count, "grad"), (float)lr, count, c->stream);
  });
}

bool tysor_cuda_dispatch_reduce_sum(void* context, void* input, void* out, uint64_t count) {
  return guarded([&] {
    Context* c = ctx_of(context);
    float* partial = scratch_floats(c, 1024);
    launch_reduce_sum(ptr_of(input, count, "input"), ptr_of(out, 1, "out"), partial, count, c->stream);
  });
}

bool tysor_cuda_dispatch_rms_norm_gain(void* context, void* input, void* gain, void* out,
                                       uint32_t rows, uint32_t width, float eps) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_rms_norm_gain(ptr_of(input, n, "input"), ptr_of(gain, width, "gain"), ptr_of(out, n, "out"), rows,
                         width, eps, c->stream);
  });
}

bool tysor_cuda_dispatch_rms_norm_gain_backward(void* context, void* input, void* gain, void* dy,
                                                void* dx, void* dgain, uint32_t rows,
                                                uint32_t width, float eps, bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    float* partial = scratch_floats(c, rms_gain_partial_elems(rows, width));
    launch_rms_norm_gain_backward(ptr_of(input, n, "input"), ptr_of(gain, width, "gain"), ptr_of(dy, n, "dy"),
                                  ptr_of(dx, n, "dx"), ptr_of(dgain, width, "dgain"), partial, rows, width,
                                  eps, accumulate, accumulate, c->stream);
  });
}

bool tysor_cuda_dispatch_cross_entropy_labels(void* context, void* logits, void* labels,
                                              void* out, uint32_t rows, uint32_t width) {
  return guarded([&] {
    Context* c = ctx_of(context);
    launch_cross_entropy_labels(ptr_of(logits, (size_t)rows * width, "logits"), ptr_of(labels, rows, "labels"),
                                ptr_of(out, rows, "out"), rows, width, c->d_err, c->stream);
  });
}

bool tysor_cuda_dispatch_cross_entropy_labels_backward(void* context, void* logits, void* labels,
                                                       void* grad, uint32_t rows, uint32_t width,
                                                       bool accumulate) {
  return guarded([&] {
    Context* c = ctx_of(context);
    const size_t n = (size_t)rows * width;
    launch_cross_entropy_labels_backward(ptr_of(logits, n, "logits"), ptr_of(labels, rows, "labels"),
                                         ptr_of(grad, n, "grad"), rows, width, accumulate, c->d_err,
                                         c->stream);
  });
}

bool tysor_cuda_dispatch_transpose(void* context, void* input, void* out, const int64_t* dims,
                                   int rank, int a, int b) {
  return guarded([&] {
    Context* c = ctx_of(context);
    if (rank < 1 || rank > 8 || a < 0 || b < 0 || a >= rank || b >= rank)
      throw CudaError("transpose axis out of range");
    size_t n = 1;
    for (int i = 0; i < rank; ++i) n *= (size_t)dims[i];
    launch_transpose(ptr_of(input, n, "input"), ptr_of(out, n, "out"), dims, rank, a < b ? a : b,
                     a < b ? b : a, 0, c->stream);
  });
}

}  // extern "C"
