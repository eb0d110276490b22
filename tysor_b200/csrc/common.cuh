// Shared definitions for the tysor CUDA backend (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <stdexcept>
#include <string>

namespace tysor {

// The low part of x for 3xTF32: x - tf32_trunc(x) (exact in fp32; the
// tensor core reads x itself as the high part and ignores its low 13 mantissa
// bits), rounded to the nearest tf32 value, ties to even.  Left unrounded, the
// tensor core would truncate the low part too, a bias toward zero of about
// 2^-22 of x on every operand; rounded, it reads the low part exactly and the
// remaining error (at most 2^-12 of the low part) is unbiased.
__device__ __forceinline__ float tf32_lo(float x) {
  const float lo = x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  const uint32_t u = __float_as_uint(lo);
  return __uint_as_float((u + 0x0FFFu + ((u >> 13) & 1u)) & 0xFFFFE000u);
}

// Kernel launches enqueued by this library (every launcher adds to it).
extern std::atomic<int64_t> g_launches;

// Error codes written by kernels into the context's device error word.  A
// kernel never traps: it records the first problem it sees and returns, and
// the host turns the word into an error message at the next check.
enum DeviceError : int {
  kErrNone = 0,
  kErrIndexRange = 1,      // embedding / label index outside [0, n)
  kErrBarrierTimeout = 2,  // an mbarrier wait ran past its time limit
  kErrTmemAlloc = 3,
};

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

#define TYSOR_CUDA(call) ::tysor::check_cuda((call), #call)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Grid size for a grid-stride elementwise loop: a few waves of the 148 SMs.
inline int elementwise_blocks(int64_t n, int threads) {
  int64_t want = ceil_div(n, threads);
  int64_t cap = 148 * 16;
  if (want > cap) want = cap;
  return (int)(want < 1 ? 1 : want);
}

// ---------------------------------------------------------------------------
// GEMM interface (gemm.cu).
// C[b] = alpha * op(A[b]) . op(B[b])  (+ bias) (relu) (+ C_old when accumulate)
// op(A) is [M, K]: A stored [M, K] row-major (trans_a = false) or [K, M]
// (trans_a = true).  op(B) is [K, N]: B stored [K, N] (trans_b = false) or
// [N, K] (trans_b = true).  All fp32.
// ---------------------------------------------------------------------------
struct GemmOperand {
  const float* ptr;
  bool trans;
  int64_t ld;            // row pitch of the stored matrix, in elements
  int64_t batch_stride;  // elements between batch items (0 for one item)
};

struct GemmOutput {
  float* ptr;
  int64_t ld;
  int64_t batch_stride;
};

struct GemmEpilogue {
  const float* bias;  // [N] or null
  float alpha;        // multiplies the product (1.0f for plain matmul)
  int accumulate;     // 1: C = C_old + result
  int relu;           // 1: result = max(result, 0)
  // Causal structure of a batched attention GEMM (tensor-core kernels only;
  // every skipped term is an exact zero or an output nobody reads):
  // 0 none; 1 skip output tiles whose columns all exceed their rows;
  // 2 contract only k < end of the tile's rows; 3 only k >= start of the
  // tile's rows; 4 only k >= start of the tile's columns.
  int tri = 0;
  // Non-null: the GEMM is the probability gradient dP of a causal
  // Softmax(causal_mask(.)) and writes, instead of dP, the mask input's
  // gradient dS = (p * (1 - p)) * dP (the reference's diagonal softmax
  // backward), 0 where col > row; `smx_p` holds p in C's layout.  Only
  // where gemm_fuses_softmax_backward holds.
  const float* smx_p = nullptr;
  // Non-null: C = residual + the result (residual in C's layout; a residual
  // connection around a linear).  Only where gemm_fuses_box_epilogue holds.
  const float* residual = nullptr;
  // Tensor-core kernels: k-blocks (16 elements of K each) accumulated in
  // tensor memory before the accumulator warps add the partial sum into
  // fp32 registers with round-to-nearest; 0 = the default (8).  The tensor
  // core adds each MMA into its accumulator rounding toward zero, so shorter
  // chunks shrink that systematic error (and cost the readout more often).
  int chunk_kb = 0;
  // Set by the launcher for the split-fp16 kernel: the per-row factors of
  // the packed A ([M]) and B ([N]) operands (see launch_pack16).
  const float* row_factor = nullptr;
  const float* col_factor = nullptr;
};

enum GemmMode : int {
  kGemmStrict = 0,    // 3xTF32 split: fp32-level accuracy
  kGemmFast = 1,      // 1xTF32
  kGemmExact = 2,     // CUDA-core fp32, products and sums in k order (bit-exact)
  kGemmStrict16 = 3,  // 3-product split over fp16 halves with per-row scaling (kind::f16):
                      // fp32-level accuracy at twice the tensor rate of 3xTF32; GEMMs it
                      // does not cover run as kGemmStrict (gemm_effective_mode)
};

// The mode a GEMM of this shape runs in: kGemmStrict16 covers unbatched,
// non-causal GEMMs with M >= 256, N > 128 and C on 16-byte strides, without
// the fused softmax backward; the others run strict 3xTF32.  Every other
// mode is returned unchanged.  Callers size scratch and launch with the
// returned mode.
int gemm_effective_mode(int mode, int batch, int64_t M, int64_t N, int64_t K, int tri, bool smx, int64_t ldc,
                        int64_t stride_c);

// Split-fp16 packing of one GEMM operand with R rows (M for A, N for B) and
// K columns, K-major: hi [R][Kp] and lo [R][Kp] fp16 (Kp = K rounded up to
// a multiple of 8), then factor [R] fp32, then (for an operand stored with
// R contiguous) R words of scratch.  Per row r, x is scaled by 2^e(r), the
// power of two that puts the row's largest magnitude in [2^14, 2^15) (e
// clamped to [-63, 63]; 0 for a zero or non-finite maximum); hi = fp16(x
// 2^e), lo = fp16(x 2^e - hi), factor = 2^-e.  hi + lo hold 22 significant
// bits of x, as 3xTF32's two parts do.  `k_contiguous`: x stored [R][ld]
// (K contiguous); else [K][ld] (R contiguous).
int64_t gemm_pack16_elems(int64_t rows, int64_t K);
void launch_pack16(const float* x, bool k_contiguous, int64_t rows, int64_t K, int64_t ld, float* packed,
                   cudaStream_t st);

// Scratch the strict-mode GEMM needs: one "lo" copy of each operand, laid
// out like the operand (no a_lo when gemm_converts_a).  With `presplit` set
// the copies already hold lo(A), lo(B) and the launcher does not recompute
// them.  In kGemmStrict16 mode a_lo and b_lo hold the packed operands
// (gemm_pack16_elems floats each; packed by the launcher unless presplit).
struct GemmScratch {
  float* a_lo;
  float* b_lo;
  int64_t a_elems;
  int64_t b_elems;
  int presplit = 0;
  // Optional workspace for split-K partial sums (16-byte aligned): a GEMM
  // whose output tiles cannot fill the GPU may split its K range into up to
  // 4 parts, written here and summed in a fixed order (deterministic).
  float* ws = nullptr;
  int64_t ws_elems = 0;
};

// Workspace elements a split-K launch of this GEMM would need (0: it would
// not split).
int64_t gemm_splitk_ws_elems(int batch, int64_t M, int64_t N, int64_t K, int mode, int64_t ldc, int64_t stride_c);

// Whether gemm_launch runs this strict GEMM (C 16-byte aligned, with these
// strides) on the kernel form that makes A's low part in shared memory:
// its scratch then needs no a_lo (only b_lo).
bool gemm_converts_a(int batch, int64_t M, int64_t N, int64_t K, int mode, int64_t ldc, int64_t stride_c);

// Whether gemm_launch can run GemmEpilogue::smx_p's softmax backward or
// GemmEpilogue::residual's addition in the GEMM's epilogue for this shape
// and operand layout (ta / tb as in GemmOperand::trans).
bool gemm_fuses_box_epilogue(int batch, int64_t M, int64_t N, int64_t K, bool ta, bool tb, int mode,
                             int64_t ldc, int64_t stride_c);

// Whether gemm_launch may use the 2-SM (cta_group::2 cluster pair) kernel.
extern bool g_two_sm_enabled;

// One thread waits, with the GEMM pipelines' bounded mbarrier wait, on a
// barrier that nothing arrives at; after `limit_cycles` the wait gives up
// and records kErrBarrierTimeout in *err.  Checks the timeout path without
// faulting or hanging the GPU.
void launch_wait_timeout_probe(int* err, long long limit_cycles, cudaStream_t st);

// lo(x) = tf32_lo(x) (x - tf32_trunc(x), rounded to tf32) over n contiguous elements.
void launch_split_lo(const float* x, float* lo, int64_t n, cudaStream_t st);
// Per batch item b: hi_t[b][c][r] = x[b][r][c] and lo_t = lo(hi_t) (lo_t may
// be null), for a contiguous [batch][rows][cols] x.
void launch_split_transpose(const float* x, float* hi_t, float* lo_t, int64_t batch, int64_t rows,
                            int64_t cols, cudaStream_t st);

// Returns the number of elements of scratch each operand needs in strict
// mode (0 when the call runs on the CUDA-core path).
void gemm_scratch_need(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A,
                       const GemmOperand& B, int mode, int64_t* a_elems, int64_t* b_elems);

// Rows per tile of the causal ranges (GemmEpilogue::tri) gemm_launch would
// use for this GEMM: with tri 2 a row's contraction ends at the end of its
// tile of this many rows (rounded up to 16), with tri 3 it starts at the
// start of its tile.  0: the CUDA-core path, which contracts all of K.
int gemm_causal_tile_rows(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A, const GemmOperand& B,
                          const GemmOutput& C, int mode);

// Launches the GEMM on `stream`.  Throws CudaError on a launch problem.
// Picks the tcgen05 path when every TMA alignment rule holds, else the
// CUDA-core path.  Returns 1 if the tensor-core path ran, 0 otherwise.
int gemm_launch(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A,
                const GemmOperand& B, const GemmOutput& C, const GemmEpilogue& ep, int mode,
                const GemmScratch& scratch, int* d_err, cudaStream_t stream);

}  // namespace tysor
