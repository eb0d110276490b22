// fp32 matmul for sm_100a.
//
// Tensor-core path: a tcgen05 kernel.  TMA (cp.async.bulk.tensor) stages
// 128 x 16 (A) and BN x 16 (B) fp32 tiles in shared memory through a 4-stage
// mbarrier ring; one elected thread issues tcgen05.mma.kind::tf32 with the
// accumulator in tensor memory (128 lanes x BN fp32 columns); four warps read
// the accumulator back with tcgen05.ld and apply the epilogue (alpha, bias,
// relu, accumulate-into-C).
//
// Strict mode (the default) is 3xTF32: each operand x is used as-is (the
// tensor core reads its top 19 bits, i.e. the tf32 truncation hi(x)) and as
// lo(x) = x - hi(x), prepared in scratch memory by split_lo_kernel; the
// products hi*hi + hi*lo + lo*hi recover fp32-level accuracy.  Fast mode
// issues only hi*hi.
//
// Both operand layouts are supported without copies: a K-contiguous operand
// is staged with 64-byte swizzle (K-major UMMA descriptor), an
// M/N-contiguous one with 128-byte swizzle (MN-major descriptor), so the
// transposed products of backward (dY.W^T, X^T.dY) read the stored tensors
// directly.
//
// Split-fp16 strict mode (kGemmStrict16): the operands are packed K-major
// into fp16 high and low halves with a power-of-two scale per row
// (launch_pack16), the persistent pair kernel issues the same three products
// with tcgen05.mma.kind::f16 (twice the tf32 rate per instruction slot: 16
// elements of K per 32-byte slice instead of 8), and the epilogue multiplies
// each output by its row's and column's inverse scales (exact powers of two).
//
// CUDA-core path: products and sums rounded separately in increasing k
// order (bit-identical to a sequential fp32 loop).  It serves shapes whose
// strides break TMA's 16-byte rules and the opt-in exact mode.
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"

namespace tysor {
namespace {

constexpr int BM = 128;
constexpr int BK = 16;  // fp32 elements of K per stage (64 bytes)
constexpr int kGroupM = 16;  // tile rows per raster group of the 1-SM kernel
constexpr long long kWaitCycles = 4000000000LL;  // about 2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the given phase parity; gives up after `limit` cycles,
// recording kErrBarrierTimeout, so a lost arrival can never hang the GPU.
__device__ bool mbar_wait_limit(uint32_t bar, uint32_t parity, int* err, long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) {
      atomicCAS(err, 0, (int)kErrBarrierTimeout);
      return false;
    }
  }
  return true;
}

__device__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
  return mbar_wait_limit(bar, parity, err, kWaitCycles);
}

// One thread initialises a barrier that expects one arrival, never arrives,
// and waits on it with the pipelines' own wait: the wait must give up after
// `limit` cycles and record kErrBarrierTimeout.  No copy or MMA is in flight.
__global__ void wait_timeout_probe_kernel(int* err, long long limit) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  mbar_wait_limit(b, 0, err, limit);
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

// Layout types of the descriptor (bits 61-63).
constexpr uint32_t kLayoutSW128Base32B = 1;  // 128-byte rows, 32-byte chunks swizzled
constexpr uint32_t kLayoutSW64 = 4;

// Descriptor of the k-th (8-deep) MMA slice of a staged operand tile.
// K-major tiles: rows of 64 bytes, 8-row swizzle atoms of 512 bytes; the
// slice offset is 32 bytes inside the atom.  MN-major tiles (32-bit
// elements admit only the "128B, 32-byte atom" swizzle): blocks of 32 M/N
// elements x 16 k-rows of 128 bytes (2 KiB per block, LBO), 4-row swizzle
// atoms (512 bytes, SBO); the slice offset is 8 k-rows (1 KiB).
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, bool mn_major, int kslice) {
  if (mn_major) return smem_desc(tile + 1024u * kslice, 2048u, 512u, kLayoutSW128Base32B);
  return smem_desc(tile + 32u * kslice, 16u, 512u, kLayoutSW64);
}

template <int BN>
struct TileCfg {
  static constexpr int kABytes = BM * BK * 4;
  static constexpr int kBBytes = BN * BK * 4;
};

template <int BN, bool kStrict>
struct PipeCfg {
  static constexpr int kA = TileCfg<BN>::kABytes;
  static constexpr int kB = TileCfg<BN>::kBBytes;
  static constexpr int kStageBytes = kStrict ? 2 * (kA + kB) : (kA + kB);
  static constexpr int kStagesRaw = (192 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

// The tensor core adds each MMA's products into the accumulator with
// round-toward-zero, so a long K run in one accumulator drifts by up to
// (number of MMAs) x 2^-24 relative.  The kernel therefore accumulates K in
// chunks of kChunkKb k-blocks (128 elements) into one of two tensor-memory
// buffers, and eight "accumulator" warps add each finished chunk into fp32
// registers with round-to-nearest while the tensor core fills the other
// buffer.  The error stays at the chunk level (about 1.4e-6 relative in
// strict mode) whatever K is.
constexpr int kChunkKb = 8;

__device__ __forceinline__ int chunk_kb(const GemmEpilogue& ep) { return ep.chunk_kb > 0 ? ep.chunk_kb : kChunkKb; }
constexpr int kAccWarps = 8;
constexpr int kThreadsTC = 64 + 32 * kAccWarps;

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Causal attention GEMMs (GemmEpilogue::tri): for a tile of rows
// [r0, r0 + rows) and columns from c0, narrows the k-block range to the
// terms that can be nonzero, or returns true when the whole output tile is
// above the diagonal and nobody reads it (mode 1).
__device__ __forceinline__ bool causal_range(int tri, int r0, int rows, int c0, int* kb_begin, int* kb_end) {
  switch (tri) {
    case 1: return c0 >= r0 + rows;
    case 2: {
      const int e = (r0 + rows + BK - 1) / BK;
      if (e < *kb_end) *kb_end = e;
      return false;
    }
    case 3: *kb_begin = r0 / BK; return false;
    case 4: *kb_begin = c0 / BK; return false;
    default: return false;
  }
}

// Tile stores from shared memory (bulk async proxy).  `add` reduces into
// global memory (C = C + tile, round-to-nearest), which is the accumulate
// epilogue's `existing + new`.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z,
                                             bool add) {
  if (add)
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            (uint64_t)map),
        "r"(src), "r"(x), "r"(y), "r"(z)
        : "memory");
  else
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     (uint64_t)map),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// Output staging for the tile-store epilogue: boxes of 32 columns x BM rows
// (128-byte rows, 128-byte swizzle: 16-byte chunk j of row r sits at chunk
// j ^ (r & 7)), so a warp writing 32 rows' chunk j touches every bank.
__device__ __forceinline__ uint32_t c_stage_addr(uint32_t base, int box, int row, int chunk) {
  return base + (uint32_t)box * (BM * 128) + (uint32_t)row * 128 + (uint32_t)((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void st_shared_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Epilogue of one CTA's 128 x BN tile, run by the 8 accumulator warps
// (thread = row quad*32 + lane, columns half*BN/2 ...): alpha, bias, relu,
// then the tile goes through shared memory.  The stage ring is idle once the
// last chunk has been read (every MMA has completed), so the tile is staged
// there; TMA then writes it in 32-column boxes (full 128-byte rows rather
// than one 16-byte piece per row per store; `accumulate` becomes a tile
// reduce-add), or, where C's strides rule TMA out, all 256 threads copy it
// out row-contiguously.
template <int BN>
__device__ __forceinline__ void tile_epilogue(float (&acc)[BN / 2], bool have, uint8_t* smem,
                                              const CUtensorMap* map_c, int c_tma, const GemmOutput& out,
                                              const GemmEpilogue& ep, int M, int N, int m0, int n0, int bz,
                                              int quad, int half, int lane, int tid) {
  constexpr int kHalf = BN / 2;
  const int col0 = n0 + half * kHalf;
  const uint32_t sbase = smem_u32(smem);
  if (have) {
#pragma unroll
    for (int i = 0; i < kHalf; ++i) {
      float r = acc[i] * ep.alpha;
      if (ep.bias != nullptr && col0 + i < N) r = r + ep.bias[col0 + i];
      if (ep.relu) r = fmaxf(r, 0.0f);
      acc[i] = r;
    }
    const int r_local = quad * 32 + lane;
#pragma unroll
    for (int b = 0; b < kHalf / 32; ++b)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        st_shared_f4(c_stage_addr(sbase, half * (kHalf / 32) + b, r_local, j), acc[b * 32 + 4 * j],
                     acc[b * 32 + 4 * j + 1], acc[b * 32 + 4 * j + 2], acc[b * 32 + 4 * j + 3]);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kAccWarps) : "memory");
  if (c_tma) {
    if (tid == 64) {
#pragma unroll 1
      for (int b = 0; b < BN / 32; ++b)
        if (n0 + 32 * b < N) tma_store_3d(map_c, sbase + (uint32_t)b * (BM * 128), n0 + 32 * b, m0, bz, ep.accumulate);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
  } else {
    const int t = tid - 64;
    float* cbase = out.ptr + (int64_t)bz * out.batch_stride;
#pragma unroll 1
    for (int idx = t; idx < BM * (BN / 4); idx += 32 * kAccWarps) {
      const int r = idx / (BN / 4), c4 = idx % (BN / 4);
      const int grow = m0 + r, gcol = n0 + 4 * c4;
      if (grow >= M || gcol >= N) continue;
      float v[4];
      asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                   : "r"(c_stage_addr(sbase, c4 >> 3, r, c4 & 7)));
      float* dst = cbase + (int64_t)grow * out.ld + gcol;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (gcol + q < N) dst[q] = ep.accumulate ? dst[q] + v[q] : v[q];
    }
  }
}

template <int BN, bool kStrict, bool kAmn, bool kBmn>
__global__ void __launch_bounds__(kThreadsTC, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_alo,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_blo,
                     const __grid_constant__ CUtensorMap map_c, GemmOutput out,
                     GemmEpilogue ep, int M, int N, int K, int c_tma, int* err) {
  using Cfg = PipeCfg<BN, kStrict>;
  static_assert(Cfg::kStages * Cfg::kStageBytes >= BM * BN * 4, "output staging must fit the stage ring");
  constexpr int kA = Cfg::kA;
  constexpr int kB = Cfg::kB;
  constexpr int kStages = Cfg::kStages;
  constexpr int kStageBytes = Cfg::kStageBytes;
  constexpr uint32_t kTxBytes = kStageBytes;
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr int kHalf = BN / 2;  // columns per accumulator warp
  constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kAmn ? 1u : 0u) << 15) |
                              ((kBmn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                              ((uint32_t)(BM >> 4) << 24);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1 KiB alignment for the swizzle atoms.
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + kStages * kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;       // [2] chunk accumulated
  uint64_t* tempty_bar = bars + 2 * kStages + 2;  // [2] chunk read back
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kStages + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // Grouped raster: consecutive CTAs take kGroupM tile rows of one tile
  // column before moving to the next column, so the CTAs resident at once
  // share a band of A rows and a few B columns in L2 instead of each wave
  // streaming all of B (an [N, K] operand larger than L2 would otherwise be
  // re-read from HBM once per tile row).
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
  const int per_group = kGroupM * tiles_n;
  const int first_m = (int)(blockIdx.x / per_group) * kGroupM;
  const int gsize = min(tiles_m - first_m, kGroupM);
  const int in_group = (int)(blockIdx.x % per_group);
  const int m0 = (first_m + in_group % gsize) * BM;
  const int n0 = (in_group / gsize) * BN;
  const int bz = blockIdx.z;
  int kb_begin = 0, kb_end = (K + BK - 1) / BK;
  if (ep.tri != 0 && causal_range(ep.tri, m0, BM, n0, &kb_begin, &kb_end)) return;  // tile not needed
  const int num_kb = kb_end > kb_begin ? kb_end - kb_begin : 0;
  const int ckb = chunk_kb(ep);
  const int nchunks = (num_kb + ckb - 1) / ckb;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), kAccWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // TMA producer.
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages) ok = mbar_wait(smem_u32(&empty_bar[s]), ((kb / kStages) - 1) & 1, err);
      if (!ok) break;
      const uint32_t fb = smem_u32(&full_bar[s]);
      mbar_expect_tx(fb, kTxBytes);
      const uint32_t base = smem_u32(smem + s * kStageBytes);
      const int k0 = (kb_begin + kb) * BK;
      const int nmaps = kStrict ? 2 : 1;
      for (int h = 0; h < nmaps; ++h) {
        const CUtensorMap* ma = h ? &map_alo : &map_a;
        const CUtensorMap* mb = h ? &map_blo : &map_b;
        const uint32_t ta = base + h * kA;
        const uint32_t tb = base + nmaps * kA + h * kB;
        if (kAmn) {
#pragma unroll
          for (int i = 0; i < BM / 32; ++i) tma_load_3d(ta + i * 2048, ma, fb, m0 + 32 * i, k0, bz);
        } else {
          tma_load_3d(ta, ma, fb, k0, m0, bz);
        }
        if (kBmn) {
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) tma_load_3d(tb + i * 2048, mb, fb, n0 + 32 * i, k0, bz);
        } else {
          tma_load_3d(tb, mb, fb, k0, n0, bz);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: chunk c accumulates into tensor-memory buffer c & 1.
    int chunk = 0, cpos = 0;  // chunk index, k-block within the chunk
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % kStages;
      const int buf = chunk & 1;
      const bool first = cpos == 0;
      const bool last = cpos == ckb - 1 || kb == num_kb - 1;
      if (first && chunk >= 2) {
        ok = mbar_wait(smem_u32(&tempty_bar[buf]), ((chunk >> 1) - 1) & 1, err);
        if (!ok) break;
        tc_fence_after();
      }
      ok = mbar_wait(smem_u32(&full_bar[s]), (kb / kStages) & 1, err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * BN);
      const uint32_t base = smem_u32(smem + s * kStageBytes);
      const int nmaps = kStrict ? 2 : 1;
      const uint32_t ta = base, talo = base + kA;
      const uint32_t tb = base + nmaps * kA, tblo = tb + kB;
#pragma unroll
      for (int j = 0; j < BK / 8; ++j) {
        const uint64_t da = operand_desc(ta, kAmn, j);
        const uint64_t db = operand_desc(tb, kBmn, j);
        const uint32_t acc = (first && j == 0) ? 0u : 1u;
        if (kStrict) {
          // Small terms first, then the leading hi*hi product.
          umma_tf32(d, operand_desc(talo, kAmn, j), db, kIdesc, acc);
          umma_tf32(d, da, operand_desc(tblo, kBmn, j), kIdesc, 1u);
          umma_tf32(d, da, db, kIdesc, 1u);
        } else {
          umma_tf32(d, da, db, kIdesc, acc);
        }
      }
      umma_commit(smem_u32(&empty_bar[s]));
      if (last) {
        umma_commit(smem_u32(&tfull_bar[buf]));
        ++chunk;
        cpos = 0;
      } else {
        ++cpos;
      }
    }
  }
  __syncwarp();

  if (warp >= 2) {
    // Accumulator warps: TMEM lane quadrant = warp % 4 (hardware rule),
    // column half = (warp - 2) / 4.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    float acc[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) acc[i] = 0.0f;
    bool have = true;
    for (int chunk = 0; chunk < nchunks; ++chunk) {
      const int buf = chunk & 1;
      have = mbar_wait(smem_u32(&tfull_bar[buf]), (chunk >> 1) & 1, err);
      if (!have) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + half * kHalf);
      // 16 columns per load keep acc[] and the loaded values within the
      // 168 registers a thread has with 10 warps per SM (3 per SMSP).
#pragma unroll
      for (int c = 0; c < kHalf; c += 16) {
        float r[16];
        tmem_ld16(taddr + c, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c + i] = acc[c + i] + r[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[buf]));
    }

    tile_epilogue<BN>(acc, have, smem, &map_c, c_tma, out, ep, M, N, m0, n0, bz, quad, half, lane, tid);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// 2-SM form (tcgen05 cta_group::2).  A cluster of two CTAs computes a
// 256 x BN tile: each CTA stages its own 128 rows of A and half (BN/2 rows or
// columns) of B; the even CTA's MMA thread issues M=256 MMAs that read both
// CTAs' shared memory and write each CTA's 128-lane accumulator.  Per SM this
// halves the B operand traffic through shared memory (TMA writes and MMA
// reads), which bounds the 1-SM tile.  Both CTAs' TMA loads complete on the
// even CTA's "full" barrier; MMA completion is multicast to both CTAs'
// "empty" / "chunk full" barriers; both CTAs' accumulator warps release a
// chunk buffer on the even CTA's "chunk empty" barrier.  No TMA load uses
// multicast.
// ---------------------------------------------------------------------------

template <int BN, bool kStrict>
struct PipeCfg2 {
  static constexpr int kA = BM * BK * 4;             // this CTA's 128 rows of A
  static constexpr int kB = (BN / 2) * BK * 4;       // this CTA's half of B
  static constexpr int kStageBytes = kStrict ? 2 * (kA + kB) : (kA + kB);
  static constexpr int kStagesRaw = (192 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of this CTA's shared variable `local` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// Arrival on a barrier of this CTA or of the peer (an address from
// map_to_rank), with the default release semantics at CTA scope.  A release
// at cluster scope measured over 1,000 cycles per arrival here, enough to
// bound a pipeline that arrives once per stage.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Loads into this CTA's shared memory; the transaction bytes complete on the
// even CTA's barrier (the peer bit of the barrier address cleared).
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar & 0xFEFFFFFFu), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same MMA over fp16 operands (both A and B fp16; fp32 accumulator).
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <bool kF16>
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  if (kF16) umma_f16_pair(d_tmem, adesc, bdesc, idesc, accumulate);
  else umma_tf32_pair(d_tmem, adesc, bdesc, idesc, accumulate);
}

// MMA completion signalled on the barrier at this offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"((uint16_t)0x3)
      : "memory");
}

template <int BN, bool kStrict, bool kAmn, bool kBmn>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsTC, 1)
    gemm_tf32_2sm_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_alo,
                         const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ CUtensorMap map_blo,
                         const __grid_constant__ CUtensorMap map_c, GemmOutput out,
                         GemmEpilogue ep, int M, int N, int K, int c_tma, int* err) {
  using Cfg = PipeCfg2<BN, kStrict>;
  static_assert(Cfg::kStages * Cfg::kStageBytes >= BM * BN * 4, "output staging must fit the stage ring");
  constexpr int kA = Cfg::kA;
  constexpr int kB = Cfg::kB;
  constexpr int kStages = Cfg::kStages;
  constexpr int kStageBytes = Cfg::kStageBytes;
  constexpr uint32_t kTxBytes = 2 * kStageBytes;  // both CTAs' loads
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr int kHalf = BN / 2;
  constexpr int kBH = BN / 2;  // rows (K-major) or columns (MN-major) of B per CTA
  constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kAmn ? 1u : 0u) << 15) |
                              ((kBmn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                              ((uint32_t)(256 >> 4) << 24);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + kStages * kStageBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* tempty_bar = bars + 2 * kStages + 2;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kStages + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  // Pair index -> (row pair, column tile) in groups of kGroupM / 2 row pairs
  // walked column by column (the 1-SM kernel's grouped raster).
  const int n_tiles = (N + BN - 1) / BN;
  const int pair_rows = (M + 255) / 256;
  constexpr int kGroupP = kGroupM / 2;
  const int pair = blockIdx.x >> 1;
  const int per_group = kGroupP * n_tiles;
  const int first_p = (pair / per_group) * kGroupP;
  const int gsize = min(pair_rows - first_p, kGroupP);
  const int in_group = pair % per_group;
  const int m0 = (first_p + in_group % gsize) * 256 + (int)rank * BM;  // this CTA's rows
  const int n0 = (in_group / gsize) * BN;
  const int nb0 = n0 + (int)rank * kBH;  // this CTA's half of B
  const int bz = blockIdx.z;
  int kb_begin = 0, kb_end = (K + BK - 1) / BK;
  // Decided on the pair's 256 rows, so both CTAs agree (and leave together,
  // before any cluster barrier, when the tile is not needed).
  if (ep.tri != 0 && causal_range(ep.tri, m0 - (int)rank * BM, 2 * BM, n0, &kb_begin, &kb_end)) return;
  const int num_kb = kb_end > kb_begin ? kb_end - kb_begin : 0;
  const int ckb = chunk_kb(ep);
  const int nchunks = (num_kb + ckb - 1) / ckb;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), 2 * kAccWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // TMA producer (both CTAs).
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages) ok = mbar_wait(smem_u32(&empty_bar[s]), ((kb / kStages) - 1) & 1, err);
      if (!ok) break;
      const uint32_t fb = smem_u32(&full_bar[s]);
      if (leader) mbar_expect_tx(fb, kTxBytes);
      const uint32_t base = smem_u32(smem + s * kStageBytes);
      const int k0 = (kb_begin + kb) * BK;
      const int nmaps = kStrict ? 2 : 1;
      for (int h = 0; h < nmaps; ++h) {
        const CUtensorMap* ma = h ? &map_alo : &map_a;
        const CUtensorMap* mb = h ? &map_blo : &map_b;
        const uint32_t ta = base + h * kA;
        const uint32_t tb = base + nmaps * kA + h * kB;
        if (kAmn) {
#pragma unroll
          for (int i = 0; i < BM / 32; ++i) tma_load_3d_pair(ta + i * 2048, ma, fb, m0 + 32 * i, k0, bz);
        } else {
          tma_load_3d_pair(ta, ma, fb, k0, m0, bz);
        }
        if (kBmn) {
#pragma unroll
          for (int i = 0; i < kBH / 32; ++i) tma_load_3d_pair(tb + i * 2048, mb, fb, nb0 + 32 * i, k0, bz);
        } else {
          tma_load_3d_pair(tb, mb, fb, k0, nb0, bz);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // MMA issuer (even CTA only): M=256 over both CTAs' operands.
    int chunk = 0, cpos = 0;  // chunk index, k-block within the chunk
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % kStages;
      const int buf = chunk & 1;
      const bool first = cpos == 0;
      const bool last = cpos == ckb - 1 || kb == num_kb - 1;
      if (first && chunk >= 2) {
        ok = mbar_wait(smem_u32(&tempty_bar[buf]), ((chunk >> 1) - 1) & 1, err);
        if (!ok) break;
        tc_fence_after();
      }
      ok = mbar_wait(smem_u32(&full_bar[s]), (kb / kStages) & 1, err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * BN);
      const uint32_t base = smem_u32(smem + s * kStageBytes);
      const int nmaps = kStrict ? 2 : 1;
      const uint32_t ta = base, talo = base + kA;
      const uint32_t tb = base + nmaps * kA, tblo = tb + kB;
#pragma unroll
      for (int j = 0; j < BK / 8; ++j) {
        const uint64_t da = operand_desc(ta, kAmn, j);
        const uint64_t db = operand_desc(tb, kBmn, j);
        const uint32_t acc = (first && j == 0) ? 0u : 1u;
        if (kStrict) {
          umma_tf32_pair(d, operand_desc(talo, kAmn, j), db, kIdesc, acc);
          umma_tf32_pair(d, da, operand_desc(tblo, kBmn, j), kIdesc, 1u);
          umma_tf32_pair(d, da, db, kIdesc, 1u);
        } else {
          umma_tf32_pair(d, da, db, kIdesc, acc);
        }
      }
      umma_commit_pair(smem_u32(&empty_bar[s]));
      if (last) {
        umma_commit_pair(smem_u32(&tfull_bar[buf]));
        ++chunk;
        cpos = 0;
      } else {
        ++cpos;
      }
    }
  }
  __syncwarp();

  if (warp >= 2) {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    float acc[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) acc[i] = 0.0f;
    bool have = true;
    for (int chunk = 0; chunk < nchunks; ++chunk) {
      const int buf = chunk & 1;
      have = mbar_wait(smem_u32(&tfull_bar[buf]), (chunk >> 1) & 1, err);
      if (!have) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * BN + half * kHalf);
#pragma unroll
      for (int c = 0; c < kHalf; c += 16) {
        float r[16];
        tmem_ld16(taddr + c, r);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c + i] = acc[c + i] + r[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[buf]), 0));
    }
    tile_epilogue<BN>(acc, have, smem, &map_c, c_tma, out, ep, M, N, m0, n0, bz, quad, half, lane, tid);
  }

  // Neither CTA may leave (releasing its shared memory and tensor memory)
  // while the pair's MMAs can still read or write them.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Persistent cluster-pair form.  One cluster of two CTAs per pair of SMs
// stays resident and walks output tiles (256 x BN, BN = 256 or 128) in the
// grouped raster order, tile t, t + clusters, ...  The TMA / MMA stage ring
// and the two tensor-memory chunk buffers keep running counters across
// tiles, so the producer loads and the MMAs of the next tile proceed while
// the accumulator warps finish the previous one: each warp writes its 32 x
// BN/2 part of the tile through two 4 KB shared-memory boxes (32 rows x 32
// columns, 128-byte swizzle) with TMA tile stores (reduce-adds for
// `accumulate`), so no tile waits for another's epilogue.  Per tile the
// protocol is the 2-SM kernel's; tiles that a causal mode skips are skipped
// by every role alike.
//
// kConvA (strict mode): the low part of A is made in shared memory instead
// of being loaded.  Each CTA's A tile lands on a barrier of its own
// ("A full"); two converter warps per CTA write lo = tf32_lo(a) beside
// it, in the same swizzled positions, and arrive on the even CTA's
// "converted" barrier, which the MMA issuer waits for besides "full".  The
// A stream read from HBM halves and no split pass over A runs; the two
// converter warps keep up with the tensor core (about 560 cycles per stage
// against 750 of MMAs for 256 x 256 tiles).
//
// kStackB (strict, BN = 128, i.e. N <= 128): B's high and low parts are
// stacked along N, so each k-slice takes two MMAs instead of three: a_hi x
// [b_hi | b_lo] (one 256-wide instruction into 256 accumulator columns) and
// a_lo x b_hi (128 wide, into the first 128).  In a pair MMA each CTA
// supplies half of B's columns at the same shared-memory offset, so the
// even CTA stages b_hi (all 128 columns) and the odd CTA b_lo in the wide
// region, and each stages its half of b_hi in the narrow one.  The
// accumulator warps add column c and c + 128 of each chunk.  A 128-wide
// instruction costs nearly as much to issue as a 256-wide one, and the
// N <= 128 GEMMs (attention with head dim 128) are bound by that.
//
// kF16 (split-fp16 strict mode, both operands K-major): the four maps
// address the packed fp16 halves (a_hi, a_lo, b_hi, b_lo); a stage holds
// the same 64-byte rows, now 32 elements of K, and each 32-byte slice is one
// kind::f16 MMA of K = 16.  Chunks of tensor-memory accumulation cover half
// as many k-blocks, i.e. the same elements of K.  The accumulator warps
// multiply each sum by row_factor[m] * col_factor[n] (a power of two) before
// the epilogue.
// ---------------------------------------------------------------------------

template <bool kConvA>
constexpr int pp_threads() {
  return kThreadsTC + (kConvA ? 64 : 0);
}

template <int BN, bool kStrict, bool kStackB = false>
struct PipeCfgP {
  static constexpr int kA = BM * BK * 4;        // this CTA's 128 rows of A
  static constexpr int kB = (BN / 2) * BK * 4;  // this CTA's half of B
  // kStackB: a 2*BN-wide stacked B region (2 kB) and a BN-wide one (kB).
  static constexpr int kStageBytes = kStackB ? 2 * kA + 3 * kB : kStrict ? 2 * (kA + kB) : (kA + kB);
  static constexpr int kEpiBytes = kAccWarps * 2 * 4096;  // two 32x32 boxes per accumulator warp
  static constexpr int kStagesRaw = (160 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kSmem = kStages * kStageBytes + kEpiBytes + 1024 + 512;
};

// Tile t of the persistent schedule: batch item, this CTA's first row, the
// tile's first column; false if the causal mode skips it.  kb range in
// [*kb_begin, *kb_end).
template <int BN>
__device__ __forceinline__ bool pp_tile(int t, int tiles_per_batch, int pair_rows, int n_tiles, int rank,
                                        int tri, int K, int* bz, int* m0, int* n0, int* kb_begin, int* kb_end,
                                        int splits = 1, int total_tiles = 0, int* ks = nullptr, int bk = BK) {
  constexpr int kGroupP = kGroupM / 2;
  // Split-K: tile t covers part t / total_tiles of the K range of output
  // tile t % total_tiles.
  int part = 0;
  if (splits > 1) {
    part = t / total_tiles;
    t -= part * total_tiles;
  }
  if (ks) *ks = part;
  *bz = t / tiles_per_batch;
  const int pair = t - *bz * tiles_per_batch;
  const int per_group = kGroupP * n_tiles;
  const int first_p = (pair / per_group) * kGroupP;
  const int gsize = min(pair_rows - first_p, kGroupP);
  const int in_group = pair % per_group;
  const int pr0 = (first_p + in_group % gsize) * 256;
  *n0 = (in_group / gsize) * BN;
  *m0 = pr0 + rank * BM;
  *kb_begin = 0;
  *kb_end = (K + bk - 1) / bk;
  if (tri != 0 && causal_range(tri, pr0, 2 * BM, *n0, kb_begin, kb_end)) return false;
  if (*kb_end < *kb_begin) *kb_end = *kb_begin;
  if (splits > 1) {
    const int per = (*kb_end - *kb_begin + splits - 1) / splits;
    const int b = *kb_begin + part * per;
    const int e = min(*kb_end, b + per);
    *kb_begin = b;
    *kb_end = e > b ? e : b;
  }
  return true;
}

template <int BN, bool kStrict, bool kAmn, bool kBmn, bool kConvA, bool kStackB, int kEpi, bool kF16 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pp_threads<kConvA>(), 1)
    gemm_tf32_pp_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_alo,
                        const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_blo,
                        const __grid_constant__ CUtensorMap map_c32,
                        const __grid_constant__ CUtensorMap map_y, GemmEpilogue ep, int M, int N, int K,
                        int batch, int splits, int* err) {
  // kEpi != 0: map_y addresses a second tensor in C's geometry; each
  // accumulator warp loads its boxes of it with TMA into its epilogue boxes
  // and rewrites them in place before storing: kEpi 1, the probabilities p,
  // as dS = (p * (1 - p)) * dP (0 above the diagonal); kEpi 2, a residual r,
  // as r + result.
  // splits > 1: map_c32 addresses the split-K workspace ([splits * batch][M]
  // [N] raw sums); alpha, bias, relu and accumulate are left to the
  // reduction that sums the parts.
  using Cfg = PipeCfgP<BN, kStrict, kStackB>;
  constexpr int kA = Cfg::kA;
  constexpr int kB = Cfg::kB;
  constexpr int kStages = Cfg::kStages;
  constexpr int kStageBytes = Cfg::kStageBytes;
  static_assert(!kConvA || kStrict, "A's low part is only used in strict mode");
  static_assert(!kStackB || (kStrict && BN == 128), "stacked B is the strict N <= 128 form");
  static_assert(!kF16 || (kStrict && !kConvA && !kStackB && !kAmn && !kBmn && kEpi != 1),
                "the split-fp16 form reads four K-major packed halves");
  constexpr int kBK = kF16 ? 2 * BK : BK;  // elements of K per stage (64-byte rows)
  static_assert(((kConvA ? 4 : 2) * kStages + 4 + 2 * kAccWarps) * 8 + 4 <= 512, "barriers exceed their reserve");
  static_assert(kA % (16 * 64) == 0, "converter warps cover the A tile in float4 rounds");
  // Both CTAs' loads on the even CTA's "full" barrier (with kConvA: B only).
  constexpr uint32_t kATx = kConvA ? 0 : (kStrict ? 2 * kA : kA);
  constexpr uint32_t kBTx = kStackB ? 3 * kB : (kStrict ? 2 * kB : kB);
  constexpr uint32_t kTxBytes = 2 * (kATx + kBTx);
  constexpr int kBufCols = kStackB ? 2 * BN : BN;  // tensor-memory columns of one chunk buffer
  constexpr uint32_t kTmemCols = 2 * kBufCols;
  constexpr int kHalf = BN / 2;  // columns per accumulator warp
  constexpr int kBH = BN / 2;    // rows (K-major) or columns (MN-major) of B per CTA
  // Operand formats: tf32 = 2; f16 = 0 (kind::f16); accumulator f32.
  constexpr uint32_t kFmt = kF16 ? 0u : 2u;
  constexpr uint32_t kIdesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((kAmn ? 1u : 0u) << 15) |
                              ((kBmn ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
                              ((uint32_t)(256 >> 4) << 24);
  constexpr uint32_t kIdescWide = (kIdesc & ~(0x3Fu << 17)) | ((uint32_t)((2 * BN) >> 3) << 17);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* epi = smem + kStages * kStageBytes;  // 1 KiB aligned: kStageBytes is a multiple of 1 KiB
  uint64_t* bars = (uint64_t*)(epi + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* tempty_bar = bars + 2 * kStages + 2;
  uint64_t* afull_bar = bars + 2 * kStages + 4;  // kConvA: this CTA's A tile landed
  uint64_t* conv_bar = bars + 3 * kStages + 4;   // kConvA: both CTAs' low parts written
  uint64_t* ybar = bars + (kConvA ? 4 * kStages + 4 : 2 * kStages + 4);  // kEpi: two per accumulator warp
  uint32_t* tmem_slot = (uint32_t*)(ybar + 2 * kAccWarps);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = (int)cluster_ctarank();
  const bool leader = rank == 0;
  const int n_tiles = (N + BN - 1) / BN;
  const int pair_rows = (M + 255) / 256;
  const int tiles_per_batch = n_tiles * pair_rows;
  const int out_tiles = tiles_per_batch * batch;
  const int total = out_tiles * splits;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), 2 * kAccWarps);
    }
    if (kConvA) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(smem_u32(&afull_bar[s]), 1);
        mbar_init(smem_u32(&conv_bar[s]), 4);  // two converter warps in each CTA
      }
    }
    if (kEpi != 0)
      for (int b = 0; b < 2 * kAccWarps; ++b) mbar_init(smem_u32(&ybar[b]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // TMA producer (both CTAs), stage ring counter across tiles.
    uint32_t it = 0;
    for (int t = cluster; t < total && ok; t += clusters) {
      int bz, m0, n0, kb0, kb1, ks;
      if (!pp_tile<BN>(t, tiles_per_batch, pair_rows, n_tiles, rank, ep.tri, K, &bz, &m0, &n0, &kb0, &kb1, splits, out_tiles, &ks, kBK))
        continue;
      const int nb0 = n0 + rank * kBH;
      for (int kb = kb0; kb < kb1 && ok; ++kb, ++it) {
        const int s = (int)(it % kStages);
        if (it >= (uint32_t)kStages) ok = mbar_wait(smem_u32(&empty_bar[s]), ((it / kStages) - 1) & 1, err);
        if (!ok) break;
        const uint32_t fb = smem_u32(&full_bar[s]);
        if (leader) mbar_expect_tx(fb, kTxBytes);
        const uint32_t afb = smem_u32(&afull_bar[s]);
        if (kConvA) mbar_expect_tx(afb, kA);
        const uint32_t base = smem_u32(smem + s * kStageBytes);
        const int k0 = kb * kBK;
        const int nmaps = kStrict ? 2 : 1;
        for (int h = 0; h < nmaps; ++h) {
          const CUtensorMap* ma = h ? &map_alo : &map_a;
          const CUtensorMap* mb = h ? &map_blo : &map_b;
          const uint32_t ta = base + h * kA;
          const uint32_t tb = base + nmaps * kA + h * kB;
          if (kConvA) {
            // The high part only, completing on this CTA's own barrier.
            if (h == 0) {
              if (kAmn) {
#pragma unroll
                for (int i = 0; i < BM / 32; ++i) tma_load_3d(ta + i * 2048, ma, afb, m0 + 32 * i, k0, bz);
              } else {
                tma_load_3d(ta, ma, afb, k0, m0, bz);
              }
            }
          } else if (kAmn) {
#pragma unroll
            for (int i = 0; i < BM / 32; ++i) tma_load_3d_pair(ta + i * 2048, ma, fb, m0 + 32 * i, k0, bz);
          } else {
            tma_load_3d_pair(ta, ma, fb, k0, m0, bz);
          }
          if (kStackB) continue;  // B below
          if (kBmn) {
#pragma unroll
            for (int i = 0; i < kBH / 32; ++i) tma_load_3d_pair(tb + i * 2048, mb, fb, nb0 + 32 * i, k0, bz);
          } else {
            tma_load_3d_pair(tb, mb, fb, k0, nb0, bz);
          }
        }
        if (kStackB) {
          // Wide region: all BN columns of b_hi (even CTA) or b_lo (odd CTA);
          // narrow region: this CTA's half of b_hi.
          const CUtensorMap* mw = rank ? &map_blo : &map_b;
          const uint32_t tw = base + 2 * kA, tn = tw + 2 * kB;
          if (kBmn) {
#pragma unroll
            for (int i = 0; i < BN / 32; ++i) tma_load_3d_pair(tw + i * 2048, mw, fb, n0 + 32 * i, k0, bz);
#pragma unroll
            for (int i = 0; i < kBH / 32; ++i) tma_load_3d_pair(tn + i * 2048, &map_b, fb, nb0 + 32 * i, k0, bz);
          } else {
            tma_load_3d_pair(tw, mw, fb, k0, n0, bz);
            tma_load_3d_pair(tw + kB, mw, fb, k0, n0 + kBH, bz);
            tma_load_3d_pair(tn, &map_b, fb, k0, nb0, bz);
          }
        }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // MMA issuer (even CTA): stage counter and chunk counter across tiles.
    const int ckb = kF16 ? (chunk_kb(ep) + 1) / 2 : chunk_kb(ep);
    uint32_t it = 0, gch = 0;  // stages and chunks issued so far (all tiles)
    for (int t = cluster; t < total && ok; t += clusters) {
      int bz, m0, n0, kb0, kb1, ks;
      if (!pp_tile<BN>(t, tiles_per_batch, pair_rows, n_tiles, 0, ep.tri, K, &bz, &m0, &n0, &kb0, &kb1, splits, out_tiles, &ks, kBK))
        continue;
      const int nkb = kb1 - kb0;
      int cpos = 0;  // k-block within the chunk
      for (int j = 0; j < nkb && ok; ++j, ++it) {
        const int s = (int)(it % kStages);
        const int buf = (int)(gch & 1);
        const bool first = cpos == 0;
        const bool last = cpos == ckb - 1 || j == nkb - 1;
        if (first && gch >= 2) {
          ok = mbar_wait(smem_u32(&tempty_bar[buf]), ((gch >> 1) - 1) & 1, err);
          if (!ok) break;
          tc_fence_after();
        }
        ok = mbar_wait(smem_u32(&full_bar[s]), (it / kStages) & 1, err);
        if (ok && kConvA) ok = mbar_wait(smem_u32(&conv_bar[s]), (it / kStages) & 1, err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * kBufCols);
        const uint32_t base = smem_u32(smem + s * kStageBytes);
        const int nmaps = kStrict ? 2 : 1;
        const uint32_t ta = base, talo = base + kA;
        const uint32_t tb = base + nmaps * kA, tblo = tb + kB;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t da = operand_desc(ta, kAmn, kk);
          const uint64_t db = operand_desc(tb, kBmn, kk);
          const uint32_t acc = (first && kk == 0) ? 0u : 1u;
          if (kStackB) {
            // tb: the wide region ([b_hi | b_lo] across the pair), tb + 2 kB:
            // the narrow one (b_hi).
            umma_tf32_pair(d, da, db, kIdescWide, acc);
            umma_tf32_pair(d, operand_desc(talo, kAmn, kk), operand_desc(tb + 2 * kB, kBmn, kk), kIdesc, 1u);
          } else if (kStrict) {
            umma_pair<kF16>(d, operand_desc(talo, kAmn, kk), db, kIdesc, acc);
            umma_pair<kF16>(d, da, operand_desc(tblo, kBmn, kk), kIdesc, 1u);
            umma_pair<kF16>(d, da, db, kIdesc, 1u);
          } else {
            umma_tf32_pair(d, da, db, kIdesc, acc);
          }
        }
        umma_commit_pair(smem_u32(&empty_bar[s]));
        if (last) {
          umma_commit_pair(smem_u32(&tfull_bar[buf]));
          ++gch;
          cpos = 0;
        } else {
          ++cpos;
        }
      }
    }
  } else if (kConvA && warp >= 2 + kAccWarps) {
    // Converter warps (both CTAs): the low part of each landed A tile,
    // elementwise, so it keeps the tile's swizzled layout at offset kA.
    const int ct = tid - 32 * (2 + kAccWarps);  // 0 .. 63
    uint32_t it = 0;
    for (int t = cluster; t < total && ok; t += clusters) {
      int bz, m0, n0, kb0, kb1, ks;
      if (!pp_tile<BN>(t, tiles_per_batch, pair_rows, n_tiles, rank, ep.tri, K, &bz, &m0, &n0, &kb0, &kb1, splits, out_tiles, &ks, kBK))
        continue;
      for (int kb = kb0; kb < kb1 && ok; ++kb, ++it) {
        const int s = (int)(it % kStages);
        ok = mbar_wait(smem_u32(&afull_bar[s]), (it / kStages) & 1, err);
        if (!ok) break;
        const uint32_t hi = smem_u32(smem + s * kStageBytes);
        constexpr int kPer = kA / (16 * 64);  // float4 per converter thread
        float4 v[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) v[i] = ld_shared_f4(hi + (uint32_t)(ct + 64 * i) * 16u);
#pragma unroll
        for (int i = 0; i < kPer; ++i)
          st_shared_f4(hi + (uint32_t)kA + (uint32_t)(ct + 64 * i) * 16u,
                       tf32_lo(v[i].x),
                       tf32_lo(v[i].y),
                       tf32_lo(v[i].z),
                       tf32_lo(v[i].w));
        // Generic-proxy writes made visible to the tensor core's reads.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&conv_bar[s]), 0));
      }
    }
  } else if (warp >= 2 && warp < 2 + kAccWarps) {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const uint32_t ebox0 = smem_u32(epi) + (uint32_t)(warp - 2) * 8192u;
    const bool smx = kEpi != 0 && splits == 1;  // boxes of map_y are loaded
    constexpr int kBoxes = kHalf / 32;  // output boxes per warp per tile
    const uint32_t ybar0 = smem_u32(&ybar[2 * (warp - 2)]);
    uint32_t yph = 0;   // phase bit of each of this warp's two probability barriers
    int y_pending = 0;  // probability boxes loading and not yet waited for
    uint32_t ch = 0;
    bool have = true;
    for (int t = cluster; t < total && have; t += clusters) {
      int bz, m0, n0, kb0, kb1, ks;
      if (!pp_tile<BN>(t, tiles_per_batch, pair_rows, n_tiles, rank, ep.tri, K, &bz, &m0, &n0, &kb0, &kb1, splits, out_tiles, &ks, kBK))
        continue;
      if (smx) {
        // The tile's first two probability boxes load while the tensor core
        // finishes the tile (once this warp's earlier stores have read the
        // boxes out).
        if (lane == 0) {
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
#pragma unroll
          for (int b = 0; b < 2 && b < kBoxes; ++b) {
            mbar_expect_tx(ybar0 + 8u * b, 4096u);
            tma_load_3d(ebox0 + (uint32_t)b * 4096u, &map_y, ybar0 + 8u * b, n0 + half * kHalf + 32 * b,
                        m0 + quad * 32, bz);
          }
        }
        y_pending += kBoxes < 2 ? kBoxes : 2;
      }
      const int ckb = kF16 ? (chunk_kb(ep) + 1) / 2 : chunk_kb(ep);
      const int nch = (kb1 - kb0 + ckb - 1) / ckb;
      float acc[kHalf];
#pragma unroll
      for (int i = 0; i < kHalf; ++i) acc[i] = 0.0f;
      for (int c = 0; c < nch; ++c) {
        const uint32_t gch = ch + (uint32_t)c;
        const int buf = (int)(gch & 1);
        have = mbar_wait(smem_u32(&tfull_bar[buf]), (gch >> 1) & 1, err);
        if (!have) break;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(buf * kBufCols + half * kHalf);
#pragma unroll
        for (int cc = 0; cc < kHalf; cc += 16) {
          float r[16];
          tmem_ld16(taddr + cc, r);
          if (kStackB) {
            // Column c + BN holds a_hi . b_lo of output column c.
            float r2[16];
            tmem_ld16(taddr + BN + cc, r2);
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = r[i] + r2[i];
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[cc + i] = acc[cc + i] + r[i];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[buf]), 0));
      }
      ch += (uint32_t)nch;
      if (!have) break;
      // Epilogue of this warp's 32 rows x kHalf columns.
      const int col0 = n0 + half * kHalf;
      // kF16: the operands' row scales are undone (exact powers of two in
      // [2^-126, 2^126]), then alpha, bias and relu applied, four columns at
      // a time as the boxes are written, which keeps the register pressure
      // at the accumulator's kHalf values.
      const int frow = m0 + quad * 32 + lane;
      const float fr = kF16 ? (frow < M ? ep.row_factor[frow] : 0.0f) : 1.0f;
      auto value4 = [&](int i) -> float4 {
        float4 v = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
        if (kF16) {
          const int c = col0 + i;  // a multiple of 4: col_factor is 16-byte aligned
          float4 f;
          if (c + 3 < N) {
            f = __ldg((const float4*)(ep.col_factor + c));
          } else {
            f.x = c < N ? ep.col_factor[c] : 0.0f;
            f.y = c + 1 < N ? ep.col_factor[c + 1] : 0.0f;
            f.z = c + 2 < N ? ep.col_factor[c + 2] : 0.0f;
            f.w = 0.0f;
          }
          v.x = v.x * (fr * f.x);
          v.y = v.y * (fr * f.y);
          v.z = v.z * (fr * f.z);
          v.w = v.w * (fr * f.w);
          if (splits == 1) {
            float* e = &v.x;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float r = e[q] * ep.alpha;
              if (ep.bias != nullptr && c + q < N) r = r + ep.bias[c + q];
              if (ep.relu) r = fmaxf(r, 0.0f);
              e[q] = r;
            }
          }
        }
        return v;
      };
      if (splits == 1 && !kF16) {
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          float r = acc[i] * ep.alpha;
          if (ep.bias != nullptr && col0 + i < N) r = r + ep.bias[col0 + i];
          if (ep.relu) r = fmaxf(r, 0.0f);
          acc[i] = r;
        }
      }
      const int zc = splits == 1 ? bz : ks * batch + bz;  // output (or workspace) batch index
      const int red = splits == 1 ? ep.accumulate : 0;
#pragma unroll
      for (int b = 0; b < kBoxes; ++b) {
        const uint32_t box = ebox0 + (uint32_t)(b & 1) * 4096u;
        if (smx) {
          // dS in place of the probability box (the output's swizzled
          // positions), 0 where the column exceeds the row.
          have = mbar_wait(ybar0 + 8u * (b & 1), (yph >> (b & 1)) & 1u, err);
          if (!have) break;
          yph ^= 1u << (b & 1);
          --y_pending;
          const int row = m0 + quad * 32 + lane;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t a = box + (uint32_t)lane * 128u + (uint32_t)((j ^ (lane & 7)) << 4);
            const float4 p = ld_shared_f4(a);
            const int c = col0 + 32 * b + 4 * j;
            const float4 v4 = value4(b * 32 + 4 * j);
            const float* v = &v4.x;
            if (kEpi == 1)
              st_shared_f4(a, c > row ? 0.0f : (p.x * (1.0f - p.x)) * v[0],
                           c + 1 > row ? 0.0f : (p.y * (1.0f - p.y)) * v[1],
                           c + 2 > row ? 0.0f : (p.z * (1.0f - p.z)) * v[2],
                           c + 3 > row ? 0.0f : (p.w * (1.0f - p.w)) * v[3]);
            else
              st_shared_f4(a, p.x + v[0], p.y + v[1], p.z + v[2], p.w + v[3]);
          }
        } else {
          // The box is reused two stores later: wait until at most one store
          // is still reading this warp's boxes.
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 v4 = value4(b * 32 + 4 * j);
            st_shared_f4(box + (uint32_t)lane * 128u + (uint32_t)((j ^ (lane & 7)) << 4), v4.x, v4.y, v4.z, v4.w);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if (col0 + 32 * b < N) tma_store_3d(&map_c32, box, col0 + 32 * b, m0 + quad * 32, zc, red);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          if (smx && b + 2 < kBoxes) {
            // This box's next probabilities, once the store has read it.
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            mbar_expect_tx(ybar0 + 8u * (b & 1), 4096u);
            tma_load_3d(box, &map_y, ybar0 + 8u * (b & 1), col0 + 32 * (b + 2), m0 + quad * 32, bz);
          }
        }
        if (smx && b + 2 < kBoxes) ++y_pending;
      }
    }
    // After a timed-out wait, probability loads may still be in flight:
    // give each a bounded wait before the shared memory is released.
    for (int b = 0; b < 2 && y_pending > 0; ++b)
      if (mbar_wait(ybar0 + 8u * b, (yph >> b) & 1u, err)) --y_pending;
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }
  __syncwarp();

  // Neither CTA may leave (releasing its shared memory and tensor memory)
  // while the pair's MMAs can still read or write them.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Split-K reduction: C (+)= epilogue(sum over parts of ws[part]), parts
// added in order 0, 1, ... (deterministic).  ws is [splits * batch][M][ldw].
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int batch, int M, int N,
                                     int64_t ldw, GemmOutput out, GemmEpilogue ep) {
  const int64_t per_batch = (int64_t)M * N;
  const int64_t total = per_batch * batch;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(e / per_batch);
    const int64_t rem = e - (int64_t)b * per_batch;
    const int row = (int)(rem / N), col = (int)(rem % N);
    float v = 0.0f;
    for (int p = 0; p < splits; ++p) v = v + ws[((int64_t)(p * batch + b) * M + row) * ldw + col];
    float r = v * ep.alpha;
    if (ep.bias != nullptr) r = r + ep.bias[col];
    if (ep.relu) r = fmaxf(r, 0.0f);
    float* dst = out.ptr + (int64_t)b * out.batch_stride + (int64_t)row * out.ld + col;
    *dst = ep.accumulate ? *dst + r : r;
  }
}

// ---------------------------------------------------------------------------
// Split-fp16 packing (kGemmStrict16 operands; layout in gemm_pack16_elems's
// declaration).
// ---------------------------------------------------------------------------

// 2^e as a float, e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }

// The row scale exponent for a row whose largest magnitude is mx: the e
// with mx 2^e in [2^14, 2^15), from mx's exponent field, clamped to
// [-63, 63] (so row and column factors multiply to a normal float); 0 when
// mx is zero or infinite (the row's products are then 0, inf or NaN
// whatever the scale).
__device__ __forceinline__ int pack16_exponent(float mx) {
  const int field = (int)((__float_as_uint(mx) >> 23) & 0xFFu);
  if (mx == 0.0f || field == 0xFF) return 0;
  const int e = 14 - (field == 0 ? -127 : field - 127);
  return e < -63 ? -63 : (e > 63 ? 63 : e);
}

__device__ __forceinline__ void pack16_one(float x, float up, __half* hi, __half* lo) {
  const float xs = x * up;  // exact: a power-of-two scale
  const __half h = __float2half_rn(xs);
  *hi = h;
  *lo = __float2half_rn(xs - __half2float(h));  // xs - h is exact in fp32
}

__device__ __forceinline__ float block_max256(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  v = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) v = fmaxf(v, red[w]);
  return v;
}

// K-contiguous operand x [R][ld]: one 256-thread block per row; the row is
// read twice (its maximum, then the halves; the second read hits cache).
__global__ void __launch_bounds__(256) pack16_rows_kernel(const float* __restrict__ x, int64_t ld, int K, int Kp,
                                                          __half* __restrict__ hi, __half* __restrict__ lo,
                                                          float* __restrict__ factor) {
  __shared__ float red[8];
  const int r = blockIdx.x;
  const float* row = x + (int64_t)r * ld;
  const bool vec = ((ld & 3) == 0) && ((((uintptr_t)x) & 15) == 0);
  const int K4 = vec ? K >> 2 : 0;
  if (vec && K4 <= 256 * 8) {
    // Rows up to 8192 wide stay in registers: one read, loads issued together.
    float4 v[8];
    float m = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = threadIdx.x + 256 * u;
      v[u] = i < K4 ? __ldg((const float4*)row + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) m = fmaxf(m, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
    for (int i = 4 * K4 + threadIdx.x; i < K; i += 256) m = fmaxf(m, fabsf(row[i]));
    m = block_max256(m, red);
    const int e = pack16_exponent(m);
    const float up = pow2f(e);
    if (threadIdx.x == 0) factor[r] = pow2f(-e);
    __half* h = hi + (int64_t)r * Kp;
    __half* l = lo + (int64_t)r * Kp;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = threadIdx.x + 256 * u;
      if (i >= K4) break;
      __align__(8) __half hv[4], lv[4];
      pack16_one(v[u].x, up, &hv[0], &lv[0]);
      pack16_one(v[u].y, up, &hv[1], &lv[1]);
      pack16_one(v[u].z, up, &hv[2], &lv[2]);
      pack16_one(v[u].w, up, &hv[3], &lv[3]);
      *(uint2*)(h + 4 * i) = *(const uint2*)hv;
      *(uint2*)(l + 4 * i) = *(const uint2*)lv;
    }
    for (int i = 4 * K4 + threadIdx.x; i < K; i += 256) pack16_one(row[i], up, h + i, l + i);
    return;
  }
  float mx = 0.0f;
  for (int i = threadIdx.x; i < K4; i += 256) {
    const float4 v = __ldg((const float4*)row + i);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  for (int i = 4 * K4 + threadIdx.x; i < K; i += 256) mx = fmaxf(mx, fabsf(row[i]));
  mx = block_max256(mx, red);
  const int e = pack16_exponent(mx);
  const float up = pow2f(e);
  if (threadIdx.x == 0) factor[r] = pow2f(-e);
  __half* h = hi + (int64_t)r * Kp;
  __half* l = lo + (int64_t)r * Kp;
  for (int i = threadIdx.x; i < K4; i += 256) {
    const float4 v = __ldg((const float4*)row + i);
    __align__(8) __half hv[4], lv[4];
    pack16_one(v.x, up, &hv[0], &lv[0]);
    pack16_one(v.y, up, &hv[1], &lv[1]);
    pack16_one(v.z, up, &hv[2], &lv[2]);
    pack16_one(v.w, up, &hv[3], &lv[3]);
    *(uint2*)(h + 4 * i) = *(const uint2*)hv;  // Kp % 8 == 0: 8-byte aligned
    *(uint2*)(l + 4 * i) = *(const uint2*)lv;
  }
  for (int i = 4 * K4 + threadIdx.x; i < K; i += 256) pack16_one(row[i], up, h + i, l + i);
}

// R-contiguous operand x [K][ld], pass 1: each column's largest magnitude,
// as float bits (non-negative floats order like their bits), atomically
// maxed into colmax[R] (zeroed before).  Block: 256 columns (64 threads x
// float4) x 4 row lanes over a slab of 64 rows, 16 independent loads per
// thread (scalar loads where ld or x breaks float4 alignment).
__global__ void __launch_bounds__(256) pack16_colmax_kernel(const float* __restrict__ x, int64_t ld, int R, int K,
                                                            uint32_t* __restrict__ colmax) {
  __shared__ float4 part[4][64];
  const int c4 = threadIdx.x & 63, lane = threadIdx.x >> 6;
  const int c = blockIdx.x * 256 + 4 * c4;
  const int k0 = blockIdx.y * 64;
  float4 m = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const bool full = c + 3 < R && (ld & 3) == 0 && (((uintptr_t)x) & 15) == 0;
  if (full && k0 + 64 <= K) {
    // A whole slab of aligned float4: the 16 loads are independent and issued together.
    float4 v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __ldg((const float4*)(x + (int64_t)(k0 + lane + 4 * i) * ld + c));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      m.x = fmaxf(m.x, fabsf(v[i].x));
      m.y = fmaxf(m.y, fabsf(v[i].y));
      m.z = fmaxf(m.z, fabsf(v[i].z));
      m.w = fmaxf(m.w, fabsf(v[i].w));
    }
  } else if (c < R) {
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int k = k0 + lane + 4 * i;
      if (k >= K) break;
      const float* p = x + (int64_t)k * ld + c;
      float4 v;
      if (full) {
        v = __ldg((const float4*)p);
      } else {
        v.x = __ldg(p);
        v.y = c + 1 < R ? __ldg(p + 1) : 0.0f;
        v.z = c + 2 < R ? __ldg(p + 2) : 0.0f;
        v.w = c + 3 < R ? __ldg(p + 3) : 0.0f;
      }
      m.x = fmaxf(m.x, fabsf(v.x));
      m.y = fmaxf(m.y, fabsf(v.y));
      m.z = fmaxf(m.z, fabsf(v.z));
      m.w = fmaxf(m.w, fabsf(v.w));
    }
  }
  part[lane][c4] = m;
  __syncthreads();
  if (threadIdx.x < 64 && c < R) {
    float4 r = part[0][c4];
#pragma unroll
    for (int l = 1; l < 4; ++l) {
      const float4 q = part[l][c4];
      r.x = fmaxf(r.x, q.x);
      r.y = fmaxf(r.y, q.y);
      r.z = fmaxf(r.z, q.z);
      r.w = fmaxf(r.w, q.w);
    }
    atomicMax(&colmax[c], __float_as_uint(r.x));
    if (c + 1 < R) atomicMax(&colmax[c + 1], __float_as_uint(r.y));
    if (c + 2 < R) atomicMax(&colmax[c + 2], __float_as_uint(r.z));
    if (c + 3 < R) atomicMax(&colmax[c + 3], __float_as_uint(r.w));
  }
}

// Pass 2: a 64 (K) x 64 (columns) tile read with float4 loads into shared
// memory, written as 64 K-major output rows of 64 halves: four threads per
// output row, 16 elements of K each, so a warp writes 8 rows' 128-byte hi
// and lo runs.  Blocks of the first K tile also write the factors.
__global__ void __launch_bounds__(256) pack16_cols_kernel(const float* __restrict__ x, int64_t ld, int R, int K, int Kp,
                                                          const uint32_t* __restrict__ colmax, __half* __restrict__ hi,
                                                          __half* __restrict__ lo, float* __restrict__ factor) {
  __shared__ float tile[64][65];
  const int c0 = blockIdx.x * 64, k0 = blockIdx.y * 64;
  {
    const int c4 = threadIdx.x & 15, r0 = threadIdx.x >> 4;
    const int c = c0 + 4 * c4;
    const bool aligned = (ld & 3) == 0 && (((uintptr_t)x) & 15) == 0;
    if (aligned && k0 + 64 <= K && c0 + 64 <= R) {
      // A whole aligned tile: four independent, unguarded float4 loads.
      float4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __ldg((const float4*)(x + (int64_t)(k0 + r0 + 16 * i) * ld + c));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kr = r0 + 16 * i;
        tile[kr][4 * c4] = v[i].x;
        tile[kr][4 * c4 + 1] = v[i].y;
        tile[kr][4 * c4 + 2] = v[i].z;
        tile[kr][4 * c4 + 3] = v[i].w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kr = r0 + 16 * i, k = k0 + kr;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (k < K && c < R) {
          const float* p = x + (int64_t)k * ld + c;
          if (aligned && c + 3 < R) {
            v = __ldg((const float4*)p);
          } else {
            v.x = __ldg(p);
            v.y = c + 1 < R ? __ldg(p + 1) : 0.0f;
            v.z = c + 2 < R ? __ldg(p + 2) : 0.0f;
            v.w = c + 3 < R ? __ldg(p + 3) : 0.0f;
          }
        }
        tile[kr][4 * c4] = v.x;
        tile[kr][4 * c4 + 1] = v.y;
        tile[kr][4 * c4 + 2] = v.z;
        tile[kr][4 * c4 + 3] = v.w;
      }
    }
  }
  __syncthreads();
  const int cc = threadIdx.x >> 2, j = threadIdx.x & 3;  // output row c0 + cc, K elements 16 j .. 16 j + 15
  const int c = c0 + cc;
  if (c >= R) return;
  const int e = pack16_exponent(__uint_as_float(colmax[c]));
  const float up = pow2f(e);
  if (blockIdx.y == 0 && j == 0) factor[c] = pow2f(-e);
  __align__(16) __half hv[16], lv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) pack16_one(tile[16 * j + i][cc], up, &hv[i], &lv[i]);
  __half* h = hi + (int64_t)c * Kp + k0 + 16 * j;
  __half* l = lo + (int64_t)c * Kp + k0 + 16 * j;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    if (k0 + 16 * j + 8 * g >= Kp) break;  // Kp % 8 == 0: whole 16-byte groups
    *(uint4*)(h + 8 * g) = *(const uint4*)(hv + 8 * g);
    *(uint4*)(l + 8 * g) = *(const uint4*)(lv + 8 * g);
  }
}

// The same reduction four columns at a time: one block row of threads per
// output row (blockIdx.y = batch item * M + row), float4 loads and stores,
// no per-element index division; the parts are added in the same order and
// the epilogue applied per element as above (bit-identical results).  Needs
// N, ldw, C's pitch and batch stride multiples of 4, C and bias 16-byte
// aligned, batch * M <= 65535.
__global__ void splitk_reduce4_kernel(const float* __restrict__ ws, int splits, int M, int N, int64_t ldw,
                                      GemmOutput out, GemmEpilogue ep) {
  const int bm = blockIdx.y;  // batch item * M + row
  const int b = bm / M, row = bm - b * M;
  const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= N) return;
  const int batch = gridDim.y / M;
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int p = 0; p < splits; ++p) {
    const float4 w = __ldg((const float4*)(ws + ((int64_t)(p * batch + b) * M + row) * ldw + c));
    v.x = v.x + w.x;
    v.y = v.y + w.y;
    v.z = v.z + w.z;
    v.w = v.w + w.w;
  }
  float* e = &v.x;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float r = e[q] * ep.alpha;
    if (ep.bias != nullptr) r = r + ep.bias[c + q];
    if (ep.relu) r = fmaxf(r, 0.0f);
    e[q] = r;
  }
  float4* dst = (float4*)(out.ptr + (int64_t)b * out.batch_stride + (int64_t)row * out.ld + c);
  if (ep.accumulate) {
    const float4 o = *dst;
    v = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
  }
  *dst = v;
}

// Launches the split-K reduction (the float4 form where its layout rules hold).
void launch_splitk_reduce(const float* ws, int splits, int batch, int M, int N, int64_t ldw, const GemmOutput& C,
                          const GemmEpilogue& ep, cudaStream_t st) {
  const bool vec = N % 4 == 0 && ldw % 4 == 0 && C.ld % 4 == 0 && (batch == 1 || C.batch_stride % 4 == 0) &&
                   (((uintptr_t)C.ptr) & 15) == 0 && (ep.bias == nullptr || (((uintptr_t)ep.bias) & 15) == 0) &&
                   (int64_t)batch * M <= 65535;
  if (vec) {
    const dim3 grid((unsigned)ceil_div(N / 4, 128), (unsigned)(batch * M));
    splitk_reduce4_kernel<<<grid, 128, 0, st>>>(ws, splits, M, N, ldw, C, ep);
  } else {
    splitk_reduce_kernel<<<elementwise_blocks((int64_t)batch * M * N, 256), 256, 0, st>>>(ws, splits, batch, M, N,
                                                                                          ldw, C, ep);
  }
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

// lo(x) = tf32_lo(x), elementwise over a contiguous span.
__global__ void split_lo_kernel(const float* __restrict__ x, float* __restrict__ lo, int64_t n) {
  const int64_t n4 = n >> 2;
  const float4* x4 = (const float4*)x;
  float4* lo4 = (float4*)lo;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = x4[i];
    float4 r;
    r.x = tf32_lo(v.x);
    r.y = tf32_lo(v.y);
    r.z = tf32_lo(v.z);
    r.w = tf32_lo(v.w);
    lo4[i] = r;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v = x[i];
    lo[i] = tf32_lo(v);
  }
}

// Transposed copy of a [batch][rows][cols] tensor plus the lo part of the
// copy, through 32 x 32 shared-memory tiles (coalesced on both sides).
__global__ void split_transpose_kernel(const float* __restrict__ x, float* __restrict__ hi_t,
                                       float* __restrict__ lo_t, int64_t rows, int64_t cols) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z;
  const float* xb = x + b * rows * cols;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = xb[r * cols + c];
  }
  __syncthreads();
  float* hb = hi_t + b * rows * cols;
  float* lb = lo_t ? lo_t + b * rows * cols : nullptr;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) {
      const float v = tile[threadIdx.x][i];
      hb[c * rows + r] = v;
      if (lb) lb[c * rows + r] = tf32_lo(v);
    }
  }
}

// The same for rows % 4 == 0 and cols % 4 == 0 (16-byte aligned x, hi_t,
// lo_t): 64 x 64 tiles moved with float4 loads and stores, so each row
// segment read or written is 256 contiguous bytes.  Edge tiles are clipped
// to whole float4 groups (the dimensions are multiples of 4).
__global__ void __launch_bounds__(256) split_transpose64_kernel(const float* __restrict__ x,
                                                                float* __restrict__ hi_t,
                                                                float* __restrict__ lo_t, int64_t rows,
                                                                int64_t cols) {
  __shared__ float tile[64][65];
  const int64_t b = blockIdx.z;
  const float* xb = x + b * rows * cols;
  const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
  const int t = threadIdx.x;
  const int q = t & 15;  // float4 group within a 64-wide row segment
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int lr = (t >> 4) + 16 * i;
    const int64_t r = r0 + lr, c = c0 + 4 * q;
    if (r < rows && c < cols) {
      const float4 v = *(const float4*)(xb + r * cols + c);
      tile[lr][4 * q] = v.x;
      tile[lr][4 * q + 1] = v.y;
      tile[lr][4 * q + 2] = v.z;
      tile[lr][4 * q + 3] = v.w;
    }
  }
  __syncthreads();
  float* hb = hi_t + b * rows * cols;
  float* lb = lo_t ? lo_t + b * rows * cols : nullptr;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int lc = (t >> 4) + 16 * i;  // output row = input column
    const int64_t c = c0 + lc, r = r0 + 4 * q;
    if (c < cols && r < rows) {
      float4 v;
      v.x = tile[4 * q][lc];
      v.y = tile[4 * q + 1][lc];
      v.z = tile[4 * q + 2][lc];
      v.w = tile[4 * q + 3][lc];
      *(float4*)(hb + c * rows + r) = v;
      if (lb) {
        float4 l;
        l.x = tf32_lo(v.x);
        l.y = tf32_lo(v.y);
        l.z = tf32_lo(v.z);
        l.w = tf32_lo(v.w);
        *(float4*)(lb + c * rows + r) = l;
      }
    }
  }
}

// CUDA-core GEMM: one output per thread, 16x16 tiles staged in shared
// memory, k walked in increasing order with separately rounded products
// and sums.
__global__ void gemm_simt_kernel(GemmOperand A, GemmOperand B, GemmOutput C, GemmEpilogue ep,
                                 int M, int N, int K) {
  __shared__ float sa[16][17];
  __shared__ float sb[16][17];
  const int bz = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int row = blockIdx.y * 16 + ty;
  const int col = blockIdx.x * 16 + tx;
  const float* a = A.ptr + (int64_t)bz * A.batch_stride;
  const float* b = B.ptr + (int64_t)bz * B.batch_stride;
  float acc = 0.0f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    {
      const int r = blockIdx.y * 16 + ty, k = k0 + tx;
      float v = 0.0f;
      if (r < M && k < K) v = A.trans ? a[(int64_t)k * A.ld + r] : a[(int64_t)r * A.ld + k];
      sa[ty][tx] = v;
    }
    {
      const int k = k0 + ty, c = blockIdx.x * 16 + tx;
      float v = 0.0f;
      if (k < K && c < N) v = B.trans ? b[(int64_t)c * B.ld + k] : b[(int64_t)k * B.ld + c];
      sb[ty][tx] = v;
    }
    __syncthreads();
    const int kmax = (K - k0) < 16 ? (K - k0) : 16;
    for (int kk = 0; kk < kmax; ++kk) acc = __fadd_rn(acc, __fmul_rn(sa[ty][kk], sb[kk][tx]));
    __syncthreads();
  }
  if (row < M && col < N) {
    float r = __fmul_rn(acc, ep.alpha);
    if (ep.alpha == 1.0f) r = acc;
    if (ep.bias != nullptr) r = __fadd_rn(r, ep.bias[col]);
    if (ep.relu) r = fmaxf(r, 0.0f);
    float* dst = C.ptr + (int64_t)bz * C.batch_stride + (int64_t)row * C.ld + col;
    *dst = ep.accumulate ? __fadd_rn(*dst, r) : r;
  }
}

// ---- host side ------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  if (!fn) throw CudaError("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Rank-3 fp32 tensor map {inner, outer, batch}.
CUtensorMap make_map(const float* base, uint64_t inner, uint64_t outer, uint64_t batch,
                     uint64_t ld, uint64_t bstride, uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swz) {
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, outer, batch};
  uint64_t bs = bstride ? bstride : ld * outer;
  bs = (bs + 3) & ~(uint64_t)3;
  cuuint64_t strides[2] = {ld * 4, bs * 4};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)base, dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return m;
}

// Rank-3 fp16 tensor map {inner, outer, 1} over a packed operand half
// (rows of ld elements, ld % 8 == 0).
CUtensorMap make_map16(const __half* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                       uint32_t box_outer) {
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, outer, 1};
  cuuint64_t strides[2] = {ld * 2, ld * 2 * outer};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, (void*)base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled (fp16) failed (" + std::to_string(r) + ")");
  return m;
}

bool tma_ok(const GemmOperand& X, int batch) {
  if (((uintptr_t)X.ptr & 15) != 0) return false;
  if ((X.ld & 3) != 0) return false;
  if (batch > 1 && (X.batch_stride & 3) != 0) return false;
  return true;
}

// Number of elements from the operand's first to its last stored element.
int64_t operand_span(const GemmOperand& X, int batch, int64_t rows, int64_t cols) {
  return (int64_t)(batch - 1) * X.batch_stride + (rows - 1) * X.ld + cols;
}

template <int BN, bool S, bool AMN, bool BMN>
void launch_tc(const CUtensorMap& ma, const CUtensorMap& malo, const CUtensorMap& mb,
               const CUtensorMap& mblo, const CUtensorMap& mc, int c_tma, const GemmOutput& C,
               const GemmEpilogue& ep, int batch, int M, int N, int K, int* d_err, cudaStream_t st) {
  constexpr int smem = PipeCfg<BN, S>::kSmem;
  auto kern = gemm_tf32_kernel<BN, S, AMN, BMN>;
  static bool configured = false;
  if (!configured) {
    TYSOR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  dim3 grid((unsigned)(ceil_div(N, BN) * ceil_div(M, BM)), 1u, (unsigned)batch);
  kern<<<grid, kThreadsTC, smem, st>>>(ma, malo, mb, mblo, mc, C, ep, M, N, K, c_tma, d_err);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

template <int BN, bool S, bool AMN, bool BMN>
void launch_tc2(const CUtensorMap& ma, const CUtensorMap& malo, const CUtensorMap& mb,
                const CUtensorMap& mblo, const CUtensorMap& mc, int c_tma, const GemmOutput& C,
                const GemmEpilogue& ep, int batch, int M, int N, int K, int* d_err, cudaStream_t st) {
  constexpr int smem = PipeCfg2<BN, S>::kSmem;
  auto kern = gemm_tf32_2sm_kernel<BN, S, AMN, BMN>;
  static bool configured = false;
  if (!configured) {
    TYSOR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  dim3 grid((unsigned)(2 * ceil_div(M, 256) * ceil_div(N, BN)), 1u, (unsigned)batch);
  kern<<<grid, kThreadsTC, smem, st>>>(ma, malo, mb, mblo, mc, C, ep, M, N, K, c_tma, d_err);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  TYSOR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (counts[dev] == 0) TYSOR_CUDA(cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev));
  return counts[dev];
}

template <int BN, bool S, bool AMN, bool BMN, bool CONV, bool STACK, int EPI = 0, bool F16 = false>
void launch_pp(const CUtensorMap& ma, const CUtensorMap& malo, const CUtensorMap& mb, const CUtensorMap& mblo,
               const CUtensorMap& mc32, const CUtensorMap& my, const GemmEpilogue& ep, int batch, int M, int N, int K,
               int splits, int* d_err, cudaStream_t st) {
  constexpr int smem = PipeCfgP<BN, S, STACK>::kSmem;
  auto kern = gemm_tf32_pp_kernel<BN, S, AMN, BMN, CONV, STACK, EPI, F16>;
  static bool configured = false;
  if (!configured) {
    TYSOR_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const int64_t tiles = (int64_t)ceil_div(M, 256) * ceil_div(N, BN) * batch * splits;
  if (tiles > INT32_MAX) throw CudaError("matmul has too many tiles");
  int64_t clusters = sm_count() / 2;
  if (clusters > tiles) clusters = tiles;
  if (clusters < 1) clusters = 1;
  kern<<<dim3((unsigned)(2 * clusters), 1u, 1u), pp_threads<CONV>(), smem, st>>>(ma, malo, mb, mblo, mc32, my, ep,
                                                                                  M, N, K, batch, splits, d_err);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

template <int BN, bool S, bool CONV = false, bool STACK = false>
void dispatch_pp(bool amn, bool bmn, const CUtensorMap& ma, const CUtensorMap& malo, const CUtensorMap& mb,
                 const CUtensorMap& mblo, const CUtensorMap& mc32, const CUtensorMap& my, const GemmEpilogue& ep,
                 int batch, int M, int N, int K, int splits, int* d_err, cudaStream_t st) {
  if (amn) {
    if (bmn) launch_pp<BN, S, true, true, CONV, STACK>(ma, malo, mb, mblo, mc32, my, ep, batch, M, N, K, splits, d_err, st);
    else launch_pp<BN, S, true, false, CONV, STACK>(ma, malo, mb, mblo, mc32, my, ep, batch, M, N, K, splits, d_err, st);
  } else {
    if (bmn) launch_pp<BN, S, false, true, CONV, STACK>(ma, malo, mb, mblo, mc32, my, ep, batch, M, N, K, splits, d_err, st);
    else launch_pp<BN, S, false, false, CONV, STACK>(ma, malo, mb, mblo, mc32, my, ep, batch, M, N, K, splits, d_err, st);
  }
}

// Split-K for the persistent kernel: when the output tiles leave the
// resident clusters idle (a weight gradient with few output tiles and a
// long K), K is cut into up to 4 parts of at least 1024 elements, choosing
// the fewest parts that minimise whole rounds of tiles per cluster.
int splitk_parts(int batch, int64_t M, int64_t N, int64_t K) {
  const int64_t BN = N <= 128 ? 128 : 256;
  const int64_t tiles = ceil_div(M, 256) * ceil_div(N, BN) * batch;
  const int64_t clusters = sm_count() / 2;
  if (clusters < 1) return 1;
  int best = 1;
  double best_cost = (double)ceil_div(tiles, clusters);
  for (int parts = 2; parts <= 4; ++parts) {
    if (K / parts < 1024) break;
    const double cost = (double)ceil_div(tiles * parts, clusters) / parts;
    if (cost < 0.9 * best_cost) {
      best = parts;
      best_cost = cost;
    }
  }
  return best;
}

template <int BN, bool S>
void dispatch_layout2(bool amn, bool bmn, const CUtensorMap& ma, const CUtensorMap& malo,
                      const CUtensorMap& mb, const CUtensorMap& mblo, const CUtensorMap& mc, int c_tma,
                      const GemmOutput& C, const GemmEpilogue& ep, int batch, int M, int N, int K,
                      int* d_err, cudaStream_t st) {
  if (amn) {
    if (bmn) launch_tc2<BN, S, true, true>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    else launch_tc2<BN, S, true, false>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
  } else {
    if (bmn) launch_tc2<BN, S, false, true>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    else launch_tc2<BN, S, false, false>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
  }
}

template <int BN, bool S>
void dispatch_layout(bool amn, bool bmn, const CUtensorMap& ma, const CUtensorMap& malo,
                     const CUtensorMap& mb, const CUtensorMap& mblo, const CUtensorMap& mc, int c_tma,
                     const GemmOutput& C, const GemmEpilogue& ep, int batch, int M, int N, int K,
                     int* d_err, cudaStream_t st) {
  if (amn) {
    if (bmn) launch_tc<BN, S, true, true>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    else launch_tc<BN, S, true, false>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
  } else {
    if (bmn) launch_tc<BN, S, false, true>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    else launch_tc<BN, S, false, false>(ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
  }
}

}  // namespace

// The 2-SM (cluster pair) kernel is the default for tiles of 256 columns
// and at least 256 rows: it halves each SM's B-operand traffic through
// shared memory, which binds the 1-SM 128 x 256 tile (3-6% faster on every
// measured shape).  TYSOR_CUDA_GEMM_2SM=0 selects the 1-SM kernel.
bool g_two_sm_enabled = [] {
  const char* v = getenv("TYSOR_CUDA_GEMM_2SM");
  return !(v && v[0] == '0');
}();

// Cluster pairs run the persistent kernel (tiles of 256 x 256, or 256 x 128
// when N <= 128) unless TYSOR_CUDA_GEMM_PERSISTENT=0.
bool g_persistent_enabled = [] {
  const char* v = getenv("TYSOR_CUDA_GEMM_PERSISTENT");
  return !(v && v[0] == '0');
}();

// Strict persistent GEMMs with N <= 128 stack B's high and low parts
// (kStackB) unless TYSOR_CUDA_GEMM_STACK_B=0.
bool g_stack_b_enabled = [] {
  const char* v = getenv("TYSOR_CUDA_GEMM_STACK_B");
  return !(v && v[0] == '0');
}();

// Strict persistent GEMMs make A's low part in shared memory (kConvA)
// unless TYSOR_CUDA_GEMM_CONV_A=0: the split pass over A and the reads of
// its low part from HBM disappear, at no cost to the tensor-core rate
// (measured 1-12% faster per GEMM, split passes included).
bool g_conv_a_enabled = [] {
  const char* v = getenv("TYSOR_CUDA_GEMM_CONV_A");
  return !(v && v[0] == '0');
}();

bool gemm_converts_a(int batch, int64_t M, int64_t N, int64_t K, int mode, int64_t ldc, int64_t stride_c) {
  return mode == kGemmStrict && K > 0 && g_two_sm_enabled && g_persistent_enabled && g_conv_a_enabled &&
         M >= 256 && (ldc & 3) == 0 && (batch == 1 || (stride_c & 3) == 0) && M <= INT32_MAX / 2 &&
         N <= INT32_MAX / 2 && K <= INT32_MAX / 2;
}

int64_t gemm_splitk_ws_elems(int batch, int64_t M, int64_t N, int64_t K, int mode, int64_t ldc, int64_t stride_c) {
  if (mode == kGemmExact || !g_two_sm_enabled || !g_persistent_enabled || M < 256 || (ldc & 3) != 0 ||
      (batch > 1 && (stride_c & 3) != 0) || M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    return 0;
  const int parts = splitk_parts(batch, M, N, K);
  if (parts <= 1) return 0;
  return (int64_t)parts * batch * M * ((N + 3) & ~(int64_t)3);
}

void launch_wait_timeout_probe(int* err, long long limit_cycles, cudaStream_t st) {
  if (limit_cycles < 1 || limit_cycles > kWaitCycles) throw CudaError("wait probe: limit outside [1, 4e9] cycles");
  wait_timeout_probe_kernel<<<1, 1, 0, st>>>(err, limit_cycles);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

int64_t gemm_pack16_elems(int64_t rows, int64_t K) {
  const int64_t kp = (K + 7) & ~(int64_t)7;
  return rows * kp + 2 * ((rows + 3) & ~(int64_t)3);
}

void launch_pack16(const float* x, bool k_contiguous, int64_t rows, int64_t K, int64_t ld, float* packed,
                   cudaStream_t st) {
  if (rows <= 0 || K <= 0) return;
  if (rows > INT32_MAX / 2 || K > INT32_MAX / 2) throw CudaError("pack16: operand too large");
  if ((((uintptr_t)packed) & 15) != 0) throw CudaError("pack16: packed buffer not 16-byte aligned");
  const int64_t kp = (K + 7) & ~(int64_t)7;
  __half* hi = (__half*)packed;
  __half* lo = hi + rows * kp;
  float* factor = (float*)(lo + rows * kp);
  if (k_contiguous) {
    if (ld < K) throw CudaError("pack16: row pitch below K");
    pack16_rows_kernel<<<(unsigned)rows, 256, 0, st>>>(x, ld, (int)K, (int)kp, hi, lo, factor);
    TYSOR_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return;
  }
  if (ld < rows) throw CudaError("pack16: row pitch below the operand's rows");
  if (ceil_div(K, 64) > 65535) throw CudaError("pack16: K too large for the column pass");
  uint32_t* colmax = (uint32_t*)(factor + ((rows + 3) & ~(int64_t)3));
  TYSOR_CUDA(cudaMemsetAsync(colmax, 0, sizeof(uint32_t) * (size_t)rows, st));
  pack16_colmax_kernel<<<dim3((unsigned)ceil_div(rows, 256), (unsigned)ceil_div(K, 64)), 256, 0, st>>>(
      x, ld, (int)rows, (int)K, colmax);
  TYSOR_CUDA(cudaGetLastError());
  pack16_cols_kernel<<<dim3((unsigned)ceil_div(rows, 64), (unsigned)ceil_div(K, 64)), 256, 0, st>>>(
      x, ld, (int)rows, (int)K, (int)kp, colmax, hi, lo, factor);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(2, std::memory_order_relaxed);
}

int gemm_effective_mode(int mode, int batch, int64_t M, int64_t N, int64_t K, int tri, bool smx, int64_t ldc,
                        int64_t stride_c) {
  (void)stride_c;
  if (mode != kGemmStrict16) return mode;
  const bool ok = batch == 1 && tri == 0 && !smx && K > 0 && M >= 256 && N > 128 && (ldc & 3) == 0 &&
                  g_two_sm_enabled && g_persistent_enabled && M <= INT32_MAX / 2 && N <= INT32_MAX / 2 &&
                  K <= INT32_MAX / 2 && ceil_div(K, 64) <= 65535;
  return ok ? kGemmStrict16 : kGemmStrict;
}

void launch_split_lo(const float* x, float* lo, int64_t n, cudaStream_t st) {
  if (n <= 0) return;
  split_lo_kernel<<<elementwise_blocks(n / 4 + 1, 256), 256, 0, st>>>(x, lo, n);
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

void launch_split_transpose(const float* x, float* hi_t, float* lo_t, int64_t batch, int64_t rows,
                            int64_t cols, cudaStream_t st) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return;
  if (batch > 65535 || ceil_div(rows, 32) > 65535) throw CudaError("split_transpose: grid too large");
  const auto a16 = [](const void* p) { return p == nullptr || (((uintptr_t)p) & 15) == 0; };
  if (rows % 4 == 0 && cols % 4 == 0 && a16(x) && a16(hi_t) && a16(lo_t)) {
    dim3 grid((unsigned)ceil_div(cols, 64), (unsigned)ceil_div(rows, 64), (unsigned)batch);
    split_transpose64_kernel<<<grid, 256, 0, st>>>(x, hi_t, lo_t, rows, cols);
  } else {
    dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)batch);
    split_transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(x, hi_t, lo_t, rows, cols);
  }
  TYSOR_CUDA(cudaGetLastError());
  g_launches.fetch_add(1, std::memory_order_relaxed);
}

void gemm_scratch_need(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A,
                       const GemmOperand& B, int mode, int64_t* a_elems, int64_t* b_elems) {
  *a_elems = 0;
  *b_elems = 0;
  if (mode == kGemmStrict16) {
    if (M > 0 && N > 0 && K > 0) {
      *a_elems = gemm_pack16_elems(M, K);
      *b_elems = gemm_pack16_elems(N, K);
    }
    return;
  }
  if (mode != kGemmStrict || !tma_ok(A, batch) || !tma_ok(B, batch) || M == 0 || N == 0 ||
      K == 0)
    return;
  *a_elems = A.trans ? operand_span(A, batch, K, M) : operand_span(A, batch, M, K);
  *b_elems = B.trans ? operand_span(B, batch, N, K) : operand_span(B, batch, K, N);
}

bool gemm_fuses_box_epilogue(int batch, int64_t M, int64_t N, int64_t K, bool ta, bool tb, int mode,
                             int64_t ldc, int64_t stride_c) {
  // The split-fp16 form packs both operands K-major and adds a residual in
  // its epilogue (it has no fused softmax backward: gemm_effective_mode
  // sends those GEMMs to 3xTF32).
  if (mode == kGemmStrict16)
    return gemm_effective_mode(mode, batch, M, N, K, 0, false, ldc, stride_c) == kGemmStrict16;
  return mode == kGemmStrict && K > 0 && !ta && tb && N > 128 && g_two_sm_enabled && g_persistent_enabled &&
         g_conv_a_enabled && M >= 256 && (ldc & 3) == 0 && (batch == 1 || (stride_c & 3) == 0) &&
         M <= INT32_MAX / 2 && N <= INT32_MAX / 2 && K <= INT32_MAX / 2;
}

int gemm_launch_impl(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A, const GemmOperand& B,
                     const GemmOutput& C, const GemmEpilogue& ep, int mode, const GemmScratch& scratch, int* d_err,
                     cudaStream_t st, bool* fused_smx);

// The split-fp16 GEMM (one batch item; gemm_effective_mode holds): packs A
// and B into the scratch (unless presplit), then the persistent pair kernel
// in its kF16 form, split-K where it pays, the residual in the epilogue.
static int launch_f16x3(int64_t M, int64_t N, int64_t K, const GemmOperand& A, const GemmOperand& B, const GemmOutput& C,
                 const GemmEpilogue& ep_in, const GemmScratch& scratch, int* d_err, cudaStream_t st, bool* fused) {
  const int64_t na = gemm_pack16_elems(M, K), nb = gemm_pack16_elems(N, K);
  if (scratch.a_lo == nullptr || scratch.b_lo == nullptr || scratch.a_elems < na || scratch.b_elems < nb)
    throw CudaError("split-fp16 matmul needs scratch for the packed operands (M " + std::to_string(M) + ", N " +
                    std::to_string(N) + ", K " + std::to_string(K) + ")");
  if ((((uintptr_t)C.ptr) & 15) != 0) throw CudaError("split-fp16 matmul needs a 16-byte aligned output");
  if (!scratch.presplit) {
    launch_pack16(A.ptr, !A.trans, M, K, A.ld, scratch.a_lo, st);
    launch_pack16(B.ptr, B.trans, N, K, B.ld, scratch.b_lo, st);
  }
  const int64_t kp = (K + 7) & ~(int64_t)7;
  const __half* ahi = (const __half*)scratch.a_lo;
  const __half* bhi = (const __half*)scratch.b_lo;
  GemmEpilogue ep = ep_in;
  ep.row_factor = (const float*)(ahi + 2 * M * kp);
  ep.col_factor = (const float*)(bhi + 2 * N * kp);
  const CUtensorMap ma = make_map16(ahi, K, M, kp, 2 * BK, BM);
  const CUtensorMap malo = make_map16(ahi + M * kp, K, M, kp, 2 * BK, BM);
  const CUtensorMap mb = make_map16(bhi, K, N, kp, 2 * BK, 128);
  const CUtensorMap mblo = make_map16(bhi + N * kp, K, N, kp, 2 * BK, 128);
  int splits = 1;
  const int64_t ldw = (N + 3) & ~(int64_t)3;
  if (!ep.residual && scratch.ws != nullptr && (((uintptr_t)scratch.ws) & 15) == 0) {
    splits = splitk_parts(1, M, N, K);
    if ((int64_t)splits * M * ldw > scratch.ws_elems) splits = 1;
  }
  const CUtensorMap mc32 = splits > 1 ? make_map(scratch.ws, N, M, (uint64_t)splits, ldw, M * ldw, 32, 32,
                                                 CU_TENSOR_MAP_SWIZZLE_128B)
                                      : make_map(C.ptr, N, M, 1, C.ld, C.batch_stride, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap my =
      ep.residual ? make_map(ep.residual, N, M, 1, C.ld, C.batch_stride, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) : mc32;
  const int im = (int)M, in = (int)N, ik = (int)K;
  if (ep.residual) {
    launch_pp<256, true, false, false, false, false, 2, true>(ma, malo, mb, mblo, mc32, my, ep, 1, im, in, ik, 1,
                                                             d_err, st);
    *fused = true;
  } else {
    launch_pp<256, true, false, false, false, false, 0, true>(ma, malo, mb, mblo, mc32, my, ep, 1, im, in, ik, splits,
                                                             d_err, st);
  }
  if (splits > 1) {
    launch_splitk_reduce(scratch.ws, splits, 1, im, in, ldw, C, ep, st);
  }
  return 1;
}

int gemm_causal_tile_rows(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A, const GemmOperand& B,
                          const GemmOutput& C, int mode) {
  // The same choice as gemm_launch_impl: the CUDA-core path contracts all
  // of K; the cluster-pair kernels (persistent or not) decide the causal
  // range on 256-row pair tiles (pp_tile, gemm_tf32_2sm_kernel), the 1-SM
  // kernel on its 128-row tiles.
  if (M <= 0 || N <= 0 || batch <= 0) return 0;
  const bool tc = mode != kGemmExact && K > 0 && tma_ok(A, batch) && tma_ok(B, batch);
  if (!tc) return 0;
  const int BN = N <= 128 ? 128 : 256;
  const GemmOperand Cview{C.ptr, false, C.ld, C.batch_stride};
  const bool persistent = g_two_sm_enabled && g_persistent_enabled && M >= 256 && tma_ok(Cview, batch);
  const bool two_sm = persistent || (g_two_sm_enabled && BN == 256 && M >= 256);
  return two_sm ? 2 * BM : BM;
}

int gemm_launch(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A,
                const GemmOperand& B, const GemmOutput& C, const GemmEpilogue& ep, int mode,
                const GemmScratch& scratch, int* d_err, cudaStream_t st) {
  if (ep.smx_p && (ep.accumulate || ep.bias || ep.relu || ep.residual))
    throw CudaError("the fused softmax backward epilogue takes no accumulate, bias, relu or residual");
  if (ep.residual && ep.accumulate) throw CudaError("a GEMM adds a residual or accumulates, not both");
  bool fused = false;
  const int r = gemm_launch_impl(batch, M, N, K, A, B, C, ep, mode, scratch, d_err, st, &fused);
  // Callers ask for the fused epilogue only where gemm_fuses_softmax_backward
  // holds; another kernel form would have written dP, not dS.
  if ((ep.smx_p || ep.residual) && !fused && M > 0 && N > 0 && batch > 0)
    throw CudaError("fused GEMM epilogue requested for a GEMM form without it");
  return r;
}

int gemm_launch_impl(int batch, int64_t M, int64_t N, int64_t K, const GemmOperand& A, const GemmOperand& B,
                     const GemmOutput& C, const GemmEpilogue& ep, int mode, const GemmScratch& scratch, int* d_err,
                     cudaStream_t st, bool* fused_smx) {
  if (M <= 0 || N <= 0 || batch <= 0) return 0;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    throw CudaError("matmul dimension too large");
  if (mode == kGemmStrict16) {
    if (gemm_effective_mode(mode, batch, M, N, K, ep.tri, ep.smx_p != nullptr, C.ld, C.batch_stride) != kGemmStrict16)
      throw CudaError("split-fp16 matmul requested for a GEMM it does not cover (gemm_effective_mode)");
    return launch_f16x3(M, N, K, A, B, C, ep, scratch, d_err, st, fused_smx);
  }
  const bool tc = mode != kGemmExact && K > 0 && tma_ok(A, batch) && tma_ok(B, batch);
  if (!tc) {
    // (K == 0 lands here too: the loop adds nothing and the epilogue writes
    // the empty product.)
    dim3 grid((unsigned)ceil_div(N, 16), (unsigned)ceil_div(M, 16), (unsigned)batch);
    gemm_simt_kernel<<<grid, dim3(16, 16), 0, st>>>(A, B, C, ep, (int)M, (int)N, (int)K);
    TYSOR_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return 0;
  }
  const bool strict = mode == kGemmStrict;
  const int BN = N <= 128 ? 128 : 256;
  // The pair forms need a full 256-row pair tile to be worth their cluster;
  // the persistent one also needs C on 16-byte strides (its TMA stores).
  const GemmOperand Cview{C.ptr, false, C.ld, C.batch_stride};
  const int c_tma = tma_ok(Cview, batch) ? 1 : 0;
  const bool persistent = g_two_sm_enabled && g_persistent_enabled && M >= 256 && c_tma;
  const bool conv_a = strict && persistent && g_conv_a_enabled;
  const float* alo = A.ptr;
  const float* blo = B.ptr;
  if (strict) {
    int64_t na, nb;
    gemm_scratch_need(batch, M, N, K, A, B, mode, &na, &nb);
    if ((!conv_a && (scratch.a_lo == nullptr || scratch.a_elems < na)) || scratch.b_lo == nullptr ||
        scratch.b_elems < nb)
      throw CudaError("strict matmul needs scratch for the split operands (batch " + std::to_string(batch) +
                      ", M " + std::to_string(M) + ", N " + std::to_string(N) + ", K " + std::to_string(K) +
                      ", A needs " + std::to_string(na) + " has " + std::to_string(scratch.a_elems) +
                      (scratch.a_lo ? "" : " (none)") + ", B needs " + std::to_string(nb) + " has " +
                      std::to_string(scratch.b_elems) + (scratch.b_lo ? "" : " (none)") + ")");
    if (!scratch.presplit) {
      if (!conv_a) launch_split_lo(A.ptr, scratch.a_lo, na, st);
      launch_split_lo(B.ptr, scratch.b_lo, nb, st);
    }
    alo = scratch.a_lo;
    blo = scratch.b_lo;
  }
  const bool two_sm = persistent || (g_two_sm_enabled && BN == 256 && M >= 256);
  const bool amn = A.trans, bmn = !B.trans;
  // A: K-major stored [M,K] -> dims {K, M}; MN-major stored [K,M] -> dims {M, K}.
  const uint64_t a_in = amn ? M : K, a_out = amn ? K : M;
  const uint64_t b_in = bmn ? N : K, b_out = bmn ? K : N;
  const uint32_t a_box_in = amn ? 32 : BK, a_box_out = amn ? BK : BM;
  const uint32_t b_rows = two_sm ? (uint32_t)BN / 2 : (uint32_t)BN;
  const uint32_t b_box_in = bmn ? 32 : BK, b_box_out = bmn ? BK : b_rows;
  const CUtensorMapSwizzle a_sw = amn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapSwizzle b_sw = bmn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap ma = make_map(A.ptr, a_in, a_out, batch, A.ld, A.batch_stride, a_box_in, a_box_out, a_sw);
  CUtensorMap mb = make_map(B.ptr, b_in, b_out, batch, B.ld, B.batch_stride, b_box_in, b_box_out, b_sw);
  CUtensorMap malo = ma, mblo = mb;
  if (strict) {
    malo = make_map(alo, a_in, a_out, batch, A.ld, A.batch_stride, a_box_in, a_box_out, a_sw);
    mblo = make_map(blo, b_in, b_out, batch, B.ld, B.batch_stride, b_box_in, b_box_out, b_sw);
  }
  if (persistent) {
    // Split-K into the caller's workspace when it has one and it pays.
    int splits = 1;
    const int64_t ldw = (N + 3) & ~(int64_t)3;
    if (ep.tri == 0 && !ep.residual && scratch.ws != nullptr && (((uintptr_t)scratch.ws) & 15) == 0) {
      splits = splitk_parts(batch, M, N, K);
      if ((int64_t)splits * batch * M * ldw > scratch.ws_elems) splits = 1;
    }
    const CUtensorMap mc32 =
        splits > 1 ? make_map(scratch.ws, N, M, (uint64_t)splits * batch, ldw, M * ldw, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B)
                   : make_map(C.ptr, N, M, batch, C.ld, C.batch_stride, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    // The probabilities of a fused softmax backward, in C's layout.
    const float* yp = ep.smx_p ? ep.smx_p : ep.residual;
    const CUtensorMap my =
        yp ? make_map(yp, N, M, batch, C.ld, C.batch_stride, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B) : mc32;
    const int im = (int)M, in = (int)N, ik = (int)K;
    if (BN == 128) {
      const bool stack_b = strict && g_stack_b_enabled;
      if (conv_a && stack_b)
        dispatch_pp<128, true, true, true>(amn, bmn, ma, ma, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else if (conv_a) dispatch_pp<128, true, true>(amn, bmn, ma, ma, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else if (stack_b)
        dispatch_pp<128, true, false, true>(amn, bmn, ma, malo, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else if (strict) dispatch_pp<128, true>(amn, bmn, ma, malo, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else dispatch_pp<128, false>(amn, bmn, ma, malo, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
    } else if (ep.smx_p && conv_a && !amn && !bmn && splits == 1) {
      // The probability gradient of a causal softmax, written as dS.
      launch_pp<256, true, false, false, true, false, true>(ma, ma, mb, mblo, mc32, my, ep, batch, im, in, ik, splits,
                                                            d_err, st);
      *fused_smx = true;
    } else if (ep.residual && conv_a && !amn && !bmn && splits == 1) {
      // C = residual + the product (a residual connection around a linear).
      launch_pp<256, true, false, false, true, false, 2>(ma, ma, mb, mblo, mc32, my, ep, batch, im, in, ik, splits,
                                                         d_err, st);
      *fused_smx = true;
    } else {
      if (conv_a) dispatch_pp<256, true, true>(amn, bmn, ma, ma, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else if (strict) dispatch_pp<256, true>(amn, bmn, ma, malo, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
      else dispatch_pp<256, false>(amn, bmn, ma, malo, mb, mblo, mc32, my, ep, batch, im, in, ik, splits, d_err, st);
    }
    if (splits > 1) {
      launch_splitk_reduce(scratch.ws, splits, batch, im, in, ldw, C, ep, st);
    }
    return 1;
  }
  // The tile-store epilogue needs C's rows and batches on 16-byte strides.
  CUtensorMap mc = ma;
  if (c_tma) mc = make_map(C.ptr, N, M, batch, C.ld, C.batch_stride, 32, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (two_sm) {
    if (strict) dispatch_layout2<256, true>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    else dispatch_layout2<256, false>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
  } else {
    if (BN == 128) {
      if (strict) dispatch_layout<128, true>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
      else dispatch_layout<128, false>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    } else {
      if (strict) dispatch_layout<256, true>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
      else dispatch_layout<256, false>(amn, bmn, ma, malo, mb, mblo, mc, c_tma, C, ep, batch, M, N, K, d_err, st);
    }
  }
  return 1;
}

}  // namespace tysor
