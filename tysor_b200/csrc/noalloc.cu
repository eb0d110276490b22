// tysor_cuda_matmul_noalloc: the strict (3xTF32) matmul for callers that
// must not allocate device memory.
//
// Who needs it: code that runs inside another runtime's memory budget —
// an inference server or training framework that reserves the GPU's memory
// up front and hands out only its own pools, or a hot path that must never
// call cudaMalloc/cudaFree because those calls synchronise the device and
// can fail once the pool owns the memory.  Such callers can provide the
// input and output buffers, but not the scratch the strict matmul needs for
// the low halves of its operands.
//
// How: the scratch lives in a file-scope __device__ array of fixed size.
// The CUDA runtime claims it on a device when it loads this library's module
// there: under the default lazy module loading that is the first call on the
// device (the address lookup below loads the module), with
// CUDA_MODULE_LOADING=EAGER it is when the process first initialises the
// device.  A caller that reserves most of the GPU's memory for its own pool
// should therefore make the first call before reserving it.  Every GPU that
// has loaded the module holds the array until the process exits.  Host code
// cannot pass the array's name to a kernel — on the host that name is only a
// stand-in, not a device address — so the first call on each device asks the
// runtime for the array's address (cudaGetSymbolAddress, with that device
// current) and keeps it.  Because that first call does this set-up work,
// make it before any stream capture.
//
// Errors inside the kernel (a tensor-core pipeline wait that ran out of
// time) cannot be returned by the call, which only enqueues work: the kernel
// records them in a device error word that starts at zero.
// tysor_cuda_matmul_noalloc_status waits for a stream, reads the word, clears
// it and reports what it held.
//
// Limits and sharing: A and B together may span at most
// kNoAllocScratchFloats elements (32 MiB); larger calls are rejected with an
// error.  All calls on a device share the one array and it keeps whatever
// the previous call left there; every call overwrites the part it reads
// before reading it, so nothing needs clearing between calls.  Two calls
// that overlap on the GPU (different streams, or different host threads)
// race on the array: order them on one stream.
#include <mutex>
#include <string>

#include "../../include/tysor_cuda.h"
#include "common.cuh"
#include "context.cuh"

namespace tysor {
namespace {

constexpr int64_t kNoAllocScratchFloats = 8LL * 1024 * 1024;  // 32 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
// Zero-initialised by the module image, so no set-up write is needed; only
// the kernels set it and only tysor_cuda_matmul_noalloc_status clears it.
static __device__ __align__(256) int g_noalloc_error[4] = {0, 0, 0, 0};

struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;
  int* error = nullptr;
};

NoAllocDevice g_devices[kMaxDevices];
std::mutex g_setup_mutex;

// Once per device, with that device current: resolve the device addresses
// of the scratch array and the error word.
NoAllocDevice& device_state() {
  int dev = 0;
  TYSOR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) throw CudaError("device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  NoAllocDevice& s = g_devices[dev];
  if (!s.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) throw CudaError(std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    s.scratch = static_cast<float*>(p);
    e = cudaGetSymbolAddress(&p, g_noalloc_error);
    if (e != cudaSuccess) throw CudaError(std::string("cudaGetSymbolAddress(error): ") + cudaGetErrorString(e));
    s.error = static_cast<int*>(p);
    s.ready = true;
  }
  return s;
}

}  // namespace
}  // namespace tysor

using namespace tysor;

extern "C" bool tysor_cuda_matmul_noalloc(void* stream, uint32_t m, uint32_t n, uint32_t k,
                                          const float* a, const float* b, float* c) {
  try {
    if (!a || !b || !c) throw CudaError("matmul_noalloc: null pointer");
    GemmOperand A{a, false, (int64_t)k, 0};
    GemmOperand B{b, false, (int64_t)n, 0};
    GemmOutput O{c, (int64_t)n, 0};
    GemmEpilogue ep{nullptr, 1.0f, 0, 0};
    int64_t na = 0, nb = 0;
    gemm_scratch_need(1, m, n, k, A, B, kGemmStrict, &na, &nb);
    const int64_t na_pad = (na + 63) & ~(int64_t)63;
    if (na_pad + nb > kNoAllocScratchFloats)
      throw CudaError("matmul_noalloc: operands span " + std::to_string(na + nb) +
                      " elements; the fixed scratch holds at most " +
                      std::to_string(kNoAllocScratchFloats) + " (use tysor_cuda_dispatch_matmul)");
    NoAllocDevice& dev = device_state();
    GemmScratch s{dev.scratch, dev.scratch + na_pad, na, nb};
    gemm_launch(1, m, n, k, A, B, O, ep, kGemmStrict, s, dev.error, (cudaStream_t)stream);
    return true;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return false;
  }
}

extern "C" bool tysor_cuda_matmul_noalloc_status(void* stream) {
  try {
    NoAllocDevice& dev = device_state();
    const cudaStream_t st = (cudaStream_t)stream;
    int code = 0;
    TYSOR_CUDA(cudaMemcpyAsync(&code, dev.error, sizeof(int), cudaMemcpyDeviceToHost, st));
    TYSOR_CUDA(cudaStreamSynchronize(st));
    if (code != 0) {
      TYSOR_CUDA(cudaMemsetAsync(dev.error, 0, sizeof(int), st));
      TYSOR_CUDA(cudaStreamSynchronize(st));
      throw CudaError(std::string("matmul_noalloc: ") + device_error_message(code));
    }
    return true;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return false;
  }
}
