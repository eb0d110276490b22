// Context, buffers and error plumbing shared by the C ABI (bridge.cu) and
// the graph executor (executor.cu).
#pragma once

#include <atomic>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"

namespace tysor {

// Kernel launches enqueued by this library (all threads, all contexts).
extern std::atomic<int64_t> g_launches;

void set_last_error(const std::string& msg);

struct Context {
  int device = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;  // device error word (DeviceError)
  int matmul_mode = kGemmStrict;
  // k-blocks per tensor-memory accumulation chunk of the tensor-core
  // matmuls (GemmEpilogue::chunk_kb; 0 = the default).
  int accum_chunk_kb = 0;
  // Scratch shared by per-op dispatches (split operands, partial sums).
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // cos/sin tables for RoPE, keyed by (seq, half, theta bits).
  std::map<std::tuple<int64_t, int64_t, uint64_t>, float2*> rope_tables;
  // NCCL communicator (opaque ncclComm_t) when data parallel.
  void* comm = nullptr;
  int nranks = 1;
  int rank = 0;

  // Grows the shared scratch (synchronising first if it must reallocate).
  void* ensure_scratch(size_t bytes);
  // Device (cos, sin) table for rope over `seq` positions and `half` freqs.
  const float2* rope_table(int64_t seq, int64_t half, double theta);
  // Waits for the stream and turns a recorded device error into a message.
  void sync_and_check();
};

struct Buffer {
  Context* ctx = nullptr;
  float* ptr = nullptr;
  size_t count = 0;
  bool owned = false;
};

const char* device_error_message(int code);

// All-reduce (sum) of `count` floats in place on the context stream.
void comm_allreduce(Context* ctx, float* data, size_t count);
// The same on another stream of the context's device.
void comm_allreduce_on(Context* ctx, float* data, size_t count, cudaStream_t stream);

}  // namespace tysor
