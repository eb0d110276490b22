// Data-parallel gradient all-reduce through NCCL (sum, fp32), reached by
// dlopen so the library links no particular NCCL build: if the process has
// already loaded libnccl.so.2 (for example through torch.distributed), that
// copy is reused.  The reference has no multi-device code; this is the
// collective of batch-sharded training.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "../../include/tysor_cuda.h"
#include "context.cuh"

namespace tysor {
namespace {

struct NcclApi {
  void* handle = nullptr;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
  decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
  decltype(&ncclCommAbort) abort_comm = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.handle = h;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.init_rank_config = (decltype(api.init_rank_config))dlsym(h, "ncclCommInitRankConfig");
    api.get_async_error = (decltype(api.get_async_error))dlsym(h, "ncclCommGetAsyncError");
    api.abort_comm = (decltype(api.abort_comm))dlsym(h, "ncclCommAbort");
    api.destroy = (decltype(api.destroy))dlsym(h, "ncclCommDestroy");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
  });
  if (!api.handle || !api.get_unique_id || !api.init_rank_config || !api.get_async_error ||
      !api.abort_comm || !api.destroy || !api.all_reduce)
    throw CudaError("NCCL (libnccl.so.2) could not be loaded");
  return api;
}

std::string nccl_msg(ncclResult_t r) {
  const char* s = nccl().error_string ? nccl().error_string(r) : nullptr;
  return s ? s : ("NCCL error " + std::to_string((int)r));
}

// Polls a non-blocking communicator until its pending operation settles.
void wait_comm(ncclComm_t comm, int timeout_ms, const char* what) {
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = nccl().get_async_error(comm, &st);
    if (r != ncclSuccess) throw CudaError(std::string(what) + ": " + nccl_msg(r));
    if (st == ncclSuccess) return;
    if (st != ncclInProgress) throw CudaError(std::string(what) + ": " + nccl_msg(st));
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0)
                  .count();
    if (timeout_ms > 0 && ms > timeout_ms)
      throw CudaError(std::string(what) + " timed out after " + std::to_string(ms) + " ms");
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

void comm_allreduce(Context* ctx, float* data, size_t count) { comm_allreduce_on(ctx, data, count, ctx->stream); }

void comm_allreduce_on(Context* ctx, float* data, size_t count, cudaStream_t stream) {
  if (!ctx->comm) throw CudaError("no communicator: call tysor_cuda_comm_init first");
  if (count == 0) return;
  ncclComm_t comm = (ncclComm_t)ctx->comm;
  ncclResult_t r = nccl().all_reduce(data, data, count, ncclFloat, ncclSum, comm, stream);
  if (r == ncclInProgress) {
    wait_comm(comm, 60000, "ncclAllReduce");
  } else if (r != ncclSuccess) {
    throw CudaError("ncclAllReduce: " + nccl_msg(r));
  }
}

}  // namespace tysor

using namespace tysor;

namespace {
template <typename F>
bool guarded_comm(F&& f) {
  try {
    f();
    return true;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return false;
  }
}
}  // namespace

extern "C" {

bool tysor_cuda_nccl_get_unique_id(uint8_t out_id[128]) {
  return guarded_comm([&] {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    ncclResult_t r = nccl().get_unique_id(&id);
    if (r != ncclSuccess) throw CudaError("ncclGetUniqueId: " + nccl_msg(r));
    std::memcpy(out_id, &id, sizeof id);
  });
}

bool tysor_cuda_comm_init(void* context, int nranks, int rank, const uint8_t id[128],
                          int timeout_ms) {
  return guarded_comm([&] {
    if (!context) throw CudaError("null context");
    Context* c = static_cast<Context*>(context);
    if (nranks < 1 || rank < 0 || rank >= nranks) throw CudaError("invalid rank / world size");
    if (c->comm) throw CudaError("context already has a communicator");
    TYSOR_CUDA(cudaSetDevice(c->device));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = nccl().init_rank_config(&comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) throw CudaError("ncclCommInitRankConfig: " + nccl_msg(r));
    try {
      wait_comm(comm, timeout_ms, "ncclCommInitRankConfig");
    } catch (...) {
      if (comm) nccl().abort_comm(comm);
      throw;
    }
    c->comm = comm;
    c->nranks = nranks;
    c->rank = rank;
  });
}

bool tysor_cuda_comm_free(void* context) {
  return guarded_comm([&] {
    if (!context) throw CudaError("null context");
    Context* c = static_cast<Context*>(context);
    if (!c->comm) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    ncclComm_t comm = (ncclComm_t)c->comm;
    c->comm = nullptr;
    ncclResult_t r = nccl().destroy(comm);
    if (r == ncclInProgress) r = ncclSuccess;
    if (r != ncclSuccess) {
      nccl().abort_comm(comm);
      throw CudaError("ncclCommDestroy: " + nccl_msg(r));
    }
    c->nranks = 1;
    c->rank = 0;
  });
}

bool tysor_cuda_allreduce_sum(void* context, void* buffer, uint64_t count) {
  return guarded_comm([&] {
    if (!context || !buffer) throw CudaError("null argument");
    Context* c = static_cast<Context*>(context);
    Buffer* b = static_cast<Buffer*>(buffer);
    if (count > b->count) throw CudaError("all-reduce past the end of the buffer");
    TYSOR_CUDA(cudaSetDevice(c->device));
    comm_allreduce(c, b->ptr, count);
  });
}

}  // extern "C"
