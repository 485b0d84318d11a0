// NCCL over NVLink / NVSwitch for the tensor-parallel decode (one allreduce
// after o_proj and one after down_proj per layer; an allgather of the
// vocab-split logits).
//
// The communicator is non-blocking (ncclConfig_t.blocking = 0): every NCCL
// call that reports ncclInProgress is polled with ncclCommGetAsyncError
// against a deadline, so a rank whose peers never join (or never enqueue)
// gets TMG_ERR_NCCL back instead of blocking in the host call for good.
// The deadline is TMG_TP_TIMEOUT_S seconds (default 300); on expiry the
// communicator is aborted (ncclCommAbort) and is unusable afterwards.
// A collective already running on the GPU waits for its peers there: that
// wait is NCCL's, not bounded by this file.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "common.cuh"
#include "tp.h"

namespace tmg {

namespace {

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*err_string)(ncclResult_t) = nullptr;
  bool ok() const { return h != nullptr; }
};

NcclApi& api() {
  static NcclApi a;
  static bool tried = false;
  if (!tried) {
    tried = true;
    // prefer an NCCL already in the process (torch's), else the system one
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
      a.init_rank_config =
          reinterpret_cast<decltype(a.init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
      a.get_async_error =
          reinterpret_cast<decltype(a.get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
      a.abort = reinterpret_cast<decltype(a.abort)>(dlsym(h, "ncclCommAbort"));
      a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
      a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
      a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
      a.err_string = reinterpret_cast<decltype(a.err_string)>(dlsym(h, "ncclGetErrorString"));
      if (a.get_unique_id && a.init_rank_config && a.get_async_error && a.abort && a.destroy &&
          a.all_reduce && a.all_gather && a.err_string)
        a.h = h;
    }
  }
  return a;
}

__global__ void interleave_kernel(const float* __restrict__ g, int64_t n_local, int world, int M,
                                  float* __restrict__ out) {
  // g: [world][M][n_local] -> out: [M][world * n_local]
  const int64_t total = int64_t(world) * M * n_local;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / (int64_t(M) * n_local);
    const int64_t rem = i % (int64_t(M) * n_local);
    const int64_t m = rem / n_local, j = rem % n_local;
    out[m * world * n_local + r * n_local + j] = g[i];
  }
}

double tp_timeout_s() {
  const char* e = getenv("TMG_TP_TIMEOUT_S");
  const double v = e ? atof(e) : 0.0;
  return v > 0.0 ? v : 300.0;
}

}  // namespace

struct TpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool aborted = false;
  float* gather_tmp = nullptr;
  size_t gather_cap = 0;
};

namespace {

// r is the result of an NCCL call on t->comm: while it is ncclInProgress,
// poll the communicator until the call has completed or the deadline has
// passed (then abort the communicator and report ncclInProgress).
ncclResult_t settle(TpComm* t, ncclResult_t r, double timeout_s) {
  if (r != ncclInProgress) return r;
  NcclApi& a = api();
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned int i = 0;; ++i) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t q = a.get_async_error(t->comm, &st);
    if (q != ncclSuccess) return q;
    if (st != ncclInProgress) return st;
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      a.abort(t->comm);
      t->aborted = true;
      return ncclInProgress;
    }
    // an enqueue usually settles within microseconds: spin first, then
    // sleep (communicator set-up can take seconds)
    if (i < 4096) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

cudaError_t as_cuda(ncclResult_t r) { return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown; }

}  // namespace

int tp_unique_id(uint8_t id[128]) {
  NcclApi& a = api();
  if (!a.ok()) return -1;
  ncclUniqueId u;
  if (a.get_unique_id(&u) != ncclSuccess) return -1;
  static_assert(sizeof(u) == 128, "ncclUniqueId size");
  std::memcpy(id, &u, 128);
  return 0;
}

TpComm* tp_create(const uint8_t id[128], int rank, int world, std::string& err) {
  NcclApi& a = api();
  if (!a.ok()) {
    err = "NCCL (libnccl.so.2) could not be loaded";
    return nullptr;
  }
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  TpComm* t = new TpComm();
  t->rank = rank;
  t->world = world;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const double limit = tp_timeout_s();
  ncclResult_t r = settle(t, a.init_rank_config(&t->comm, world, u, rank, &cfg), limit);
  if (r == ncclInProgress) {
    err = "ncclCommInitRankConfig: the other ranks did not join within " +
          std::to_string(int(limit)) + " s (communicator aborted)";
    delete t;
    return nullptr;
  }
  if (r != ncclSuccess) {
    err = std::string("ncclCommInitRankConfig: ") + a.err_string(r);
    if (t->comm) a.abort(t->comm);
    delete t;
    return nullptr;
  }
  return t;
}

void tp_destroy(TpComm* t) {
  if (!t) return;
  if (t->comm && !t->aborted) api().destroy(t->comm);
  if (t->gather_tmp) cudaFree(t->gather_tmp);
  delete t;
}

cudaError_t tp_allreduce_sum(TpComm* t, float* buf, int64_t n, cudaStream_t s) {
  if (!t || t->aborted) return cudaErrorInvalidValue;
  return as_cuda(settle(t, api().all_reduce(buf, buf, size_t(n), ncclFloat32, ncclSum, t->comm, s),
                        tp_timeout_s()));
}

cudaError_t tp_allgather_rows(TpComm* t, const float* local, int64_t n_local, float* out,
                              int64_t n_full, int M, cudaStream_t s) {
  if (!t || t->aborted || n_full != n_local * t->world) return cudaErrorInvalidValue;
  if (M == 1)
    return as_cuda(settle(t, api().all_gather(local, out, size_t(n_local), ncclFloat32, t->comm, s),
                          tp_timeout_s()));
  const size_t need = size_t(n_full) * M;
  if (t->gather_cap < need) {
    if (t->gather_tmp) cudaFree(t->gather_tmp);
    t->gather_tmp = nullptr;
    t->gather_cap = 0;
    TMG_CUDA_TRY(cudaMalloc(&t->gather_tmp, need * sizeof(float)));
    t->gather_cap = need;
  }
  const ncclResult_t r = settle(
      t, api().all_gather(local, t->gather_tmp, size_t(n_local) * M, ncclFloat32, t->comm, s),
      tp_timeout_s());
  if (r != ncclSuccess) return cudaErrorUnknown;
  interleave_kernel<<<296, 256, 0, s>>>(t->gather_tmp, n_local, t->world, M, out);
  return cudaGetLastError();
}

cudaError_t tp_barrier(TpComm* t, float* scratch, cudaStream_t s) {
  return tp_allreduce_sum(t, scratch, 1, s);
}

}  // namespace tmg
