// NCCL over NVLink / NVSwitch for the tensor-parallel decode (one allreduce
// after o_proj and one after down_proj per layer; an allgather of the
// vocab-split logits).
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>

#include "common.cuh"
#include "tp.h"

namespace tmg {

namespace {

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
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
      a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
      a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
      a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
      a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
      a.err_string = reinterpret_cast<decltype(a.err_string)>(dlsym(h, "ncclGetErrorString"));
      if (a.get_unique_id && a.init_rank && a.destroy && a.all_reduce && a.all_gather &&
          a.err_string)
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

}  // namespace

struct TpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  float* gather_tmp = nullptr;
  size_t gather_cap = 0;
};

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
  ncclResult_t r = a.init_rank(&t->comm, world, u, rank);
  if (r != ncclSuccess) {
    err = std::string("ncclCommInitRank: ") + a.err_string(r);
    delete t;
    return nullptr;
  }
  return t;
}

void tp_destroy(TpComm* t) {
  if (!t) return;
  if (t->comm) api().destroy(t->comm);
  if (t->gather_tmp) cudaFree(t->gather_tmp);
  delete t;
}

cudaError_t tp_allreduce_sum(TpComm* t, float* buf, int64_t n, cudaStream_t s) {
  if (!t) return cudaErrorInvalidValue;
  ncclResult_t r = api().all_reduce(buf, buf, size_t(n), ncclFloat32, ncclSum, t->comm, s);
  return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
}

cudaError_t tp_allgather_rows(TpComm* t, const float* local, int64_t n_local, float* out,
                              int64_t n_full, int M, cudaStream_t s) {
  if (!t || n_full != n_local * t->world) return cudaErrorInvalidValue;
  if (M == 1) {
    ncclResult_t r = api().all_gather(local, out, size_t(n_local), ncclFloat32, t->comm, s);
    return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
  }
  const size_t need = size_t(n_full) * M;
  if (t->gather_cap < need) {
    if (t->gather_tmp) cudaFree(t->gather_tmp);
    t->gather_tmp = nullptr;
    t->gather_cap = 0;
    TMG_CUDA_TRY(cudaMalloc(&t->gather_tmp, need * sizeof(float)));
    t->gather_cap = need;
  }
  ncclResult_t r =
      api().all_gather(local, t->gather_tmp, size_t(n_local) * M, ncclFloat32, t->comm, s);
  if (r != ncclSuccess) return cudaErrorUnknown;
  interleave_kernel<<<296, 256, 0, s>>>(t->gather_tmp, n_local, t->world, M, out);
  return cudaGetLastError();
}

}  // namespace tmg
