// Tensor-parallel communicator: NCCL, loaded at run time (libnccl.so.2) so
// that the library itself does not link it; only contexts that call
// tmg_tp_init need it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace tmg {

struct TpComm;

int tp_unique_id(uint8_t id[128]);
TpComm* tp_create(const uint8_t id[128], int rank, int world, std::string& err);
void tp_destroy(TpComm* t);
// In-place sum of n floats over the ranks.
cudaError_t tp_allreduce_sum(TpComm* t, float* buf, int64_t n, cudaStream_t s);
// Every rank holds rows [M, n_local] (its vocab shard); out [M, n_full]
// receives the shards side by side (n_full = world * n_local).
cudaError_t tp_allgather_rows(TpComm* t, const float* local, int64_t n_local, float* out,
                              int64_t n_full, int M, cudaStream_t s);
// Every rank's stream reaches this point before any passes it (a one-float
// allreduce on `scratch`, a device float).
cudaError_t tp_barrier(TpComm* t, float* scratch, cudaStream_t s);

}  // namespace tmg
