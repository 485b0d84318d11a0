// Shared device/host helpers for the sm_100a token-loop kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace tmg {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  Every kernel calls pdl_trigger() at
// its start, so the next kernel in the stream may be scheduled while this
// one drains, and pdl_wait() before it touches anything an earlier kernel
// wrote.  Work that depends on nothing earlier (streaming this kernel's own
// weights) goes between the two.  Both are no-ops without the launch
// attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// BF16 bit pattern -> f32 (exact: the reference's `(w as u32) << 16`).
__device__ __forceinline__ float bf16lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16hi(uint32_t packed) {
  return __uint_as_float(packed & 0xffff0000u);
}
__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// Streaming 16-byte load that bypasses L1 allocation (weights are read once
// per token; keep L1 for activations).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Order-preserving key for (value, index) argmax with the reference's rule
// (src/tensor.rs:1063-1073): the largest value wins, ties go to the lowest
// index, NaN and -inf never win.  Larger key = better; 0 = "no candidate".
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  if (!(v > -INFINITY)) return 0ull;  // NaN or -inf
  uint32_t b = __float_as_uint(v + 0.0f);  // -0 -> +0
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(~idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
  return k == 0ull ? 0u : ~static_cast<uint32_t>(k & 0xffffffffull);
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// ---------------------------------------------------------------------------
// mbarriers and bulk (TMA) copies, shared-memory side.
// ---------------------------------------------------------------------------
// A healthy wait lasts microseconds; one that exceeds this gives up.
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the phase of parity `parity` to complete; false after
// kWaitNs (the caller records an error and stops waiting).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (unsigned int i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 63) == 0) {
      const unsigned long long t = global_ns();
      if (i == 0) t0 = t;
      else if (t - t0 > kWaitNs) return false;
    }
  }
}
// Non-blocking test: has the phase of parity `parity` completed?
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Contiguous global -> shared bulk copy (TMA engine), completing `bytes`
// of transaction on `bar`.  Both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Block-wide sum for blockDim.x == NT (a multiple of 32); `red` holds
// NT/32 floats.  All threads get the result.
template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / kWarp, l = threadIdx.x % kWarp;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / kWarp; ++i) t += red[i];
  return t;
}

}  // namespace tmg

// Host-side error plumbing: every launcher returns cudaError_t; the API
// layer turns it into a status code + message.
#define TMG_CUDA_TRY(expr)                       \
  do {                                           \
    cudaError_t _e = (expr);                     \
    if (_e != cudaSuccess) return _e;            \
  } while (0)

namespace tmg {
// Every kernel of the library asks for the largest shared-memory carveout,
// so consecutive kernels never make an SM switch its L1 / shared split
// (which drains the SM and keeps the next kernel's CTAs from co-residing
// with the previous kernel's under programmatic dependent launch).
template <typename K>
inline cudaError_t set_carveout(K kern, int max_dynamic_smem = -1) {
  cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                       cudaFuncAttributePreferredSharedMemoryCarveout,
                                       int(cudaSharedmemCarveoutMaxShared));
  if (e == cudaSuccess && max_dynamic_smem >= 0)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_dynamic_smem);
  return e;
}
}  // namespace tmg
