// The int8 weight path of the decode GEMV: the reference's TMG_I8=1
// (wmat_maybe_i8, src/model.rs:57-76; WMat::quantize_i8, src/tensor.rs:
// 282-297; the I8 arm of matmul_w_into, src/tensor.rs:341-357, with
// quantize_row_i8 and dot_i8, src/tensor.rs:128-170).
//
// Layer matrices are quantized once at load, per row: scale = max|w| / 127
// (1 for an all-zero row), q = round(w / scale) clamped to +-127.  A GEMV
// quantizes its activation row the same way (scale s = max|x| / 127, q =
// round(x * (1 / s)); an all-zero row has s = 0), takes exact integer dots
// (dp4a, i32: the order of the sum does not matter) and writes
// y[o] = f32(dot) * s * scale[o].  With the same quantized inputs the
// result is bit-identical to the reference's.  HBM-bound: algorithmic bytes
// = N * K (+ 4 N of scales) per launch, half of the BF16 GEMV's.
//
// Kernels:
//  * quantize_w_kernel: the load-time weight quantization (one CTA per row).
//  * gemv_i8_tma_kernel (one activation row): a producer warp streams groups
//    of whole int8 rows through a shared-memory ring (cp.async.bulk +
//    mbarriers) from before griddepcontrol.wait; the consumer warps
//    quantize the activation row themselves (optionally RMSNorm'd first:
//    the same row in every CTA, from registers), keep their K segment of it
//    in registers and reduce with dp4a and warp shuffles.
//  * quantize_x_kernel + gemv_i8_gen_kernel: up to 16 activation rows (the
//    multi-stream step): the rows are quantized once into global memory,
//    then one warp per weight row serves every stream.
#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kQThreads = 256;            // quantize kernels
constexpr int kI8Consumers = 8;           // consumer warps of gemv_i8_tma
constexpr int kI8Threads = (kI8Consumers + 1) * kWarp;
constexpr int kI8Ring = 96 * 1024;        // ring bytes per CTA (two CTAs per SM)
constexpr int kI8MaxStages = 12;
constexpr int kI8MaxPerThread = 64;       // activation values per consumer thread (K <= 16384)
constexpr int kI8GenThreads = 256;

// f32::round (halves away from zero), clamped to +-127, as an integer.
__device__ __forceinline__ int q8(float v) {
  float r = roundf(v);
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return int(r);
}

__device__ __forceinline__ void i8_consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kI8Consumers * kWarp) : "memory");
}

// A barrier among the NT threads that run the quantization: the whole CTA
// (NT = kQThreads), or the consumer warps of gemv_i8_tma (named barrier 1;
// its producer warp never joins).
template <int NT>
__device__ __forceinline__ void q_sync() {
  if constexpr (NT == kI8Consumers * kWarp && kI8Threads != NT) i8_consumer_sync();
  else __syncthreads();
}

template <int NT>
__device__ __forceinline__ float block_max_q(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  q_sync<NT>();
  float m = 0.0f;
  for (int i = 0; i < NT / kWarp; ++i) m = fmaxf(m, red[i]);
  q_sync<NT>();
  return m;
}

// ---------------------------------------------------------------------------
// WMat::quantize_i8 of a BF16 [N, K] matrix (values widened exactly).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kQThreads) quantize_w_kernel(const uint16_t* __restrict__ w,
                                                               int64_t N, int K,
                                                               int8_t* __restrict__ q,
                                                               float* __restrict__ scales) {
  __shared__ float red[kQThreads / kWarp];
  for (int64_t r = blockIdx.x; r < N; r += gridDim.x) {
    const uint16_t* row = w + r * K;
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += kQThreads) m = fmaxf(fabsf(bf16f(row[k])), m);
    m = block_max_q<kQThreads>(m, red);
    const float sc = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    if (threadIdx.x == 0) scales[r] = sc;
    int8_t* qr = q + r * K;
    for (int k = threadIdx.x; k < K; k += kQThreads) qr[k] = int8_t(q8(__fdiv_rn(bf16f(row[k]), sc)));
  }
}

// RMSNorm scaling of one element in either of the reference's orders.
__device__ __forceinline__ float nscale(float v, float inv, float w, int mode) {
  if (mode == 0) return (v * inv) * w;
  return v * (inv * w);
}

// quantize_row_i8 (with an optional RMSNorm first) of one K-row, by the
// block of `nthreads` threads that calls it.  Thread t holds the values
// k = 4 (t + nthreads i) .. +3 in registers; the quantized row goes to
// xq (shared or global), its scale is returned.
template <int NT>
__device__ __forceinline__ float quantize_row_block(const float* __restrict__ x,
                                                    const float* __restrict__ norm_w, float eps,
                                                    int mode, int K, int8_t* xq, float* red) {
  constexpr int NV = kI8MaxPerThread / 4;
  float4 v[NV];
  float ss = 0.0f, m = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (threadIdx.x + NT * i);
    if (k < K) {
      v[i] = *reinterpret_cast<const float4*>(x + k);
      ss = fmaf(v[i].x, v[i].x, ss);
      ss = fmaf(v[i].y, v[i].y, ss);
      ss = fmaf(v[i].z, v[i].z, ss);
      ss = fmaf(v[i].w, v[i].w, ss);
    }
  }
  if (norm_w) {
    ss = warp_sum(ss);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = ss;
    q_sync<NT>();
    float tot = 0.0f;
    for (int i = 0; i < NT / kWarp; ++i) tot += red[i];
    q_sync<NT>();
    const float inv = 1.0f / sqrtf(tot / float(K) + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int k = 4 * (threadIdx.x + NT * i);
      if (k < K) {
        const float4 g = *reinterpret_cast<const float4*>(norm_w + k);
        v[i] = make_float4(nscale(v[i].x, inv, g.x, mode), nscale(v[i].y, inv, g.y, mode),
                           nscale(v[i].z, inv, g.z, mode), nscale(v[i].w, inv, g.w, mode));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (threadIdx.x + NT * i);
    if (k < K)
      m = fmaxf(fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))), m);
  }
  m = block_max_q<NT>(m, red);
  const float s = m == 0.0f ? 0.0f : __fdiv_rn(m, 127.0f);
  const float inv = m == 0.0f ? 0.0f : __fdiv_rn(1.0f, s);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = 4 * (threadIdx.x + NT * i);
    if (k < K) {
      const uint32_t b0 = uint32_t(q8(__fmul_rn(v[i].x, inv))) & 0xffu;
      const uint32_t b1 = uint32_t(q8(__fmul_rn(v[i].y, inv))) & 0xffu;
      const uint32_t b2 = uint32_t(q8(__fmul_rn(v[i].z, inv))) & 0xffu;
      const uint32_t b3 = uint32_t(q8(__fmul_rn(v[i].w, inv))) & 0xffu;
      *reinterpret_cast<uint32_t*>(xq + k) = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
  }
  return s;
}

__device__ __forceinline__ int dp16(const int4& w, const int4& x, int acc) {
  acc = __dp4a(w.x, x.x, acc);
  acc = __dp4a(w.y, x.y, acc);
  acc = __dp4a(w.z, x.z, acc);
  return __dp4a(w.w, x.w, acc);
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// y = f32(dot) * s * scale, the reference's order.
__device__ __forceinline__ float i8_out(int dot, float s, float scale) {
  return __fmul_rn(__fmul_rn(__int2float_rn(dot), s), scale);
}

// ---------------------------------------------------------------------------
// gemv_i8_tma: one activation row.  Groups of rpc = 8 / ksplit row slots
// (SwiGLU: rpc / 2 gate rows then as many up rows); warp w takes K segment
// w % ksplit (chunks x 512 int8) of row slot w / ksplit.
// ---------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(kI8Threads, 2)
    gemv_i8_tma_kernel(const GemvI8Args a, const int chunks, const int ksplit) {
  extern __shared__ __align__(128) uint8_t dsm[];  // ring | xq (K bytes)
  __shared__ __align__(8) uint64_t full[kI8MaxStages];
  __shared__ __align__(8) uint64_t empty[kI8MaxStages];
  __shared__ int part[2][kI8Consumers];
  __shared__ float red[kI8Consumers];
  __shared__ volatile int abort_s[2];

  constexpr bool SW = EPI == EPI_SWIGLU;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  const int rpc = kI8Consumers / ksplit;
  const int rpg = SW ? rpc / 2 : rpc;
  const int64_t ngroups = (a.N + rpg - 1) / rpg;
  const uint32_t stage_bytes = uint32_t(rpc) * uint32_t(K);
  const int nst = min(kI8MaxStages, int(kI8Ring / stage_bytes));
  uint8_t* ring = dsm;
  int8_t* xq = reinterpret_cast<int8_t*>(dsm + size_t(nst) * stage_bytes);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kI8Consumers);
    }
    abort_s[0] = abort_s[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kI8Consumers) {
    // ---- producer: weights only, so no wait on the previous kernel ----
    if (lane == 0) {
      int it = 0;
      for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
        const int s = it % nst;
        const uint32_t ph = (it / nst) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          abort_s[0] = abort_s[1] = 1;
          if (a.err) atomicExch(a.err, 2);
          break;
        }
        uint8_t* dst = ring + size_t(s) * stage_bytes;
        const int64_t r0 = g * rpg;
        const int64_t nr = min(int64_t(rpg), a.N - r0);
        const uint32_t bytes = uint32_t(nr) * uint32_t(K);
        mbar_expect_tx(&full[s], SW ? 2 * bytes : bytes);
        bulk_g2s(dst, a.q + r0 * K, bytes, &full[s]);
        if (SW) bulk_g2s(dst + size_t(rpg) * K, a.q2 + r0 * K, bytes, &full[s]);
      }
    }
    return;
  }

  // ---- consumers: quantize the activation row (every CTA alike) ----
  pdl_wait();
  const float xs = quantize_row_block<kI8Consumers * kWarp>(a.x, a.norm_w, a.eps, a.norm_mode, K,
                                                            xq, red);
  i8_consumer_sync();
  const int ks = warp % ksplit, slot = warp / ksplit;
  const int kbase = ks * chunks * 512;
  int4 xr[8];
#pragma unroll
  for (int c = 0; c < 8; ++c)
    if (c < chunks) xr[c] = *reinterpret_cast<const int4*>(xq + kbase + c * 512 + lane * 16);
  const bool need_sync = ksplit > 1 || SW;
  int it = 0;
  for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
    const int s = it % nst;
    const uint32_t ph = (it / nst) & 1;
    const int64_t r0 = g * rpg;
    const int rslot = SW ? slot % rpg : slot;
    const bool valid = r0 + rslot < a.N;
    int acc = 0;
    const bool ok = !(abort_s[0] | abort_s[1]) && mbar_wait(&full[s], ph);
    if (ok) {
      if (valid) {
        const int8_t* wr = reinterpret_cast<const int8_t*>(ring + size_t(s) * stage_bytes) +
                           size_t(slot) * K + kbase + lane * 16;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          if (c < chunks) acc = dp16(*reinterpret_cast<const int4*>(wr + c * 512), xr[c], acc);
      }
    } else if (lane == 0) {
      abort_s[it & 1] = 1;
      if (a.err) atomicExch(a.err, 2);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    acc = warp_sum_i(acc);
    bool stop = !ok;
    if (need_sync) {
      if (lane == 0) part[it & 1][warp] = acc;
      i8_consumer_sync();
      stop = abort_s[it & 1] != 0;
    }
    if (!stop && lane == 0 && ks == 0 && valid && (!SW || slot < rpg)) {
      if (ksplit > 1)
        for (int j = 1; j < ksplit; ++j) acc += part[it & 1][warp + j];
      const int64_t r = r0 + rslot;
      const float v = i8_out(acc, xs, a.scales[r]);
      if (SW) {
        int up = 0;
        for (int j = 0; j < ksplit; ++j) up += part[it & 1][(slot + rpg) * ksplit + j];
        const float u = i8_out(up, xs, a.scales2[r]);
        a.y[r] = v / (1.0f + expf(-v)) * u;
      } else if (EPI == EPI_ADD) {
        a.y[r] += v;
      } else {
        a.y[r] = v;
      }
    }
    if (stop) break;
  }
}

// ---------------------------------------------------------------------------
// Multi-stream: quantize_x (one CTA per activation row) then gemv_i8_gen.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kQThreads) quantize_x_kernel(const GemvI8Args a) {
  __shared__ float red[kQThreads / kWarp];
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const float s = quantize_row_block<kQThreads>(a.x + size_t(m) * a.K, a.norm_w, a.eps,
                                                a.norm_mode, a.K, a.xq + size_t(m) * a.K, red);
  if (threadIdx.x == 0) a.xs[m] = s;
}

template <int EPI>
__global__ void __launch_bounds__(kI8GenThreads) gemv_i8_gen_kernel(const GemvI8Args a) {
  constexpr bool SW = EPI == EPI_SWIGLU;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K, M = a.M;
  pdl_trigger();
  pdl_wait();
  for (int64_t r = int64_t(blockIdx.x) * (kI8GenThreads / kWarp) + warp; r < a.N;
       r += int64_t(gridDim.x) * (kI8GenThreads / kWarp)) {
    int acc[kMaxStreams], acc2[kMaxStreams];
#pragma unroll
    for (int m = 0; m < kMaxStreams; ++m) acc[m] = acc2[m] = 0;
    const int8_t* wr = a.q + r * K;
    const int8_t* wr2 = SW ? a.q2 + r * K : nullptr;
    for (int k = lane * 16; k < K; k += 512) {
      const uint4 wu = ld_stream(wr + k);
      const int4 w = make_int4(int(wu.x), int(wu.y), int(wu.z), int(wu.w));
      int4 w2 = make_int4(0, 0, 0, 0);
      if (SW) {
        const uint4 u2 = ld_stream(wr2 + k);
        w2 = make_int4(int(u2.x), int(u2.y), int(u2.z), int(u2.w));
      }
#pragma unroll
      for (int m = 0; m < kMaxStreams; ++m) {
        if (m < M) {
          const int4 xv = __ldg(reinterpret_cast<const int4*>(a.xq + size_t(m) * K + k));
          acc[m] = dp16(w, xv, acc[m]);
          if (SW) acc2[m] = dp16(w2, xv, acc2[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < kMaxStreams; ++m) {
      if (m < M) {
        const int d = warp_sum_i(acc[m]);
        const int d2 = SW ? warp_sum_i(acc2[m]) : 0;
        if (lane == 0) {
          float* y = a.y + size_t(m) * a.ldy;
          const float xs = a.xs[m];
          const float v = i8_out(d, xs, a.scales[r]);
          if (SW) {
            const float u = i8_out(d2, xs, a.scales2[r]);
            y[r] = v / (1.0f + expf(-v)) * u;
          } else if (EPI == EPI_ADD) {
            y[r] += v;
          } else {
            y[r] = v;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Prefill: q widened to BF16 (exact: |q| <= 127) for the tensor-core GEMM,
// then the row scale (y = acc * scale[o], matmul_batch_w_into's writeback,
// src/tensor.rs:736-738), optionally added into the residual.
// ---------------------------------------------------------------------------
__global__ void widen_i8_kernel(const int8_t* __restrict__ q, size_t n, uint16_t* __restrict__ out) {
  for (size_t i = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n;
       i += size_t(gridDim.x) * blockDim.x * 4) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(q + i);
    uint16_t b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f = float(int8_t(u >> (8 * j)));
      b[j] = uint16_t(__float_as_uint(f) >> 16);  // exact: an integer of at most 7 bits
    }
    *reinterpret_cast<uint2*>(out + i) =
        make_uint2(uint32_t(b[0]) | (uint32_t(b[1]) << 16), uint32_t(b[2]) | (uint32_t(b[3]) << 16));
  }
}

__global__ void scale_rows_kernel(const float* __restrict__ acc, int64_t T, int64_t N,
                                  const float* __restrict__ scales, float* __restrict__ y,
                                  int64_t ldy, int add) {
  const int64_t total = T * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / N, o = i % N;
    const float v = __fmul_rn(acc[t * N + o], scales[o]);
    if (add) y[t * ldy + o] += v;
    else y[t * ldy + o] = v;
  }
}

// K split over 1, 2, 4 or 8 warps: a warp's segment is a whole number of
// 512-byte chunks, at most 8.
int i8_ksplit(int K) {
  for (int ks = 1; ks <= 8; ks *= 2)
    if (K % (ks * 512) == 0 && K / (ks * 512) <= 8) return ks;
  return 0;
}

}  // namespace

bool gemv_i8_tma_ok(int K, int M) {
  if (M != 1 || K % 512 || K > kI8MaxPerThread * kI8Consumers * kWarp) return false;
  const int ks = i8_ksplit(K);
  return ks > 0 && (kI8Consumers / ks) * K <= kI8Ring;
}

cudaError_t launch_quantize_w_i8(const uint16_t* w, int64_t N, int K, int8_t* q, float* scales,
                                 cudaStream_t s) {
  if (N <= 0 || K <= 0) return cudaErrorInvalidValue;
  const int grid = int(std::min<int64_t>(N, 16384));
  quantize_w_kernel<<<grid, kQThreads, 0, s>>>(w, N, K, q, scales);
  return cudaGetLastError();
}

cudaError_t launch_gemv_i8(const GemvI8Args& args, GemvEpi epi, cudaStream_t s, bool pdl,
                           int num_sms) {
  GemvI8Args a = args;
  if (a.M < 1 || a.M > kMaxStreams || a.K % 16 || a.K > kI8MaxPerThread * kQThreads ||
      (epi != EPI_STORE && epi != EPI_ADD && epi != EPI_SWIGLU))
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (gemv_i8_tma_ok(a.K, a.M)) {
    const int ks = i8_ksplit(a.K);
    const int chunks = a.K / (ks * 512);
    const uint32_t stage = uint32_t(kI8Consumers / ks) * uint32_t(a.K);
    const int nst = std::min(kI8MaxStages, int(kI8Ring / stage));
    cfg.gridDim = dim3(2 * num_sms);
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = size_t(nst) * stage + size_t(a.K);
    switch (epi) {
      case EPI_ADD: return cudaLaunchKernelEx(&cfg, gemv_i8_tma_kernel<EPI_ADD>, a, chunks, ks);
      case EPI_SWIGLU:
        return cudaLaunchKernelEx(&cfg, gemv_i8_tma_kernel<EPI_SWIGLU>, a, chunks, ks);
      default: return cudaLaunchKernelEx(&cfg, gemv_i8_tma_kernel<EPI_STORE>, a, chunks, ks);
    }
  }
  if (!a.xq || !a.xs) return cudaErrorInvalidValue;
  cfg.gridDim = dim3(a.M);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = 0;
  TMG_CUDA_TRY(cudaLaunchKernelEx(&cfg, quantize_x_kernel, a));
  cfg.gridDim = dim3(4 * num_sms);
  cfg.blockDim = dim3(kI8GenThreads);
  switch (epi) {
    case EPI_ADD: return cudaLaunchKernelEx(&cfg, gemv_i8_gen_kernel<EPI_ADD>, a);
    case EPI_SWIGLU: return cudaLaunchKernelEx(&cfg, gemv_i8_gen_kernel<EPI_SWIGLU>, a);
    default: return cudaLaunchKernelEx(&cfg, gemv_i8_gen_kernel<EPI_STORE>, a);
  }
}

cudaError_t launch_widen_i8(const int8_t* q, size_t n, uint16_t* out, cudaStream_t s) {
  if (n % 4) return cudaErrorInvalidValue;
  const size_t blocks = std::min<size_t>((n / 4 + 255) / 256, 4096);
  widen_i8_kernel<<<unsigned(std::max<size_t>(blocks, 1)), 256, 0, s>>>(q, n, out);
  return cudaGetLastError();
}

cudaError_t launch_scale_rows(const float* acc, int64_t T, int64_t N, const float* scales, float* y,
                              int64_t ldy, bool add, cudaStream_t s) {
  const int64_t total = T * N;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 8192);
  scale_rows_kernel<<<unsigned(std::max<int64_t>(blocks, 1)), 256, 0, s>>>(acc, T, N, scales, y, ldy,
                                                                           add ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t gemv_i8_prepare() {
  TMG_CUDA_TRY(set_carveout(gemv_i8_tma_kernel<EPI_STORE>, kI8Ring + 16384));
  TMG_CUDA_TRY(set_carveout(gemv_i8_tma_kernel<EPI_ADD>, kI8Ring + 16384));
  TMG_CUDA_TRY(set_carveout(gemv_i8_tma_kernel<EPI_SWIGLU>, kI8Ring + 16384));
  TMG_CUDA_TRY(set_carveout(gemv_i8_gen_kernel<EPI_STORE>));
  TMG_CUDA_TRY(set_carveout(gemv_i8_gen_kernel<EPI_ADD>));
  TMG_CUDA_TRY(set_carveout(gemv_i8_gen_kernel<EPI_SWIGLU>));
  TMG_CUDA_TRY(set_carveout(quantize_x_kernel));
  return set_carveout(quantize_w_kernel);
}

}  // namespace tmg
