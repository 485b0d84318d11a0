// Decode GEMV: the BF16 matrix-vector products of forward_token
// (matmul_w_into, src/tensor.rs:331-460; call sites src/model.rs:417-419,
// 461, 471-472, 476, 489).
//
// y[n] = sum_k x[k] * W[n, k] with W BF16 [N, K] row-major, f32 math.  The
// reference runs 8-lane AVX2 FMA chains per row; here every weight byte is
// streamed once from HBM, widened to f32 in registers (exact), and reduced
// with warp shuffles.  HBM-bound: algorithmic bytes = 2 * N * K per launch
// (+ 4 * K of x).
//
// Two kernels:
//  * gemv_tma (one activation row: the batch-1 token loop; K % 256 == 0).
//    One persistent CTA per SM: a producer warp streams groups of whole
//    weight rows (contiguous, <= 32 KB) with cp.async.bulk into a 3-stage
//    shared-memory ring guarded by mbarriers, starting before
//    griddepcontrol.wait so the stream overlaps the previous kernel; eight
//    consumer warps keep their K segment of x (normalised when RMSNorm is
//    fused) in registers and reduce each row with warp shuffles, split-K
//    across warps when K > 2048.  The 96 KB ring leaves room for the next
//    kernel's CTA on the same SM.
//  * gemv_gen: up to 16 activation rows, any K (the multi-stream step and
//    odd shapes).  One row per warp task, x read through L1.
//
// Epilogues fuse the residual add (src/model.rs:462-464, 477-479), SwiGLU
// (473-475: gate / (1 + exp(-gate)) * up), and for the LM head the end of a
// forward (pos += 1) plus, in greedy mode, the argmax of generate
// (src/tensor.rs:1063-1073) with generate's bookkeeping.
#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / kWarp;
constexpr int kConsumerWarps = 8;
constexpr int kTmaThreads = (kConsumerWarps + 1) * kWarp;
constexpr int kRingBytes = 96 * 1024;  // bytes in flight per SM (HBM latency x bandwidth share)
constexpr int kMaxStages = 12;
constexpr int kStageMax = 32 * 1024;  // bytes of one ring stage

__device__ __forceinline__ float dot8(const float4& xa, const float4& xb, const uint4& w,
                                      float acc) {
  acc = fmaf(xa.x, bf16lo(w.x), acc);
  acc = fmaf(xa.y, bf16hi(w.x), acc);
  acc = fmaf(xa.z, bf16lo(w.y), acc);
  acc = fmaf(xa.w, bf16hi(w.y), acc);
  acc = fmaf(xb.x, bf16lo(w.z), acc);
  acc = fmaf(xb.y, bf16hi(w.z), acc);
  acc = fmaf(xb.z, bf16lo(w.w), acc);
  acc = fmaf(xb.w, bf16hi(w.w), acc);
  return acc;
}

// Eight independent accumulators (one per element of a 16-byte chunk): the
// FMA chains stay 'chunks' long instead of 8 * chunks, so a warp issues
// back to back instead of waiting on its own previous FMA.
__device__ __forceinline__ void fma8(const float4& xa, const float4& xb, const uint4& w,
                                     float (&s)[8]) {
  s[0] = fmaf(xa.x, bf16lo(w.x), s[0]);
  s[1] = fmaf(xa.y, bf16hi(w.x), s[1]);
  s[2] = fmaf(xa.z, bf16lo(w.y), s[2]);
  s[3] = fmaf(xa.w, bf16hi(w.y), s[3]);
  s[4] = fmaf(xb.x, bf16lo(w.z), s[4]);
  s[5] = fmaf(xb.y, bf16hi(w.z), s[5]);
  s[6] = fmaf(xb.z, bf16lo(w.w), s[6]);
  s[7] = fmaf(xb.w, bf16hi(w.w), s[7]);
}
__device__ __forceinline__ float sum8(const float (&s)[8]) {
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

// RMSNorm scaling of one element, in either of the reference's orders.
__device__ __forceinline__ float norm_scale(float v, float inv, float w, int mode) {
  if (mode == 0) {
    float t = v * inv;  // rms_norm_into: v * inv * w
    return t * w;
  }
  float f = inv * w;  // rms_norm_batch: v *= inv * w
  return v * f;
}

// End of a forward for the streams of this launch: the last CTA to finish
// advances pos (one appended position) and, with argmax, reduces the
// per-CTA candidates and records the token.  Ticket-based, no waiting.
template <bool ARGMAX>
__device__ void head_finish(const GemvArgs& a, int M, unsigned long long* red_s, bool* last_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int t = atomicAdd(a.ticket, 1u);
    *last_s = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!*last_s) return;
  __threadfence();
  for (int m = 0; m < M; ++m) {
    unsigned long long b = 0ull;
    if (ARGMAX) {
      for (int i = threadIdx.x; i < gridDim.x; i += blockDim.x) {
        unsigned long long v = __ldcg(&a.am_part[size_t(i) * M + m]);
        b = v > b ? v : b;
      }
      b = warp_max_u64(b);
      if ((threadIdx.x & 31) == 0) red_s[threadIdx.x >> 5] = b;
      __syncthreads();
      if (threadIdx.x == 0)
        for (int w = 1; w < int(blockDim.x >> 5); ++w) b = red_s[w] > b ? red_s[w] : b;
    }
    if (threadIdx.x == 0) {
      if (!a.st.done[m]) a.st.pos[m] += 1;
      if (ARGMAX) finish_step(a.st, m, argmax_key_index(b));
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *a.ticket = 0u;
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * kWarp) : "memory");
}

// ---------------------------------------------------------------------------
// gemv_tma
//
// Row groups: `rpc` = 8 / ksplit row slots per group; warp w owns K segment
// ks = w % ksplit (chunks x 256 elements) of row slot w / ksplit.  With
// SwiGLU the first rpc/2 slots are gate rows and the rest the up rows of
// the same outputs.  Group g is one contiguous block of rows per matrix,
// loaded by one (two for SwiGLU) bulk copies.
// ---------------------------------------------------------------------------
// Two CTAs fit on one SM (registers and shared memory), so under
// programmatic dependent launch the next GEMV's producer starts streaming
// while this one drains.
template <int PRO, int EPI>
__global__ void __launch_bounds__(kTmaThreads, 2)
    gemv_tma_kernel(const GemvArgs a, const int chunks, const int ksplit) {
  extern __shared__ __align__(128) uint8_t dsm[];  // ring | x (K floats, with a norm)
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ float part[2][kConsumerWarps];
  __shared__ float ssq[kConsumerWarps];
  __shared__ unsigned long long best_s[kConsumerWarps + 1];
  __shared__ volatile int abort_s[2];  // set by a wait that gave up, per iteration parity
  __shared__ bool last_s;

  constexpr bool SW = EPI == EPI_SWIGLU;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  const int rpc = kConsumerWarps / ksplit;
  const int rpg = SW ? rpc / 2 : rpc;  // output rows per group
  const int64_t ngroups = (a.N + rpg - 1) / rpg;
  const size_t row_bytes = size_t(K) * 2;
  const uint32_t stage_bytes = uint32_t(rpc * row_bytes);
  const int nst = min(kMaxStages, int(kRingBytes / stage_bytes));
  uint8_t* ring = dsm;
  float* xs = reinterpret_cast<float*>(dsm + nst * stage_bytes);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    abort_s[0] = abort_s[1] = 0;
    mbar_fence_init();
    trace_mark(a.trace, 0);
  }
  __syncthreads();
  pdl_trigger();

  unsigned long long best = 0ull;
  if (warp == kConsumerWarps) {
    // ---- producer: weights only, so no wait on the previous kernel ----
    if (lane == 0) {
      int it = 0;
      for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
        const int s = it % nst;
        const uint32_t ph = (it / nst) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          abort_s[0] = abort_s[1] = 1;  // consumers stop waiting for stages
          if (a.err) atomicExch(a.err, 2);
          break;
        }
        uint8_t* dst = ring + s * stage_bytes;
        const int64_t r0 = g * rpg;
        const int64_t nr = min(int64_t(rpg), a.N - r0);
        const uint32_t bytes = uint32_t(nr * row_bytes);
        mbar_expect_tx(&full[s], SW ? 2 * bytes : bytes);
        bulk_g2s(dst, a.w + r0 * K, bytes, &full[s]);
        if (SW) bulk_g2s(dst + rpg * row_bytes, a.w2 + r0 * K, bytes, &full[s]);
      }
    }
  } else {
    // ---- consumers ----
    pdl_wait();
    if (threadIdx.x == 0) {
      trace_mark(a.trace, 1);
      trace_mark(a.trace, 2);
    }
    const int ks = warp % ksplit, slot = warp / ksplit;
    const int kbase = ks * chunks * 256;
    // with a norm: stage x (embedding row or activations) in shared memory,
    // since the sum of squares spans all of K
    const uint16_t* erow = PRO == PRO_EMBED_NORM ? a.embed + size_t(a.tokens[0]) * K : nullptr;
    float ss = 0.f;
    for (int k8 = threadIdx.x * 8; PRO != PRO_NONE && k8 < K; k8 += kConsumerWarps * kWarp * 8) {
      float4 p, q;
      if (PRO == PRO_EMBED_NORM) {
        const uint4 u = *reinterpret_cast<const uint4*>(erow + k8);
        p = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
        q = make_float4(bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w));
        if (blockIdx.x == 0) {
          *reinterpret_cast<float4*>(a.x_out + k8) = p;
          *reinterpret_cast<float4*>(a.x_out + k8 + 4) = q;
        }
      } else {
        p = *reinterpret_cast<const float4*>(a.x + k8);
        q = *reinterpret_cast<const float4*>(a.x + k8 + 4);
      }
      *reinterpret_cast<float4*>(xs + k8) = p;
      *reinterpret_cast<float4*>(xs + k8 + 4) = q;
      if (PRO != PRO_NONE) {
        ss = fmaf(p.x, p.x, ss); ss = fmaf(p.y, p.y, ss); ss = fmaf(p.z, p.z, ss); ss = fmaf(p.w, p.w, ss);
        ss = fmaf(q.x, q.x, ss); ss = fmaf(q.y, q.y, ss); ss = fmaf(q.z, q.z, ss); ss = fmaf(q.w, q.w, ss);
      }
    }
    float inv = 1.0f;
    if (PRO != PRO_NONE) {
      ss = warp_sum(ss);
      if (lane == 0) ssq[warp] = ss;
      consumer_sync();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) tot += ssq[w];
      inv = 1.0f / sqrtf(tot / float(K) + a.eps);
    }
    // this warp's K segment, in registers (without a norm, straight from
    // global memory: the rows of x are produced by the previous kernel)
    const float* xsrc = PRO == PRO_NONE ? a.x : xs;
    float4 xa[8], xb[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (c < chunks) {
        const int k = kbase + c * 256 + lane * 8;
        float4 p = *reinterpret_cast<const float4*>(xsrc + k);
        float4 q = *reinterpret_cast<const float4*>(xsrc + k + 4);
        if (PRO != PRO_NONE) {
          const float4 wa = __ldg(reinterpret_cast<const float4*>(a.norm_w + k));
          const float4 wb = __ldg(reinterpret_cast<const float4*>(a.norm_w + k + 4));
          const int md = a.norm_mode;
          p = make_float4(norm_scale(p.x, inv, wa.x, md), norm_scale(p.y, inv, wa.y, md),
                          norm_scale(p.z, inv, wa.z, md), norm_scale(p.w, inv, wa.w, md));
          q = make_float4(norm_scale(q.x, inv, wb.x, md), norm_scale(q.y, inv, wb.y, md),
                          norm_scale(q.z, inv, wb.z, md), norm_scale(q.w, inv, wb.w, md));
        }
        xa[c] = p;
        xb[c] = q;
      }
    }
    const bool need_sync = ksplit > 1 || SW;
    int it = 0;
    for (int64_t g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
      const int s = it % nst;
      const uint32_t ph = (it / nst) & 1;
      const int64_t r0 = g * rpg;
      const int rslot = SW ? slot % rpg : slot;
      const bool valid = r0 + rslot < a.N;
      float acc = 0.f;
      const bool ok = !(abort_s[0] | abort_s[1]) && mbar_wait(&full[s], ph);
      if (ok) {
        if (valid) {
          const uint16_t* wr = reinterpret_cast<const uint16_t*>(ring + s * stage_bytes +
                                                                 slot * row_bytes) +
                               kbase + lane * 8;
          float sacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c < chunks) fma8(xa[c], xb[c], *reinterpret_cast<const uint4*>(wr + c * 256), sacc);
          acc = sum8(sacc);
        }
      } else if (lane == 0) {
        abort_s[it & 1] = 1;
        if (a.err) atomicExch(a.err, 2);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      acc = warp_sum(acc);
      bool stop = !ok;
      if (need_sync) {
        // every consumer warp passes this barrier each iteration, so the
        // stop decision (this iteration's flag) is the same for all of them
        if (lane == 0) part[it & 1][warp] = acc;
        consumer_sync();
        stop = abort_s[it & 1] != 0;
      }
      if (!stop && lane == 0 && ks == 0 && valid && (!SW || slot < rpg)) {
        if (ksplit > 1)
          for (int j = 1; j < ksplit; ++j) acc += part[it & 1][warp + j];
        const int64_t r = r0 + rslot;
        if (SW) {
          float up = 0.f;
          for (int j = 0; j < ksplit; ++j) up += part[it & 1][(slot + rpg) * ksplit + j];
          const float sg = acc / (1.0f + expf(-acc));
          a.y[r] = sg * up;
        } else if (EPI == EPI_ADD) {
          a.y[r] += acc;
        } else {
          a.y[r] = acc;
          if (EPI == EPI_HEAD_ARGMAX) {
            const unsigned long long kk = argmax_key(acc, uint32_t(r));
            best = kk > best ? kk : best;
          }
        }
      }
      if (stop) break;
    }
  }

  if (EPI == EPI_HEAD_ARGMAX) {
    best = warp_max_u64(best);
    if (lane == 0) best_s[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = best_s[0];
      for (int w = 1; w <= kConsumerWarps; ++w) b = best_s[w] > b ? best_s[w] : b;
      a.am_part[blockIdx.x] = b;
    }
  }
  if (EPI == EPI_HEAD || EPI == EPI_HEAD_ARGMAX)
    head_finish<EPI == EPI_HEAD_ARGMAX>(a, 1, best_s, &last_s);
  if (threadIdx.x == 0) trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------------------
// gemv_gen: M <= 16 rows, any K; x read through L1.  PRO_NONE only (the
// host runs the embedding / norm kernels first).
// ---------------------------------------------------------------------------
template <int EPI, bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_gen_kernel(const GemvArgs a) {
  __shared__ unsigned long long best_s[kWarps][kMaxStreams];
  __shared__ unsigned long long red_s[kWarps];
  __shared__ bool last_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K, M = a.M;
  const int64_t ntasks = a.N;
  pdl_trigger();
  pdl_wait();

  unsigned long long best[kMaxStreams];
#pragma unroll
  for (int m = 0; m < kMaxStreams; ++m) best[m] = 0ull;

  for (int64_t r = int64_t(blockIdx.x) * kWarps + warp; r < ntasks;
       r += int64_t(gridDim.x) * kWarps) {
    float acc[kMaxStreams], acc2[kMaxStreams];
#pragma unroll
    for (int m = 0; m < kMaxStreams; ++m) acc[m] = acc2[m] = 0.f;
    const uint16_t* wr = a.w + r * K;
    const uint16_t* wr2 = (EPI == EPI_SWIGLU) ? a.w2 + r * K : nullptr;
    if (VEC) {
      for (int k = lane * 8; k < K; k += 256) {
        const uint4 w = ld_stream(wr + k);
        uint4 w2 = make_uint4(0, 0, 0, 0);
        if (EPI == EPI_SWIGLU) w2 = ld_stream(wr2 + k);
#pragma unroll
        for (int m = 0; m < kMaxStreams; ++m) {
          if (m < M) {
            const float4 xa = __ldg(reinterpret_cast<const float4*>(a.x + size_t(m) * K + k));
            const float4 xb = __ldg(reinterpret_cast<const float4*>(a.x + size_t(m) * K + k + 4));
            acc[m] = dot8(xa, xb, w, acc[m]);
            if (EPI == EPI_SWIGLU) acc2[m] = dot8(xa, xb, w2, acc2[m]);
          }
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
        const float w = bf16f(wr[k]);
        const float w2 = (EPI == EPI_SWIGLU) ? bf16f(wr2[k]) : 0.f;
#pragma unroll
        for (int m = 0; m < kMaxStreams; ++m) {
          if (m < M) {
            const float xv = __ldg(a.x + size_t(m) * K + k);
            acc[m] = fmaf(xv, w, acc[m]);
            if (EPI == EPI_SWIGLU) acc2[m] = fmaf(xv, w2, acc2[m]);
          }
        }
      }
    }
#pragma unroll
    for (int m = 0; m < kMaxStreams; ++m) {
      if (m < M) {
        const float v = warp_sum(acc[m]);
        const float v2 = (EPI == EPI_SWIGLU) ? warp_sum(acc2[m]) : 0.f;
        if (lane == 0) {
          float* y = a.y + size_t(m) * a.ldy;
          if (EPI == EPI_SWIGLU) {
            const float sg = v / (1.0f + expf(-v));
            y[r] = sg * v2;
          } else if (EPI == EPI_ADD) {
            y[r] += v;
          } else {
            y[r] = v;
          }
          if (EPI == EPI_HEAD_ARGMAX) {
            unsigned long long kk = argmax_key(v, uint32_t(r));
            best[m] = kk > best[m] ? kk : best[m];
          }
        }
      }
    }
  }
  if (EPI == EPI_HEAD_ARGMAX) {
    if (lane == 0)
      for (int m = 0; m < kMaxStreams; ++m) best_s[warp][m] = best[m];
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kWarps; ++w) b = best_s[w][threadIdx.x] > b ? best_s[w][threadIdx.x] : b;
      a.am_part[size_t(blockIdx.x) * M + threadIdx.x] = b;
    }
  }
  if (EPI == EPI_HEAD || EPI == EPI_HEAD_ARGMAX)
    head_finish<EPI == EPI_HEAD_ARGMAX>(a, M, red_s, &last_s);
}


template <typename Kern>
cudaError_t launch_k(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                     const GemvArgs& a, int c, int ks) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a, c, ks);
}

template <typename Kern>
cudaError_t launch_k2(Kern kern, dim3 grid, dim3 block, cudaStream_t s, bool pdl,
                      const GemvArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

bool use_tma(const GemvArgs& a) {
  return a.M == 1 && a.K % 256 == 0 && a.K <= 256 * 8 * 8 &&
         (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
         (a.w2 == nullptr || (reinterpret_cast<uintptr_t>(a.w2) & 15) == 0) &&
         (a.x == nullptr || (reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
}

// Split-K factor: segments of at most 8 x 256 elements per warp, a stage of
// at most 32 KB, and (when possible) at least 4 row groups per SM.
void pick_split(const GemvArgs& a, GemvEpi epi, int num_sms, int* chunks, int* ksplit) {
  const int tc = a.K / 256;
  int best = -1;
  for (int ks : {1, 2, 4, 8}) {
    if (tc % ks != 0 || tc / ks > 8) continue;
    const int rpc = kConsumerWarps / ks;
    if (epi == EPI_SWIGLU && rpc < 2) continue;
    if (size_t(rpc) * a.K * 2 > size_t(kStageMax)) continue;
    best = ks;
    const int rpg = epi == EPI_SWIGLU ? rpc / 2 : rpc;
    if ((a.N + rpg - 1) / rpg >= int64_t(num_sms) * 4) break;
  }
  *ksplit = best;
  *chunks = best > 0 ? tc / best : 0;
}

int tma_grid(const GemvArgs& a, GemvEpi epi, int ksplit, int num_sms) {
  const int rpc = kConsumerWarps / ksplit;
  const int rpg = epi == EPI_SWIGLU ? rpc / 2 : rpc;
  const int64_t ngroups = (a.N + rpg - 1) / rpg;
  return int(std::min<int64_t>(ngroups, int64_t(num_sms)));
}

int gen_grid(const GemvArgs& a, int num_sms) {
  const int64_t need = (a.N + kWarps - 1) / kWarps;
  return int(std::min<int64_t>(need, int64_t(num_sms) * 4));
}

// ring (as many whole stages as fit kRingBytes) + x staging when normed
size_t tma_smem(const GemvArgs& a, int ksplit, GemvPro pro) {
  const size_t stage = size_t(kConsumerWarps / ksplit) * a.K * 2;
  const size_t nst = std::min<size_t>(kMaxStages, kRingBytes / stage);
  return nst * stage + (pro != PRO_NONE ? size_t(a.K) * 4 : 0);
}

constexpr int kMaxTmaSmem = kRingBytes + 256 * 8 * 8 * 4;  // ring + x (K <= 16384)

template <int PRO, int EPI>
cudaError_t set_tma_attr() {
  TMG_CUDA_TRY((set_carveout(gemv_gen_kernel<EPI, true>)));
  TMG_CUDA_TRY((set_carveout(gemv_gen_kernel<EPI, false>)));
  return set_carveout(gemv_tma_kernel<PRO, EPI>, kMaxTmaSmem);
}

template <int PRO>
cudaError_t set_tma_attrs() {
  TMG_CUDA_TRY((set_tma_attr<PRO, EPI_STORE>()));
  TMG_CUDA_TRY((set_tma_attr<PRO, EPI_ADD>()));
  TMG_CUDA_TRY((set_tma_attr<PRO, EPI_SWIGLU>()));
  TMG_CUDA_TRY((set_tma_attr<PRO, EPI_HEAD>()));
  return set_tma_attr<PRO, EPI_HEAD_ARGMAX>();
}

template <int PRO, int EPI>
cudaError_t launch_tma(const GemvArgs& a, cudaStream_t s, bool pdl, int num_sms, int chunks,
                       int ksplit) {
  const int grid = tma_grid(a, GemvEpi(EPI), ksplit, num_sms);
  return launch_k(gemv_tma_kernel<PRO, EPI>, dim3(grid), dim3(kTmaThreads),
                  tma_smem(a, ksplit, GemvPro(PRO)),
                  s, pdl, a, chunks, ksplit);
}

template <int PRO>
cudaError_t launch_tma_epi(const GemvArgs& a, GemvEpi epi, cudaStream_t s, bool pdl, int num_sms,
                           int chunks, int ksplit) {
  switch (epi) {
    case EPI_STORE: return launch_tma<PRO, EPI_STORE>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_ADD: return launch_tma<PRO, EPI_ADD>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_SWIGLU: return launch_tma<PRO, EPI_SWIGLU>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_HEAD: return launch_tma<PRO, EPI_HEAD>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_HEAD_ARGMAX: return launch_tma<PRO, EPI_HEAD_ARGMAX>(a, s, pdl, num_sms, chunks, ksplit);
  }
  return cudaErrorInvalidValue;
}

template <bool VEC>
cudaError_t launch_gen(const GemvArgs& a, GemvEpi epi, cudaStream_t s, bool pdl, int num_sms) {
  const dim3 grid(gen_grid(a, num_sms)), block(kThreads);
  switch (epi) {
    case EPI_STORE: return launch_k2(gemv_gen_kernel<EPI_STORE, VEC>, grid, block, s, pdl, a);
    case EPI_ADD: return launch_k2(gemv_gen_kernel<EPI_ADD, VEC>, grid, block, s, pdl, a);
    case EPI_SWIGLU: return launch_k2(gemv_gen_kernel<EPI_SWIGLU, VEC>, grid, block, s, pdl, a);
    case EPI_HEAD: return launch_k2(gemv_gen_kernel<EPI_HEAD, VEC>, grid, block, s, pdl, a);
    case EPI_HEAD_ARGMAX:
      return launch_k2(gemv_gen_kernel<EPI_HEAD_ARGMAX, VEC>, grid, block, s, pdl, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t gemv_prepare() {
  TMG_CUDA_TRY(set_tma_attrs<PRO_NONE>());
  TMG_CUDA_TRY(set_tma_attrs<PRO_NORM>());
  return set_tma_attrs<PRO_EMBED_NORM>();
}

bool gemv_fused_ok(const GemvArgs& a, GemvEpi epi) {
  if (!use_tma(a)) return false;
  int chunks, ks;
  pick_split(a, epi, 148, &chunks, &ks);
  return ks > 0;
}

int gemv_grid(const GemvArgs& a, GemvEpi epi, int num_sms) {
  if (use_tma(a)) {
    int chunks, ks;
    pick_split(a, epi, num_sms, &chunks, &ks);
    if (ks > 0) return tma_grid(a, epi, ks, num_sms);
  }
  return gen_grid(a, num_sms);
}

cudaError_t launch_gemv(const GemvArgs& a, GemvPro pro, GemvEpi epi, cudaStream_t s, bool pdl,
                        int num_sms) {
  if (a.N <= 0 || a.K <= 0 || a.M < 1 || a.M > kMaxStreams) return cudaErrorInvalidValue;
  if (use_tma(a)) {
    int chunks, ks;
    pick_split(a, epi, num_sms, &chunks, &ks);
    if (ks > 0) {
      switch (pro) {
        case PRO_NONE: return launch_tma_epi<PRO_NONE>(a, epi, s, pdl, num_sms, chunks, ks);
        case PRO_NORM: return launch_tma_epi<PRO_NORM>(a, epi, s, pdl, num_sms, chunks, ks);
        case PRO_EMBED_NORM:
          return launch_tma_epi<PRO_EMBED_NORM>(a, epi, s, pdl, num_sms, chunks, ks);
      }
    }
  }
  if (pro != PRO_NONE) return cudaErrorInvalidValue;  // host must pre-normalise
  const bool vec = a.K % 8 == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
                   (a.w2 == nullptr || (reinterpret_cast<uintptr_t>(a.w2) & 15) == 0) &&
                   (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  return vec ? launch_gen<true>(a, epi, s, pdl, num_sms) : launch_gen<false>(a, epi, s, pdl, num_sms);
}

}  // namespace tmg
