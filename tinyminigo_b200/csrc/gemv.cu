// Decode GEMV: the BF16 matrix-vector products of forward_token
// (matmul_w_into, src/tensor.rs:331-460; call sites src/model.rs:417-419,
// 461, 471-472, 476, 489).
//
// y[n] = sum_k x[k] * W[n, k] with W BF16 [N, K] row-major, f32 math.  The
// reference runs 8-lane AVX2 FMA chains per row; here every weight byte is
// streamed once from HBM with 16-byte L1-bypassing loads, widened to f32 in
// registers (exact), and reduced with warp shuffles.  This kernel family is
// HBM-bound: algorithmic bytes = 2 * N * K per launch (+ 4 * K of x).
//
// Two kernels:
//  * gemv_m1: one activation row (the batch-1 token loop).  K % 256 == 0.
//    A CTA of 8 warps stages x (normalised when fused with RMSNorm) in
//    shared memory in a permuted layout that makes every warp's float4
//    reads conflict-free; each warp owns a fixed K segment (split-K inside
//    the CTA when N is small) and two output rows per task, so a lane keeps
//    2 x chunks x 16 B of weights in flight.  The first task's weights are
//    requested before griddepcontrol.wait, overlapping the previous kernel.
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

// ---------------------------------------------------------------------------
// gemv_m1
// ---------------------------------------------------------------------------
template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_m1_kernel(const GemvArgs a, const int chunks, const int ksplit) {
  extern __shared__ float4 xs4[];  // K floats, permuted
  __shared__ float red[kWarps];
  __shared__ float part[kWarps][2];
  __shared__ unsigned long long best_s[kWarps];
  __shared__ bool last_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = a.K;
  const int ks = warp % ksplit, slot = warp / ksplit, rpc = kWarps / ksplit;
  constexpr int RPT = (EPI == EPI_SWIGLU) ? 1 : 2;
  const int64_t ngroups = (a.N + int64_t(rpc) * RPT - 1) / (int64_t(rpc) * RPT);
  const int kbase = ks * chunks * 256;

  pdl_trigger();

  uint4 w0[8], w1[8];
  auto issue = [&](int64_t g) {
    const int64_t r0 = (EPI == EPI_SWIGLU) ? g * rpc + slot : (g * rpc + slot) * 2;
    const bool v0 = r0 < a.N;
    const bool v1 = (EPI == EPI_SWIGLU) ? v0 : (r0 + 1 < a.N);
    const uint16_t* p0 = a.w + r0 * K + kbase + lane * 8;
    const uint16_t* p1 = (EPI == EPI_SWIGLU) ? a.w2 + r0 * K + kbase + lane * 8 : p0 + K;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (c < chunks) {
        w0[c] = v0 ? ld_stream(p0 + c * 256) : make_uint4(0, 0, 0, 0);
        w1[c] = v1 ? ld_stream(p1 + c * 256) : make_uint4(0, 0, 0, 0);
      }
    }
  };

  int64_t g = blockIdx.x;
  if (g < ngroups) issue(g);  // independent of earlier kernels
  pdl_wait();

  // ---- prologue: x (or rmsnorm(x)) into shared memory ---------------------
  const int k8_step = kThreads * 8;
  float inv = 1.0f;
  const uint16_t* erow = nullptr;
  if (PRO == PRO_EMBED_NORM) erow = a.embed + size_t(a.tokens[0]) * K;
  auto load8 = [&](int k8, float* v) {
    if (PRO == PRO_EMBED_NORM) {
      uint4 u = *reinterpret_cast<const uint4*>(erow + k8);
      v[0] = bf16lo(u.x); v[1] = bf16hi(u.x); v[2] = bf16lo(u.y); v[3] = bf16hi(u.y);
      v[4] = bf16lo(u.z); v[5] = bf16hi(u.z); v[6] = bf16lo(u.w); v[7] = bf16hi(u.w);
    } else {
      float4 p = *reinterpret_cast<const float4*>(a.x + k8);
      float4 q = *reinterpret_cast<const float4*>(a.x + k8 + 4);
      v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
      v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
    }
  };
  if (PRO != PRO_NONE) {
    float ss = 0.f;
    for (int k8 = threadIdx.x * 8; k8 < K; k8 += k8_step) {
      float v[8];
      load8(k8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    }
    ss = block_sum<kThreads>(ss, red);
    inv = 1.0f / sqrtf(ss / float(K) + a.eps);
  }
  for (int k8 = threadIdx.x * 8; k8 < K; k8 += k8_step) {
    float v[8];
    load8(k8, v);
    if (PRO == PRO_EMBED_NORM && blockIdx.x == 0) {
      *reinterpret_cast<float4*>(a.x_out + k8) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(a.x_out + k8 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    if (PRO != PRO_NONE) {
      float4 wa = *reinterpret_cast<const float4*>(a.norm_w + k8);
      float4 wb = *reinterpret_cast<const float4*>(a.norm_w + k8 + 4);
      v[0] = norm_scale(v[0], inv, wa.x, a.norm_mode); v[1] = norm_scale(v[1], inv, wa.y, a.norm_mode);
      v[2] = norm_scale(v[2], inv, wa.z, a.norm_mode); v[3] = norm_scale(v[3], inv, wa.w, a.norm_mode);
      v[4] = norm_scale(v[4], inv, wb.x, a.norm_mode); v[5] = norm_scale(v[5], inv, wb.y, a.norm_mode);
      v[6] = norm_scale(v[6], inv, wb.z, a.norm_mode); v[7] = norm_scale(v[7], inv, wb.w, a.norm_mode);
    }
    const int i4 = ((k8 >> 8) * 2) * 32 + ((k8 & 255) >> 3);
    xs4[i4] = make_float4(v[0], v[1], v[2], v[3]);
    xs4[i4 + 32] = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();

  // ---- main loop over row groups -----------------------------------------
  unsigned long long best = 0ull;
  const int cg0 = kbase >> 8;
  for (; g < ngroups; g += gridDim.x) {
    if (g != blockIdx.x) issue(g);
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (c < chunks) {
        const float4 xa = xs4[((cg0 + c) * 2) * 32 + lane];
        const float4 xb = xs4[((cg0 + c) * 2 + 1) * 32 + lane];
        acc0 = dot8(xa, xb, w0[c], acc0);
        acc1 = dot8(xa, xb, w1[c], acc1);
      }
    }
    acc0 = warp_sum(acc0);
    acc1 = warp_sum(acc1);
    if (ksplit > 1) {
      if (lane == 0) {
        part[warp][0] = acc0;
        part[warp][1] = acc1;
      }
      __syncthreads();
      if (ks == 0 && lane == 0)
        for (int j = 1; j < ksplit; ++j) {
          acc0 += part[warp + j][0];
          acc1 += part[warp + j][1];
        }
    }
    if (ks == 0 && lane == 0) {
      if (EPI == EPI_SWIGLU) {
        const int64_t r = g * rpc + slot;
        if (r < a.N) {
          const float sg = acc0 / (1.0f + expf(-acc0));
          a.y[r] = sg * acc1;
        }
      } else {
        const int64_t r0 = (g * rpc + slot) * 2;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int64_t r = r0 + i;
          const float v = i == 0 ? acc0 : acc1;
          if (r < a.N) {
            if (EPI == EPI_ADD) a.y[r] += v;
            else a.y[r] = v;
            if (EPI == EPI_HEAD_ARGMAX) {
              unsigned long long kk = argmax_key(v, uint32_t(r));
              best = kk > best ? kk : best;
            }
          }
        }
      }
    }
    if (ksplit > 1) __syncthreads();
  }

  if (EPI == EPI_HEAD_ARGMAX) {
    best = warp_max_u64(best);
    if (lane == 0) best_s[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = best_s[0];
      for (int w = 1; w < kWarps; ++w) b = best_s[w] > b ? best_s[w] : b;
      a.am_part[blockIdx.x] = b;
    }
  }
  if (EPI == EPI_HEAD || EPI == EPI_HEAD_ARGMAX)
    head_finish<EPI == EPI_HEAD_ARGMAX>(a, 1, best_s, &last_s);
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

bool use_m1(const GemvArgs& a) {
  return a.M == 1 && a.K % 256 == 0 && a.K <= 256 * 8 * 8 &&
         (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
         (a.w2 == nullptr || (reinterpret_cast<uintptr_t>(a.w2) & 15) == 0) &&
         (a.x == nullptr || (reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
}

// Split-K factor inside a CTA: the smallest that gives every warp of a
// 2-CTA-per-SM grid a task, with at most 8 chunks of 256 per warp.
void pick_split(const GemvArgs& a, GemvEpi epi, int num_sms, int* chunks, int* ksplit) {
  const int tc = a.K / 256;
  const int64_t tasks1 = (epi == EPI_SWIGLU) ? a.N : (a.N + 1) / 2;
  const int64_t want = int64_t(num_sms) * 2 * kWarps;
  int best = -1;
  for (int ks : {1, 2, 4, 8}) {
    if (tc % ks != 0 || tc / ks > 8) continue;
    best = ks;
    if (tasks1 * ks >= want) break;
  }
  *ksplit = best;
  *chunks = best > 0 ? tc / best : 0;
}

int m1_grid(const GemvArgs& a, GemvEpi epi, int ksplit, int num_sms) {
  const int rpc = kWarps / ksplit;
  const int64_t per = int64_t(rpc) * ((epi == EPI_SWIGLU) ? 1 : 2);
  const int64_t ngroups = (a.N + per - 1) / per;
  return int(std::min<int64_t>(ngroups, int64_t(num_sms) * 2));
}

int gen_grid(const GemvArgs& a, int num_sms) {
  const int64_t need = (a.N + kWarps - 1) / kWarps;
  return int(std::min<int64_t>(need, int64_t(num_sms) * 4));
}

constexpr int kMaxM1Smem = 256 * 8 * 8 * sizeof(float);  // K <= 16384

template <int PRO, int EPI>
cudaError_t set_m1_attr() {
  return cudaFuncSetAttribute(gemv_m1_kernel<PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kMaxM1Smem);
}

template <int PRO>
cudaError_t set_m1_attrs() {
  TMG_CUDA_TRY((set_m1_attr<PRO, EPI_STORE>()));
  TMG_CUDA_TRY((set_m1_attr<PRO, EPI_ADD>()));
  TMG_CUDA_TRY((set_m1_attr<PRO, EPI_SWIGLU>()));
  TMG_CUDA_TRY((set_m1_attr<PRO, EPI_HEAD>()));
  return set_m1_attr<PRO, EPI_HEAD_ARGMAX>();
}

template <int PRO, int EPI>
cudaError_t launch_m1(const GemvArgs& a, cudaStream_t s, bool pdl, int num_sms, int chunks,
                      int ksplit) {
  auto kern = gemv_m1_kernel<PRO, EPI>;
  const size_t smem = size_t(a.K) * sizeof(float);
  const int grid = m1_grid(a, GemvEpi(EPI), ksplit, num_sms);
  return launch_k(kern, dim3(grid), dim3(kThreads), smem, s, pdl, a, chunks, ksplit);
}

template <int PRO>
cudaError_t launch_m1_epi(const GemvArgs& a, GemvEpi epi, cudaStream_t s, bool pdl, int num_sms,
                          int chunks, int ksplit) {
  switch (epi) {
    case EPI_STORE: return launch_m1<PRO, EPI_STORE>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_ADD: return launch_m1<PRO, EPI_ADD>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_SWIGLU: return launch_m1<PRO, EPI_SWIGLU>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_HEAD: return launch_m1<PRO, EPI_HEAD>(a, s, pdl, num_sms, chunks, ksplit);
    case EPI_HEAD_ARGMAX: return launch_m1<PRO, EPI_HEAD_ARGMAX>(a, s, pdl, num_sms, chunks, ksplit);
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
  TMG_CUDA_TRY(set_m1_attrs<PRO_NONE>());
  TMG_CUDA_TRY(set_m1_attrs<PRO_NORM>());
  return set_m1_attrs<PRO_EMBED_NORM>();
}

bool gemv_fused_ok(const GemvArgs& a, GemvEpi epi) {
  if (!use_m1(a)) return false;
  int chunks, ks;
  pick_split(a, epi, 148, &chunks, &ks);
  return ks > 0;
}

int gemv_grid(const GemvArgs& a, GemvEpi epi, int num_sms) {
  if (use_m1(a)) {
    int chunks, ks;
    pick_split(a, epi, num_sms, &chunks, &ks);
    if (ks > 0) return m1_grid(a, epi, ks, num_sms);
  }
  return gen_grid(a, num_sms);
}

cudaError_t launch_gemv(const GemvArgs& a, GemvPro pro, GemvEpi epi, cudaStream_t s, bool pdl,
                        int num_sms) {
  if (a.N <= 0 || a.K <= 0 || a.M < 1 || a.M > kMaxStreams) return cudaErrorInvalidValue;
  if (use_m1(a)) {
    int chunks, ks;
    pick_split(a, epi, num_sms, &chunks, &ks);
    if (ks > 0) {
      switch (pro) {
        case PRO_NONE: return launch_m1_epi<PRO_NONE>(a, epi, s, pdl, num_sms, chunks, ks);
        case PRO_NORM: return launch_m1_epi<PRO_NORM>(a, epi, s, pdl, num_sms, chunks, ks);
        case PRO_EMBED_NORM:
          return launch_m1_epi<PRO_EMBED_NORM>(a, epi, s, pdl, num_sms, chunks, ks);
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
