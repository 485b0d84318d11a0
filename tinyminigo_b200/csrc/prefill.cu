// Prefill building blocks (forward_seq, src/model.rs:503-590) and small
// helpers: embedding gather (515-519), RMSNorm rows (rms_norm_batch /
// rms_norm_into, src/tensor.rs:946-977), SwiGLU (577-580), a SIMT GEMM for
// shapes the tensor-core GEMM does not take, and argmax rows
// (src/tensor.rs:1063-1073).
#include <math.h>

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

__global__ void embed_kernel(const uint16_t* __restrict__ embed, const uint32_t* __restrict__ tok,
                             int h, float* __restrict__ x) {
  const int64_t t = blockIdx.x;
  const uint16_t* row = embed + size_t(tok[t]) * h;
  for (int k = threadIdx.x; k < h; k += blockDim.x) x[t * h + k] = bf16f(row[k]);
}

template <int NT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const float* __restrict__ x,
                                                     const float* __restrict__ w, float eps,
                                                     int64_t n, int mode, float* __restrict__ out) {
  __shared__ float red[NT / 32];
  const int64_t r = blockIdx.x;
  const float* xr = x + r * n;
  float ss = 0.f;
  for (int64_t k = threadIdx.x; k < n; k += NT) ss = fmaf(xr[k], xr[k], ss);
  ss = block_sum<NT>(ss, red);
  const float inv = 1.0f / sqrtf(ss / float(n) + eps);
  for (int64_t k = threadIdx.x; k < n; k += NT) {
    const float v = xr[k];
    if (mode == 0) {
      const float t = v * inv;
      out[r * n + k] = t * w[k];
    } else {
      const float f = inv * w[k];
      out[r * n + k] = v * f;
    }
  }
}

// rmsnorm_kernel's mode 1 (rms_norm_batch) written straight as the next
// GEMM's BF16 hi/lo operands: the same value v * (inv * w[k]), then hi =
// bf16(value), lo = bf16(value - hi) as the split kernels compute them.
template <int NT>
__global__ void __launch_bounds__(NT) rmsnorm_split_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ w, float eps,
                                                           int64_t n, __nv_bfloat16* __restrict__ hi,
                                                           __nv_bfloat16* __restrict__ lo) {
  __shared__ float red[NT / 32];
  const int64_t r = blockIdx.x;
  const float* xr = x + r * n;
  float ss = 0.f;
  for (int64_t k = threadIdx.x; k < n; k += NT) ss = fmaf(xr[k], xr[k], ss);
  ss = block_sum<NT>(ss, red);
  const float inv = 1.0f / sqrtf(ss / float(n) + eps);
  for (int64_t k = threadIdx.x; k < n; k += NT) {
    const float f = inv * w[k];
    const float v = xr[k] * f;
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[r * n + k] = h;
    lo[r * n + k] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t n,
                              float* __restrict__ out) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float gv = g[i];
    const float sg = gv / (1.0f + expf(-gv));
    out[i] = sg * u[i];
  }
}

// 64x64 output tile, K step 16, 256 threads each computing 4x4.
constexpr int BM = 64, BN = 64, BK = 16;
__global__ void __launch_bounds__(256) gemm_simt_kernel(const float* __restrict__ x,
                                                        const uint16_t* __restrict__ w, int64_t T,
                                                        int64_t N, int64_t K, float* __restrict__ y,
                                                        int64_t ldy, int accumulate) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, c = i % BK;
      const int64_t gm = m0 + r, gk = k0 + c;
      xs[c][r] = (gm < T && gk < K) ? x[gm * K + gk] : 0.f;
      const int64_t gn = n0 + r;
      ws[c][r] = (gn < N && gk < K) ? bf16f(w[gn * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < T && gn < N) {
        if (accumulate) y[gm * ldy + gn] += acc[i][j];
        else y[gm * ldy + gn] = acc[i][j];
      }
    }
}

__global__ void argmax_rows_kernel(const float* __restrict__ logits, int64_t V,
                                   uint32_t* __restrict__ out) {
  __shared__ unsigned long long red[32];
  const float* l = logits + size_t(blockIdx.x) * V;
  unsigned long long b = 0ull;
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    unsigned long long k = argmax_key(l[i], uint32_t(i));
    b = k > b ? k : b;
  }
  b = warp_max_u64(b);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < int(blockDim.x >> 5); ++i) b = red[i] > b ? red[i] : b;
    out[blockIdx.x] = argmax_key_index(b);
  }
}

__global__ void set_pos_kernel(StreamState st, int m, int32_t v) { st.pos[m] = v; }

__global__ void add_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    dst[i] += src[i];
}

// One CTA per stream.
__global__ void step_end_kernel(StreamState st, const float* __restrict__ logits, int64_t V) {
  __shared__ unsigned long long red[32];
  const int m = blockIdx.x;
  unsigned long long b = 0ull;
  if (logits) {
    const float* l = logits + size_t(m) * V;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
      unsigned long long k = argmax_key(l[i], uint32_t(i));
      b = k > b ? k : b;
    }
    b = warp_max_u64(b);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (logits)
      for (int i = 1; i < int(blockDim.x >> 5); ++i) b = red[i] > b ? red[i] : b;
    if (!st.done[m]) st.pos[m] += 1;
    if (logits) finish_step(st, m, argmax_key_index(b));
  }
}

}  // namespace

cudaError_t prefill_prepare() {
  TMG_CUDA_TRY(set_carveout(embed_kernel));
  TMG_CUDA_TRY(set_carveout(rmsnorm_kernel<256>));
  TMG_CUDA_TRY(set_carveout(rmsnorm_split_kernel<256>));
  TMG_CUDA_TRY(set_carveout(swiglu_kernel));
  TMG_CUDA_TRY(set_carveout(gemm_simt_kernel));
  TMG_CUDA_TRY(set_carveout(argmax_rows_kernel));
  TMG_CUDA_TRY(set_carveout(set_pos_kernel));
  TMG_CUDA_TRY(set_carveout(add_kernel));
  return set_carveout(step_end_kernel);
}

cudaError_t launch_embed(const uint16_t* embed, const uint32_t* tokens, int64_t T, int h, float* x,
                         cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  embed_kernel<<<unsigned(T), 256, 0, s>>>(embed, tokens, h, x);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int64_t n, int64_t rows,
                           int mode, float* out, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  rmsnorm_kernel<256><<<unsigned(rows), 256, 0, s>>>(x, w, eps, n, mode, out);
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_split(const float* x, const float* w, float eps, int64_t n,
                                 int64_t rows, uint16_t* hi, uint16_t* lo, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  rmsnorm_split_kernel<256><<<unsigned(rows), 256, 0, s>>>(
      x, w, eps, n, reinterpret_cast<__nv_bfloat16*>(hi), reinterpret_cast<__nv_bfloat16*>(lo));
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const float* gate, const float* up, int64_t n, float* out,
                          cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  swiglu_kernel<<<unsigned(blocks), 256, 0, s>>>(gate, up, n, out);
  return cudaGetLastError();
}

cudaError_t launch_gemm_simt(const float* x, const uint16_t* w, int64_t T, int64_t N, int64_t K,
                             float* y, int64_t ldy, bool accumulate, cudaStream_t s) {
  if (T <= 0 || N <= 0) return cudaSuccess;
  dim3 grid(unsigned((N + BN - 1) / BN), unsigned((T + BM - 1) / BM));
  gemm_simt_kernel<<<grid, 256, 0, s>>>(x, w, T, N, K, y, ldy, accumulate ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const float* logits, int64_t V, int rows, uint32_t* out,
                               cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  argmax_rows_kernel<<<rows, 1024, 0, s>>>(logits, V, out);
  return cudaGetLastError();
}

cudaError_t launch_add(const float* src, float* dst, int64_t n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
  add_kernel<<<unsigned(blocks), 256, 0, s>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_step_end(StreamState st, int M, const float* logits, int64_t V,
                            cudaStream_t s) {
  step_end_kernel<<<M, 1024, 0, s>>>(st, logits, V);
  return cudaGetLastError();
}

cudaError_t launch_set_pos(StreamState st, int m, int32_t value, cudaStream_t s) {
  set_pos_kernel<<<1, 1, 0, s>>>(st, m, value);
  return cudaGetLastError();
}

}  // namespace tmg
