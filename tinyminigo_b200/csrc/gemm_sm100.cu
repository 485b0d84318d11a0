// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// matmul_batch_w_into (src/tensor.rs:573-792): Y[T, N] = X[T, K] . W[N, K]^T
// with X f32 activations and W BF16 weights.  The reference accumulates in
// f32; a plain BF16 MMA on the activations would keep only 8 mantissa bits,
// so X is split into two BF16 operands, X = Xhi + Xlo (Xhi = bf16(X), Xlo =
// bf16(X - Xhi), ~16 bits together), and every K step issues two MMAs into
// the same f32 TMEM accumulator: Xhi.W and Xlo.W.  W is exact in BF16.
//
// Persistent: one CTA per SM walks the output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... (128 x bn, bn <= 256 chosen per launch so the
// tiles fill the SMs evenly; consecutive tiles share their 128 rows of X).
// An optional second (W, Y) segment extends N (gate and up from one split
// of their common input in one launch).  Roles:
//   warp 0      TMA producer: per 64-wide K block, Xhi / Xlo [128 x 64] and
//               W [bn x 64] tiles (128-byte swizzle) into a 3-stage ring;
//   warp 1      allocates 2 x 256 TMEM columns (two accumulators), issues
//               tcgen05.mma (one elected lane; M=128, N=bn, K=16 per
//               instruction) into the tile's accumulator, commits each stage
//               back to the producer and the finished tile to the epilogue;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 16 columns at a time, then
//               store (or add into) Y in f32, and hand the accumulator back,
//               so tile i's epilogue overlaps tile i+1's MMAs.
// Every mbarrier wait is bounded; a wait that gives up sets the error word
// and the CTA skips the rest of its work (the host reports TMG_ERR_TIMEOUT).
// Single-GPU code: every CTA loads its own tiles; no peer memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB (a narrower tile uses its first bn rows)
constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int kThreadsG = 192;
constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators

// The launch: rows T of X; output columns [0, N1) from W1 into Y1 and
// [N1, N1 + N2) from W2 into Y2 (N2 = 0: one segment).
struct GemmTcArgs {
  float* y1;
  int64_t ldy1;
  float* y2;
  int64_t ldy2;
  int T, K, N1, N2;
  int bn;              // tile width (multiple of 16, <= 256)
  int nt1, nt2, mt;    // tiles along N1, N2 and T
  int accumulate;
  int32_t* err;
  // SwiGLU mode: each tile holds bn/2 gate rows (W1) and the same bn/2 up
  // rows (W2) of the columns [n0, n0 + bn/2), and the epilogue writes
  // act = g / (1 + exp(-g)) * u straight as BF16 hi/lo parts (the next GEMM's
  // operands) instead of y1 / y2.
  int swiglu;
  uint16_t* act_hi;
  uint16_t* act_lo;
  int64_t ld_act;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO), the
// second 16-byte K chunk 16 B away (LBO = 1), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3fff);
  d |= uint64_t(1) << 16;                 // LBO (16 B units)
  d |= uint64_t(1024 >> 4) << 32;         // SBO
  d |= uint64_t(1) << 46;                 // version
  d |= uint64_t(2) << 61;                 // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: BF16 x BF16 -> F32, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t idesc_for(int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(bn >> 3) << 17) |
         (uint32_t(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                     uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15},"
      " [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                   const __grid_constant__ CUtensorMap map_w1,
                   const __grid_constant__ CUtensorMap map_w2, const GemmTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2] a tile's accumulator is complete
  uint64_t* acc_empty = acc_full + 2;    // [2] the epilogue has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ volatile int failed;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (a.K + BK - 1) / BK;
  const int ntn = a.nt1 + a.nt2;
  const int tiles = a.mt * ntn;
  const uint32_t b_bytes = uint32_t(a.bn) * BK * 2;
  const uint32_t idesc = idesc_for(a.bn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // TMA producer: every tile's K blocks through the ring
    int it = 0;
    for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
      const int m0 = (t / ntn) * BM, nt = t % ntn;
      const bool seg2 = nt >= a.nt1;
      const int n0 = a.swiglu ? nt * (a.bn / 2) : (seg2 ? nt - a.nt1 : nt) * a.bn;
      const CUtensorMap* mw = seg2 ? &map_w2 : &map_w1;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1)) {
          atomicExch(a.err, 2);
          failed = 1;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_expect_tx(&full[s], 2 * A_BYTES + b_bytes);
        tma_load_2d(st, &map_hi, &full[s], kb * BK, m0);
        tma_load_2d(st + A_BYTES, &map_lo, &full[s], kb * BK, m0);
        if (a.swiglu) {  // gate rows, then the same up rows
          tma_load_2d(st + 2 * A_BYTES, &map_w1, &full[s], kb * BK, n0);
          tma_load_2d(st + 2 * A_BYTES + (a.bn / 2) * BK * 2, &map_w2, &full[s], kb * BK, n0);
        } else {
          tma_load_2d(st + 2 * A_BYTES, mw, &full[s], kb * BK, n0);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: tile i into accumulator i & 1
    int it = 0, tl = 0;
    for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (!mbar_wait(&acc_empty[buf], ((tl >> 1) & 1) ^ 1)) {
        atomicExch(a.err, 2);
        failed = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t acc_t = tmem + uint32_t(buf * BN);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_hi = smem_u32(smem + s * STAGE_BYTES);
        const uint32_t a_lo = a_hi + A_BYTES;
        const uint32_t b = a_hi + 2 * A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t db = umma_desc(b + k * 32);
          umma(acc_t, umma_desc(a_hi + k * 32), db, idesc, (kb | k) != 0);
          umma(acc_t, umma_desc(a_lo + k * 32), db, idesc, 1);
        }
        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      if (!ok) {
        atomicExch(a.err, 2);
        failed = 1;
        break;
      }
      umma_commit(&acc_full[buf]);
    }
  } else if (warp >= 2) {
    // epilogue: warp w reads TMEM lanes 32 * (w % 4) ...
    const int q = warp & 3;
    int tl = 0;
    for (int t = blockIdx.x; t < tiles && !failed; t += gridDim.x, ++tl) {
      const int buf = tl & 1;
      if (!mbar_wait(&acc_full[buf], (tl >> 1) & 1)) {
        atomicExch(a.err, 2);
        failed = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (t / ntn) * BM, nt = t % ntn;
      const int row = m0 + q * 32 + lane;
      const uint32_t tacc = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * BN);
      if (a.swiglu) {
        // columns [0, bn/2) hold gate, [bn/2, bn) up, for act columns n0 ..
        const int half = a.bn / 2, n0 = nt * half;
        for (int c = 0; c < half; c += 16) {
          float g[16], u[16];
          tmem_ld16(tacc + uint32_t(c), g);
          tmem_ld16(tacc + uint32_t(half + c), u);
          if (row < a.T && n0 + c < a.N1) {
            uint32_t hw[8], lw[8];
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              // SwiGLU (src/model.rs:473-475) as swiglu_split4_kernel computes it
              const float a0 = (g[i] / (1.0f + expf(-g[i]))) * u[i];
              const float a1 = (g[i + 1] / (1.0f + expf(-g[i + 1]))) * u[i + 1];
              const __nv_bfloat16 h0 = __float2bfloat16_rn(a0), h1 = __float2bfloat16_rn(a1);
              const __nv_bfloat16 l0 = __float2bfloat16_rn(a0 - __bfloat162float(h0));
              const __nv_bfloat16 l1 = __float2bfloat16_rn(a1 - __bfloat162float(h1));
              hw[i / 2] = uint32_t(__bfloat16_as_ushort(h0)) | (uint32_t(__bfloat16_as_ushort(h1)) << 16);
              lw[i / 2] = uint32_t(__bfloat16_as_ushort(l0)) | (uint32_t(__bfloat16_as_ushort(l1)) << 16);
            }
            const int64_t o = int64_t(row) * a.ld_act + n0 + c;
            if (n0 + c + 16 <= a.N1) {
              uint4* ph = reinterpret_cast<uint4*>(a.act_hi + o);
              uint4* pl = reinterpret_cast<uint4*>(a.act_lo + o);
              ph[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
              ph[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
              pl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
              pl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (n0 + c + i < a.N1) {
                  a.act_hi[o + i] = uint16_t(hw[i / 2] >> (16 * (i & 1)));
                  a.act_lo[o + i] = uint16_t(lw[i / 2] >> (16 * (i & 1)));
                }
            }
          }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      const bool seg2 = nt >= a.nt1;
      const int n0 = (seg2 ? nt - a.nt1 : nt) * a.bn;
      const int N = seg2 ? a.N2 : a.N1;
      float* y = seg2 ? a.y2 : a.y1;
      const int64_t ldy = seg2 ? a.ldy2 : a.ldy1;
      for (int c = 0; c < a.bn; c += 16) {
        float v[16];
        tmem_ld16(tacc + uint32_t(c), v);
        if (row < a.T && n0 + c < N) {
          float* yr = y + int64_t(row) * ldy + n0 + c;
          if (n0 + c + 16 <= N && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              float4* p = reinterpret_cast<float4*>(yr + i);
              float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              if (a.accumulate) {
                const float4 old = *p;
                o.x += old.x;
                o.y += old.y;
                o.z += old.z;
                o.w += old.w;
              }
              *p = o;
            }
          } else {
            for (int i = 0; i < 16; ++i)
              if (n0 + c + i < N) yr[i] = a.accumulate ? yr[i] + v[i] : v[i];
          }
        }
      }
      // the accumulator goes back to the MMA warp
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

__global__ void split_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ hi,
                             __nv_bfloat16* __restrict__ lo) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float v = x[i];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
  }
}

// Four elements per thread: a float4 in, the hi and lo halves out as 8-byte
// words (element 0 in the low bits).
__device__ __forceinline__ void split4(float4 v, uint2* hi, uint2* lo) {
  const float a[4] = {v.x, v.y, v.z, v.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat16 hb = __float2bfloat16_rn(a[e]);
    h[e] = __bfloat16_as_ushort(hb);
    l[e] = __bfloat16_as_ushort(__float2bfloat16_rn(a[e] - __bfloat162float(hb)));
  }
  *hi = make_uint2(h[0] | h[1] << 16, h[2] | h[3] << 16);
  *lo = make_uint2(l[0] | l[1] << 16, l[2] | l[3] << 16);
}

__global__ void split4_kernel(const float4* __restrict__ x, int64_t n4, uint2* __restrict__ hi,
                              uint2* __restrict__ lo) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4;
       i += int64_t(gridDim.x) * blockDim.x)
    split4(x[i], hi + i, lo + i);
}

// SwiGLU (src/model.rs:473-475, the same arithmetic as swiglu_kernel:
// g / (1 + exp(-g)) * u) written straight as the down GEMM's hi/lo operands.
__global__ void swiglu_split4_kernel(const float4* __restrict__ g, const float4* __restrict__ u,
                                     int64_t n4, uint2* __restrict__ hi, uint2* __restrict__ lo) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float4 gv = g[i], uv = u[i];
    float4 a;
    a.x = (gv.x / (1.0f + expf(-gv.x))) * uv.x;
    a.y = (gv.y / (1.0f + expf(-gv.y))) * uv.y;
    a.z = (gv.z / (1.0f + expf(-gv.z))) * uv.z;
    a.w = (gv.w / (1.0f + expf(-gv.w))) * uv.w;
    split4(a, hi + i, lo + i);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D bf16 [rows, K] row-major map with a (64 x box_rows) box, 128B swizzle.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool gemm_tc_supported(int64_t K, const void* w) {
  return K % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t gemm_tc_prepare() {
  TMG_CUDA_TRY(set_carveout(split_kernel));
  TMG_CUDA_TRY(set_carveout(split4_kernel));
  TMG_CUDA_TRY(set_carveout(swiglu_split4_kernel));
  return set_carveout(gemm_tc_kernel, SMEM_BYTES);
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }
}  // namespace

cudaError_t launch_split(const float* x, int64_t n, uint16_t* hi, uint16_t* lo, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (n % 4 == 0 && aligned16(x) && aligned8(hi) && aligned8(lo)) {
    const int64_t n4 = n / 4;
    const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 148 * 16);
    split4_kernel<<<unsigned(blocks), 256, 0, s>>>(reinterpret_cast<const float4*>(x), n4,
                                                   reinterpret_cast<uint2*>(hi),
                                                   reinterpret_cast<uint2*>(lo));
    return cudaGetLastError();
  }
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  split_kernel<<<unsigned(blocks), 256, 0, s>>>(x, n, reinterpret_cast<__nv_bfloat16*>(hi),
                                                reinterpret_cast<__nv_bfloat16*>(lo));
  return cudaGetLastError();
}

bool swiglu_split_supported(const float* g, const float* u, int64_t n, const uint16_t* hi,
                            const uint16_t* lo) {
  return n % 4 == 0 && aligned16(g) && aligned16(u) && aligned8(hi) && aligned8(lo);
}

cudaError_t launch_swiglu_split(const float* g, const float* u, int64_t n, uint16_t* hi,
                                uint16_t* lo, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (!swiglu_split_supported(g, u, n, hi, lo)) return cudaErrorInvalidValue;
  const int64_t n4 = n / 4;
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 148 * 16);
  swiglu_split4_kernel<<<unsigned(blocks), 256, 0, s>>>(
      reinterpret_cast<const float4*>(g), reinterpret_cast<const float4*>(u), n4,
      reinterpret_cast<uint2*>(hi), reinterpret_cast<uint2*>(lo));
  return cudaGetLastError();
}

namespace {
// Tile width for N columns over m_tiles 128-row blocks on num_sms SMs:
// the widest of 256, 192, 128 (multiples of 16 the MMA takes) whose tiles
// fill the last round of the persistent grid best.
int pick_bn(int64_t N, int64_t m_tiles, int num_sms) {
  int best = 256;
  double best_eff = -1.0;
  for (int bn : {256, 192, 128}) {
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    const int64_t rounds = (tiles + num_sms - 1) / num_sms;
    const double eff = double(tiles) / double(rounds * num_sms) * double(N) /
                       double(((N + bn - 1) / bn) * bn);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}
}  // namespace

cudaError_t launch_gemm_tc2(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* w1,
                            int64_t N1, float* y1, int64_t ldy1, const uint16_t* w2, int64_t N2,
                            float* y2, int64_t ldy2, int64_t T, int64_t K, bool accumulate,
                            int32_t* err, cudaStream_t s) {
  if (T <= 0 || N1 + N2 <= 0) return cudaSuccess;
  if (K % 8 != 0 || N1 <= 0 || N2 < 0 || (N2 > 0 && !w2) || T > (int64_t(1) << 30) ||
      N1 > (int64_t(1) << 30) || N2 > (int64_t(1) << 30) || K > (int64_t(1) << 30) || !err)
    return cudaErrorInvalidValue;
  static int num_sms = 0;
  if (!num_sms) {
    int dev = 0;
    TMG_CUDA_TRY(cudaGetDevice(&dev));
    TMG_CUDA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int64_t mt = (T + BM - 1) / BM;
  // one width for both segments (gate and up have the same N)
  const int bn = pick_bn(N1 + N2, mt, num_sms);
  CUtensorMap mh, ml, mw1, mw2;
  if (!make_map(&mh, x_hi, T, K, BM) || !make_map(&ml, x_lo, T, K, BM) ||
      !make_map(&mw1, w1, N1, K, bn) || !make_map(&mw2, N2 > 0 ? w2 : w1, N2 > 0 ? N2 : N1, K, bn))
    return cudaErrorInvalidValue;
  GemmTcArgs a;
  a.y1 = y1;
  a.ldy1 = ldy1;
  a.y2 = y2;
  a.ldy2 = ldy2;
  a.T = int(T);
  a.K = int(K);
  a.N1 = int(N1);
  a.N2 = int(N2);
  a.bn = bn;
  a.nt1 = int((N1 + bn - 1) / bn);
  a.nt2 = int((N2 + bn - 1) / bn);
  a.mt = int(mt);
  a.accumulate = accumulate ? 1 : 0;
  a.err = err;
  a.swiglu = 0;
  a.act_hi = a.act_lo = nullptr;
  a.ld_act = 0;
  const int64_t tiles = mt * (a.nt1 + a.nt2);
  const unsigned grid = unsigned(std::min<int64_t>(tiles, num_sms));
  gemm_tc_kernel<<<grid, kThreadsG, SMEM_BYTES, s>>>(mh, ml, mw1, mw2, a);
  return cudaGetLastError();
}

bool gemm_swiglu_supported(int64_t I, const void* act_hi, const void* act_lo) {
  return I % 16 == 0 && (reinterpret_cast<uintptr_t>(act_hi) & 31) == 0 &&
         (reinterpret_cast<uintptr_t>(act_lo) & 31) == 0;
}

cudaError_t launch_gemm_tc_swiglu(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* wg,
                                  const uint16_t* wu, int64_t I, int64_t T, int64_t K,
                                  uint16_t* act_hi, uint16_t* act_lo, int32_t* err,
                                  cudaStream_t s) {
  if (T <= 0 || I <= 0) return cudaSuccess;
  if (K % 8 != 0 || T > (int64_t(1) << 30) || I > (int64_t(1) << 30) || K > (int64_t(1) << 30) ||
      !err || !gemm_swiglu_supported(I, act_hi, act_lo))
    return cudaErrorInvalidValue;
  static int num_sms = 0;
  if (!num_sms) {
    int dev = 0;
    TMG_CUDA_TRY(cudaGetDevice(&dev));
    TMG_CUDA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int64_t mt = (T + BM - 1) / BM;
  const int bn = pick_bn(2 * I, mt, num_sms);  // bn / 2 gate + bn / 2 up columns per tile
  CUtensorMap mh, ml, mg, mu;
  if (!make_map(&mh, x_hi, T, K, BM) || !make_map(&ml, x_lo, T, K, BM) ||
      !make_map(&mg, wg, I, K, bn / 2) || !make_map(&mu, wu, I, K, bn / 2))
    return cudaErrorInvalidValue;
  GemmTcArgs a;
  a.y1 = a.y2 = nullptr;
  a.ldy1 = a.ldy2 = 0;
  a.T = int(T);
  a.K = int(K);
  a.N1 = int(I);
  a.N2 = 0;
  a.bn = bn;
  a.nt1 = int((I + bn / 2 - 1) / (bn / 2));
  a.nt2 = 0;
  a.mt = int(mt);
  a.accumulate = 0;
  a.err = err;
  a.swiglu = 1;
  a.act_hi = act_hi;
  a.act_lo = act_lo;
  a.ld_act = I;
  const int64_t tiles = mt * a.nt1;
  const unsigned grid = unsigned(std::min<int64_t>(tiles, num_sms));
  gemm_tc_kernel<<<grid, kThreadsG, SMEM_BYTES, s>>>(mh, ml, mg, mu, a);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* w,
                           int64_t T, int64_t N, int64_t K, float* y, int64_t ldy,
                           bool accumulate, int32_t* err, cudaStream_t s) {
  return launch_gemm_tc2(x_hi, x_lo, w, N, y, ldy, nullptr, 0, nullptr, 0, T, K, accumulate, err,
                         s);
}

}  // namespace tmg
