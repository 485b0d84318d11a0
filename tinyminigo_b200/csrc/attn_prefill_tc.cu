// Causal prefill attention on the 5th-generation tensor cores (tcgen05 +
// TMEM + TMA), head dim 64.
//
// The reference's prefill attention (src/model.rs:526-571: per query row t
// and head, scores q.k * scale over keys 0..pos0+t, softmax, weighted sum of
// the values) in f32.  Here S = Q K^T and O = P V are tcgen05 MMAs on BF16
// operands that together carry the f32 values:
//   * scores: q (pre-multiplied by scale * log2 e, so S comes out in base-2
//     units) and k are each split into three BF16 parts x = hi + mid + lo
//     (hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid): ~24 bits)
//     and S accumulates the six products hi.hi, hi.mid, mid.hi, hi.lo,
//     lo.hi, mid.mid in f32 (the dropped terms are below 2^-26 relative);
//   * values: p and v are split in two (~16 bits each) and O accumulates
//     p_hi.v_hi + p_hi.v_lo + p_lo.v_hi.  p lies in [0, 1] and O is a
//     weighted mean, so this keeps the output within ~2^-16 of |v|.
// The splits are written by attn_pf_split_* into scratch arrays laid out
// for TMA: q parts [n_q][Tq][64], k parts [n_kv][Lk][64] and the value
// parts transposed, [n_kv][64][Lk] (the PV MMA's B operand is K-major).
//
// One CTA = 128 query rows of one q head; grid (n_q, query blocks), the
// heaviest (last) query blocks first.  320 threads:
//   warp 0     TMA producer: the q parts once, then per 64-key block the k
//              parts into a 3-stage ring (free again once S_j is computed)
//              and the v parts into a 2-stage ring (free once O_j is), with
//              the 128-byte swizzle;
//   warp 1     allocates 256 TMEM columns and issues the MMAs (one lane):
//              S_j into one of two S buffers, then, once the softmax has
//              written P_j, O_j = P_j V_j into one of two O buffers;
//   warps 2-9  softmax, two threads per query row (TMEM lane = row; one
//              takes keys and output dims 0-31, the other 32-63): load S_j
//              (tcgen05.ld), mask the blocks that reach the diagonal or past
//              the keys, running max (shared by the pair through shared
//              memory) and sum, p = 2^(s - m) into the P buffer as BF16
//              hi/lo in the swizzled K-major layout the MMA reads, then fold
//              O_{j-1} from TMEM into registers (o = o * alpha + O_blk), one
//              block behind so that PV_j overlaps softmax_{j+1}.
// Every mbarrier wait is bounded; a wait that gives up sets the error word
// and the CTA stops (the host reports TMG_ERR_TIMEOUT).  Single-GPU code:
// every CTA loads its own tiles; no peer memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kPD = 64;                       // head dim
constexpr int kQB = 128;                      // query rows per CTA (MMA M)
constexpr int kKB = 64;                       // keys per block (S: N; PV: K)
constexpr int kKStages = 3;  // k ring: a stage is free once S_j has read it
constexpr int kVStages = 2;  // v ring: once O_j = P_j V_j has
constexpr int kQPart = kQB * kPD * 2;         // 16 KB: one BF16 part of the q tile
constexpr int kKPart = kKB * kPD * 2;         // 8 KB: one part of a k block
constexpr int kVPart = kPD * kKB * 2;         // 8 KB: one part of a v^T block
constexpr int kKStage = 3 * kKPart;          // 24 KB: k hi, mid, lo
constexpr int kVStage = 2 * kVPart;          // 16 KB: v^T hi, lo
constexpr int kPPart = kQB * kKB * 2;         // 16 KB: one part of a P block
constexpr int kOffQ = 0;                      // q hi, mid, lo
constexpr int kOffK = 3 * kQPart;                      // 48 KB
constexpr int kOffV = kOffK + kKStages * kKStage;      // 120 KB
constexpr int kOffP = kOffV + kVStages * kVStage;      // 152 KB; P[2] x {hi, lo}
constexpr int kOffBar = kOffP + 2 * 2 * kPPart;        // 216 KB
constexpr int kSmemPf = kOffBar + 256 + 1024;          // + barriers + alignment slack
constexpr int kPfThreads = 320;  // producer, MMA, 8 softmax warps
constexpr uint32_t kPfTmemCols = 256;  // S[2] at 0, 64; O[2] at 128, 192
// kind::f16: BF16 x BF16 -> F32, both K-major, M = 128, N = 64.
constexpr uint32_t kIdescPf =
    (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(64 >> 3) << 17) | (uint32_t(128 >> 4) << 24);
constexpr float kLog2ePf = 1.4426950408889634f;

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                      int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Shared-memory descriptor of a K-major BF16 tile of 128-byte rows written
// with the 128-byte swizzle (8-row groups 1024 B apart).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3fff);
  d |= uint64_t(1) << 16;
  d |= uint64_t(1024 >> 4) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(kIdescPf), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes (one row per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
#pragma unroll
  for (int c = 0; c < 32; c += 16)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(r[c + 0]), "=r"(r[c + 1]), "=r"(r[c + 2]), "=r"(r[c + 3]), "=r"(r[c + 4]),
          "=r"(r[c + 5]), "=r"(r[c + 6]), "=r"(r[c + 7]), "=r"(r[c + 8]), "=r"(r[c + 9]),
          "=r"(r[c + 10]), "=r"(r[c + 11]), "=r"(r[c + 12]), "=r"(r[c + 13]), "=r"(r[c + 14]),
          "=r"(r[c + 15])
        : "r"(taddr + uint32_t(c)));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Barrier `id` (1..15) among `n` threads (whole warps).
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
// The same barrier, returning the AND of every participant's `pred`.
__device__ __forceinline__ bool bar_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

// (bf16(a), bf16(b)) packed, a in the low half.
__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct PfArgs {
  float* out;        // [T, out_ld]: head h at columns h * 64
  uint16_t* out_hi;  // or (when set) its BF16 hi/lo parts, same layout
  uint16_t* out_lo;
  int64_t out_ld;
  int32_t* err;
  int T;             // query rows
  int64_t pos0;      // position of query row 0
  int Lk;            // keys: pos0 + T
  int Tq;            // query rows per head in the q arrays (multiple of 128)
  int Lkp;           // keys per kv head in the k arrays (multiple of 64)
  int G;             // q heads per kv head
};

__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap mq_hi,
                           const __grid_constant__ CUtensorMap mq_mid,
                           const __grid_constant__ CUtensorMap mq_lo,
                           const __grid_constant__ CUtensorMap mk_hi,
                           const __grid_constant__ CUtensorMap mk_mid,
                           const __grid_constant__ CUtensorMap mk_lo,
                           const __grid_constant__ CUtensorMap mv_hi,
                           const __grid_constant__ CUtensorMap mv_lo, const PfArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~uintptr_t(1023));
  uint64_t* kfull = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [3] k stage loaded
  uint64_t* kempty = kfull + kKStages;                             // [3] k stage free
  uint64_t* vfull = kempty + kKStages;                             // [2] v stage loaded
  uint64_t* vempty = vfull + kVStages;                             // [2] v stage free
  uint64_t* qfull = vempty + kVStages;                             // q parts loaded
  uint64_t* s_full = qfull + 1;                                  // [2] S_j in TMEM
  uint64_t* p_full = s_full + 2;                                 // [2] P_j in smem (S_j read)
  uint64_t* o_full = p_full + 2;                                 // [2] O_j in TMEM
  uint64_t* o_free = o_full + 2;                                 // [2] O_j read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);
  __shared__ volatile int failed;
  __shared__ float red_mx[2][2][kQB];  // [block parity][half][row]: a half's max of the block
  __shared__ float red_l[2][kQB];      // [half][row]: a half's share of the row's sum

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, kvh = h / a.G;
  const int qb = int(gridDim.y) - 1 - int(blockIdx.y);
  const int q0 = qb * kQB;
  const int64_t last_key = min(int64_t(a.Lk), a.pos0 + q0 + kQB);  // keys [0, last_key)
  const int nb = int((last_key + kKB - 1) / kKB);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(qfull, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_free[b], 8);
    }
    failed = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      mbar_expect_tx(qfull, 3 * kQPart);
      const int qy = h * a.Tq + q0;
      tma2d(sm + kOffQ, &mq_hi, qfull, 0, qy);
      tma2d(sm + kOffQ + kQPart, &mq_mid, qfull, 0, qy);
      tma2d(sm + kOffQ + 2 * kQPart, &mq_lo, qfull, 0, qy);
      for (int j = 0; j < nb; ++j) {
        const int sk = j % kKStages, sv = j % kVStages;
        if (failed || !mbar_wait(&kempty[sk], ((j / kKStages) & 1) ^ 1)) {
          failed = 1;
          atomicExch(a.err, 2);
          break;
        }
        uint8_t* kst = sm + kOffK + sk * kKStage;
        mbar_expect_tx(&kfull[sk], kKStage);
        const int ky = kvh * a.Lkp + j * kKB;
        tma2d(kst, &mk_hi, &kfull[sk], 0, ky);
        tma2d(kst + kKPart, &mk_mid, &kfull[sk], 0, ky);
        tma2d(kst + 2 * kKPart, &mk_lo, &kfull[sk], 0, ky);
        if (failed || !mbar_wait(&vempty[sv], ((j / kVStages) & 1) ^ 1)) {
          failed = 1;
          atomicExch(a.err, 2);
          break;
        }
        uint8_t* vst = sm + kOffV + sv * kVStage;
        mbar_expect_tx(&vfull[sv], kVStage);
        tma2d(vst, &mv_hi, &vfull[sv], j * kKB, kvh * kPD);
        tma2d(vst + kVPart, &mv_lo, &vfull[sv], j * kKB, kvh * kPD);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      bool ok = mbar_wait(qfull, 0);
      const uint32_t qa = smem_u32(sm + kOffQ);
      const uint32_t qh = qa, qm = qa + kQPart, ql = qa + 2 * kQPart;
      for (int j = 0; j <= nb && ok; ++j) {
        if (j < nb) {
          // S_j = Q K_j^T into S buffer j & 1 (its previous user, S_{j-2},
          // was read before P_{j-2} arrived, which PV_{j-2} waited for)
          const int s = j % kKStages;
          if (failed || !mbar_wait(&kfull[s], (j / kKStages) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t kb = smem_u32(sm + kOffK + s * kKStage);
          const uint32_t kh = kb, km = kb + kKPart, kl = kb + 2 * kKPart;
          const uint32_t ts = tmem + uint32_t((j & 1) * 64);
#pragma unroll
          for (int k = 0; k < kPD / 16; ++k) {
            const uint32_t o = uint32_t(k * 32);
            mma(ts, sdesc(qh + o), sdesc(kh + o), k != 0);
            mma(ts, sdesc(qh + o), sdesc(km + o), 1);
            mma(ts, sdesc(qm + o), sdesc(kh + o), 1);
            mma(ts, sdesc(qh + o), sdesc(kl + o), 1);
            mma(ts, sdesc(ql + o), sdesc(kh + o), 1);
            mma(ts, sdesc(qm + o), sdesc(km + o), 1);
          }
          commit(&s_full[j & 1]);
          commit(&kempty[s]);  // k stage s is free once these MMAs have read it
        }
        if (j >= 1) {
          // O_i = P_i V_i for i = j - 1 into O buffer i & 1
          const int i = j - 1, b = i & 1;
          const int s = i % kVStages;
          if (failed || !mbar_wait(&p_full[b], (i >> 1) & 1) ||
              (i >= 2 && !mbar_wait(&o_free[b], ((i - 2) >> 1) & 1)) ||
              !mbar_wait(&vfull[s], (i / kVStages) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t vb = smem_u32(sm + kOffV + s * kVStage);
          const uint32_t vh = vb, vl = vb + kVPart;
          const uint32_t pb = smem_u32(sm + kOffP + b * 2 * kPPart);
          const uint32_t ph = pb, pl = pb + kPPart;
          const uint32_t to = tmem + 128u + uint32_t(b * 64);
#pragma unroll
          for (int k = 0; k < kKB / 16; ++k) {
            const uint32_t o = uint32_t(k * 32);
            mma(to, sdesc(ph + o), sdesc(vh + o), k != 0);
            mma(to, sdesc(ph + o), sdesc(vl + o), 1);
            mma(to, sdesc(pl + o), sdesc(vh + o), 1);
          }
          commit(&o_full[b]);
          commit(&vempty[s]);  // v stage s is free once these MMAs have read it
        }
      }
      if (!ok) {
        failed = 1;
        atomicExch(a.err, 2);
      }
    }
  } else {
    // ---- softmax / output: two threads per query row ----
    // Warps 2-5 and 6-9: warp w reads TMEM lanes 32 (w % 4) .. (its rows);
    // the first four take keys 0-31 of each block and dims 0-31 of O, the
    // other four keys 32-63 and dims 32-63.  The two threads of a row
    // agree on the row's running max through shared memory (named barrier
    // of the two warps); each keeps its share of the running sum.
    const int qd = warp & 3;                 // TMEM lane quadrant of this warp
    const int hf = (warp - 2) >> 2;          // which half of the keys and dims
    const int r = qd * 32 + lane;            // row in the query block
    const int64_t tq = a.pos0 + q0 + r;      // its position
    const uint32_t lanes = uint32_t(qd * 32) << 16;
    const uint32_t cofs = uint32_t(hf * 32);
    const int64_t row0 = a.pos0 + q0;        // the first row's position
    float o[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) o[c] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    // A failed wait does not leave the loop on its own: the pair's barrier
    // below ANDs both threads' status, so both leave at the same block and
    // every barrier of the pair is met.
    for (int j = 0; j < nb; ++j) {
      const int b = j & 1;
      const bool got = mbar_wait(&s_full[b], (j >> 1) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float sv[32];
      tmem_ld32(tmem + lanes + uint32_t(b * 64) + cofs, sv);
      const int64_t k0 = int64_t(j) * kKB + hf * 32;
      // only blocks that reach past the first row's position or past the
      // keys need the mask (the same for every row of the CTA)
      if (int64_t(j) * kKB + kKB - 1 > row0 || int64_t(j) * kKB + kKB > a.Lk) {
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (k0 + c > tq || k0 + c >= a.Lk) sv[c] = -INFINITY;
      }
      // four independent chains (max is exact in any order)
      float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < 32; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], sv[c]);
      const float lmx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      red_mx[b][hf][r] = lmx;
      if (!bar_and(2 + qd, 64, ok && got)) {
        ok = false;
        break;
      }
      const float mx = fmaxf(m, fmaxf(lmx, red_mx[b][hf ^ 1][r]));
      const float alpha = m == -INFINITY ? 0.f : ex2f(m - mx);
      // mx is finite (key 0 is visible to every row), so a masked score
      // gives ex2(-inf) = 0 without a test; the sum in four chains
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      // P_j (row r, this half's 32 keys) into P buffer b: BF16 hi and lo,
      // 16-byte chunk e of the 128-byte row at chunk e ^ (r & 7) (the
      // 128-byte swizzle).  The buffer was last read by PV_{j-2}, which
      // completed before O_{j-2} was folded.
      uint8_t* prow_h = sm + kOffP + b * 2 * kPPart + r * 128;
      uint8_t* prow_l = prow_h + kPPart;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int t = 0; t < 8; t += 2) {
          const float p0 = ex2f(sv[8 * e + t] - mx);
          const float p1 = ex2f(sv[8 * e + t + 1] - mx);
          sum4[t >> 1] += p0;
          sum4[t >> 1] += p1;
          const uint32_t hb = bf16x2_bits(p0, p1);
          const float r0 = p0 - __uint_as_float(hb << 16);
          const float r1 = p1 - __uint_as_float(hb & 0xffff0000u);
          hw[t / 2] = hb;
          lw[t / 2] = bf16x2_bits(r0, r1);
        }
        const int off = (((hf * 4 + e) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(prow_h + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(prow_l + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
      l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      m = mx;
      // the P writes (generic proxy) before the MMA (async proxy) reads them
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      if (j >= 1) {
        const int i = j - 1, bi = i & 1;
        if (!mbar_wait(&o_full[bi], (i >> 1) & 1)) ok = false;  // leaves at the next barrier
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float ob[32];
        tmem_ld32(tmem + lanes + 128u + uint32_t(bi * 64) + cofs, ob);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = fmaf(o[c], alpha_prev, ob[c]);
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[bi]);
      }
      alpha_prev = alpha;
    }
    if (ok) {
      const int i = nb - 1, bi = i & 1;
      if (!mbar_wait(&o_full[bi], (i >> 1) & 1)) {
        ok = false;
      } else {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        float ob[32];
        tmem_ld32(tmem + lanes + 128u + uint32_t(bi * 64) + cofs, ob);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = fmaf(o[c], alpha_prev, ob[c]);
      }
    }
    // the row's sum: this thread's share and its partner's (every thread
    // reaches this barrier, also after a failed wait)
    red_l[hf][r] = l;
    named_sync(2 + qd, 64);
    const float lt = l + red_l[hf ^ 1][r];
    if (!ok) {
      failed = 1;
      atomicExch(a.err, 2);
    } else if (q0 + r < a.T) {
      const int64_t base = int64_t(q0 + r) * a.out_ld + int64_t(h) * kPD + hf * 32;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      if (a.out_hi) {
        // the O GEMM's operands: hi = bf16(v), lo = bf16(v - hi)
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int t = 0; t < 8; t += 2) {
            const float v0 = o[c + t] * inv, v1 = o[c + t + 1] * inv;
            const uint32_t hb = bf16x2_bits(v0, v1);
            hw[t / 2] = hb;
            lw[t / 2] = bf16x2_bits(v0 - __uint_as_float(hb << 16),
                                    v1 - __uint_as_float(hb & 0xffff0000u));
          }
          *reinterpret_cast<uint4*>(a.out_hi + base + c) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(a.out_lo + base + c) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      } else {
        float* dst = a.out + base;
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(dst + c) =
              make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kPfTmemCols));
  }
}

// Three-way BF16 split of x: hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid).
__device__ __forceinline__ void split3(float x, uint16_t* hi, uint16_t* mid, uint16_t* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(h);
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(m);
  *hi = __bfloat16_as_ushort(h);
  *mid = __bfloat16_as_ushort(m);
  *lo = __bfloat16_as_ushort(__float2bfloat16_rn(r2));
}

// q rows (T of them, row stride q_ld, head h at columns h * 64) times qs,
// split three ways into [n_q][Tq][64] (rows T..Tq-1 zero).  Grid (Tq / 4,
// n_q), 256 threads: 4 rows of 64 per block.
__global__ void attn_pf_split_q_kernel(const float* __restrict__ q, int64_t q_ld, int T, int Tq,
                                       float qs, uint16_t* __restrict__ hi,
                                       uint16_t* __restrict__ mid, uint16_t* __restrict__ lo) {
  const int h = blockIdx.y;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 6), c = threadIdx.x & 63;
  const float x = t < T ? q[int64_t(t) * q_ld + int64_t(h) * kPD + c] * qs : 0.f;
  const int64_t o = (int64_t(h) * Tq + t) * kPD + c;
  split3(x, hi + o, mid + o, lo + o);
}

// The cache rows [0, Lk) of one kv head: k split three ways into
// [n_kv][Lkp][64]; v split in two and transposed into [n_kv][64][Lkp]
// (keys Lk..Lkp-1 zero).  Grid (Lkp / 64, n_kv), 256 threads: one 64-key
// block per CTA.
// Keys at or past `kend` are left alone (attn_pf_prep_kernel writes them).
__global__ void attn_pf_split_kv_kernel(const float* __restrict__ kc, const float* __restrict__ vc,
                                        int64_t kvd, int Lk, int Lkp, int kend,
                                        uint16_t* __restrict__ khi, uint16_t* __restrict__ kmid,
                                        uint16_t* __restrict__ klo, uint16_t* __restrict__ vhi,
                                        uint16_t* __restrict__ vlo) {
  __shared__ float vs[kKB][kPD + 1];
  const int kvh = blockIdx.y, key0 = blockIdx.x * kKB;
  for (int i = threadIdx.x; i < kKB * kPD; i += blockDim.x) {
    const int kk = i / kPD, c = i % kPD;
    const int key = key0 + kk;
    if (key >= kend) continue;
    const bool in = key < Lk;
    const float kx = in ? kc[int64_t(key) * kvd + int64_t(kvh) * kPD + c] : 0.f;
    vs[kk][c] = in ? vc[int64_t(key) * kvd + int64_t(kvh) * kPD + c] : 0.f;
    const int64_t o = (int64_t(kvh) * Lkp + key) * kPD + c;
    split3(kx, khi + o, kmid + o, klo + o);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kKB * kPD; i += blockDim.x) {
    const int c = i / kKB, kk = i % kKB;
    if (key0 + kk >= kend) continue;
    const float v = vs[kk][c];
    const __nv_bfloat16 hb = __float2bfloat16_rn(v);
    const int64_t o = (int64_t(kvh) * kPD + c) * Lkp + key0 + kk;
    vhi[o] = __bfloat16_as_ushort(hb);
    vlo[o] = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(hb)));
  }
}

// RoPE with the reference's rounding (each product rounded, then the sum),
// as the decode kernels apply it.
__device__ __forceinline__ void rot_pf(float a, float b, float c, float s, float* o0, float* o1) {
  const float ac = __fmul_rn(a, c), bs = __fmul_rn(b, s), as = __fmul_rn(a, s), bc = __fmul_rn(b, c);
  *o0 = __fsub_rn(ac, bs);
  *o1 = __fadd_rn(as, bc);
}

// The new rows of a prefill chunk in one pass over the projections
// (src/model.rs:533-553): RoPE of q and k at pos0 + t, k and v appended to
// the cache, and the attention's operand parts: q (times qs) three ways
// into [n_q][Tq][64] (rows T..Tq-1 zero), k three ways into [n_kv][Lkp][64]
// and v two ways transposed into [n_kv][64][Lkp] for keys pos0 .. Lkp-1
// (keys past pos0 + T zero).  Grid (row blocks of 64, n_q + n_kv), 256
// threads: a q head's rows, or a kv head's keys.
__global__ void attn_pf_prep_kernel(const float* __restrict__ qkv, int64_t ld, int nq, int nkv,
                                    int T, int64_t pos0, int Tq, int Lkp,
                                    const float* __restrict__ cs, const float* __restrict__ sn,
                                    float qs, float* __restrict__ kc, float* __restrict__ vc,
                                    uint16_t* __restrict__ qh, uint16_t* __restrict__ qm,
                                    uint16_t* __restrict__ ql, uint16_t* __restrict__ kh,
                                    uint16_t* __restrict__ km, uint16_t* __restrict__ kl,
                                    uint16_t* __restrict__ vh, uint16_t* __restrict__ vl) {
  __shared__ float vs[kKB][kPD + 1];
  constexpr int half = kPD / 2;
  const int hs = blockIdx.y, t0 = blockIdx.x * kKB;
  const int64_t kvd = int64_t(nkv) * kPD;
  if (hs < nq) {
    if (t0 >= Tq) return;
    for (int i = threadIdx.x; i < kKB * half; i += blockDim.x) {
      const int tt = i / half, j = i % half, t = t0 + tt;
      float o0 = 0.f, o1 = 0.f;
      if (t < T) {
        const float* v = qkv + int64_t(t) * ld + int64_t(hs) * kPD;
        const int64_t pos = pos0 + t;
        rot_pf(v[j], v[j + half], cs[pos * half + j], sn[pos * half + j], &o0, &o1);
      }
      const int64_t o = (int64_t(hs) * Tq + t) * kPD;
      split3(o0 * qs, qh + o + j, qm + o + j, ql + o + j);
      split3(o1 * qs, qh + o + j + half, qm + o + j + half, ql + o + j + half);
    }
    return;
  }
  const int kvh = hs - nq;
  const int64_t key0 = pos0 + t0;
  if (key0 >= Lkp) return;
  for (int i = threadIdx.x; i < kKB * half; i += blockDim.x) {
    const int tt = i / half, j = i % half, t = t0 + tt;
    const int64_t key = key0 + tt;
    if (key >= Lkp) continue;
    float o0 = 0.f, o1 = 0.f, v0 = 0.f, v1 = 0.f;
    if (t < T) {
      const float* row = qkv + int64_t(t) * ld;
      const float* kv = row + int64_t(nq + kvh) * kPD;
      rot_pf(kv[j], kv[j + half], cs[key * half + j], sn[key * half + j], &o0, &o1);
      const float* vv = row + int64_t(nq + nkv + kvh) * kPD;
      v0 = vv[j];
      v1 = vv[j + half];
      float* kd = kc + key * kvd + int64_t(kvh) * kPD;
      float* vd = vc + key * kvd + int64_t(kvh) * kPD;
      kd[j] = o0;
      kd[j + half] = o1;
      vd[j] = v0;
      vd[j + half] = v1;
    }
    const int64_t o = (int64_t(kvh) * Lkp + key) * kPD;
    split3(o0, kh + o + j, km + o + j, kl + o + j);
    split3(o1, kh + o + j + half, km + o + j + half, kl + o + j + half);
    vs[tt][j] = v0;
    vs[tt][j + half] = v1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kKB * kPD; i += blockDim.x) {
    const int c = i / kKB, tt = i % kKB;
    const int64_t key = key0 + tt;
    if (key >= Lkp) continue;
    const float v = vs[tt][c];
    const __nv_bfloat16 hb = __float2bfloat16_rn(v);
    const int64_t o = (int64_t(kvh) * kPD + c) * Lkp + key;
    vh[o] = __bfloat16_as_ushort(hb);
    vl[o] = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(hb)));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_pf() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D BF16 [rows, cols] row-major map with a (64 x box_rows) box and the
// 128-byte swizzle.
bool map_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto fn = encode_pf();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  cuuint32_t box[2] = {64u, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

}  // namespace

size_t attn_prefill_tc_scratch(int nq, int nkv, int64_t T, int64_t Lk) {
  const int64_t Tq = round_up(T, kQB), Lkp = round_up(Lk, kKB);
  return size_t(3 * nq * Tq * kPD + 3 * nkv * Lkp * kPD + 2 * nkv * kPD * Lkp) * 2 + 6 * 256;
}

bool attn_prefill_tc_ok(const float* q, int64_t q_ld, const float* kc, const float* vc, int64_t T,
                        int64_t pos0, int nq, int nkv, int d, const void* out, int64_t out_ld) {
  if (d != kPD || nkv <= 0 || nq % nkv || T <= 0 || pos0 < 0) return false;
  if (pos0 + T > (int64_t(1) << 30) || int64_t(nq) * round_up(T, kQB) > (int64_t(1) << 30) ||
      int64_t(nkv) * round_up(pos0 + T, kKB) > (int64_t(1) << 30))
    return false;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || out_ld % 8) return false;
  (void)q;
  (void)q_ld;
  (void)kc;
  (void)vc;
  return encode_pf() != nullptr;
}

cudaError_t attn_prefill_tc_prepare() {
  return set_carveout(attn_prefill_tc_kernel, kSmemPf);
}

cudaError_t launch_attn_prefill_tc(const float* q, int64_t q_ld, const float* kc, const float* vc,
                                   int64_t T, int64_t pos0, int nq, int nkv, float scale,
                                   float* out, uint16_t* out_hi, uint16_t* out_lo, int64_t out_ld,
                                   void* scratch, size_t scratch_bytes, int32_t* err,
                                   cudaStream_t s, const float* rope_cos, const float* rope_sin) {
  const void* dst = out_hi ? static_cast<const void*>(out_hi) : static_cast<const void*>(out);
  if (!attn_prefill_tc_ok(q, q_ld, kc, vc, T, pos0, nq, nkv, kPD, dst, out_ld) ||
      !err || (out_hi && ((reinterpret_cast<uintptr_t>(out_lo) & 15) || !out_lo)) ||
      (!out_hi && !out))
    return cudaErrorInvalidValue;
  const int64_t Lk = pos0 + T;
  const int64_t Tq = round_up(T, kQB), Lkp = round_up(Lk, kKB);
  if (scratch_bytes < attn_prefill_tc_scratch(nq, nkv, T, Lk)) return cudaErrorInvalidValue;
  // carve the scratch: every array 256-byte aligned
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(scratch) + 255) &
                                          ~uintptr_t(255));
  auto take = [&](int64_t elems) {
    uint16_t* r = reinterpret_cast<uint16_t*>(p);
    p += (elems * 2 + 255) / 256 * 256;
    return r;
  };
  const int64_t nqe = int64_t(nq) * Tq * kPD, nke = int64_t(nkv) * Lkp * kPD;
  uint16_t *qh = take(nqe), *qm = take(nqe), *ql = take(nqe);
  uint16_t *kh = take(nke), *km = take(nke), *kl = take(nke);
  uint16_t *vh = take(nke), *vl = take(nke);
  if (p > reinterpret_cast<uint8_t*>(scratch) + scratch_bytes) return cudaErrorInvalidValue;
  const int64_t kvd = int64_t(nkv) * kPD;
  if (rope_cos) {
    // q, k, v of the chunk's rows un-rotated in q (rows of q_ld: q | k | v):
    // one pass rotates, appends to the cache and writes their parts; the
    // older cache rows [0, pos0) are split from the cache
    if (pos0 > 0) {
      attn_pf_split_kv_kernel<<<dim3(unsigned((pos0 + kKB - 1) / kKB), unsigned(nkv)), 256, 0, s>>>(
          kc, vc, kvd, int(Lk), int(Lkp), int(pos0), kh, km, kl, vh, vl);
      TMG_CUDA_TRY(cudaGetLastError());
    }
    const int64_t rows = std::max<int64_t>(Tq, Lkp - pos0);
    attn_pf_prep_kernel<<<dim3(unsigned((rows + kKB - 1) / kKB), unsigned(nq + nkv)), 256, 0, s>>>(
        q, q_ld, nq, nkv, int(T), pos0, int(Tq), int(Lkp), rope_cos, rope_sin,
        scale * kLog2ePf, const_cast<float*>(kc), const_cast<float*>(vc), qh, qm, ql, kh, km, kl,
        vh, vl);
    TMG_CUDA_TRY(cudaGetLastError());
  } else {
    attn_pf_split_q_kernel<<<dim3(unsigned(Tq / 4), unsigned(nq)), 256, 0, s>>>(
        q, q_ld, int(T), int(Tq), scale * kLog2ePf, qh, qm, ql);
    TMG_CUDA_TRY(cudaGetLastError());
    attn_pf_split_kv_kernel<<<dim3(unsigned(Lkp / kKB), unsigned(nkv)), 256, 0, s>>>(
        kc, vc, kvd, int(Lk), int(Lkp), int(Lkp), kh, km, kl, vh, vl);
    TMG_CUDA_TRY(cudaGetLastError());
  }
  CUtensorMap mqh, mqm, mql, mkh, mkm, mkl, mvh, mvl;
  if (!map_bf16(&mqh, qh, int64_t(nq) * Tq, kPD, kQB) ||
      !map_bf16(&mqm, qm, int64_t(nq) * Tq, kPD, kQB) ||
      !map_bf16(&mql, ql, int64_t(nq) * Tq, kPD, kQB) ||
      !map_bf16(&mkh, kh, int64_t(nkv) * Lkp, kPD, kKB) ||
      !map_bf16(&mkm, km, int64_t(nkv) * Lkp, kPD, kKB) ||
      !map_bf16(&mkl, kl, int64_t(nkv) * Lkp, kPD, kKB) ||
      !map_bf16(&mvh, vh, int64_t(nkv) * kPD, Lkp, kPD) ||
      !map_bf16(&mvl, vl, int64_t(nkv) * kPD, Lkp, kPD))
    return cudaErrorInvalidValue;
  PfArgs a;
  a.out = out;
  a.out_hi = out_hi;
  a.out_lo = out_lo;
  a.out_ld = out_ld;
  a.err = err;
  a.T = int(T);
  a.pos0 = pos0;
  a.Lk = int(Lk);
  a.Tq = int(Tq);
  a.Lkp = int(Lkp);
  a.G = nq / nkv;
  attn_prefill_tc_kernel<<<dim3(unsigned(nq), unsigned(Tq / kQB)), kPfThreads, kSmemPf, s>>>(
      mqh, mqm, mql, mkh, mkm, mkl, mvh, mvl, a);
  return cudaGetLastError();
}

}  // namespace tmg
