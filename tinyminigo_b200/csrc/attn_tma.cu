// Decode attention with the cache rows staged by TMA (src/model.rs:434-459:
// per query head, scores over the stream's cached rows, softmax, weighted sum
// of the values; GQA: kv_head = head / (n_q / n_kv)).
//
// Grid (n_kv, nsplit, M), 160 threads: four consumer warps and one producer
// warp.  The producer streams the split's K and V rows of this kv head as
// [32 positions x head_dim] f32 tiles with cp.async.bulk.tensor (a 2D tensor
// map over the layer's [M * capacity, n_kv * head_dim] cache) into a ring of
// shared-memory stages guarded by mbarriers, so several tiles per CTA are in
// flight while the consumers work on an earlier one.  Each consumer
// half-warp takes 4 of a tile's 32 rows: lane l16 holds columns
// 4 l16 .. (and 64 + 4 l16 .. for head dim 128) of q (all G heads), reads its
// columns of each row from shared memory, meets the other 15 lanes in a
// shuffle butterfly for the scores, and keeps its own running max, sum and
// output per head (online softmax); the eight half-warps meet in shared
// memory at the end, and the last split of a (stream, kv head) combines the
// partials (ticket).  The decoded position's rotated k and raw v are
// appended to the cache by the CTA whose range holds it, which uses them
// from shared memory for its own row.  HBM roofline: 2 * n_ctx * head_dim * 4
// bytes per (stream, kv head).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kTmaConsumers = 4;                    // consumer warps
constexpr int kTmaThreads = (kTmaConsumers + 1) * kWarp;
constexpr int kTmaRows = 32;                        // positions per tile
constexpr int kTmaRowsPerHalf = kTmaRows / (2 * kTmaConsumers);  // 4
constexpr int kTmaMinChunk = 64;                    // fewest positions a split takes
constexpr int kTmaMaxStages = 6;

__device__ __forceinline__ void rot_rn(float a, float b, float c, float s, float* o0, float* o1) {
  const float ac = __fmul_rn(a, c), bs = __fmul_rn(b, s), as = __fmul_rn(a, s), bc = __fmul_rn(b, c);
  *o0 = __fsub_rn(ac, bs);
  *o1 = __fadd_rn(as, bc);
}

constexpr float kLog2e = 1.4426950408889634f;

// 2^x by the SFU's ex2 instruction (relative error about 2^-22; 2^-inf = 0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Reduce-scatter of 16 values over the 16 lanes of a half-warp: afterwards
// v[0] of lane l16 holds the sum over the half-warp of value l16.  Level
// xor m (8, 4, 2, 1) pairs value j with j + m among the values still held;
// a lane keeps the half its lane bit selects and adds the partner's copy.
__device__ __forceinline__ void reduce_scatter16(float (&v)[16], int l16) {
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) {
    const bool hi = (l16 & m) != 0;
#pragma unroll
    for (int j = 0; j < m; ++j) {
      const float keep = hi ? v[j + m] : v[j];
      const float send = hi ? v[j] : v[j + m];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Stages of the ring for head dim D (a stage: the K and V tiles).
template <int D>
constexpr int tma_stages() { return 3; }
template <int D>
constexpr int tma_stage_floats() { return 2 * kTmaRows * D; }

template <int D>
__global__ void __launch_bounds__(kTmaThreads, D == 64 ? 3 : 2)
    attn_decode_tma_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const AttnDecodeArgs a) {
  constexpr int d = D, GM = 4, NS = tma_stages<D>(), SF = tma_stage_floats<D>();
  constexpr int DL = D / 64;  // float4 column groups per lane (head dim 128: two)
  extern __shared__ __align__(128) float stg[];  // NS stages of [K tile | V tile]; later the combine weights
  __shared__ __align__(8) uint64_t full[NS];
  __shared__ __align__(8) uint64_t empty[NS];
  __shared__ __align__(16) float qs[GM * D];
  __shared__ __align__(16) float kp_s[D];
  __shared__ __align__(16) float vp_s[D];
  __shared__ __align__(16) float wo[kTmaConsumers * GM * D];
  __shared__ __align__(16) float ofin[GM * D];
  __shared__ float wm[kTmaConsumers * GM], wl[kTmaConsumers * GM];
  __shared__ float m_s[16], l_s[16];
  __shared__ __align__(16) float p_s[kTmaConsumers][2][16];  // [warp][half-warp][row * 4 + head]
  __shared__ volatile int abort_s;
  __shared__ volatile int issued_s;  // tiles the producer has issued
  __shared__ bool last_s;
  const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
  const int half = d / 2, G = a.nq / a.nkv, kvd = a.nkv * d;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) trace_mark(a.trace, 0);
  pdl_trigger();
  pdl_wait();
  if (tid == 0) {
    trace_mark(a.trace, 1);
    trace_mark(a.trace, 2);
  }

  const bool fixed = a.pos_override != nullptr;
  const int pos = fixed ? a.pos_override[m] : a.st.pos[m];
  const bool done = fixed ? true : (a.st.done[m] != 0);
  const bool append = !done && pos < a.cap;
  const int n_ctx = fixed ? pos + 1 : (append ? pos + 1 : pos);
  const float* qkv = a.qkv + size_t(m) * a.qkv_ld;
  float* kc = a.kc + size_t(m) * a.cap * kvd;
  float* vc = a.vc + size_t(m) * a.cap * kvd;

  int chunk = (n_ctx + a.nsplit - 1) / a.nsplit;
  chunk = max(kTmaMinChunk, (chunk + kTmaRows - 1) / kTmaRows * kTmaRows);
  const int n_used = (n_ctx + chunk - 1) / chunk;
  const int c0 = split * chunk;
  const int c1 = min(n_ctx, c0 + chunk);
  if (n_used == 1 && split > 0) {  // one-split launches need no ticket
    if (tid == 0) trace_mark(a.trace, 3);
    return;
  }
  const bool own_pos = append && pos >= c0 && pos < c1;
  const int ntiles = c1 > c0 ? (c1 - c0 + kTmaRows - 1) / kTmaRows : 0;

  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTmaConsumers);
    }
    abort_s = 0;
    issued_s = 0;
    mbar_fence_init();
  }
  // q heads of this group rotated at pos (model.rs:422-426)
  const int rp = pos < a.cap ? pos : 0;
  for (int i = tid; i < G * half; i += blockDim.x) {
    const int g = i / half, j = i % half;
    const float* qh = qkv + (kvh * G + g) * d;
    if (fixed) {
      qs[g * d + j] = qh[j];
      qs[g * d + j + half] = qh[j + half];
    } else {
      float o0, o1;
      rot_rn(qh[j], qh[j + half], a.rope_cos[size_t(rp) * half + j],
             a.rope_sin[size_t(rp) * half + j], &o0, &o1);
      qs[g * d + j] = o0;
      qs[g * d + j + half] = o1;
    }
  }
  // the CTA whose range holds pos appends the rotated k and raw v
  // (KvCache::push, model.rs:432) and keeps them for its own row
  if (own_pos) {
    const float* kh = qkv + a.nq * d + kvh * d;
    const float* vh = qkv + (a.nq + a.nkv) * d + kvh * d;
    float* kdst = kc + size_t(pos) * kvd + kvh * d;
    float* vdst = vc + size_t(pos) * kvd + kvh * d;
    for (int j = tid; j < half; j += blockDim.x) {
      float o0, o1;
      rot_rn(kh[j], kh[j + half], a.rope_cos[size_t(pos) * half + j],
             a.rope_sin[size_t(pos) * half + j], &o0, &o1);
      kdst[j] = o0;
      kdst[j + half] = o1;
      kp_s[j] = o0;
      kp_s[j + half] = o1;
    }
    for (int j = tid; j < d; j += blockDim.x) {
      const float v = vh[j];
      vdst[j] = v;
      vp_s[j] = v;
    }
  }
  __syncthreads();

  if (warp == kTmaConsumers) {
    // ---- producer: the split's tiles, NS in flight ----
    if (lane == 0) {
      const int y0 = m * int(a.cap) + c0;
      for (int i = 0; i < ntiles; ++i) {
        const int s = i % NS;
        const uint32_t ph = (i / NS) & 1;
        if (abort_s || !mbar_wait(&empty[s], ph ^ 1)) {
          abort_s = 1;
          if (a.err) atomicExch(a.err, 2);
          break;
        }
        float* kt = stg + s * SF;
        mbar_expect_tx(&full[s], uint32_t(SF * 4));
        tma_load_2d(kt, &kmap, &full[s], kvh * d, y0 + i * kTmaRows);
        tma_load_2d(kt + kTmaRows * d, &vmap, &full[s], kvh * d, y0 + i * kTmaRows);
        issued_s = i + 1;
      }
    }
  } else {
    // ---- consumers ----
    // A half-warp takes 4 rows of each tile.  Each lane dots its columns of
    // the 4 rows with its columns of the G <= 4 q heads (16 partial sums),
    // then a reduce-scatter over the half-warp's 16 lanes (xor 8, 4, 2, 1:
    // the same pairs, so the same sums, as a butterfly) leaves lane l16
    // with the whole score of row l16 / 4 and head l16 % 4.  Scores are
    // kept in base-2 units (scale * log2 e folded into the scale), so one
    // ex2 per lane gives its probability; the lane keeps its head's running
    // max and its own share of the head's running sum, and the 16
    // probabilities reach every lane through shared memory for the weighted
    // sum of the values it holds.  The outputs are rescaled only in tiles where
    // some head's max grew (alpha is exactly 1 otherwise).
    const int hw = lane >> 4, l16 = lane & 15, hb = lane & 16;
    const int my_g = l16 & 3, my_r = l16 >> 2;
    const float qscale = a.scale * kLog2e;
    float4 q4[GM][DL], o4[GM][DL];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
#pragma unroll
      for (int c = 0; c < DL; ++c) {
        q4[g][c] = g < G ? *reinterpret_cast<const float4*>(qs + g * d + 64 * c + 4 * l16)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        o4[g][c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float m_own = -INFINITY;  // running max of head my_g (equal in its 4 lanes)
    float l_own = 0.f;        // this lane's rows' share of head my_g's running sum
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % NS;
      const uint32_t ph = (i / NS) & 1;
      const bool ok = !abort_s && mbar_wait(&full[s], ph);
      if (!ok) {
        if (lane == 0) {
          abort_s = 1;
          if (a.err) atomicExch(a.err, 2);
        }
        break;
      }
      const float* kt = stg + s * SF;
      const float* vt = kt + kTmaRows * d;
      const int r0 = warp * 2 * kTmaRowsPerHalf + hw * kTmaRowsPerHalf;  // row in the tile
      const int tb = c0 + i * kTmaRows + r0;                               // its position
      float4 kr[kTmaRowsPerHalf][DL], vr[kTmaRowsPerHalf][DL];
      // the tile's rows as loaded, unless it reaches past the range or holds
      // the decoded position (the same for the whole CTA)
      const int tile0 = c0 + i * kTmaRows;
      if (tile0 + kTmaRows <= c1 && !(own_pos && pos >= tile0 && pos < tile0 + kTmaRows)) {
#pragma unroll
        for (int r = 0; r < kTmaRowsPerHalf; ++r)
#pragma unroll
          for (int c = 0; c < DL; ++c) {
            const int col = 64 * c + 4 * l16;
            kr[r][c] = *reinterpret_cast<const float4*>(kt + (r0 + r) * d + col);
            vr[r][c] = *reinterpret_cast<const float4*>(vt + (r0 + r) * d + col);
          }
      } else {
#pragma unroll
        for (int r = 0; r < kTmaRowsPerHalf; ++r) {
          // rows past the range hold whatever the cache held (or the map's
          // zero fill): they enter as zeros with a masked score
          const bool mine = own_pos && tb + r == pos;
          const bool live = tb + r < c1;
#pragma unroll
          for (int c = 0; c < DL; ++c) {
            const int col = 64 * c + 4 * l16;
            kr[r][c] = mine ? *reinterpret_cast<const float4*>(kp_s + col)
                            : *reinterpret_cast<const float4*>(kt + (r0 + r) * d + col);
            vr[r][c] = mine ? *reinterpret_cast<const float4*>(vp_s + col)
                            : *reinterpret_cast<const float4*>(vt + (r0 + r) * d + col);
            if (!live) {
              kr[r][c] = make_float4(0.f, 0.f, 0.f, 0.f);
              vr[r][c] = kr[r][c];
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // the tile is in registers
      // partial scores over this lane's columns, index r * 4 + g
      float sp[16];
#pragma unroll
      for (int r = 0; r < kTmaRowsPerHalf; ++r) {
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          float acc = q4[g][0].x * kr[r][0].x;
          acc = fmaf(q4[g][0].y, kr[r][0].y, acc);
          acc = fmaf(q4[g][0].z, kr[r][0].z, acc);
          acc = fmaf(q4[g][0].w, kr[r][0].w, acc);
#pragma unroll
          for (int c = 1; c < DL; ++c) {
            acc = fmaf(q4[g][c].x, kr[r][c].x, acc);
            acc = fmaf(q4[g][c].y, kr[r][c].y, acc);
            acc = fmaf(q4[g][c].z, kr[r][c].z, acc);
            acc = fmaf(q4[g][c].w, kr[r][c].w, acc);
          }
          sp[r * 4 + g] = acc;
        }
      }
      reduce_scatter16(sp, l16);
      const bool live = tb + my_r < c1 && my_g < G;
      const float sc = live ? sp[0] * qscale : -INFINITY;
      float mt = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      const float mn = fmaxf(m_own, mt);
      const float p = sc == -INFINITY ? 0.f : ex2_approx(sc - mn);
      if (__any_sync(0xffffffffu, mn != m_own)) {
        const float alpha = mn == m_own ? 1.f : (m_own == -INFINITY ? 0.f : ex2_approx(m_own - mn));
        l_own *= alpha;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          const float ag = __shfl_sync(0xffffffffu, alpha, hb + g);
#pragma unroll
          for (int c = 0; c < DL; ++c)
            o4[g][c] = make_float4(o4[g][c].x * ag, o4[g][c].y * ag, o4[g][c].z * ag,
                                   o4[g][c].w * ag);
        }
      }
      m_own = mn;
      l_own += p;
      // the half-warp's 16 probabilities to every lane of it: one store and
      // four broadcast loads (row r's heads at p_s[r * 4 ..])
      float* ps_h = p_s[warp][hw];
      __syncwarp();  // the previous tile's reads are done
      ps_h[l16] = p;
      __syncwarp();
#pragma unroll
      for (int r = 0; r < kTmaRowsPerHalf; ++r) {
        const float4 pr = *reinterpret_cast<const float4*>(ps_h + r * 4);
        const float pv[4] = {pr.x, pr.y, pr.z, pr.w};
#pragma unroll
        for (int g = 0; g < GM; ++g) {
#pragma unroll
          for (int c = 0; c < DL; ++c) {
            o4[g][c].x = fmaf(pv[g], vr[r][c].x, o4[g][c].x);
            o4[g][c].y = fmaf(pv[g], vr[r][c].y, o4[g][c].y);
            o4[g][c].z = fmaf(pv[g], vr[r][c].z, o4[g][c].z);
            o4[g][c].w = fmaf(pv[g], vr[r][c].w, o4[g][c].w);
          }
        }
      }
    }
    // per head: the half-warp's max and sum (the 4 lanes of a head hold
    // shares of its sum)
    float l_h = l_own + __shfl_xor_sync(0xffffffffu, l_own, 4);
    l_h += __shfl_xor_sync(0xffffffffu, l_h, 8);
    float m_g[GM], l_g[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m_g[g] = __shfl_sync(0xffffffffu, m_own, hb + g);
      l_g[g] = __shfl_sync(0xffffffffu, l_h, hb + g);
    }
    // the warp's two half-warps meet (lanes l16 and l16 + 16)
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m_g[g], 16);
        const float l2 = __shfl_xor_sync(0xffffffffu, l_g[g], 16);
        const float M = fmaxf(m_g[g], m2);
        const float a1 = m_g[g] == -INFINITY ? 0.f : ex2_approx(m_g[g] - M);
        const float a2 = m2 == -INFINITY ? 0.f : ex2_approx(m2 - M);
#pragma unroll
        for (int c = 0; c < DL; ++c) {
          float4 o2;
          o2.x = __shfl_xor_sync(0xffffffffu, o4[g][c].x, 16);
          o2.y = __shfl_xor_sync(0xffffffffu, o4[g][c].y, 16);
          o2.z = __shfl_xor_sync(0xffffffffu, o4[g][c].z, 16);
          o2.w = __shfl_xor_sync(0xffffffffu, o4[g][c].w, 16);
          if (hw == 0) {
            float4 o;
            o.x = fmaf(o2.x, a2, o4[g][c].x * a1);
            o.y = fmaf(o2.y, a2, o4[g][c].y * a1);
            o.z = fmaf(o2.z, a2, o4[g][c].z * a1);
            o.w = fmaf(o2.w, a2, o4[g][c].w * a1);
            *reinterpret_cast<float4*>(wo + (warp * G + g) * d + 64 * c + 4 * l16) = o;
          }
        }
        if (hw == 0 && l16 == 0) {
          wm[warp * GM + g] = M;
          wl[warp * GM + g] = fmaf(l2, a2, l_g[g] * a1);
        }
      }
    }
  }
  __syncthreads();
  // every issued tile has completed (the consumers waited on all of them,
  // or an abort stopped the producer before it issued more); the stage
  // memory is free for the combine weights below
  if (abort_s) {
    // a wait gave up: let the copies still in flight (the last NS issued)
    // land before the CTA leaves
    if (tid == 0) {
      const int n = issued_s;
      for (int j = max(0, n - NS); j < n; ++j) mbar_wait(&full[j % NS], (j / NS) & 1);
      trace_mark(a.trace, 3);
    }
    return;
  }
  // one thread per head: the CTA's (m, l); then o per (head, column)
  if (tid < G) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTmaConsumers; ++w) M = fmaxf(M, wm[w * GM + tid]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < kTmaConsumers; ++w) {
      const float mw = wm[w * GM + tid];
      L = fmaf(wl[w * GM + tid], mw == -INFINITY ? 0.f : ex2_approx(mw - M), L);
    }
    m_s[tid] = M;
    l_s[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * d; idx += blockDim.x) {
    const int g = idx / d;
    const float M = m_s[g];
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kTmaConsumers; ++w) {
      const float mw = wm[w * GM + g];
      O = fmaf(wo[(w * G + g) * d + (idx % d)], mw == -INFINITY ? 0.f : ex2_approx(mw - M), O);
    }
    ofin[idx] = O;
  }
  __syncthreads();
  float* out = a.out + size_t(m) * a.nq * d + kvh * G * d;
  if (n_used == 1) {
    if (split == 0) {
      for (int idx = tid; idx < G * d; idx += blockDim.x) {
        const float L = l_s[idx / d];
        out[idx] = L > 0.f ? ofin[idx] / L : 0.f;
      }
    }
    if (tid == 0) trace_mark(a.trace, 3);
    return;
  }
  // partial (m, l, o[d]) per head
  if (split < n_used) {
    float* part = a.part + ((size_t(m) * a.nkv + kvh) * a.nsplit + split) * G * (d + 2);
    for (int idx = tid; idx < G * d; idx += blockDim.x)
      part[(idx / d) * (d + 2) + 2 + (idx % d)] = ofin[idx];
    if (tid < G) {
      part[tid * (d + 2)] = m_s[tid];
      part[tid * (d + 2) + 1] = l_s[tid];
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(&a.ticket[m * a.nkv + kvh], 1u);
    last_s = (t == gridDim.y - 1);
  }
  __syncthreads();
  if (!last_s) {
    if (tid == 0) trace_mark(a.trace, 3);
    return;
  }
  __threadfence();
  // combine: the per-split weights once per (split, head), then every
  // output sums its column over the splits
  const float* pb = a.part + (size_t(m) * a.nkv + kvh) * a.nsplit * G * (d + 2);
  float* wts = stg;  // [G][n_used] (n_used * G <= NS * SF floats)
  for (int g = warp; g < G; g += blockDim.x / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < n_used; s += 32) mx = fmaxf(mx, __ldcg(pb + (s * G + g) * (d + 2)));
    mx = warp_max(mx);
    float L = 0.f;
    for (int s = lane; s < n_used; s += 32) {
      const float ms = __ldcg(pb + (s * G + g) * (d + 2));
      const float w = ms == -INFINITY ? 0.f : ex2_approx(ms - mx);
      wts[g * n_used + s] = w;
      L = fmaf(__ldcg(pb + (s * G + g) * (d + 2) + 1), w, L);
    }
    L = warp_sum(L);
    if (lane == 0) l_s[g] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * d; idx += blockDim.x) {
    const int g = idx / d, j = idx % d;
    float acc = 0.f;
    int s = 0;
    for (; s + 4 <= n_used; s += 4) {
      const float o0 = __ldcg(pb + ((s + 0) * G + g) * (d + 2) + 2 + j);
      const float o1 = __ldcg(pb + ((s + 1) * G + g) * (d + 2) + 2 + j);
      const float o2 = __ldcg(pb + ((s + 2) * G + g) * (d + 2) + 2 + j);
      const float o3 = __ldcg(pb + ((s + 3) * G + g) * (d + 2) + 2 + j);
      acc = fmaf(o0, wts[g * n_used + s], acc);
      acc = fmaf(o1, wts[g * n_used + s + 1], acc);
      acc = fmaf(o2, wts[g * n_used + s + 2], acc);
      acc = fmaf(o3, wts[g * n_used + s + 3], acc);
    }
    for (; s < n_used; ++s) acc = fmaf(__ldcg(pb + (s * G + g) * (d + 2) + 2 + j), wts[g * n_used + s], acc);
    const float L = l_s[g];
    out[idx] = L > 0.f ? acc / L : 0.f;
  }
  if (tid == 0) {
    a.ticket[m * a.nkv + kvh] = 0u;
    trace_mark(a.trace, 3);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

// A 2D f32 map over a layer's cache [rows, kvd] with a [32 x D] box.
bool cache_map(CUtensorMap* m, const float* base, int64_t rows, int kvd, int D) {
  auto fn = encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(kvd), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(kvd) * 4};
  cuuint32_t box[2] = {cuuint32_t(D), cuuint32_t(kTmaRows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attn_decode_tma_ok(int nq, int nkv, int d, int64_t cap, int M, const void* kc, const void* vc) {
  if (nkv <= 0 || nq % nkv || nq / nkv > 4 || (d != 64 && d != 128)) return false;
  if (int64_t(M) * cap > int64_t(INT32_MAX) - kTmaRows) return false;
  if ((reinterpret_cast<uintptr_t>(kc) & 15) || (reinterpret_cast<uintptr_t>(vc) & 15)) return false;
  return encode_tiled() != nullptr;
}

size_t attn_decode_tma_smem(int d) {
  return d == 64 ? size_t(tma_stages<64>()) * tma_stage_floats<64>() * 4
                 : size_t(tma_stages<128>()) * tma_stage_floats<128>() * 4;
}

cudaError_t launch_attn_decode_tma(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  if (!attn_decode_tma_ok(a.nq, a.nkv, a.d, a.cap, a.M, a.kc, a.vc)) return cudaErrorInvalidValue;
  const int kvd = a.nkv * a.d;
  // the combine's per-split weights reuse the stage memory
  if (size_t(a.nq / a.nkv) * a.nsplit * 4 > attn_decode_tma_smem(a.d)) return cudaErrorInvalidValue;
  CUtensorMap km, vm;
  if (!cache_map(&km, a.kc, int64_t(a.M) * a.cap, kvd, a.d) ||
      !cache_map(&vm, a.vc, int64_t(a.M) * a.cap, kvd, a.d))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nkv, a.nsplit, a.M);
  cfg.blockDim = dim3(kTmaThreads);
  cfg.dynamicSmemBytes = attn_decode_tma_smem(a.d);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (a.d == 64) return cudaLaunchKernelEx(&cfg, attn_decode_tma_kernel<64>, km, vm, a);
  return cudaLaunchKernelEx(&cfg, attn_decode_tma_kernel<128>, km, vm, a);
}

cudaError_t attn_tma_prepare() {
  TMG_CUDA_TRY(set_carveout(attn_decode_tma_kernel<64>, int(attn_decode_tma_smem(64))));
  return set_carveout(attn_decode_tma_kernel<128>, int(attn_decode_tma_smem(128)));
}

}  // namespace tmg
