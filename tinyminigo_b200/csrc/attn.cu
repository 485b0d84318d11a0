// Attention for the token loop.
//
// Decode (src/model.rs:420-459): RoPE of q and k at pos (Rope::rotate,
// src/tensor.rs:1026-1037, from the host-built cos/sin table), the KV append
// (KvCache::push, model.rs:288-293), and GQA attention of each query head
// over the stream's cached rows, kv_head = head / (n_q / n_kv).  The context
// is split over CTAs (split-KV); each CTA keeps an online softmax per head
// of its GQA group and reads every K/V row of its range once for all G heads
// of the group; the last CTA of a (stream, kv head) combines the partials.
// HBM-bound for long contexts: algorithmic bytes = 2 * n_ctx * kv_dim * 4
// per layer and stream.
//
// Prefill (attention_batch, src/tensor.rs:1099-1139): causal attention of T
// query rows over the cache with an online softmax in f32.  Head dim 64:
// 64-row x 64-key register-tiled blocks (attn_prefill_tiled_kernel); other
// head dims: one thread (or two, for head_dim 128) per query row, K/V tiles
// staged in shared memory.
#include <math.h>

#include <algorithm>
#include <cstring>
#include <stdlib.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kTile = 64;      // decode split lengths are multiples of this
constexpr int kMinChunk = 64;  // fewest positions a decode split takes
constexpr int kPTile = 32;     // key positions per prefill tile

// Rotate pair (a, b) by (c, s): (a c - b s, a s + b c), rounded like the
// reference (two products, then one add/sub; no FMA contraction).
__device__ __forceinline__ void rot(float a, float b, float c, float s, float* o0, float* o1) {
  float ac = __fmul_rn(a, c), bs = __fmul_rn(b, s), as = __fmul_rn(a, s), bc = __fmul_rn(b, c);
  *o0 = __fsub_rn(ac, bs);
  *o1 = __fadd_rn(as, bc);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// K/V tile buffers of the decode kernel: two (the next tile loads while the
// current one is used) where they fit the shared-memory budget.
constexpr int kTileD = 32;     // positions per shared-memory tile of the decode kernel
constexpr int kAttnBufs = 2;   // its K/V tile buffers (the next tile loads during this one)
// K tile row stride (floats) and the float4 swizzle of row t: rows of d >= 32
// unpadded with float4 index j4 stored at j4 ^ 4 on odd rows, so that the
// eight lanes of a 16-byte phase (two rows, four quarters) hit distinct banks
template <int D>
constexpr int attn_kstride() { return D >= 32 ? D : D + 16; }
template <int D>
__device__ __forceinline__ int attn_kswz(int t) { return D >= 32 ? (t & 1) << 2 : 0; }

// Grid (n_kv, nsplit, M); 128 threads.  Dynamic smem: q [G][d], K tiles
// [NB][kTileD][d+16], V tiles [NB][kTileD][d], p [kTileD][G rounded up to
// 4], and the decoded position's rotated k and raw v [2][d].
template <int D, int GM>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnDecodeArgs a) {
  extern __shared__ float sm[];
  __shared__ float m_s[16], l_s[16];
  __shared__ bool last_s;
  constexpr int NB = kAttnBufs;
  const int kvh = blockIdx.x, split = blockIdx.y, m = blockIdx.z;
  constexpr int d = D;
  const int half = d / 2, G = a.nq / a.nkv, kvd = a.nkv * d;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int GP = (G + 3) & ~3;               // heads per p row, padded to float4
  float* qs = sm;                           // [G][d]
  float* ks_ = qs + G * d;                    // [NB][kTileD][d+16]
  constexpr int KS = attn_kstride<D>();
  float* vs = ks_ + NB * kTileD * KS;         // [NB][kTileD][d]
  float* ps = vs + NB * kTileD * d;           // [kTileD][GP] p, a warp's rows each
  float* kp_s = ps + kTileD * GP;             // [d] k of the decoded position (rotated)
  float* vp_s = kp_s + d;                   // [d] its v

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

  // context range of this split: at least kMinChunk positions per split, so
  // short contexts use few CTAs (the rest only take their ticket)
  int chunk = (n_ctx + a.nsplit - 1) / a.nsplit;
  chunk = max(kMinChunk, (chunk + kTile - 1) / kTile * kTile);
  const int n_used = (n_ctx + chunk - 1) / chunk;
  const int c0 = split * chunk;
  const int c1 = min(n_ctx, c0 + chunk);
  if (n_used == 1 && split > 0) {  // one-split launches need no ticket
    if (tid == 0) trace_mark(a.trace, 3);
    return;
  }
  const bool own_pos = append && pos >= c0 && pos < c1;
  const int d4 = d / 4;

  // q heads of this group rotated at pos (model.rs:422-426), and the first
  // K/V tile, requested together
  const int rp = pos < a.cap ? pos : 0;
  for (int i = tid; i < G * half; i += blockDim.x) {
    const int g = i / half, j = i % half;
    const float* qh = qkv + (kvh * G + g) * d;
    if (fixed) {
      qs[g * d + j] = qh[j];
      qs[g * d + j + half] = qh[j + half];
    } else {
      float o0, o1;
      rot(qh[j], qh[j + half], a.rope_cos[size_t(rp) * half + j], a.rope_sin[size_t(rp) * half + j],
          &o0, &o1);
      qs[g * d + j] = o0;
      qs[g * d + j + half] = o1;
    }
  }
  // the CTA whose range holds pos appends the rotated k and raw v
  // (KvCache::push, model.rs:432) and keeps them for its tile
  if (own_pos) {
    const float* kh = qkv + a.nq * d + kvh * d;
    const float* vh = qkv + (a.nq + a.nkv) * d + kvh * d;
    float* kdst = kc + size_t(pos) * kvd + kvh * d;
    float* vdst = vc + size_t(pos) * kvd + kvh * d;
    for (int j = tid; j < half; j += blockDim.x) {
      float o0, o1;
      rot(kh[j], kh[j + half], a.rope_cos[size_t(pos) * half + j],
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
  // tile (t0, nt) into buffer b: cache rows by cp.async, the decoded
  // position's row (when in range) from kp_s/vp_s (the caller commits)
  auto load_tile = [&](int b, int t0, int nt) {
    float* kb = ks_ + b * kTileD * KS;
    float* vb = vs + b * kTileD * d;
    for (int i = tid; i < nt * d4; i += blockDim.x) {
      const int t = i / d4, j4 = i % d4;
      const int pk = (j4 ^ attn_kswz<D>(t)) * 4;
      if (own_pos && t0 + t == pos) {
        *reinterpret_cast<float4*>(kb + t * KS + pk) =
            *reinterpret_cast<const float4*>(kp_s + j4 * 4);
        *reinterpret_cast<float4*>(vb + t * d + j4 * 4) =
            *reinterpret_cast<const float4*>(vp_s + j4 * 4);
        continue;
      }
      cp_async16(kb + t * KS + pk, kc + size_t(t0 + t) * kvd + kvh * d + j4 * 4);
      cp_async16(vb + t * d + j4 * 4, vc + size_t(t0 + t) * kvd + kvh * d + j4 * 4);
    }
  };
  // the first NB - 1 tiles, one commit group each (empty past the range)
#pragma unroll
  for (int k = 0; k < NB - 1; ++k) {
    const int tk = c0 + k * kTileD;
    if (tk < c1) load_tile(k, tk, min(kTileD, c1 - tk));
    cp_async_commit();
  }
  // Work split (flash-decoding inside the CTA; GM: heads per kv head, at
  // most): warp w takes positions 8w .. 8w+7 of every 32-position tile with
  // its own running max m, sum l and output o per head, so one CTA barrier
  // per tile (the tile's arrival) is all the warps share:
  //  * scores: lane -> position lane / 4 of the warp's eight and every
  //    fourth float4 of its K row (lane & 3), all heads; the quarters meet
  //    by two shuffles (K rows swizzled, see attn_kswz);
  //  * softmax: max and sum over the warp's positions by shuffles; p goes
  //    to a warp-private [8][GP] table;
  //  * P.V: lane -> DL consecutive columns, all heads: V rows coalesced
  //    across the warp, p by one broadcast float4 per 4 heads.
  // The four warps' (m, l, o) meet in shared memory at the end.
  constexpr int kWarps = kAttnThreads / 32;
  constexpr int kPerW = kTileD / kWarps;  // positions per warp and tile (8)
  constexpr int DL = D >= 32 ? D / 32 : 1;
  const bool pv_lane = D >= 32 || lane < D;  // lanes with columns in P.V
  const int tw = lane >> 2, dq = lane & 3;
  float* pw = ps + warp * kPerW * GP;  // this warp's p table [kPerW][GP]
  float m_g[GM], l_g[GM], o_acc[GM][DL];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    m_g[g] = -INFINITY;
    l_g[g] = 0.f;
#pragma unroll
    for (int e = 0; e < DL; ++e) o_acc[g][e] = 0.f;
  }

  for (int t0 = c0, it = 0; t0 < c1; t0 += kTileD, ++it) {
    const int nt = min(kTileD, c1 - t0);
    const int b = it % NB;
    cp_async_wait<NB - 2>();  // this tile's group (one group is committed per tile)
    __syncthreads();          // ... visible to all, and every warp is done with tile it - 1
    {
      const int tn = t0 + (NB - 1) * kTileD;  // into the buffer of tile it - 1
      if (tn < c1) load_tile((it + NB - 1) % NB, tn, min(kTileD, c1 - tn));
      cp_async_commit();
    }
    const float* kt = ks_ + b * kTileD * KS;
    const float* vt = vs + b * kTileD * d;
    const int tb = warp * kPerW;                    // first tile row of this warp
    const int nw = max(0, min(kPerW, nt - tb));     // its rows in this tile
    if (nw > 0) {
      // raw scores of position tb + tw
      const int t = tb + tw;
      float sc[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) sc[g] = 0.f;
      if (tw < nw) {
        const float* kr = kt + t * KS;
        const int sw = attn_kswz<D>(t);
#pragma unroll
        for (int j = 0; j < d; j += 16) {
          const float4 k4 = *reinterpret_cast<const float4*>(kr + ((((j >> 2) + dq) ^ sw) << 2));
#pragma unroll
          for (int g = 0; g < GM; ++g) {
            if (g < G) {
              const float4 q4 = *reinterpret_cast<const float4*>(qs + g * d + dq * 4 + j);
              sc[g] = fmaf(q4.x, k4.x, sc[g]);
              sc[g] = fmaf(q4.y, k4.y, sc[g]);
              sc[g] = fmaf(q4.z, k4.z, sc[g]);
              sc[g] = fmaf(q4.w, k4.w, sc[g]);
            }
          }
        }
      }
      // online softmax over the warp's positions (lane bits 2..4), per head
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g < G) {
          float full = sc[g] + __shfl_xor_sync(0xffffffffu, sc[g], 1);
          full += __shfl_xor_sync(0xffffffffu, full, 2);
          const float s = tw < nw ? full * a.scale : -INFINITY;
          float mt = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 4));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
          mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
          const float mn = fmaxf(m_g[g], mt);
          const float p = tw < nw ? expf(s - mn) : 0.f;
          float ls = p + __shfl_xor_sync(0xffffffffu, p, 4);
          ls += __shfl_xor_sync(0xffffffffu, ls, 8);
          ls += __shfl_xor_sync(0xffffffffu, ls, 16);
          const float alpha = m_g[g] == -INFINITY ? 0.f : expf(m_g[g] - mn);
          l_g[g] = l_g[g] * alpha + ls;
          m_g[g] = mn;
#pragma unroll
          for (int e = 0; e < DL; ++e) o_acc[g][e] *= alpha;
          if (dq == (g & 3)) pw[tw * GP + g] = p;
        }
      }
      __syncwarp();
      // P.V over the warp's rows
      if (pv_lane) {
#pragma unroll 4
        for (int u = 0; u < nw; ++u) {
          const float* vr = vt + (tb + u) * d + lane * DL;
          float v[DL];
          if (DL == 4) {
            const float4 w4 = *reinterpret_cast<const float4*>(vr);
            v[0] = w4.x; v[DL > 1 ? 1 : 0] = w4.y; v[DL > 2 ? 2 : 0] = w4.z; v[DL > 3 ? 3 : 0] = w4.w;
          } else if (DL == 2) {
            const float2 w2 = *reinterpret_cast<const float2*>(vr);
            v[0] = w2.x; v[DL > 1 ? 1 : 0] = w2.y;
          } else {
            v[0] = vr[0];
          }
#pragma unroll
          for (int c = 0; c < GM / 4; ++c) {
            if (4 * c < G) {
              const float4 p4 = *reinterpret_cast<const float4*>(pw + u * GP + 4 * c);
              const float pr[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (4 * c + q < G) {
#pragma unroll
                  for (int e = 0; e < DL; ++e)
                    o_acc[4 * c + q][e] = fmaf(pr[q], v[e], o_acc[4 * c + q][e]);
                }
              }
            }
          }
        }
      }
      __syncwarp();
    }
  }
  cp_async_wait<0>();  // (only empty groups can remain)
  __syncthreads();     // the tile buffers are free: the warps' (m, l, o) go there
  {
    float* wo = ks_;                      // [kWarps][G][d]
    float* wm = ks_ + kWarps * G * d;     // [kWarps][GM]
    float* wl = wm + kWarps * GM;         // [kWarps][GM]
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        if (pv_lane) {
#pragma unroll
          for (int e = 0; e < DL; ++e) wo[(warp * G + g) * d + lane * DL + e] = o_acc[g][e];
        }
        if (lane == 0) {
          wm[warp * GM + g] = m_g[g];
          wl[warp * GM + g] = l_g[g];
        }
      }
    }
    __syncthreads();
    // one thread per (head, column): the CTA's (m, l) per head and o
    if (tid < G) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * GM + tid]);
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = wm[w * GM + tid];
        L = fmaf(wl[w * GM + tid], mw == -INFINITY ? 0.f : expf(mw - M), L);
      }
      m_s[tid] = M;
      l_s[tid] = L;
    }
    __syncthreads();
    for (int idx = tid; idx < G * d; idx += kAttnThreads) {
      const int g = idx / d;
      const float M = m_s[g];
      float O = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = wm[w * GM + g];
        O = fmaf(wo[(w * G + g) * d + (idx % d)], mw == -INFINITY ? 0.f : expf(mw - M), O);
      }
      wo[kWarps * G * d + 2 * kWarps * GM + idx] = O;  // after wm/wl
    }
    __syncthreads();
  }
  const float* ofin = ks_ + kWarps * G * d + 2 * kWarps * GM;  // [G][d] o of this CTA
  float* out = a.out + size_t(m) * a.nq * d + kvh * G * d;
  if (n_used == 1) {
    // the whole context in one CTA: finish here, no partials
    if (split == 0) {
      for (int idx = tid; idx < G * d; idx += kAttnThreads) {
        const float L = l_s[idx / d];
        out[idx] = L > 0.f ? ofin[idx] / L : 0.f;
      }
    }
    if (tid == 0) trace_mark(a.trace, 3);
    return;  // one-split launches need no ticket
  }
  // partial (m, l, o[d]) per head
  if (split < n_used) {
    float* part = a.part + ((size_t(m) * a.nkv + kvh) * a.nsplit + split) * G * (d + 2);
    for (int idx = tid; idx < G * d; idx += kAttnThreads)
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
  // combine: the per-split weights w = exp(m_s - max) once per (split, head)
  // in shared memory, then every output sums its column over the splits
  const float* pb = a.part + (size_t(m) * a.nkv + kvh) * a.nsplit * G * (d + 2);
  float* wts = sm;  // [G][n_used] (the tiles are no longer needed)
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < n_used; s += 32) mx = fmaxf(mx, __ldcg(pb + (s * G + g) * (d + 2)));
    mx = warp_max(mx);
    float L = 0.f;
    for (int s = lane; s < n_used; s += 32) {
      const float ms = __ldcg(pb + (s * G + g) * (d + 2));
      const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
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

// ---------------------------------------------------------------------------
// Decode attention for head dim 64 and at most 4 query heads per kv head (the
// 1B-class shapes), with K and V streamed from HBM straight into registers:
// each K/V element serves only the G heads of its group, so staging tiles in
// shared memory bought nothing but shared-memory latency.  Same grid, split,
// append, partials and ticketed merge as attn_decode_kernel.  Inside the CTA
// eight row streams (4 warps x 2 half-warps) take blocks of kRegRows
// consecutive positions in turn; lane l16 of a half-warp holds columns
// 4 l16 .. 4 l16 + 3 of q (all heads), of each K/V row it loads (one 16-byte
// non-coherent load per row, a half-warp reads a row's 256 contiguous bytes)
// and of its output.  Scores meet over the 16 lanes by a shuffle butterfly;
// each stream keeps its own running max, sum and output per head; the
// streams meet in shared memory at the end.  The decoded position's row
// comes from shared memory (this CTA wrote it to the cache).
// Dynamic shared memory: the merge weights [G][nsplit].
// ---------------------------------------------------------------------------
constexpr int kRegRows = 4;

__global__ void __launch_bounds__(kAttnThreads, 4) attn_decode_reg_kernel(const AttnDecodeArgs a) {
  constexpr int D = 64, d = D, GM = 4, kWarps = kAttnThreads / 32;
  extern __shared__ float wts_s[];
  __shared__ __align__(16) float qs[GM * D];
  __shared__ __align__(16) float kp_s[D];
  __shared__ __align__(16) float vp_s[D];
  __shared__ __align__(16) float wo[kWarps * GM * D];
  __shared__ __align__(16) float ofin[GM * D];
  __shared__ float wm[kWarps * GM], wl[kWarps * GM];
  __shared__ float m_s[16], l_s[16];
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

  // context range of this split: at least kMinChunk positions per split, so
  // short contexts use few CTAs (the rest only take their ticket)
  int chunk = (n_ctx + a.nsplit - 1) / a.nsplit;
  chunk = max(kMinChunk, (chunk + kTile - 1) / kTile * kTile);
  const int n_used = (n_ctx + chunk - 1) / chunk;
  const int c0 = split * chunk;
  const int c1 = min(n_ctx, c0 + chunk);
  if (n_used == 1 && split > 0) {  // one-split launches need no ticket
    if (tid == 0) trace_mark(a.trace, 3);
    return;
  }
  const bool own_pos = append && pos >= c0 && pos < c1;

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
      rot(qh[j], qh[j + half], a.rope_cos[size_t(rp) * half + j], a.rope_sin[size_t(rp) * half + j],
          &o0, &o1);
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
      rot(kh[j], kh[j + half], a.rope_cos[size_t(pos) * half + j],
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

  const int hw = lane >> 4, l16 = lane & 15;
  float4 q4[GM], o4[GM];
  float m_g[GM], l_g[GM];
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    q4[g] = g < G ? *reinterpret_cast<const float4*>(qs + g * d + 4 * l16) : make_float4(0.f, 0.f, 0.f, 0.f);
    o4[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    m_g[g] = -INFINITY;
    l_g[g] = 0.f;
  }
  const float* kcol = kc + kvh * d + 4 * l16;
  const float* vcol = vc + kvh * d + 4 * l16;
  // warp-uniform trip count: the warp's two streams take the blocks at
  // wb and wb + kRegRows; rows past c1 are masked
  for (int wb = c0 + warp * 2 * kRegRows; wb < c1; wb += kWarps * 2 * kRegRows) {
    const int rb = wb + hw * kRegRows;
    float4 kr[kRegRows], vr[kRegRows];
#pragma unroll
    for (int r = 0; r < kRegRows; ++r) {
      const int t = rb + r;
      if (t < c1) {
        if (own_pos && t == pos) {
          kr[r] = *reinterpret_cast<const float4*>(kp_s + 4 * l16);
          vr[r] = *reinterpret_cast<const float4*>(vp_s + 4 * l16);
        } else {
          const uint4 ku = ld_stream(kcol + size_t(t) * kvd);
          const uint4 vu = ld_stream(vcol + size_t(t) * kvd);
          kr[r] = make_float4(__uint_as_float(ku.x), __uint_as_float(ku.y), __uint_as_float(ku.z),
                              __uint_as_float(ku.w));
          vr[r] = make_float4(__uint_as_float(vu.x), __uint_as_float(vu.y), __uint_as_float(vu.z),
                              __uint_as_float(vu.w));
        }
      } else {
        kr[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        vr[r] = kr[r];
      }
    }
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      if (g < G) {
        float sc[kRegRows];
        float mt = -INFINITY;
#pragma unroll
        for (int r = 0; r < kRegRows; ++r) {
          float acc = q4[g].x * kr[r].x;
          acc = fmaf(q4[g].y, kr[r].y, acc);
          acc = fmaf(q4[g].z, kr[r].z, acc);
          acc = fmaf(q4[g].w, kr[r].w, acc);
          acc += __shfl_xor_sync(0xffffffffu, acc, 8);
          acc += __shfl_xor_sync(0xffffffffu, acc, 4);
          acc += __shfl_xor_sync(0xffffffffu, acc, 2);
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          sc[r] = rb + r < c1 ? acc * a.scale : -INFINITY;
          mt = fmaxf(mt, sc[r]);
        }
        const float mn = fmaxf(m_g[g], mt);
        const float alpha = m_g[g] == -INFINITY ? 0.f : expf(m_g[g] - mn);
        float4 o = make_float4(o4[g].x * alpha, o4[g].y * alpha, o4[g].z * alpha, o4[g].w * alpha);
        float ls = l_g[g] * alpha;
#pragma unroll
        for (int r = 0; r < kRegRows; ++r) {
          const float p = sc[r] == -INFINITY ? 0.f : expf(sc[r] - mn);
          ls += p;
          o.x = fmaf(p, vr[r].x, o.x);
          o.y = fmaf(p, vr[r].y, o.y);
          o.z = fmaf(p, vr[r].z, o.z);
          o.w = fmaf(p, vr[r].w, o.w);
        }
        o4[g] = o;
        l_g[g] = ls;
        m_g[g] = mn;
      }
    }
  }
  // the warp's two streams meet (lanes l16 and l16 + 16), then the warps
#pragma unroll
  for (int g = 0; g < GM; ++g) {
    if (g < G) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m_g[g], 16);
      const float l2 = __shfl_xor_sync(0xffffffffu, l_g[g], 16);
      float4 o2;
      o2.x = __shfl_xor_sync(0xffffffffu, o4[g].x, 16);
      o2.y = __shfl_xor_sync(0xffffffffu, o4[g].y, 16);
      o2.z = __shfl_xor_sync(0xffffffffu, o4[g].z, 16);
      o2.w = __shfl_xor_sync(0xffffffffu, o4[g].w, 16);
      const float M = fmaxf(m_g[g], m2);
      const float a1 = m_g[g] == -INFINITY ? 0.f : expf(m_g[g] - M);
      const float a2 = m2 == -INFINITY ? 0.f : expf(m2 - M);
      if (hw == 0) {
        float4 o;
        o.x = fmaf(o2.x, a2, o4[g].x * a1);
        o.y = fmaf(o2.y, a2, o4[g].y * a1);
        o.z = fmaf(o2.z, a2, o4[g].z * a1);
        o.w = fmaf(o2.w, a2, o4[g].w * a1);
        *reinterpret_cast<float4*>(wo + (warp * G + g) * d + 4 * l16) = o;
        if (l16 == 0) {
          wm[warp * GM + g] = M;
          wl[warp * GM + g] = fmaf(l2, a2, l_g[g] * a1);
        }
      }
    }
  }
  __syncthreads();
  // one thread per head: the CTA's (m, l); then o per (head, column)
  if (tid < G) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w * GM + tid]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = wm[w * GM + tid];
      L = fmaf(wl[w * GM + tid], mw == -INFINITY ? 0.f : expf(mw - M), L);
    }
    m_s[tid] = M;
    l_s[tid] = L;
  }
  __syncthreads();
  for (int idx = tid; idx < G * d; idx += kAttnThreads) {
    const int g = idx / d;
    const float M = m_s[g];
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = wm[w * GM + g];
      O = fmaf(wo[(w * G + g) * d + (idx % d)], mw == -INFINITY ? 0.f : expf(mw - M), O);
    }
    ofin[idx] = O;
  }
  __syncthreads();
  float* out = a.out + size_t(m) * a.nq * d + kvh * G * d;
  if (n_used == 1) {
    // the whole context in one CTA: finish here, no partials
    if (split == 0) {
      for (int idx = tid; idx < G * d; idx += kAttnThreads) {
        const float L = l_s[idx / d];
        out[idx] = L > 0.f ? ofin[idx] / L : 0.f;
      }
    }
    if (tid == 0) trace_mark(a.trace, 3);
    return;  // one-split launches need no ticket
  }
  // partial (m, l, o[d]) per head
  if (split < n_used) {
    float* part = a.part + ((size_t(m) * a.nkv + kvh) * a.nsplit + split) * G * (d + 2);
    for (int idx = tid; idx < G * d; idx += kAttnThreads)
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
  // combine: the per-split weights w = exp(m_s - max) once per (split, head)
  // in shared memory, then every output sums its column over the splits
  const float* pb = a.part + (size_t(m) * a.nkv + kvh) * a.nsplit * G * (d + 2);
  float* wts = wts_s;  // [G][n_used]
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < n_used; s += 32) mx = fmaxf(mx, __ldcg(pb + (s * G + g) * (d + 2)));
    mx = warp_max(mx);
    float L = 0.f;
    for (int s = lane; s < n_used; s += 32) {
      const float ms = __ldcg(pb + (s * G + g) * (d + 2));
      const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
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

// ---------------------------------------------------------------------------
// Prefill causal attention.  Template on head_dim; DPT dims per thread,
// TPR = D / DPT threads per query row.  Grid (n_q, ceil(T / rows_per_cta)).
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(
    const float* __restrict__ q, int64_t q_ld, const float* __restrict__ kc,
    const float* __restrict__ vc, int64_t T, int64_t pos0, int nq, int nkv, float scale,
    float* __restrict__ out, int64_t out_ld) {
  constexpr int DPT = D < 64 ? D : 64;
  constexpr int TPR = D / DPT;
  constexpr int ROWS = kAttnThreads / TPR;
  __shared__ float ks[kPTile][D];
  __shared__ float vs[kPTile][D];
  const int h = blockIdx.x;
  const int kvh = h / (nq / nkv);
  const int kvd = nkv * D;
  const int tid = threadIdx.x;
  const int rloc = tid / TPR, part = tid % TPR;
  const int64_t row = int64_t(blockIdx.y) * ROWS + rloc;
  const bool valid = row < T;
  const int64_t my_pos = pos0 + (valid ? row : 0);
  const int64_t last_row = (T - 1 < int64_t(blockIdx.y) * ROWS + ROWS - 1 ? T - 1 : int64_t(blockIdx.y) * ROWS + ROWS - 1);
  const int64_t n_keys = pos0 + last_row + 1;

  float qr[DPT], o[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) {
    qr[j] = valid ? q[row * q_ld + h * D + part * DPT + j] : 0.f;
    o[j] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;

  for (int64_t t0 = 0; t0 < n_keys; t0 += kPTile) {
    const int nt = int(n_keys - t0 < kPTile ? n_keys - t0 : kPTile);
    __syncthreads();
    for (int i = tid; i < kPTile * (D / 4); i += kAttnThreads) {
      const int t = i / (D / 4), j4 = i % (D / 4);
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;  // rows past nt: zeros, not
      if (t < nt) {                                              // stale smem (0 * NaN)
        kv4 = *reinterpret_cast<const float4*>(kc + (t0 + t) * kvd + kvh * D + j4 * 4);
        vv4 = *reinterpret_cast<const float4*>(vc + (t0 + t) * kvd + kvh * D + j4 * 4);
      }
      *reinterpret_cast<float4*>(&ks[t][j4 * 4]) = kv4;
      *reinterpret_cast<float4*>(&vs[t][j4 * 4]) = vv4;
    }
    __syncthreads();
    float s[kPTile];
    float mt = -INFINITY;
#pragma unroll
    for (int t = 0; t < kPTile; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < DPT; ++j) acc = fmaf(qr[j], ks[t][part * DPT + j], acc);
#pragma unroll
      for (int o2 = 1; o2 < TPR; o2 <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o2);
      const bool ok = t < nt && (t0 + t) <= my_pos;
      s[t] = ok ? acc * scale : -INFINITY;
      mt = fmaxf(mt, s[t]);
    }
    const float m_new = fmaxf(m_run, mt);
    if (m_new == -INFINITY) continue;  // nothing visible in this tile yet
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    float lsum = 0.f;
#pragma unroll
    for (int t = 0; t < kPTile; ++t) {
      s[t] = s[t] == -INFINITY ? 0.f : expf(s[t] - m_new);
      lsum += s[t];
    }
    l_run = l_run * alpha + lsum;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < DPT; ++j) {
      float acc = o[j] * alpha;
#pragma unroll
      for (int t = 0; t < kPTile; ++t) acc = fmaf(s[t], vs[t][part * DPT + j], acc);
      o[j] = acc;
    }
  }
  if (valid) {
    const float inv = 1.0f / l_run;
#pragma unroll
    for (int j = 0; j < DPT; ++j) out[row * out_ld + h * D + part * DPT + j] = o[j] * inv;
  }
}

// ---------------------------------------------------------------------------
// Prefill causal attention, register-tiled (head_dim a multiple of 64).  A CTA
// of 256 threads takes kPfBR query rows of one head (the longest row blocks
// launch first) and walks the visible keys in kPfBC-position tiles, K and V
// double-buffered in shared memory by cp.async.  Thread (ty, tx) = (tid / 16,
// tid % 16) owns rows ty + 16 i (i < 4): S = Q K^T as a 4 x 4 register tile
// over keys tx + 16 j (Q and K rows read as float4 along d; the K row stride
// D + 4 puts the 8 rows of a 16-byte phase on distinct banks), the row max
// and sum by shuffles over the 16 lanes that share a row, P through shared
// memory, then O += P V as a 4-row x (D / 16)-column register tile (columns
// tx * 4 + 64 c).  Every product is an f32 FMA; only the order of the sums
// differs from the reference's sequential ones.
// ---------------------------------------------------------------------------
constexpr int kPfBR = 64, kPfBC = 64, kPfThreads = 256;

template <int D>
constexpr size_t attn_prefill_tiled_smem() {
  return sizeof(float) * (size_t(kPfBR) * (D + 4) + 2 * size_t(kPfBC) * (D + 4) +
                          2 * size_t(kPfBC) * D + size_t(kPfBR) * (kPfBC + 4));
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 2) attn_prefill_tiled_kernel(
    const float* __restrict__ q, int64_t q_ld, const float* __restrict__ kc,
    const float* __restrict__ vc, int64_t T, int64_t pos0, int nq, int nkv, float scale,
    float* __restrict__ out, int64_t out_ld) {
  static_assert(D % 64 == 0, "columns are float4 groups of 16 lanes");
  constexpr int QS = D + 4, PS = kPfBC + 4, NC = D / 64, D4 = D / 4;
  extern __shared__ __align__(16) float pf_smem[];
  float* qs = pf_smem;                 // [kPfBR][QS]
  float* ks = qs + kPfBR * QS;         // [2][kPfBC][QS]
  float* vs = ks + 2 * kPfBC * QS;     // [2][kPfBC][D]
  float* ps = vs + 2 * kPfBC * D;      // [kPfBR][PS]
  const int h = blockIdx.x;
  const int kvh = h / (nq / nkv);
  const int64_t kvd = int64_t(nkv) * D;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t r0 = int64_t(gridDim.y - 1 - blockIdx.y) * kPfBR;
  const int64_t last_row = T - 1 < r0 + kPfBR - 1 ? T - 1 : r0 + kPfBR - 1;
  const int64_t n_keys = pos0 + last_row + 1;  // keys 0 .. n_keys-1 are visible to some row
  const int ntiles = int((n_keys + kPfBC - 1) / kPfBC);

  for (int i = tid; i < kPfBR * D4; i += kPfThreads) {
    const int r = i / D4, j4 = i % D4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < T) v = *reinterpret_cast<const float4*>(q + (r0 + r) * q_ld + int64_t(h) * D + j4 * 4);
    *reinterpret_cast<float4*>(qs + r * QS + j4 * 4) = v;
  }
  // positions past n_keys are zero-filled (never stale shared memory: 0 * NaN)
  auto load_tile = [&](int n, int b) {
    const int64_t t0 = int64_t(n) * kPfBC;
    float* kb = ks + b * kPfBC * QS;
    float* vb = vs + b * kPfBC * D;
    for (int i = tid; i < kPfBC * D4; i += kPfThreads) {
      const int t = i / D4, j4 = i % D4;
      float* kd = kb + t * QS + j4 * 4;
      float* vd = vb + t * D + j4 * 4;
      if (t0 + t < n_keys) {
        const int64_t off = (t0 + t) * kvd + int64_t(kvh) * D + j4 * 4;
        cp_async16(kd, kc + off);
        cp_async16(vd, vc + off);
      } else {
        *reinterpret_cast<float4*>(kd) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(vd) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };

  // a row's position, clamped so rows past T (not stored) see only real keys
  int64_t pos[4];
  float m_run[4], l_run[4], o[4][4 * NC];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t p = pos0 + r0 + ty + 16 * i;
    pos[i] = p < n_keys - 1 ? p : n_keys - 1;
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 4 * NC; ++c) o[i][c] = 0.f;
  }

  load_tile(0, 0);
  for (int n = 0; n < ntiles; ++n) {
    cp_async_wait<0>();
    __syncthreads();  // tile n (and the Q tile) visible; tile n-1's P.V finished
    if (n + 1 < ntiles) load_tile(n + 1, (n + 1) & 1);
    const float* kb = ks + (n & 1) * kPfBC * QS;
    const float* vb = vs + (n & 1) * kPfBC * D;
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll
    for (int k = 0; k < D; k += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(qs + (ty + 16 * i) * QS + k);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(kb + (tx + 16 * j) * QS + k);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float acc = s[i][j];
          acc = fmaf(a[i].x, b[j].x, acc);
          acc = fmaf(a[i].y, b[j].y, acc);
          acc = fmaf(a[i].z, b[j].z, acc);
          acc = fmaf(a[i].w, b[j].w, acc);
          s[i][j] = acc;
        }
    }
    const int64_t t0 = int64_t(n) * kPfBC;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mt = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = (t0 + tx + 16 * j) <= pos[i] ? s[i][j] * scale : -INFINITY;
        mt = fmaxf(mt, s[i][j]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_run[i], mt);
      const float alpha = m_run[i] == -INFINITY ? 0.f : expf(m_run[i] - m_new);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - m_new);
        ps[(ty + 16 * i) * PS + tx + 16 * j] = p;
        ls += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      l_run[i] = l_run[i] * alpha + ls;
      m_run[i] = m_new;
#pragma unroll
      for (int c = 0; c < 4 * NC; ++c) o[i][c] *= alpha;
    }
    __syncthreads();  // P visible
#pragma unroll 4
    for (int t = 0; t < kPfBC; t += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(ps + (ty + 16 * i) * PS + t);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const float4 v = *reinterpret_cast<const float4*>(vb + (t + e) * D + 64 * c + tx * 4);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = e == 0 ? pv[i].x : e == 1 ? pv[i].y : e == 2 ? pv[i].z : pv[i].w;
            o[i][4 * c + 0] = fmaf(p, v.x, o[i][4 * c + 0]);
            o[i][4 * c + 1] = fmaf(p, v.y, o[i][4 * c + 1]);
            o[i][4 * c + 2] = fmaf(p, v.z, o[i][4 * c + 2]);
            o[i][4 * c + 3] = fmaf(p, v.w, o[i][4 * c + 3]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t row = r0 + ty + 16 * i;
    if (row < T) {
      const float inv = 1.0f / l_run[i];
#pragma unroll
      for (int c = 0; c < NC; ++c)
        *reinterpret_cast<float4*>(out + row * out_ld + int64_t(h) * D + 64 * c + tx * 4) =
            make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv, o[i][4 * c + 2] * inv,
                        o[i][4 * c + 3] * inv);
    }
  }
}

// RoPE of q and k for T prefill rows + KV append (model.rs:533-553).
// Grid (T); threads over (heads x half).
__global__ void rope_append_kernel(float* qkv, int64_t ld, int nq, int nkv, int d,
                                   const float* __restrict__ cs, const float* __restrict__ sn,
                                   int64_t pos0, float* kc, float* vc) {
  const int64_t t = blockIdx.x;
  const int64_t pos = pos0 + t;
  const int half = d / 2, kvd = nkv * d;
  float* row = qkv + t * ld;
  for (int i = threadIdx.x; i < (nq + nkv) * half; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    float* v = row + hh * d;
    float o0, o1;
    rot(v[j], v[j + half], cs[pos * half + j], sn[pos * half + j], &o0, &o1);
    if (hh < nq) {
      v[j] = o0;
      v[j + half] = o1;
    } else {
      float* kdst = kc + pos * kvd + (hh - nq) * d;
      kdst[j] = o0;
      kdst[j + half] = o1;
    }
  }
  const float* vsrc = row + (nq + nkv) * d;
  for (int j = threadIdx.x; j < kvd; j += blockDim.x) vc[pos * kvd + j] = vsrc[j];
}

__global__ void rope_rows_kernel(float* x, int64_t ld, int n_heads, int d,
                                 const float* __restrict__ cs, const float* __restrict__ sn,
                                 int64_t pos0) {
  const int64_t t = blockIdx.x, pos = pos0 + t;
  const int half = d / 2;
  float* row = x + t * ld;
  for (int i = threadIdx.x; i < n_heads * half; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    float* v = row + hh * d;
    float o0, o1;
    rot(v[j], v[j + half], cs[pos * half + j], sn[pos * half + j], &o0, &o1);
    v[j] = o0;
    v[j + half] = o1;
  }
}

}  // namespace

int attn_decode_nsplit(int nkv, int M, int64_t cap, int num_sms) {
  // enough CTAs to fill the GPU, and for long contexts at most ~512
  // positions (8 tiles) per split
  const int64_t fill = (int64_t(num_sms) * 8 + int64_t(nkv) * M - 1) / (int64_t(nkv) * M);
  const int64_t want = std::max<int64_t>(fill, (cap + 511) / 512);
  const int64_t maxs = (cap + kTile - 1) / kTile;
  int64_t n = std::min<int64_t>(want, maxs);
  return int(std::max<int64_t>(1, std::min<int64_t>(n, 1024)));
}

constexpr int kMaxAttnSmem = 96 * 1024;

template <int D>
cudaError_t attn_attr() {
  TMG_CUDA_TRY(set_carveout(attn_prefill_kernel<D>));
  TMG_CUDA_TRY((set_carveout(attn_decode_kernel<D, 4>, kMaxAttnSmem)));
  return set_carveout(attn_decode_kernel<D, 16>, kMaxAttnSmem);
}

cudaError_t attn_prepare() {
  TMG_CUDA_TRY(set_carveout(attn_decode_reg_kernel));
  TMG_CUDA_TRY(set_carveout(attn_prefill_tiled_kernel<64>, int(attn_prefill_tiled_smem<64>())));
  TMG_CUDA_TRY(set_carveout(rope_append_kernel));
  TMG_CUDA_TRY(set_carveout(rope_rows_kernel));
  TMG_CUDA_TRY(attn_attr<16>());
  TMG_CUDA_TRY(attn_attr<32>());
  TMG_CUDA_TRY(attn_attr<64>());
  return attn_attr<128>();
}

// The shapes launch_attn_decode takes (checked before anything is enqueued
// by the op entry points): head dim 16/32/64/128, at most 16 query heads
// per kv head, and the tiled kernel's shared memory within kMaxAttnSmem.
bool attn_decode_shape_ok(int nq, int nkv, int d, int64_t n_ctx, int nsplit, std::string* why) {
  if (nkv <= 0 || nq <= 0 || nq % nkv) {
    *why = "n_q must be a positive multiple of n_kv";
    return false;
  }
  const int G = nq / nkv;
  if (d != 16 && d != 32 && d != 64 && d != 128) {
    *why = "head_dim must be 16, 32, 64 or 128";
    return false;
  }
  if (G > 16 || G * d > 8 * kAttnThreads) {
    *why = "at most 16 query heads per kv head (and n_q/n_kv * head_dim <= 1024)";
    return false;
  }
  if (n_ctx < 1 || n_ctx > int64_t(INT32_MAX)) {
    *why = "n_ctx must be in [1, 2^31 - 1]";
    return false;
  }
  const size_t gp = (size_t(G) + 3) & ~size_t(3);
  const size_t ks = d >= 32 ? size_t(d) : size_t(d) + 16;
  const size_t tiles = size_t(G) * d + size_t(kAttnBufs) * kTileD * ks +
                       size_t(kAttnBufs) * kTileD * d + kTileD * gp + 2 * size_t(d);
  if (sizeof(float) * std::max<size_t>(tiles, size_t(G) * nsplit) > size_t(kMaxAttnSmem)) {
    *why = "shape needs more shared memory than the decode attention kernel has";
    return false;
  }
  return true;
}

cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t s, bool pdl) {
  const int G = a.nq / a.nkv;
  if (G * a.nkv != a.nq || G * a.d > 8 * kAttnThreads || G > 16) return cudaErrorInvalidValue;
  // head dim 64 or 128 with at most 4 heads per kv head: the TMA-staged
  // kernel (attn_tma.cu).  TMG_ATTN_KERNEL=reg / tiled selects the
  // register-streaming kernel (head dim 64) or the cp.async tiled one, for
  // comparison.
  static const int choice = [] {
    const char* e = getenv("TMG_ATTN_KERNEL");
    if (e && std::strcmp(e, "reg") == 0) return 1;
    if (e && std::strcmp(e, "tiled") == 0) return 2;
    const char* t = getenv("TMG_ATTN_TILED");
    return t && t[0] == '1' ? 2 : 0;
  }();
  if (choice == 0 && attn_decode_tma_ok(a.nq, a.nkv, a.d, a.cap, a.M, a.kc, a.vc) &&
      size_t(G) * a.nsplit * 4 <= attn_decode_tma_smem(a.d))
    return launch_attn_decode_tma(a, s, pdl);
  if (a.d == 64 && G <= 4 && choice != 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nkv, a.nsplit, a.M);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = sizeof(float) * std::max<size_t>(4, size_t(G) * a.nsplit);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_decode_reg_kernel, a);
  }
  void (*kern)(const AttnDecodeArgs) = nullptr;
  const bool g4 = G <= 4;
  switch (a.d) {
    case 16: kern = g4 ? attn_decode_kernel<16, 4> : attn_decode_kernel<16, 16>; break;
    case 32: kern = g4 ? attn_decode_kernel<32, 4> : attn_decode_kernel<32, 16>; break;
    case 64: kern = g4 ? attn_decode_kernel<64, 4> : attn_decode_kernel<64, 16>; break;
    case 128: kern = g4 ? attn_decode_kernel<128, 4> : attn_decode_kernel<128, 16>; break;
    default: return cudaErrorInvalidValue;
  }
  // tiles, or the combine's per-split weights when those are larger
  const size_t gp = (size_t(G) + 3) & ~size_t(3);
  const size_t ks = a.d >= 32 ? size_t(a.d) : size_t(a.d) + 16;  // attn_kstride<D>()
  const size_t tiles = size_t(G) * a.d + size_t(kAttnBufs) * kTileD * ks +
                       size_t(kAttnBufs) * kTileD * a.d + kTileD * gp + 2 * size_t(a.d);
  // (the end-of-loop combine of the warps reuses the K and V tiles)
  const size_t smem = sizeof(float) * std::max<size_t>(tiles, size_t(G) * a.nsplit);
  if (smem > size_t(kMaxAttnSmem)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.nkv, a.nsplit, a.M);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_attn_prefill(const float* q, int64_t q_ld, const float* kc, const float* vc,
                                int64_t T, int64_t pos0, int nq, int nkv, int d, float scale,
                                float* out, int64_t out_ld, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  // the register-tiled kernel reads q and writes out as float4 rows
  const bool vec = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) == 0 &&
                   q_ld % 4 == 0 && out_ld % 4 == 0;
  if (d == 64 && vec && nkv > 0 && nq % nkv == 0) {
    dim3 grid(nq, unsigned((T + kPfBR - 1) / kPfBR));
    attn_prefill_tiled_kernel<64><<<grid, kPfThreads, attn_prefill_tiled_smem<64>(), s>>>(
        q, q_ld, kc, vc, T, pos0, nq, nkv, scale, out, out_ld);
    return cudaGetLastError();
  }
  switch (d) {
#define TMG_ATTN_CASE(D)                                                                   \
  case D: {                                                                                \
    constexpr int ROWS = kAttnThreads / (D / (D < 64 ? D : 64));                           \
    dim3 grid(nq, unsigned((T + ROWS - 1) / ROWS));                                        \
    attn_prefill_kernel<D><<<grid, kAttnThreads, 0, s>>>(q, q_ld, kc, vc, T, pos0, nq, nkv, \
                                                         scale, out, out_ld);              \
    return cudaGetLastError();                                                             \
  }
    TMG_ATTN_CASE(16)
    TMG_ATTN_CASE(32)
    TMG_ATTN_CASE(64)
    TMG_ATTN_CASE(128)
#undef TMG_ATTN_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rope_append(float* qkv, int64_t qkv_ld, int64_t T, int nq, int nkv, int d,
                               const float* rope_cos, const float* rope_sin, int64_t pos0,
                               float* kc, float* vc, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  rope_append_kernel<<<unsigned(T), 256, 0, s>>>(qkv, qkv_ld, nq, nkv, d, rope_cos, rope_sin, pos0,
                                                 kc, vc);
  return cudaGetLastError();
}

cudaError_t launch_rope_rows(float* x, int64_t ld, int64_t rows, int n_heads, int d,
                             const float* rope_cos, const float* rope_sin, int64_t pos0,
                             cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  rope_rows_kernel<<<unsigned(rows), 256, 0, s>>>(x, ld, n_heads, d, rope_cos, rope_sin, pos0);
  return cudaGetLastError();
}

}  // namespace tmg
