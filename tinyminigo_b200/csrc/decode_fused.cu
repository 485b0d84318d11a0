// Fused batch-1 decode: n_steps greedy steps of generate's loop
// (src/model.rs:631-656: forward_token, src/model.rs:392-491, then argmax,
// src/tensor.rs:1063-1073) in ONE persistent kernel.
//
// One CTA per SM (cooperative launch), 9 warps:
//  * a producer warp streams, in consumption order, every weight row this
//    CTA needs for all n_steps tokens -- q/k/v, o, gate/up, down of each
//    layer, then the LM head -- through a ring of 32 KB shared-memory stages
//    with cp.async.bulk (TMA) and mbarriers.  Weights never depend on
//    activations, so this stream runs ahead of the math, across phase and
//    token boundaries, limited only by free ring stages: HBM stays busy
//    while the consumers sit at a grid barrier.
//  * eight consumer warps run the phases of each layer, each followed by a
//    grid barrier (bounded spin; a barrier that gives up sets the error word
//    and every CTA leaves):
//      QKV   rmsnorm(x) . Wqkv^T           -> qkv          (rows split over CTAs)
//      ATTN  RoPE, KV append at pos, split-KV attention   -> partials
//      O     combine partials, . Wo^T      -> x += ...
//      GU    rmsnorm(x) . Wgate^T, Wup^T   -> act = silu(g) * u
//      DOWN  act . Wdown^T                 -> x += ...
//    then HEAD: rmsnorm(x) . Wlm^T -> logits + per-CTA argmax; after one more
//    barrier every CTA reduces the argmax (the same token everywhere), CTA 0
//    records it, and the next token starts.
// Row groups of a phase are dealt to CTAs round-robin with a rotating offset
// so every CTA streams the same number of bytes per token within one group.
// All arithmetic is f32 with BF16 weights widened exactly, as in the
// separate kernels; cross-CTA activations are read through L2 (ld.cg).
#include <math.h>

#include "common.cuh"
#include "fused.cuh"

namespace tmg {

namespace {

constexpr int kCWarps = 8;                         // consumer warps
constexpr int kCThreads = kCWarps * kWarp;         // 256
constexpr int kFThreads = kCThreads + kWarp;       // + producer warp
constexpr int kStage = 32 * 1024;                  // ring stage bytes
constexpr int kMaxStagesF = 6;
constexpr int kTileF = 64;                         // attention positions per tile
constexpr int kMaxDefer = 512;                     // deferred residual rows per phase

enum Phase : int { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_HEAD = 4 };

__device__ __forceinline__ void csync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");
}

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

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

__device__ __forceinline__ void rot(float a, float b, float c, float s, float* o0, float* o1) {
  float ac = __fmul_rn(a, c), bs = __fmul_rn(b, s), as = __fmul_rn(a, s), bc = __fmul_rn(b, c);
  *o0 = __fsub_rn(ac, bs);
  *o1 = __fadd_rn(as, bc);
}

// The geometry of one GEMV phase: rows of K elements in groups of `rpc` row
// slots (for SwiGLU, rpg gate rows + rpg up rows), one 32 KB stage each.
struct PhaseGeo {
  const uint16_t* w;
  const uint16_t* w2;
  int64_t N;       // output rows
  int K;
  int ks;          // K split over warps
  int chunks;      // 256-element chunks per warp segment
  int rpc;         // row slots per group (8 / ks)
  int rpg;         // output rows per group
  int64_t ngroups;
  uint32_t bytes;  // stage bytes of a full group
};

__device__ __forceinline__ PhaseGeo geo(const FusedArgs& a, int ph, int l) {
  PhaseGeo g;
  const FusedLayer& L = a.layers[l];
  g.w2 = nullptr;
  switch (ph) {
    case PH_QKV: g.w = L.wqkv; g.N = (a.nq + 2 * a.nkv) * a.d; g.K = a.h; break;
    case PH_O: g.w = L.wo; g.N = a.h; g.K = a.nq * a.d; break;
    case PH_GU: g.w = L.wg; g.w2 = L.wu; g.N = a.I; g.K = a.h; break;
    case PH_DOWN: g.w = L.wd; g.N = a.h; g.K = a.I; break;
    default: g.w = a.lm_head; g.N = a.V; g.K = a.h; break;
  }
  g.ks = 1;
  while (g.K / g.ks > 2048) g.ks *= 2;
  g.chunks = g.K / g.ks / 256;
  g.rpc = kCWarps / g.ks;
  g.rpg = ph == PH_GU ? g.rpc / 2 : g.rpc;
  g.ngroups = (g.N + g.rpg - 1) / g.rpg;
  g.bytes = uint32_t(g.rpc) * g.K * 2;
  return g;
}

// First group of this CTA in a phase whose groups start at rotation `off`.
__device__ __forceinline__ int64_t first_group(int off) {
  const int n = gridDim.x;
  return int64_t(((int(blockIdx.x) - off) % n + n) % n);
}

struct Shared {
  uint64_t full[kMaxStagesF];
  uint64_t empty[kMaxStagesF];
  float part[2][kCWarps];
  float ssq[kCWarps];
  unsigned long long best[kCWarps];
  float defer_v[kMaxDefer];
  float defer_old[kMaxDefer];
  int gen_ok;
  volatile int abort;      // consumers -> producer: stop issuing
  volatile int issued;     // producer: stages issued so far
  volatile int prod_done;  // producer: no more stages will be issued
  float m_s[8], l_s[8], alpha_s[8];
};

// ---------------------------------------------------------------------------
// Grid barrier among the consumer warps of all CTAs.  Generation counting,
// reusable across launches; every wait is bounded in time.
// ---------------------------------------------------------------------------
__device__ bool grid_sync(const FusedArgs& a, unsigned int& gen, Shared& S) {
  csync();
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    const unsigned int g = gen;
    if (atomicAdd(&a.bar[0], 1u) == gridDim.x - 1) {
      atomicExch(&a.bar[0], 0u);
      __threadfence();
      atomicExch(&a.bar[1], g + 1);
    } else {
      const unsigned long long t0 = global_ns();
      unsigned int spins = 0;
      while (ld_acquire(&a.bar[1]) == g) {
        if ((++spins & 255) == 0) {
          if (ld_acquire(&a.bar[2]) != 0 || global_ns() - t0 > kWaitNs) {
            ok = 0;
            break;
          }
        }
      }
    }
    gen = g + 1;
    __threadfence();
    if (!ok) {
      atomicExch(&a.bar[2], 1u);
      if (a.err) atomicExch(a.err, 2);
    }
    S.gen_ok = ok;
  }
  csync();
  return S.gen_ok != 0;
}

// ---------------------------------------------------------------------------
// Producer: the weight stream of all steps, in consumption order.
// ---------------------------------------------------------------------------
__device__ void producer(const FusedArgs& a, Shared& S, uint8_t* ring, int nst) {
  int it = 0;
  int off = 0;
  for (int step = 0; step < a.n_steps; ++step) {
    for (int l = 0; l <= a.L; ++l) {
      for (int ph = (l == a.L ? PH_HEAD : PH_QKV); ph <= (l == a.L ? PH_HEAD : PH_DOWN); ++ph) {
        const PhaseGeo g = geo(a, ph, l < a.L ? l : 0);
        for (int64_t grp = first_group(off); grp < g.ngroups; grp += gridDim.x, ++it) {
          const int s = it % nst;
          const uint32_t par = (it / nst) & 1;
          if (S.abort) return;
          if (!mbar_wait(&S.empty[s], par ^ 1)) {
            S.abort = 1;
            if (a.err) atomicExch(a.err, 2);
            return;
          }
          uint8_t* dst = ring + size_t(s) * kStage;
          const int64_t r0 = grp * g.rpg;
          const int64_t nr = min(int64_t(g.rpg), g.N - r0);
          const uint32_t bytes = uint32_t(nr) * g.K * 2;
          mbar_expect_tx(&S.full[s], ph == PH_GU ? 2 * bytes : bytes);
          bulk_g2s(dst, g.w + r0 * g.K, bytes, &S.full[s]);
          if (ph == PH_GU) bulk_g2s(dst + size_t(g.rpg) * g.K * 2, g.w2 + r0 * g.K, bytes, &S.full[s]);
          S.issued = it + 1;
        }
        off = int((off + g.ngroups) % gridDim.x);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
struct XSeg {
  float4 a[8], b[8];
};

// Load this warp's K segment of the phase input into registers: from the
// staged (normalised) x in shared memory or straight from global memory.
__device__ __forceinline__ void load_seg(XSeg& x, const float* src, bool via_l2, int kbase,
                                         int chunks, int lane) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < chunks) {
      const int k = kbase + c * 256 + lane * 8;
      if (via_l2) {
        x.a[c] = ldcg4(src + k);
        x.b[c] = ldcg4(src + k + 4);
      } else {
        x.a[c] = *reinterpret_cast<const float4*>(src + k);
        x.b[c] = *reinterpret_cast<const float4*>(src + k + 4);
      }
    }
  }
}

// rmsnorm of v[0..n) (already in shared memory `xs`) in place:
// v * inv * w (rms_norm_into's order).
__device__ __forceinline__ void norm_in_smem(float* xs, const float* w, int n, float eps, Shared& S) {
  float ss = 0.f;
  for (int k = threadIdx.x; k < n; k += kCThreads) ss = fmaf(xs[k], xs[k], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) S.ssq[threadIdx.x >> 5] = ss;
  csync();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kCWarps; ++i) tot += S.ssq[i];
  const float inv = 1.0f / sqrtf(tot / float(n) + eps);
  for (int k = threadIdx.x; k < n; k += kCThreads) {
    const float t = xs[k] * inv;
    xs[k] = t * __ldg(w + k);
  }
  csync();
}

// One GEMV phase over this CTA's groups.  EPI: 0 store y, 1 deferred
// residual add into y, 2 SwiGLU into y, 3 LM head (store + argmax).
template <int EPI>
__device__ __forceinline__ bool gemv_phase(const PhaseGeo& g, const XSeg& x, float* y, int off, int& it, int nst,
                           uint8_t* ring, Shared& S, unsigned long long& best, int& n_def) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = warp % g.ks, slot = warp / g.ks;
  const int kbase = ks * g.chunks * 256;
  const bool need_sync = g.ks > 1 || EPI == 2;
  int k_local = 0;
  for (int64_t grp = first_group(off); grp < g.ngroups; grp += gridDim.x, ++it, ++k_local) {
    const int s = it % nst;
    const uint32_t par = (it / nst) & 1;
    const int64_t r0 = grp * g.rpg;
    const int rslot = EPI == 2 ? slot % g.rpg : slot;
    const bool valid = r0 + rslot < g.N;
    float acc = 0.f;
    const bool ok = !S.abort && mbar_wait(&S.full[s], par);
    if (ok && valid) {
      const uint16_t* wr = reinterpret_cast<const uint16_t*>(ring + size_t(s) * kStage +
                                                             size_t(slot) * g.K * 2) +
                           kbase + lane * 8;
      float sacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c < g.chunks) fma8(x.a[c], x.b[c], *reinterpret_cast<const uint4*>(wr + c * 256), sacc);
      acc = sum8(sacc);
    }
    if (!ok && lane == 0) S.abort = 1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    acc = warp_sum(acc);
    if (need_sync) {
      if (lane == 0) S.part[it & 1][warp] = acc;
      csync();
    }
    if (lane == 0 && ks == 0 && valid && (EPI != 2 || slot < g.rpg)) {
      for (int j = 1; j < g.ks; ++j) acc += S.part[it & 1][warp + j];
      const int64_t r = r0 + rslot;
      if (EPI == 2) {
        float up = 0.f;
        for (int j = 0; j < g.ks; ++j) up += S.part[it & 1][(slot + g.rpg) * g.ks + j];
        const float sg = acc / (1.0f + expf(-acc));
        y[r] = sg * up;
      } else if (EPI == 1) {
        S.defer_v[k_local * g.rpg + rslot] = acc;
      } else {
        y[r] = acc;
        if (EPI == 3) {
          const unsigned long long kk = argmax_key(acc, uint32_t(r));
          best = kk > best ? kk : best;
        }
      }
    }
  }
  if (EPI == 1) n_def = k_local * g.rpg;
  return !S.abort;
}

// Prefetch the residual rows this CTA will update in a deferred-add phase.
__device__ __forceinline__ void prefetch_residual(const PhaseGeo& g, const float* x, int off, Shared& S) {
  const int64_t f = first_group(off);
  const int64_t my_groups = f < g.ngroups ? (g.ngroups - 1 - f) / gridDim.x + 1 : 0;
  const int n = int(my_groups) * g.rpg;
  for (int k = threadIdx.x; k < n && k < kMaxDefer; k += kCThreads) {
    const int64_t r = (f + int64_t(k / g.rpg) * gridDim.x) * g.rpg + k % g.rpg;
    S.defer_old[k] = r < g.N ? ldcg(x + r) : 0.f;
  }
}

__device__ __forceinline__ void apply_residual(const PhaseGeo& g, float* x, int off, int n_def, Shared& S) {
  csync();
  const int64_t f = first_group(off);
  for (int k = threadIdx.x; k < n_def && k < kMaxDefer; k += kCThreads) {
    const int64_t r = (f + int64_t(k / g.rpg) * gridDim.x) * g.rpg + k % g.rpg;
    if (r < g.N) x[r] = S.defer_old[k] + S.defer_v[k];
  }
}

// Attention partials of one (kv head, split) item: RoPE, KV append by the
// owner of pos, online softmax over the split's positions.
template <int D>
__device__ __forceinline__ void attn_item(const FusedArgs& a, const FusedLayer& L, int kvh, int split, int chunk,
                          int n_ctx, int pos, bool append, float* sm, Shared& S) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.nq / a.nkv, half = D / 2, kvd = a.nkv * D;
  float* qs = sm;                       // [G][D]
  float* ks_ = qs + G * D;              // [kTileF][D+4]
  float* vs = ks_ + kTileF * (D + 4);   // [kTileF][D]
  float* ps = vs + kTileF * D;          // [G][kTileF]
  const int c0 = split * chunk, c1 = min(n_ctx, c0 + chunk);
  const bool own = append && pos >= c0 && pos < c1;
  const int64_t rp = pos < a.cap ? pos : a.cap - 1;  // the host keeps pos < cap
  for (int i = tid; i < G * half; i += kCThreads) {
    const int g = i / half, j = i % half;
    const float* qh = a.qkv + (kvh * G + g) * D;
    float o0, o1;
    rot(ldcg(qh + j), ldcg(qh + j + half), a.rope_cos[rp * half + j], a.rope_sin[rp * half + j],
        &o0, &o1);
    qs[g * D + j] = o0;
    qs[g * D + j + half] = o1;
  }
  if (own) {
    const float* kh = a.qkv + a.nq * D + kvh * D;
    const float* vh = a.qkv + (a.nq + a.nkv) * D + kvh * D;
    for (int j = tid; j < half; j += kCThreads) {
      float o0, o1;
      rot(ldcg(kh + j), ldcg(kh + j + half), a.rope_cos[size_t(pos) * half + j],
          a.rope_sin[size_t(pos) * half + j], &o0, &o1);
      L.kc[size_t(pos) * kvd + kvh * D + j] = o0;
      L.kc[size_t(pos) * kvd + kvh * D + j + half] = o1;
    }
    for (int j = tid; j < D; j += kCThreads) L.vc[size_t(pos) * kvd + kvh * D + j] = ldcg(vh + j);
  }
  if (tid < G) {
    S.m_s[tid] = -INFINITY;
    S.l_s[tid] = 0.f;
  }
  float o_acc[4] = {0.f, 0.f, 0.f, 0.f};  // G * D <= 1024 outputs, tid + 256 r
  csync();  // the append is visible to this CTA's tile loads
  for (int t0 = c0; t0 < c1; t0 += kTileF) {
    const int nt = min(kTileF, c1 - t0);
    for (int i = tid; i < nt * (D / 4); i += kCThreads) {
      const int t = i / (D / 4), j4 = i % (D / 4);
      cp_async16(ks_ + t * (D + 4) + j4 * 4, L.kc + size_t(t0 + t) * kvd + kvh * D + j4 * 4);
      cp_async16(vs + t * D + j4 * 4, L.vc + size_t(t0 + t) * kvd + kvh * D + j4 * 4);
    }
    cp_async_wait_all();
    csync();
    if (warp < G) {
      const int g = warp;
      const float* qr = qs + g * D;
      float sc[2];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int t = lane + 32 * h2;
        sc[h2] = -INFINITY;
        if (t < nt) {
          const float* kr = ks_ + t * (D + 4);
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
          for (int j = 0; j < D; j += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(kr + j);
            const float4 q4 = *reinterpret_cast<const float4*>(qr + j);
            a0 = fmaf(q4.x, k4.x, a0);
            a1 = fmaf(q4.y, k4.y, a1);
            a2 = fmaf(q4.z, k4.z, a2);
            a3 = fmaf(q4.w, k4.w, a3);
          }
          sc[h2] = ((a0 + a1) + (a2 + a3)) * a.scale;
        }
      }
      const float mt = warp_max(fmaxf(sc[0], sc[1]));
      const float m_old = S.m_s[g];
      const float m_new = fmaxf(m_old, mt);
      const float p0 = lane < nt ? expf(sc[0] - m_new) : 0.f;
      const float p1 = lane + 32 < nt ? expf(sc[1] - m_new) : 0.f;
      const float lsum = warp_sum(p0 + p1);
      ps[g * kTileF + lane] = p0;
      ps[g * kTileF + lane + 32] = p1;
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
        S.alpha_s[g] = alpha;
        S.l_s[g] = S.l_s[g] * alpha + lsum;
        S.m_s[g] = m_new;
      }
    }
    csync();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int idx = tid + r * kCThreads;
      if (idx < G * D) {
        const int g = idx / D, j = idx % D;
        float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        int t = 0;
        for (; t + 4 <= nt; t += 4) {
          b0 = fmaf(ps[g * kTileF + t], vs[t * D + j], b0);
          b1 = fmaf(ps[g * kTileF + t + 1], vs[(t + 1) * D + j], b1);
          b2 = fmaf(ps[g * kTileF + t + 2], vs[(t + 2) * D + j], b2);
          b3 = fmaf(ps[g * kTileF + t + 3], vs[(t + 3) * D + j], b3);
        }
        for (; t < nt; ++t) b0 = fmaf(ps[g * kTileF + t], vs[t * D + j], b0);
        o_acc[r] = fmaf(o_acc[r], S.alpha_s[g], (b0 + b1) + (b2 + b3));
      }
    }
    csync();
  }
  float* part = a.part + (size_t(kvh) * a.nsplit + split) * G * (D + 2);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int idx = tid + r * kCThreads;
    if (idx < G * D) part[(idx / D) * (D + 2) + 2 + (idx % D)] = o_acc[r];
  }
  if (tid < G) {
    part[tid * (D + 2)] = S.m_s[tid];
    part[tid * (D + 2) + 1] = S.l_s[tid];
  }
  csync();
}

// attention output (q_dim floats) into shared memory from the partials.
template <int D>
__device__ __forceinline__ void combine(const FusedArgs& a, int n_used, float* out, float* wts, Shared& S) {
  const int G = a.nq / a.nkv, tid = threadIdx.x;
  const int nh = a.nkv * G;  // query heads
  // per (kv head, g): the weights exp(m_s - max) of the used splits
  for (int hq = tid; hq < nh; hq += kCThreads) {
    const int kvh = hq / G, g = hq % G;
    const float* pb = a.part + size_t(kvh) * a.nsplit * G * (D + 2) + g * (D + 2);
    float mx = -INFINITY;
    for (int s = 0; s < n_used; ++s) mx = fmaxf(mx, ldcg(pb + size_t(s) * G * (D + 2)));
    float L = 0.f;
    for (int s = 0; s < n_used; ++s) {
      const float ms = ldcg(pb + size_t(s) * G * (D + 2));
      const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
      wts[hq * n_used + s] = w;
      L = fmaf(ldcg(pb + size_t(s) * G * (D + 2) + 1), w, L);
    }
    wts[nh * n_used + hq] = L;
  }
  csync();
  for (int idx = tid; idx < nh * D; idx += kCThreads) {
    const int hq = idx / D, j = idx % D, kvh = hq / G, g = hq % G;
    const float* pb = a.part + size_t(kvh) * a.nsplit * G * (D + 2) + g * (D + 2) + 2 + j;
    float acc = 0.f;
    for (int s = 0; s < n_used; ++s) acc = fmaf(ldcg(pb + size_t(s) * G * (D + 2)), wts[hq * n_used + s], acc);
    const float L = wts[nh * n_used + hq];
    out[idx] = L > 0.f ? acc / L : 0.f;
  }
  csync();
}

template <int D>
__global__ void __launch_bounds__(kFThreads, 1) decode_fused_kernel(const FusedArgs a, int nst) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ Shared S;
  uint8_t* ring = dsm;
  float* xs = reinterpret_cast<float*>(dsm + size_t(nst) * kStage);  // max(h, q_dim, I) floats
  float* asm_ = xs + a.xs_floats;  // attention tiles / combine weights
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], kCWarps);
    }
    S.abort = 0;
    S.issued = 0;
    S.prod_done = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kCWarps) {
    if (lane == 0) {
      producer(a, S, ring, nst);
      __threadfence_block();
      S.prod_done = 1;
    }
    return;
  }

  // ---------------- consumers ----------------
  unsigned int gen = 0;
  if (threadIdx.x == 0) gen = ld_acquire(&a.bar[1]);
  const StreamState& st = a.st;
  int pos = st.pos[0];
  int done = st.done[0];
  int n_gen = st.n_gen[0];
  uint32_t tok = st.token[0];
  const int G = a.nq / a.nkv;
  int it = 0, off = 0;
  bool ok = true;
  XSeg x;  // this warp's K segment of the current phase's input
  for (int step = 0; step < a.n_steps && ok && !done; ++step) {
    const bool append = pos < a.cap;
    const int n_ctx = append ? pos + 1 : pos;
    int chunk = (n_ctx + a.nsplit - 1) / a.nsplit;
    chunk = max(kTileF, (chunk + kTileF - 1) / kTileF * kTileF);
    const int n_used = (n_ctx + chunk - 1) / chunk;
    for (int l = 0; l < a.L && ok; ++l) {
      const FusedLayer& Lw = a.layers[l];
      // ---- QKV: x (the embedding row at layer 0) -> rmsnorm -> Wqkv ----
      {
        const PhaseGeo g = geo(a, PH_QKV, l);
        if (l == 0) {
          const uint16_t* erow = a.embed + size_t(tok) * a.h;
          for (int k = threadIdx.x; k < a.h; k += kCThreads) {
            const float v = bf16f(erow[k]);
            xs[k] = v;
            if (blockIdx.x == 0) a.x[k] = v;
          }
        } else {
          for (int k = threadIdx.x; k < a.h; k += kCThreads) xs[k] = ldcg(a.x + k);
        }
        csync();
        norm_in_smem(xs, Lw.in_norm, a.h, a.eps, S);
        load_seg(x, xs, false, (warp % g.ks) * g.chunks * 256, g.chunks, lane);
        unsigned long long b = 0;
        int nd = 0;
        ok = gemv_phase<0>(g, x, a.qkv, off, it, nst, ring, S, b, nd);
        off = int((off + g.ngroups) % gridDim.x);
        ok = ok && grid_sync(a, gen, S);
      }
      if (!ok) break;
      // ---- ATTN: partials per (kv head, split) item ----
      for (int item = blockIdx.x; item < a.nkv * n_used; item += gridDim.x)
        attn_item<D>(a, Lw, item / n_used, item % n_used, chunk, n_ctx, pos, append, asm_, S);
      ok = grid_sync(a, gen, S);
      if (!ok) break;
      // ---- O: combine -> Wo -> x += ----
      {
        const PhaseGeo g = geo(a, PH_O, l);
        prefetch_residual(g, a.x, off, S);
        combine<D>(a, n_used, xs, asm_, S);
        load_seg(x, xs, false, (warp % g.ks) * g.chunks * 256, g.chunks, lane);
        unsigned long long b = 0;
        int nd = 0;
        ok = gemv_phase<1>(g, x, a.x, off, it, nst, ring, S, b, nd);
        apply_residual(g, a.x, off, nd, S);
        off = int((off + g.ngroups) % gridDim.x);
        ok = ok && grid_sync(a, gen, S);
      }
      if (!ok) break;
      // ---- GU: rmsnorm(x) -> Wgate, Wup -> act ----
      {
        const PhaseGeo g = geo(a, PH_GU, l);
        for (int k = threadIdx.x; k < a.h; k += kCThreads) xs[k] = ldcg(a.x + k);
        csync();
        norm_in_smem(xs, Lw.post_norm, a.h, a.eps, S);
        load_seg(x, xs, false, (warp % g.ks) * g.chunks * 256, g.chunks, lane);
        unsigned long long b = 0;
        int nd = 0;
        ok = gemv_phase<2>(g, x, a.act, off, it, nst, ring, S, b, nd);
        off = int((off + g.ngroups) % gridDim.x);
        ok = ok && grid_sync(a, gen, S);
      }
      if (!ok) break;
      // ---- DOWN: act -> Wdown -> x += ----
      {
        const PhaseGeo g = geo(a, PH_DOWN, l);
        prefetch_residual(g, a.x, off, S);
        load_seg(x, a.act, true, (warp % g.ks) * g.chunks * 256, g.chunks, lane);
        unsigned long long b = 0;
        int nd = 0;
        ok = gemv_phase<1>(g, x, a.x, off, it, nst, ring, S, b, nd);
        apply_residual(g, a.x, off, nd, S);
        off = int((off + g.ngroups) % gridDim.x);
        ok = ok && grid_sync(a, gen, S);
      }
    }
    if (!ok) break;
    // ---- HEAD: final rmsnorm -> LM head -> logits, argmax ----
    {
      const PhaseGeo g = geo(a, PH_HEAD, 0);
      for (int k = threadIdx.x; k < a.h; k += kCThreads) xs[k] = ldcg(a.x + k);
      csync();
      norm_in_smem(xs, a.final_norm, a.h, a.eps, S);
      load_seg(x, xs, false, (warp % g.ks) * g.chunks * 256, g.chunks, lane);
      unsigned long long best = 0;
      int nd = 0;
      ok = gemv_phase<3>(g, x, a.logits, off, it, nst, ring, S, best, nd);
      off = int((off + g.ngroups) % gridDim.x);
      best = warp_max_u64(best);
      if (lane == 0) S.best[warp] = best;
      csync();
      if (threadIdx.x == 0) {
        unsigned long long bb = 0;
        for (int w = 0; w < kCWarps; ++w) bb = S.best[w] > bb ? S.best[w] : bb;
        a.am_part[blockIdx.x] = bb;
      }
      ok = ok && grid_sync(a, gen, S);
    }
    if (!ok) break;
    // every CTA reduces the argmax partials: the same token everywhere
    {
      unsigned long long b = 0;
      for (int i = threadIdx.x; i < int(gridDim.x); i += kCThreads) {
        const unsigned long long v = __ldcg(a.am_part + i);
        b = v > b ? v : b;
      }
      b = warp_max_u64(b);
      if (lane == 0) S.best[warp] = b;
      csync();
      unsigned long long bb = 0;
      for (int w = 0; w < kCWarps; ++w) bb = S.best[w] > bb ? S.best[w] : bb;
      const uint32_t next = argmax_key_index(bb);
      csync();
      // end of forward + generate's bookkeeping (finish_step semantics)
      if (!done) pos += 1;
      if (n_gen >= st.gen_cap) {
        done = 1;
      } else {
        if (blockIdx.x == 0 && threadIdx.x == 0) st.gen[n_gen] = next;
        n_gen += 1;
        tok = next;
        for (int e = 0; e < st.n_eos; ++e)
          if (st.eos[e] == next) done = 1;
      }
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        st.pos[0] = pos;
        st.n_gen[0] = n_gen;
        st.token[0] = tok;
        st.done[0] = done;
      }
    }
  }
  // The stream stops here.  When generation ended early (EOS) the producer
  // has issued stages ahead: tell it to stop, then consume (wait for and
  // release) every stage it issued, so no copy is in flight when the CTA
  // exits.  In the normal case it has issued exactly what was consumed.
  if (threadIdx.x == 0) S.abort = 1;
  {
    const unsigned long long t0 = global_ns();
    for (;;) {
      const int pdone = S.prod_done;
      const int issued = S.issued;
      if (it < issued) {
        const int s = it % nst;
        mbar_wait(&S.full[s], (it / nst) & 1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[s]);
        ++it;
      } else if (pdone || global_ns() - t0 > kWaitNs) {
        break;
      }
    }
  }
  (void)G;
}

}  // namespace

namespace {
// K is split over 1, 2, 4 or 8 warps so that a warp's segment is a whole
// number of 256-element chunks, at most 2048 elements.
bool seg_ok(int K) {
  int ks = 1;
  while (K / ks > 2048) ks *= 2;
  return ks <= 8 && K % (ks * 256) == 0;
}
}  // namespace

bool fused_supported(int h, int q_dim, int I, int d, int G) {
  return seg_ok(h) && seg_ok(q_dim) && seg_ok(I) && (d == 64 || d == 128) && G >= 1 && G <= 8 &&
         G * d <= 4 * kCThreads;
}

// Dynamic shared memory: the ring (as many 32 KB stages as fit, <= 6), x
// staging (max(h, q_dim) floats), and the attention tiles or the combine's
// weights (n_q * (nsplit + 1) floats), whichever is larger.
size_t fused_smem(int h, int q_dim, int nq, int d, int G, int nsplit, int* nst_out) {
  const size_t xs = size_t(std::max(h, q_dim)) * 4;
  const size_t att = std::max<size_t>(
      size_t(G) * d + size_t(kTileF) * (d + 4) + size_t(kTileF) * d + size_t(G) * kTileF,
      size_t(nq) * (nsplit + 1)) * 4;
  const size_t budget = 227 * 1024 - sizeof(Shared) - 1024;
  int nst = budget > xs + att ? int((budget - xs - att) / kStage) : 0;
  nst = std::min(nst, kMaxStagesF);
  *nst_out = nst;
  return size_t(nst) * kStage + xs + att;
}

cudaError_t fused_prepare() {
  const int max_smem = 227 * 1024 - int(sizeof(Shared));
  TMG_CUDA_TRY(set_carveout(decode_fused_kernel<64>, max_smem));
  return set_carveout(decode_fused_kernel<128>, max_smem);
}

cudaError_t launch_decode_fused(const FusedArgs& a, int num_sms, cudaStream_t s) {
  int nst = 0;
  const int G = a.nq / a.nkv;
  const size_t smem = fused_smem(a.h, a.nq * a.d, a.nq, a.d, G, a.nsplit, &nst);
  if (nst < 2 || a.xs_floats < std::max(a.h, a.nq * a.d)) return cudaErrorInvalidValue;
  // rows of the residual one CTA updates in the o and down phases must fit
  // the deferred-update arrays
  for (int K : {a.nq * a.d, a.I}) {
    int ks = 1;
    while (K / ks > 2048) ks *= 2;
    const int64_t rpg = kCWarps / ks;
    const int64_t groups = (a.h + rpg - 1) / rpg;
    if ((groups + num_sms - 1) / num_sms * rpg > kMaxDefer) return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.d == 64) return cudaLaunchKernelEx(&cfg, decode_fused_kernel<64>, a, nst);
  if (a.d == 128) return cudaLaunchKernelEx(&cfg, decode_fused_kernel<128>, a, nst);
  return cudaErrorInvalidValue;
}

}  // namespace tmg
