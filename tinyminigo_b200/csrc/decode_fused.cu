// Fused batch-1 decode: n_steps greedy steps of generate's loop
// (src/model.rs:631-656: forward_token, src/model.rs:392-491, then argmax,
// src/tensor.rs:1063-1073) in ONE persistent kernel.
//
// One CTA per SM (cooperative launch), three warpgroups:
//  * a producer warp streams, in consumption order, every weight row this
//    CTA needs for all n_steps tokens -- q/k/v, o, gate/up, down of each
//    layer, then the LM head -- through a ring of 32 KB shared-memory stages
//    with cp.async.bulk (TMA) and mbarriers.  Weights never depend on
//    activations, so the stream runs ahead of the math across phase and
//    token boundaries.  (An optional L2 prefetch of the stages past the
//    ring while the consumers sit in the attention chain exists for
//    measurement; it is off by default.)
//  * eight consumer warps run the phases of each layer:
//      QKV   rmsnorm(x) . Wqkv^T; RoPE on q and k, k/v appended at pos
//      ATTN  split-KV attention per (kv head, split); the owner of a head's
//            first split merges the partials into the attention output
//      O     att . Wo^T              -> x += ...
//      GU    rmsnorm(x) . Wgate^T, Wup^T -> act = silu(g) * u
//      DOWN  act . Wdown^T           -> x += ...
//    then HEAD: rmsnorm(x) . Wlm^T -> logits + per-CTA argmax.
//  * Between phases CTAs exchange activations as tagged {value, tag}
//    words (see ll_store): a reader polls the words it needs until each
//    carries the producing phase's tag, so no grid barrier sits inside a
//    token.  One grid barrier per token (after HEAD) publishes the argmax
//    partials and the cache rows appended during the step; every CTA then
//    reduces the argmax (the same token everywhere), CTA 0 records it, and
//    the next token starts.  Every wait (mbarrier, tag poll, grid barrier)
//    is bounded in time and sets the error word instead of hanging.
// Inside a GEMV phase each warp works alone: it waits for a stage, dots its
// K segment of the stage's rows against the input it holds in registers and
// parks the partial sums in shared memory; one epilogue at the end of the
// phase combines the K segments in warp order and applies the phase's
// output step.
// Row groups of a phase are dealt to CTAs round-robin with a rotating offset
// so every CTA streams the same number of bytes per token within one group.
// QKV groups pair rows j and j + d/2 of one q or k head (RoPE partners), so
// the rotation and the KV append happen in the QKV epilogue.
// All arithmetic is f32 with BF16 weights widened exactly, as in the
// separate kernels.
// Compiled twice: for one GPU (this file) and for a group of GPUs
// (decode_fused_group.cu, TMG_FUSED_GROUP = 1), where the CTAs of every rank
// form one grid for the GEMV phases, exchanged words and KV appends are
// stored into every rank's memory over NVLink, and each rank runs all
// attention items itself.
#include <math.h>

#include "common.cuh"
#include "fused.cuh"

// 0: the single-GPU kernels (and the host side); 1: the same kernels for a
// group of GPUs (decode_fused_group.cu), where exchanged words, KV appends
// and the grid barrier reach every rank.  A compile-time switch, so the
// single-GPU kernels carry none of the group's branches.
#ifndef TMG_FUSED_GROUP
#define TMG_FUSED_GROUP 0
#endif

namespace tmg {

namespace {

constexpr bool kGroup = TMG_FUSED_GROUP != 0;

constexpr int kCWarps = 8;                         // consumer warps
constexpr int kCThreads = kCWarps * kWarp;         // 256
constexpr int kFThreads = kCThreads + 4 * kWarp;   // + the producer's warpgroup
// Registers per thread: the launch gives every thread kLaunchRegs (65536 /
// 384, rounded down to the allocation unit); the producer's warpgroup (one
// working warp, three idle) then gives registers back and the two consumer
// warpgroups take them: 128 * 56 + 256 * 224 = 64512 = 384 * 168.
constexpr int kLaunchRegs = 168;
constexpr int kProducerRegs = 56;
constexpr int kConsumerRegs = 224;
static_assert(4 * kWarp * kProducerRegs + 2 * 4 * kWarp * kConsumerRegs <= kFThreads * kLaunchRegs,
              "register split exceeds the launch's registers");
constexpr int kStage = 32 * 1024;                  // ring stage bytes
constexpr int kMaxStagesF = 6;
constexpr int kTileF = 32;                         // attention positions per tile
constexpr int kMaxRes = 2048;                      // per-warp results of one phase
constexpr int kMaxLocal = kMaxRes / kCWarps;       // LM head groups of one CTA (deferred)
constexpr int kBarWords = 128;                     // words of the barrier block
constexpr int kTraceWords = 12;                    // trace record per CTA and phase

enum Phase : int { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_HEAD = 4 };

__device__ __forceinline__ void csync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// The same at system scope (a word other GPUs write over NVLink).
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// Stage n floats (n % 4 == 0, 16-byte aligned) into shared memory with
// cp.async; the reader waits (cp.async.wait_all, then a CTA barrier).
__device__ __forceinline__ void stage_vec(float* dst, const float* src, int n) {
  for (int i = threadIdx.x * 4; i < n; i += kCThreads * 4) cp_async16(dst + i, src + i);
}

// GEMV inputs live in shared memory in a lane-major layout: within each
// 256-element chunk, the 8 elements lane l multiplies with one 16-byte
// weight load (l*8 .. l*8+7) sit as two float4 at l*4 and 128 + l*4, so a
// warp's two float4 loads per chunk are contiguous (no bank conflicts).
__device__ __forceinline__ int perm_idx(int k) {
  const int e = k & 255;
  return (k - e) + ((e >> 2) & 1) * 128 + (e >> 3) * 4 + (e & 3);
}
// stage_vec into the lane-major layout (n % 8 == 0).
__device__ __forceinline__ void stage_vec_perm(float* dst, const float* src, int n) {
  for (int i = threadIdx.x * 4; i < n; i += kCThreads * 4) cp_async16(dst + perm_idx(i), src + i);
}

// L2 policy for weight rows: once copied to shared memory they are dead.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_ef(void* dst, const void* src, uint32_t bytes,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Bring [src, src + bytes) into L2 (no completion to wait for).
__device__ __forceinline__ void l2_prefetch(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
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

// RoPE of one pair (rotate-half form), without FMA contraction.
__device__ __forceinline__ void rot(float a, float b, float c, float s, float* o0, float* o1) {
  float ac = __fmul_rn(a, c), bs = __fmul_rn(b, s), as = __fmul_rn(a, s), bc = __fmul_rn(b, c);
  *o0 = __fsub_rn(ac, bs);
  *o1 = __fadd_rn(as, bc);
}

// ---------------------------------------------------------------------------
// Phase geometry.  A group is one stage of rpc = 8 / ks rows of K elements
// (at most 32 KB).  Layer phases (QKV, O, GU, DOWN): warp w takes K segment
// w of 8 (K / 8 elements) of every row.  LM head: warp w takes row slot
// w / ks and K segment w % ks.
// ---------------------------------------------------------------------------
struct PhaseGeo {
  const uint16_t* w;
  const uint16_t* w2;      // up rows (GU)
  int N;                   // output rows
  int K;
  int ks;                  // K split over warps (LM head)
  int chunks;              // 256-element chunks per warp segment (LM head)
  int rpc;                 // row slots per group (8 / ks)
  int rpg;                 // output rows per group (GU: rpc / 2 gate + as many up)
  int lrpc, lrpg;          // their log2 (all of rpc, rpg, D are powers of two)
  int ngroups;
  int pair_groups;         // QKV: leading groups holding RoPE partner rows
  int D;                   // head dim
  int lD;
};

__device__ __forceinline__ int ilog2(int p) { return __ffs(p) - 1; }  // p a power of two

__device__ __forceinline__ int ksplit(int K) {
  int ks = 1;
  while (K / ks > 2048) ks *= 2;
  return ks;
}

__device__ __forceinline__ PhaseGeo geo(const FusedArgs& a, const FusedLayer* layers, int ph, int l) {
  PhaseGeo g;
  const FusedLayer& L = layers[l];
  g.w2 = nullptr;
  g.pair_groups = 0;
  g.D = a.d;
  g.lD = ilog2(a.d);
  switch (ph) {
    case PH_QKV: g.w = L.wqkv; g.N = (a.nq + 2 * a.nkv) * a.d; g.K = a.h; break;
    case PH_O: g.w = L.wo; g.N = a.h; g.K = a.nq * a.d; break;
    case PH_GU: g.w = L.wg; g.w2 = L.wu; g.N = a.I; g.K = a.h; break;
    case PH_DOWN: g.w = L.wd; g.N = a.h; g.K = a.I; break;
    default: g.w = a.lm_head; g.N = int(a.V); g.K = a.h; break;
  }
  g.ks = ksplit(g.K);
  g.chunks = g.K / g.ks / 256;
  g.rpc = kCWarps / g.ks;
  g.rpg = ph == PH_GU ? g.rpc / 2 : g.rpc;
  g.lrpc = ilog2(g.rpc);
  g.lrpg = ilog2(g.rpg);
  g.ngroups = (g.N + g.rpg - 1) >> g.lrpg;
  if (ph == PH_QKV) g.pair_groups = ((a.nq + a.nkv) * a.d) >> g.lrpc;
  return g;
}

// Output row held by `slot` of group grp (GU: the gate/up row index).
__device__ __forceinline__ int slot_row(const PhaseGeo& g, int grp, int slot) {
  if (g.pair_groups > 0) {
    if (grp < g.pair_groups) {
      // rpc / 2 rows from each RoPE half of a head; D / rpc groups per head
      const int hp = g.rpc >> 1, half = g.D >> 1;
      const int lgph = g.lD - g.lrpc;  // log2 of groups per head
      const int ra = ((grp >> lgph) << g.lD) + ((grp & ((1 << lgph) - 1)) << (g.lrpc - 1));
      return slot < hp ? ra + slot : ra + half + (slot - hp);
    }
    return (grp << g.lrpc) + slot;  // v rows follow the q and k rows
  }
  return (grp << g.lrpg) + (slot & (g.rpg - 1));
}

// The (at most two) contiguous row ranges a group copies into its stage.
struct Ranges {
  const uint16_t* src[2];
  uint32_t bytes[2];
  uint32_t doff[2];
  int n;
};
__device__ __forceinline__ Ranges group_ranges(const PhaseGeo& g, int grp) {
  Ranges r;
  const uint32_t rowb = uint32_t(g.K) * 2;
  if (g.pair_groups > 0) {
    const int ra = slot_row(g, grp, 0);
    if (grp < g.pair_groups) {
      const int hp = g.rpc / 2;
      r.n = 2;
      r.src[0] = g.w + size_t(ra) * g.K;
      r.src[1] = g.w + size_t(ra + g.D / 2) * g.K;
      r.bytes[0] = r.bytes[1] = uint32_t(hp) * rowb;
      r.doff[0] = 0;
      r.doff[1] = uint32_t(hp) * rowb;
    } else {
      r.n = 1;
      r.src[0] = g.w + size_t(ra) * g.K;
      r.bytes[0] = uint32_t(g.rpc) * rowb;
      r.doff[0] = 0;
    }
    return r;
  }
  const int r0 = grp << g.lrpg;
  const int nr = min(g.rpg, g.N - r0);
  r.n = g.w2 ? 2 : 1;
  r.src[0] = g.w + size_t(r0) * g.K;
  r.bytes[0] = uint32_t(nr) * rowb;
  r.doff[0] = 0;
  if (g.w2) {
    r.src[1] = g.w2 + size_t(r0) * g.K;
    r.bytes[1] = r.bytes[0];
    r.doff[1] = uint32_t(g.rpg) * rowb;
  }
  return r;
}

// First group of CTA gid of a grid of gn CTAs (all ranks') in a phase whose
// groups start at rotation `off` (0 <= off < gn).
__device__ __forceinline__ int first_group(int off, int gid, int gn) {
  const int d = gid - off;
  return d < 0 ? d + gn : d;
}

// Upper bound on the kernel's static shared memory, checked at prepare time.
constexpr size_t kStaticReserve = 12 * 1024;

struct Shared {
  uint64_t full[kMaxStagesF];
  uint64_t empty[kMaxStagesF];
  float res[kMaxRes];  // per-warp sums of this phase: [local group][warp]
  float ssq[kCWarps];
  unsigned long long best[kCWarps];
  float m_s[8], l_s[8], alpha_s[8];
  int fail[2];  // a poll gave up (indexed by the parity of the poll count)
  unsigned long long poll_ns;  // limit of one tag poll
  int gid, gn;                 // this CTA in the grid of all ranks, and its size
  int world;                   // GPUs of that grid (1: this one alone)
  unsigned long long* ll_base;    // this rank's exchange words ...
  unsigned long long* ll_peer[kMaxGroupRanks];    // ... and every rank's (by rank)
  int gen_ok;
  volatile int abort;      // stop issuing / waiting (error or early end)
  volatile int issued;     // producer: stages issued so far
  volatile int prod_done;  // producer: no more stages will be issued
  volatile int streaming;  // consumers: inside a GEMV's stage loop
  volatile int in_attn;    // consumers: in an attention phase
};

// This CTA's index in the grid of all ranks, and that grid's size: the
// special registers on one GPU, the values the kernel computed at entry in a
// group (kept in shared memory).
__device__ __forceinline__ int cta_gid(const Shared& S) {
  return kGroup ? S.gid : int(blockIdx.x);
}
__device__ __forceinline__ int cta_gn(const Shared& S) {
  return kGroup ? S.gn : int(gridDim.x);
}

// ---------------------------------------------------------------------------
// Grid barrier among the consumer warps of all CTAs: one monotonic arrival
// counter (zeroed before the launch); the k-th barrier waits until it reaches
// k times the CTAs of the grid (of all ranks: on several GPUs every CTA adds
// to every rank's counter and waits on its own).  Every wait is bounded in time; a CTA that has aborted does
// not arrive and raises bar[2], which releases the others.
// ---------------------------------------------------------------------------
__device__ bool grid_sync(const FusedArgs& a, unsigned int& target, Shared& S,
                          unsigned long long* tr) {
  csync();
  if (threadIdx.x == 0) {
    if (tr) tr[0] = global_ns();
    int ok = S.abort ? 0 : 1;
    target += cta_gn(S);
    constexpr bool sys = kGroup;
    if (ok) {
      if (sys) {
        // every rank's counter: this CTA's writes of the step (KV appends,
        // argmax partial) are released to all GPUs first
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < a.world; ++r)
          asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(a.bar_peer[r]) : "memory");
      } else {
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
      }
      const unsigned long long t0 = global_ns();
      unsigned int spins = 0;
      while (int((sys ? ld_acquire_sys(a.bar) : ld_acquire(a.bar)) - target) < 0) {
        if ((++spins & 255) == 0) {
          if ((sys ? ld_acquire_sys(a.bar + 2) : ld_acquire(a.bar + 2)) != 0 ||
              global_ns() - t0 > S.poll_ns) {
            ok = 0;
            break;
          }
        }
      }
    }
    if (!ok) {
      if (sys)
        for (int r = 0; r < a.world; ++r) atomicExch_system(a.bar_peer[r] + 2, 1u);
      else
        atomicExch(a.bar + 2, 1u);
      if (a.err) atomicExch(a.err, 2);
    }
    if (tr) tr[1] = global_ns();
    S.gen_ok = ok;
  }
  csync();
  return S.gen_ok != 0;
}

// ---------------------------------------------------------------------------
// Producer: the weight stream of all steps, in consumption order.
// ---------------------------------------------------------------------------
struct Cursor {
  const FusedLayer* layers;  // the per-layer table in shared memory
  int step, l, ph, off;
  int grp;
  int gid, gn;  // this CTA in the grid of all ranks
  PhaseGeo g;
  bool valid;
};

__device__ __forceinline__ void cur_settle(const FusedArgs& a, Cursor& c) {
  while (c.valid && c.grp >= c.g.ngroups) {
    c.off = (c.off + c.g.ngroups) % c.gn;
    if (c.ph == PH_HEAD) {
      if (++c.step >= a.n_steps) {
        c.valid = false;
        break;
      }
      c.l = 0;
      c.ph = PH_QKV;
    } else if (c.ph == PH_DOWN) {
      ++c.l;
      c.ph = c.l == a.L ? PH_HEAD : PH_QKV;
    } else {
      ++c.ph;
    }
    c.g = geo(a, c.layers, c.ph, c.l < a.L ? c.l : 0);
    c.grp = first_group(c.off, c.gid, c.gn);
  }
}
__device__ __forceinline__ void cur_begin(const FusedArgs& a, const FusedLayer* layers,
                                          const Shared& S, Cursor& c) {
  c.layers = layers;
  c.gid = cta_gid(S);
  c.gn = cta_gn(S);
  c.step = 0;
  c.l = 0;
  c.ph = PH_QKV;
  c.off = 0;
  c.g = geo(a, c.layers, PH_QKV, 0);
  c.grp = first_group(0, c.gid, c.gn);
  c.valid = a.n_steps > 0;
  cur_settle(a, c);
}
__device__ __forceinline__ void cur_next(const FusedArgs& a, Cursor& c) {
  c.grp += c.gn;
  cur_settle(a, c);
}

__device__ void producer(const FusedArgs& a, const FusedLayer* layers, Shared& S, uint8_t* ring,
                         int nst) {
  const uint64_t pol = evict_first_policy();
  const int nph = a.L * 5 + 1;
  Cursor ic, pc;
  cur_begin(a, layers, S, ic);
  // pc: the first stage past the ring (stage it + nst), the next one the
  // stall-time L2 prefetch may bring in; pf counts the stages it passed
  pc = ic;
  int it = 0, pf = 0;
  for (int k = 0; k < nst && pc.valid; ++k, ++pf) cur_next(a, pc);
  long long pf_next = 0;  // clock of the next prefetch allowed (pacing)
  unsigned long long* tr_cur = nullptr;  // diagnostics of the phase being issued
  unsigned long long t_last = 0, c_wait = 0, c_issue = 0;
  while (ic.valid) {
    const int s = it % nst;
    const uint32_t par = (it / nst) & 1;
    if (S.abort) return;
    const long long c0 = clock64();
    // While the slot is busy and the consumers are in the attention chain
    // (ATTN entry to O's input; most CTAs only wait there), the weight
    // stream would stall: bring the stages after the ring into L2 instead,
    // at most pf_ahead past it, one every pf_pace cycles.
    bool got = mbar_try(&S.empty[s], par ^ 1);
    if (!got && a.pf_ahead > 0) {
      // poll the slot, prefetching while the condition holds (bounded in
      // time like mbar_wait)
      const unsigned long long tw0 = global_ns();
      for (unsigned int i = 1; !got; ++i) {
        if ((a.pf_mode == 1 || S.in_attn != 0) && pc.valid && pf < it + nst + a.pf_ahead) {
          const long long now = clock64();
          if (now >= pf_next) {
            const Ranges r = group_ranges(pc.g, pc.grp);
            l2_prefetch(r.src[0], r.bytes[0]);
            if (r.n > 1) l2_prefetch(r.src[1], r.bytes[1]);
            cur_next(a, pc);
            ++pf;
            pf_next = now + a.pf_pace;
          }
        }
        got = mbar_try(&S.empty[s], par ^ 1);
        if (!got && (i & 255) == 0 && (S.abort || global_ns() - tw0 > kWaitNs)) break;
      }
    }
    if (!got && S.abort) return;
    if (!got && !mbar_wait(&S.empty[s], par ^ 1)) {
      S.abort = 1;
      if (a.err) atomicExch(a.err, 2);
      return;
    }
    const long long c1 = clock64();
    const Ranges r = group_ranges(ic.g, ic.grp);
    mbar_expect_tx(&S.full[s], r.bytes[0] + (r.n > 1 ? r.bytes[1] : 0u));
    uint8_t* dst = ring + size_t(s) * kStage;
    bulk_g2s_ef(dst + r.doff[0], r.src[0], r.bytes[0], &S.full[s], pol);
    if (r.n > 1) bulk_g2s_ef(dst + r.doff[1], r.src[1], r.bytes[1], &S.full[s], pol);
    S.issued = it + 1;
    if (a.trace && ic.step == 0) {
      const int p = ic.l == a.L ? a.L * 5 : ic.l * 5 + (ic.ph == PH_QKV ? 0 : ic.ph + 1);
      unsigned long long* tr = a.trace + (size_t(blockIdx.x) * nph + p) * kTraceWords;
      if (tr != tr_cur) {
        if (tr_cur) {
          tr_cur[3] = t_last;
          tr_cur[10] = c_wait;
          tr_cur[11] = c_issue;
        }
        tr_cur = tr;
        tr[2] = global_ns();
        c_wait = c_issue = 0;
      }
      t_last = global_ns();
      c_wait += c1 - c0;
      c_issue += clock64() - c1;
    }
    cur_next(a, ic);
    ++it;
    if (pf < it + nst) {  // the ring moved past pc
      if (pc.valid) cur_next(a, pc);
      ++pf;
    }
  }
  if (tr_cur) {
    tr_cur[3] = t_last;
    tr_cur[10] = c_wait;
    tr_cur[11] = c_issue;
  }
}

// ---------------------------------------------------------------------------
// Flag-in-data exchange between CTAs.  Every activation that crosses CTAs
// inside a step (x after O and after DOWN, the rotated q/k/v of the
// position, the attention partials and output, act) travels as 8-byte
// words {value, tag} written with one relaxed 64-bit store; a reader polls
// the words it needs until each carries the tag of the phase that writes
// it.  A 64-bit access is single-copy atomic, so a matching tag comes with
// its value, and neither a fence nor a barrier sits between producer and
// consumer.  Tags number the phases of a launch from 1 (the host zeroes the
// buffers before each launch).  A buffer is written again only after a
// chain of phases that needs every CTA to have finished reading it (every
// CTA owns groups in every GEMV phase), so a reader never misses its tag.
// On several GPUs the writer stores each word into every rank's copy (peer
// stores over NVLink, system scope) and readers poll their own copy, except
// for the attention: every rank runs all attention items of a layer itself
// (it holds all of q/k/v and the whole cache), so the partials and the
// attention output stay in its own memory and two of a layer's hops never
// cross GPUs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_tag(unsigned long long* p, unsigned long long w, bool sys) {
  if (sys) asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
  else asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long tag_word(float v, uint32_t tag) {
  return (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
}
// (v, tag) at word p of this rank's exchange block, and of every rank's.
__device__ __forceinline__ void ll_store(const Shared& S, unsigned long long* p, float v,
                                         uint32_t tag) {
  const unsigned long long w = tag_word(v, tag);
  if (!kGroup) {
    st_tag(p, w, false);
    return;
  }
  const size_t o = size_t(p - S.ll_base);
  for (int r = 0; r < S.world; ++r) st_tag(S.ll_peer[r] + o, w, true);
}
__device__ __forceinline__ void ll_store_rep(const Shared& S, unsigned long long* base, int n,
                                             int rep, int r, float v, uint32_t tag) {
  for (int c = 0; c < rep; ++c) ll_store(S, base + size_t(c) * n + r, v, tag);
}
// This rank's copy only: the attention partials and outputs (in a group
// every rank runs all attention items itself, so they never cross GPUs).
__device__ __forceinline__ void ll_store_local(unsigned long long* p, float v, uint32_t tag) {
  st_tag(p, tag_word(v, tag), false);
}
__device__ __forceinline__ void ll_store_rep_local(unsigned long long* base, int n, int rep, int r,
                                                   float v, uint32_t tag) {
  for (int c = 0; c < rep; ++c) ll_store_local(base + size_t(c) * n + r, v, tag);
}
__device__ __forceinline__ ulonglong2 ll_load2(const unsigned long long* p, bool sys) {
  ulonglong2 r;
  if (sys)
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];"
                 : "=l"(r.x), "=l"(r.y)
                 : "l"(p)
                 : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];"
                 : "=l"(r.x), "=l"(r.y)
                 : "l"(p)
                 : "memory");
  return r;
}
__device__ __forceinline__ unsigned int ld_abort(const unsigned int* p, bool sys) {
  return sys ? ld_acquire_sys(p) : ld_acquire(p);
}

// The copy of a replicated exchange vector (n words per copy) this CTA reads.
__device__ __forceinline__ const unsigned long long* ll_mine(const unsigned long long* base, int n,
                                                             int rep) {
  return base + size_t(blockIdx.x % unsigned(rep)) * n;
}

constexpr int kGatherPairs = 16;                            // word pairs per thread
constexpr unsigned kBackoffNs = 0;                          // pause between polls
constexpr int kMaxGather = kGatherPairs * 2 * kCThreads;   // 8192 words

// All consumer threads: wait until src[0..n) (n even, <= kMaxGather) carry
// `tag`, then copy the values to dst in shared memory (in the lane-major
// layout when asked; n % 8 == 0 then).  With wx (an rmsnorm input; wx holds
// the norm weights in dst's layout, staged and waited for), also
// wx <- wx * x in place and each warp's share of sum(x^2) into S.ssq.  Returns false, in
// every thread alike, when a wait gave up or the kernel is aborting; `gc`
// counts the polls (the failure flag alternates slots so that a slow reader
// of one poll never sees the next poll's flag).
__device__ __noinline__ bool ll_gather(float* dst, const unsigned long long* src, int n, uint32_t tag,
                          const unsigned int* abort_word, Shared& S, uint32_t& gc,
                          bool lane_major = false, float* wx = nullptr) {
  const unsigned long long t0 = global_ns();
  unsigned int spins = 0;
  bool ok = true;
  float ss = 0.f;
  constexpr bool sys = kGroup;
  ulonglong2 v[kGatherPairs];
  uint32_t need = 0;  // bit k: pair k still to come
#pragma unroll
  for (int k = 0; k < kGatherPairs; ++k) {
    const int i = (threadIdx.x + k * kCThreads) * 2;
    if (i < n) {
      v[k] = ll_load2(src + i, sys);
      need |= 1u << k;
    }
  }
  for (;;) {
#pragma unroll
    for (int k = 0; k < kGatherPairs; ++k) {
      if ((need >> k) & 1u) {
        if (uint32_t(v[k].x >> 32) == tag && uint32_t(v[k].y >> 32) == tag) {
          const int i = (threadIdx.x + k * kCThreads) * 2;
          const int j = lane_major ? perm_idx(i) : i;
          const float2 val =
              make_float2(__uint_as_float(uint32_t(v[k].x)), __uint_as_float(uint32_t(v[k].y)));
          *reinterpret_cast<float2*>(dst + j) = val;
          if (wx) {  // rmsnorm input: weights * x in place, and sum(x^2)
            float2 w = *reinterpret_cast<const float2*>(wx + j);
            w.x *= val.x;
            w.y *= val.y;
            *reinterpret_cast<float2*>(wx + j) = w;
            ss = fmaf(val.x, val.x, ss);
            ss = fmaf(val.y, val.y, ss);
          }
          need &= ~(1u << k);
        }
      }
    }
    if (!need) break;
    if ((++spins & 15) == 0 && (ld_abort(abort_word, sys) != 0 || global_ns() - t0 > S.poll_ns)) {
      ok = false;
      break;
    }
    if (kBackoffNs) __nanosleep(kBackoffNs);
#pragma unroll
    for (int k = 0; k < kGatherPairs; ++k)
      if ((need >> k) & 1u) v[k] = ll_load2(src + (threadIdx.x + k * kCThreads) * 2, sys);
  }
  if (wx) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) S.ssq[threadIdx.x >> 5] = ss;
  }
  const int slot = gc & 1;
  ++gc;
  if (!ok || (threadIdx.x == 0 && S.abort)) S.fail[slot] = 1;
  csync();
  return S.fail[slot] == 0;
}

// Up to three short ranges (each at most 2 kCThreads words, even) gathered
// in one poll, as ll_gather.
struct LLRange {
  float* dst;
  const unsigned long long* src;
  int n;
};
__device__ __forceinline__ bool ll_gather3(const LLRange* r, int nr, uint32_t tag,
                                        const unsigned int* abort_word, Shared& S, uint32_t& gc) {
  ulonglong2 v[3];
  uint32_t need = 0;
  constexpr bool sys = kGroup;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    if (k < nr && threadIdx.x * 2 < r[k].n) {
      v[k] = ll_load2(r[k].src + threadIdx.x * 2, sys);
      need |= 1u << k;
    }
  }
  const unsigned long long t0 = global_ns();
  unsigned int spins = 0;
  bool ok = true;
  for (;;) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      if (((need >> k) & 1u) && uint32_t(v[k].x >> 32) == tag && uint32_t(v[k].y >> 32) == tag) {
        r[k].dst[threadIdx.x * 2] = __uint_as_float(uint32_t(v[k].x));
        r[k].dst[threadIdx.x * 2 + 1] = __uint_as_float(uint32_t(v[k].y));
        need &= ~(1u << k);
      }
    }
    if (!need) break;
    if ((++spins & 15) == 0 && (ld_abort(abort_word, sys) != 0 || global_ns() - t0 > S.poll_ns)) {
      ok = false;
      break;
    }
    if (kBackoffNs) __nanosleep(kBackoffNs);
#pragma unroll
    for (int k = 0; k < 3; ++k)
      if ((need >> k) & 1u) v[k] = ll_load2(r[k].src + threadIdx.x * 2, sys);
  }
  const int slot = gc & 1;
  ++gc;
  if (!ok || (threadIdx.x == 0 && S.abort)) S.fail[slot] = 1;
  csync();
  return S.fail[slot] == 0;
}

// Give up: raise the kernel-wide abort word and the error word.
__device__ __forceinline__ void raise_abort(const FusedArgs& a) {
  if (threadIdx.x == 0) {
    if (kGroup)
      for (int r = 0; r < a.world; ++r) atomicExch_system(a.bar_peer[r] + 2, 1u);
    else
      atomicExch(a.bar + 2, 1u);
    if (a.err) atomicExch(a.err, 2);
  }
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
struct XSeg {
  float4 a[8], b[8];
};

// This warp's K segment of the phase input from shared memory (lane-major
// layout, see perm_idx).
__device__ __forceinline__ void load_seg_smem(XSeg& x, const float* src, int kbase, int chunks,
                                              int lane) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < chunks) {
      const float* p = src + kbase + c * 256 + lane * 4;  // lane-major layout
      x.a[c] = *reinterpret_cast<const float4*>(p);
      x.b[c] = *reinterpret_cast<const float4*>(p + 128);
    }
  }
}

// rmsnorm of the n-vector whose K segments the warps hold (warps slot*ks ..
// slot*ks + ks - 1 cover all of it): x <- (x * inv) * w, rms_norm_into's
// order, w staged in shared memory.  With ks > 1 the segment sums meet in
// shared memory.
__device__ __forceinline__ void norm_seg(XSeg& x, const float* w, int kbase, int chunks, int ks,
                                         int n, float eps, Shared& S) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < chunks) {
      s0 = fmaf(x.a[c].x, x.a[c].x, s0);
      s1 = fmaf(x.a[c].y, x.a[c].y, s1);
      s0 = fmaf(x.a[c].z, x.a[c].z, s0);
      s1 = fmaf(x.a[c].w, x.a[c].w, s1);
      s0 = fmaf(x.b[c].x, x.b[c].x, s0);
      s1 = fmaf(x.b[c].y, x.b[c].y, s1);
      s0 = fmaf(x.b[c].z, x.b[c].z, s0);
      s1 = fmaf(x.b[c].w, x.b[c].w, s1);
    }
  }
  float tot = warp_sum(s0 + s1);
  if (ks > 1) {
    if (lane == 0) S.ssq[warp] = tot;
    csync();
    tot = 0.f;
    for (int j = 0; j < ks; ++j) tot += S.ssq[(warp / ks) * ks + j];
  }
  const float inv = 1.0f / sqrtf(tot / float(n) + eps);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c < chunks) {
      const float* p = w + kbase + c * 256 + lane * 4;  // lane-major, as x
      const float4 wa = *reinterpret_cast<const float4*>(p);
      const float4 wb = *reinterpret_cast<const float4*>(p + 128);
      x.a[c] = make_float4((x.a[c].x * inv) * wa.x, (x.a[c].y * inv) * wa.y,
                           (x.a[c].z * inv) * wa.z, (x.a[c].w * inv) * wa.w);
      x.b[c] = make_float4((x.b[c].x * inv) * wb.x, (x.b[c].y * inv) * wb.y,
                           (x.b[c].z * inv) * wb.z, (x.b[c].w * inv) * wb.w);
    }
  }
}

// 1/rms(x) from the warps' shares in S.ssq (after a CTA barrier).
__device__ __forceinline__ float rms_scale(const Shared& S, int n, float eps) {
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kCWarps; ++w) tot += S.ssq[w];
  return 1.0f / sqrtf(tot / float(n) + eps);
}

// Position in the stage ring: stage count, slot, phase parity.
struct RingPos {
  int it, s;
  uint32_t par;
  __device__ __forceinline__ void next(int nst) {
    ++it;
    if (++s == nst) {
      s = 0;
      par ^= 1u;
    }
  }
};

// One GEMV phase over this CTA's groups: the warp's K segment of the input
// from shared memory (src), rmsnorm'd with nw when given; then each warp
// dots its slot/segment of every stage.  imm (LM
// head with ks == 1): logits and the argmax candidate directly; otherwise
// the sums go to S.res for the phase's epilogue.  Returns the number of
// local groups; tw (diagnostics) receives the first stage's arrival time.
__device__ __forceinline__ int gemv_block(int ngroups, int K, int ks, int rpg, int N,
                                       int chunks, const float* src, const float* nw,
                                       float eps, int n_norm, int off,
                                       RingPos& rp_io, int nst, const uint8_t* ring, Shared& S,
                                       bool imm, float* logits, unsigned long long& best_io,
                                       unsigned long long* tw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp / ks;
  const int kbase = (warp % ks) * chunks * 256;
  const long long c0 = tw ? clock64() : 0;
  XSeg x;
  load_seg_smem(x, src, kbase, chunks, lane);
  const long long c1 = tw ? clock64() : 0;
  if (nw) norm_seg(x, nw, kbase, chunks, ks, n_norm, eps, S);
  const long long c2 = tw ? clock64() : 0;
  if (tw && threadIdx.x == 0) {
    tw[8] = c1 - c0;
    tw[9] = c2 - c1;
  }
  RingPos rp = rp_io;
  unsigned long long best = best_io;
  if (threadIdx.x == 0) S.streaming = 1;
  // this lane's first weight element in stage 0
  const uint16_t* wbase =
      reinterpret_cast<const uint16_t*>(ring + size_t(slot) * K * 2) + kbase + lane * 8;
  int kl = 0;
  for (int grp = first_group(off, cta_gid(S), cta_gn(S)); grp < ngroups;
       grp += cta_gn(S), rp.next(nst), ++kl) {
    const int s = rp.s;
    float acc = 0.f;
    const bool ok = !S.abort && mbar_wait(&S.full[s], rp.par);
    if (tw && kl == 0 && threadIdx.x == 0) {
      tw[6] = global_ns();
      tw[4] = clock64() - c2;
    }
    if (ok) {
      const uint16_t* wr = wbase + s * (kStage / 2);
      float sacc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c < chunks) fma8(x.a[c], x.b[c], *reinterpret_cast<const uint4*>(wr + c * 256), sacc);
      acc = sum8(sacc);
    } else if (lane == 0) {
      S.abort = 1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    acc = warp_sum(acc);
    if (lane == 0) {
      if (imm) {
        const int r = grp * rpg + slot;
        if (r < N) {
          logits[r] = acc;
          const unsigned long long kk = argmax_key(acc, uint32_t(r));
          best = kk > best ? kk : best;
        }
      } else if (kl < kMaxLocal) {
        S.res[kl * kCWarps + warp] = acc;
      }
    }
  }
  if (threadIdx.x == 0) S.streaming = 0;
  rp_io = rp;
  best_io = best;
  return kl;
}

// Sum of slot `slot` of local group kl over its K segments, in order.
__device__ __forceinline__ float res_val(const Shared& S, int kl, int slot, int ks) {
  float v = S.res[kl * kCWarps + slot * ks];
  for (int j = 1; j < ks; ++j) v += S.res[kl * kCWarps + slot * ks + j];
  return v;
}

// Layer phases: row `slot` of local group kl, the sum of the 8 warps' K
// segments in warp order.
__device__ __forceinline__ float res_k(const Shared& S, int kl, int slot, int rpc) {
  const float* r = S.res + (kl * rpc + slot) * kCWarps;
  return ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
}

// One layer-phase GEMV over this CTA's groups (R = rpc rows per stage):
// warp w holds x[w*K/8, (w+1)*K/8) (chunks 256-element chunks, lane-major
// in shared memory) and dots it with that segment of all R rows of every
// stage; a transposed butterfly (R values per lane -> one row per lane
// group) reduces over the lanes, and each warp's R partial sums go to
// S.res[(kl * R + row) * 8 + warp] for the epilogue.  Returns the number
// of local groups.
template <int R>
__device__ __forceinline__ int gemv_kseg(int ngroups, int K, int chunks, const float* src,
                                         int off, RingPos& rp_io, int nst, const uint8_t* ring,
                                         Shared& S, unsigned long long* tw) {
  constexpr int M = R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0;  // log2 R
  constexpr int NC = 8 / R;                                      // most chunks a warp holds
  constexpr int NA = 8 / R;                                      // accumulators per row
  // one or two rows per stage (segments of 4 to 8 chunks): x is read from
  // shared memory with each stage instead of held in registers
  constexpr bool XS = R <= 2;
  static_assert(R == 8 || R == 4 || R == 2 || R == 1, "rows per stage");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kbase = warp * chunks * 256;
  const long long c0 = tw ? clock64() : 0;
  float4 xa[XS ? 1 : NC], xb[XS ? 1 : NC];
#pragma unroll
  for (int c = 0; c < (XS ? 0 : NC); ++c) {
    if (c < chunks) {
      const float* p = src + kbase + c * 256 + lane * 4;  // lane-major layout
      xa[c] = *reinterpret_cast<const float4*>(p);
      xb[c] = *reinterpret_cast<const float4*>(p + 128);
    }
  }
  if (tw && threadIdx.x == 0) tw[8] = clock64() - c0;
  const long long c2 = tw ? clock64() : 0;
  if (threadIdx.x == 0) S.streaming = 1;
  RingPos rp = rp_io;
  const uint16_t* wbase = reinterpret_cast<const uint16_t*>(ring) + kbase + lane * 8;
  const int myrow = M > 0 ? (lane >> (5 - M)) & (R - 1) : 0;
  const bool writer = (lane & ((32 >> M) - 1)) == 0;
  int kl = 0;
  for (int grp = first_group(off, cta_gid(S), cta_gn(S)); grp < ngroups;
       grp += cta_gn(S), rp.next(nst), ++kl) {
    const int s = rp.s;
    float acc[R][NA];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int i = 0; i < NA; ++i) acc[r][i] = 0.f;
    const bool ok = !S.abort && mbar_wait(&S.full[s], rp.par);
    if (tw && kl == 0 && threadIdx.x == 0) {
      tw[6] = global_ns();
      tw[4] = clock64() - c2;
    }
    if (ok) {
      const uint16_t* wr = wbase + s * (kStage / 2);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (c < chunks) {
          const float* xp = src + kbase + c * 256 + lane * 4;
          const float4 ua = XS ? *reinterpret_cast<const float4*>(xp) : xa[XS ? 0 : c];
          const float4 ub = XS ? *reinterpret_cast<const float4*>(xp + 128) : xb[XS ? 0 : c];
          const float xv[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint4 w = *reinterpret_cast<const uint4*>(wr + size_t(r) * K + c * 256);
            const float wv[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                                 bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r][e % NA] = fmaf(xv[e], wv[e], acc[r][e % NA]);
          }
        }
      }
    } else if (lane == 0) {
      S.abort = 1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
    float v[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float t = acc[r][0];
#pragma unroll
      for (int i = 1; i < NA; ++i) t += acc[r][i];
      v[r] = t;
    }
    // halve the rows held per lane M times (lane bit 16, 8, 4 picks the
    // upper half), then sum over the lanes that share a row
#pragma unroll
    for (int st = 0; st < M; ++st) {
      const int h = R >> (st + 1), bit = 16 >> st;
      const bool up = (lane & bit) != 0;
#pragma unroll
      for (int i = 0; i < h; ++i) {
        const float send = up ? v[i] : v[i + h];
        const float keep = up ? v[i + h] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
      }
    }
#pragma unroll
    for (int bit = 16 >> M; bit >= 1; bit >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], bit);
    if (writer && (kl + 1) * R * kCWarps <= kMaxRes) S.res[(kl * R + myrow) * kCWarps + warp] = v[0];
  }
  if (threadIdx.x == 0) S.streaming = 0;
  rp_io = rp;
  return kl;
}

// QKV epilogue: the rmsnorm factor (scale), then RoPE on the q/k partner
// rows at position pos (rope_s: the cos then sin row of pos).  q, k and v of the position go out as tagged
// words; k and v are also appended to the cache at pos (when there is room),
// where later steps read them.
// On several GPUs the appends go to every rank's cache (plain stores; the
// step's grid barrier releases them before any rank reads those rows).
__device__ __forceinline__ void kv_put(const FusedArgs& a, const FusedLayer& L, int l, int which,
                                       size_t idx, float v) {
  if (!kGroup) {
    (which ? L.vc : L.kc)[idx] = v;
    return;
  }
  for (int r = 0; r < a.world; ++r) a.kv_peer[(size_t(r) * a.L + l) * 2 + which][idx] = v;
}

__device__ __forceinline__ void epi_qkv(const FusedArgs& a, const FusedLayer& L, int l,
                                        const PhaseGeo& g, int off, int nloc, int pos, bool append,
                                        const float* rope_s, float scale, uint32_t tag, Shared& S) {
  const int D = g.D, half = D / 2, hp = g.rpc / 2, kvd = a.nkv * D;
  const int f = first_group(off, cta_gid(S), cta_gn(S));
  const int vbase = (a.nq + a.nkv) * D;
  for (int i = threadIdx.x; i < (nloc << g.lrpc); i += kCThreads) {
    const int kl = i >> g.lrpc, slot = i & (g.rpc - 1);
    const int grp = f + kl * cta_gn(S);
    if (grp < g.pair_groups) {
      if (slot >= hp) continue;  // done with its partner
      const int ra = slot_row(g, grp, slot);
      const int head = ra >> g.lD;
      const int j = ra & (D - 1);
      float o0, o1;
      rot(res_k(S, kl, slot, g.rpc) * scale, res_k(S, kl, slot + hp, g.rpc) * scale, rope_s[j],
          rope_s[half + j], &o0, &o1);
      ll_store(S, a.qkv_ll + ra, o0, tag);
      ll_store(S, a.qkv_ll + ra + half, o1, tag);
      if (head >= a.nq && append) {
        const size_t kb = size_t(pos) * kvd + (head - a.nq) * D;
        kv_put(a, L, l, 0, kb + j, o0);
        kv_put(a, L, l, 0, kb + j + half, o1);
      }
    } else {
      const int r = slot_row(g, grp, slot);
      const float v = res_k(S, kl, slot, g.rpc) * scale;
      ll_store(S, a.qkv_ll + r, v, tag);
      if (append) kv_put(a, L, l, 1, size_t(pos) * kvd + (r - vbase), v);
    }
  }
}

// O / DOWN epilogue: x[r] = x_s[r] + y[r] out as tagged words (x_s: x as
// this CTA last gathered it, lane-major).
__device__ __forceinline__ void epi_residual(unsigned long long* x_ll, int rep, const float* x_s,
                                             const PhaseGeo& g, int off, int nloc, uint32_t tag,
                                             const Shared& S) {
  const int f = first_group(off, cta_gid(S), cta_gn(S));
  for (int i = threadIdx.x; i < (nloc << g.lrpc); i += kCThreads) {
    const int kl = i >> g.lrpc, slot = i & (g.rpc - 1);
    const int r = ((f + kl * cta_gn(S)) << g.lrpg) + slot;
    if (r < g.N)
      ll_store_rep(S, x_ll, g.N, rep, r, x_s[perm_idx(r)] + res_k(S, kl, slot, g.rpc), tag);
  }
}

// GU epilogue: the rmsnorm factor (scale), then act = silu(gate) * up, out
// as tagged words.
__device__ __forceinline__ void epi_swiglu(unsigned long long* act_ll, int rep, const PhaseGeo& g,
                                           int off, int nloc, float scale, uint32_t tag,
                                           const Shared& S) {
  const int f = first_group(off, cta_gid(S), cta_gn(S));
  for (int i = threadIdx.x; i < (nloc << g.lrpg); i += kCThreads) {
    const int kl = i >> g.lrpg, q = i & (g.rpg - 1);
    const int r = ((f + kl * cta_gn(S)) << g.lrpg) + q;
    if (r < g.N) {
      const float gv = res_k(S, kl, q, g.rpc) * scale, uv = res_k(S, kl, q + g.rpg, g.rpc) * scale;
      ll_store_rep(S, act_ll, g.N, rep, r, gv / (1.0f + expf(-gv)) * uv, tag);
    }
  }
}

// LM head epilogue (ks > 1): logits and this thread's argmax candidate.
__device__ __forceinline__ void epi_head(float* logits, const PhaseGeo& g, int off, int nloc,
                                         const Shared& S, unsigned long long& best) {
  const int f = first_group(off, cta_gid(S), cta_gn(S));
  for (int i = threadIdx.x; i < (nloc << g.lrpc); i += kCThreads) {
    const int kl = i >> g.lrpc, slot = i & (g.rpc - 1);
    const int r = ((f + kl * cta_gn(S)) << g.lrpg) + slot;
    if (r < g.N) {
      const float v = res_val(S, kl, slot, g.ks);
      logits[r] = v;
      const unsigned long long kk = argmax_key(v, uint32_t(r));
      best = kk > best ? kk : best;
    }
  }
}

// What the attention items of one layer read and write.
struct AttnArgs {
  const unsigned long long* qkv_ll;  // q | k | v of the position, tagged
  const float* kc;                   // cache rows < pos
  const float* vc;
  unsigned long long* part_ll;       // [n_kv, nsplit, G, D + 2] tagged partials
  unsigned long long* att_ll;        // [n_q * D] tagged output
  const unsigned int* abort_word;
  int nq, nkv, nsplit;
  int rep;                           // copies of att_ll
  float scale;
};

// Attention of one (kv head, split) item over positions [split*chunk,
// min(n_ctx, (split+1)*chunk)) with online softmax.  q and, when the
// position is in range, its k and v come as tagged words from the QKV
// epilogues; earlier positions from the cache.  A single split writes the
// output; otherwise the partial (m, l, o) goes out for the merge.
// Start loading the cached K/V rows of the first tile of attention item
// (kvh, split) into its tile buffers in sm (the layout attn_item uses).  The
// rows below the decoded position do not depend on this step, so a CTA
// issues this as soon as the region is free (in its QKV phase) and the load
// overlaps the QKV GEMV instead of sitting in the attention chain.  The
// copies complete at attn_item's cp.async wait.
template <int D>
__device__ __forceinline__ void attn_prefetch(const float* kc, const float* vc, int nkv, int G,
                                              int kvh, int split, int chunk, int n_ctx,
                                              int cache_end, float* sm) {
  float* ks_ = sm + G * D;
  float* vs = ks_ + kTileF * (D + 4);
  const int kvd = nkv * D;
  const int c0 = split * chunk, c1 = min(n_ctx, c0 + chunk);
  const int nt = min(kTileF, c1 - c0);
  const int nc = max(0, min(nt, cache_end - c0));
  for (int i = threadIdx.x; i < nc * (D / 4); i += kCThreads) {
    const int t = i / (D / 4), j4 = i % (D / 4);
    cp_async16(ks_ + t * (D + 4) + j4 * 4, kc + size_t(c0 + t) * kvd + kvh * D + j4 * 4);
    cp_async16(vs + t * D + j4 * 4, vc + size_t(c0 + t) * kvd + kvh * D + j4 * 4);
  }
}

// tile0_ready: attn_prefetch already issued the first tile's cache rows.
template <int D>
__device__ __forceinline__ bool attn_item(const AttnArgs a, int kvh, int split, int chunk, int n_ctx,
                                       int pos, bool append, int n_used, uint32_t tag_qkv,
                                       uint32_t tag_att, float* sm, Shared& S, uint32_t& gc,
                                       unsigned long long* tp, bool tile0_ready) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.nq / a.nkv, kvd = a.nkv * D;
  float* qs = sm;                       // [G][D]
  float* ks_ = qs + G * D;              // [kTileF][D+4]
  float* vs = ks_ + kTileF * (D + 4);   // [kTileF][D]
  float* ps = vs + kTileF * D;          // [G][kTileF]
  const int c0 = split * chunk, c1 = min(n_ctx, c0 + chunk);
  const int cache_end = append ? pos : n_ctx;  // rows below come from the cache
  if (tid < G) {
    S.m_s[tid] = -INFINITY;
    S.l_s[tid] = 0.f;
  }
  float o_acc[4] = {0.f, 0.f, 0.f, 0.f};  // G * D <= 1024 outputs: tid + 256 r
  for (int t0 = c0; t0 < c1; t0 += kTileF) {
    const int nt = min(kTileF, c1 - t0);
    const int nc = max(0, min(nt, cache_end - t0));
    if (!(t0 == c0 && tile0_ready)) {
      for (int i = tid; i < nc * (D / 4); i += kCThreads) {
        const int t = i / (D / 4), j4 = i % (D / 4);
        cp_async16(ks_ + t * (D + 4) + j4 * 4, a.kc + size_t(t0 + t) * kvd + kvh * D + j4 * 4);
        cp_async16(vs + t * D + j4 * 4, a.vc + size_t(t0 + t) * kvd + kvh * D + j4 * 4);
      }
    }
    if (t0 == c0 || nc < nt) {
      // q (first tile) and the position's own k and v (its last row) in one poll
      LLRange r[3];
      int nr = 0;
      if (t0 == c0) r[nr++] = LLRange{qs, a.qkv_ll + size_t(kvh) * G * D, G * D};
      if (nc < nt) {
        r[nr++] = LLRange{ks_ + nc * (D + 4), a.qkv_ll + size_t(a.nq) * D + kvh * D, D};
        r[nr++] = LLRange{vs + nc * D, a.qkv_ll + size_t(a.nq + a.nkv) * D + kvh * D, D};
      }
      if (!ll_gather3(r, nr, tag_qkv, a.abort_word, S, gc)) {
        cp_async_wait_all();
        return false;
      }
      if (t0 == c0 && tp && tid == 0) tp[1] = global_ns();
    }
    cp_async_wait_all();
    csync();
    if (t0 == c0 && tp && tid == 0) tp[2] = global_ns();
    if (warp < G) {
      const int g = warp;
      const float* qr = qs + g * D;
      float sc = -INFINITY;
      if (lane < nt) {
        const float* kr = ks_ + lane * (D + 4);
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
        sc = ((a0 + a1) + (a2 + a3)) * a.scale;
      }
      const float mt = warp_max(sc);
      const float m_old = S.m_s[g];
      const float m_new = fmaxf(m_old, mt);
      const float p = lane < nt ? expf(sc - m_new) : 0.f;
      const float lsum = warp_sum(p);
      ps[g * kTileF + lane] = p;
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
    if (t0 == c0 && tp && tid == 0) tp[3] = global_ns();
  }
  if (n_used == 1) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int idx = tid + r * kCThreads;
      if (idx < G * D) {
        const float l = S.l_s[idx / D];
        ll_store_rep_local(a.att_ll, a.nq * D, a.rep, kvh * G * D + idx, l > 0.f ? o_acc[r] / l : 0.f,
                     tag_att);
      }
    }
  } else {
    unsigned long long* part = a.part_ll + (size_t(kvh) * a.nsplit + split) * G * (D + 2);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int idx = tid + r * kCThreads;
      if (idx < G * D) ll_store_local(part + (idx / D) * (D + 2) + 2 + (idx % D), o_acc[r], tag_att);
    }
    if (tid < G) {
      ll_store_local(part + tid * (D + 2), S.m_s[tid], tag_att);
      ll_store_local(part + tid * (D + 2) + 1, S.l_s[tid], tag_att);
    }
  }
  if (tp && tid == 0) tp[8] = global_ns();
  csync();
  if (tp && tid == 0) tp[9] = global_ns();
  return true;
}

// Merge the n_used split partials of kv head kvh into its attention output.
template <int D>
__device__ __forceinline__ bool merge_head(const AttnArgs a, int kvh, int n_used, uint32_t tag_att,
                                        float* sm, Shared& S, uint32_t& gc) {
  const int G = a.nq / a.nkv, tid = threadIdx.x, rec = G * (D + 2);
  float* P = sm;                   // [n_used][G][D + 2]
  float* wv = P + n_used * rec;    // [G][n_used]
  float* Ls = wv + G * n_used;     // [G]
  if (!ll_gather(P, a.part_ll + size_t(kvh) * a.nsplit * rec, n_used * rec, tag_att, a.abort_word,
                 S, gc))
    return false;
  if (tid < G) {
    float mx = -INFINITY;
    for (int s = 0; s < n_used; ++s) mx = fmaxf(mx, P[s * rec + tid * (D + 2)]);
    float L = 0.f;
    for (int s = 0; s < n_used; ++s) {
      const float ms = P[s * rec + tid * (D + 2)];
      const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
      wv[tid * n_used + s] = w;
      L = fmaf(P[s * rec + tid * (D + 2) + 1], w, L);
    }
    Ls[tid] = L;
  }
  csync();
  for (int idx = tid; idx < G * D; idx += kCThreads) {
    const int g = idx / D, j = idx % D;
    float acc = 0.f;
    for (int s = 0; s < n_used; ++s) acc = fmaf(P[s * rec + g * (D + 2) + 2 + j], wv[g * n_used + s], acc);
    const float L = Ls[g];
    ll_store_rep_local(a.att_ll, a.nq * D, a.rep, kvh * G * D + idx, L > 0.f ? acc / L : 0.f,
                       tag_att);
  }
  csync();
  return true;
}

// D: head dim.  RA: rows per stage of the phases with K = h or n_q * d
// (QKV, O, GU); RB: of DOWN (K = I).  The LM head's warp segments are 2048
// elements (8 chunks).
template <int D, int RA, int RB>
__global__ void __launch_bounds__(kFThreads, 1) decode_fused_kernel(const FusedArgs a, int nst) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  __shared__ Shared S;
  uint8_t* ring = dsm;
  // attention tiles / merge, then the gathered att (O) or act (DOWN)
  float* asm_ = reinterpret_cast<float*>(dsm + size_t(nst) * kStage);
  float* x_s = asm_ + a.attn_floats;  // [h] x as last gathered (the residual), lane-major
  float* nw_s = x_s + a.h;            // [h] the next rmsnorm weight vector, lane-major
  float* rope_s = nw_s + a.h;         // [D] cos, sin of the step's position
  // [L] the per-layer pointer table, read every phase by every role
  FusedLayer* layers_s = reinterpret_cast<FusedLayer*>(rope_s + D);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(a.layers);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(layers_s);
    const int words = a.L * int(sizeof(FusedLayer) / 8);
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], kCWarps);
    }
    S.abort = 0;
    S.issued = 0;
    S.prod_done = 0;
    S.streaming = 0;
    S.in_attn = 0;
    S.fail[0] = S.fail[1] = 0;
    S.poll_ns = a.poll_ns ? a.poll_ns : kWaitNs;
    S.world = a.world;
    S.gid = a.rank * int(gridDim.x) + int(blockIdx.x);
    S.gn = a.world * int(gridDim.x);
    S.ll_base = a.ll_base;
    for (int r = 0; r < kMaxGroupRanks; ++r) S.ll_peer[r] = a.ll_peer[r];
    mbar_fence_init();
  }
  __syncthreads();

  if (warp >= kCWarps) {
    // warpgroup 2: the producer warp and three idle warps hand registers back
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    if (warp == kCWarps && lane == 0) {
      producer(a, layers_s, S, ring, nst);
      __threadfence_block();
      S.prod_done = 1;
    }
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));

  // ---------------- consumers ----------------
  unsigned int target = 0;  // arrivals the last grid barrier waited for
  uint32_t gc = 0;          // polls so far
  const StreamState& st = a.st;
  int pos = st.pos[0];
  int done = st.done[0];
  int n_gen = st.n_gen[0];
  uint32_t tok = st.token[0];
  RingPos rp{0, 0, 0u};
  int off = 0;
  bool ok = true;
  const int nph = a.L * 5 + 1;
  for (int step = 0; step < a.n_steps && ok && !done; ++step) {
    unsigned long long* trs =
        a.trace && step == 0 ? a.trace + size_t(blockIdx.x) * nph * kTraceWords : nullptr;
    auto tslot = [&](int i) { return trs ? trs + i * kTraceWords : nullptr; };
    const uint32_t tag0 = uint32_t(step) * uint32_t(nph);  // phase p writes tag0 + p + 1
    // the first rmsnorm's weights and the RoPE row of this position
    stage_vec_perm(nw_s, layers_s[0].in_norm, a.h);
    {
      const int64_t rrow = pos < a.cap ? pos : a.cap - 1;  // the host keeps pos < cap
      stage_vec(rope_s, a.rope_cos + rrow * (D / 2), D / 2);
      stage_vec(rope_s + D / 2, a.rope_sin + rrow * (D / 2), D / 2);
    }
    const bool append = pos < a.cap;
    const int n_ctx = append ? pos + 1 : pos;
    int chunk = (n_ctx + a.max_splits - 1) / a.max_splits;
    chunk = max(kTileF, (chunk + kTileF - 1) / kTileF * kTileF);
    const int n_used = (n_ctx + chunk - 1) / chunk;
    // phases of the step: per layer QKV, ATTN, O, GU, DOWN; then HEAD
    for (int p = 0; p < nph && ok; ++p) {
      const int l = p / 5;
      const int kind = p == a.L * 5 ? 5 : p % 5;
      const uint32_t tag = tag0 + uint32_t(p) + 1u;
      unsigned long long* tp = tslot(p);
      if (tp && threadIdx.x == 0) tp[0] = global_ns();
      if (kind == 1) {
        // ---- ATTN: partials of this CTA's items, then the merges it owns ----
        if (threadIdx.x == 0) S.in_attn = 1;
        AttnArgs aa;
        aa.qkv_ll = a.qkv_ll;
        aa.kc = layers_s[l].kc;
        aa.vc = layers_s[l].vc;
        aa.part_ll = a.part_ll;
        aa.att_ll = a.att_ll;
        aa.rep = a.ll_rep;
        aa.abort_word = a.bar + 2;
        aa.nq = a.nq;
        aa.nkv = a.nkv;
        aa.nsplit = a.nsplit;
        aa.scale = a.scale;
        for (int item = int(blockIdx.x); item < a.nkv * n_used && ok; item += int(gridDim.x))
          ok = attn_item<D>(aa, item / n_used, item % n_used, chunk, n_ctx, pos, append, n_used,
                            tag - 1u, tag, asm_, S, gc, item == int(blockIdx.x) ? tp : nullptr,
                            item == int(blockIdx.x));
        if (tp && threadIdx.x == 0) tp[5] = global_ns();
        if (n_used > 1)
          for (int item = int(blockIdx.x); item < a.nkv * n_used && ok; item += int(gridDim.x))
            if (item % n_used == 0) ok = merge_head<D>(aa, item / n_used, n_used, tag, asm_, S, gc);
        if (tp && threadIdx.x == 0) tp[6] = global_ns();
        if (!ok) raise_abort(a);
        continue;
      }
      const int ph = kind == 0 ? PH_QKV : kind == 2 ? PH_O : kind == 3 ? PH_GU
                   : kind == 4 ? PH_DOWN : PH_HEAD;
      const int lw = ph == PH_HEAD ? 0 : l;
      const PhaseGeo g = geo(a, layers_s, ph, lw);
      // the rmsnorm weights two phases ahead go to nw_s now (its last reader,
      // the previous rmsnorm, is behind a CTA barrier)
      if (ph == PH_O) stage_vec_perm(nw_s, layers_s[l].post_norm, a.h);
      if (ph == PH_DOWN)
        stage_vec_perm(nw_s, l + 1 < a.L ? layers_s[l + 1].in_norm : a.final_norm, a.h);
      // the phase input in shared memory (lane-major): for QKV and GU the
      // rmsnorm input x * w (in place over the staged weights nw_s, the raw x
      // kept in x_s for the residual, each warp's share of sum(x^2) in
      // S.ssq; the 1/rms factor goes on each row's dot product in the
      // epilogue); x for HEAD (normalised per warp); att for O; act for DOWN
      const float* src = x_s;
      // the tag this phase's input carries (a never-written one in the
      // failure-path test)
      const uint32_t want = step == 0 && p == a.stall_phase ? (tag - 1u) ^ 0x80000000u : tag - 1u;
      if (ph == PH_QKV && l == 0) {
        cp_async_wait_all();  // nw_s (staged at the step's start)
        csync();
        src = nw_s;
        const uint16_t* erow = a.embed + size_t(tok) * a.h;
        float ss = 0.f;
        for (int k = threadIdx.x * 8; k < a.h; k += kCThreads * 8) {
          const uint4 u = *reinterpret_cast<const uint4*>(erow + k);
          const int j = perm_idx(k);  // lane-major: the 8 values split 4 + 4
          const float4 v0 = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
          const float4 v1 = make_float4(bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w));
          *reinterpret_cast<float4*>(x_s + j) = v0;
          *reinterpret_cast<float4*>(x_s + j + 128) = v1;
          float4 w0 = *reinterpret_cast<const float4*>(nw_s + j);
          float4 w1 = *reinterpret_cast<const float4*>(nw_s + j + 128);
          w0 = make_float4(w0.x * v0.x, w0.y * v0.y, w0.z * v0.z, w0.w * v0.w);
          w1 = make_float4(w1.x * v1.x, w1.y * v1.y, w1.z * v1.z, w1.w * v1.w);
          *reinterpret_cast<float4*>(nw_s + j) = w0;
          *reinterpret_cast<float4*>(nw_s + j + 128) = w1;
          ss = fmaf(v0.x, v0.x, ss); ss = fmaf(v0.y, v0.y, ss);
          ss = fmaf(v0.z, v0.z, ss); ss = fmaf(v0.w, v0.w, ss);
          ss = fmaf(v1.x, v1.x, ss); ss = fmaf(v1.y, v1.y, ss);
          ss = fmaf(v1.z, v1.z, ss); ss = fmaf(v1.w, v1.w, ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) S.ssq[warp] = ss;
        csync();
      } else if (ph == PH_O) {
        ok = ll_gather(asm_, ll_mine(a.att_ll, a.nq * a.d, a.ll_rep), a.nq * a.d, want,
                       a.bar + 2, S, gc, true);
        if (threadIdx.x == 0) S.in_attn = 0;  // the attention chain ends with att here
        src = asm_;
      } else if (ph == PH_DOWN) {
        // act in pieces of at most one gather (whole 256-element chunks)
        const unsigned long long* act = ll_mine(a.act_ll, a.I, a.ll_rep);
        for (int o = 0; o < a.I && ok; o += kMaxGather)
          ok = ll_gather(asm_ + o, act + o, min(kMaxGather, a.I - o), want, a.bar + 2, S, gc, true);
        src = asm_;
      } else {
        // x after the phase just before: the previous layer's DOWN (QKV,
        // HEAD) or this layer's O (GU)
        ok = ll_gather(x_s, ll_mine(a.x_ll, a.h, a.ll_rep), a.h, want, a.bar + 2, S, gc, true);
        cp_async_wait_all();  // nw_s (staged a phase or more ago)
        if (ok && ph != PH_HEAD) {
          // nw_s <- nw_s * x (same layout) and each warp's share of sum(x^2)
          float ss = 0.f;
          for (int j = threadIdx.x * 4; j < a.h; j += kCThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(x_s + j);
            float4 w = *reinterpret_cast<const float4*>(nw_s + j);
            w = make_float4(w.x * v.x, w.y * v.y, w.z * v.z, w.w * v.w);
            *reinterpret_cast<float4*>(nw_s + j) = w;
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
          }
          ss = warp_sum(ss);
          if (lane == 0) S.ssq[warp] = ss;
          src = nw_s;
        }
        csync();
      }
      if (!ok) {
        raise_abort(a);
        break;
      }
      // the cache rows of this CTA's first attention item of the layer start
      // loading now (the region is free until the attention phase; no
      // cp.async wait comes before attn_item's)
      if (ph == PH_QKV && int(blockIdx.x) < a.nkv * n_used) {
        const int item = int(blockIdx.x);
        attn_prefetch<D>(layers_s[l].kc, layers_s[l].vc, a.nkv, a.nq / a.nkv, item / n_used,
                         item % n_used, chunk, n_ctx, append ? pos : n_ctx, asm_);
      }
      if (tp && threadIdx.x == 0) tp[1] = global_ns();
      const bool imm = ph == PH_HEAD && g.ks == 1;
      unsigned long long best = 0;
      // the rmsnorm factor of QKV / GU (S.ssq is complete after the gather's
      // barrier), ready before the epilogue needs it
      const float rscale = (ph == PH_QKV || ph == PH_GU) ? rms_scale(S, a.h, a.eps) : 1.f;
      int nloc = 0;
      if (ph == PH_HEAD) {
        nloc = gemv_block(g.ngroups, g.K, g.ks, g.rpg, g.N, 8, src, nw_s, a.eps, a.h, off, rp,
                          nst, ring, S, imm, a.logits, best, tp);
      } else if (ph == PH_DOWN) {
        nloc = gemv_kseg<RB>(g.ngroups, g.K, g.K / (kCWarps * 256), src, off, rp, nst, ring, S, tp);
      } else {
        nloc = gemv_kseg<RA>(g.ngroups, g.K, g.K / (kCWarps * 256), src, off, rp, nst, ring, S, tp);
      }
      if (tp && threadIdx.x == 0) {
        tp[5] = global_ns();
        tp[7] = nloc;
      }
      if (!imm) {
        csync();
        const long long ce = tp ? clock64() : 0;
        switch (ph) {
          case PH_QKV:
            epi_qkv(a, layers_s[lw], lw, g, off, nloc, pos, append, rope_s, rscale, tag, S);
            break;
          case PH_GU: epi_swiglu(a.act_ll, a.ll_rep, g, off, nloc, rscale, tag, S); break;
          case PH_HEAD: epi_head(a.logits, g, off, nloc, S, best); break;
          default: epi_residual(a.x_ll, a.ll_rep, x_s, g, off, nloc, tag, S); break;
        }
        if (tp && threadIdx.x == 0) tp[9] = clock64() - ce;
      }
      csync();  // x_s, asm_ and S.res are free for the next phase
      off = (off + g.ngroups) % cta_gn(S);
      if (ph == PH_HEAD) {
        best = warp_max_u64(best);
        if (lane == 0) S.best[warp] = best;
        csync();
        if (threadIdx.x == 0) {
          unsigned long long bb = 0;
          for (int w = 0; w < kCWarps; ++w) bb = S.best[w] > bb ? S.best[w] : bb;
          if (!kGroup) {
            a.am_part[blockIdx.x] = bb;
          } else {  // every rank's table, at this CTA's index in the joint grid
            for (int r = 0; r < a.world; ++r)
              asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(a.am_peer[r] + cta_gid(S)),
                           "l"(bb)
                           : "memory");
          }
        }
        // the one grid barrier of a step: the argmax partials, and the cache
        // rows appended this step, are visible everywhere after it
        ok = grid_sync(a, target, S, nullptr);
      }
    }
    if (!ok) break;
    // every CTA reduces the argmax partials: the same token everywhere
    {
      unsigned long long b = 0;
      for (int i = threadIdx.x; i < cta_gn(S); i += kCThreads) {
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
  // The stream stops here.  When generation ended early (EOS) or a wait gave
  // up, the producer may have issued stages nobody consumed: tell it to
  // stop, keep releasing what it issued until it has stopped, then wait for
  // the copies of the last nst issued stages (the only ones that can still
  // be in flight), so no copy lands after the CTA exits.
  if (threadIdx.x == 0) S.abort = 1;
  {
    const unsigned long long t0 = global_ns();
    for (;;) {
      const int pdone = S.prod_done;
      const int issued = S.issued;
      if (rp.it < issued) {
        mbar_wait(&S.full[rp.s], rp.par);
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.empty[rp.s]);
        rp.next(nst);
      } else if (pdone || global_ns() - t0 > kWaitNs) {
        break;
      }
    }
  }
  csync();
  if (threadIdx.x == 0) {
    const int issued = S.issued;
    for (int j = max(0, issued - nst); j < issued; ++j) mbar_wait(&S.full[j % nst], (j / nst) & 1);
  }
}

// Whether every instance was compiled with the register count the
// warpgroup split assumes (set by fused_prepare; otherwise the fused path is
// not used, since a consumer's setmaxnreg.inc could then wait forever).
bool g_regs_ok = true;

template <int D, int RA, int RB>
cudaError_t prepare_one() {
  cudaFuncAttributes fa{};
  TMG_CUDA_TRY(cudaFuncGetAttributes(&fa, decode_fused_kernel<D, RA, RB>));
  if (fa.sharedSizeBytes > kStaticReserve) return cudaErrorInvalidConfiguration;
  if (fa.numRegs != kLaunchRegs) g_regs_ok = false;
  int dev = 0, optin = 0;
  TMG_CUDA_TRY(cudaGetDevice(&dev));
  TMG_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  return set_carveout(decode_fused_kernel<D, RA, RB>, optin - int(fa.sharedSizeBytes));
}

int ksplit_host(int K) {
  int ks = 1;
  while (K / ks > 2048) ks *= 2;
  return ks;
}

// K is split over 1, 2, 4 or 8 warps so that a warp's segment is a whole
// number of 256-element chunks, at most 2048 elements.
bool seg_ok(int K) {
  const int ks = ksplit_host(K);
  return ks <= 8 && K % (ks * 256) == 0;
}

// Groups one CTA takes in a phase of ngroups groups (deferred phases hold
// one result per warp and group in shared memory).
bool local_ok(int64_t ngroups, int num_sms) {
  return (ngroups + num_sms - 1) / num_sms <= kMaxLocal;
}
// The (QKV/O/GU, DOWN) rows-per-stage pairs with a kernel instance: 2048-
// and 8192-wide rows (1B-class shapes), 4096- and 14336-wide rows (8B-class
// shapes).
bool rows_ok(int ra, int rb) { return (ra == 8 && rb == 2) || (ra == 4 && rb == 1); }

// The same for a layer phase of rpc rows per group (8 partial sums per row).
bool local_ok_k(int64_t ngroups, int num_sms, int rpc) {
  return (ngroups + num_sms - 1) / num_sms * rpc * kCWarps <= kMaxRes;
}

}  // namespace

#if TMG_FUSED_GROUP
// The group instances: prepared with the single-GPU ones and launched by
// launch_decode_fused when the arguments name more than one rank.
cudaError_t fused_group_prepare(bool* regs_ok) {
  TMG_CUDA_TRY((prepare_one<64, 8, 2>()));
  TMG_CUDA_TRY((prepare_one<128, 4, 1>()));
  TMG_CUDA_TRY((prepare_one<128, 8, 2>()));
  *regs_ok = g_regs_ok;
  return cudaSuccess;
}

cudaError_t fused_group_launch(const cudaLaunchConfig_t& cfg, const FusedArgs& a, int nst, int ra,
                               int rb) {
  if (a.d == 64 && ra == 8 && rb == 2) return cudaLaunchKernelEx(&cfg, decode_fused_kernel<64, 8, 2>, a, nst);
  if (a.d == 128 && ra == 8 && rb == 2)
    return cudaLaunchKernelEx(&cfg, decode_fused_kernel<128, 8, 2>, a, nst);
  if (a.d == 128 && ra == 4 && rb == 1)
    return cudaLaunchKernelEx(&cfg, decode_fused_kernel<128, 4, 1>, a, nst);
  return cudaErrorInvalidValue;
}
#else
namespace {
bool g_group_regs_ok = true;  // the group instances' register counts (fused_group_prepare)
}  // namespace

bool fused_supported(int h, int nq, int nkv, int d, int I, int64_t V, int num_sms) {
  if (!g_regs_ok || nkv <= 0 || nq % nkv != 0) return false;
  const int G = nq / nkv, q_dim = nq * d;
  // layer GEMVs split K over the 8 warps in whole 256-element chunks; the
  // LM head's warp segments are 2048 wide; a kernel instance for the rows
  // per stage
  if (h % (kCWarps * 256) != 0 || q_dim % (kCWarps * 256) != 0 || I % (kCWarps * 256) != 0)
    return false;
  if (h / ksplit_host(h) != 2048 || ksplit_host(q_dim) != ksplit_host(h) ||
      !rows_ok(kCWarps / ksplit_host(h), kCWarps / ksplit_host(I)))
    return false;
  if (!(seg_ok(h) && seg_ok(q_dim) && seg_ok(I) && (d == 64 || d == 128) && G >= 1 && G <= 8 &&
        G * d <= 4 * kCThreads))
    return false;
  // every tagged exchange but act fits one gather (a kv head's queries: one
  // word pair per thread; act is gathered in pieces)
  if (h > kMaxGather || q_dim > kMaxGather || G * (d + 2) > kMaxGather || G * d > 2 * kCThreads)
    return false;
  if ((d == 64 && !rows_ok(8, kCWarps / ksplit_host(I))) ||
      (kCWarps / ksplit_host(h) == 4 && d != 128))
    return false;  // the kernel instances: <64, 8, 2>, <128, 8, 2>, <128, 4, 1>
  // QKV groups hold rpc/2 rows from each RoPE half of a head
  const int rpc_h = kCWarps / ksplit_host(h);
  if (rpc_h < 2 || d % rpc_h != 0 || (d / 2) % (rpc_h / 2) != 0) return false;
  const int rpc_q = kCWarps / ksplit_host(q_dim), rpc_i = kCWarps / ksplit_host(I);
  const int64_t groups[5] = {int64_t(nq + 2 * nkv) * d / rpc_h, (h + rpc_q - 1) / rpc_q,
                             (I + rpc_h / 2 - 1) / (rpc_h / 2), (h + rpc_i - 1) / rpc_i,
                             (V + rpc_h - 1) / rpc_h};
  // every CTA owns groups in every phase (what makes reusing the tagged
  // buffers safe), and the deferred phases fit the per-warp result table
  for (int i = 0; i < 5; ++i)
    if (groups[i] < num_sms) return false;
  return local_ok_k(groups[0], num_sms, rpc_h) && local_ok_k(groups[1], num_sms, rpc_q) &&
         local_ok_k(groups[2], num_sms, rpc_h) && local_ok_k(groups[3], num_sms, rpc_i) &&
         (ksplit_host(h) == 1 || local_ok(groups[4], num_sms));
}

int fused_bar_words() { return kBarWords; }

// Attention splits per kv head the fused kernel may use for a cache of
// `capacity` positions: one kTileF-position tile per split, as many as one
// merge can gather.
int fused_nsplit(int G, int d, int64_t capacity) {
  const int64_t tiles = (capacity + kTileF - 1) / kTileF;
  const int64_t most = kMaxGather / (int64_t(G) * (d + 2));
  return int(std::max<int64_t>(1, std::min(tiles, most)));
}

// Dynamic shared memory: the ring (as many 32 KB stages as fit, at most
// max_stages or 6); a region for the attention tiles, the merge's gathered
// partials, the gathered att or act (the largest; *attn_floats); x as last
// gathered (h); one rmsnorm weight vector (h); a RoPE row (d); the per-layer
// pointer table (L FusedLayer).  *max_splits:
// the most attention splits one merge can gather.
size_t fused_smem(int h, int q_dim, int I, int d, int G, int nsplit, int L, int max_stages,
                  int* nst_out, int* attn_floats, int* max_splits) {
  *max_splits = std::max(1, std::min(nsplit, kMaxGather / (G * (d + 2))));
  const size_t tiles =
      size_t(G) * d + size_t(kTileF) * (d + 4) + size_t(kTileF) * d + size_t(G) * kTileF;
  const size_t merge = size_t(*max_splits) * G * (d + 2) + size_t(G) * *max_splits + G;
  const size_t att = std::max(std::max(tiles, merge), std::max(size_t(q_dim), size_t(I)));
  *attn_floats = int((att + 3) / 4 * 4);  // keep what follows 16-byte aligned
  const size_t rest = (size_t(*attn_floats) + 2 * size_t(h) + d) * 4 + size_t(L) * sizeof(FusedLayer);
  // the kernel's static shared memory and the 1 KB alignment slack of the
  // dynamic segment come out of the 227 KB
  const size_t budget = 227 * 1024 - kStaticReserve - 1024;
  int nst = budget > rest ? int((budget - rest) / kStage) : 0;
  nst = std::min(nst, max_stages > 0 ? std::min(max_stages, kMaxStagesF) : kMaxStagesF);
  *nst_out = nst;
  return size_t(nst) * kStage + rest;
}

cudaError_t fused_prepare() {
  TMG_CUDA_TRY((prepare_one<64, 8, 2>()));
  TMG_CUDA_TRY((prepare_one<128, 4, 1>()));
  TMG_CUDA_TRY((prepare_one<128, 8, 2>()));
  return fused_group_prepare(&g_group_regs_ok);
}

int fused_group_ctas(int h, int nq, int nkv, int d, int I, int64_t V, int num_sms, int world) {
  if (world < 1 || world > kMaxGroupRanks || !fused_supported(h, nq, nkv, d, I, V, num_sms) ||
      (world > 1 && !g_group_regs_ok))
    return 0;
  const int rpc_h = kCWarps / ksplit_host(h), rpc_q = kCWarps / ksplit_host(nq * d),
            rpc_i = kCWarps / ksplit_host(I);
  const int64_t groups[5] = {int64_t(nq + 2 * nkv) * d / rpc_h, (h + rpc_q - 1) / rpc_q,
                             (I + rpc_h / 2 - 1) / (rpc_h / 2), (h + rpc_i - 1) / rpc_i,
                             (V + rpc_h - 1) / rpc_h};
  // every CTA of the joint grid owns a group of every phase
  int64_t ctas = num_sms;
  for (int i = 0; i < 5; ++i) ctas = std::min<int64_t>(ctas, groups[i] / world);
  return int(std::max<int64_t>(ctas, 0));
}

cudaError_t fused_zero(const FusedArgs& a, cudaStream_t s) {
  // the grid barrier counts from zero in every launch, and the tagged
  // exchange buffers hold no tag of this launch
  const int G = a.nq / a.nkv;
  TMG_CUDA_TRY(cudaMemsetAsync(a.bar, 0, 4 * sizeof(unsigned int), s));
  TMG_CUDA_TRY(cudaMemsetAsync(a.ll_base, 0, a.ll_bytes, s));
  return cudaMemsetAsync(a.part_ll, 0,
                         size_t(a.nkv) * a.nsplit * G * (a.d + 2) * sizeof(unsigned long long), s);
}

cudaError_t launch_decode_fused(const FusedArgs& args, int grid, cudaStream_t s, bool zero) {
  FusedArgs a = args;
  int nst = 0;
  const int G = a.nq / a.nkv;
  const size_t smem = fused_smem(a.h, a.nq * a.d, a.I, a.d, G, a.nsplit, a.L, a.max_stages, &nst,
                                 &a.attn_floats, &a.max_splits);
  if (nst < 2 || !a.x_ll || !a.att_ll || !a.act_ll || !a.qkv_ll || !a.part_ll || a.pf_ahead < 0 || a.pf_pace < 0 ||
      a.ll_rep < 1 || grid < 1 || a.world < 1 || a.world > kMaxGroupRanks || a.rank < 0 ||
      a.rank >= a.world)
    return cudaErrorInvalidValue;
  if (a.world > 1) {
    for (int r = 0; r < a.world; ++r)
      if (!a.ll_peer[r] || !a.part_peer[r] || !a.bar_peer[r] || !a.am_peer[r])
        return cudaErrorInvalidValue;
    if (!a.kv_peer || a.trace) return cudaErrorInvalidValue;
  }
  const int ra = kCWarps / ksplit_host(a.h), rb = kCWarps / ksplit_host(a.I);
  if (!rows_ok(ra, rb)) return cudaErrorInvalidValue;
  if (zero) TMG_CUDA_TRY(fused_zero(a, s));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.world > 1) return fused_group_launch(cfg, a, nst, ra, rb);
  if (a.d == 64 && ra == 8 && rb == 2) return cudaLaunchKernelEx(&cfg, decode_fused_kernel<64, 8, 2>, a, nst);
  if (a.d == 128 && ra == 8 && rb == 2)
    return cudaLaunchKernelEx(&cfg, decode_fused_kernel<128, 8, 2>, a, nst);
  if (a.d == 128 && ra == 4 && rb == 1)
    return cudaLaunchKernelEx(&cfg, decode_fused_kernel<128, 4, 1>, a, nst);
  return cudaErrorInvalidValue;
}
#endif  // TMG_FUSED_GROUP

}  // namespace tmg
