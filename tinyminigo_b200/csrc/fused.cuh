// The fused batch-1 decode kernel (decode_fused.cu): arguments and launcher.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"

namespace tmg {

// Per-layer device pointers (an array of these lives in device memory).
struct FusedLayer {
  const uint16_t* wqkv;  // [(nq + 2 nkv) d, h]
  const uint16_t* wo;    // [h, nq d]
  const uint16_t* wg;    // [I, h]
  const uint16_t* wu;    // [I, h]
  const uint16_t* wd;    // [h, I]
  const float* in_norm;
  const float* post_norm;
  float* kc;  // [cap, nkv d] (stream 0)
  float* vc;
};

// Most GPUs one fused decode can span (fused_group in api.cu).
constexpr int kMaxGroupRanks = 8;

struct FusedArgs {
  const FusedLayer* layers = nullptr;
  int L = 0, h = 0, nq = 0, nkv = 0, d = 0, I = 0, V = 0;
  float eps = 0.f, scale = 1.f;
  const uint16_t* embed = nullptr;
  const uint16_t* lm_head = nullptr;
  const float* final_norm = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int64_t cap = 0;
  // tagged exchange words {value, tag} (see decode_fused.cu), zeroed by the
  // launcher: x [h], att [nq d], act [I], qkv [(nq + 2 nkv) d] in one block
  // at ll_base (ll_bytes), the attention partials [nkv, nsplit, G, d + 2]
  unsigned long long* ll_base = nullptr;
  size_t ll_bytes = 0;
  unsigned long long* x_ll = nullptr;
  unsigned long long* att_ll = nullptr;
  unsigned long long* act_ll = nullptr;
  unsigned long long* qkv_ll = nullptr;
  unsigned long long* part_ll = nullptr;
  float* logits = nullptr;  // [V]
  unsigned long long* am_part = nullptr;  // [grid]
  // fused_bar_words() words: [0] barrier arrivals, [2] abort
  unsigned int* bar = nullptr;
  int nsplit = 1;
  int pf_ahead = 0;    // stages of stall-time L2 prefetch beyond the ring
  int pf_pace = 0;     // clock cycles between two such prefetches
  int pf_mode = 0;     // 0: prefetch only in the attention chain; 1: whenever the ring is full
  int ll_rep = 1;      // copies of x_ll, att_ll and act_ll (each n words apart)
  int max_stages = 0;  // cap on the ring's stages (0: as many as fit)
  int attn_floats = 0; // set by the launcher: attention region of shared memory
  int max_splits = 1;  // set by the launcher: attention splits per kv head
  StreamState st{};
  int n_steps = 0;
  int32_t* err = nullptr;
  // limit of the tag polls and the grid barrier (ns; 0: the 2 s default)
  unsigned long long poll_ns = 0;
  // Several GPUs (world > 1): the CTAs of all ranks form one grid of world
  // x gridDim.x CTAs (this rank's are rank x gridDim.x + blockIdx.x); every
  // exchange word, attention partial, KV-cache append, argmax partial and
  // barrier arrival is written into every rank's copy (index: rank; the own
  // rank's entry is the local buffer).  Each rank holds the full weights and
  // streams the row groups its CTAs own.
  int rank = 0, world = 1;
  unsigned long long* ll_peer[kMaxGroupRanks] = {};
  unsigned long long* part_peer[kMaxGroupRanks] = {};
  unsigned int* bar_peer[kMaxGroupRanks] = {};
  unsigned long long* am_peer[kMaxGroupRanks] = {};
  float* const* kv_peer = nullptr;  // [world][L][2]: every rank's K and V cache of each layer
  // failure-path test only (-1: off): in the first step, the input gather of
  // phase stall_phase (a GEMV phase that gathers: O, GU, DOWN, a later
  // layer's QKV, HEAD) waits for a tag no phase writes, so the poll gives up
  // after poll_ns and the launch ends with the timeout error word
  int stall_phase = -1;
  // diagnostics: [grid][L * 5 + 1][12] records of the first step per CTA
  // and phase (globaltimer ns: work done, barrier passed, producer's first
  // and last issue, input ready, GEMV done, first stage ready; the group
  // count; SM cycles of stage waits and math of consumer warp 0, of free-
  // stage waits and issue work of the producer), or null
  unsigned long long* trace = nullptr;
};

bool fused_supported(int h, int nq, int nkv, int d, int I, int64_t V, int num_sms);
int fused_bar_words();
int fused_nsplit(int G, int d, int64_t capacity);
size_t fused_smem(int h, int q_dim, int I, int d, int G, int nsplit, int L, int max_stages,
                  int* nst_out, int* attn_floats, int* max_splits);
// Words of the tagged exchange block (x, att, act, qkv) of a model.
// Tagged exchange words: x, att and act in `rep` copies each (readers spread
// over the copies), then the position's q/k/v.
inline size_t fused_ll_words(int h, int q_dim, int I, int qkv_rows, int rep) {
  return size_t(rep) * (size_t(h) + q_dim + I) + qkv_rows;
}
cudaError_t fused_prepare();
// CTAs per rank when `world` GPUs share one fused decode of this shape (every
// CTA of the joint grid must own a row group of every phase), or 0.
int fused_group_ctas(int h, int nq, int nkv, int d, int I, int64_t V, int num_sms, int world);
// Zero the launch's barrier and tagged-exchange words (the launcher does it
// unless told not to: a multi-GPU launch zeroes every rank before any rank
// starts, between two host-side barriers).
cudaError_t fused_zero(const FusedArgs& a, cudaStream_t s);
// Cooperative launch of `grid` CTAs (one per SM at most).
cudaError_t launch_decode_fused(const FusedArgs& a, int grid, cudaStream_t s, bool zero = true);
// The group instances (decode_fused_group.cu): prepared by fused_prepare,
// launched by launch_decode_fused for world > 1.
cudaError_t fused_group_prepare(bool* regs_ok);
cudaError_t fused_group_launch(const cudaLaunchConfig_t& cfg, const FusedArgs& a, int nst, int ra,
                               int rb);

}  // namespace tmg
