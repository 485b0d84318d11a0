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
  float* x = nullptr;       // [h] residual
  float* qkv = nullptr;     // [(nq + 2 nkv) d]
  float* part = nullptr;    // [nkv, nsplit, G, d + 2] attention partials
  float* att = nullptr;     // [nq d] attention output
  float* act = nullptr;     // [I]
  float* logits = nullptr;  // [V]
  unsigned long long* am_part = nullptr;  // [grid]
  // fused_bar_words() words: [0] barrier arrivals, [2] abort, [64 + kv head]
  // attention tickets (zero between launches)
  unsigned int* bar = nullptr;
  int nsplit = 1;
  int pf_ahead = 0;    // stages of L2 prefetch beyond the ring
  int max_stages = 0;  // cap on the ring's stages (0: as many as fit)
  int attn_floats = 0; // set by the launcher: attention region of shared memory
  StreamState st{};
  int n_steps = 0;
  int32_t* err = nullptr;
  // diagnostics: [grid][L * 5 + 1][12] records of the first step per CTA
  // and phase (globaltimer ns: work done, barrier passed, producer's first
  // and last issue, input ready, GEMV done, first stage ready; the group
  // count; SM cycles of stage waits and math of consumer warp 0, of free-
  // stage waits and issue work of the producer), or null
  unsigned long long* trace = nullptr;
};

bool fused_supported(int h, int nq, int nkv, int d, int I, int64_t V, int num_sms);
int fused_bar_words();
size_t fused_smem(int h, int d, int G, int nsplit, int max_stages, int* nst_out, int* attn_floats);
cudaError_t fused_prepare();
// Cooperative launch: one CTA per SM (num_sms CTAs).
cudaError_t launch_decode_fused(const FusedArgs& a, int num_sms, cudaStream_t s);

}  // namespace tmg
