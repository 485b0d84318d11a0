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
  float* act = nullptr;     // [I]
  float* logits = nullptr;  // [V]
  unsigned long long* am_part = nullptr;  // [grid]
  unsigned int* bar = nullptr;            // [0] arrivals, [1] generation, [2] abort
  int nsplit = 1;
  int xs_floats = 0;  // max(h, nq d)
  StreamState st{};
  int n_steps = 0;
  int32_t* err = nullptr;
};

bool fused_supported(int h, int q_dim, int I, int d, int G);
size_t fused_smem(int h, int q_dim, int nq, int d, int G, int nsplit, int* nst_out);
cudaError_t fused_prepare();
// Cooperative launch: one CTA per SM (num_sms CTAs).
cudaError_t launch_decode_fused(const FusedArgs& a, int num_sms, cudaStream_t s);

}  // namespace tmg
