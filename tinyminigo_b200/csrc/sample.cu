// On-device sampling: apply_repetition_penalty + sample (src/tensor.rs:
// 1142-1213; call site src/model.rs:631-646).
//
// Three phases in one kernel launch per step:
//  1. penalty: each distinct generated id once (the reference's HashSet),
//     l > 0 -> l / p else l * p, in place on the logits;
//  2. per vocab slice (grid.x slices per stream): the slice's top-k of
//     (scaled = l / temperature, index) with the reference's ordering --
//     larger value first, ties to the lower index (the order a stable sort
//     gives; sort_unstable_by leaves it unspecified) -- NaN and -inf never
//     selected (NaN logits set the error word; the reference panics);
//  3. the last CTA of a stream merges the slices' candidates, then one
//     thread replays the reference's sequential tail in candidate order:
//     softmax (max, exp(v - max), sequential sum, divide), the top-p cutoff
//     at the first rank whose running sum exceeds p, renormalisation over the
//     kept ranks, and the draw (first i with r < cumulative prob).
//
// exp here is f64 exp rounded to f32 (correctly rounded in practice); the
// reference's glibc expf is within 0.502 ulp, so single probabilities can
// differ by 1 ulp while the candidate set, order and cutoff are identical
// except when a running sum lies within an ulp of p or of r.
#include <math.h>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 16;
constexpr int kSlice = kThreads * kPerThread;

__device__ __forceinline__ float key_value(unsigned long long k) {
  uint32_t b = uint32_t(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7fffffffu) : ~b;
  return __uint_as_float(b);
}

// Iterative block-wide top-k over per-thread key arrays (descending).
// Thread 0's `out` receives the k best keys (0 when fewer exist).
__device__ void block_topk(unsigned long long (&keys)[kPerThread], int k, unsigned long long* out,
                           unsigned long long* warp_s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = 0; r < k; ++r) {
    unsigned long long b = 0ull;
#pragma unroll
    for (int i = 0; i < kPerThread; ++i) b = keys[i] > b ? keys[i] : b;
    b = warp_max_u64(b);
    if (lane == 0) warp_s[warp] = b;
    __syncthreads();
    unsigned long long w = warp_s[0];
    for (int i = 1; i < kThreads / 32; ++i) w = warp_s[i] > w ? warp_s[i] : w;
    if (threadIdx.x == 0) out[r] = w;
    if (w != 0ull) {
#pragma unroll
      for (int i = 0; i < kPerThread; ++i)
        if (keys[i] == w) keys[i] = 0ull;  // keys are unique (index bits)
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const SampleArgs a) {
  __shared__ unsigned long long warp_s[kThreads / 32];
  __shared__ unsigned long long top_s[kMaxTopK];
  __shared__ bool last_s;
  const int slice = blockIdx.x, m = blockIdx.y, nslices = gridDim.x;
  const int k = a.temperature <= 0.f ? 1 : a.top_k;
  float* logits = a.logits + size_t(m) * a.V;

  pdl_trigger();
  pdl_wait();
  // A finished stream skips the step in every one of its CTAs (done[m] only
  // changes in this stream's last CTA, after all the others took a ticket).
  if (a.record && a.st.done[m]) return;

  // 1. penalty: each CTA penalises the distinct generated ids that fall in
  //    its own slice, before reading the slice
  const int64_t n_gen = a.n_gen_fixed >= 0 ? a.n_gen_fixed
                        : (a.n_generated ? a.n_generated[m] : a.st.n_gen[m]);
  const uint32_t* gen = a.generated ? a.generated + size_t(m) * a.gen_ld
                                    : a.st.gen + size_t(m) * a.st.gen_cap;
  const bool pen = a.penalty != 1.0f && n_gen > 0;

  // 2. this slice's top-k of the scaled logits
  const int64_t lo = int64_t(slice) * kSlice;
  const int64_t hi = lo + kSlice < a.V ? lo + kSlice : a.V;
  if (pen) {
    for (int64_t j = threadIdx.x; j < n_gen; j += blockDim.x) {
      const uint32_t tok = gen[j];
      if (int64_t(tok) < lo || int64_t(tok) >= hi) continue;
      bool first = true;
      for (int64_t i = 0; i < j && first; ++i) first = gen[i] != tok;
      if (first) {
        const float l = logits[tok];
        logits[tok] = l > 0.0f ? l / a.penalty : l * a.penalty;
      }
    }
    __syncthreads();
  }
  unsigned long long keys[kPerThread];
#pragma unroll
  for (int i = 0; i < kPerThread; ++i) {
    const int64_t idx = lo + threadIdx.x + int64_t(i) * kThreads;
    unsigned long long kk = 0ull;
    if (idx < hi) {
      const float l = logits[idx];
      if (isnan(l) && a.err) atomicExch(a.err, 1);
      const float v = a.temperature <= 0.f ? l : l / a.temperature;
      kk = argmax_key(v, uint32_t(idx));
    }
    keys[i] = kk;
  }
  block_topk(keys, k, top_s, warp_s);
  unsigned long long* part = a.part + (size_t(m) * nslices + slice) * kMaxTopK;
  if (threadIdx.x < k) part[threadIdx.x] = top_s[threadIdx.x];

  // 3. the last slice CTA of this stream merges and draws
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(&a.ticket[m], 1u);
    last_s = (t == unsigned(nslices) - 1);
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const unsigned long long* pb = a.part + size_t(m) * nslices * kMaxTopK;
  // merge nslices * k candidates (<= kSlice of them)
#pragma unroll
  for (int i = 0; i < kPerThread; ++i) {
    const int j = threadIdx.x + i * kThreads;  // j over [0, nslices * k)
    keys[i] = j < nslices * k ? __ldcg(pb + size_t(j / k) * kMaxTopK + (j % k)) : 0ull;
  }
  block_topk(keys, k, top_s, warp_s);
  if (threadIdx.x == 0) {
    a.ticket[m] = 0u;
    uint32_t tok;
    if (a.temperature <= 0.f) {
      tok = argmax_key_index(top_s[0]);
      if (a.cutoff) a.cutoff[m] = 1;
    } else {
      // softmax over the candidates, in candidate order (tensor.rs:1177-1179)
      float vals[kMaxTopK], probs[kMaxTopK];
      int nc = 0;
      while (nc < k && top_s[nc] != 0ull) ++nc;
      float mx = -INFINITY;
      for (int i = 0; i < nc; ++i) {
        vals[i] = key_value(top_s[i]);
        mx = fmaxf(mx, vals[i]);
      }
      float sum = 0.f;
      for (int i = 0; i < nc; ++i) {
        probs[i] = float(exp(double(vals[i] - mx)));
        sum += probs[i];
      }
      for (int i = 0; i < nc; ++i) probs[i] = probs[i] / sum;
      int cut = nc;
      if (a.top_p < 1.0f) {
        // probs are non-increasing in candidate order, so the reference's
        // sort by probability (tensor.rs:1183-1184) is the identity here
        float cum = 0.f;
        for (int r = 0; r < nc; ++r) {
          cum += probs[r];
          if (cum > a.top_p) {
            cut = r + 1;
            break;
          }
        }
        float s2 = 0.f;
        for (int r = 0; r < cut; ++r) s2 += probs[r];
        for (int r = 0; r < nc; ++r) probs[r] = r < cut ? probs[r] / s2 : 0.f;
      }
      const int64_t step = n_gen;
      const float r = a.uniforms ? a.uniforms[size_t(m) * a.uni_ld + (a.record ? step : 0)] : 0.f;
      int pick = -1;
      float cum = 0.f;
      for (int i = 0; i < nc; ++i) {
        cum += probs[i];
        if (r < cum) {
          pick = i;
          break;
        }
      }
      if (pick < 0)
        for (int i = 0; i < nc && pick < 0; ++i)
          if (probs[i] > 0.f) pick = i;
      if (pick < 0) pick = 0;
      tok = argmax_key_index(top_s[pick]);
      if (a.cand_ids)
        for (int i = 0; i < k; ++i) {
          a.cand_ids[size_t(m) * k + i] = i < nc ? argmax_key_index(top_s[i]) : 0u;
          a.cand_probs[size_t(m) * k + i] = i < nc ? probs[i] : 0.f;
        }
      if (a.cutoff) a.cutoff[m] = cut;
    }
    if (a.next) a.next[m] = tok;
    if (a.record) finish_step(a.st, m, tok);
  }
}

}  // namespace

cudaError_t sample_prepare() { return set_carveout(sample_kernel); }

int sample_slices(int64_t V, int M, int num_sms) {
  (void)M;
  (void)num_sms;
  return int((V + kSlice - 1) / kSlice);
}

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t s, bool pdl, int num_sms) {
  const int k = a.temperature <= 0.f ? 1 : a.top_k;
  if (k < 1 || k > kMaxTopK || a.V <= k || a.M < 1) return cudaErrorInvalidValue;
  const int ns = sample_slices(a.V, a.M, num_sms);
  // the merge holds ns * k candidates; part buffers hold 64 slices per stream
  if (int64_t(ns) * k > kSlice || ns > 64) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ns, a.M);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, sample_kernel, a);
}

}  // namespace tmg
