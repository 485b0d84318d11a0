// Kernel launchers of the token-loop library (host-callable).  Every
// launcher enqueues on `s` and returns the launch status.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace tmg {

constexpr int kMaxStreams = 16;  // streams batched in one decode step
constexpr int kMaxEos = 8;

// Per-stream state of the token loop, resident in device memory so that a
// captured CUDA graph can be replayed step after step.
struct StreamState {
  uint32_t* token;  // [M] token fed to the next forward
  int32_t* pos;     // [M] KV length = position of the next token
  int32_t* done;    // [M] 1 once EOS was sampled or max_tokens reached
  int32_t* n_gen;   // [M] tokens generated so far
  uint32_t* gen;    // [M, gen_cap] generated ids
  int32_t gen_cap;  // max_tokens; 0 = plain forward (nothing recorded)
  int32_t n_eos;
  uint32_t eos[kMaxEos];
};

// Optional device timeline of one forward (tmg_trace_decode): per launch
// slot, [0] first CTA start, [1] first CTA past griddepcontrol.wait,
// [2] last CTA past the wait, [3] last CTA end (globaltimer ns).
struct Trace {
  unsigned long long* buf = nullptr;
  int slot = 0;
};
__device__ __forceinline__ void trace_mark(const Trace& t, int what) {
  if (t.buf == nullptr) return;
  unsigned long long now;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(now));
  unsigned long long* p = t.buf + t.slot * 4 + what;
  if (what == 0 || what == 1) atomicMin(p, now);
  else atomicMax(p, now);
}

// Record a chosen token for stream m (the body of generate's loop after
// sampling, src/model.rs:648-653): push it, stop on EOS.  After max_tokens
// tokens the next call only marks the stream done (the reference's final,
// unused forward_token has run by then, model.rs:655).
__device__ __forceinline__ void finish_step(const StreamState& st, int m, uint32_t tok) {
  if (st.done[m]) return;
  int n = st.n_gen[m];
  if (n >= st.gen_cap) {
    st.done[m] = 1;
    return;
  }
  st.gen[size_t(m) * st.gen_cap + n] = tok;
  st.n_gen[m] = n + 1;
  st.token[m] = tok;
  for (int e = 0; e < st.n_eos; ++e)
    if (st.eos[e] == tok) st.done[m] = 1;
}

// ---------------------------------------------------------------------------
// Decode GEMV: y[m, n] = sum_k xin[m, k] * W[n, k] for M <= 16 rows.
// ---------------------------------------------------------------------------
enum GemvPro : int {
  PRO_NONE = 0,        // xin = x
  PRO_NORM = 1,        // xin = rmsnorm(x) * norm_w
  PRO_EMBED_NORM = 2,  // x = embed[token] (written to x_out), xin = rmsnorm(x) * norm_w
};
enum GemvEpi : int {
  EPI_STORE = 0,        // y = acc
  EPI_ADD = 1,          // y += acc (residual add)
  EPI_SWIGLU = 2,       // rows come in (gate, up) pairs: y = silu(gate) * up
  EPI_HEAD = 3,         // y = acc; the last CTA advances pos (end of a forward)
  EPI_HEAD_ARGMAX = 4,  // EPI_HEAD + argmax per stream + finish_step
};

struct GemvArgs {
  const uint16_t* w = nullptr;   // [N, K] bf16 (gate rows for SwiGLU)
  const uint16_t* w2 = nullptr;  // [N, K] up rows (SwiGLU)
  const float* x = nullptr;      // [M, K]
  const uint16_t* embed = nullptr;
  const uint32_t* tokens = nullptr;
  float* x_out = nullptr;        // [M, K] residual written by PRO_EMBED_NORM
  const float* norm_w = nullptr;
  float eps = 0.f;
  int norm_mode = 0;  // 0: (v*inv)*w (rms_norm_into); 1: v*(inv*w) (rms_norm_batch)
  float* y = nullptr;  // [M, ldy]
  int64_t ldy = 0;
  int64_t N = 0;
  int K = 0;
  int M = 1;
  // EPI_HEAD / EPI_HEAD_ARGMAX
  unsigned long long* am_part = nullptr;  // [grid, M]
  unsigned int* ticket = nullptr;
  StreamState st{};
  int32_t* err = nullptr;  // device error word (2 = a bounded wait gave up)
  Trace trace{};
};

cudaError_t launch_gemv(const GemvArgs& a, GemvPro pro, GemvEpi epi, cudaStream_t s, bool pdl,
                        int num_sms);

// ---------------------------------------------------------------------------
// Int8 weights (gemv_i8.cu): per-row quantized matrices, the reference's
// TMG_I8=1 path.
// ---------------------------------------------------------------------------
struct GemvI8Args {
  const int8_t* q = nullptr;        // [N, K] (gate rows for SwiGLU)
  const int8_t* q2 = nullptr;       // [N, K] up rows (SwiGLU)
  const float* scales = nullptr;    // [N]
  const float* scales2 = nullptr;   // [N] (SwiGLU up rows)
  const float* x = nullptr;         // [M, K] activation rows (f32)
  const float* norm_w = nullptr;    // RMSNorm weights applied to x first, or null
  float eps = 0.f;
  int norm_mode = 0;
  int8_t* xq = nullptr;             // [M, K] scratch: quantized rows (M > 1)
  float* xs = nullptr;              // [M] scratch: their scales (M > 1)
  float* y = nullptr;               // [M, ldy]
  int64_t ldy = 0;
  int64_t N = 0;
  int K = 0;
  int M = 1;
  int32_t* err = nullptr;
};
// y = quantize_row_i8(x) . Q^T scaled (EPI_STORE, EPI_ADD or EPI_SWIGLU).
cudaError_t launch_gemv_i8(const GemvI8Args& a, GemvEpi epi, cudaStream_t s, bool pdl, int num_sms);
// Whether one activation row of this K takes the fused-prologue TMA kernel.
bool gemv_i8_tma_ok(int K, int M);
// WMat::quantize_i8 of a BF16 [N, K] matrix: q [N, K], scales [N].
cudaError_t launch_quantize_w_i8(const uint16_t* w, int64_t N, int K, int8_t* q, float* scales,
                                 cudaStream_t s);
// out = q widened to BF16 (exact), n % 4 == 0.
cudaError_t launch_widen_i8(const int8_t* q, size_t n, uint16_t* out, cudaStream_t s);
// y[t, o] (+)= acc[t, o] * scales[o] for T rows of N.
cudaError_t launch_scale_rows(const float* acc, int64_t T, int64_t N, const float* scales, float* y,
                              int64_t ldy, bool add, cudaStream_t s);
cudaError_t gemv_i8_prepare();
// True when the fused one-row kernel takes this shape (prologues need it).
bool gemv_fused_ok(const GemvArgs& a, GemvEpi epi);
// Once per device, before any launch or capture: kernel attributes
// (dynamic shared memory limits).
cudaError_t gemv_prepare();
cudaError_t attn_prepare();
cudaError_t prefill_prepare();
cudaError_t sample_prepare();
// Scratch the launcher needs for EPI_HEAD*: number of CTAs it will use.
int gemv_grid(const GemvArgs& a, GemvEpi epi, int num_sms);

// ---------------------------------------------------------------------------
// Decode attention (split-KV, online softmax, in-kernel combine), with RoPE
// of q/k and the KV append fused in.
// ---------------------------------------------------------------------------
struct AttnDecodeArgs {
  const float* qkv = nullptr;  // [M, qkv_ld]: q | k | v, before RoPE
  int64_t qkv_ld = 0;
  float* kc = nullptr;  // layer cache [M, cap, kv_dim]
  float* vc = nullptr;
  int64_t cap = 0;
  const float* rope_cos = nullptr;  // [cap, d/2]
  const float* rope_sin = nullptr;
  float* out = nullptr;  // [M, n_q * d]
  float* part = nullptr;  // [M, n_kv, nsplit, G, d + 2]
  unsigned int* ticket = nullptr;  // [M, n_kv]
  StreamState st{};
  const int32_t* pos_override = nullptr;  // op-level: fixed n_ctx - 1 (no append)
  int32_t* err = nullptr;  // device error word (2 = a bounded wait gave up), or null
  int nq = 0, nkv = 0, d = 0, nsplit = 1, M = 1;
  float scale = 1.f;
  Trace trace{};
};
cudaError_t launch_attn_decode(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);
// The TMA-staged decode attention (attn_tma.cu): head dim 64 or 128, at most
// 4 query heads per kv head; launch_attn_decode picks it when it applies.
bool attn_decode_tma_ok(int nq, int nkv, int d, int64_t cap, int M, const void* kc, const void* vc);
size_t attn_decode_tma_smem(int d);
cudaError_t launch_attn_decode_tma(const AttnDecodeArgs& a, cudaStream_t s, bool pdl);
cudaError_t attn_tma_prepare();
int attn_decode_nsplit(int nkv, int M, int64_t cap, int num_sms);
// Whether launch_attn_decode takes this op-level shape (n_q, n_kv, head dim,
// context length, split count); *why says why not.
bool attn_decode_shape_ok(int nq, int nkv, int d, int64_t n_ctx, int nsplit, std::string* why);
// Decode attention on the static per-device scratch (attn_noalloc.cu):
// enqueues on s, allocates nothing.  0 = enqueued; 1 bad device, 2 too
// large for the scratch, 3 CUDA error; *why says which.
int attn_decode_noalloc(int device, int num_sms, cudaStream_t s, const float* q, const float* keys,
                        const float* values, int64_t n_ctx, int n_q, int n_kv, int head_dim,
                        float* out, std::string* why);

// ---------------------------------------------------------------------------
// Prefill pieces.
// ---------------------------------------------------------------------------
// x[t, :] = embed[tokens[t], :] (bf16 -> f32).
cudaError_t launch_embed(const uint16_t* embed, const uint32_t* tokens, int64_t T, int h, float* x,
                         cudaStream_t s);
// out = rmsnorm rows (mode 0: (v*inv)*w, mode 1: v*(inv*w)).
cudaError_t launch_rmsnorm(const float* x, const float* w, float eps, int64_t n, int64_t rows,
                           int mode, float* out, cudaStream_t s);
// rms_norm_batch (mode 1) written as the BF16 hi/lo parts of its result
// (the tcgen05 GEMM's operands) instead of f32.
cudaError_t launch_rmsnorm_split(const float* x, const float* w, float eps, int64_t n,
                                 int64_t rows, uint16_t* hi, uint16_t* lo, cudaStream_t s);
// Rotate q and k of T rows in place (qkv layout) at positions pos0.., and
// append rotated k and raw v to the cache at pos0...
cudaError_t launch_rope_append(float* qkv, int64_t qkv_ld, int64_t T, int nq, int nkv, int d,
                               const float* rope_cos, const float* rope_sin, int64_t pos0,
                               float* kc, float* vc, cudaStream_t s);
// Rotate rows of n_heads heads in place (op level).
cudaError_t launch_rope_rows(float* x, int64_t ld, int64_t rows, int n_heads, int d,
                             const float* rope_cos, const float* rope_sin, int64_t pos0,
                             cudaStream_t s);
// Causal attention of T query rows (positions pos0..pos0+T-1) over cache
// rows [0, pos0 + T).
cudaError_t launch_attn_prefill(const float* q, int64_t q_ld, const float* kc, const float* vc,
                                int64_t T, int64_t pos0, int nq, int nkv, int d, float scale,
                                float* out, int64_t out_ld, cudaStream_t s);
// The same attention on tcgen05 tensor cores (attn_prefill_tc.cu), head dim
// 64: q, k and v^T are split into BF16 parts in `scratch` (at least
// attn_prefill_tc_scratch bytes) by two kernels before the MMA kernel.
bool attn_prefill_tc_ok(const float* q, int64_t q_ld, const float* kc, const float* vc, int64_t T,
                        int64_t pos0, int nq, int nkv, int d, const void* out, int64_t out_ld);
size_t attn_prefill_tc_scratch(int nq, int nkv, int64_t T, int64_t Lk);
cudaError_t attn_prefill_tc_prepare();
// out_hi / out_lo (both or neither): the output written as its BF16 hi/lo
// parts (the O GEMM's operands) instead of f32 into out.  With rope_cos /
// rope_sin, q points at the chunk's un-rotated projections (rows of q_ld:
// q | k | v): RoPE, the KV append to kc / vc and the operand parts are done
// in one pass (launch_rope_append is then not needed).
cudaError_t launch_attn_prefill_tc(const float* q, int64_t q_ld, const float* kc, const float* vc,
                                   int64_t T, int64_t pos0, int nq, int nkv, float scale,
                                   float* out, uint16_t* out_hi, uint16_t* out_lo, int64_t out_ld,
                                   void* scratch, size_t scratch_bytes, int32_t* err,
                                   cudaStream_t s, const float* rope_cos = nullptr,
                                   const float* rope_sin = nullptr);
// out = gate / (1 + exp(-gate)) * up.
cudaError_t launch_swiglu(const float* gate, const float* up, int64_t n, float* out,
                          cudaStream_t s);
// y[T, N] (+)= x[T, K] . W^T  (SIMT f32 path, any shape).
cudaError_t launch_gemm_simt(const float* x, const uint16_t* w, int64_t T, int64_t N, int64_t K,
                             float* y, int64_t ldy, bool accumulate, cudaStream_t s);
// Tensor-core prefill GEMM (tcgen05): y[T, N] (+)= (x_hi + x_lo)[T, K] . W^T
// with x split into two BF16 operands by launch_split.  err: device error
// word (2 when a bounded wait gave up).
bool gemm_tc_supported(int64_t K, const void* w);
cudaError_t gemm_tc_prepare();
cudaError_t launch_split(const float* x, int64_t n, uint16_t* hi, uint16_t* lo, cudaStream_t s);
// The SwiGLU of launch_swiglu written as the hi/lo BF16 split of its result
// (the down GEMM's operands); needs n % 4 == 0, g and u 16-byte aligned.
bool swiglu_split_supported(const float* g, const float* u, int64_t n, const uint16_t* hi,
                            const uint16_t* lo);
cudaError_t launch_swiglu_split(const float* g, const float* u, int64_t n, uint16_t* hi,
                                uint16_t* lo, cudaStream_t s);
cudaError_t launch_gemm_tc(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* w,
                           int64_t T, int64_t N, int64_t K, float* y, int64_t ldy,
                           bool accumulate, int32_t* err, cudaStream_t s);
// gate and up of one input in one launch with the SwiGLU in the epilogue:
// act[T, I] = silu(x . Wg^T) * (x . Wu^T) written as its BF16 hi/lo parts
// (the down GEMM's operands); I % 16 == 0, act_hi / act_lo 32-byte aligned.
bool gemm_swiglu_supported(int64_t I, const void* act_hi, const void* act_lo);
cudaError_t launch_gemm_tc_swiglu(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* wg,
                                  const uint16_t* wu, int64_t I, int64_t T, int64_t K,
                                  uint16_t* act_hi, uint16_t* act_lo, int32_t* err,
                                  cudaStream_t s);
// The same over two weight matrices of one input in one launch: columns
// [0, N1) of W1 into y1, then [0, N2) of W2 into y2 (N2 = 0: W1 only).
cudaError_t launch_gemm_tc2(const uint16_t* x_hi, const uint16_t* x_lo, const uint16_t* w1,
                            int64_t N1, float* y1, int64_t ldy1, const uint16_t* w2, int64_t N2,
                            float* y2, int64_t ldy2, int64_t T, int64_t K, bool accumulate,
                            int32_t* err, cudaStream_t s);
// argmax per row (op level and the first greedy step).
cudaError_t launch_argmax_rows(const float* logits, int64_t V, int rows, uint32_t* out,
                               cudaStream_t s);
// dst[i] += src[i].
cudaError_t launch_add(const float* src, float* dst, int64_t n, cudaStream_t s);
// End of a forward outside the LM-head kernel (tensor parallel): pos += 1
// for the live streams and, when logits is given ([M, V]), the argmax +
// finish_step of generate.
cudaError_t launch_step_end(StreamState st, int M, const float* logits, int64_t V,
                            cudaStream_t s);
// Set pos[m] = value (device).
cudaError_t launch_set_pos(StreamState st, int m, int32_t value, cudaStream_t s);

// ---------------------------------------------------------------------------
// Sampling (apply_repetition_penalty + sample, src/tensor.rs:1142-1213).
// ---------------------------------------------------------------------------
constexpr int kMaxTopK = 64;
struct SampleArgs {
  float* logits = nullptr;  // [M, V], penalised in place
  int64_t V = 0;
  int M = 1;
  const uint32_t* generated = nullptr;  // [M, gen_ld] (NULL: use st.gen)
  int64_t gen_ld = 0;
  const int32_t* n_generated = nullptr;  // [M] (NULL: use st.n_gen)
  int64_t n_gen_fixed = -1;              // op level: same count for all rows
  float temperature = 0.f;
  int top_k = 0;
  float top_p = 1.f;
  float penalty = 1.f;
  const float* uniforms = nullptr;  // [M, uni_ld]; indexed by the step
  int64_t uni_ld = 0;
  uint32_t* next = nullptr;  // [M] (op level)
  uint32_t* cand_ids = nullptr;  // [M, top_k] (op level)
  float* cand_probs = nullptr;
  int32_t* cutoff = nullptr;
  unsigned long long* part = nullptr;  // [M, nslices, top_k]
  unsigned int* ticket = nullptr;      // [M]
  int32_t* err = nullptr;              // device error word (NaN)
  StreamState st{};
  bool record = false;  // finish_step into st
};
cudaError_t launch_sample(const SampleArgs& a, cudaStream_t s, bool pdl, int num_sms);
int sample_slices(int64_t V, int M, int num_sms);

}  // namespace tmg
