/*
 * tmg_cuda.h — C ABI of the B200 (sm_100a) token-loop library.
 *
 * This is the boundary that replaces the CPU kernels and the forward pass of
 * HanzCEO/TinyMiniGo (citations are `path:line` in that project).  A Rust
 * engine binds it with an `extern "C"` block (the rust/tmg-cuda-sys crate of
 * this repository); the parity tests and bench.py bind it with ctypes.
 *
 * Conventions
 *  - Every call returns an int status: TMG_OK (0) or a negative TMG_ERR_*.
 *    tmg_last_error(ctx) gives the message of the last failure on ctx.
 *    (The reference returns anyhow::Result and panics on shape errors or
 *    NaN logits; here every such case is a status code.)
 *  - Model-level calls take HOST pointers.  tmg_op_* calls take DEVICE
 *    pointers (16-byte aligned) and run on the context's stream; they return
 *    after the work completes.
 *  - A context is single-threaded (the reference's `&mut self`): one host
 *    thread per context, one context per GPU.
 *  - Weights are BF16 bit patterns (uint16) laid out [out, in] row-major, as
 *    nn.Linear and the reference store them (src/tensor.rs:313-314).  All
 *    arithmetic is f32 with BF16 widened exactly.
 */
#ifndef TMG_CUDA_H
#define TMG_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMG_OK 0
#define TMG_ERR_INVALID (-1)  /* bad argument, shape or call order */
#define TMG_ERR_CUDA (-2)     /* a CUDA runtime/driver call failed */
#define TMG_ERR_IO (-3)       /* file missing or unparsable */
#define TMG_ERR_CAPACITY (-4) /* KV cache full */
#define TMG_ERR_NAN (-5)      /* NaN logits reached the sampler */
#define TMG_ERR_TIMEOUT (-6)  /* a bounded device-side wait gave up */
#define TMG_ERR_NCCL (-7)     /* a collective failed */

#define TMG_MAX_EOS 8

/* ModelConfig, src/config.rs:6-20. */
typedef struct tmg_config {
  int32_t hidden_size;
  int32_t num_hidden_layers;
  int32_t num_attention_heads;
  int32_t num_key_value_heads;
  int32_t head_dim;
  int32_t intermediate_size;
  int32_t vocab_size;
  float rms_norm_eps;
  float rope_theta;
  uint32_t bos_token_id;
  int32_t n_eos;
  uint32_t eos_token_ids[TMG_MAX_EOS];
} tmg_config;

/* GenParams, src/model.rs:597-604. */
typedef struct tmg_gen_params {
  int64_t max_tokens;
  float temperature;
  int64_t top_k;
  float top_p;
  float repetition_penalty;
  uint64_t seed;
} tmg_gen_params;

typedef struct tmg_ctx tmg_ctx; /* Model: weights, scratch, stream (src/model.rs:338-346) */
typedef struct tmg_kv tmg_kv;   /* KvCache on the device (src/model.rs:250-260) */
typedef struct tmg_wmat tmg_wmat; /* WMat on the device (src/tensor.rs:198-206) */

/* Called once per generated token from inside tmg_generate (the on_token
 * callback of src/model.rs:618; main.rs:94-100 detokenises there).  Return
 * non-zero to stop generation early. */
typedef int (*tmg_token_cb)(uint32_t token, void* user);

/* ---------------------------------------------------------------------------
 * Host-only calls (no GPU needed).
 * ------------------------------------------------------------------------ */

/* ModelConfig::load, src/config.rs:112-172 (config.json next to the weights:
 * config_path_for_model, src/config.rs:174-185, is done by the caller). */
int tmg_config_load(const char* config_json_path, tmg_config* out, char* err, int errlen);
/* ModelConfig::from_json, src/config.rs:39-93, on JSON text. */
int tmg_config_parse(const char* json_text, tmg_config* out, char* err, int errlen);
/* Safetensors header inspection, src/safetensors_loader.rs:83-147: number of
 * tensors, and for index i its name, dtype (0 F32, 1 BF16, 2 F16), rank and
 * shape (up to 4 dims), data offset and byte length. */
int tmg_safetensors_count(const char* path, int64_t* n, char* err, int errlen);
int tmg_safetensors_info(const char* path, int64_t i, char* name, int namelen, int32_t* dtype,
                         int32_t* rank, int64_t shape[4], int64_t* offset, int64_t* nbytes,
                         char* err, int errlen);
/* TMB1 (the reference's load-optimised repack) header inspection,
 * parse_tmb_header, src/tmb.rs:80-121: the embedded config (cfg may be NULL;
 * ModelConfig::from_json, src/config.rs:39-93, so an EOS list written under
 * the repack's "eos_token_ids" key is not read back, as in the reference),
 * the number of tensors, and for index i its name, absolute data offset and
 * byte length.  TMG_ERR_IO with the reference's messages on a bad file. */
int tmg_tmb_count(const char* path, tmg_config* cfg, int64_t* n, char* err, int errlen);
int tmg_tmb_info(const char* path, int64_t i, char* name, int namelen, int64_t* offset,
                 int64_t* nbytes, char* err, int errlen);
/* The reference's f16 -> f32 widening, src/safetensors_loader.rs:149-173. */
float tmg_f16_to_f32(uint16_t h);
/* Library version string. */
const char* tmg_version(void);

/* ---------------------------------------------------------------------------
 * Context and weights (Model::load, src/model.rs:383-389, 90-96, 181-244).
 * ------------------------------------------------------------------------ */

/* A context on `device` for a model of shape `cfg` (NULL: an op-only
 * context for the tmg_op_* calls). */
int tmg_create(int device, const tmg_config* cfg, tmg_ctx** out);
/* Frees the context.  KV caches and WMat handles still alive lose their
 * device memory here; their handles then accept only tmg_kv_destroy /
 * tmg_wmat_free (in either order relative to this call). */
int tmg_destroy(tmg_ctx* ctx);
/* The message of the last failure on ctx; with ctx NULL, why the last
 * tmg_create on the calling thread failed. */
const char* tmg_last_error(const tmg_ctx* ctx);

/* Upload every tensor of a safetensors file (load_model_safetensors,
 * src/model.rs:181-244): BF16 matrices (and the BF16 embedding) go to HBM
 * once, bits unchanged; norm vectors may be F32, F16 or BF16 and are kept in
 * f32.  F32/F16 matrices are rejected with TMG_ERR_INVALID: the device path
 * streams BF16 only.  A missing lm_head.weight ties the head to the
 * embedding (model.rs:230-233). */
int tmg_load_safetensors(tmg_ctx* ctx, const char* path);
/* Upload every tensor of a TMB1 file (load_model_tmb, src/model.rs:108-179)
 * straight from its mapping: BF16 matrices bits unchanged, f32 norms, and the
 * f32 embedding back to its BF16 bits (a value that is not a widened BF16 is
 * refused with TMG_ERR_INVALID).  The file's model shape must equal the
 * context's (create the context from tmg_tmb_count's config).  A missing
 * lm_head.weight ties the head to the embedding. */
int tmg_load_tmb(tmg_ctx* ctx, const char* path);
/* Upload one tensor by its HF name from host memory (a WMat, src/tensor.rs:
 * 198-206, and the f32 vectors of src/model.rs:27-28).  dtype: 0 F32, 1 BF16.
 * Matrices must be BF16; vectors may be F32 or BF16. */
int tmg_set_tensor(tmg_ctx* ctx, const char* name, int32_t dtype, const void* host,
                   int64_t numel);
/* Check that every tensor is present; ties lm_head when absent. */
int tmg_finalize(tmg_ctx* ctx);
/* Bytes of weights resident in HBM on this context (this rank's shard). */
int64_t tmg_weight_bytes(const tmg_ctx* ctx);

/* ---------------------------------------------------------------------------
 * KV cache (KvCache, src/model.rs:250-332).  Per layer and stream an f32
 * [capacity, n_kv*head_dim] buffer in HBM, the reference's flat
 * [pos, kv_dim] row layout, preallocated instead of grown.
 * ------------------------------------------------------------------------ */

int tmg_kv_create(tmg_ctx* ctx, int32_t n_streams, int64_t capacity, tmg_kv** out);
int tmg_kv_destroy(tmg_kv* kv);
/* KvCache::len(layer) for one stream (src/model.rs:283-285). */
int tmg_kv_len(const tmg_kv* kv, int32_t layer, int32_t stream, int64_t* out);
/* KvCache::reset, src/model.rs:325-331 (all streams). */
int tmg_kv_reset(tmg_kv* kv);
/* Keep only the first len positions of one stream (len <= its length); the
 * next forward appends at len.  No counterpart in the reference, whose cache
 * only grows or resets: it lets a server reuse a prefilled prompt. */
int tmg_kv_truncate(tmg_kv* kv, int32_t stream, int64_t len);
/* keys_flat / values_flat, src/model.rs:310-317: copy [len, kv_dim] rows of
 * one layer and stream to host buffers (either may be NULL). */
int tmg_kv_read(tmg_kv* kv, int32_t layer, int32_t stream, float* keys, float* values);

/* ---------------------------------------------------------------------------
 * Forward passes.
 * ------------------------------------------------------------------------ */

/* Model::forward_token, src/model.rs:392-491, for all n_streams of `kv` at
 * once: tokens[n_streams] in, logits[n_streams * vocab] out (NULL: keep them
 * on the device).  Appends one position per stream. */
int tmg_forward_token(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* tokens, float* logits);
/* Model::forward_seq / prefill, src/model.rs:494-590, for one stream: T
 * tokens appended from the stream's current position; logits of the last
 * token out (NULL: keep on the device).  T == 0 is an error (prefill bails
 * on an empty prompt, model.rs:495-497). */
int tmg_forward_seq(tmg_ctx* ctx, tmg_kv* kv, int32_t stream, const uint32_t* tokens, int64_t T,
                    float* logits);
/* generate, src/model.rs:614-663, for stream 0 of `kv` (reset first):
 * prefill, then up to max_tokens steps of penalty -> argmax/sample -> EOS
 * check -> forward_token, all on the device.  tokens_out[max_tokens];
 * *n_out = tokens produced; first_logits (vocab floats, may be NULL) =
 * GenOutput::logits_first_step; *prefill_secs may be NULL.  `uniforms`
 * (max_tokens floats, may be NULL) supplies each sampled step's draw; when
 * NULL the library's restatement of the reference's StdRng(seed) does. */
int tmg_generate(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* prompt, int64_t T,
                 const tmg_gen_params* params, const float* uniforms, uint32_t* tokens_out,
                 int64_t* n_out, float* first_logits, double* prefill_secs, tmg_token_cb cb,
                 void* user);
/* generate over all n_streams of `kv` at once (weights read once per step
 * for every stream; no counterpart in the reference, which runs one stream):
 * prompts[n_streams * T]; params[n_streams] (the same temperature/top-k/top-p/
 * penalty/max_tokens for all; the seeds differ); uniforms (may be NULL)
 * [n_streams * max_tokens]; tokens_out[n_streams * max_tokens];
 * n_out[n_streams]. */
int tmg_generate_batch(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* prompts, int64_t T,
                       const tmg_gen_params* params, const float* uniforms,
                       uint32_t* tokens_out, int64_t* n_out);

/* The reference's StdRng draws (rand 0.10.2 StdRng::seed_from_u64(seed),
 * StandardUniform f32), n values: the `r` of src/tensor.rs:1204. */
int tmg_rng_uniforms(uint64_t seed, int64_t n, float* out);

/* The greedy step of generate's loop (src/model.rs:636-655) repeated
 * n_steps times for every stream of kv, with no host round trip: step i runs
 * forward_token(t_i) and takes t_{i+1} = argmax of its logits; t_0 =
 * tokens[m].  out[m * n_steps + i] = t_{i+1} (NULL: do not wait; the work is
 * queued on the context's stream -- see tmg_sync).  No EOS check: exactly
 * n_steps positions are appended per stream. */
int tmg_decode(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* tokens, int64_t n_steps, uint32_t* out);
/* Wait for all work queued on the context. */
int tmg_sync(tmg_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t), for timing with CUDA events. */
void* tmg_stream(tmg_ctx* ctx);
/* Profiling aid: the same greedy steps as tmg_decode, launched one kernel at
 * a time with CUDA events around each kernel (so without the overlap of the
 * captured graph).  ms[8] / launches[8] receive the summed device time and
 * the launch count of: 0 qkv GEMV, 1 attention, 2 o GEMV, 3 gate/up GEMV,
 * 4 down GEMV, 5 LM head, 6 allreduce + residual add and 7 logits
 * allgather + end of step (6 and 7 under tensor parallelism only). */
int tmg_profile_decode(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* tokens, int64_t n_steps,
                       double* ms, int64_t* launches);
/* Profiling aid: the device timeline of one captured greedy step (the real
 * graph, with its launch overlap), from %globaltimer stamps.  For each
 * kernel i of the step (n_slots of them, at most max_slots): out[4i..4i+3] =
 * first CTA start, first CTA past griddepcontrol.wait, last CTA past it, last
 * CTA end (ns); kinds[i] = 0 qkv GEMV, 1 attention, 2 o GEMV, 3 gate/up
 * GEMV, 4 down GEMV, 5 LM head.  Appends two positions per stream. */
int tmg_trace_decode(tmg_ctx* ctx, tmg_kv* kv, const uint32_t* tokens, uint64_t* out,
                     int32_t* kinds, int32_t max_slots, int32_t* n_slots);
/* Profiling aid for the fused single-stream decode kernel: one greedy step
 * with %globaltimer stamps (ns) and SM cycle counts.  out receives
 * n_ctas * (5 L + 1) records of 12 words per CTA and phase (per layer: qkv,
 * attention, o, gate/up, down; then the LM head).  GEMV phases: [0] entry,
 * [1] input ready, [2] / [3] the weight stream's first / last copy of the
 * phase issued, [4] cycles from the input loaded to the first stage ready,
 * [5] GEMV loop end, [6] first stage ready, [7] groups (stages) of the CTA,
 * [8] cycles loading the input into registers, [9] epilogue cycles (LM
 * head: rmsnorm cycles), [10] / [11] producer cycles waiting for a free
 * stage / issuing.  Attention phase (first item of the CTA): [0] entry,
 * [1] q/k/v gathered, [2] first tile loaded, [3] its P.V done, [5] items
 * done, [6] merges done, [8] outputs written, [9] after the item's closing
 * barrier.  max_u64 is the room in out; *n_ctas is set.  Appends one
 * position. */
int tmg_trace_fused(tmg_ctx* ctx, tmg_kv* kv, uint32_t token, uint64_t* out, int64_t max_u64,
                    int32_t* n_ctas);

/* ---------------------------------------------------------------------------
 * Tensor parallel (8B-class config, 2/4/8 GPUs of one node).  Call before
 * the weights are uploaded: each rank keeps its shard (q/k/v and gate/up
 * column-split by heads and rows, o/down row-split, lm_head split by vocab).
 * ------------------------------------------------------------------------ */
int tmg_tp_unique_id(uint8_t id[128]);
/* Greedy decode of one sequence spread over `world` GPUs of one node (2 to
 * 8, one process per GPU) by the fused decode kernel.  No counterpart in the
 * reference (tensor parallelism of the 8B config).  Every rank calls this
 * with its own context (created WITHOUT tmg_tp_init, holding the full
 * weights: the 8B model is 16 GB of a B200's 180 GB) and a 1-stream cache of
 * the same capacity, and the same `id` (tmg_tp_unique_id on rank 0).
 * Afterwards tmg_decode / tmg_generate (greedy) on that cache run the fused
 * kernel with its row groups and attention items dealt over the SMs of all
 * ranks, so each GPU streams 1/world of the weights per token; every
 * exchanged value, KV-cache row and argmax candidate is written into every
 * rank's memory over NVLink (peer stores), so each output row is computed
 * whole on one GPU and the tokens are bit-identical to one GPU's.  All ranks
 * must make the same decode calls (prefill runs on each rank alone).  The
 * group ends with the cache (tmg_kv_destroy on every rank).  Returns
 * TMG_ERR_INVALID for a shape the fused kernel does not take or with too
 * few row groups for `world`, or when two ranks share a GPU. */
int tmg_fused_group_init(tmg_ctx* ctx, tmg_kv* kv, const uint8_t id[128], int32_t rank,
                         int32_t world);
/* Host-only: the block of the full tensor `name` (HF name, e.g.
 * "model.layers.3.mlp.down_proj.weight") that rank `rank` of `world` keeps,
 * as out = {row0, rows, col0, cols} of its [out, in] layout (vectors:
 * [n, 1]).  q/k/v and gate/up are split by output rows (whole heads,
 * I / world rows), o and down by input columns, lm_head by vocabulary rows
 * (ceil(V / world) per rank); the embedding and norms are replicated.  This
 * is the split tmg_set_tensor / tmg_load_* apply after tmg_tp_init. */
int tmg_tp_shard(const tmg_config* cfg, const char* name, int32_t rank, int32_t world,
                 int64_t out[4]);
int tmg_tp_init(tmg_ctx* ctx, const uint8_t id[128], int32_t rank, int32_t world);

/* ---------------------------------------------------------------------------
 * Op-level entry points (device pointers; for parity tests and profiling).
 * Each mirrors one reference kernel.
 * ------------------------------------------------------------------------ */

/* matmul_w_into, src/tensor.rs:331-460, for M activation rows at once:
 * y[M, N] = x[M, K] . W[N, K]^T. */
int tmg_op_gemv_bf16(tmg_ctx* ctx, const float* x, const uint16_t* w, int64_t N, int64_t K,
                     int32_t M, float* y);
/* matmul_batch_w_into, src/tensor.rs:573-792 (the prefill GEMM on tcgen05
 * tensor cores): y[T, N] = x[T, K] . W[N, K]^T. */
int tmg_op_gemm_bf16(tmg_ctx* ctx, const float* x, const uint16_t* w, int64_t N, int64_t K,
                     int64_t T, float* y);
/* WMat handles (src/tensor.rs:198-206): a BF16 weight matrix [rows, cols]
 * (row-major, [out, in]) uploaded once to HBM and owned by the handle; the
 * host buffer (it may be the safetensors mapping) is not retained.  Free a
 * handle with tmg_wmat_free before destroying its context (tmg_destroy
 * releases any that are left, after which their pointers dangle). */
int tmg_wmat_upload_bf16(tmg_ctx* ctx, const uint16_t* host, int64_t rows, int64_t cols,
                         tmg_wmat** out);
int tmg_wmat_free(tmg_wmat* w);
int tmg_wmat_shape(const tmg_wmat* w, int64_t* rows, int64_t* cols);
/* matmul_w_into(x, &WMat, out, in, y), src/tensor.rs:331-460, over a handle:
 * y[M, rows] = x[M, cols] . W^T (device pointers, M <= 16). */
int tmg_op_gemv_wmat(tmg_ctx* ctx, const float* x, const tmg_wmat* w, int32_t M, float* y);
/* matmul_batch_w_into, src/tensor.rs:573-792, over a handle: y[T, rows] =
 * x[T, cols] . W^T on the tcgen05 prefill GEMM (device pointers). */
int tmg_op_gemm_wmat(tmg_ctx* ctx, const float* x, const tmg_wmat* w, int64_t T, float* y);
/* Int8 weights: the reference's TMG_I8=1 (wmat_maybe_i8, src/model.rs:
 * 57-76).  With TMG_I8=1 in the environment when a model's weights are
 * first set, its layer matrices (q/k/v/o, gate/up/down) are quantized at
 * upload and every forward runs the int8 path (the LM head and norms stay
 * BF16 / f32, as there); single GPU only (tmg_tp_init + TMG_I8=1 is
 * refused).  The two op entries below expose its kernels.
 * WMat::quantize_i8, src/tensor.rs:282-297, of a BF16 [N, K] matrix:
 * q[N, K] int8 and scales[N] (device pointers). */
int tmg_op_quantize_i8(tmg_ctx* ctx, const uint16_t* w, int64_t N, int64_t K, int8_t* q,
                       float* scales);
/* The I8 arm of matmul_w_into, src/tensor.rs:341-357, for M <= 16 rows:
 * each row of x[M, K] quantized (quantize_row_i8, src/tensor.rs:128-141),
 * integer dots with q[N, K] (dot_i8, 146-170), y[M, N] = f32(dot) * s_x *
 * scales[n].  K % 16 == 0, K <= 16384. */
int tmg_op_gemv_i8(tmg_ctx* ctx, const float* x, const int8_t* q, const float* scales, int64_t N,
                   int64_t K, int32_t M, float* y);
/* rms_norm_into (mode 0, src/tensor.rs:969-977) or rms_norm_batch (mode 1,
 * 946-954) over `rows` rows of n. */
int tmg_op_rmsnorm(tmg_ctx* ctx, const float* x, const float* w, float eps, int64_t n,
                   int64_t rows, int32_t mode, float* out);
/* Rope::rotate, src/tensor.rs:1026-1037, in place on rows of n_heads heads
 * of head_dim at positions pos0, pos0+1, ... (one row per position). */
int tmg_op_rope(tmg_ctx* ctx, float* x, int64_t rows, int32_t n_heads, int32_t head_dim,
                int64_t pos0, float theta);
/* SwiGLU, src/model.rs:473-475: out = gate / (1 + exp(-gate)) * up. */
int tmg_op_swiglu(tmg_ctx* ctx, const float* gate, const float* up, int64_t n, float* out);
/* Decode attention, src/model.rs:434-459: one query row of n_q heads over
 * n_ctx cached rows of [n_kv * head_dim] (keys already rotated).  head_dim
 * 16, 32, 64 or 128; at most 16 query heads per kv head; other shapes return
 * TMG_ERR_INVALID before anything is enqueued. */
int tmg_op_attn_decode(tmg_ctx* ctx, const float* q, const float* keys, const float* values,
                       int64_t n_ctx, int32_t n_q, int32_t n_kv, int32_t head_dim, float* out);
/* The same decode attention as tmg_op_attn_decode (same split count, same
 * results), for callers that may not allocate device memory at call time.
 * No counterpart in the reference.  It allocates nothing: partials,
 * tickets and the position word live in a 4 MiB static per-device scratch
 * (requests needing more return TMG_ERR_CAPACITY before enqueuing
 * anything).  It only enqueues on the context's stream (results are ready
 * after tmg_sync).  Shapes as tmg_op_attn_decode (others return
 * TMG_ERR_INVALID before anything is enqueued).  The first call on a device
 * sets the scratch up and should precede any stream capture.  Calls that
 * overlap on one device race on the shared scratch: order them. */
int tmg_op_attn_decode_noalloc(tmg_ctx* ctx, const float* q, const float* keys,
                               const float* values, int64_t n_ctx, int32_t n_q, int32_t n_kv,
                               int32_t head_dim, float* out);
/* attention_batch, src/tensor.rs:1099-1139: T causal query rows at
 * start_pos.. over [start_pos + T, n_kv * head_dim] cached rows. */
int tmg_op_attn_prefill(tmg_ctx* ctx, const float* q, const float* keys, const float* values,
                        int64_t T, int64_t start_pos, int32_t n_q, int32_t n_kv,
                        int32_t head_dim, float* out);
/* argmax, src/tensor.rs:1063-1073, per row of `rows` x V logits. */
int tmg_op_argmax(tmg_ctx* ctx, const float* logits, int64_t V, int32_t rows, uint32_t* out);
/* apply_repetition_penalty + sample, src/tensor.rs:1142-1213, per row:
 * logits[rows, V] (penalised in place), generated[rows, n_gen] ids,
 * uniforms[rows] draws; next[rows] out.  Also returns the candidate set of
 * each row when cand_ids/cand_probs are not NULL ([rows, top_k] each) and
 * the top-p cutoff in cutoff[rows] (may be NULL). */
int tmg_op_sample(tmg_ctx* ctx, float* logits, int64_t V, int32_t rows, const uint32_t* generated,
                  int64_t n_gen, float temperature, int64_t top_k, float top_p, float penalty,
                  const float* uniforms, uint32_t* next, uint32_t* cand_ids, float* cand_probs,
                  int32_t* cutoff);

#ifdef __cplusplus
}
#endif
#endif /* TMG_CUDA_H */
