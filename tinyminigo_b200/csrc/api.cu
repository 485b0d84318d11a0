// The token-loop engine behind the C ABI (include/tmg_cuda.h): Model
// (weights + scratch on one GPU), KvCache, forward_token, forward_seq and
// generate of src/model.rs, driving the kernels of this directory.
//
// Decode is one CUDA graph per step: 5 kernels per layer (qkv GEMV with the
// input RMSNorm fused in, attention with RoPE + KV append fused in, o GEMV +
// residual, gate/up GEMV with the post-attention RMSNorm and SwiGLU fused in,
// down GEMV + residual) and the LM head (final RMSNorm fused in; in greedy
// mode the argmax and generate's bookkeeping too), launched with
// programmatic dependent launch so each kernel's weight stream starts while
// the previous kernel drains.  generate runs its whole loop on the device;
// the host only launches graph replays and reads tokens back in chunks.
#include <dlfcn.h>
#include <math.h>

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "../../include/tmg_cuda.h"
#include "common.cuh"
#include "kernels.cuh"
#include "loader.h"
#include "tp.h"
#include "fused.cuh"

using namespace tmg;

namespace {

struct Layer {
  uint16_t* wqkv = nullptr;  // [(nq + 2 nkv) d, h]: q rows, then k, then v
  uint16_t* wo = nullptr;    // [h, nq d]
  uint16_t* wg = nullptr;    // [I, h]
  uint16_t* wu = nullptr;    // [I, h]
  uint16_t* wd = nullptr;    // [h, I]
  // int8 weights (TMG_I8=1): the same matrices quantized per row, and
  // their row scales (the BF16 pointers above are then null)
  int8_t *qqkv = nullptr, *qo = nullptr, *qg = nullptr, *qu = nullptr, *qd = nullptr;
  float *sqkv = nullptr, *so = nullptr, *sg = nullptr, *su = nullptr, *sd = nullptr;
  float* in_norm = nullptr;
  float* post_norm = nullptr;
  unsigned have = 0;  // bit per tensor
};

constexpr unsigned kHaveQ = 1, kHaveK = 2, kHaveV = 4, kHaveO = 8, kHaveG = 16, kHaveU = 32,
                   kHaveD = 64, kHaveIn = 128, kHavePost = 256, kHaveAll = 511;

}  // namespace

struct tmg_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  bool has_model = false;
  bool finalized = false;
  // TMG_DEBUG set when the context was created (src/model.rs:406): the
  // per-token forward prints the first 8 values of the embedding and of
  // each layer's residual stream after attention and after the MLP
  bool debug = false;
  tmg_config cfg{};
  // tensor parallel
  int rank = 0, world = 1;
  TpComm* tp = nullptr;
  // dims (local shard)
  int h = 0, d = 0, L = 0, nq = 0, nkv = 0, I = 0, V = 0;
  int nq_g = 0, nkv_g = 0, I_g = 0;  // global
  int64_t V_l = 0, v_off = 0;         // vocab shard of the LM head
  int qkv_rows = 0;
  // weights
  std::vector<Layer> layers;
  uint16_t* embed = nullptr;  // [V, h], replicated
  uint16_t* lm_head = nullptr;  // [V_l, h]
  float* final_norm = nullptr;
  bool lm_tied = true;
  int64_t weight_bytes = 0;
  std::vector<void*> allocs;
  // decode scratch (kMaxStreams rows)
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr,
        *logits = nullptr, *partial = nullptr;
  unsigned long long *am_part = nullptr, *sm_part = nullptr;
  unsigned int* tickets = nullptr;  // [0]: head, [1..16]: sampler
  int32_t* d_err = nullptr;
  float* logits_full = nullptr;  // [M, V] gathered logits under TP
  unsigned int* bar = nullptr;   // grid barrier of the fused decode kernel
  unsigned long long* ll = nullptr;  // its tagged exchange words (x, att, act, qkv)
  int fused_pf = 0;              // its stall-time L2 prefetch distance (stages; TMG_FUSED_PF)
  int fused_pf_pace = 0;         // cycles between those prefetches (TMG_FUSED_PF_PACE)
  int fused_pf_mode = 0;         // when: 0 attention chain only, 1 ring full (TMG_FUSED_PF_MODE)
  int fused_rep = 4;             // copies of its x/att/act exchange words (TMG_FUSED_REP)
  bool fused_rep_set = false;    // TMG_FUSED_REP given (else a group of GPUs uses one copy)
  int fused_stages = 4;          // its ring depth cap (0: all that fit; TMG_FUSED_STAGES)
  bool fused_ok = false;         // the fused batch-1 decode kernel takes this shape
  // int8 layer weights (the reference's TMG_I8=1, read when the weights are
  // allocated): BF16 staging for the load-time quantization, the quantized
  // activation rows of the multi-stream GEMV, and the prefill's widened
  // weights and accumulator
  bool i8 = false;
  uint16_t* i8_stage = nullptr;
  int8_t* xq8 = nullptr;
  float* xs8 = nullptr;
  uint16_t* dq = nullptr;
  size_t dq_cap = 0;
  float* i8acc = nullptr;
  // failure-path test of the fused kernel (TMG_TEST_FUSED_STALL=<phase>,
  // TMG_TEST_FUSED_POLL_MS=<ms>): the context's next fused launch waits in
  // that phase for a tag nobody writes, with polls limited to that many ms
  int test_stall = -1;
  int test_poll_ms = 50;
  // prefill scratch
  int64_t pf_cap = 0;
  float *X = nullptr, *Xn = nullptr, *QKV = nullptr, *ATT = nullptr, *G = nullptr, *U = nullptr;
  uint32_t* d_tok = nullptr;
  // op-level scratch
  void* op_buf = nullptr;
  size_t op_cap = 0;
  // hi/lo BF16 split of the prefill GEMM's activations
  uint16_t *sp_hi = nullptr, *sp_lo = nullptr;
  size_t sp_cap = 0;
  // hi/lo parts of the SwiGLU output written by the gate/up GEMM's epilogue
  uint16_t *sa_hi = nullptr, *sa_lo = nullptr;
  size_t sa_cap = 0;
  // BF16 parts of q, k and v^T for the tensor-core prefill attention
  void* pfa = nullptr;
  size_t pfa_cap = 0;
  // pinned staging
  void* pinned = nullptr;
  size_t pinned_cap = 0;
  // WMat handles and KV caches still alive: tmg_destroy releases their
  // device memory and detaches them (the handles then only accept their
  // own destroy call, in any order relative to the context's)
  std::vector<tmg_wmat*> wmats;
  std::vector<tmg_kv*> kvs;
  std::string err;
};

// One fused decode spread over several GPUs (tmg_fused_group_init): every
// rank's exchange buffers, argmax table, barrier words and KV caches mapped
// into this process (CUDA IPC), and the communicator whose collectives
// separate the launches (no rank zeroes its buffers while another still
// writes into them, none starts before all have zeroed).
struct FusedGroup {
  TpComm* comm = nullptr;
  int rank = 0, world = 1, ctas = 0;
  unsigned long long* ll_peer[tmg::kMaxGroupRanks] = {};
  unsigned long long* part_peer[tmg::kMaxGroupRanks] = {};
  unsigned int* bar_peer[tmg::kMaxGroupRanks] = {};
  unsigned long long* am_peer[tmg::kMaxGroupRanks] = {};
  float** d_kv_peer = nullptr;         // [world][L][2] on the device
  unsigned long long* am = nullptr;    // this rank's argmax table [world * ctas]
  float* sync = nullptr;               // the barriers' one float
  std::vector<void*> opened;           // peer mappings to close
};

// A device weight matrix handle (WMat, src/tensor.rs:198-206): row-major
// [rows, cols] BF16 bits in HBM, owned by the handle.
struct tmg_wmat {
  tmg_ctx* ctx = nullptr;
  int64_t rows = 0, cols = 0;
  uint16_t* w = nullptr;
};

struct tmg_kv {
  tmg_ctx* ctx = nullptr;
  int M = 1;
  int64_t cap = 0;
  int kvd = 0;
  std::vector<float*> k, v;  // per layer [M, cap, kvd]
  float *rope_cos = nullptr, *rope_sin = nullptr;
  int32_t* d_state = nullptr;  // token | pos | done | n_gen, kMaxStreams each
  StreamState st{};
  uint32_t* d_gen = nullptr;
  int64_t gen_alloc = 0;
  float* d_uni = nullptr;
  int64_t uni_alloc = 0;
  float* part = nullptr;
  unsigned int* att_ticket = nullptr;
  int nsplit = 1;
  std::vector<int64_t> lens;
  cudaGraphExec_t g_plain = nullptr;
  cudaGraphExec_t g_dec = nullptr;  // forward + argmax with gen_cap = dec_cap
  int64_t dec_cap = 0;
  int32_t* h_state = nullptr;  // pinned staging of the state block
  FusedLayer* d_layers = nullptr;  // per-layer pointers for the fused kernel (stream 0)
  unsigned long long* part_ll = nullptr;  // its tagged attention partials
  int nsplit_f = 1;                       // their split capacity per kv head
  cudaEvent_t state_ev = nullptr;  // the last upload from h_state
  FusedGroup* grp = nullptr;       // set by tmg_fused_group_init
  std::vector<void*> allocs;
};

namespace {

constexpr int64_t kPrefillChunk = 4096;

// Why the last tmg_create on this thread failed (there is no context to hold it).
thread_local std::string g_create_err;

int fail(tmg_ctx* c, int code, const std::string& m) {
  if (c) c->err = m;
  return code;
}
int cuda_fail(tmg_ctx* c, cudaError_t e, const char* where) {
  return fail(c, TMG_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}
#define CK(expr, where)                               \
  do {                                                \
    cudaError_t _e = (expr);                          \
    if (_e != cudaSuccess) return cuda_fail(c, _e, where); \
  } while (0)

template <typename T>
cudaError_t dalloc(std::vector<void*>& list, T** p, size_t count) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T));
  if (e != cudaSuccess) return e;
  list.push_back(q);
  *p = static_cast<T*>(q);
  return cudaSuccess;
}

void free_all(std::vector<void*>& list) {
  for (void* p : list) cudaFree(p);
  list.clear();
}

cudaError_t ensure_pinned(tmg_ctx* c, size_t bytes) {
  if (c->pinned_cap >= bytes) return cudaSuccess;
  if (c->pinned) cudaFreeHost(c->pinned);
  c->pinned = nullptr;
  c->pinned_cap = 0;
  size_t want = std::max<size_t>(bytes, 1 << 20);
  TMG_CUDA_TRY(cudaHostAlloc(&c->pinned, want, cudaHostAllocDefault));
  c->pinned_cap = want;
  return cudaSuccess;
}

// Every copy and fill is ordered on the context's (non-blocking) stream:
// legacy-stream cudaMemcpy / cudaMemset do not order against it, and a
// pageable host-to-device cudaMemcpy may return before its DMA lands.
cudaError_t copy_sync(tmg_ctx* c, void* dst, const void* src, size_t n, cudaMemcpyKind k) {
  TMG_CUDA_TRY(cudaMemcpyAsync(dst, src, n, k, c->stream));
  return cudaStreamSynchronize(c->stream);
}

cudaError_t zero_sync(tmg_ctx* c, void* p, size_t n) {
  TMG_CUDA_TRY(cudaMemsetAsync(p, 0, n, c->stream));
  return cudaStreamSynchronize(c->stream);
}

// The device error word: 1 = NaN logits reached the sampler, 2 = a bounded
// device-side wait gave up.
int err_status(tmg_ctx* c, int32_t w) {
  if (w == 1) return fail(c, TMG_ERR_NAN, "NaN logits reached the sampler");
  return fail(c, TMG_ERR_TIMEOUT, "a bounded device-side wait gave up (pipeline stalled)");
}

// Wait for the stream, then read and clear the device error word.
int sync_check(tmg_ctx* c, const char* where) {
  int32_t w = 0;
  cudaError_t e = copy_sync(c, &w, c->d_err, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(c, e, where);
  if (w) {
    e = zero_sync(c, c->d_err, 4);
    // a fused launch that gave up may have left its grid barrier mid-way
    if (e == cudaSuccess && c->bar) e = zero_sync(c, c->bar, fused_bar_words() * sizeof(unsigned int));
    if (e != cudaSuccess) return cuda_fail(c, e, where);
    return err_status(c, w);
  }
  return TMG_OK;
}

cudaError_t ensure_op(tmg_ctx* c, size_t bytes) {
  if (c->op_cap >= bytes) return cudaSuccess;
  TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (c->op_buf) cudaFree(c->op_buf);
  c->op_buf = nullptr;
  c->op_cap = 0;
  TMG_CUDA_TRY(cudaMalloc(&c->op_buf, bytes));
  TMG_CUDA_TRY(zero_sync(c, c->op_buf, bytes));
  c->op_cap = bytes;
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// Weight placement (with the tensor-parallel shard of this rank).
// ---------------------------------------------------------------------------
int check_shape(tmg_ctx* c, const std::string& name, int64_t numel, int64_t want) {
  if (numel != want)
    return fail(c, TMG_ERR_INVALID,
                "tensor " + name + ": " + std::to_string(numel) + " elements, expected " +
                    std::to_string(want));
  return TMG_OK;
}

// Copy rows [r0, r0 + nr) x cols [c0, c0 + nc) of a host [R, C] bf16 matrix
// into a device [nr, nc] matrix at dst.
int upload_block(tmg_ctx* c, uint16_t* dst, const uint16_t* src, int64_t C, int64_t r0,
                 int64_t nr, int64_t c0, int64_t nc) {
  CK(cudaMemcpy2DAsync(dst, size_t(nc) * 2, src + r0 * C + c0, size_t(C) * 2, size_t(nc) * 2,
                       size_t(nr), cudaMemcpyHostToDevice, c->stream),
     "upload");
  return TMG_OK;
}

int upload_vec(tmg_ctx* c, float* dst, int32_t dtype, const void* host, int64_t n) {
  std::vector<float> tmp(n);
  if (dtype == 0) std::memcpy(tmp.data(), host, n * 4);
  else if (dtype == 1)
    for (int64_t i = 0; i < n; ++i) {
      uint32_t u = uint32_t(static_cast<const uint16_t*>(host)[i]) << 16;
      std::memcpy(&tmp[i], &u, 4);
    }
  else
    for (int64_t i = 0; i < n; ++i) tmp[i] = f16_to_f32(static_cast<const uint16_t*>(host)[i]);
  CK(cudaMemcpyAsync(dst, tmp.data(), n * 4, cudaMemcpyHostToDevice, c->stream), "upload");
  CK(cudaStreamSynchronize(c->stream), "upload");
  return TMG_OK;
}

// The tensor-parallel split: the block of the full tensor `name` (HF name)
// that `rank` of `world` keeps, as rows [r0, r0 + nr) x columns
// [c0, c0 + nc) of its [rows, cols] layout (vectors are [n, 1]).  q/k/v and
// gate/up are split by output rows (whole heads, I / world rows), o and down
// by input columns, the LM head by vocabulary rows (ceil(V / world) per
// rank, the last rank keeps the rest); the embedding and the norm vectors
// are replicated.  With world 1 every block is the whole tensor.
// full = {rows, cols} of the whole tensor.  False for an unknown name.
bool tp_shard_rect(const tmg_config& f, const std::string& name, int rank, int world,
                   int64_t rect[4], int64_t full[2]) {
  const int64_t h = f.hidden_size, d = f.head_dim, V = f.vocab_size;
  const int64_t qg = int64_t(f.num_attention_heads) * d, kg = int64_t(f.num_key_value_heads) * d;
  const int64_t Ig = f.intermediate_size;
  const int64_t ql = qg / world, kl = kg / world, Il = Ig / world;
  auto set = [&](int64_t R, int64_t C, int64_t r0, int64_t nr, int64_t c0, int64_t nc) {
    full[0] = R;
    full[1] = C;
    rect[0] = r0;
    rect[1] = nr;
    rect[2] = c0;
    rect[3] = nc;
    return true;
  };
  if (name == "model.embed_tokens.weight") return set(V, h, 0, V, 0, h);
  if (name == "model.norm.weight") return set(h, 1, 0, h, 0, 1);
  if (name == "lm_head.weight") {
    const int64_t vl = (V + world - 1) / world, v0 = int64_t(rank) * vl;
    return set(V, h, v0, std::max<int64_t>(0, std::min<int64_t>(vl, V - v0)), 0, h);
  }
  const std::string pre = "model.layers.";
  if (name.compare(0, pre.size(), pre) != 0) return false;
  const size_t dot = name.find('.', pre.size());
  if (dot == std::string::npos) return false;
  const std::string suf = name.substr(dot + 1);
  if (suf == "self_attn.q_proj.weight") return set(qg, h, rank * ql, ql, 0, h);
  if (suf == "self_attn.k_proj.weight" || suf == "self_attn.v_proj.weight")
    return set(kg, h, rank * kl, kl, 0, h);
  if (suf == "self_attn.o_proj.weight") return set(h, qg, 0, h, rank * ql, ql);
  if (suf == "mlp.gate_proj.weight" || suf == "mlp.up_proj.weight")
    return set(Ig, h, rank * Il, Il, 0, h);
  if (suf == "mlp.down_proj.weight") return set(h, Ig, 0, h, rank * Il, Il);
  if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight")
    return set(h, 1, 0, h, 0, 1);
  return false;
}

// Upload this rank's block of a full host matrix (tp_shard_rect) to dst.
int upload_shard(tmg_ctx* c, const std::string& name, uint16_t* dst, const void* host,
                 int64_t numel) {
  int64_t r[4], full[2];
  if (!tp_shard_rect(c->cfg, name, c->rank, c->world, r, full))
    return fail(c, TMG_ERR_INVALID, "unknown tensor " + name);
  int rc = check_shape(c, name, numel, full[0] * full[1]);
  if (rc) return rc;
  return upload_block(c, dst, static_cast<const uint16_t*>(host), full[1], r[0], r[1], r[2], r[3]);
}

// The same through the BF16 staging buffer, quantized on the device into
// int8 rows at q with their scales (wmat_maybe_i8, src/model.rs:57-76).
// Stream order keeps the staging buffer's next upload behind this
// quantization.
int upload_shard_i8(tmg_ctx* c, const std::string& name, int8_t* q, float* scales,
                    const void* host, int64_t numel) {
  int64_t r[4], full[2];
  if (!tp_shard_rect(c->cfg, name, c->rank, c->world, r, full))
    return fail(c, TMG_ERR_INVALID, "unknown tensor " + name);
  int rc = upload_shard(c, name, c->i8_stage, host, numel);
  if (rc) return rc;
  CK(launch_quantize_w_i8(c->i8_stage, r[1], int(r[3]), q, scales, c->stream), "quantize");
  return TMG_OK;
}

int set_tensor(tmg_ctx* c, const std::string& name, int32_t dtype, const void* host,
               int64_t numel) {
  if (!c->has_model) return fail(c, TMG_ERR_INVALID, "context has no model config");
  if (c->finalized) return fail(c, TMG_ERR_INVALID, "weights already finalized");
  const int64_t h = c->h, d = c->d;
  const bool is_vec = name == "model.norm.weight" || name.find("layernorm.weight") != std::string::npos;
  if (!is_vec && dtype != 1)
    return fail(c, TMG_ERR_INVALID, "tensor " + name + ": the device path needs BF16 matrices");
  int rc;
  if (name == "model.embed_tokens.weight") {
    if ((rc = check_shape(c, name, numel, int64_t(c->V) * h))) return rc;
    CK(cudaMemcpyAsync(c->embed, host, size_t(numel) * 2, cudaMemcpyHostToDevice, c->stream),
       "upload");
    return TMG_OK;
  }
  if (name == "model.norm.weight") {
    if ((rc = check_shape(c, name, numel, h))) return rc;
    return upload_vec(c, c->final_norm, dtype, host, numel);
  }
  if (name == "lm_head.weight") {
    if ((rc = check_shape(c, name, numel, int64_t(c->V) * h))) return rc;
    if (c->lm_tied) {
      CK(dalloc(c->allocs, &c->lm_head, size_t(c->V_l) * h), "alloc");
      c->weight_bytes += c->V_l * h * 2;
      c->lm_tied = false;
    }
    return upload_shard(c, name, c->lm_head, host, numel);
  }
  const std::string pre = "model.layers.";
  if (name.compare(0, pre.size(), pre) != 0)
    return fail(c, TMG_ERR_INVALID, "unknown tensor " + name);
  size_t dot = name.find('.', pre.size());
  if (dot == std::string::npos) return fail(c, TMG_ERR_INVALID, "unknown tensor " + name);
  const int li = std::atoi(name.substr(pre.size(), dot - pre.size()).c_str());
  if (li < 0 || li >= c->L) return fail(c, TMG_ERR_INVALID, "layer out of range: " + name);
  const std::string suf = name.substr(dot + 1);
  Layer& Lw = c->layers[li];
  const int64_t ql = int64_t(c->nq) * d, kl = int64_t(c->nkv) * d;
  const bool q8 = c->i8;
  if (suf == "self_attn.q_proj.weight") {
    Lw.have |= kHaveQ;
    return q8 ? upload_shard_i8(c, name, Lw.qqkv, Lw.sqkv, host, numel)
              : upload_shard(c, name, Lw.wqkv, host, numel);
  }
  if (suf == "self_attn.k_proj.weight") {
    Lw.have |= kHaveK;
    return q8 ? upload_shard_i8(c, name, Lw.qqkv + ql * h, Lw.sqkv + ql, host, numel)
              : upload_shard(c, name, Lw.wqkv + ql * h, host, numel);
  }
  if (suf == "self_attn.v_proj.weight") {
    Lw.have |= kHaveV;
    return q8 ? upload_shard_i8(c, name, Lw.qqkv + (ql + kl) * h, Lw.sqkv + ql + kl, host, numel)
              : upload_shard(c, name, Lw.wqkv + (ql + kl) * h, host, numel);
  }
  if (suf == "self_attn.o_proj.weight") {
    Lw.have |= kHaveO;
    return q8 ? upload_shard_i8(c, name, Lw.qo, Lw.so, host, numel)
              : upload_shard(c, name, Lw.wo, host, numel);
  }
  if (suf == "mlp.gate_proj.weight" || suf == "mlp.up_proj.weight") {
    const bool gate = suf[4] == 'g';
    Lw.have |= gate ? kHaveG : kHaveU;
    if (q8)
      return upload_shard_i8(c, name, gate ? Lw.qg : Lw.qu, gate ? Lw.sg : Lw.su, host, numel);
    return upload_shard(c, name, gate ? Lw.wg : Lw.wu, host, numel);
  }
  if (suf == "mlp.down_proj.weight") {
    Lw.have |= kHaveD;
    return q8 ? upload_shard_i8(c, name, Lw.qd, Lw.sd, host, numel)
              : upload_shard(c, name, Lw.wd, host, numel);
  }
  if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight") {
    if ((rc = check_shape(c, name, numel, h))) return rc;
    const bool in = suf[0] == 'i';
    Lw.have |= in ? kHaveIn : kHavePost;
    return upload_vec(c, in ? Lw.in_norm : Lw.post_norm, dtype, host, numel);
  }
  return fail(c, TMG_ERR_INVALID, "unknown tensor " + name);
}

int alloc_model(tmg_ctx* c) {
  const tmg_config& f = c->cfg;
  if (f.hidden_size <= 0 || f.num_hidden_layers <= 0 || f.num_attention_heads <= 0 ||
      f.num_key_value_heads <= 0 || f.head_dim <= 0 || f.intermediate_size <= 0 ||
      f.vocab_size <= 0 || f.head_dim % 2 != 0 ||
      f.num_attention_heads % f.num_key_value_heads != 0)
    return fail(c, TMG_ERR_INVALID, "invalid model config");
  if (f.num_key_value_heads % c->world != 0 || f.intermediate_size % c->world != 0 ||
      f.num_attention_heads % c->world != 0)
    return fail(c, TMG_ERR_INVALID, "heads / intermediate size do not divide by the TP world");
  c->h = f.hidden_size;
  c->d = f.head_dim;
  c->L = f.num_hidden_layers;
  c->nq_g = f.num_attention_heads;
  c->nkv_g = f.num_key_value_heads;
  c->I_g = f.intermediate_size;
  c->V = f.vocab_size;
  c->nq = c->nq_g / c->world;
  c->nkv = c->nkv_g / c->world;
  c->I = c->I_g / c->world;
  c->V_l = (int64_t(c->V) + c->world - 1) / c->world;
  c->v_off = int64_t(c->rank) * c->V_l;
  c->V_l = std::min<int64_t>(c->V_l, int64_t(c->V) - c->v_off);
  c->qkv_rows = (c->nq + 2 * c->nkv) * c->d;
  const int64_t h = c->h;
  if (const char* e8 = getenv("TMG_I8")) c->i8 = std::strcmp(e8, "1") == 0;
  if (c->i8 && c->world > 1)
    return fail(c, TMG_ERR_INVALID, "int8 weights (TMG_I8=1) with tensor parallelism are not supported");
  if (c->i8 && (h % 16 || (int64_t(c->nq) * c->d) % 16 || c->I % 16))
    return fail(c, TMG_ERR_INVALID, "int8 weights need hidden, n_q * head_dim and intermediate % 16 == 0");
  c->layers.assign(c->L, Layer());
  const int64_t qd = int64_t(c->nq) * c->d;
  for (auto& Lw : c->layers) {
    if (c->i8) {
      CK(dalloc(c->allocs, &Lw.qqkv, size_t(c->qkv_rows) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.qo, size_t(h) * qd), "alloc weights");
      CK(dalloc(c->allocs, &Lw.qg, size_t(c->I) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.qu, size_t(c->I) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.qd, size_t(h) * c->I), "alloc weights");
      CK(dalloc(c->allocs, &Lw.sqkv, size_t(c->qkv_rows)), "alloc weights");
      CK(dalloc(c->allocs, &Lw.so, size_t(h)), "alloc weights");
      CK(dalloc(c->allocs, &Lw.sg, size_t(c->I)), "alloc weights");
      CK(dalloc(c->allocs, &Lw.su, size_t(c->I)), "alloc weights");
      CK(dalloc(c->allocs, &Lw.sd, size_t(h)), "alloc weights");
      c->weight_bytes += (int64_t(c->qkv_rows) * h + h * qd + 3 * int64_t(c->I) * h) +
                         4 * (int64_t(c->qkv_rows) + 2 * h + 2 * int64_t(c->I));
    } else {
      CK(dalloc(c->allocs, &Lw.wqkv, size_t(c->qkv_rows) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.wo, size_t(h) * qd), "alloc weights");
      CK(dalloc(c->allocs, &Lw.wg, size_t(c->I) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.wu, size_t(c->I) * h), "alloc weights");
      CK(dalloc(c->allocs, &Lw.wd, size_t(h) * c->I), "alloc weights");
      c->weight_bytes += 2 * (int64_t(c->qkv_rows) * h + h * qd + 3 * int64_t(c->I) * h);
    }
    CK(dalloc(c->allocs, &Lw.in_norm, size_t(h)), "alloc weights");
    CK(dalloc(c->allocs, &Lw.post_norm, size_t(h)), "alloc weights");
  }
  if (c->i8) {
    // staging of one BF16 matrix (the largest of a layer) for quantization
    const size_t most = std::max<size_t>({size_t(c->qkv_rows) * h, size_t(h) * qd, size_t(c->I) * h});
    CK(dalloc(c->allocs, &c->i8_stage, most), "alloc staging");
    const int64_t kmax = std::max<int64_t>({h, qd, int64_t(c->I)});
    CK(dalloc(c->allocs, &c->xq8, size_t(kMaxStreams) * kmax), "alloc scratch");
    CK(dalloc(c->allocs, &c->xs8, size_t(kMaxStreams)), "alloc scratch");
  }
  CK(dalloc(c->allocs, &c->embed, size_t(c->V) * h), "alloc weights");
  CK(dalloc(c->allocs, &c->final_norm, size_t(h)), "alloc weights");
  c->weight_bytes += int64_t(c->V) * h * 2;
  c->lm_tied = true;
  c->lm_head = c->embed + c->v_off * h;
  // decode scratch
  const int M = kMaxStreams;
  CK(dalloc(c->allocs, &c->x, size_t(M) * h), "alloc scratch");
  CK(dalloc(c->allocs, &c->xn, size_t(M) * h), "alloc scratch");
  CK(dalloc(c->allocs, &c->partial, size_t(M) * h), "alloc scratch");
  CK(dalloc(c->allocs, &c->qkv, size_t(M) * c->qkv_rows), "alloc scratch");
  CK(dalloc(c->allocs, &c->attn, size_t(M) * c->nq * c->d), "alloc scratch");
  CK(dalloc(c->allocs, &c->act, size_t(M) * c->I), "alloc scratch");
  CK(dalloc(c->allocs, &c->logits, size_t(M) * c->V_l), "alloc scratch");
  if (c->world > 1) CK(dalloc(c->allocs, &c->logits_full, size_t(M) * c->V), "alloc scratch");
  CK(dalloc(c->allocs, &c->am_part, size_t(M) * c->num_sms * 8), "alloc scratch");
  CK(dalloc(c->allocs, &c->sm_part, size_t(M) * 64 * kMaxTopK), "alloc scratch");
  CK(dalloc(c->allocs, &c->tickets, 64), "alloc scratch");
  CK(zero_sync(c, c->tickets, 64 * sizeof(unsigned int)), "memset");
  if (const char* rp = getenv("TMG_FUSED_REP")) {
    c->fused_rep = std::max(1, std::min(16, atoi(rp)));
    c->fused_rep_set = true;
  }
  CK(dalloc(c->allocs, &c->ll, fused_ll_words(h, c->nq * c->d, c->I, c->qkv_rows, c->fused_rep)),
     "alloc scratch");
  CK(dalloc(c->allocs, &c->bar, fused_bar_words()), "alloc scratch");
  CK(zero_sync(c, c->bar, fused_bar_words() * sizeof(unsigned int)), "memset");
  c->fused_ok = c->world == 1 && !c->i8 &&
                fused_supported(c->h, c->nq, c->nkv, c->d, c->I, c->V_l, c->num_sms);
  if (const char* pf = getenv("TMG_FUSED_PF")) c->fused_pf = atoi(pf);
  if (const char* pp = getenv("TMG_FUSED_PF_PACE")) c->fused_pf_pace = atoi(pp);
  if (const char* pm = getenv("TMG_FUSED_PF_MODE")) c->fused_pf_mode = atoi(pm);
  if (const char* ns = getenv("TMG_FUSED_STAGES")) c->fused_stages = atoi(ns);
  if (const char* ts = getenv("TMG_TEST_FUSED_STALL")) {
    // only a GEMV phase that gathers its input: O, GU, DOWN (p % 5 = 2, 3,
    // 4), a later layer's QKV or the LM head (p % 5 = 0, p > 0)
    const int p = atoi(ts);
    if (p > 0 && p <= 5 * c->L && p % 5 != 1) c->test_stall = p;
  }
  if (const char* tm = getenv("TMG_TEST_FUSED_POLL_MS")) c->test_poll_ms = std::max(1, atoi(tm));
  c->debug = getenv("TMG_DEBUG") != nullptr;
  c->has_model = true;
  return TMG_OK;
}

int finalize(tmg_ctx* c) {
  if (!c->has_model) return fail(c, TMG_ERR_INVALID, "context has no model config");
  if (c->finalized) return TMG_OK;
  for (int l = 0; l < c->L; ++l)
    if (c->layers[l].have != kHaveAll)
      return fail(c, TMG_ERR_INVALID,
                  "missing tensor in layer " + std::to_string(l) + " (have mask " +
                      std::to_string(c->layers[l].have) + ")");
  CK(cudaStreamSynchronize(c->stream), "finalize");
  c->finalized = true;
  return TMG_OK;
}

int ensure_prefill(tmg_ctx* c, int64_t T) {
  const int64_t Tc = std::min<int64_t>(T, kPrefillChunk);
  if (c->pf_cap >= Tc) return TMG_OK;
  for (void* p : {(void*)c->X, (void*)c->Xn, (void*)c->QKV, (void*)c->ATT, (void*)c->G,
                  (void*)c->U, (void*)c->d_tok, (void*)c->i8acc})
    if (p) cudaFree(p);
  c->i8acc = nullptr;
  c->pf_cap = 0;
  std::vector<void*> tmp;
  if (c->i8) CK(dalloc(tmp, &c->i8acc, size_t(Tc) * c->h), "alloc prefill");
  CK(dalloc(tmp, &c->X, size_t(Tc) * c->h), "alloc prefill");
  CK(dalloc(tmp, &c->Xn, size_t(Tc) * c->h), "alloc prefill");
  CK(dalloc(tmp, &c->QKV, size_t(Tc) * c->qkv_rows), "alloc prefill");
  CK(dalloc(tmp, &c->ATT, size_t(Tc) * c->nq * c->d), "alloc prefill");
  CK(dalloc(tmp, &c->G, size_t(Tc) * c->I), "alloc prefill");
  CK(dalloc(tmp, &c->U, size_t(Tc) * c->I), "alloc prefill");
  CK(dalloc(tmp, &c->d_tok, size_t(Tc)), "alloc prefill");
  c->pf_cap = Tc;
  return TMG_OK;
}

// A profiler (NVTX) range for the life of a scope; no cost without a tool.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

cudaError_t ensure_act_split(tmg_ctx* c, size_t n) {
  if (c->sa_cap >= n) return cudaSuccess;
  TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (c->sa_hi) cudaFree(c->sa_hi);
  if (c->sa_lo) cudaFree(c->sa_lo);
  c->sa_hi = c->sa_lo = nullptr;
  c->sa_cap = 0;
  TMG_CUDA_TRY(cudaMalloc(&c->sa_hi, n * 2));
  TMG_CUDA_TRY(cudaMalloc(&c->sa_lo, n * 2));
  c->sa_cap = n;
  return cudaSuccess;
}

cudaError_t ensure_split(tmg_ctx* c, size_t n) {
  if (c->sp_cap >= n) return cudaSuccess;
  TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (c->sp_hi) cudaFree(c->sp_hi);
  if (c->sp_lo) cudaFree(c->sp_lo);
  c->sp_hi = c->sp_lo = nullptr;
  c->sp_cap = 0;
  TMG_CUDA_TRY(cudaMalloc(&c->sp_hi, n * 2));
  TMG_CUDA_TRY(cudaMalloc(&c->sp_lo, n * 2));
  c->sp_cap = n;
  return cudaSuccess;
}

// Causal prefill attention of T query rows at pos0.. over cache rows
// [0, pos0 + T): the tcgen05 kernel for head dim 64 (TMG_PREFILL_ATTN=simt
// keeps the CUDA-core kernel), else the CUDA-core one.
// With parts (out_hi, out_lo) the tensor-core kernel writes the output as
// the O GEMM's hi/lo operands and *wrote_parts is set; the CUDA-core kernel
// always writes f32 into out.
// TMG_PREFILL_ATTN=simt: the CUDA-core prefill attention instead of the
// tensor-core one.
bool prefill_attn_simt() {
  static const bool simt = [] {
    const char* e = std::getenv("TMG_PREFILL_ATTN");
    return e && std::strcmp(e, "simt") == 0;
  }();
  return simt;
}

// rope_cos / rope_sin: q holds the chunk's un-rotated projections and the
// tensor-core path does RoPE and the KV append itself (*roped set); the
// caller runs launch_rope_append when *roped stays false.
cudaError_t prefill_attention(tmg_ctx* c, const float* q, int64_t q_ld, const float* kc,
                              const float* vc, int64_t T, int64_t pos0, float scale, float* out,
                              int64_t out_ld, int nq, int nkv, int d, uint16_t* out_hi = nullptr,
                              uint16_t* out_lo = nullptr, bool* wrote_parts = nullptr,
                              const float* rope_cos = nullptr, const float* rope_sin = nullptr,
                              bool* roped = nullptr) {
  const bool simt = prefill_attn_simt();
  if (wrote_parts) *wrote_parts = false;
  if (roped) *roped = false;
  if (!simt && attn_prefill_tc_ok(q, q_ld, kc, vc, T, pos0, nq, nkv, d, out, out_ld)) {
    const size_t need = attn_prefill_tc_scratch(nq, nkv, T, pos0 + T);
    if (c->pfa_cap < need) {
      TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
      if (c->pfa) cudaFree(c->pfa);
      c->pfa = nullptr;
      c->pfa_cap = 0;
      const size_t bytes = need + need / 4;  // room for a few more keys
      TMG_CUDA_TRY(cudaMalloc(&c->pfa, bytes));
      c->pfa_cap = bytes;
    }
    const bool parts = out_hi && out_lo;
    if (wrote_parts) *wrote_parts = parts;
    const bool rope = rope_cos && rope_sin && roped;
    if (rope) *roped = true;
    return launch_attn_prefill_tc(q, q_ld, kc, vc, T, pos0, nq, nkv, scale, out,
                                  parts ? out_hi : nullptr, parts ? out_lo : nullptr, out_ld,
                                  c->pfa, c->pfa_cap, c->d_err, c->stream,
                                  rope ? rope_cos : nullptr, rope ? rope_sin : nullptr);
  }
  return launch_attn_prefill(q, q_ld, kc, vc, T, pos0, nq, nkv, d, scale, out, out_ld, c->stream);
}

// y (+)= x . W^T for T rows (the prefill GEMM): tcgen05 tensor cores on the
// hi/lo BF16 split of x; the SIMT kernel only for rows of K % 8 != 0.
cudaError_t gemm(tmg_ctx* c, const float* x, const uint16_t* w, int64_t T, int64_t N, int64_t K,
                 float* y, int64_t ldy, bool acc) {
  if (gemm_tc_supported(K, w)) {
    TMG_CUDA_TRY(ensure_split(c, size_t(T) * K));
    TMG_CUDA_TRY(launch_split(x, T * K, c->sp_hi, c->sp_lo, c->stream));
    return launch_gemm_tc(c->sp_hi, c->sp_lo, w, T, N, K, y, ldy, acc, c->d_err, c->stream);
  }
  return launch_gemm_simt(x, w, T, N, K, y, ldy, acc, c->stream);
}

// The prefill GEMM of one layer matrix: BF16 as is, or (TMG_I8=1) the int8
// rows widened to BF16 (exact) for the tensor cores, then scaled per row
// (matmul_batch_w_into's I8 writeback: acc * scale[o], src/tensor.rs:
// 736-738), and added into y when acc.
cudaError_t gemm_layer(tmg_ctx* c, const float* x, const uint16_t* w, const int8_t* q,
                       const float* sc, int64_t T, int64_t N, int64_t K, float* y, int64_t ldy,
                       bool acc) {
  if (!q) return gemm(c, x, w, T, N, K, y, ldy, acc);
  const size_t n = size_t(N) * size_t(K);
  if (c->dq_cap < n) {
    TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (c->dq) cudaFree(c->dq);
    c->dq = nullptr;
    c->dq_cap = 0;
    TMG_CUDA_TRY(cudaMalloc(&c->dq, n * 2));
    c->dq_cap = n;
  }
  TMG_CUDA_TRY(launch_widen_i8(q, n, c->dq, c->stream));
  float* tmp = (acc || ldy != N) ? c->i8acc : y;
  if (tmp == nullptr) return cudaErrorInvalidValue;
  TMG_CUDA_TRY(gemm(c, x, c->dq, T, N, K, tmp, N, false));
  return launch_scale_rows(tmp, T, N, sc, y, ldy, acc, c->stream);
}

// GEMV with an optional fused prologue; falls back to separate embedding /
// norm kernels when the fused kernel does not take the shape.
cudaError_t gemv(tmg_ctx* c, GemvArgs a, GemvPro pro, GemvEpi epi, bool pdl) {
  a.err = c->d_err;
  if (!gemv_fused_ok(a, epi) && pro != PRO_NONE) {
    if (pro == PRO_EMBED_NORM) {
      TMG_CUDA_TRY(launch_embed(a.embed, a.tokens, a.M, a.K, a.x_out, c->stream));
      a.x = a.x_out;
    }
    TMG_CUDA_TRY(launch_rmsnorm(a.x, a.norm_w, a.eps, a.K, a.M, a.norm_mode, c->xn, c->stream));
    a.x = c->xn;
    pro = PRO_NONE;
  }
  return launch_gemv(a, pro, epi, c->stream, pdl, c->num_sms);
}

// Sum the partial [M, n] over the TP ranks and add it into dst.
cudaError_t tp_reduce_add(tmg_ctx* c, float* partial, float* dst, int64_t n) {
  TMG_CUDA_TRY(tp_allreduce_sum(c->tp, partial, n, c->stream));
  return launch_add(partial, dst, n, c->stream);
}

// Per-kernel CUDA events of the profiling pass (tmg_profile_decode): classes
// 0 qkv GEMV, 1 attention, 2 o GEMV, 3 gate/up GEMV, 4 down GEMV, 5 LM head,
// 6 allreduce + residual add (tensor parallel), 7 logits allgather + end of
// step (tensor parallel).
constexpr int kProfClasses = 8;
struct Prof {
  cudaStream_t s;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
  cudaEvent_t open = nullptr;
  void begin() {
    cudaEventCreate(&open);
    cudaEventRecord(open, s);
  }
  void end(int cls) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, s);
    marks.push_back({cls, {open, e}});
    open = nullptr;
  }
  ~Prof() {
    for (auto& m : marks) {
      cudaEventDestroy(m.second.first);
      cudaEventDestroy(m.second.second);
    }
  }
};

// One forward_token for the M streams of kv (model.rs:392-491).
// Trace slots of one captured forward (tmg_trace_decode): kernel i of the
// forward writes its timeline into slot i; kinds[i] = its class.
struct TraceCtx {
  unsigned long long* buf = nullptr;
  int next = 0;
  std::vector<int> kinds;
  Trace take(int kind) {
    Trace t;
    if (buf) {
      t.buf = buf;
      t.slot = next++;
      kinds.push_back(kind);
    }
    return t;
  }
};

// A host callback at a point of the forward (debug prints): (layer, what)
// with what 0 = the embedding (layer -1), 1 = after the attention residual,
// 2 = after the MLP residual.  The forward is then enqueued eagerly.
using DebugHook = std::function<cudaError_t(int, int)>;

cudaError_t enqueue_forward(tmg_ctx* c, tmg_kv* kv, const StreamState& st, bool argmax,
                            Prof* prof = nullptr, TraceCtx* trc = nullptr,
                            const DebugHook* dbg = nullptr) {
  TraceCtx none;
  TraceCtx& tc = trc ? *trc : none;
  const int M = kv->M;
  const bool pdl = prof == nullptr && dbg == nullptr;
  auto B = [&]() {
    if (prof) prof->begin();
  };
  auto E = [&](int cls) {
    if (prof) prof->end(cls);
  };
  const float eps = c->cfg.rms_norm_eps;
  const bool tp = c->world > 1;
  // an int8 GEMV of this forward (TMG_I8=1): x (RMSNorm'd by norm_w when
  // given) quantized per row, integer dots, y (+)= the scaled result
  auto gemv8 = [&](const int8_t* q, const float* sc, const int8_t* q2, const float* sc2,
                   const float* x, const float* norm_w, float* y, int64_t ldy, int64_t N, int K,
                   GemvEpi epi) {
    GemvI8Args a;
    a.q = q;
    a.scales = sc;
    a.q2 = q2;
    a.scales2 = sc2;
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.norm_mode = 0;
    a.xq = c->xq8;
    a.xs = c->xs8;
    a.y = y;
    a.ldy = ldy;
    a.N = N;
    a.K = K;
    a.M = M;
    a.err = c->d_err;
    return launch_gemv_i8(a, epi, c->stream, pdl, c->num_sms);
  };
  for (int l = 0; l < c->L; ++l) {
    const Layer& Lw = c->layers[l];
    if (c->i8) {
      B();
      if (l == 0) TMG_CUDA_TRY(launch_embed(c->embed, st.token, M, c->h, c->x, c->stream));
      if (l == 0 && dbg) TMG_CUDA_TRY((*dbg)(-1, 0));
      TMG_CUDA_TRY(gemv8(Lw.qqkv, Lw.sqkv, nullptr, nullptr, c->x, Lw.in_norm, c->qkv,
                         c->qkv_rows, c->qkv_rows, c->h, EPI_STORE));
      E(0);
    }
    GemvArgs A;
    A.w = Lw.wqkv;
    A.N = c->qkv_rows;
    A.K = c->h;
    A.M = M;
    A.y = c->qkv;
    A.ldy = c->qkv_rows;
    A.norm_w = Lw.in_norm;
    A.eps = eps;
    A.norm_mode = 0;
    A.trace = tc.take(0);
    if (c->i8) {
      // done above
    } else if (l == 0) {
      A.embed = c->embed;
      A.tokens = st.token;
      A.x_out = c->x;
      B();
      TMG_CUDA_TRY(gemv(c, A, PRO_EMBED_NORM, EPI_STORE, pdl));
      E(0);
      if (dbg) TMG_CUDA_TRY((*dbg)(-1, 0));
    } else {
      A.x = c->x;
      B();
      TMG_CUDA_TRY(gemv(c, A, PRO_NORM, EPI_STORE, pdl));
      E(0);
    }
    AttnDecodeArgs T;
    T.qkv = c->qkv;
    T.qkv_ld = c->qkv_rows;
    T.kc = kv->k[l];
    T.vc = kv->v[l];
    T.cap = kv->cap;
    T.rope_cos = kv->rope_cos;
    T.rope_sin = kv->rope_sin;
    T.out = c->attn;
    T.part = kv->part;
    T.ticket = kv->att_ticket;
    T.st = st;
    T.nq = c->nq;
    T.nkv = c->nkv;
    T.d = c->d;
    T.nsplit = kv->nsplit;
    T.M = M;
    T.scale = 1.0f / sqrtf(float(c->d));
    T.err = c->d_err;
    T.trace = tc.take(1);
    B();
    TMG_CUDA_TRY(launch_attn_decode(T, c->stream, pdl));
    E(1);
    GemvArgs O;
    O.w = Lw.wo;
    O.N = c->h;
    O.K = c->nq * c->d;
    O.M = M;
    O.x = c->attn;
    O.y = tp ? c->partial : c->x;
    O.ldy = c->h;
    O.trace = tc.take(2);
    B();
    if (c->i8)
      TMG_CUDA_TRY(gemv8(Lw.qo, Lw.so, nullptr, nullptr, c->attn, nullptr, c->x, c->h, c->h,
                         c->nq * c->d, EPI_ADD));
    else
      TMG_CUDA_TRY(gemv(c, O, PRO_NONE, tp ? EPI_STORE : EPI_ADD, pdl));
    E(2);
    if (tp) {
      B();
      TMG_CUDA_TRY(tp_reduce_add(c, c->partial, c->x, int64_t(M) * c->h));
      E(6);
    }
    if (dbg) TMG_CUDA_TRY((*dbg)(l, 1));
    GemvArgs GU;
    GU.w = Lw.wg;
    GU.w2 = Lw.wu;
    GU.N = c->I;
    GU.K = c->h;
    GU.M = M;
    GU.x = c->x;
    GU.norm_w = Lw.post_norm;
    GU.eps = eps;
    GU.y = c->act;
    GU.ldy = c->I;
    GU.trace = tc.take(3);
    B();
    if (c->i8)
      TMG_CUDA_TRY(gemv8(Lw.qg, Lw.sg, Lw.qu, Lw.su, c->x, Lw.post_norm, c->act, c->I, c->I, c->h,
                         EPI_SWIGLU));
    else
      TMG_CUDA_TRY(gemv(c, GU, PRO_NORM, EPI_SWIGLU, pdl));
    E(3);
    GemvArgs D;
    D.w = Lw.wd;
    D.N = c->h;
    D.K = c->I;
    D.M = M;
    D.x = c->act;
    D.y = tp ? c->partial : c->x;
    D.ldy = c->h;
    D.trace = tc.take(4);
    B();
    if (c->i8)
      TMG_CUDA_TRY(gemv8(Lw.qd, Lw.sd, nullptr, nullptr, c->act, nullptr, c->x, c->h, c->h, c->I,
                         EPI_ADD));
    else
      TMG_CUDA_TRY(gemv(c, D, PRO_NONE, tp ? EPI_STORE : EPI_ADD, pdl));
    E(4);
    if (tp) {
      B();
      TMG_CUDA_TRY(tp_reduce_add(c, c->partial, c->x, int64_t(M) * c->h));
      E(6);
    }
    if (dbg) TMG_CUDA_TRY((*dbg)(l, 2));
  }
  GemvArgs H;
  H.w = c->lm_head;
  H.N = c->V_l;
  H.K = c->h;
  H.M = M;
  H.x = c->x;
  H.norm_w = c->final_norm;
  H.eps = eps;
  H.norm_mode = 0;
  H.y = c->logits;
  H.ldy = c->V_l;
  H.am_part = c->am_part;
  H.ticket = &c->tickets[0];
  H.st = st;
  H.trace = tc.take(5);
  if (!tp) {
    B();
    cudaError_t e = gemv(c, H, PRO_NORM, argmax ? EPI_HEAD_ARGMAX : EPI_HEAD, pdl);
    E(5);
    return e;
  }
  // TP: vocab-split head; gather the logits, then the same end of step
  B();
  TMG_CUDA_TRY(gemv(c, H, PRO_NORM, EPI_STORE, pdl));
  E(5);
  B();
  TMG_CUDA_TRY(tp_allgather_rows(c->tp, c->logits, c->V_l, c->logits_full, c->V, M, c->stream));
  TMG_CUDA_TRY(launch_step_end(st, M, argmax ? c->logits_full : nullptr, c->V, c->stream));
  E(7);
  return cudaSuccess;
}

// forward_seq for one stream (model.rs:503-590): chunks of kPrefillChunk
// tokens through all layers; the last row's logits land in row `stream` of
// the decode logits buffer.
int forward_seq(tmg_ctx* c, tmg_kv* kv, int stream, const uint32_t* tokens, int64_t T,
                bool host_tokens) {
  int rc;
  if ((rc = ensure_prefill(c, T))) return rc;
  const int64_t p0 = kv->lens[stream];
  const int64_t kvd = kv->kvd;
  const float eps = c->cfg.rms_norm_eps;
  const float scale = 1.0f / sqrtf(float(c->d));
  const bool tp = c->world > 1;
  if (host_tokens) CK(ensure_pinned(c, size_t(T) * 4), "pinned");
  for (int64_t t0 = 0; t0 < T; t0 += c->pf_cap) {
    const int64_t Tc = std::min<int64_t>(c->pf_cap, T - t0);
    const int64_t pos0 = p0 + t0;
    const uint32_t* dtok;
    if (host_tokens) {
      CK(cudaStreamSynchronize(c->stream), "prefill");
      std::memcpy(c->pinned, tokens + t0, size_t(Tc) * 4);
      CK(cudaMemcpyAsync(c->d_tok, c->pinned, size_t(Tc) * 4, cudaMemcpyHostToDevice, c->stream),
         "prefill tokens");
      dtok = c->d_tok;
    } else {
      dtok = tokens + t0;
    }
    CK(launch_embed(c->embed, dtok, Tc, c->h, c->X, c->stream), "embed");
    for (int l = 0; l < c->L; ++l) {
      const Layer& Lw = c->layers[l];
      // one profiler range per layer of the chunk (host side: the enqueues)
      char rname[48];
      std::snprintf(rname, sizeof rname, "prefill layer %d", l);
      NvtxRange layer_range(rname);
      float* kc = kv->k[l] + size_t(stream) * kv->cap * kvd;
      float* vc = kv->v[l] + size_t(stream) * kv->cap * kvd;
      if (!c->i8 && gemm_tc_supported(c->h, Lw.wqkv)) {
        // rmsnorm written straight as the qkv GEMM's hi/lo operands
        CK(ensure_split(c, size_t(Tc) * c->h), "split");
        CK(launch_rmsnorm_split(c->X, Lw.in_norm, eps, c->h, Tc, c->sp_hi, c->sp_lo, c->stream),
           "rmsnorm");
        CK(launch_gemm_tc(c->sp_hi, c->sp_lo, Lw.wqkv, Tc, c->qkv_rows, c->h, c->QKV, c->qkv_rows,
                          false, c->d_err, c->stream),
           "gemm qkv");
      } else {
        CK(launch_rmsnorm(c->X, Lw.in_norm, eps, c->h, Tc, 1, c->Xn, c->stream), "rmsnorm");
        CK(gemm_layer(c, c->Xn, Lw.wqkv, Lw.qqkv, Lw.sqkv, Tc, c->qkv_rows, c->h, c->QKV,
                      c->qkv_rows, false),
           "gemm qkv");
      }
      // the attention output straight as the O GEMM's hi/lo operands when
      // that GEMM runs on the tensor cores; RoPE and the KV append inside
      // the tensor-core attention's first pass (else rope_append first)
      const int64_t qd = int64_t(c->nq) * c->d;
      const bool o_parts = !tp && !c->i8 && gemm_tc_supported(qd, Lw.wo) &&
                           ensure_split(c, size_t(Tc) * std::max<int64_t>(qd, c->h)) == cudaSuccess;
      bool att_parts = false, roped = false;
      const bool tc_attn = attn_prefill_tc_ok(c->QKV, c->qkv_rows, kc, vc, Tc, pos0, c->nq, c->nkv,
                                              c->d, c->ATT, qd) &&
                           !prefill_attn_simt();
      if (!tc_attn)
        CK(launch_rope_append(c->QKV, c->qkv_rows, Tc, c->nq, c->nkv, c->d, kv->rope_cos,
                              kv->rope_sin, pos0, kc, vc, c->stream),
           "rope");
      CK(prefill_attention(c, c->QKV, c->qkv_rows, kc, vc, Tc, pos0, scale, c->ATT, qd, c->nq,
                           c->nkv, c->d, o_parts ? c->sp_hi : nullptr,
                           o_parts ? c->sp_lo : nullptr, &att_parts,
                           tc_attn ? kv->rope_cos : nullptr, tc_attn ? kv->rope_sin : nullptr,
                           &roped),
         "attention");
      if (tc_attn && !roped) return fail(c, TMG_ERR_CUDA, "prefill attention: RoPE not applied");
      if (att_parts) {
        CK(launch_gemm_tc(c->sp_hi, c->sp_lo, Lw.wo, Tc, c->h, qd, c->X, c->h, true, c->d_err,
                          c->stream),
           "gemm o");
      } else if (tp) {
        CK(gemm(c, c->ATT, Lw.wo, Tc, c->h, int64_t(c->nq) * c->d, c->Xn, c->h, false), "gemm o");
        CK(tp_reduce_add(c, c->Xn, c->X, Tc * c->h), "allreduce");
      } else {
        CK(gemm_layer(c, c->ATT, Lw.wo, Lw.qo, Lw.so, Tc, c->h, int64_t(c->nq) * c->d, c->X, c->h,
                      true),
           "gemm o");
      }
      // the MLP's input: rmsnorm as f32 (int8 weights, tensor parallel, other
      // shapes) or straight as the gate/up GEMM's hi/lo operands
      const bool fuse_mlp = !c->i8 && gemm_tc_supported(c->h, Lw.wg) &&
                            gemm_tc_supported(c->h, Lw.wu) && gemm_tc_supported(c->I, Lw.wd) &&
                            ensure_act_split(c, size_t(Tc) * c->I) == cudaSuccess &&
                            gemm_swiglu_supported(c->I, c->sa_hi, c->sa_lo);
      if (fuse_mlp) {
        CK(ensure_split(c, size_t(Tc) * c->h), "split");
        CK(launch_rmsnorm_split(c->X, Lw.post_norm, eps, c->h, Tc, c->sp_hi, c->sp_lo,
                                c->stream),
           "rmsnorm");
      } else {
        CK(launch_rmsnorm(c->X, Lw.post_norm, eps, c->h, Tc, 1, c->Xn, c->stream), "rmsnorm");
      }
      bool swiglu_done = false;  // act already split for the down GEMM
      if (c->i8) {
        CK(gemm_layer(c, c->Xn, Lw.wg, Lw.qg, Lw.sg, Tc, c->I, c->h, c->G, c->I, false),
           "gemm gate");
        CK(gemm_layer(c, c->Xn, nullptr, Lw.qu, Lw.su, Tc, c->I, c->h, c->U, c->I, false), "gemm up");
      } else if (fuse_mlp) {
        // gate and up read the same input: one launch whose tiles hold
        // matching gate and up columns, SwiGLU in its epilogue written as the
        // down GEMM's hi/lo operands
        CK(launch_gemm_tc_swiglu(c->sp_hi, c->sp_lo, Lw.wg, Lw.wu, c->I, Tc, c->h, c->sa_hi,
                                 c->sa_lo, c->d_err, c->stream),
           "gemm gate/up + swiglu");
        swiglu_done = true;
      } else if (gemm_tc_supported(c->h, Lw.wg) && gemm_tc_supported(c->h, Lw.wu)) {
        // gate and up read the same input: one hi/lo split, one launch whose
        // tiles cover both outputs
        CK(ensure_split(c, size_t(Tc) * c->h), "split");
        CK(launch_split(c->Xn, Tc * c->h, c->sp_hi, c->sp_lo, c->stream), "split");
        CK(launch_gemm_tc2(c->sp_hi, c->sp_lo, Lw.wg, c->I, c->G, c->I, Lw.wu, c->I, c->U, c->I,
                           Tc, c->h, false, c->d_err, c->stream),
           "gemm gate/up");
      } else {
        CK(gemm(c, c->Xn, Lw.wg, Tc, c->I, c->h, c->G, c->I, false), "gemm gate");
        CK(gemm(c, c->Xn, Lw.wu, Tc, c->I, c->h, c->U, c->I, false), "gemm up");
      }
      float* down_y = tp ? c->Xn : c->X;
      if (swiglu_done) {
        CK(launch_gemm_tc(c->sa_hi, c->sa_lo, Lw.wd, Tc, c->h, c->I, down_y, c->h, !tp, c->d_err,
                          c->stream),
           "gemm down");
      } else if (c->i8) {
        CK(launch_swiglu(c->G, c->U, Tc * c->I, c->G, c->stream), "swiglu");
        CK(gemm_layer(c, c->G, nullptr, Lw.qd, Lw.sd, Tc, c->h, c->I, down_y, c->h, !tp), "gemm down");
      } else if (gemm_tc_supported(c->I, Lw.wd) && (ensure_split(c, size_t(Tc) * c->I) == cudaSuccess) &&
          swiglu_split_supported(c->G, c->U, Tc * c->I, c->sp_hi, c->sp_lo)) {
        // SwiGLU written straight as the down GEMM's hi/lo operands
        CK(launch_swiglu_split(c->G, c->U, Tc * c->I, c->sp_hi, c->sp_lo, c->stream), "swiglu");
        CK(launch_gemm_tc(c->sp_hi, c->sp_lo, Lw.wd, Tc, c->h, c->I, down_y, c->h, !tp, c->d_err,
                          c->stream),
           "gemm down");
      } else {
        CK(launch_swiglu(c->G, c->U, Tc * c->I, c->G, c->stream), "swiglu");
        CK(gemm(c, c->G, Lw.wd, Tc, c->h, c->I, down_y, c->h, !tp), "gemm down");
      }
      if (tp) CK(tp_reduce_add(c, c->Xn, c->X, Tc * c->h), "allreduce");
    }
    if (t0 + Tc == T) {
      GemvArgs H;
      H.w = c->lm_head;
      H.N = c->V_l;
      H.K = c->h;
      H.M = 1;
      H.x = c->X + size_t(Tc - 1) * c->h;
      H.norm_w = c->final_norm;
      H.eps = eps;
      H.norm_mode = 1;  // forward_seq's final norm is rms_norm_batch (model.rs:587)
      H.y = c->logits + size_t(stream) * c->V_l;
      H.ldy = c->V_l;
      CK(gemv(c, H, PRO_NORM, EPI_STORE, false), "lm_head");
      if (tp)
        CK(tp_allgather_rows(c->tp, c->logits + size_t(stream) * c->V_l, c->V_l,
                             c->logits_full + size_t(stream) * c->V, c->V, 1, c->stream),
           "allgather");
    }
  }
  CK(launch_set_pos(kv->st, stream, int32_t(p0 + T), c->stream), "set pos");
  kv->lens[stream] = p0 + T;
  return TMG_OK;
}

const float* logits_row(tmg_ctx* c, int m) {
  return c->world > 1 ? c->logits_full + size_t(m) * c->V : c->logits + size_t(m) * c->V_l;
}

std::vector<float> rope_table(int d, float theta, int64_t n_pos, bool sin_part) {
  // Rope::new / ensure, src/tensor.rs:1005-1023: f32 powf, recip, f32
  // angle, glibc sinf / cosf -- the same values the reference computes.
  const int half = d / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) {
    const float e = (2.0f * float(i)) / float(d);
    inv[i] = 1.0f / powf(theta, e);
  }
  std::vector<float> t(size_t(n_pos) * half);
  for (int64_t p = 0; p < n_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const float ang = float(p) * inv[i];
      t[size_t(p) * half + i] = sin_part ? sinf(ang) : cosf(ang);
    }
  return t;
}

int reset_state(tmg_ctx* c, tmg_kv* kv) {
  CK(cudaMemsetAsync(kv->d_state, 0, sizeof(int32_t) * 4 * kMaxStreams, c->stream), "reset");
  for (auto& v : kv->lens) v = 0;
  return TMG_OK;
}

int check_sampling(tmg_ctx* c, const tmg_gen_params* p) {
  if (!p || p->max_tokens < 0) return fail(c, TMG_ERR_INVALID, "bad generation params");
  if (p->temperature > 0.f && (p->top_k < 1 || p->top_k > kMaxTopK || p->top_k >= c->V))
    return fail(c, TMG_ERR_INVALID,
                "device sampling needs 1 <= top_k <= 64 (top_k = 0 / full-vocabulary "
                "sampling is not implemented on the device)");
  return TMG_OK;
}

// n_steps greedy steps (forward + argmax + generate's bookkeeping) of the
// single stream of kv in one persistent launch (decode_fused.cu).
cudaError_t launch_fused(tmg_ctx* c, tmg_kv* kv, const StreamState& st, int64_t n_steps,
                         unsigned long long* trace = nullptr) {
  FusedArgs f;
  f.layers = kv->d_layers;
  f.L = c->L;
  f.h = c->h;
  f.nq = c->nq;
  f.nkv = c->nkv;
  f.d = c->d;
  f.I = c->I;
  f.V = int(c->V_l);
  f.eps = c->cfg.rms_norm_eps;
  f.scale = 1.0f / sqrtf(float(c->d));
  f.embed = c->embed;
  f.lm_head = c->lm_head;
  f.final_norm = c->final_norm;
  f.rope_cos = kv->rope_cos;
  f.rope_sin = kv->rope_sin;
  f.cap = kv->cap;
  const int q_dim = c->nq * c->d;
  f.ll_base = c->ll;
  f.ll_bytes =
      fused_ll_words(c->h, q_dim, c->I, c->qkv_rows, c->fused_rep) * sizeof(unsigned long long);
  f.ll_rep = c->fused_rep;
  f.x_ll = c->ll;
  f.att_ll = f.x_ll + size_t(c->fused_rep) * c->h;
  f.act_ll = f.att_ll + size_t(c->fused_rep) * q_dim;
  f.qkv_ll = f.act_ll + size_t(c->fused_rep) * c->I;
  f.part_ll = kv->part_ll;
  f.logits = c->logits;
  f.am_part = c->am_part;
  f.bar = c->bar;
  f.nsplit = kv->nsplit_f;
  f.pf_ahead = c->fused_pf;
  f.pf_pace = c->fused_pf_pace;
  f.pf_mode = c->fused_pf_mode;
  f.max_stages = c->fused_stages;
  f.st = st;
  f.n_steps = int(n_steps);
  f.err = c->d_err;
  f.trace = trace;
  if (c->test_stall >= 0) {
    f.stall_phase = c->test_stall;
    f.poll_ns = (unsigned long long)(c->test_poll_ms) * 1000000ull;
    c->test_stall = -1;
  }
  FusedGroup* g = kv->grp;
  if (!g) return launch_decode_fused(f, c->num_sms, c->stream);
  f.rank = g->rank;
  f.world = g->world;
  // every copy of an exchange word is stored into every rank's memory: one
  // copy (measured on 2 GPUs: 516 tok/s with one, 505 with four)
  if (!c->fused_rep_set) f.ll_rep = 1;
  for (int r = 0; r < g->world; ++r) {
    f.ll_peer[r] = g->ll_peer[r];
    f.part_peer[r] = g->part_peer[r];
    f.bar_peer[r] = g->bar_peer[r];
    f.am_peer[r] = g->am_peer[r];
  }
  f.kv_peer = g->d_kv_peer;
  f.am_part = g->am;
  // every rank has finished the previous launch (its writes into this
  // rank's buffers included) before any zeroes; every rank has zeroed
  // before any starts
  TMG_CUDA_TRY(tp_barrier(g->comm, g->sync, c->stream));
  TMG_CUDA_TRY(fused_zero(f, c->stream));
  TMG_CUDA_TRY(tp_barrier(g->comm, g->sync, c->stream));
  return launch_decode_fused(f, g->ctas, c->stream, false);
}

bool use_fused(tmg_ctx* c, tmg_kv* kv) { return c->fused_ok && kv->M == 1 && kv->d_layers && kv->part_ll; }

// The generate loop for all streams of kv (model.rs:614-663).
int run_generate(tmg_ctx* c, tmg_kv* kv, const uint32_t* prompts, int64_t T,
                 const tmg_gen_params* params, const float* uniforms, uint32_t* tokens_out,
                 int64_t* n_out, float* first_logits, double* prefill_secs, tmg_token_cb cb,
                 void* user) {
  int rc;
  if (!c->finalized) return fail(c, TMG_ERR_INVALID, "weights not finalized");
  if ((rc = check_sampling(c, params))) return rc;
  const int M = kv->M;
  const int64_t maxt = params->max_tokens;
  for (int m = 1; m < M; ++m)
    if (params[m].max_tokens != maxt || params[m].temperature != params[0].temperature ||
        params[m].top_k != params[0].top_k || params[m].top_p != params[0].top_p ||
        params[m].repetition_penalty != params[0].repetition_penalty)
      return fail(c, TMG_ERR_INVALID, "batched streams must share sampling settings");
  if (T <= 0) return fail(c, TMG_ERR_INVALID, "empty prompt");
  if (T + maxt > kv->cap) return fail(c, TMG_ERR_CAPACITY, "prompt + max_tokens exceeds KV capacity");
  for (int64_t i = 0; i < int64_t(M) * T; ++i)
    if (prompts[i] >= uint32_t(c->V)) return fail(c, TMG_ERR_INVALID, "token id out of range");
  if ((rc = reset_state(c, kv))) return rc;
  auto t0 = std::chrono::steady_clock::now();
  for (int m = 0; m < M; ++m)
    if ((rc = forward_seq(c, kv, m, prompts + size_t(m) * T, T, true))) return rc;
  CK(cudaStreamSynchronize(c->stream), "prefill");
  auto t1 = std::chrono::steady_clock::now();
  if (prefill_secs) *prefill_secs = std::chrono::duration<double>(t1 - t0).count();
  if (first_logits)
    for (int m = 0; m < M; ++m)
      CK(copy_sync(c, first_logits + size_t(m) * c->V, logits_row(c, m), size_t(c->V) * 4,
                   cudaMemcpyDeviceToHost),
         "first logits");
  for (int m = 0; m < M; ++m) n_out[m] = 0;
  if (maxt == 0) return TMG_OK;

  // device state for the loop
  if (kv->gen_alloc < int64_t(M) * maxt) {
    if (kv->d_gen) cudaFree(kv->d_gen);
    kv->d_gen = nullptr;
    kv->gen_alloc = 0;
    CK(cudaMalloc(&kv->d_gen, size_t(M) * maxt * 4), "alloc");
    kv->gen_alloc = int64_t(M) * maxt;
  }
  const bool sampled = params->temperature > 0.f;
  const bool greedy_fused = !sampled && params->repetition_penalty == 1.0f;
  if (sampled) {
    if (kv->uni_alloc < int64_t(M) * maxt) {
      if (kv->d_uni) cudaFree(kv->d_uni);
      kv->d_uni = nullptr;
      kv->uni_alloc = 0;
      CK(cudaMalloc(&kv->d_uni, size_t(M) * maxt * 4), "alloc");
      kv->uni_alloc = int64_t(M) * maxt;
    }
    std::vector<float> u(size_t(M) * maxt);
    if (uniforms) std::memcpy(u.data(), uniforms, u.size() * 4);
    else
      for (int m = 0; m < M; ++m) stdrng_uniforms(params[m].seed, maxt, u.data() + size_t(m) * maxt);
    CK(cudaMemcpyAsync(kv->d_uni, u.data(), u.size() * 4, cudaMemcpyHostToDevice, c->stream),
       "uniforms");
    CK(cudaStreamSynchronize(c->stream), "uniforms");
  }
  StreamState st = kv->st;
  st.gen = kv->d_gen;
  st.gen_cap = int32_t(maxt);
  st.n_eos = c->cfg.n_eos;
  for (int e = 0; e < c->cfg.n_eos && e < kMaxEos; ++e) st.eos[e] = c->cfg.eos_token_ids[e];

  SampleArgs S;
  S.logits = const_cast<float*>(logits_row(c, 0));
  S.V = c->V;
  S.M = M;
  S.temperature = params->temperature;
  S.top_k = int(params->top_k);
  S.top_p = params->top_p;
  S.penalty = params->repetition_penalty;
  S.uniforms = kv->d_uni;
  S.uni_ld = maxt;
  S.part = c->sm_part;
  S.ticket = &c->tickets[1];
  S.err = c->d_err;
  S.st = st;
  S.record = true;

  // first token from the prefill logits
  if (greedy_fused) {
    CK(launch_sample(S, c->stream, false, c->num_sms), "argmax");
  } else {
    CK(launch_sample(S, c->stream, false, c->num_sms), "sample");
  }
  // the per-step work: the fused persistent kernel (greedy, one stream), or
  // a graph of forward (+ argmax) [+ sampler]
  const bool fused = greedy_fused && use_fused(c, kv);
  cudaGraphExec_t exec = nullptr;
  if (!fused) {
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "capture");
    cudaError_t ce = enqueue_forward(c, kv, st, greedy_fused);
    if (ce == cudaSuccess && !greedy_fused) ce = launch_sample(S, c->stream, true, c->num_sms);
    cudaError_t ee = cudaStreamEndCapture(c->stream, &graph);
    if (ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return cuda_fail(c, ce, "capture step");
    }
    CK(ee, "capture");
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(ce, "instantiate");
  }

  // launch max_tokens steps in chunks; read back tokens a chunk behind
  const int64_t chunk = fused ? 32 : 8;
  std::vector<int32_t> h_state(4 * kMaxStreams);
  std::vector<uint32_t> h_gen(size_t(M) * maxt);
  int64_t launched = 0;
  std::vector<int64_t> reported(M, 0);
  bool stop = false;
  cudaEvent_t ev[2];
  CK(cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming), "event");
  CK(cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming), "event");
  int32_t* pinned_state = nullptr;
  CK(ensure_pinned(c, sizeof(int32_t) * (4 * kMaxStreams + 1) * 2 + size_t(M) * maxt * 4 * 2),
     "pinned");
  pinned_state = static_cast<int32_t*>(c->pinned);
  uint32_t* pinned_gen = reinterpret_cast<uint32_t*>(pinned_state + 8 * kMaxStreams);
  // the device error word after each chunk (a failed step ends the loop)
  int32_t* pinned_err = reinterpret_cast<int32_t*>(pinned_gen + size_t(M) * maxt * 2);
  int pending = -1;
  auto drain = [&](int slot) -> int {
    CK(cudaEventSynchronize(ev[slot]), "sync");
    int32_t* s = pinned_state + slot * 4 * kMaxStreams;
    uint32_t* g = pinned_gen + size_t(slot) * M * maxt;
    bool all_done = true;
    for (int m = 0; m < M; ++m) {
      const int32_t ng = s[3 * kMaxStreams + m];
      if (cb && m == 0)
        for (int64_t i = reported[0]; i < ng && !stop; ++i)
          if (cb(g[i], user) != 0) stop = true;
      reported[m] = ng;
      if (!s[2 * kMaxStreams + m]) all_done = false;
    }
    if (all_done || pinned_err[slot] != 0) stop = true;
    return TMG_OK;
  };
  int n_chunks = 0;
  while (launched < maxt && !stop) {
    const int64_t n = std::min<int64_t>(chunk, maxt - launched);
    if (fused)
      CK(launch_fused(c, kv, st, n), "fused decode");
    else
      for (int64_t i = 0; i < n; ++i) CK(cudaGraphLaunch(exec, c->stream), "graph launch");
    launched += n;
    const int slot = (n_chunks++) & 1;
    CK(cudaMemcpyAsync(pinned_state + slot * 4 * kMaxStreams, kv->d_state,
                       sizeof(int32_t) * 4 * kMaxStreams, cudaMemcpyDeviceToHost, c->stream),
       "state");
    CK(cudaMemcpyAsync(pinned_gen + size_t(slot) * M * maxt, kv->d_gen, size_t(M) * maxt * 4,
                       cudaMemcpyDeviceToHost, c->stream),
       "tokens");
    CK(cudaMemcpyAsync(pinned_err + slot, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream), "err");
    CK(cudaEventRecord(ev[slot], c->stream), "event");
    if (pending >= 0 && (rc = drain(pending))) return rc;
    pending = slot;
  }
  if (pending >= 0 && (rc = drain(pending))) return rc;
  CK(cudaStreamSynchronize(c->stream), "generate");
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  if (exec) cudaGraphExecDestroy(exec);
  int32_t err_word = 0;
  CK(copy_sync(c, &err_word, c->d_err, 4, cudaMemcpyDeviceToHost), "err");
  CK(copy_sync(c, h_state.data(), kv->d_state, h_state.size() * 4, cudaMemcpyDeviceToHost),
     "state");
  CK(copy_sync(c, h_gen.data(), kv->d_gen, h_gen.size() * 4, cudaMemcpyDeviceToHost), "tokens");
  if (err_word) {
    CK(zero_sync(c, c->d_err, 4), "err");
    return err_status(c, err_word);
  }
  for (int m = 0; m < M; ++m) {
    const int32_t ng = h_state[3 * kMaxStreams + m];
    n_out[m] = ng;
    std::memcpy(tokens_out + size_t(m) * maxt, h_gen.data() + size_t(m) * maxt, size_t(ng) * 4);
    kv->lens[m] = h_state[kMaxStreams + m];
    if (cb && m == 0)
      for (int64_t i = reported[0]; i < ng && !stop; ++i)
        if (cb(h_gen[i], user) != 0) stop = true;
  }
  return TMG_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* tmg_version(void) { return "tinyminigo_b200 0.1 (sm_100a)"; }

float tmg_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

int tmg_config_parse(const char* json_text, tmg_config* out, char* err, int errlen) {
  std::string e;
  Json j;
  if (!json_text || !out) return TMG_ERR_INVALID;
  if (!json_parse(json_text, std::strlen(json_text), j, e) || !config_from_json(j, out, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  return TMG_OK;
}

int tmg_config_load(const char* path, tmg_config* out, char* err, int errlen) {
  std::string text, e;
  if (!path || !out) return TMG_ERR_INVALID;
  if (!read_file(path, text, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  int rc = tmg_config_parse(text.c_str(), out, err, errlen);
  return rc;
}

int tmg_safetensors_count(const char* path, int64_t* n, char* err, int errlen) {
  MappedFile f;
  std::string e;
  std::vector<StTensor> ts;
  if (!path || !n) return TMG_ERR_INVALID;
  if (!f.open(path, e) || !safetensors_parse(f.data(), f.size, ts, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  *n = int64_t(ts.size());
  return TMG_OK;
}

int tmg_safetensors_info(const char* path, int64_t i, char* name, int namelen, int32_t* dtype,
                         int32_t* rank, int64_t shape[4], int64_t* offset, int64_t* nbytes,
                         char* err, int errlen) {
  MappedFile f;
  std::string e;
  std::vector<StTensor> ts;
  if (!path) return TMG_ERR_INVALID;
  if (!f.open(path, e) || !safetensors_parse(f.data(), f.size, ts, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  if (i < 0 || i >= int64_t(ts.size())) return TMG_ERR_INVALID;
  const StTensor& t = ts[size_t(i)];
  if (name && namelen > 0) std::snprintf(name, size_t(namelen), "%s", t.name.c_str());
  if (dtype) *dtype = t.dtype;
  if (rank) *rank = int32_t(t.shape.size());
  if (shape)
    for (int k = 0; k < 4; ++k) shape[k] = k < int(t.shape.size()) ? t.shape[k] : 0;
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  return TMG_OK;
}

int tmg_tmb_count(const char* path, tmg_config* cfg, int64_t* n, char* err, int errlen) {
  MappedFile f;
  std::string e;
  std::vector<TmbTensor> ts;
  if (!path || !n) return TMG_ERR_INVALID;
  if (!f.open(path, e) || !tmb_parse(f.data(), f.size, cfg, ts, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  *n = int64_t(ts.size());
  return TMG_OK;
}

int tmg_tmb_info(const char* path, int64_t i, char* name, int namelen, int64_t* offset,
                 int64_t* nbytes, char* err, int errlen) {
  MappedFile f;
  std::string e;
  std::vector<TmbTensor> ts;
  if (!path) return TMG_ERR_INVALID;
  if (!f.open(path, e) || !tmb_parse(f.data(), f.size, nullptr, ts, e)) {
    if (err && errlen > 0) std::snprintf(err, size_t(errlen), "%s", e.c_str());
    return TMG_ERR_IO;
  }
  if (i < 0 || i >= int64_t(ts.size())) return TMG_ERR_INVALID;
  const TmbTensor& t = ts[size_t(i)];
  if (name && namelen > 0) std::snprintf(name, size_t(namelen), "%s", t.name.c_str());
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  return TMG_OK;
}

int tmg_rng_uniforms(uint64_t seed, int64_t n, float* out) {
  if (n < 0 || (n > 0 && !out)) return TMG_ERR_INVALID;
  stdrng_uniforms(seed, n, out);
  return TMG_OK;
}

int tmg_create(int device, const tmg_config* cfg, tmg_ctx** out) {
  if (!out) return TMG_ERR_INVALID;
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n <= device || device < 0) {
    g_create_err = e != cudaSuccess ? std::string("tmg_create: ") + cudaGetErrorString(e)
                                    : std::string("tmg_create: no such device");
    return TMG_ERR_CUDA;
  }
  tmg_ctx* c = new tmg_ctx();
  c->device = device;
  const char* step = nullptr;
  cudaError_t ce = cudaSuccess;
  auto run = [&](const char* name, cudaError_t r) {
    if (!step && r != cudaSuccess) { step = name; ce = r; }
    return !step;
  };
  run("cudaSetDevice", cudaSetDevice(device)) &&
      run("stream", cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) &&
      run("sm count", cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device)) &&
      run("gemv_prepare", gemv_prepare()) && run("attn_prepare", attn_prepare()) &&
      run("gemm_tc_prepare", gemm_tc_prepare()) && run("prefill_prepare", prefill_prepare()) &&
      run("fused_prepare", fused_prepare()) && run("sample_prepare", sample_prepare()) &&
      run("gemv_i8_prepare", gemv_i8_prepare()) && run("attn_tma_prepare", attn_tma_prepare()) &&
      run("attn_prefill_tc_prepare", attn_prefill_tc_prepare()) &&
      run("error word", dalloc(c->allocs, &c->d_err, 4)) && run("error word", zero_sync(c, c->d_err, 16));
  if (step) {
    g_create_err = std::string("tmg_create: ") + step + ": " + cudaGetErrorString(ce);
    free_all(c->allocs);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return TMG_ERR_CUDA;
  }
  if (cfg) {
    c->cfg = *cfg;
    c->has_model = true;  // allocation happens at the first weight (after a TP init)
    c->h = 0;
  }
  *out = c;
  return TMG_OK;
}

static void kv_release(tmg_kv* kv);

int tmg_destroy(tmg_ctx* c) {
  if (!c) return TMG_ERR_INVALID;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (tmg_kv* kv : c->kvs) {  // caches the caller did not destroy first
    kv_release(kv);
    kv->ctx = nullptr;
  }
  free_all(c->allocs);
  for (void* p : {(void*)c->X, (void*)c->Xn, (void*)c->QKV, (void*)c->ATT, (void*)c->G,
                  (void*)c->U, (void*)c->d_tok, c->op_buf, (void*)c->sp_hi, (void*)c->sp_lo, c->pfa,
                  (void*)c->sa_hi, (void*)c->sa_lo,
                  (void*)c->dq, (void*)c->i8acc})
    if (p) cudaFree(p);
  if (c->pinned) cudaFreeHost(c->pinned);
  for (tmg_wmat* m : c->wmats) {
    cudaFree(m->w);
    m->w = nullptr;
    m->ctx = nullptr;  // the handle stays valid for tmg_wmat_free only
  }
  if (c->tp) tp_destroy(c->tp);
  cudaStreamDestroy(c->stream);
  delete c;
  return TMG_OK;
}

const char* tmg_last_error(const tmg_ctx* c) { return c ? c->err.c_str() : g_create_err.c_str(); }

static int ensure_alloc(tmg_ctx* c) {
  if (!c->has_model) return fail(c, TMG_ERR_INVALID, "context has no model config");
  if (c->h == 0) return alloc_model(c);
  return TMG_OK;
}

int tmg_set_tensor(tmg_ctx* c, const char* name, int32_t dtype, const void* host, int64_t numel) {
  if (!c || !name || !host || numel <= 0) return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  int rc = ensure_alloc(c);
  if (rc) return rc;
  return set_tensor(c, name, dtype, host, numel);
}

int tmg_load_safetensors(tmg_ctx* c, const char* path) {
  if (!c || !path) return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  int rc = ensure_alloc(c);
  if (rc) return rc;
  MappedFile f;
  std::string e;
  std::vector<StTensor> ts;
  if (!f.open(path, e) || !safetensors_parse(f.data(), f.size, ts, e))
    return fail(c, TMG_ERR_IO, e);
  for (const StTensor& t : ts) {
    int64_t numel = t.nbytes / (t.dtype == 0 ? 4 : 2);
    rc = set_tensor(c, t.name, t.dtype, f.data() + t.offset, numel);
    if (rc) return rc;
  }
  CK(cudaStreamSynchronize(c->stream), "load");
  return finalize(c);
}

// load_model_tmb, src/model.rs:108-179: the file's BF16 matrices go to HBM
// straight from the mapping, norms as f32; the embedding, stored as f32
// there, returns to its BF16 bits (exact for a file repacked from a BF16
// checkpoint; any other value is refused rather than rounded).
int tmg_load_tmb(tmg_ctx* c, const char* path) {
  if (!c || !path) return fail(c, TMG_ERR_INVALID, "bad argument");
  if (!c->has_model) return fail(c, TMG_ERR_INVALID, "context has no model config");
  cudaSetDevice(c->device);
  MappedFile f;
  std::string e;
  std::vector<TmbTensor> ts;
  tmg_config fc{};
  if (!f.open(path, e) || !tmb_parse(f.data(), f.size, &fc, ts, e)) return fail(c, TMG_ERR_IO, e);
  const tmg_config& cc = c->cfg;
  if (fc.hidden_size != cc.hidden_size || fc.num_hidden_layers != cc.num_hidden_layers ||
      fc.num_attention_heads != cc.num_attention_heads ||
      fc.num_key_value_heads != cc.num_key_value_heads || fc.head_dim != cc.head_dim ||
      fc.intermediate_size != cc.intermediate_size || fc.vocab_size != cc.vocab_size)
    return fail(c, TMG_ERR_INVALID, "TMB config does not match the context's model shape");
  int rc = ensure_alloc(c);
  if (rc) return rc;
  for (const TmbTensor& t : ts) {
    const uint8_t* p = f.data() + t.offset;
    const bool is_vec = t.name == "model.norm.weight" ||
                        t.name.find("layernorm.weight") != std::string::npos;
    if (t.name == "model.embed_tokens.weight") {
      if (t.nbytes % 4) return fail(c, TMG_ERR_INVALID, "TMB f32 tensor has non-multiple-of-4 byte length");
      const int64_t numel = t.nbytes / 4;
      if (numel != int64_t(c->V) * c->h)
        return fail(c, TMG_ERR_INVALID, "TMB embed size " + std::to_string(numel) +
                                            " != vocab*hidden " + std::to_string(int64_t(c->V) * c->h));
      std::vector<uint16_t> bits(static_cast<size_t>(numel));
      for (int64_t i = 0; i < numel; ++i) {
        uint32_t u;
        std::memcpy(&u, p + 4 * i, 4);
        if (u & 0xffffu)
          return fail(c, TMG_ERR_INVALID, "TMB embedding value " + std::to_string(i) +
                                              " is not a BF16 value (the device embedding is BF16)");
        bits[size_t(i)] = uint16_t(u >> 16);
      }
      rc = set_tensor(c, t.name, 1, bits.data(), numel);
      if (rc) return rc;
      CK(cudaStreamSynchronize(c->stream), "load");  // `bits` is freed on return
    } else if (is_vec) {
      if (t.nbytes % 4) return fail(c, TMG_ERR_INVALID, "TMB f32 tensor has non-multiple-of-4 byte length");
      rc = set_tensor(c, t.name, 0, p, t.nbytes / 4);
      if (rc) return rc;
    } else {
      if (t.nbytes % 2) return fail(c, TMG_ERR_INVALID, "TMB BF16 tensor has odd byte length");
      rc = set_tensor(c, t.name, 1, p, t.nbytes / 2);
      if (rc) return rc;
    }
  }
  CK(cudaStreamSynchronize(c->stream), "load");
  return finalize(c);
}

int tmg_finalize(tmg_ctx* c) {
  if (!c) return TMG_ERR_INVALID;
  cudaSetDevice(c->device);
  return finalize(c);
}

int64_t tmg_weight_bytes(const tmg_ctx* c) { return c ? c->weight_bytes : 0; }

int tmg_kv_create(tmg_ctx* c, int32_t n_streams, int64_t capacity, tmg_kv** out) {
  if (!c || !out || n_streams < 1 || n_streams > kMaxStreams || capacity < 1)
    return fail(c, TMG_ERR_INVALID, "bad KV cache shape (1..16 streams)");
  if (!c->finalized) return fail(c, TMG_ERR_INVALID, "weights not finalized");
  cudaSetDevice(c->device);
  tmg_kv* kv = new tmg_kv();
  kv->ctx = c;
  kv->M = n_streams;
  kv->cap = capacity;
  kv->kvd = c->nkv * c->d;
  kv->lens.assign(n_streams, 0);
  auto bail = [&](cudaError_t e) {
    free_all(kv->allocs);
    delete kv;
    return cuda_fail(c, e, "KV cache allocation");
  };
  cudaError_t e;
  for (int l = 0; l < c->L; ++l) {
    float *kp, *vp;
    if ((e = dalloc(kv->allocs, &kp, size_t(n_streams) * capacity * kv->kvd)) != cudaSuccess) return bail(e);
    if ((e = dalloc(kv->allocs, &vp, size_t(n_streams) * capacity * kv->kvd)) != cudaSuccess) return bail(e);
    kv->k.push_back(kp);
    kv->v.push_back(vp);
  }
  const int half = c->d / 2;
  if ((e = dalloc(kv->allocs, &kv->rope_cos, size_t(capacity) * half)) != cudaSuccess) return bail(e);
  if ((e = dalloc(kv->allocs, &kv->rope_sin, size_t(capacity) * half)) != cudaSuccess) return bail(e);
  std::vector<float> tc = rope_table(c->d, c->cfg.rope_theta, capacity, false);
  std::vector<float> ts = rope_table(c->d, c->cfg.rope_theta, capacity, true);
  if ((e = copy_sync(c, kv->rope_cos, tc.data(), tc.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return bail(e);
  if ((e = copy_sync(c, kv->rope_sin, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return bail(e);
  if ((e = dalloc(kv->allocs, &kv->d_state, 4 * kMaxStreams)) != cudaSuccess) return bail(e);
  if ((e = zero_sync(c, kv->d_state, 16 * kMaxStreams)) != cudaSuccess) return bail(e);
  kv->st.token = reinterpret_cast<uint32_t*>(kv->d_state);
  kv->st.pos = kv->d_state + kMaxStreams;
  kv->st.done = kv->d_state + 2 * kMaxStreams;
  kv->st.n_gen = kv->d_state + 3 * kMaxStreams;
  kv->st.gen = nullptr;
  kv->st.gen_cap = 0;
  kv->st.n_eos = 0;
  kv->nsplit = attn_decode_nsplit(c->nkv, n_streams, capacity, c->num_sms);
  if (c->fused_ok && n_streams == 1) {
    std::vector<FusedLayer> fl(c->L);
    for (int l = 0; l < c->L; ++l) {
      const Layer& Lw = c->layers[l];
      fl[l] = FusedLayer{Lw.wqkv, Lw.wo, Lw.wg, Lw.wu, Lw.wd, Lw.in_norm, Lw.post_norm, kv->k[l],
                         kv->v[l]};
    }
    if ((e = dalloc(kv->allocs, &kv->d_layers, size_t(c->L))) != cudaSuccess) return bail(e);
    if ((e = copy_sync(c, kv->d_layers, fl.data(), fl.size() * sizeof(FusedLayer),
                       cudaMemcpyHostToDevice)) != cudaSuccess)
      return bail(e);
    kv->nsplit_f = fused_nsplit(c->nq / c->nkv, c->d, capacity);
    const size_t pw = size_t(c->nkv) * kv->nsplit_f * (c->nq / c->nkv) * (c->d + 2);
    if ((e = dalloc(kv->allocs, &kv->part_ll, pw)) != cudaSuccess) return bail(e);
  }
  const int G = c->nq / c->nkv;
  if ((e = dalloc(kv->allocs, &kv->part, size_t(n_streams) * c->nkv * kv->nsplit * G * (c->d + 2))) != cudaSuccess) return bail(e);
  if ((e = dalloc(kv->allocs, &kv->att_ticket, size_t(n_streams) * c->nkv)) != cudaSuccess) return bail(e);
  if ((e = zero_sync(c, kv->att_ticket, size_t(n_streams) * c->nkv * 4)) != cudaSuccess) return bail(e);
  c->kvs.push_back(kv);
  *out = kv;
  return TMG_OK;
}

// Free a KV cache's device resources (its context is current and alive).
static void kv_release(tmg_kv* kv) {
  if (FusedGroup* g = kv->grp) {
    // the other ranks stop writing into this rank's memory first
    tp_barrier(g->comm, g->sync, kv->ctx->stream);
    cudaStreamSynchronize(kv->ctx->stream);
    for (void* p : g->opened) cudaIpcCloseMemHandle(p);
    if (g->d_kv_peer) cudaFree(g->d_kv_peer);
    if (g->am) cudaFree(g->am);
    if (g->sync) cudaFree(g->sync);
    tp_destroy(g->comm);
    delete g;
    kv->grp = nullptr;
  }
  cudaStreamSynchronize(kv->ctx->stream);
  if (kv->g_plain) cudaGraphExecDestroy(kv->g_plain);
  if (kv->g_dec) cudaGraphExecDestroy(kv->g_dec);
  if (kv->state_ev) cudaEventDestroy(kv->state_ev);
  if (kv->h_state) cudaFreeHost(kv->h_state);
  if (kv->d_gen) cudaFree(kv->d_gen);
  if (kv->d_uni) cudaFree(kv->d_uni);
  free_all(kv->allocs);
  kv->g_plain = kv->g_dec = nullptr;
  kv->state_ev = nullptr;
  kv->h_state = nullptr;
  kv->d_gen = nullptr;
  kv->d_uni = nullptr;
}

int tmg_kv_destroy(tmg_kv* kv) {
  if (!kv) return TMG_ERR_INVALID;
  if (kv->ctx) {  // null: released with its context already
    cudaSetDevice(kv->ctx->device);
    kv_release(kv);
    auto& v = kv->ctx->kvs;
    v.erase(std::remove(v.begin(), v.end(), kv), v.end());
  }
  delete kv;
  return TMG_OK;
}

int tmg_kv_len(const tmg_kv* kv, int32_t layer, int32_t stream, int64_t* out) {
  if (!kv || !kv->ctx || !out || stream < 0 || stream >= kv->M || layer < 0 || layer >= kv->ctx->L)
    return TMG_ERR_INVALID;
  *out = kv->lens[stream];
  return TMG_OK;
}

int tmg_kv_reset(tmg_kv* kv) {
  if (!kv || !kv->ctx) return TMG_ERR_INVALID;
  tmg_ctx* c = kv->ctx;
  cudaSetDevice(c->device);
  int rc = reset_state(c, kv);
  if (rc) return rc;
  CK(cudaStreamSynchronize(c->stream), "reset");
  return TMG_OK;
}

int tmg_kv_truncate(tmg_kv* kv, int32_t stream, int64_t len) {
  if (!kv || !kv->ctx || stream < 0 || stream >= kv->M || len < 0 || len > kv->lens[stream])
    return fail(kv ? kv->ctx : nullptr, TMG_ERR_INVALID, "bad truncate length");
  kv->lens[stream] = len;  // the device position is uploaded by the next forward
  return TMG_OK;
}

int tmg_kv_read(tmg_kv* kv, int32_t layer, int32_t stream, float* keys, float* values) {
  if (!kv || !kv->ctx || stream < 0 || stream >= kv->M || layer < 0 || layer >= kv->ctx->L)
    return TMG_ERR_INVALID;
  tmg_ctx* c = kv->ctx;
  cudaSetDevice(c->device);
  CK(cudaStreamSynchronize(c->stream), "kv read");
  const size_t n = size_t(kv->lens[stream]) * kv->kvd;
  const size_t off = size_t(stream) * kv->cap * kv->kvd;
  if (keys) CK(copy_sync(c, keys, kv->k[layer] + off, n * 4, cudaMemcpyDeviceToHost), "kv read");
  if (values)
    CK(copy_sync(c, values, kv->v[layer] + off, n * 4, cudaMemcpyDeviceToHost), "kv read");
  return TMG_OK;
}

// One f32 as Rust's `{:?}` writes it: the shortest decimal that reads back
// as the same f32, with ".0" on integral values.
std::string f32_debug(float v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "inf" : "-inf";
  char buf[48];
  for (int prec = 1; prec <= 9; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*g", prec, double(v));
    if (std::strtof(buf, nullptr) == v) break;
  }
  std::string t(buf);
  const size_t e = t.find('e');
  if (e != std::string::npos) {  // 1e-07 -> 1e-7
    std::string mant = t.substr(0, e), ex = t.substr(e + 1);
    const bool neg = !ex.empty() && ex[0] == '-';
    if (!ex.empty() && (ex[0] == '-' || ex[0] == '+')) ex = ex.substr(1);
    while (ex.size() > 1 && ex[0] == '0') ex = ex.substr(1);
    return mant + "e" + (neg ? "-" : "") + ex;
  }
  if (t.find('.') == std::string::npos) t += ".0";
  return t;
}

// The TMG_DEBUG lines of src/model.rs:406-409, 468-470, 480-482 for stream
// 0 of a per-token forward: "embed first8: [...]", "L<i> attn_out first8:
// [...]" (the residual stream after attention), "L<i> out first8: [...]".
cudaError_t debug_print(tmg_ctx* c, int layer, int what) {
  TMG_CUDA_TRY(cudaStreamSynchronize(c->stream));
  float v[8];
  const int n = std::min(8, c->h);
  TMG_CUDA_TRY(cudaMemcpy(v, c->x, size_t(n) * 4, cudaMemcpyDeviceToHost));
  std::string line = what == 0 ? std::string("embed first8: [")
                               : "L" + std::to_string(layer) +
                                     (what == 1 ? " attn_out first8: [" : " out first8: [");
  for (int i = 0; i < n; ++i) line += (i ? ", " : "") + f32_debug(v[i]);
  line += "]\n";
  std::fputs(line.c_str(), stderr);
  return cudaSuccess;
}

int tmg_forward_token(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens, float* logits) {
  if (!c || !kv || !tokens || kv->ctx != c) return fail(c, TMG_ERR_INVALID, "bad argument");
  if (!c->finalized) return fail(c, TMG_ERR_INVALID, "weights not finalized");
  cudaSetDevice(c->device);
  for (int m = 0; m < kv->M; ++m) {
    if (tokens[m] >= uint32_t(c->V)) return fail(c, TMG_ERR_INVALID, "token id out of range");
    if (kv->lens[m] + 1 > kv->cap) return fail(c, TMG_ERR_CAPACITY, "KV cache full");
  }
  // state: the tokens; not done; no recording; pos from the host mirror
  std::vector<int32_t> s(4 * kMaxStreams, 0);
  for (int m = 0; m < kv->M; ++m) {
    s[m] = int32_t(tokens[m]);
    s[kMaxStreams + m] = int32_t(kv->lens[m]);
  }
  CK(ensure_pinned(c, s.size() * 4), "pinned");
  CK(cudaStreamSynchronize(c->stream), "forward");
  std::memcpy(c->pinned, s.data(), s.size() * 4);
  CK(cudaMemcpyAsync(kv->d_state, c->pinned, s.size() * 4, cudaMemcpyHostToDevice, c->stream),
     "tokens");
  if (c->debug) {
    // eagerly, with the reference's debug lines between the sublayers
    const DebugHook hook = [c](int l, int what) { return debug_print(c, l, what); };
    nvtxRangePushA("forward_token");
    const cudaError_t ce = enqueue_forward(c, kv, kv->st, false, nullptr, nullptr, &hook);
    nvtxRangePop();
    CK(ce, "forward (TMG_DEBUG)");
  } else if (!kv->g_plain) {
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "capture");
    cudaError_t ce = enqueue_forward(c, kv, kv->st, false);
    cudaError_t ee = cudaStreamEndCapture(c->stream, &g);
    if (ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return cuda_fail(c, ce, "capture forward");
    }
    CK(ee, "capture");
    ce = cudaGraphInstantiate(&kv->g_plain, g, 0);
    cudaGraphDestroy(g);
    CK(ce, "instantiate");
  }
  if (!c->debug) {
    nvtxRangePushA("forward_token");
    const cudaError_t ce = cudaGraphLaunch(kv->g_plain, c->stream);
    nvtxRangePop();
    CK(ce, "forward");
  }
  if (logits)
    for (int m = 0; m < kv->M; ++m)
      CK(cudaMemcpyAsync(logits + size_t(m) * c->V, logits_row(c, m), size_t(c->V) * 4,
                         cudaMemcpyDeviceToHost, c->stream),
         "logits");
  for (int m = 0; m < kv->M; ++m) kv->lens[m] += 1;
  return sync_check(c, "forward");
}

int tmg_forward_seq(tmg_ctx* c, tmg_kv* kv, int32_t stream, const uint32_t* tokens, int64_t T,
                    float* logits) {
  if (!c || !kv || kv->ctx != c || stream < 0 || stream >= kv->M)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  if (T <= 0 || !tokens) return fail(c, TMG_ERR_INVALID, "empty prompt");
  if (!c->finalized) return fail(c, TMG_ERR_INVALID, "weights not finalized");
  if (kv->lens[stream] + T > kv->cap) return fail(c, TMG_ERR_CAPACITY, "KV cache full");
  for (int64_t i = 0; i < T; ++i)
    if (tokens[i] >= uint32_t(c->V)) return fail(c, TMG_ERR_INVALID, "token id out of range");
  cudaSetDevice(c->device);
  int rc = forward_seq(c, kv, stream, tokens, T, true);
  if (rc) return rc;
  if (logits)
    CK(cudaMemcpyAsync(logits, logits_row(c, stream), size_t(c->V) * 4, cudaMemcpyDeviceToHost,
                       c->stream),
       "logits");
  return sync_check(c, "forward_seq");
}

int tmg_generate(tmg_ctx* c, tmg_kv* kv, const uint32_t* prompt, int64_t T,
                 const tmg_gen_params* params, const float* uniforms, uint32_t* tokens_out,
                 int64_t* n_out, float* first_logits, double* prefill_secs, tmg_token_cb cb,
                 void* user) {
  if (!c || !kv || kv->ctx != c || !prompt || !params || !n_out ||
      (params->max_tokens > 0 && !tokens_out))
    return fail(c, TMG_ERR_INVALID, "bad argument");
  if (kv->M != 1) return fail(c, TMG_ERR_INVALID, "tmg_generate needs a 1-stream cache");
  cudaSetDevice(c->device);
  return run_generate(c, kv, prompt, T, params, uniforms, tokens_out, n_out, first_logits,
                      prefill_secs, cb, user);
}

int tmg_generate_batch(tmg_ctx* c, tmg_kv* kv, const uint32_t* prompts, int64_t T,
                       const tmg_gen_params* params, const float* uniforms, uint32_t* tokens_out,
                       int64_t* n_out) {
  if (!c || !kv || kv->ctx != c || !prompts || !params || !n_out)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  return run_generate(c, kv, prompts, T, params, uniforms, tokens_out, n_out, nullptr, nullptr,
                      nullptr, nullptr);
}

// Upload (token, pos = host length, done = 0, n_gen = 0) for every stream
// through a pinned staging block that is reused only after its previous
// copy has executed.
static int upload_state(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens) {
  if (!kv->h_state) {
    CK(cudaHostAlloc(reinterpret_cast<void**>(&kv->h_state), 16 * kMaxStreams,
                     cudaHostAllocDefault),
       "pinned");
    CK(cudaEventCreateWithFlags(&kv->state_ev, cudaEventDisableTiming), "event");
  } else {
    CK(cudaEventSynchronize(kv->state_ev), "state");
  }
  std::memset(kv->h_state, 0, 16 * kMaxStreams);
  for (int m = 0; m < kv->M; ++m) {
    kv->h_state[m] = int32_t(tokens[m]);
    kv->h_state[kMaxStreams + m] = int32_t(kv->lens[m]);
  }
  CK(cudaMemcpyAsync(kv->d_state, kv->h_state, 16 * kMaxStreams, cudaMemcpyHostToDevice,
                     c->stream),
     "state");
  CK(cudaEventRecord(kv->state_ev, c->stream), "state");
  return TMG_OK;
}

static int prepare_decode(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens, int64_t n_steps,
                          StreamState* st) {
  if (!c->finalized) return fail(c, TMG_ERR_INVALID, "weights not finalized");
  if (n_steps < 1 || n_steps > (int64_t(1) << 30)) return fail(c, TMG_ERR_INVALID, "bad n_steps");
  for (int m = 0; m < kv->M; ++m) {
    if (tokens[m] >= uint32_t(c->V)) return fail(c, TMG_ERR_INVALID, "token id out of range");
    if (kv->lens[m] + n_steps > kv->cap) return fail(c, TMG_ERR_CAPACITY, "KV cache full");
  }
  if (kv->gen_alloc < int64_t(kv->M) * n_steps) {
    CK(cudaStreamSynchronize(c->stream), "decode");
    if (kv->d_gen) cudaFree(kv->d_gen);
    kv->d_gen = nullptr;
    kv->gen_alloc = 0;
    CK(cudaMalloc(&kv->d_gen, size_t(kv->M) * n_steps * 4), "alloc");
    kv->gen_alloc = int64_t(kv->M) * n_steps;
    if (kv->g_dec) cudaGraphExecDestroy(kv->g_dec);
    kv->g_dec = nullptr;
  }
  int rc = upload_state(c, kv, tokens);
  if (rc) return rc;
  *st = kv->st;
  st->gen = kv->d_gen;
  st->gen_cap = int32_t(n_steps);
  st->n_eos = 0;
  return TMG_OK;
}

int tmg_decode(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens, int64_t n_steps, uint32_t* out) {
  if (!c || !kv || kv->ctx != c || !tokens) return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  NvtxRange range("decode");
  StreamState st;
  int rc = prepare_decode(c, kv, tokens, n_steps, &st);
  if (rc) return rc;
  if (!use_fused(c, kv) && (!kv->g_dec || kv->dec_cap != n_steps)) {
    if (kv->g_dec) cudaGraphExecDestroy(kv->g_dec);
    kv->g_dec = nullptr;
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "capture");
    cudaError_t ce = enqueue_forward(c, kv, st, true);
    cudaError_t ee = cudaStreamEndCapture(c->stream, &g);
    if (ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return cuda_fail(c, ce, "capture decode");
    }
    CK(ee, "capture");
    ce = cudaGraphInstantiate(&kv->g_dec, g, 0);
    cudaGraphDestroy(g);
    CK(ce, "instantiate");
    kv->dec_cap = n_steps;
  }
  if (use_fused(c, kv)) {
    CK(launch_fused(c, kv, st, n_steps), "fused decode");
  } else {
    for (int64_t i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(kv->g_dec, c->stream), "decode");
  }
  for (int m = 0; m < kv->M; ++m) kv->lens[m] += n_steps;
  if (out) {
    CK(cudaMemcpyAsync(out, kv->d_gen, size_t(kv->M) * n_steps * 4, cudaMemcpyDeviceToHost,
                       c->stream),
       "tokens");
    return sync_check(c, "decode");
  }
  return TMG_OK;
}

int tmg_sync(tmg_ctx* c) {
  if (!c) return TMG_ERR_INVALID;
  cudaSetDevice(c->device);
  if (!c->d_err) {
    CK(cudaStreamSynchronize(c->stream), "sync");
    return TMG_OK;
  }
  return sync_check(c, "sync");
}

void* tmg_stream(tmg_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

int tmg_profile_decode(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens, int64_t n_steps,
                       double* ms, int64_t* launches) {
  if (!c || !kv || kv->ctx != c || !tokens || !ms || !launches)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  StreamState st;
  int rc = prepare_decode(c, kv, tokens, n_steps, &st);
  if (rc) return rc;
  Prof prof;
  prof.s = c->stream;
  for (int64_t i = 0; i < n_steps; ++i) {
    cudaError_t e = enqueue_forward(c, kv, st, true, &prof);
    if (e != cudaSuccess) return cuda_fail(c, e, "profile");
  }
  CK(cudaStreamSynchronize(c->stream), "profile");
  for (int k = 0; k < kProfClasses; ++k) {
    ms[k] = 0.0;
    launches[k] = 0;
  }
  for (auto& m : prof.marks) {
    float t = 0.f;
    CK(cudaEventElapsedTime(&t, m.second.first, m.second.second), "elapsed");
    ms[m.first] += t;
    launches[m.first] += 1;
  }
  for (int m = 0; m < kv->M; ++m) kv->lens[m] += n_steps;
  return TMG_OK;
}

int tmg_trace_decode(tmg_ctx* c, tmg_kv* kv, const uint32_t* tokens, uint64_t* out,
                     int32_t* kinds, int32_t max_slots, int32_t* n_slots) {
  if (!c || !kv || kv->ctx != c || !tokens || !out || !kinds || !n_slots)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  StreamState st;
  int rc = prepare_decode(c, kv, tokens, 2, &st);
  if (rc) return rc;
  const int cap = 4096;
  unsigned long long* buf = nullptr;
  CK(cudaMalloc(&buf, size_t(cap) * 4 * 8), "trace");
  std::vector<unsigned long long> init(size_t(cap) * 4);
  for (int i = 0; i < cap; ++i) {
    init[size_t(i) * 4 + 0] = init[size_t(i) * 4 + 1] = ~0ull;
    init[size_t(i) * 4 + 2] = init[size_t(i) * 4 + 3] = 0ull;
  }
  TraceCtx tc;
  tc.buf = buf;
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    cudaError_t ce = enqueue_forward(c, kv, st, true, nullptr, &tc);
    e = cudaStreamEndCapture(c->stream, &g);
    if (ce != cudaSuccess) e = ce;
  }
  if (e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
  // one untraced-warm replay, then the traced one
  for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
    e = cudaMemcpyAsync(buf, init.data(), init.size() * 8, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaGraphLaunch(ex, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  }
  const int n = std::min<int>(tc.next, std::min<int>(cap, max_slots));
  if (e == cudaSuccess)
    e = cudaMemcpy(out, buf, size_t(n) * 4 * 8, cudaMemcpyDeviceToHost);
  if (ex) cudaGraphExecDestroy(ex);
  if (g) cudaGraphDestroy(g);
  cudaFree(buf);
  if (e != cudaSuccess) return cuda_fail(c, e, "trace");
  for (int i = 0; i < n; ++i) kinds[i] = tc.kinds[i];
  *n_slots = n;
  for (int m = 0; m < kv->M; ++m) kv->lens[m] += 2;
  return sync_check(c, "trace");
}

int tmg_trace_fused(tmg_ctx* c, tmg_kv* kv, uint32_t token, uint64_t* out, int64_t max_u64,
                    int32_t* n_ctas) {
  if (!c || !kv || kv->ctx != c || !out || !n_ctas) return fail(c, TMG_ERR_INVALID, "bad argument");
  if (!use_fused(c, kv)) return fail(c, TMG_ERR_INVALID, "the fused decode kernel does not apply");
  const size_t n = size_t(c->num_sms) * (size_t(c->L) * 5 + 1) * 12;
  if (max_u64 < int64_t(n)) return fail(c, TMG_ERR_INVALID, "trace buffer too small");
  cudaSetDevice(c->device);
  StreamState st;
  int rc = prepare_decode(c, kv, &token, 1, &st);
  if (rc) return rc;
  unsigned long long* buf = nullptr;
  CK(cudaMalloc(&buf, n * 8), "trace");
  cudaError_t e = cudaMemsetAsync(buf, 0, n * 8, c->stream);
  if (e == cudaSuccess) e = launch_fused(c, kv, st, 1, buf);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(out, buf, n * 8, cudaMemcpyDeviceToHost);
  cudaFree(buf);
  if (e != cudaSuccess) return cuda_fail(c, e, "trace");
  *n_ctas = c->num_sms;
  kv->lens[0] += 1;
  return sync_check(c, "trace");
}

int tmg_tp_shard(const tmg_config* cfg, const char* name, int32_t rank, int32_t world,
                 int64_t out[4]) {
  if (!cfg || !name || !out || world < 1 || rank < 0 || rank >= world) return TMG_ERR_INVALID;
  if (cfg->num_attention_heads % world || cfg->num_key_value_heads % world ||
      cfg->intermediate_size % world)
    return TMG_ERR_INVALID;
  int64_t full[2];
  return tp_shard_rect(*cfg, name, rank, world, out, full) ? TMG_OK : TMG_ERR_INVALID;
}

int tmg_tp_unique_id(uint8_t id[128]) { return tp_unique_id(id) == 0 ? TMG_OK : TMG_ERR_NCCL; }

int tmg_fused_group_init(tmg_ctx* c, tmg_kv* kv, const uint8_t id[128], int32_t rank,
                         int32_t world) {
  if (!c || !kv || kv->ctx != c || !id || world < 2 || world > kMaxGroupRanks || rank < 0 ||
      rank >= world)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  if (c->world != 1 || !use_fused(c, kv) || kv->grp)
    return fail(c, TMG_ERR_INVALID,
                "a fused group needs a single-GPU context with full weights whose shape the fused "
                "decode kernel takes, and a 1-stream cache not yet in a group");
  cudaSetDevice(c->device);
  const int ctas = fused_group_ctas(c->h, c->nq, c->nkv, c->d, c->I, c->V_l, c->num_sms, world);
  if (ctas < 1)
    return fail(c, TMG_ERR_INVALID, "the model's phases have too few row groups for this many GPUs");
  std::string e;
  TpComm* comm = tp_create(id, rank, world, e);
  if (!comm) return fail(c, TMG_ERR_NCCL, e);
  FusedGroup* g = new FusedGroup();
  g->comm = comm;
  g->rank = rank;
  g->world = world;
  g->ctas = ctas;
  float* dbuf = nullptr;
  auto bail = [&](int code, const std::string& m) {
    for (void* p : g->opened) cudaIpcCloseMemHandle(p);
    if (g->d_kv_peer) cudaFree(g->d_kv_peer);
    if (g->am) cudaFree(g->am);
    if (g->sync) cudaFree(g->sync);
    if (dbuf) cudaFree(dbuf);
    tp_destroy(g->comm);
    delete g;
    return fail(c, code, "tmg_fused_group_init: " + m);
  };
  cudaError_t ce = cudaMalloc(&g->am, size_t(world) * ctas * sizeof(unsigned long long));
  if (ce == cudaSuccess) ce = cudaMalloc(&g->sync, sizeof(float));
  if (ce == cudaSuccess) ce = zero_sync(c, g->sync, sizeof(float));
  if (ce != cudaSuccess) return bail(TMG_ERR_CUDA, cudaGetErrorString(ce));
  // what every rank publishes: its GPU, shape, and the IPC handles of its
  // exchange words, partials, barrier words, argmax table and KV caches
  struct Head {
    char bus[32];
    int32_t h, L, ctas, pad;
    int64_t cap;
  };
  const int nh = 4 + 2 * c->L;
  const size_t blob = (sizeof(Head) + size_t(nh) * sizeof(cudaIpcMemHandle_t) + 15) / 16 * 16;
  std::vector<char> mine(blob, 0), all(blob * world, 0);
  Head hd{};
  hd.h = c->h;
  hd.L = c->L;
  hd.ctas = ctas;
  hd.cap = kv->cap;
  ce = cudaDeviceGetPCIBusId(hd.bus, sizeof(hd.bus), c->device);
  std::memcpy(mine.data(), &hd, sizeof(hd));
  std::vector<void*> bases = {c->ll, kv->part_ll, c->bar, g->am};
  for (int l = 0; l < c->L; ++l) {
    bases.push_back(kv->k[l]);
    bases.push_back(kv->v[l]);
  }
  for (int i = 0; i < nh && ce == cudaSuccess; ++i) {
    cudaIpcMemHandle_t hh;
    ce = cudaIpcGetMemHandle(&hh, bases[i]);
    std::memcpy(mine.data() + sizeof(Head) + size_t(i) * sizeof(hh), &hh, sizeof(hh));
  }
  if (ce != cudaSuccess) return bail(TMG_ERR_CUDA, cudaGetErrorString(ce));
  const int64_t nf = int64_t(blob / 4);
  ce = cudaMalloc(&dbuf, blob * (world + 1));
  if (ce == cudaSuccess) ce = copy_sync(c, dbuf, mine.data(), blob, cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = tp_allgather_rows(comm, dbuf, nf, dbuf + nf, nf * world, 1, c->stream);
  if (ce == cudaSuccess) ce = copy_sync(c, all.data(), dbuf + nf, blob * world, cudaMemcpyDeviceToHost);
  cudaFree(dbuf);
  dbuf = nullptr;
  if (ce != cudaSuccess) return bail(TMG_ERR_NCCL, std::string("handle exchange: ") + cudaGetErrorString(ce));
  // one distinct GPU per rank, and the same model shape and cache everywhere
  // (ranks that wait on one another must run at the same time)
  for (int r = 0; r < world; ++r) {
    Head o;
    std::memcpy(&o, all.data() + size_t(r) * blob, sizeof(o));
    if (o.h != hd.h || o.L != hd.L || o.ctas != hd.ctas || o.cap != hd.cap)
      return bail(TMG_ERR_INVALID, "the ranks' model shapes or cache capacities differ");
    for (int q = 0; q < r; ++q)
      if (std::strncmp(o.bus, all.data() + size_t(q) * blob, sizeof(o.bus)) == 0)
        return bail(TMG_ERR_INVALID, "two ranks share one GPU");
  }
  std::vector<float*> kvp(size_t(world) * c->L * 2);
  for (int r = 0; r < world; ++r) {
    std::vector<void*> p(nh);
    for (int i = 0; i < nh; ++i) {
      if (r == rank) {
        p[i] = bases[i];
        continue;
      }
      cudaIpcMemHandle_t hh;
      std::memcpy(&hh, all.data() + size_t(r) * blob + sizeof(Head) + size_t(i) * sizeof(hh),
                  sizeof(hh));
      ce = cudaIpcOpenMemHandle(&p[i], hh, cudaIpcMemLazyEnablePeerAccess);
      if (ce != cudaSuccess) return bail(TMG_ERR_CUDA, std::string("peer mapping: ") + cudaGetErrorString(ce));
      g->opened.push_back(p[i]);
    }
    g->ll_peer[r] = static_cast<unsigned long long*>(p[0]);
    g->part_peer[r] = static_cast<unsigned long long*>(p[1]);
    g->bar_peer[r] = static_cast<unsigned int*>(p[2]);
    g->am_peer[r] = static_cast<unsigned long long*>(p[3]);
    for (int l = 0; l < c->L; ++l) {
      kvp[(size_t(r) * c->L + l) * 2] = static_cast<float*>(p[4 + 2 * l]);
      kvp[(size_t(r) * c->L + l) * 2 + 1] = static_cast<float*>(p[5 + 2 * l]);
    }
  }
  ce = cudaMalloc(&g->d_kv_peer, kvp.size() * sizeof(float*));
  if (ce == cudaSuccess)
    ce = copy_sync(c, g->d_kv_peer, kvp.data(), kvp.size() * sizeof(float*), cudaMemcpyHostToDevice);
  if (ce == cudaSuccess) ce = tp_barrier(comm, g->sync, c->stream);  // every rank mapped
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->stream);
  if (ce != cudaSuccess) return bail(TMG_ERR_CUDA, cudaGetErrorString(ce));
  kv->grp = g;
  return TMG_OK;
}

int tmg_tp_init(tmg_ctx* c, const uint8_t id[128], int32_t rank, int32_t world) {
  if (!c || !id || world < 1 || rank < 0 || rank >= world) return fail(c, TMG_ERR_INVALID, "bad argument");
  if (c->h != 0) return fail(c, TMG_ERR_INVALID, "tmg_tp_init must precede the weight upload");
  cudaSetDevice(c->device);
  std::string e;
  c->tp = tp_create(id, rank, world, e);
  if (!c->tp) return fail(c, TMG_ERR_NCCL, e);
  // one allreduce and one allgather before any stream capture: NCCL sets up
  // its connections on a communicator's first collectives
  float* w = nullptr;
  cudaError_t ce = cudaMalloc(&w, sizeof(float) * (1 + world));
  if (ce == cudaSuccess) ce = cudaMemsetAsync(w, 0, sizeof(float) * (1 + world), c->stream);
  if (ce == cudaSuccess) ce = tp_allreduce_sum(c->tp, w, 1, c->stream);
  if (ce == cudaSuccess) ce = tp_allgather_rows(c->tp, w, 1, w + 1, world, 1, c->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(c->stream);
  if (w) cudaFree(w);
  if (ce != cudaSuccess) {
    tp_destroy(c->tp);
    c->tp = nullptr;
    return fail(c, TMG_ERR_NCCL, std::string("tmg_tp_init: first collectives failed: ") +
                                     cudaGetErrorString(ce));
  }
  c->rank = rank;
  c->world = world;
  return TMG_OK;
}

// --- op level ---------------------------------------------------------------
int tmg_op_gemv_bf16(tmg_ctx* c, const float* x, const uint16_t* w, int64_t N, int64_t K,
                     int32_t M, float* y) {
  if (!c || !x || !w || !y || N <= 0 || K <= 0 || M < 1 || M > kMaxStreams)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  GemvArgs a;
  a.w = w;
  a.x = x;
  a.y = y;
  a.ldy = N;
  a.N = N;
  a.K = int(K);
  a.M = M;
  CK(launch_gemv(a, PRO_NONE, EPI_STORE, c->stream, false, c->num_sms), "gemv");
  CK(cudaStreamSynchronize(c->stream), "gemv");
  return TMG_OK;
}

int tmg_op_gemm_bf16(tmg_ctx* c, const float* x, const uint16_t* w, int64_t N, int64_t K,
                     int64_t T, float* y) {
  if (!c || !x || !w || !y || N <= 0 || K <= 0 || T <= 0)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(gemm(c, x, w, T, N, K, y, N, false), "gemm");
  CK(cudaStreamSynchronize(c->stream), "gemm");
  return TMG_OK;
}

int tmg_wmat_upload_bf16(tmg_ctx* c, const uint16_t* host, int64_t rows, int64_t cols,
                         tmg_wmat** out) {
  if (!c || !host || !out || rows <= 0 || cols <= 0 || rows > INT32_MAX || cols > INT32_MAX)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  *out = nullptr;
  cudaSetDevice(c->device);
  tmg_wmat* m = new tmg_wmat();
  m->ctx = c;
  m->rows = rows;
  m->cols = cols;
  const size_t bytes = size_t(rows) * size_t(cols) * 2;
  cudaError_t e = cudaMalloc(&m->w, bytes);
  if (e == cudaSuccess) e = copy_sync(c, m->w, host, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (m->w) cudaFree(m->w);
    delete m;
    return cuda_fail(c, e, "tmg_wmat_upload_bf16");
  }
  c->wmats.push_back(m);
  *out = m;
  return TMG_OK;
}

int tmg_wmat_free(tmg_wmat* m) {
  if (!m) return TMG_ERR_INVALID;
  tmg_ctx* c = m->ctx;
  if (!c) {  // released with its context already
    delete m;
    return TMG_OK;
  }
  auto it = std::find(c->wmats.begin(), c->wmats.end(), m);
  if (it == c->wmats.end()) return fail(c, TMG_ERR_INVALID, "unknown WMat handle");
  c->wmats.erase(it);
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  cudaFree(m->w);
  delete m;
  return TMG_OK;
}

int tmg_wmat_shape(const tmg_wmat* m, int64_t* rows, int64_t* cols) {
  if (!m || !rows || !cols) return TMG_ERR_INVALID;
  *rows = m->rows;
  *cols = m->cols;
  return TMG_OK;
}

int tmg_op_gemv_wmat(tmg_ctx* c, const float* x, const tmg_wmat* w, int32_t M, float* y) {
  if (!c || !w || w->ctx != c) return fail(c, TMG_ERR_INVALID, "bad WMat handle");
  return tmg_op_gemv_bf16(c, x, w->w, w->rows, w->cols, M, y);
}

int tmg_op_gemm_wmat(tmg_ctx* c, const float* x, const tmg_wmat* w, int64_t T, float* y) {
  if (!c || !w || w->ctx != c) return fail(c, TMG_ERR_INVALID, "bad WMat handle");
  return tmg_op_gemm_bf16(c, x, w->w, w->rows, w->cols, T, y);
}

int tmg_op_quantize_i8(tmg_ctx* c, const uint16_t* w, int64_t N, int64_t K, int8_t* q,
                       float* scales) {
  if (!c || !w || !q || !scales || N <= 0 || K <= 0 || K > INT32_MAX)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(launch_quantize_w_i8(w, N, int(K), q, scales, c->stream), "quantize");
  CK(cudaStreamSynchronize(c->stream), "quantize");
  return TMG_OK;
}

int tmg_op_gemv_i8(tmg_ctx* c, const float* x, const int8_t* q, const float* scales, int64_t N,
                   int64_t K, int32_t M, float* y) {
  if (!c || !x || !q || !scales || !y || N <= 0 || K <= 0 || K % 16 || K > 16384 || M < 1 ||
      M > kMaxStreams)
    return fail(c, TMG_ERR_INVALID, "bad argument (K % 16 == 0, K <= 16384, 1 <= M <= 16)");
  cudaSetDevice(c->device);
  GemvI8Args a;
  a.q = q;
  a.scales = scales;
  a.x = x;
  a.y = y;
  a.ldy = N;
  a.N = N;
  a.K = int(K);
  a.M = M;
  if (!gemv_i8_tma_ok(a.K, M)) {
    CK(ensure_op(c, size_t(M) * K + 256 + 4 * kMaxStreams), "op scratch");
    a.xs = static_cast<float*>(c->op_buf);
    a.xq = static_cast<int8_t*>(c->op_buf) + 256;
  }
  CK(launch_gemv_i8(a, EPI_STORE, c->stream, false, c->num_sms), "gemv_i8");
  CK(cudaStreamSynchronize(c->stream), "gemv_i8");
  return TMG_OK;
}

int tmg_op_rmsnorm(tmg_ctx* c, const float* x, const float* w, float eps, int64_t n, int64_t rows,
                   int32_t mode, float* out) {
  if (!c || !x || !w || !out || n <= 0 || rows <= 0 || (mode != 0 && mode != 1))
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(launch_rmsnorm(x, w, eps, n, rows, mode, out, c->stream), "rmsnorm");
  CK(cudaStreamSynchronize(c->stream), "rmsnorm");
  return TMG_OK;
}

int tmg_op_rope(tmg_ctx* c, float* x, int64_t rows, int32_t n_heads, int32_t head_dim,
                int64_t pos0, float theta) {
  if (!c || !x || rows <= 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2 || pos0 < 0)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  const int64_t np = pos0 + rows;
  std::vector<float> tc = rope_table(head_dim, theta, np, false);
  std::vector<float> ts = rope_table(head_dim, theta, np, true);
  const size_t bytes = tc.size() * 4;
  CK(ensure_op(c, 2 * bytes + 64), "op scratch");
  float* dc = static_cast<float*>(c->op_buf);
  float* ds = dc + tc.size();
  CK(copy_sync(c, dc, tc.data(), bytes, cudaMemcpyHostToDevice), "rope table");
  CK(copy_sync(c, ds, ts.data(), bytes, cudaMemcpyHostToDevice), "rope table");
  CK(launch_rope_rows(x, int64_t(n_heads) * head_dim, rows, n_heads, head_dim, dc, ds, pos0,
                      c->stream),
     "rope");
  CK(cudaStreamSynchronize(c->stream), "rope");
  return TMG_OK;
}

int tmg_op_swiglu(tmg_ctx* c, const float* gate, const float* up, int64_t n, float* out) {
  if (!c || !gate || !up || !out || n <= 0) return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(launch_swiglu(gate, up, n, out, c->stream), "swiglu");
  CK(cudaStreamSynchronize(c->stream), "swiglu");
  return TMG_OK;
}

int tmg_op_attn_decode(tmg_ctx* c, const float* q, const float* keys, const float* values,
                       int64_t n_ctx, int32_t n_q, int32_t n_kv, int32_t head_dim, float* out) {
  if (!c || !q || !keys || !values || !out || n_ctx <= 0 || n_q <= 0 || n_kv <= 0 ||
      n_q % n_kv || head_dim <= 0 || head_dim % 8)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  const int G = n_q / n_kv;
  const int nsplit = attn_decode_nsplit(n_kv, 1, n_ctx, c->num_sms);
  std::string why;
  if (!attn_decode_shape_ok(n_q, n_kv, head_dim, n_ctx, nsplit, &why))
    return fail(c, TMG_ERR_INVALID, "tmg_op_attn_decode: " + why);
  // op scratch: the partials, then one ticket per kv head, then the
  // position word (each region 256-byte aligned)
  const size_t part_b = (size_t(n_kv) * nsplit * G * (head_dim + 2) * 4 + 255) & ~size_t(255);
  const size_t tick_b = (size_t(n_kv) * 4 + 255) & ~size_t(255);
  CK(ensure_op(c, part_b + tick_b + 256), "op scratch");
  AttnDecodeArgs a;
  a.qkv = q;
  a.qkv_ld = 0;
  a.kc = const_cast<float*>(keys);
  a.vc = const_cast<float*>(values);
  a.cap = n_ctx;
  a.out = out;
  a.part = static_cast<float*>(c->op_buf);
  a.ticket = reinterpret_cast<unsigned int*>(static_cast<char*>(c->op_buf) + part_b);
  int32_t* posv = reinterpret_cast<int32_t*>(static_cast<char*>(c->op_buf) + part_b + tick_b);
  const int32_t pv = int32_t(n_ctx - 1);
  CK(cudaMemsetAsync(a.ticket, 0, size_t(n_kv) * 4, c->stream), "memset");
  CK(cudaMemcpyAsync(posv, &pv, 4, cudaMemcpyHostToDevice, c->stream), "pos");
  a.pos_override = posv;
  a.nq = n_q;
  a.nkv = n_kv;
  a.d = head_dim;
  a.nsplit = nsplit;
  a.M = 1;
  a.scale = 1.0f / sqrtf(float(head_dim));
  CK(launch_attn_decode(a, c->stream, false), "attention");
  CK(cudaStreamSynchronize(c->stream), "attention");
  return TMG_OK;
}

int tmg_op_attn_decode_noalloc(tmg_ctx* c, const float* q, const float* keys, const float* values,
                               int64_t n_ctx, int32_t n_q, int32_t n_kv, int32_t head_dim,
                               float* out) {
  if (!c || !q || !keys || !values || !out || n_ctx <= 0 || n_q <= 0 || n_kv <= 0 ||
      n_q % n_kv || head_dim <= 0 || head_dim % 8)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  std::string why;
  const int r = attn_decode_noalloc(c->device, c->num_sms, c->stream, q, keys, values, n_ctx, n_q,
                                    n_kv, head_dim, out, &why);
  if (r == 2) return fail(c, TMG_ERR_CAPACITY, "tmg_op_attn_decode_noalloc: " + why);
  if (r == 1) return fail(c, TMG_ERR_INVALID, "tmg_op_attn_decode_noalloc: " + why);
  if (r != 0) return fail(c, TMG_ERR_CUDA, "tmg_op_attn_decode_noalloc: " + why);
  return TMG_OK;
}

int tmg_op_attn_prefill(tmg_ctx* c, const float* q, const float* keys, const float* values,
                        int64_t T, int64_t start_pos, int32_t n_q, int32_t n_kv, int32_t head_dim,
                        float* out) {
  if (!c || !q || !keys || !values || !out || T <= 0 || start_pos < 0 || n_q <= 0 ||
      n_kv <= 0 || n_q % n_kv)
    return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(prefill_attention(c, q, int64_t(n_q) * head_dim, keys, values, T, start_pos,
                       1.0f / sqrtf(float(head_dim)), out, int64_t(n_q) * head_dim, n_q, n_kv,
                       head_dim),
     "attention");
  return sync_check(c, "tmg_op_attn_prefill");
}

int tmg_op_argmax(tmg_ctx* c, const float* logits, int64_t V, int32_t rows, uint32_t* out) {
  if (!c || !logits || !out || V <= 0 || rows <= 0) return fail(c, TMG_ERR_INVALID, "bad argument");
  cudaSetDevice(c->device);
  CK(launch_argmax_rows(logits, V, rows, out, c->stream), "argmax");
  CK(cudaStreamSynchronize(c->stream), "argmax");
  return TMG_OK;
}

int tmg_op_sample(tmg_ctx* c, float* logits, int64_t V, int32_t rows, const uint32_t* generated,
                  int64_t n_gen, float temperature, int64_t top_k, float top_p, float penalty,
                  const float* uniforms, uint32_t* next, uint32_t* cand_ids, float* cand_probs,
                  int32_t* cutoff) {
  if (!c || !logits || !next || V <= 0 || rows < 1 || rows > kMaxStreams || n_gen < 0 ||
      (n_gen > 0 && !generated))
    return fail(c, TMG_ERR_INVALID, "bad argument");
  if (temperature > 0.f && (top_k < 1 || top_k > kMaxTopK || top_k >= V))
    return fail(c, TMG_ERR_INVALID, "device sampling needs 1 <= top_k <= 64");
  if (temperature > 0.f && !uniforms) return fail(c, TMG_ERR_INVALID, "uniforms required");
  cudaSetDevice(c->device);
  const int ns = sample_slices(V, rows, c->num_sms);
  const size_t part_b = size_t(rows) * ns * kMaxTopK * 8;
  CK(ensure_op(c, part_b + 4096), "op scratch");
  SampleArgs a;
  a.logits = logits;
  a.V = V;
  a.M = rows;
  a.generated = generated;
  a.gen_ld = n_gen;
  a.n_gen_fixed = n_gen;
  a.temperature = temperature;
  a.top_k = int(top_k);
  a.top_p = top_p;
  a.penalty = penalty;
  a.uniforms = uniforms;
  a.uni_ld = 1;
  a.next = next;
  a.cand_ids = cand_ids;
  a.cand_probs = cand_probs;
  a.cutoff = cutoff;
  a.part = static_cast<unsigned long long*>(c->op_buf);
  a.ticket = reinterpret_cast<unsigned int*>(static_cast<char*>(c->op_buf) + part_b);
  a.err = reinterpret_cast<int32_t*>(static_cast<char*>(c->op_buf) + part_b + 1024);
  CK(cudaMemsetAsync(a.ticket, 0, 2048, c->stream), "memset");
  CK(launch_sample(a, c->stream, false, c->num_sms), "sample");
  int32_t errw = 0;
  CK(cudaMemcpyAsync(&errw, a.err, 4, cudaMemcpyDeviceToHost, c->stream), "err");
  CK(cudaStreamSynchronize(c->stream), "sample");
  if (errw) return fail(c, TMG_ERR_NAN, "NaN logits reached the sampler");
  return TMG_OK;
}

}  // extern "C"
