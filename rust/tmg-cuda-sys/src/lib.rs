//! Raw declarations of the C ABI in `include/tmg_cuda.h` (libtmg_cuda.so),
//! for TinyMiniGo's Rust engine.  `Model` keeps a `*mut TmgCtx`, `KvCache` a
//! `*mut TmgKv`, and a `WMat` that lives on the GPU a `*mut TmgWmat`; the
//! engine's `forward_token` / `forward_seq` / `generate` (src/model.rs:392,
//! 494, 614) call `tmg_forward_token` / `tmg_forward_seq` / `tmg_generate`.
//! Every call returns 0 or a negative `TMG_ERR_*`; `check` turns that into a
//! `Result` carrying `tmg_last_error`'s message (the reference's functions
//! return `anyhow::Result`).
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_void, CStr};

pub const TMG_OK: i32 = 0;
pub const TMG_ERR_INVALID: i32 = -1;
pub const TMG_ERR_CUDA: i32 = -2;
pub const TMG_ERR_IO: i32 = -3;
pub const TMG_ERR_CAPACITY: i32 = -4;
pub const TMG_ERR_NAN: i32 = -5;
pub const TMG_ERR_TIMEOUT: i32 = -6;
pub const TMG_ERR_NCCL: i32 = -7;
pub const TMG_MAX_EOS: usize = 8;

/// ModelConfig (src/config.rs:6-20).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct TmgConfig {
    pub hidden_size: i32,
    pub num_hidden_layers: i32,
    pub num_attention_heads: i32,
    pub num_key_value_heads: i32,
    pub head_dim: i32,
    pub intermediate_size: i32,
    pub vocab_size: i32,
    pub rms_norm_eps: f32,
    pub rope_theta: f32,
    pub bos_token_id: u32,
    pub n_eos: i32,
    pub eos_token_ids: [u32; TMG_MAX_EOS],
}

/// GenParams (src/model.rs:597-604).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct TmgGenParams {
    pub max_tokens: i64,
    pub temperature: f32,
    pub top_k: i64,
    pub top_p: f32,
    pub repetition_penalty: f32,
    pub seed: u64,
}

#[repr(C)]
pub struct TmgCtx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct TmgKv {
    _p: [u8; 0],
}
#[repr(C)]
pub struct TmgWmat {
    _p: [u8; 0],
}

/// Called once per generated token inside `tmg_generate`; non-zero stops.
pub type TmgTokenCb = Option<unsafe extern "C" fn(token: u32, user: *mut c_void) -> i32>;

#[link(name = "tmg_cuda")]
unsafe extern "C" {
    // host-only
    pub fn tmg_config_load(path: *const c_char, out: *mut TmgConfig, err: *mut c_char, errlen: i32) -> i32;
    pub fn tmg_config_parse(json: *const c_char, out: *mut TmgConfig, err: *mut c_char, errlen: i32) -> i32;
    pub fn tmg_safetensors_count(path: *const c_char, n: *mut i64, err: *mut c_char, errlen: i32) -> i32;
    pub fn tmg_safetensors_info(path: *const c_char, i: i64, name: *mut c_char, namelen: i32,
                                dtype: *mut i32, rank: *mut i32, shape: *mut i64, offset: *mut i64,
                                nbytes: *mut i64, err: *mut c_char, errlen: i32) -> i32;
    pub fn tmg_tmb_count(path: *const c_char, cfg: *mut TmgConfig, n: *mut i64, err: *mut c_char,
                         errlen: i32) -> i32;
    pub fn tmg_tmb_info(path: *const c_char, i: i64, name: *mut c_char, namelen: i32, offset: *mut i64,
                        nbytes: *mut i64, err: *mut c_char, errlen: i32) -> i32;
    pub fn tmg_f16_to_f32(h: u16) -> f32;
    pub fn tmg_version() -> *const c_char;

    // context and weights
    pub fn tmg_create(device: i32, cfg: *const TmgConfig, out: *mut *mut TmgCtx) -> i32;
    pub fn tmg_destroy(ctx: *mut TmgCtx) -> i32;
    pub fn tmg_last_error(ctx: *const TmgCtx) -> *const c_char;
    pub fn tmg_load_safetensors(ctx: *mut TmgCtx, path: *const c_char) -> i32;
    pub fn tmg_load_tmb(ctx: *mut TmgCtx, path: *const c_char) -> i32;
    pub fn tmg_set_tensor(ctx: *mut TmgCtx, name: *const c_char, dtype: i32, host: *const c_void,
                          numel: i64) -> i32;
    pub fn tmg_finalize(ctx: *mut TmgCtx) -> i32;
    pub fn tmg_weight_bytes(ctx: *const TmgCtx) -> i64;

    // KV cache
    pub fn tmg_kv_create(ctx: *mut TmgCtx, n_streams: i32, capacity: i64, out: *mut *mut TmgKv) -> i32;
    pub fn tmg_kv_destroy(kv: *mut TmgKv) -> i32;
    pub fn tmg_kv_len(kv: *const TmgKv, layer: i32, stream: i32, out: *mut i64) -> i32;
    pub fn tmg_kv_reset(kv: *mut TmgKv) -> i32;
    pub fn tmg_kv_truncate(kv: *mut TmgKv, stream: i32, len: i64) -> i32;
    pub fn tmg_kv_read(kv: *mut TmgKv, layer: i32, stream: i32, keys: *mut f32, values: *mut f32) -> i32;

    // forward passes and generation
    pub fn tmg_forward_token(ctx: *mut TmgCtx, kv: *mut TmgKv, tokens: *const u32, logits: *mut f32) -> i32;
    pub fn tmg_forward_seq(ctx: *mut TmgCtx, kv: *mut TmgKv, stream: i32, tokens: *const u32, t: i64,
                           logits: *mut f32) -> i32;
    pub fn tmg_generate(ctx: *mut TmgCtx, kv: *mut TmgKv, prompt: *const u32, t: i64,
                        params: *const TmgGenParams, uniforms: *const f32, tokens_out: *mut u32,
                        n_out: *mut i64, first_logits: *mut f32, prefill_secs: *mut f64,
                        cb: TmgTokenCb, user: *mut c_void) -> i32;
    pub fn tmg_generate_batch(ctx: *mut TmgCtx, kv: *mut TmgKv, prompts: *const u32, t: i64,
                              params: *const TmgGenParams, uniforms: *const f32,
                              tokens_out: *mut u32, n_out: *mut i64) -> i32;
    pub fn tmg_rng_uniforms(seed: u64, n: i64, out: *mut f32) -> i32;
    pub fn tmg_decode(ctx: *mut TmgCtx, kv: *mut TmgKv, tokens: *const u32, n_steps: i64, out: *mut u32) -> i32;
    pub fn tmg_sync(ctx: *mut TmgCtx) -> i32;
    pub fn tmg_stream(ctx: *mut TmgCtx) -> *mut c_void;
    pub fn tmg_profile_decode(ctx: *mut TmgCtx, kv: *mut TmgKv, tokens: *const u32, n_steps: i64,
                              ms: *mut f64, launches: *mut i64) -> i32;
    pub fn tmg_trace_decode(ctx: *mut TmgCtx, kv: *mut TmgKv, tokens: *const u32, out: *mut u64,
                            kinds: *mut i32, max_slots: i32, n_slots: *mut i32) -> i32;
    pub fn tmg_trace_fused(ctx: *mut TmgCtx, kv: *mut TmgKv, token: u32, out: *mut u64, max_u64: i64,
                           n_ctas: *mut i32) -> i32;

    // tensor parallel
    pub fn tmg_tp_unique_id(id: *mut u8) -> i32;
    pub fn tmg_tp_init(ctx: *mut TmgCtx, id: *const u8, rank: i32, world: i32) -> i32;
    pub fn tmg_tp_shard(cfg: *const TmgConfig, name: *const c_char, rank: i32, world: i32,
                        out: *mut i64) -> i32;
    pub fn tmg_fused_group_init(ctx: *mut TmgCtx, kv: *mut TmgKv, id: *const u8, rank: i32,
                                world: i32) -> i32;

    // WMat handles and op-level entry points (device pointers)
    pub fn tmg_wmat_upload_bf16(ctx: *mut TmgCtx, host: *const u16, rows: i64, cols: i64,
                                out: *mut *mut TmgWmat) -> i32;
    pub fn tmg_wmat_free(w: *mut TmgWmat) -> i32;
    pub fn tmg_wmat_shape(w: *const TmgWmat, rows: *mut i64, cols: *mut i64) -> i32;
    pub fn tmg_op_gemv_wmat(ctx: *mut TmgCtx, x: *const f32, w: *const TmgWmat, m: i32, y: *mut f32) -> i32;
    pub fn tmg_op_gemm_wmat(ctx: *mut TmgCtx, x: *const f32, w: *const TmgWmat, t: i64, y: *mut f32) -> i32;
    pub fn tmg_op_quantize_i8(ctx: *mut TmgCtx, w: *const u16, n: i64, k: i64, q: *mut i8,
                              scales: *mut f32) -> i32;
    pub fn tmg_op_gemv_i8(ctx: *mut TmgCtx, x: *const f32, q: *const i8, scales: *const f32, n: i64,
                          k: i64, m: i32, y: *mut f32) -> i32;
    pub fn tmg_op_gemv_bf16(ctx: *mut TmgCtx, x: *const f32, w: *const u16, n: i64, k: i64, m: i32,
                            y: *mut f32) -> i32;
    pub fn tmg_op_gemm_bf16(ctx: *mut TmgCtx, x: *const f32, w: *const u16, n: i64, k: i64, t: i64,
                            y: *mut f32) -> i32;
    pub fn tmg_op_rmsnorm(ctx: *mut TmgCtx, x: *const f32, w: *const f32, eps: f32, n: i64, rows: i64,
                          mode: i32, out: *mut f32) -> i32;
    pub fn tmg_op_rope(ctx: *mut TmgCtx, x: *mut f32, rows: i64, n_heads: i32, head_dim: i32, pos0: i64,
                       theta: f32) -> i32;
    pub fn tmg_op_swiglu(ctx: *mut TmgCtx, gate: *const f32, up: *const f32, n: i64, out: *mut f32) -> i32;
    pub fn tmg_op_attn_decode(ctx: *mut TmgCtx, q: *const f32, keys: *const f32, values: *const f32,
                              n_ctx: i64, n_q: i32, n_kv: i32, head_dim: i32, out: *mut f32) -> i32;
    pub fn tmg_op_attn_decode_noalloc(ctx: *mut TmgCtx, q: *const f32, keys: *const f32,
                                      values: *const f32, n_ctx: i64, n_q: i32, n_kv: i32,
                                      head_dim: i32, out: *mut f32) -> i32;
    pub fn tmg_op_attn_prefill(ctx: *mut TmgCtx, q: *const f32, keys: *const f32, values: *const f32,
                               t: i64, start_pos: i64, n_q: i32, n_kv: i32, head_dim: i32,
                               out: *mut f32) -> i32;
    pub fn tmg_op_argmax(ctx: *mut TmgCtx, logits: *const f32, v: i64, rows: i32, out: *mut u32) -> i32;
    pub fn tmg_op_sample(ctx: *mut TmgCtx, logits: *mut f32, v: i64, rows: i32, generated: *const u32,
                         n_gen: i64, temperature: f32, top_k: i64, top_p: f32, penalty: f32,
                         uniforms: *const f32, next: *mut u32, cand_ids: *mut u32,
                         cand_probs: *mut f32, cutoff: *mut i32) -> i32;
}

/// A failed call: its status and `tmg_last_error`'s message.
#[derive(Debug, Clone)]
pub struct TmgError {
    pub code: i32,
    pub message: String,
}

impl std::fmt::Display for TmgError {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "tmg error {}: {}", self.code, self.message)
    }
}

impl std::error::Error for TmgError {}

/// `Ok(())` for TMG_OK, else the status with the context's last message
/// (`ctx` may be null: the message of the last failed `tmg_create`).
pub fn check(rc: i32, ctx: *const TmgCtx) -> Result<(), TmgError> {
    if rc == TMG_OK {
        return Ok(());
    }
    // SAFETY: tmg_last_error returns a NUL-terminated string owned by the
    // library (valid until the next call on that context).
    let message = unsafe {
        let p = tmg_last_error(ctx);
        if p.is_null() { String::new() } else { CStr::from_ptr(p).to_string_lossy().into_owned() }
    };
    Err(TmgError { code: rc, message })
}
