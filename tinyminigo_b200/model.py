"""The reference's engine API (HanzCEO/TinyMiniGo src/model.rs, src/config.rs)
over the B200 library: same names, argument meaning and error behaviour.

    cfg   = ModelConfig.load(path)                 # src/config.rs:112-172
    model = Model.load("dir/model.safetensors")     # src/model.rs:384-389
    cache = model.new_cache()                       # KvCache::new + set_kv_dim
    logits = model.prefill(prompt, cache)           # src/model.rs:494-499
    logits = model.forward_token(tok, cache)        # src/model.rs:392-491
    out = generate(model, prompt, GenParams(...), on_token)  # 614-663

Differences forced by the device: a KvCache has a fixed capacity (HBM is
preallocated; the reference grows a Vec), and may hold up to 16 streams
that one forward_token advances together.  All math runs in the CUDA
library; logits come back to the host only when asked for.
"""
from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import TmgError, check, lib


def _ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


# ---------------------------------------------------------------------------
# ModelConfig, src/config.rs:6-185
# ---------------------------------------------------------------------------
@dataclass
class ModelConfig:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rms_norm_eps: float
    rope_theta: float
    vocab_size: int
    eos_token_ids: list = field(default_factory=list)
    bos_token_id: int = 0

    @staticmethod
    def _from_c(c: _lib.Config) -> "ModelConfig":
        return ModelConfig(c.hidden_size, c.num_hidden_layers, c.num_attention_heads,
                           c.num_key_value_heads, c.head_dim, c.intermediate_size,
                           float(c.rms_norm_eps), float(c.rope_theta), c.vocab_size,
                           [int(c.eos_token_ids[i]) for i in range(c.n_eos)], int(c.bos_token_id))

    def to_c(self) -> _lib.Config:
        c = _lib.Config()
        c.hidden_size = self.hidden_size
        c.num_hidden_layers = self.num_hidden_layers
        c.num_attention_heads = self.num_attention_heads
        c.num_key_value_heads = self.num_key_value_heads
        c.head_dim = self.head_dim
        c.intermediate_size = self.intermediate_size
        c.vocab_size = self.vocab_size
        c.rms_norm_eps = self.rms_norm_eps
        c.rope_theta = self.rope_theta
        c.bos_token_id = self.bos_token_id
        if len(self.eos_token_ids) > 8:
            raise ValueError("at most 8 eos_token_id values")
        c.n_eos = len(self.eos_token_ids)
        for i, e in enumerate(self.eos_token_ids):
            c.eos_token_ids[i] = e
        return c

    @staticmethod
    def from_json(text: str) -> "ModelConfig":
        c = _lib.Config()
        err = ctypes.create_string_buffer(512)
        rc = lib().tmg_config_parse(text.encode(), ctypes.byref(c), err, 512)
        if rc != 0:
            raise TmgError(rc, err.value.decode())
        return ModelConfig._from_c(c)

    @staticmethod
    def load(path) -> "ModelConfig":
        c = _lib.Config()
        err = ctypes.create_string_buffer(512)
        rc = lib().tmg_config_load(str(path).encode(), ctypes.byref(c), err, 512)
        if rc != 0:
            raise TmgError(rc, err.value.decode())
        return ModelConfig._from_c(c)

    @staticmethod
    def config_path_for_model(model_path) -> Path | None:
        p = Path(model_path).parent / "config.json"
        return p if p.exists() else None

    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim


def safetensors_index(path) -> list:
    """(name, dtype, shape, offset, nbytes) of every tensor in a file."""
    n = ctypes.c_int64(0)
    err = ctypes.create_string_buffer(512)
    rc = lib().tmg_safetensors_count(str(path).encode(), ctypes.byref(n), err, 512)
    if rc != 0:
        raise TmgError(rc, err.value.decode())
    out = []
    for i in range(n.value):
        name = ctypes.create_string_buffer(512)
        dt, rank = ctypes.c_int32(), ctypes.c_int32()
        shape = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_int64(), ctypes.c_int64()
        rc = lib().tmg_safetensors_info(str(path).encode(), i, name, 512, ctypes.byref(dt),
                                        ctypes.byref(rank), shape, ctypes.byref(off),
                                        ctypes.byref(nb), err, 512)
        if rc != 0:
            raise TmgError(rc, err.value.decode())
        out.append((name.value.decode(), ["F32", "BF16", "F16"][dt.value],
                    [shape[k] for k in range(rank.value)], off.value, nb.value))
    return out


def f16_to_f32(h: int) -> float:
    return float(lib().tmg_f16_to_f32(h))


def rng_uniforms(seed: int, n: int) -> np.ndarray:
    """The reference's StdRng::seed_from_u64(seed) StandardUniform f32 draws."""
    out = np.zeros(n, np.float32)
    check(lib().tmg_rng_uniforms(seed, n, _ptr(out)))
    return out


# ---------------------------------------------------------------------------
# Model + KvCache
# ---------------------------------------------------------------------------
class Model:
    """Weights resident in HBM on one GPU (or one tensor-parallel rank)."""

    def __init__(self, config: ModelConfig, device: int = 0, tp=None):
        self.config = config
        self.device = device
        h = ctypes.c_void_p()
        cc = config.to_c()
        self._c = cc
        check(lib().tmg_create(device, ctypes.byref(cc), ctypes.byref(h)), None, "tmg_create")
        self._h = h
        self._gen_cache = None
        self._caches = []
        if tp is not None:
            uid, rank, world = tp
            buf = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(uid))
            check(lib().tmg_tp_init(self._h, buf, rank, world), self._h, "tmg_tp_init")

    # --- construction ---
    @staticmethod
    def load(model_path, device: int = 0, tp=None) -> "Model":
        """Model::load (src/model.rs:384-389): a TMB1 repack (recognised by its
        magic, load_model, src/model.rs:90-96) carries its own config; a
        safetensors file needs config.json beside it.  Weights go to HBM once."""
        p = Path(model_path)
        if not p.exists():
            raise FileNotFoundError(f"model file not found: {p}")
        from . import tmb

        if tmb.is_tmb(p):
            cfg, _ = tmb.index(p)
            m = Model(cfg, device, tp)
            try:
                check(lib().tmg_load_tmb(m._h, str(p).encode()), m._h, "load")
            except TmgError:
                m.close()
                raise
            return m
        cp = ModelConfig.config_path_for_model(p)
        if cp is None:
            raise FileNotFoundError(f"config.json not found next to {p}")
        m = Model(ModelConfig.load(cp), device, tp)
        check(lib().tmg_load_safetensors(m._h, str(p).encode()), m._h, "load")
        return m

    @staticmethod
    def from_tensors(config: ModelConfig, tensors: dict, device: int = 0, tp=None) -> "Model":
        """Build from in-memory tensors keyed by HF name: BF16 bit patterns as
        uint16 arrays (matrices must be BF16), norms as f32 or BF16.
        `tensors` is a dict or an iterable of (name, array) pairs (each array
        may be dropped once it has been uploaded)."""
        m = Model(config, device, tp)
        for name, a in (tensors.items() if hasattr(tensors, "items") else tensors):
            a = np.ascontiguousarray(a)
            dtype = 1 if a.dtype == np.uint16 else 0
            if dtype == 0:
                a = np.ascontiguousarray(a, np.float32)
            check(lib().tmg_set_tensor(m._h, name.encode(), dtype, _ptr(a), a.size), m._h, name)
        check(lib().tmg_finalize(m._h), m._h, "finalize")
        return m

    def close(self):
        """Free the device state; caches made from this model are closed
        first (a cache cannot outlive its model's context)."""
        if getattr(self, "_gen_cache", None) is not None:
            self._gen_cache.close()
            self._gen_cache = None
        for ref in getattr(self, "_caches", []):
            c = ref()
            if c is not None:
                c.close()
        self._caches = []
        if getattr(self, "_h", None):
            lib().tmg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self) -> int:
        return int(lib().tmg_weight_bytes(self._h))

    def last_error(self) -> str:
        return lib().tmg_last_error(self._h).decode()

    def new_cache(self, capacity: int = 4096, n_streams: int = 1) -> "KvCache":
        return KvCache(self, capacity, n_streams)

    # --- forwards ---
    def forward_token(self, token, cache: "KvCache", want_logits: bool = True):
        """Model::forward_token: one token per stream of the cache; returns
        logits [vocab] (or [n_streams, vocab])."""
        toks = np.ascontiguousarray(np.atleast_1d(np.asarray(token, np.uint32)))
        if toks.size != cache.n_streams:
            raise ValueError(f"need {cache.n_streams} tokens, got {toks.size}")
        V = self.config.vocab_size
        out = np.zeros((cache.n_streams, V), np.float32) if want_logits else None
        check(lib().tmg_forward_token(self._h, cache._h, _ptr(toks),
                                      _ptr(out) if out is not None else None), self._h,
              "forward_token")
        if out is None:
            return None
        return out[0] if cache.n_streams == 1 else out

    def forward_seq(self, tokens, cache: "KvCache", stream: int = 0, want_logits: bool = True):
        """Model::forward_seq: tokens appended from the stream's current
        position; returns the last token's logits."""
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        out = np.zeros(self.config.vocab_size, np.float32) if want_logits else None
        check(lib().tmg_forward_seq(self._h, cache._h, stream, _ptr(t), t.size,
                                    _ptr(out) if out is not None else None), self._h,
              "forward_seq")
        return out

    def prefill(self, tokens, cache: "KvCache", stream: int = 0):
        """Model::prefill: forward_seq that rejects an empty prompt."""
        if len(tokens) == 0:
            raise ValueError("empty prompt")
        return self.forward_seq(tokens, cache, stream)

    def decode(self, tokens, cache: "KvCache", n_steps: int, wait: bool = True):
        """n_steps greedy steps (forward_token + argmax) per stream on the
        device, starting from tokens[m]; returns [n_streams, n_steps] ids
        (or None when wait=False: the work stays queued, see sync())."""
        t = np.ascontiguousarray(np.atleast_1d(np.asarray(tokens, np.uint32)))
        out = np.zeros((cache.n_streams, n_steps), np.uint32) if wait else None
        check(lib().tmg_decode(self._h, cache._h, _ptr(t), n_steps,
                               _ptr(out) if out is not None else None), self._h, "decode")
        return out

    def sync(self):
        check(lib().tmg_sync(self._h), self._h, "sync")

    def stream_handle(self) -> int:
        """The library's cudaStream_t (for CUDA events on the launching stream)."""
        return int(lib().tmg_stream(self._h) or 0)

    def fused_group(self, cache: "KvCache", uid: bytes, rank: int, world: int):
        """Join `cache` to a greedy decode spread over `world` GPUs (one
        process each, every rank holding the full weights): tmg_decode on it
        then deals the fused kernel's work over all ranks' SMs."""
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(uid))
        check(lib().tmg_fused_group_init(self._h, cache._h, buf, rank, world), self._h,
              "tmg_fused_group_init")

    def profile_decode(self, tokens, cache: "KvCache", n_steps: int) -> dict:
        """Per-kernel-class device time (ms) and launches of n_steps greedy
        steps launched one kernel at a time with CUDA events between them."""
        t = np.ascontiguousarray(np.atleast_1d(np.asarray(tokens, np.uint32)))
        ms = np.zeros(8, np.float64)
        n = np.zeros(8, np.int64)
        check(lib().tmg_profile_decode(self._h, cache._h, _ptr(t), n_steps, _ptr(ms), _ptr(n)),
              self._h, "profile_decode")
        names = ["qkv_gemv", "attn_decode", "o_gemv", "gateup_gemv", "down_gemv", "lm_head",
                 "allreduce", "allgather_step_end"]
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(names)}

    def trace_decode(self, tokens, cache: "KvCache") -> list:
        """Device timeline of one captured greedy step: per kernel (kind,
        first start, first past wait, last past wait, last end) in ns."""
        t = np.ascontiguousarray(np.atleast_1d(np.asarray(tokens, np.uint32)))
        cap = 1024
        out = np.zeros((cap, 4), np.uint64)
        kinds = np.zeros(cap, np.int32)
        n = ctypes.c_int32(0)
        check(lib().tmg_trace_decode(self._h, cache._h, _ptr(t), _ptr(out), _ptr(kinds), cap,
                                     ctypes.byref(n)), self._h, "trace_decode")
        names = ["qkv_gemv", "attn_decode", "o_gemv", "gateup_gemv", "down_gemv", "lm_head"]
        return [(names[kinds[i]], *[int(v) for v in out[i]]) for i in range(n.value)]

    def trace_fused(self, token: int, cache: "KvCache", n_ctas_max: int = 1024) -> np.ndarray:
        """One greedy step of the fused decode kernel with timestamps:
        [n_ctas, 5 L + 1, 12] per CTA and phase (see tmg_trace_fused)."""
        nph = self.config.num_hidden_layers * 5 + 1
        out = np.zeros(n_ctas_max * nph * 12, np.uint64)
        n = ctypes.c_int32(0)
        check(lib().tmg_trace_fused(self._h, cache._h, int(token), _ptr(out), out.size,
                                    ctypes.byref(n)), self._h, "trace_fused")
        return out[: n.value * nph * 12].reshape(n.value, nph, 12)


class KvCache:
    """KvCache (src/model.rs:250-332) on the device: per layer and stream an
    f32 [capacity, n_kv * head_dim] row buffer."""

    def __init__(self, model: Model, capacity: int, n_streams: int = 1):
        self.model = model
        self.capacity = capacity
        self.n_streams = n_streams
        h = ctypes.c_void_p()
        check(lib().tmg_kv_create(model._h, n_streams, capacity, ctypes.byref(h)), model._h,
              "kv_create")
        self._h = h
        if not hasattr(model, "_caches"):
            model._caches = []
        model._caches.append(weakref.ref(self))

    def close(self):
        if getattr(self, "_h", None):
            lib().tmg_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def kv_dim(self) -> int:
        return self.model.config.kv_dim()

    def len(self, layer: int = 0, stream: int = 0) -> int:
        n = ctypes.c_int64()
        check(lib().tmg_kv_len(self._h, layer, stream, ctypes.byref(n)), self.model._h, "kv_len")
        return n.value

    def total_len(self, stream: int = 0) -> int:
        return self.len(0, stream)

    def reset(self):
        check(lib().tmg_kv_reset(self._h), self.model._h, "kv_reset")

    def truncate(self, length: int, stream: int = 0):
        """Keep the first `length` positions of a stream."""
        check(lib().tmg_kv_truncate(self._h, stream, length), self.model._h, "kv_truncate")

    def keys_flat(self, layer: int, stream: int = 0) -> np.ndarray:
        k = np.zeros((self.len(layer, stream), self.kv_dim()), np.float32)
        check(lib().tmg_kv_read(self._h, layer, stream, _ptr(k), None), self.model._h, "kv_read")
        return k

    def values_flat(self, layer: int, stream: int = 0) -> np.ndarray:
        v = np.zeros((self.len(layer, stream), self.kv_dim()), np.float32)
        check(lib().tmg_kv_read(self._h, layer, stream, None, _ptr(v)), self.model._h, "kv_read")
        return v


# ---------------------------------------------------------------------------
# generate, src/model.rs:597-663
# ---------------------------------------------------------------------------
@dataclass
class GenParams:
    max_tokens: int = 256
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    seed: int = 42

    def to_c(self) -> _lib.GenParamsC:
        return _lib.GenParamsC(self.max_tokens, self.temperature, self.top_k, self.top_p,
                               self.repetition_penalty, self.seed)


@dataclass
class GenOutput:
    tokens: list
    logits_first_step: np.ndarray
    prefill_secs: float


def _gen_cache(model: Model, need: int, n_streams: int) -> KvCache:
    c = model._gen_cache
    if c is None or c.capacity < need or c.n_streams != n_streams:
        if c is not None:
            c.close()
        c = KvCache(model, need, n_streams)
        model._gen_cache = c
    return c


def generate(model: Model, prompt_tokens, params: GenParams, on_token=None,
             uniforms=None) -> GenOutput:
    """generate(): prefill, then the greedy / sampled token loop, all on the
    device; on_token(id) is called for every generated token, in order.
    `uniforms` overrides the draws of the reference's StdRng(seed)."""
    p = np.ascontiguousarray(np.asarray(prompt_tokens, np.uint32))
    if p.size == 0:
        raise ValueError("empty prompt")
    cache = _gen_cache(model, p.size + max(params.max_tokens, 0) + 1, 1)
    maxt = max(params.max_tokens, 0)
    out = np.zeros(max(maxt, 1), np.uint32)
    first = np.zeros(model.config.vocab_size, np.float32)
    n = ctypes.c_int64(0)
    ps = ctypes.c_double(0)
    cp = params.to_c()
    u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
    if on_token is not None:
        def _cb(tok, _user):
            on_token(int(tok))
            return 0
        cb = _lib.TOKEN_CB(_cb)
    else:
        cb = _lib.TOKEN_CB()
    check(lib().tmg_generate(model._h, cache._h, _ptr(p), p.size, ctypes.byref(cp),
                             None if u is None else _ptr(u), _ptr(out), ctypes.byref(n),
                             _ptr(first), ctypes.byref(ps), cb, None), model._h, "generate")
    return GenOutput([int(t) for t in out[:n.value]], first, ps.value)


def generate_batch(model: Model, prompts, params: list, uniforms=None, cache: KvCache = None):
    """generate() for up to 16 equal-length prompts at once (weights streamed
    once per step for all of them).  Returns a list of token lists."""
    P = np.ascontiguousarray(np.asarray(prompts, np.uint32))
    M, T = P.shape
    if len(params) != M:
        raise ValueError("one GenParams per stream")
    maxt = params[0].max_tokens
    if cache is None:
        cache = _gen_cache(model, T + maxt + 1, M)
    arr = (_lib.GenParamsC * M)(*[q.to_c() for q in params])
    out = np.zeros((M, max(maxt, 1)), np.uint32)
    n = np.zeros(M, np.int64)
    u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
    check(lib().tmg_generate_batch(model._h, cache._h, _ptr(P), T, arr,
                                   None if u is None else _ptr(u), _ptr(out),
                                   n.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))), model._h,
          "generate_batch")
    return [[int(t) for t in out[m, :n[m]]] for m in range(M)]
