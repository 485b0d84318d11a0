"""TEST INFRASTRUCTURE ONLY — ctypes bindings of the CPU oracle (ref_cpu.cpp).

The oracle restates the reference engine's CPU arithmetic (HanzCEO/TinyMiniGo
src/tensor.rs and src/model.rs) in C++.  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg use this module, always as the checker or the
timed CPU baseline, never as the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "ref_cpu.cpp"
LIB = HERE / "build" / "libtmg_oracle.so"

CXXFLAGS = [
    "-O2", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-fast-math",
    "-fPIC", "-std=c++17", "-pthread", "-shared",
]


def build(force: bool = False) -> Path:
    """Compile ref_cpu.cpp into build/libtmg_oracle.so (g++, seconds)."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run(["g++", *CXXFLAGS, "-o", str(tmp), str(SRC)], check=True)
    os.replace(tmp, LIB)
    return LIB


class OrcConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("num_hidden_layers", ctypes.c_int32),
        ("num_attention_heads", ctypes.c_int32),
        ("num_key_value_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
    ]


_lib = None

_F = ctypes.POINTER(ctypes.c_float)
_U16 = ctypes.POINTER(ctypes.c_uint16)
_U32 = ctypes.POINTER(ctypes.c_uint32)
_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_I8 = ctypes.POINTER(ctypes.c_int8)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        sig = {
            "orc_set_num_threads": (None, [_I64]),
            "orc_num_threads": (_I64, []),
            "orc_dot_bf16": (ctypes.c_float, [_F, _U16, _I64]),
            "orc_dot_f32": (ctypes.c_float, [_F, _F, _I64]),
            "orc_matmul_w_bf16": (None, [_F, _U16, _I64, _I64, _F]),
            "orc_matmul_w_f32": (None, [_F, _F, _I64, _I64, _F]),
            "orc_matmul_batch_w_bf16": (None, [_F, _U16, _I64, _I64, _I64, _F]),
            "orc_quantize_i8": (None, [_F, _I64, _I64, _I8, _F]),
            "orc_quantize_row_i8": (ctypes.c_float, [_F, _I64, _I8]),
            "orc_dot_i8": (ctypes.c_int32, [_I8, _I8, _I64]),
            "orc_matmul_w_i8": (None, [_F, _I8, _F, _I64, _I64, _F]),
            "orc_matmul_batch_w_i8": (None, [_F, _I8, _F, _I64, _I64, _I64, _F]),
            "orc_model_set_i8": (None, [_P, ctypes.c_int]),
            "orc_rms_norm_into": (None, [_F, _F, ctypes.c_float, _I64, _F]),
            "orc_rms_norm_batch": (None, [_F, _F, ctypes.c_float, _I64, _I64]),
            "orc_rope_rotate": (None, [_F, _I64, _I64, ctypes.c_float]),
            "orc_rope_table_rotate": (None, [_F, _I64, _I64, _I64, ctypes.c_float]),
            "orc_rope_tables": (None, [_I64, ctypes.c_float, _I64, _F, _F]),
            "orc_softmax": (None, [_F, _I64, _F]),
            "orc_argmax": (_I64, [_F, _I64]),
            "orc_silu": (ctypes.c_float, [ctypes.c_float]),
            "orc_attention_batch": (None, [_F, _F, _F, _I64, _I64, _I64, _I64, _I64, _F]),
            "orc_apply_repetition_penalty": (None, [_F, _U32, _I64, ctypes.c_float]),
            "orc_sample_select": (_I64, [_F, _I64, ctypes.c_float, _I64, ctypes.c_float, _U32, _F,
                                         ctypes.POINTER(ctypes.c_int64)]),
            "orc_sample": (_I64, [_F, _I64, ctypes.c_float, _I64, ctypes.c_float, ctypes.c_float]),
            "orc_stdrng_uniforms": (None, [ctypes.c_uint64, _I64, _F]),
            "orc_model_new": (_P, [ctypes.POINTER(OrcConfig)]),
            "orc_model_free": (None, [_P]),
            "orc_model_set": (ctypes.c_int, [_P, ctypes.c_char_p, _P, ctypes.c_int, _I64]),
            "orc_kv_new": (_P, [_P]),
            "orc_kv_free": (None, [_P]),
            "orc_kv_len": (_I64, [_P, _I64]),
            "orc_kv_reset": (None, [_P]),
            "orc_kv_read": (None, [_P, _I64, _F, _F]),
            "orc_kv_load": (None, [_P, _I64, _F, _F, _I64]),
            "orc_forward_token": (ctypes.c_int, [_P, _P, ctypes.c_uint32, _F]),
            "orc_forward_seq": (ctypes.c_int, [_P, _P, _U32, _I64, _F]),
            "orc_generate": (_I64, [_P, _P, _U32, _I64, _I64, ctypes.c_float, _I64, ctypes.c_float,
                                    ctypes.c_float, ctypes.c_uint64, _F, _U32, _I64, _U32, _F,
                                    ctypes.POINTER(ctypes.c_double),
                                    ctypes.POINTER(ctypes.c_double)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def _u16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_U16)


def _u32(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_U32)


# --- op level ---------------------------------------------------------------

def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(n)


def num_threads() -> int:
    return int(lib().orc_num_threads())


def _i8(a: np.ndarray):
    assert a.dtype == np.int8 and a.flags.c_contiguous
    return a.ctypes.data_as(_I8)


def quantize_i8(w: np.ndarray):
    """WMat::quantize_i8 (src/tensor.rs:282-297) of an f32 [out, in] matrix:
    (int8 rows, per-row f32 scales)."""
    w = np.ascontiguousarray(w, np.float32)
    out, inn = w.shape
    q = np.zeros((out, inn), np.int8)
    sc = np.zeros(out, np.float32)
    lib().orc_quantize_i8(_f(w), out, inn, _i8(q), _f(sc))
    return q, sc


def quantize_row_i8(x: np.ndarray):
    """quantize_row_i8 (src/tensor.rs:128-141): (int8 values, scale)."""
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = lib().orc_quantize_row_i8(_f(x), x.size, _i8(q))
    return q, np.float32(s)


def dot_i8(a: np.ndarray, b: np.ndarray) -> int:
    return int(lib().orc_dot_i8(_i8(np.ascontiguousarray(a, np.int8)),
                                _i8(np.ascontiguousarray(b, np.int8)), a.size))


def matmul_w_i8(x: np.ndarray, q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """The decode GEMV of an I8 matrix (src/tensor.rs:341-357)."""
    out, inn = q.shape
    y = np.zeros(out, np.float32)
    lib().orc_matmul_w_i8(_f(np.ascontiguousarray(x, np.float32)), _i8(np.ascontiguousarray(q)),
                          _f(np.ascontiguousarray(scales, np.float32)), out, inn, _f(y))
    return y


def matmul_batch_w_i8(x: np.ndarray, q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """The prefill GEMM of an I8 matrix (src/tensor.rs:573-592, 799-858)."""
    out, inn = q.shape
    T = x.shape[0]
    y = np.zeros((T, out), np.float32)
    lib().orc_matmul_batch_w_i8(_f(np.ascontiguousarray(x, np.float32)),
                                _i8(np.ascontiguousarray(q)),
                                _f(np.ascontiguousarray(scales, np.float32)), out, inn, T, _f(y))
    return y


def matmul_w(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """y = x @ W^T for one activation row; W is [out, in] (bf16 bits or f32)."""
    out, inn = w.shape
    y = np.zeros(out, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    if w.dtype == np.uint16:
        lib().orc_matmul_w_bf16(_f(x), _u16(w), out, inn, _f(y))
    else:
        lib().orc_matmul_w_f32(_f(x), _f(np.ascontiguousarray(w, np.float32)), out, inn, _f(y))
    return y


def matmul_batch_w(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    T, inn = x.shape
    out = w.shape[0]
    y = np.zeros((T, out), np.float32)
    lib().orc_matmul_batch_w_bf16(_f(np.ascontiguousarray(x, np.float32)), _u16(w), out, inn, T, _f(y))
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_rms_norm_into(_f(x), _f(np.ascontiguousarray(w, np.float32)), eps, x.size, _f(out))
    return out


def rms_norm_batch(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    lib().orc_rms_norm_batch(_f(x), _f(np.ascontiguousarray(w, np.float32)), eps, x.shape[-1],
                             x.size // x.shape[-1])
    return x


def rope_rotate(v: np.ndarray, pos: int, theta: float) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    lib().orc_rope_rotate(_f(v), v.size, pos, theta)
    return v


def rope_table_rotate(v: np.ndarray, n_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    lib().orc_rope_table_rotate(_f(v), n_heads, head_dim, pos, theta)
    return v


def rope_tables(head_dim: int, theta: float, n_pos: int):
    c = np.zeros((n_pos, head_dim // 2), np.float32)
    s = np.zeros_like(c)
    lib().orc_rope_tables(head_dim, theta, n_pos, _f(c), _f(s))
    return c, s


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_softmax(_f(x), x.size, _f(out))
    return out


def argmax(x: np.ndarray) -> int:
    return int(lib().orc_argmax(_f(np.ascontiguousarray(x, np.float32)), x.size))


def silu(g: float) -> float:
    return float(lib().orc_silu(g))


def attention_batch(q, keys, vals, n_q, n_kv, head_dim, start_pos) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    T = q.size // (n_q * head_dim)
    out = np.zeros((T, n_q * head_dim), np.float32)
    lib().orc_attention_batch(_f(q), _f(np.ascontiguousarray(keys, np.float32)),
                              _f(np.ascontiguousarray(vals, np.float32)), T, n_q, n_kv, head_dim,
                              start_pos, _f(out))
    return out


def apply_repetition_penalty(logits: np.ndarray, generated, penalty: float) -> np.ndarray:
    logits = np.array(logits, np.float32, copy=True)
    g = np.ascontiguousarray(np.asarray(generated, np.uint32))
    lib().orc_apply_repetition_penalty(_f(logits), _u32(g), g.size, penalty)
    return logits


def sample_select(logits: np.ndarray, temperature: float, top_k: int, top_p: float):
    """Candidate ids (in order), their probabilities after top-p, the cutoff."""
    logits = np.ascontiguousarray(logits, np.float32)
    V = logits.size
    n = top_k if 0 < top_k < V else V
    idx = np.zeros(n, np.uint32)
    probs = np.zeros(n, np.float32)
    cut = ctypes.c_int64(0)
    k = lib().orc_sample_select(_f(logits), V, temperature, top_k, top_p, _u32(idx), _f(probs),
                                ctypes.byref(cut))
    return idx[:k], probs[:k], int(cut.value)


def sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, r: float) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample(_f(logits), logits.size, temperature, top_k, top_p, r))


def stdrng_uniforms(seed: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    lib().orc_stdrng_uniforms(seed, n, _f(out))
    return out


# --- model ------------------------------------------------------------------

class OracleModel:
    """The reference's Model + KvCache + generate on the CPU.

    `tensors` maps HF names to numpy arrays: BF16 as uint16 bits, else f32.
    Matrices are borrowed: the arrays are kept alive by this object.
    """

    def __init__(self, cfg: dict, tensors: dict, i8: bool = False):
        """i8: the reference's TMG_I8=1 (layer matrices quantized at load,
        src/model.rs:57-76; the LM head and norms keep their precision)."""
        self.cfg = cfg
        c = OrcConfig(cfg["hidden_size"], cfg["num_hidden_layers"], cfg["num_attention_heads"],
                      cfg["num_key_value_heads"], cfg["head_dim"], cfg["intermediate_size"],
                      cfg["vocab_size"], cfg["rms_norm_eps"], cfg["rope_theta"])
        self._h = lib().orc_model_new(ctypes.byref(c))
        lib().orc_model_set_i8(self._h, 1 if i8 else 0)
        self._keep = []
        # the embedding first, so a dedicated lm_head (if any) overrides the tie
        names = sorted(tensors, key=lambda n: (n != "model.embed_tokens.weight", n))
        for name in names:
            a = np.ascontiguousarray(tensors[name])
            self._keep.append(a)
            dtype = 1 if a.dtype == np.uint16 else 0
            if dtype == 0:
                a = np.ascontiguousarray(a, np.float32)
                self._keep.append(a)
            rc = lib().orc_model_set(self._h, name.encode(), a.ctypes.data_as(_P), dtype, a.size)
            if rc != 0:
                raise ValueError(f"oracle rejected tensor {name}: {rc}")
        self.kv = self.new_cache()

    def __del__(self):
        try:
            if getattr(self, "kv", None):
                lib().orc_kv_free(self.kv)
            if getattr(self, "_h", None):
                lib().orc_model_free(self._h)
        except Exception:
            pass

    def new_cache(self):
        return lib().orc_kv_new(self._h)

    def reset(self):
        lib().orc_kv_reset(self.kv)

    def kv_len(self, layer: int = 0) -> int:
        return int(lib().orc_kv_len(self.kv, layer))

    def kv_read(self, layer: int):
        n = self.kv_len(layer)
        kvd = self.cfg["num_key_value_heads"] * self.cfg["head_dim"]
        k = np.zeros((n, kvd), np.float32)
        v = np.zeros((n, kvd), np.float32)
        lib().orc_kv_read(self.kv, layer, _f(k), _f(v))
        return k, v

    def kv_load(self, layer: int, keys: np.ndarray, values: np.ndarray):
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        lib().orc_kv_load(self.kv, layer, _f(keys), _f(values), keys.shape[0])

    def forward_token(self, token: int) -> np.ndarray:
        logits = np.zeros(self.cfg["vocab_size"], np.float32)
        if lib().orc_forward_token(self._h, self.kv, token, _f(logits)) != 0:
            raise ValueError("forward_token failed")
        return logits

    def forward_seq(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        logits = np.zeros(self.cfg["vocab_size"], np.float32)
        if lib().orc_forward_seq(self._h, self.kv, _u32(t), t.size, _f(logits)) != 0:
            raise ValueError("forward_seq failed")
        return logits

    def generate(self, prompt, max_tokens: int, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, repetition_penalty: float = 1.0, seed: int = 42,
                 uniforms=None, eos=()):
        """generate() from a fresh cache; returns (tokens, first_logits, prefill_s, decode_s)."""
        self.reset()
        p = np.ascontiguousarray(np.asarray(prompt, np.uint32))
        out = np.zeros(max(1, max_tokens), np.uint32)
        first = np.zeros(self.cfg["vocab_size"], np.float32)
        e = np.ascontiguousarray(np.asarray(list(eos) or [0], np.uint32))
        u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
        ps, ds = ctypes.c_double(0), ctypes.c_double(0)
        n = lib().orc_generate(self._h, self.kv, _u32(p), p.size, max_tokens, temperature, top_k,
                               top_p, repetition_penalty, seed, None if u is None else _f(u),
                               _u32(e), len(eos), _u32(out), _f(first), ctypes.byref(ps),
                               ctypes.byref(ds))
        if n < 0:
            raise ValueError("generate failed")
        return out[:n].copy(), first, ps.value, ds.value
