"""ctypes bindings of the C ABI in include/tmg_cuda.h (libtmg_cuda.so, built
in-tree by tinyminigo_b200.build).  There is no fallback: if the library is
missing, every call raises."""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libtmg_cuda.so"

TMG_OK = 0
ERRORS = {
    -1: "invalid argument",
    -2: "CUDA error",
    -3: "I/O error",
    -4: "KV cache capacity exceeded",
    -5: "NaN logits",
    -6: "device wait timed out",
    -7: "collective failed",
}


class TmgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, 'error')} ({code}): {msg}")
        self.code = code


class Config(ctypes.Structure):
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
        ("bos_token_id", ctypes.c_uint32),
        ("n_eos", ctypes.c_int32),
        ("eos_token_ids", ctypes.c_uint32 * 8),
    ]


class GenParamsC(ctypes.Structure):
    _fields_ = [
        ("max_tokens", ctypes.c_int64),
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_int64),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("seed", ctypes.c_uint64),
    ]


TOKEN_CB = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p)

_P = ctypes.c_void_p
_PP = ctypes.POINTER(ctypes.c_void_p)
_I = ctypes.c_int
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float
_CP = ctypes.c_char_p
_PI64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); every symbol include/tmg_cuda.h declares.
SIGNATURES = {
    "tmg_version": (_CP, []),
    "tmg_f16_to_f32": (_F, [ctypes.c_uint16]),
    "tmg_config_load": (_I, [_CP, ctypes.POINTER(Config), _CP, _I]),
    "tmg_config_parse": (_I, [_CP, ctypes.POINTER(Config), _CP, _I]),
    "tmg_safetensors_count": (_I, [_CP, _PI64, _CP, _I]),
    "tmg_safetensors_info": (_I, [_CP, _I64, _CP, _I, ctypes.POINTER(_I32), ctypes.POINTER(_I32),
                                  ctypes.POINTER(_I64), _PI64, _PI64, _CP, _I]),
    "tmg_tmb_count": (_I, [_CP, ctypes.POINTER(Config), _PI64, _CP, _I]),
    "tmg_tmb_info": (_I, [_CP, _I64, _CP, _I, _PI64, _PI64, _CP, _I]),
    "tmg_create": (_I, [_I, ctypes.POINTER(Config), _PP]),
    "tmg_destroy": (_I, [_P]),
    "tmg_last_error": (_CP, [_P]),
    "tmg_load_safetensors": (_I, [_P, _CP]),
    "tmg_load_tmb": (_I, [_P, _CP]),
    "tmg_set_tensor": (_I, [_P, _CP, _I32, _P, _I64]),
    "tmg_finalize": (_I, [_P]),
    "tmg_weight_bytes": (_I64, [_P]),
    "tmg_kv_create": (_I, [_P, _I32, _I64, _PP]),
    "tmg_kv_destroy": (_I, [_P]),
    "tmg_kv_len": (_I, [_P, _I32, _I32, _PI64]),
    "tmg_kv_reset": (_I, [_P]),
    "tmg_kv_truncate": (_I, [_P, _I32, _I64]),
    "tmg_kv_read": (_I, [_P, _I32, _I32, _P, _P]),
    "tmg_forward_token": (_I, [_P, _P, _P, _P]),
    "tmg_forward_seq": (_I, [_P, _P, _I32, _P, _I64, _P]),
    "tmg_generate": (_I, [_P, _P, _P, _I64, ctypes.POINTER(GenParamsC), _P, _P, _PI64, _P,
                          ctypes.POINTER(ctypes.c_double), TOKEN_CB, _P]),
    "tmg_generate_batch": (_I, [_P, _P, _P, _I64, ctypes.POINTER(GenParamsC), _P, _P, _PI64]),
    "tmg_rng_uniforms": (_I, [ctypes.c_uint64, _I64, _P]),
    "tmg_decode": (_I, [_P, _P, _P, _I64, _P]),
    "tmg_sync": (_I, [_P]),
    "tmg_stream": (_P, [_P]),
    "tmg_profile_decode": (_I, [_P, _P, _P, _I64, _P, _P]),
    "tmg_trace_decode": (_I, [_P, _P, _P, _P, _P, _I32, ctypes.POINTER(_I32)]),
    "tmg_trace_fused": (_I, [_P, _P, ctypes.c_uint32, _P, ctypes.c_int64, ctypes.POINTER(_I32)]),
    "tmg_tp_unique_id": (_I, [_P]),
    "tmg_tp_init": (_I, [_P, _P, _I32, _I32]),
    "tmg_tp_shard": (_I, [_P, ctypes.c_char_p, _I32, _I32, _P]),
    "tmg_fused_group_init": (_I, [_P, _P, _P, _I32, _I32]),
    "tmg_op_gemv_bf16": (_I, [_P, _P, _P, _I64, _I64, _I32, _P]),
    "tmg_wmat_upload_bf16": (_I, [_P, _P, _I64, _I64, _PP]),
    "tmg_wmat_free": (_I, [_P]),
    "tmg_wmat_shape": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "tmg_op_gemv_wmat": (_I, [_P, _P, _P, _I32, _P]),
    "tmg_op_gemm_wmat": (_I, [_P, _P, _P, _I64, _P]),
    "tmg_op_quantize_i8": (_I, [_P, _P, _I64, _I64, _P, _P]),
    "tmg_op_gemv_i8": (_I, [_P, _P, _P, _P, _I64, _I64, _I32, _P]),
    "tmg_op_gemm_bf16": (_I, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "tmg_op_rmsnorm": (_I, [_P, _P, _P, _F, _I64, _I64, _I32, _P]),
    "tmg_op_rope": (_I, [_P, _P, _I64, _I32, _I32, _I64, _F]),
    "tmg_op_swiglu": (_I, [_P, _P, _P, _I64, _P]),
    "tmg_op_attn_decode": (_I, [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _P]),
    "tmg_op_attn_decode_noalloc": (_I, [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _P]),
    "tmg_op_attn_prefill": (_I, [_P, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _P]),
    "tmg_op_argmax": (_I, [_P, _P, _I64, _I32, _P]),
    "tmg_op_sample": (_I, [_P, _P, _I64, _I32, _P, _I64, _F, _I64, _F, _F, _P, _P, _P, _P, _P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libtmg_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"the CUDA library {LIB_PATH} is missing: run `python -m tinyminigo_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int, ctx=None, what: str = "") -> None:
    if rc != TMG_OK:
        msg = ""
        # a null context reads why the last tmg_create on this thread failed
        m = lib().tmg_last_error(ctx)
        msg = m.decode() if m else ""
        raise TmgError(rc, f"{what}: {msg}" if what else msg)
