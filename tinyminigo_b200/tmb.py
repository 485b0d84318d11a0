"""TMB1, the reference's load-optimised repack of a checkpoint (src/tmb.rs).

One file: magic "TMB1" | u64 config length | u32 tensor count | config JSON |
u64 weights length | zero padding to 8 bytes | weights | index (per tensor:
u32 name length, name, u64 absolute offset, u64 byte length) | trailer (u64
index offset, metadata offset, weights length, file size).  Tensors sit in
consumption order, 8-byte aligned: the embedding (f32), then per layer q, k,
v, o, gate, up, down (BF16 bits) and the two norms (f32), the final norm
(f32), and lm_head (BF16) when the checkpoint has one.

`repack` is the offline tool (`--repack`, src/main.rs:29-35 -> write_tmb,
src/tmb.rs:127-247); `index` reads a file's header through the library's
parser (parse_tmb_header, src/tmb.rs:80-121); `Model.load` of a TMB1 file
uploads it with tmg_load_tmb (load_model_tmb, src/model.rs:108-179).
"""
from __future__ import annotations

import ctypes
import json
import struct
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import TmgError, lib

MAGIC = b"TMB1"
ALIGN = 8  # TENSOR_ALIGN, src/tmb.rs:26

LAYER_TENSORS = [  # (suffix, stored as BF16 bits) in consumption order, src/tmb.rs:160-170
    ("self_attn.q_proj.weight", True),
    ("self_attn.k_proj.weight", True),
    ("self_attn.v_proj.weight", True),
    ("self_attn.o_proj.weight", True),
    ("mlp.gate_proj.weight", True),
    ("mlp.up_proj.weight", True),
    ("mlp.down_proj.weight", True),
    ("input_layernorm.weight", False),
    ("post_attention_layernorm.weight", False),
]


def is_tmb(path) -> bool:
    """is_tmb, src/model.rs:97-103: the file starts with the magic."""
    try:
        with open(path, "rb") as f:
            return f.read(4) == MAGIC
    except OSError:
        return False


def config_json(cfg: dict) -> bytes:
    """ModelConfig::to_json (src/config.rs:96-110), compact, keys sorted as
    serde_json's default map writes them.  The EOS list goes under
    "eos_token_ids", which from_json does not read back (it reads
    "eos_token_id"): a repacked model has no EOS ids, as in the reference."""
    d = {
        "hidden_size": int(cfg["hidden_size"]),
        "num_hidden_layers": int(cfg["num_hidden_layers"]),
        "num_attention_heads": int(cfg["num_attention_heads"]),
        "num_key_value_heads": int(cfg["num_key_value_heads"]),
        "head_dim": int(cfg["head_dim"]),
        "intermediate_size": int(cfg["intermediate_size"]),
        "rms_norm_eps": float(np.float32(cfg["rms_norm_eps"])),
        "rope_theta": float(np.float32(cfg["rope_theta"])),
        "vocab_size": int(cfg["vocab_size"]),
        "eos_token_ids": [int(e) for e in cfg.get("eos_token_ids", [])],
        "bos_token_id": int(cfg.get("bos_token_id", 0)),
    }
    return json.dumps(d, sort_keys=True, separators=(",", ":")).encode()


def _as_f32(a: np.ndarray) -> np.ndarray:
    """push_f32's conversion (src/tmb.rs:143-154): BF16 bits widened exactly,
    f32 as is."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def write(dst, cfg: dict, tensors: dict) -> int:
    """write_tmb (src/tmb.rs:127-247) from in-memory tensors keyed by HF name
    (BF16 bit patterns as uint16 arrays, vectors as f32 or BF16).  Returns the
    file size."""
    order = [("model.embed_tokens.weight", False)]
    for layer in range(int(cfg["num_hidden_layers"])):
        order += [(f"model.layers.{layer}.{s}", bf) for s, bf in LAYER_TENSORS]
    order.append(("model.norm.weight", False))
    if "lm_head.weight" in tensors:
        order.append(("lm_head.weight", True))
    blobs, index, off = [], [], 0
    for name, bf16 in order:
        if name not in tensors:
            raise KeyError(f"missing {name}")
        a = np.ascontiguousarray(tensors[name])
        if bf16:
            if a.dtype != np.uint16:
                raise TypeError(f"{name}: BF16 bits (uint16) expected")
            b = a
        else:
            b = _as_f32(a)
        pad = (-off) % ALIGN
        off += pad
        blobs.append((pad, b))
        index.append((name, off, b.nbytes))
        off += b.nbytes
    weights_len = off
    cb = config_json(cfg)
    field = 16 + len(cb)  # where the weights-length field sits
    weights_off = (field + 8 + ALIGN - 1) // ALIGN * ALIGN
    index_off = weights_off + weights_len
    meta_off = index_off + sum(4 + len(n.encode()) + 16 for n, _, _ in index)
    size = meta_off + 32
    with open(dst, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<QI", len(cb), len(index)))
        f.write(cb)
        f.write(struct.pack("<Q", weights_len))
        f.write(b"\0" * (weights_off - field - 8))
        for pad, b in blobs:
            f.write(b"\0" * pad)
            f.write(b.tobytes())
        for name, o, n in index:
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)))
            f.write(nb)
            f.write(struct.pack("<QQ", weights_off + o, n))
        f.write(struct.pack("<QQQQ", index_off, meta_off, weights_len, size))
    return size


def repack(model_path, dst) -> int:
    """The `--repack` tool: a safetensors checkpoint with config.json beside
    it -> a TMB1 file.  Matrices must be BF16; vectors may be F32, F16 or
    BF16 (F16 widened with the reference's f16_to_f32)."""
    from .model import ModelConfig, f16_to_f32, safetensors_index

    p = Path(model_path)
    mc = ModelConfig.load(p.parent / "config.json")
    cfg = {k: getattr(mc, k) for k in ("hidden_size", "num_hidden_layers", "num_attention_heads",
                                         "num_key_value_heads", "head_dim", "intermediate_size",
                                         "rms_norm_eps", "rope_theta", "vocab_size",
                                         "bos_token_id")}
    cfg["eos_token_ids"] = list(mc.eos_token_ids)
    raw = np.memmap(p, dtype=np.uint8, mode="r")
    tensors = {}
    for name, dt, shape, off, nb in safetensors_index(p):
        b = raw[off:off + nb]
        if dt == "BF16":
            tensors[name] = b.view(np.uint16).reshape(shape)
        elif dt == "F32":
            tensors[name] = b.view(np.float32).reshape(shape)
        else:  # F16
            tensors[name] = np.array([f16_to_f32(int(h)) for h in b.view(np.uint16)],
                                     np.float32).reshape(shape)
    return write(dst, cfg, tensors)


def index(path):
    """(config, [(name, offset, nbytes), ...]) of a TMB1 file, parsed by the
    library (tmg_tmb_count / tmg_tmb_info)."""
    from .model import ModelConfig

    c = _lib.Config()
    n = ctypes.c_int64(0)
    err = ctypes.create_string_buffer(512)
    rc = lib().tmg_tmb_count(str(path).encode(), ctypes.byref(c), ctypes.byref(n), err, 512)
    if rc != 0:
        raise TmgError(rc, err.value.decode())
    out = []
    for i in range(n.value):
        name = ctypes.create_string_buffer(512)
        off, nb = ctypes.c_int64(), ctypes.c_int64()
        rc = lib().tmg_tmb_info(str(path).encode(), i, name, 512, ctypes.byref(off),
                                ctypes.byref(nb), err, 512)
        if rc != 0:
            raise TmgError(rc, err.value.decode())
        out.append((name.value.decode(), off.value, nb.value))
    return ModelConfig._from_c(c), out
