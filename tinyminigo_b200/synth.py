"""Seeded synthetic Llama-style checkpoints for the benchmark configurations.

There is no network for real checkpoints, so every benchmark and parity test
runs on random weights with the reference's tensor names and layout
(src/model.rs:181-244): BF16 matrices drawn from N(0, 0.02^2) in f32 and
rounded to BF16 (round-to-nearest-even), norm weights = 1, and no
`lm_head.weight` when the embeddings are tied.  Files are written in the
safetensors format the reference loads (src/safetensors_loader.rs:103-147),
with a `config.json` beside them (src/config.rs:174-185).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

# The benchmark configurations (BASELINE.json "configs", in order).
CONFIGS = {
    "c1": dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
               head_dim=16, intermediate_size=128, vocab_size=32000, rope_theta=10000.0,
               rms_norm_eps=1e-6, tie_word_embeddings=False),
    "c2": dict(hidden_size=2048, num_hidden_layers=16, num_attention_heads=32,
               num_key_value_heads=8, head_dim=64, intermediate_size=8192, vocab_size=128256,
               rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=True),
    "c4": dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
               num_key_value_heads=8, head_dim=128, intermediate_size=14336, vocab_size=128256,
               rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=False),
}
# C3 (prefill stress) and C5 (long-context sampled decode) use the C2 shape.
CONFIGS["c3"] = CONFIGS["c2"]
CONFIGS["c5"] = CONFIGS["c2"]


def with_layers(cfg: dict, layers: int) -> dict:
    c = dict(cfg)
    c["num_hidden_layers"] = layers
    return c


def tensor_specs(cfg: dict):
    """(name, shape, kind) in file order; kind is 'w' (random) or 'norm' (ones)."""
    h, i = cfg["hidden_size"], cfg["intermediate_size"]
    qd = cfg["num_attention_heads"] * cfg["head_dim"]
    kd = cfg["num_key_value_heads"] * cfg["head_dim"]
    specs = [("model.embed_tokens.weight", (cfg["vocab_size"], h), "w")]
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        specs += [
            (p + "self_attn.q_proj.weight", (qd, h), "w"),
            (p + "self_attn.k_proj.weight", (kd, h), "w"),
            (p + "self_attn.v_proj.weight", (kd, h), "w"),
            (p + "self_attn.o_proj.weight", (h, qd), "w"),
            (p + "mlp.gate_proj.weight", (i, h), "w"),
            (p + "mlp.up_proj.weight", (i, h), "w"),
            (p + "mlp.down_proj.weight", (h, i), "w"),
            (p + "input_layernorm.weight", (h,), "norm"),
            (p + "post_attention_layernorm.weight", (h,), "norm"),
        ]
    specs.append(("model.norm.weight", (h,), "norm"))
    if not cfg.get("tie_word_embeddings", False):
        specs.append(("lm_head.weight", (cfg["vocab_size"], h), "w"))
    return specs


def iter_weights(cfg: dict, seed: int, device: str = "cpu", std: float = 0.02):
    """(name, BF16 bit patterns as numpy uint16) for every tensor, drawn in
    file order from one torch Generator seeded with `seed` on `device`, one
    tensor at a time (a consumer that uploads and drops each holds one
    tensor in host memory at most)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for name, shape, kind in tensor_specs(cfg):
        if kind == "norm":
            t = torch.ones(shape, dtype=torch.bfloat16)
        else:
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(0.0, std, generator=g)
            t = t.to(torch.bfloat16)
        yield name, t.view(torch.int16).cpu().numpy().view(np.uint16)


def make_weights(cfg: dict, seed: int, device: str = "cpu", std: float = 0.02) -> dict:
    """iter_weights collected into a dict keyed by tensor name."""
    return dict(iter_weights(cfg, seed, device, std))


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def config_json(cfg: dict, eos=None) -> dict:
    d = {
        "architectures": ["LlamaForCausalLM"],
        "model_type": "llama",
        "hidden_size": cfg["hidden_size"],
        "num_hidden_layers": cfg["num_hidden_layers"],
        "num_attention_heads": cfg["num_attention_heads"],
        "num_key_value_heads": cfg["num_key_value_heads"],
        "head_dim": cfg["head_dim"],
        "intermediate_size": cfg["intermediate_size"],
        "vocab_size": cfg["vocab_size"],
        "rope_theta": cfg["rope_theta"],
        "rms_norm_eps": cfg["rms_norm_eps"],
        "tie_word_embeddings": bool(cfg.get("tie_word_embeddings", False)),
        "bos_token_id": 0,
    }
    if eos is not None:
        d["eos_token_id"] = eos
    return d


def write_safetensors(path: Path, tensors: dict) -> None:
    """Write BF16 (uint16 bits) / F32 arrays in the safetensors layout:
    u64 LE header length, JSON header (padded to 8 bytes), raw data."""
    header, off, items = {}, 0, []
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        dt = "BF16" if a.dtype == np.uint16 else "F32"
        if dt == "F32":
            a = a.astype(np.float32)
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        items.append(a)
        off += a.nbytes
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in items:
            f.write(a.tobytes())


def write_model(directory: str | Path, cfg: dict, tensors: dict, eos=None) -> Path:
    """Write model.safetensors + config.json; returns the safetensors path."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(config_json(cfg, eos), indent=1))
    p = d / "model.safetensors"
    write_safetensors(p, tensors)
    return p


def random_prompt(vocab: int, n: int, seed: int) -> np.ndarray:
    """Uniform random token ids in [0, vocab) from numpy's default_rng(seed)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)
