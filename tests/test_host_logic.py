"""Host logic of the library that needs no GPU: config.json parsing
(src/config.rs), the safetensors reader (src/safetensors_loader.rs), the
f16 widening, and the sampler's uniform draws."""
import json
import struct

import numpy as np
import pytest

from tinyminigo_b200 import synth
from tinyminigo_b200._lib import TmgError
from tinyminigo_b200.model import ModelConfig, f16_to_f32, rng_uniforms, safetensors_index

TINY_RANDOM_MINICPM5 = """{
    "architectures": ["LlamaForCausalLM"],
    "bos_token_id": 0,
    "eos_token_id": [1, 130073],
    "head_dim": 32,
    "hidden_size": 16,
    "intermediate_size": 64,
    "model_type": "llama",
    "num_attention_heads": 16,
    "num_hidden_layers": 2,
    "num_key_value_heads": 2,
    "rms_norm_eps": 1e-06,
    "rope_parameters": {"rope_theta": 5000000.0, "rope_type": "default"},
    "tie_word_embeddings": false,
    "vocab_size": 130560
}"""


def test_parses_tiny_random_minicpm5_config(tmp_path):  # src/config.rs:191-225
    p = tmp_path / "config.json"
    p.write_text(TINY_RANDOM_MINICPM5)
    c = ModelConfig.load(p)
    assert (c.hidden_size, c.num_hidden_layers, c.num_attention_heads) == (16, 2, 16)
    assert (c.num_key_value_heads, c.head_dim, c.intermediate_size) == (2, 32, 64)
    assert c.rms_norm_eps == np.float32(1e-6)
    assert c.rope_theta == 5_000_000.0
    assert c.vocab_size == 130560
    assert c.eos_token_ids == [1, 130073]
    assert c.bos_token_id == 0
    assert c.num_attention_heads // c.num_key_value_heads == 8


def test_config_defaults():  # src/config.rs:42-91
    c = ModelConfig.from_json(json.dumps(dict(hidden_size=64, num_attention_heads=4,
                                              num_hidden_layers=1, intermediate_size=8,
                                              vocab_size=10)))
    assert c.num_key_value_heads == 4 and c.head_dim == 16
    assert c.rope_theta == 10000.0 and c.rms_norm_eps == np.float32(1e-5)
    assert c.eos_token_ids == [] and c.bos_token_id == 0


def test_config_scalar_eos_and_top_level_theta():
    c = ModelConfig.from_json(json.dumps(dict(hidden_size=8, num_attention_heads=2,
                                              num_hidden_layers=1, intermediate_size=8,
                                              vocab_size=10, eos_token_id=7, rope_theta=500000.0,
                                              rope_parameters={"rope_theta": 1.0})))
    assert c.eos_token_ids == [7] and c.rope_theta == 500000.0


def test_config_missing_field_is_an_error():
    with pytest.raises(TmgError, match="hidden_size"):
        ModelConfig.from_json('{"num_attention_heads": 2}')
    with pytest.raises(TmgError, match="JSON"):
        ModelConfig.from_json('{"hidden_size": 2,')
    with pytest.raises(TmgError, match="eos"):
        ModelConfig.from_json(json.dumps(dict(hidden_size=8, num_attention_heads=2,
                                              num_hidden_layers=1, intermediate_size=8,
                                              vocab_size=10, eos_token_id=-1)))


def test_config_load_missing_file(tmp_path):
    with pytest.raises(TmgError):
        ModelConfig.load(tmp_path / "nope.json")


def test_f16_conversions():  # src/safetensors_loader.rs:184-189
    assert f16_to_f32(0x3C00) == 1.0
    assert f16_to_f32(0) == 0.0
    assert f16_to_f32(0xBC00) == -1.0
    assert np.isinf(f16_to_f32(0x7C00))
    assert f16_to_f32(0x3555) == np.float32(np.float16(0.333251953125))


def test_f16_subnormal_follows_reference():
    # src/safetensors_loader.rs:153-166 starts the subnormal exponent at
    # 127 - 1 instead of 127 - 15, so f16 subnormals widen 2^13 too large
    # (0x0001 -> 2^-11, IEEE says 2^-24).  The library keeps the
    # reference's result: parity is with the reference, not with IEEE.
    assert f16_to_f32(0x0001) == 2.0 ** -11
    assert f16_to_f32(0x8200) == -(2.0 ** 13) * float(np.float16(np.frombuffer(
        np.uint16(0x0200).tobytes(), np.float16)[0]))


def test_safetensors_roundtrip(tmp_path):  # src/safetensors_loader.rs:198-226
    p = tmp_path / "t.safetensors"
    synth.write_safetensors(p, {"w": np.array([[1, 2], [3, 4]], np.float32),
                                "b": np.array([0x3F80, 0xC000], np.uint16)})
    idx = {n: (dt, sh, off, nb) for n, dt, sh, off, nb in safetensors_index(p)}
    assert idx["w"][0] == "F32" and idx["w"][1] == [2, 2] and idx["w"][3] == 16
    assert idx["b"][0] == "BF16" and idx["b"][1] == [2] and idx["b"][3] == 4
    raw = p.read_bytes()
    assert np.frombuffer(raw[idx["b"][2]:idx["b"][2] + 4], np.uint16).tolist() == [0x3F80, 0xC000]
    assert np.frombuffer(raw[idx["w"][2]:idx["w"][2] + 16], np.float32).tolist() == [1, 2, 3, 4]


def test_safetensors_rejects_bad_files(tmp_path):
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(TmgError, match="too small"):
        safetensors_index(p)
    q = tmp_path / "trunc.safetensors"
    q.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(TmgError, match="truncated"):
        safetensors_index(q)
    r = tmp_path / "dtype.safetensors"
    h = json.dumps({"x": {"dtype": "I64", "shape": [1], "data_offsets": [0, 8]}}).encode()
    r.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(TmgError, match="unsupported dtype"):
        safetensors_index(r)
    s = tmp_path / "off.safetensors"
    h = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    s.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(TmgError, match="data_offsets"):
        safetensors_index(s)


def test_synthetic_model_file_layout(tmp_path):
    cfg = synth.with_layers(synth.CONFIGS["c1"], 1)
    t = synth.make_weights(cfg, 5)
    p = synth.write_model(tmp_path, cfg, t)
    idx = {n: (dt, sh) for n, dt, sh, _, _ in safetensors_index(p)}
    assert idx["model.embed_tokens.weight"] == ("BF16", [32000, 64])
    assert idx["lm_head.weight"] == ("BF16", [32000, 64])
    assert idx["model.layers.0.self_attn.k_proj.weight"] == ("BF16", [32, 64])
    c = ModelConfig.load(tmp_path / "config.json")
    assert c.vocab_size == 32000 and c.head_dim == 16 and c.rope_theta == 10000.0


def test_rng_uniforms_match_oracle_restatement(orc):
    for seed in [0, 1, 42, 2**63 + 5]:
        assert np.array_equal(rng_uniforms(seed, 100), orc.stdrng_uniforms(seed, 100))
    u = rng_uniforms(7, 10000)
    assert u.min() >= 0 and u.max() < 1 and len(set(u.tolist())) > 9990


def test_entry_points_refuse_bad_arguments_before_any_device_call():
    # argument errors come back as TMG_ERR_INVALID (-1) without touching a
    # GPU: a null context or cache, a group of one rank or of more than 8,
    # a rank outside the group
    import ctypes

    from tinyminigo_b200._lib import lib

    uid = (ctypes.c_uint8 * 128)()
    L = lib()
    assert L.tmg_fused_group_init(None, None, uid, 0, 2) == -1
    assert L.tmg_fused_group_init(None, None, None, 0, 2) == -1
    assert L.tmg_fused_group_init(None, None, uid, 0, 1) == -1
    assert L.tmg_fused_group_init(None, None, uid, 2, 2) == -1
    assert L.tmg_fused_group_init(None, None, uid, 0, 9) == -1
    assert L.tmg_op_attn_prefill(None, None, None, None, 16, 0, 4, 2, 64, None) == -1
