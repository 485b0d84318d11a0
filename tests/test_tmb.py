"""TMB1 repack format (src/tmb.rs) on the host: the writer (write_tmb,
src/tmb.rs:127-247) and the library's header parser (parse_tmb_header,
src/tmb.rs:80-121), without a GPU.

The reference has no test of its own for this file; these pin the layout it
writes (consumption order, 8-byte aligned tensors, f32 embedding and norms,
raw BF16 matrices, the 32-byte trailer) and the errors its reader gives.
"""
import struct

import numpy as np
import pytest

from tinyminigo_b200 import synth, tmb
from tinyminigo_b200._lib import TmgError

C1 = synth.CONFIGS["c1"]


@pytest.fixture(scope="module")
def c1w():
    return synth.make_weights(C1, 7)


def cfg_with_eos(eos=(3, 5)):
    c = dict(C1)
    c["eos_token_ids"] = list(eos)
    c["bos_token_id"] = 1
    return c


def test_layout_and_index(tmp_path, c1w):
    p = tmp_path / "m.tmb"
    size = tmb.write(p, cfg_with_eos(), c1w)
    raw = p.read_bytes()
    assert len(raw) == size and raw[:4] == b"TMB1"
    cfg, idx = tmb.index(p)
    assert (cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads,
            cfg.num_key_value_heads, cfg.head_dim, cfg.intermediate_size,
            cfg.vocab_size) == (64, 2, 4, 2, 16, 128, 32000)
    assert np.float32(cfg.rms_norm_eps) == np.float32(1e-6)
    assert np.float32(cfg.rope_theta) == np.float32(10000.0)
    assert cfg.bos_token_id == 1
    # the repack writes "eos_token_ids", from_json reads "eos_token_id":
    # a TMB model has no EOS ids (src/config.rs:64-72, 96-110)
    assert cfg.eos_token_ids == []
    names = [n for n, _, _ in idx]
    expect = ["model.embed_tokens.weight"]
    for layer in range(2):
        expect += [f"model.layers.{layer}.{s}" for s, _ in tmb.LAYER_TENSORS]
    expect += ["model.norm.weight", "lm_head.weight"]
    assert names == expect
    for name, off, nb in idx:
        assert off % 8 == 0
        a = c1w[name]
        if name.endswith("proj.weight") or name == "lm_head.weight":
            assert nb == a.nbytes
            assert np.array_equal(np.frombuffer(raw, np.uint16, a.size, off), a.ravel())
        else:  # embedding and norms are stored widened to f32
            assert nb == a.size * 4
            got = np.frombuffer(raw, np.float32, a.size, off)
            assert np.array_equal(got, synth.bf16_to_f32(a).ravel())
    # trailer: index offset, metadata offset, weights length, file size
    index_off, meta_off, wlen, fsize = struct.unpack("<QQQQ", raw[-32:])
    assert fsize == len(raw) and meta_off == len(raw) - 32
    assert index_off == idx[-1][1] + idx[-1][2]
    assert wlen == index_off - idx[0][1]


def test_tied_checkpoint_has_no_lm_head(tmp_path, c1w):
    t = {k: v for k, v in c1w.items() if k != "lm_head.weight"}
    p = tmp_path / "tied.tmb"
    tmb.write(p, C1, t)
    _, idx = tmb.index(p)
    assert idx[-1][0] == "model.norm.weight" and len(idx) == 1 + 2 * 9 + 1


def test_repack_from_safetensors_equals_direct_write(tmp_path, c1w):
    st = synth.write_model(tmp_path / "src", C1, c1w, eos=[7])
    a, b = tmp_path / "a.tmb", tmp_path / "b.tmb"
    tmb.repack(st, a)
    tmb.write(b, dict(C1, eos_token_ids=[7]), c1w)
    assert a.read_bytes() == b.read_bytes()
    assert tmb.is_tmb(a) and not tmb.is_tmb(st)


def test_reader_errors(tmp_path, c1w):
    good = tmp_path / "g.tmb"
    tmb.write(good, C1, c1w)
    raw = good.read_bytes()
    cases = {
        "short": (raw[:10], "too small"),
        "magic": (b"TMB2" + raw[4:], "wrong magic"),
        "config": (raw[:40], "truncated"),
        "index": (raw[:-200], "truncated"),
    }
    # a tensor whose range runs past the end of the file
    _, idx = tmb.index(good)
    name = idx[0][0].encode()
    at = raw.index(struct.pack("<I", len(name)) + name) + 4 + len(name)
    bad = bytearray(raw)
    bad[at:at + 8] = struct.pack("<Q", len(raw) - 4)
    cases["range"] = (bytes(bad), "out of bounds")
    # a config that ModelConfig::from_json rejects (hidden_size missing)
    cfg_len = struct.unpack("<Q", raw[4:12])[0]
    cj = raw[16:16 + cfg_len].replace(b'"hidden_size"', b'"hidden_sizX"')
    cases["json"] = (raw[:16] + cj + raw[16 + cfg_len:], "hidden_size")
    for key, (data, msg) in cases.items():
        p = tmp_path / f"{key}.tmb"
        p.write_bytes(data)
        with pytest.raises(TmgError) as ei:
            tmb.index(p)
        assert msg in str(ei.value), (key, str(ei.value))


def test_writer_needs_bf16_matrices(tmp_path, c1w):
    t = dict(c1w)
    t["model.layers.0.mlp.up_proj.weight"] = synth.bf16_to_f32(t["model.layers.0.mlp.up_proj.weight"])
    with pytest.raises(TypeError):
        tmb.write(tmp_path / "x.tmb", C1, t)
    t = {k: v for k, v in c1w.items() if k != "model.norm.weight"}
    with pytest.raises(KeyError):
        tmb.write(tmp_path / "y.tmb", C1, t)


def test_repack_widens_f16_and_f32_norms(tmp_path, c1w):
    # norm vectors may be F16 or F32 in the checkpoint; the repack stores f32
    # (push_f32, src/tmb.rs:143-154; F16 widened as src/safetensors_loader.rs:149-173)
    import json as _json
    import struct as _struct

    from tinyminigo_b200.model import f16_to_f32

    t = dict(c1w)
    n16 = np.array([1.0, -2.5, 0.0001, 65504.0] * 16, np.float16)
    n32 = np.linspace(-1, 1, 64).astype(np.float32)
    src = synth.write_model(tmp_path / "m", C1, {k: v for k, v in t.items()
                                                 if k not in ("model.norm.weight",
                                                              "model.layers.0.input_layernorm.weight")})
    # rewrite the file with an F16 final norm and an F32 input norm
    header = {}
    blobs, off = [], 0
    items = dict(t)
    items["model.norm.weight"] = n16
    items["model.layers.0.input_layernorm.weight"] = n32
    for name, a in items.items():
        a = np.ascontiguousarray(a)
        dt = {np.dtype(np.uint16): "BF16", np.dtype(np.float16): "F16",
              np.dtype(np.float32): "F32"}[a.dtype]
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    hb = _json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    src.write_bytes(_struct.pack("<Q", len(hb)) + hb + b"".join(blobs))
    out = tmp_path / "n.tmb"
    tmb.repack(src, out)
    raw = out.read_bytes()
    _, idx = tmb.index(out)
    at = {n: (o, nb) for n, o, nb in idx}
    o, nb = at["model.norm.weight"]
    got = np.frombuffer(raw, np.float32, 64, o)
    assert np.array_equal(got, np.float32([f16_to_f32(int(h)) for h in n16.view(np.uint16)]))
    o, nb = at["model.layers.0.input_layernorm.weight"]
    assert np.array_equal(np.frombuffer(raw, np.float32, 64, o), n32)
