"""The oracle's int8 arms (the reference's TMG_I8=1 path): the checker for a
device int8 path.  The reference has no int8 tests of its own, so these pin
the restatement to its definitions (src/tensor.rs:128-170, 282-297,
341-357, 799-858, 860-893) with independent numpy arithmetic in f32."""
import numpy as np
import pytest

from tinyminigo_b200 import synth


def rnd(v):  # f32::round: halves away from zero
    return np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))


def test_quantize_i8_rules(orc):
    w = np.array([[127.0, 2.5, -2.5, 0.49, -127.0],   # scale exactly 1
                  [0.0, 0.0, 0.0, 0.0, 0.0],          # all zero: scale 1, q 0
                  [1e-3, -3e-3, 2e-3, 0.0, 5e-4]], np.float32)
    q, s = orc.quantize_i8(w)
    assert s[0] == 1.0 and s[1] == 1.0
    assert q[0].tolist() == [127, 3, -3, 0, -127]
    assert q[1].tolist() == [0] * 5
    assert s[2] == np.float32(np.float32(3e-3) / np.float32(127.0))
    assert q[2].tolist() == rnd(w[2] / s[2]).astype(np.int8).tolist()


def test_quantize_i8_random_rows(orc):
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (64, 200)).astype(np.float32)
    q, s = orc.quantize_i8(w)
    ms = np.abs(w).max(1) / np.float32(127.0)
    assert np.array_equal(s, ms.astype(np.float32))
    ref = np.clip(rnd(w / s[:, None]), -127, 127).astype(np.int8)
    assert np.array_equal(q, ref)


def test_quantize_row_i8(orc):
    q, s = orc.quantize_row_i8(np.zeros(9, np.float32))
    assert s == 0.0 and not q.any()
    x = np.random.default_rng(1).normal(0, 1, 300).astype(np.float32)
    q, s = orc.quantize_row_i8(x)
    s_ref = np.float32(np.abs(x).max() / np.float32(127.0))
    inv = np.float32(1.0) / s_ref
    assert s == s_ref
    assert np.array_equal(q, np.clip(rnd(x * inv), -127, 127).astype(np.int8))


def test_int8_gemv_is_integer_dot(orc):
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, (33, 2048)).astype(np.float32)
    x = rng.normal(0, 1, 2048).astype(np.float32)
    q, s = orc.quantize_i8(w)
    xq, xs = orc.quantize_row_i8(x)
    y = orc.matmul_w_i8(x, q, s)
    dots = q.astype(np.int64) @ xq.astype(np.int64)
    assert orc.dot_i8(xq, q[0]) == dots[0]
    ref = (dots.astype(np.float32) * xs) * s  # (dot as f32) * xs * scale, in that order
    assert np.array_equal(y, ref.astype(np.float32))


def test_int8_prefill_gemm(orc):
    # T = 6: one 4-token tile and a 2-token tail; 7 rows: three row pairs and
    # an odd row; K = 20: two 8-lane chunks and a 4-element tail, whose I8
    # elements enter the tile as q * scale before the row scale (as the
    # reference's wf_elem + w_row_scale do)
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (7, 20)).astype(np.float32)
    x = rng.normal(0, 1, (6, 20)).astype(np.float32)
    q, s = orc.quantize_i8(w)
    y = orc.matmul_batch_w_i8(x, q, s)
    qf = q.astype(np.float64)
    plain = (x.astype(np.float64) @ qf.T) * s  # scale once
    tail = x[:, 16:].astype(np.float64) @ (qf[:, 16:] * s[:, None]).T
    quirk = ((x[:, :16].astype(np.float64) @ qf[:, :16].T) + tail) * s
    expect = plain.copy()
    expect[:4, :6] = quirk[:4, :6]  # tiles: tokens 0-3, row pairs 0-5
    assert np.allclose(y, expect, rtol=1e-5, atol=1e-6)
    assert not np.allclose(quirk[:4, :6], plain[:4, :6], rtol=1e-3, atol=0)


def test_int8_model_decodes(orc):
    cfg = synth.CONFIGS["c1"]
    w = synth.make_weights(cfg, 5)
    a = orc.OracleModel(cfg, w, i8=True)
    b = orc.OracleModel(cfg, w)
    prompt = [3, 99, 1000, 31999, 7]
    la, lb = a.forward_seq(prompt), b.forward_seq(prompt)
    ta, tb = a.forward_token(42), b.forward_token(42)
    # lossy but close: the LM head stays BF16, the layers are per-row int8
    for u, v in ((la, lb), (ta, tb)):
        assert 0 < np.max(np.abs(u - v)) < 0.05
