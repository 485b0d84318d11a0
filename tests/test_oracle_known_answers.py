"""The oracle against the reference's own known-answer unit tests.

Each test restates one `#[test]` of the reference (path:line given) with the
same inputs and the same expected values, run on the C++ restatement.
"""
import math

import numpy as np
import pytest


def f32(*v):
    return np.array(v, np.float32)


def bf16_bits(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_matmul_identity(orc):  # src/tensor.rs:1224-1230
    y = orc.matmul_w(f32(3, -4), f32(1, 0, 0, 1).reshape(2, 2))
    assert list(y) == [3.0, -4.0]


def test_matmul_linear_weights(orc):  # src/tensor.rs:1233-1240
    y = orc.matmul_w(f32(1, 1), f32(1, 2, 3, 4).reshape(2, 2))
    assert list(y) == [3.0, 7.0]


def test_matmul_bf16_equals_f32_widened(orc):  # src/tensor.rs:38-41
    rng = np.random.default_rng(0)
    w = bf16_bits(rng.normal(0, 0.02, (37, 83)))
    x = rng.normal(0, 1, 83).astype(np.float32)
    wf = (w.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(orc.matmul_w(x, w), orc.matmul_w(x, wf))


def test_batch_gemm_matches_gemv_bitwise(orc):  # src/tensor.rs:735-738
    rng = np.random.default_rng(1)
    for T, out, inn in [(2, 9, 13), (5, 17, 64), (7, 3, 8), (4, 64, 100)]:
        w = bf16_bits(rng.normal(0, 0.02, (out, inn)))
        x = rng.normal(0, 1, (T, inn)).astype(np.float32)
        yb = orc.matmul_batch_w(x, w)
        for t in range(T):
            assert np.array_equal(yb[t], orc.matmul_w(x[t], w))


def test_rms_norm_known(orc):  # src/tensor.rs:1243-1250
    y = orc.rms_norm(f32(3, 4), f32(1, 1), 0.0)
    inv = np.float32(1.0) / np.sqrt(np.float32(12.5))
    assert abs(y[0] - 3 * inv) < 1e-6 and abs(y[1] - 4 * inv) < 1e-6


def test_rms_norm_weighted(orc):  # src/tensor.rs:1253-1259
    y = orc.rms_norm(f32(3, 4), f32(2, 0.5), 1e-6)
    inv = np.float32(1.0) / np.sqrt(np.float32(12.5) + np.float32(1e-6))
    assert abs(y[0] - 3 * inv * 2) < 1e-6 and abs(y[1] - 4 * inv * 0.5) < 1e-6


def test_rope_preserves_norm(orc):  # src/tensor.rs:1262-1268
    v = (np.arange(8, dtype=np.float32) * 0.5 - 1.75).astype(np.float32)
    r = orc.rope_rotate(v, 17, 5000000.0)
    assert abs(float((v * v).sum()) - float((r * r).sum())) < 1e-4


def test_rope_zero_pos_identity(orc):  # src/tensor.rs:1271-1275
    assert list(orc.rope_rotate(f32(1, 2, 3, 4), 0, 10000.0)) == [1, 2, 3, 4]


def test_rope_matches_reference(orc):  # src/tensor.rs:1278-1292
    v = orc.rope_rotate(f32(1, 0, 0, 1), 1, 10000.0)
    assert abs(v[0] - math.cos(1.0)) < 1e-5 and abs(v[2] - math.sin(1.0)) < 1e-5
    assert abs(v[1] - (-math.sin(0.01))) < 1e-5 and abs(v[3] - math.cos(0.01)) < 1e-5


def test_rope_table_equals_direct(orc):  # src/tensor.rs:983-1038: both forms agree
    rng = np.random.default_rng(2)
    v = rng.normal(0, 1, 3 * 16).astype(np.float32)
    for pos in [0, 1, 5, 1000, 40000]:
        t = orc.rope_table_rotate(v, 3, 16, pos, 500000.0)
        d = np.concatenate([orc.rope_rotate(v[h * 16:(h + 1) * 16], pos, 500000.0) for h in range(3)])
        assert np.array_equal(t, d)


def test_silu_known(orc):  # src/tensor.rs:1295-1298
    assert abs(orc.silu(0.0)) < 1e-6
    assert abs(orc.silu(1.0) - 1.0 / (1.0 + math.exp(-1.0))) < 1e-6


def test_softmax_sums_to_one(orc):  # src/tensor.rs:1301-1305
    p = orc.softmax(f32(1, 2, 3))
    assert abs(float(p.sum()) - 1.0) < 1e-6 and p[2] > p[1] > p[0]


def test_argmax_basic(orc):  # src/tensor.rs:1308-1312
    assert orc.argmax(f32(0.1, 3.0, 2.0)) == 1
    assert orc.argmax(f32(2.0, 2.0)) == 0


def test_argmax_nan_never_wins(orc):  # src/tensor.rs:1063-1073 (strict >)
    assert orc.argmax(f32(np.nan, 1.0, np.nan)) == 1
    assert orc.argmax(f32(-np.inf, -np.inf)) == 0


def test_attention_row_shapes(orc):  # src/tensor.rs:1315-1324 (via attention_batch)
    # one query row, 1 head, head_dim 2, two cached positions; causal row at pos 1
    q = f32(1, 0)
    keys = f32(1, 0, 0, 1)
    vals = f32(1, 2, 3, 4)
    out = orc.attention_batch(q, keys, vals, 1, 1, 2, 1)
    p = orc.softmax(f32(1.0 / math.sqrt(2.0), 0.0))
    assert abs(out[0, 0] - (p[0] * 1 + p[1] * 3)) < 1e-5
    assert abs(out[0, 1] - (p[0] * 2 + p[1] * 4)) < 1e-5


def test_repetition_penalty_applied(orc):  # src/tensor.rs:1327-1333
    l = orc.apply_repetition_penalty(f32(2.0, -2.0, 1.0), [0, 1], 2.0)
    assert list(l) == [1.0, -4.0, 1.0]


def test_repetition_penalty_unique_ids(orc):  # src/tensor.rs:1146-1153 (HashSet)
    l = orc.apply_repetition_penalty(f32(2.0, -2.0, 1.0), [0, 0, 0, 1, 1], 2.0)
    assert list(l) == [1.0, -4.0, 1.0]


def test_greedy_sample_is_argmax(orc):  # src/tensor.rs:1336-1339
    assert orc.sample(f32(0.1, 5.0, 3.0), 0.0, 0, 1.0, 0.5) == 1


def test_temperature_sample_peaked(orc):  # src/tensor.rs:1342-1352
    u = orc.stdrng_uniforms(123, 1)
    assert orc.sample(f32(0.1, 0.2, 0.3, 0.4, 5.0), 1.0, 0, 1.0, float(u[0])) == 4
    assert np.array_equal(orc.stdrng_uniforms(123, 4), orc.stdrng_uniforms(123, 4))


def test_top_k_restricts_candidates(orc):  # src/tensor.rs:1355-1364
    logits = f32(0.0, 5.0, 1.0, 4.0, 2.0)
    for seed in range(50):
        r = float(orc.stdrng_uniforms(seed, 1)[0])
        assert orc.sample(logits, 1.0, 2, 1.0, r) in (1, 3)


def test_top_p_cutoff_is_strict(orc):  # src/tensor.rs:1182-1201
    # probs for [ln 6, ln 3, ln 1] at T=1: 0.6, 0.3, 0.1 (approximately)
    logits = np.log(f32(6, 3, 1)).astype(np.float32)
    idx, probs, cut = orc.sample_select(logits, 1.0, 0, 0.85)
    assert cut == 2 and probs[2] == 0.0
    assert abs(float(probs[0] + probs[1]) - 1.0) < 1e-6


def test_uniforms_in_unit_interval(orc):  # StandardUniform f32 is [0, 1)
    u = orc.stdrng_uniforms(42, 4096)
    assert u.min() >= 0.0 and u.max() < 1.0 and 0.45 < u.mean() < 0.55
