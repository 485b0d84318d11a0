"""The tensor-core prefill attention (attn_prefill_tc.cu) against the CPU
oracle's prefill attention (src/model.rs:526-571), through tmg_op_attn_prefill
(head dim 64 takes the tcgen05 kernel).

Shapes cover one and many 128-row query blocks, partial query blocks,
start offsets that are not multiples of the 64-key block (the causal mask
inside a block and keys past the end), GQA groups of 1 to 8 q heads, the
C3 layer shape (2048 rows, 32/8 heads) and a chunk late in a long prompt.

Bar: |out - ref| <= 1e-5 * max|v| (the CUDA-core kernel's bound): the
scores are carried as three BF16 parts per operand (~24 bits) and the
values as two (the output is a weighted mean, so its error is bounded by
~2^-17 of |v| per term and averages down).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU box
    pytest.skip("needs a GPU", allow_module_level=True)

from tinyminigo_b200._lib import check, lib  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    h = ctypes.c_void_p()
    check(lib().tmg_create(0, None, ctypes.byref(h)))
    yield h
    lib().tmg_destroy(h)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def P(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("T,start,nq,nkv", [(1, 0, 4, 4), (63, 0, 8, 2), (128, 0, 4, 1),
                                            (129, 5, 8, 8), (300, 77, 32, 8), (1000, 0, 16, 2),
                                            (2048, 0, 32, 8), (384, 3000, 32, 8)])
def test_prefill_attention_tc_matches_oracle(ctx, orc, T, start, nq, nkv):
    d = 64
    rng = np.random.default_rng(1000 * T + start + nq)
    q = rng.normal(0, 1, (T, nq * d)).astype(np.float32)
    keys = rng.normal(0, 1, (start + T, nkv * d)).astype(np.float32)
    vals = rng.normal(0, 1, (start + T, nkv * d)).astype(np.float32)
    od = torch.zeros((T, nq * d), dtype=torch.float32, device="cuda")
    qd, kd, vd = dev(q), dev(keys), dev(vals)
    check(lib().tmg_op_attn_prefill(ctx, P(qd), P(kd), P(vd), T, start, nq, nkv, d, P(od)), ctx)
    ref = orc.attention_batch(q, keys, vals, nq, nkv, d, start)
    err = np.max(np.abs(od.cpu().numpy() - ref))
    assert err <= 1e-5 * np.abs(vals).max(), err


def test_prefill_attention_tc_large_scores(ctx, orc):
    # scores of tens (q, k ~ N(0, 3^2)): the running max moves often and
    # most probabilities underflow; the output must still follow the oracle
    T, start, nq, nkv, d = 256, 40, 8, 2, 64
    rng = np.random.default_rng(7)
    q = rng.normal(0, 3, (T, nq * d)).astype(np.float32)
    keys = rng.normal(0, 3, (start + T, nkv * d)).astype(np.float32)
    vals = rng.normal(0, 1, (start + T, nkv * d)).astype(np.float32)
    od = torch.zeros((T, nq * d), dtype=torch.float32, device="cuda")
    qd, kd, vd = dev(q), dev(keys), dev(vals)
    check(lib().tmg_op_attn_prefill(ctx, P(qd), P(kd), P(vd), T, start, nq, nkv, d, P(od)), ctx)
    ref = orc.attention_batch(q, keys, vals, nq, nkv, d, start)
    err = np.max(np.abs(od.cpu().numpy() - ref))
    assert err <= 1e-4 * np.abs(vals).max(), err
