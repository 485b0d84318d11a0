"""tmg_op_attn_decode_noalloc (decode attention on a static per-device
scratch, no allocation at call time) against tmg_op_attn_decode on the same
inputs, through the C ABI.

Both enqueue the same attention kernel with the same split count, so the
outputs should agree bit for bit; the check allows 1e-6 of the largest
|value| for headroom.  Each case calls the new entry point twice in a row
(the second call must find the tickets reset and give the same result).
The cases cover both kernels behind the entry point: head dim 64 with at
most 4 query heads per kv head (register-streaming kernel) and the tiled
kernel (head dims 16/32/128, and 16 query heads per kv head).  One case is
also checked against the CPU oracle (attention_batch, src/tensor.rs:
1099-1139) within the decode attention tests' bound (1e-5 of max |V|).
Also: the device's free memory does not move across calls after the first
(which sets the scratch up), and a request larger than the static scratch
is rejected with TMG_ERR_CAPACITY (an unsupported head dim with
TMG_ERR_INVALID) before anything is enqueued.

The file name sorts last so the test also runs after every other test in
the session; it passes alone as well (its context is its own).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU box
    pytest.skip("needs a GPU", allow_module_level=True)

from tinyminigo_b200._lib import TmgError, check, lib  # noqa: E402

TMG_ERR_INVALID = -1
TMG_ERR_CAPACITY = -4


@pytest.fixture(scope="module")
def ctx():
    h = ctypes.c_void_p()
    check(lib().tmg_create(0, None, ctypes.byref(h)))
    yield h
    lib().tmg_destroy(h)


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def inputs(n_ctx, nq, nkv, d, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(nq * d, generator=g).cuda()
    k = torch.randn(n_ctx, nkv * d, generator=g).cuda()
    v = torch.randn(n_ctx, nkv * d, generator=g).cuda()
    return q, k, v


@pytest.mark.parametrize("n_ctx,nq,nkv,d", [(1, 4, 2, 16), (33, 32, 8, 64), (300, 32, 8, 128),
                                             (2000, 8, 2, 128), (4097, 4, 1, 64),
                                             (700, 64, 4, 64), (129, 16, 2, 32)])
def test_noalloc_matches_op(ctx, n_ctx, nq, nkv, d):
    q, k, v = inputs(n_ctx, nq, nkv, d, n_ctx + d)
    ref = torch.zeros(nq * d, device="cuda")
    check(lib().tmg_op_attn_decode(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(ref)), ctx)
    outs = [torch.full((nq * d,), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    for o in outs:  # two calls in a row
        check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(o)),
              ctx)
    check(lib().tmg_sync(ctx), ctx)
    tol = 1e-6 * float(ref.abs().max()) + 1e-30
    for o in outs:
        assert torch.isfinite(o).all()
        assert float((o - ref).abs().max()) <= tol


def test_noalloc_matches_oracle(ctx, orc):
    n_ctx, nq, nkv, d = 1031, 32, 8, 64
    q, k, v = inputs(n_ctx, nq, nkv, d, 21)
    out = torch.zeros(nq * d, device="cuda")
    check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(out)), ctx)
    check(lib().tmg_sync(ctx), ctx)
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))
    ref = orc.attention_batch(qh, kh, vh, nq, nkv, d, n_ctx - 1)[0]
    assert np.max(np.abs(out.cpu().numpy() - ref)) < 1e-5 * (np.abs(vh).max() + 1e-6)


def test_noalloc_leaves_free_memory_alone(ctx):
    n_ctx, nq, nkv, d = 777, 32, 8, 128
    q, k, v = inputs(n_ctx, nq, nkv, d, 5)
    out = torch.zeros(nq * d, device="cuda")
    # first call: setup (symbol lookup, module load)
    check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(out)), ctx)
    check(lib().tmg_sync(ctx), ctx)
    torch.cuda.synchronize()
    # free memory is device-wide: another process can move it, so a change
    # is measured twice before it counts
    moved = []
    for _ in range(2):
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(3):
            check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d,
                                                   P(out)), ctx)
        check(lib().tmg_sync(ctx), ctx)
        free1, _ = torch.cuda.mem_get_info()
        moved.append(free0 - free1)
        if free1 == free0:
            break
    assert moved[-1] == 0, moved


def test_noalloc_rejects_unsupported_head_dim(ctx):
    n_ctx, nq, nkv, d = 16, 4, 2, 48
    q, k, v = inputs(n_ctx, nq, nkv, d, 3)
    out = torch.zeros(nq * d, device="cuda")
    with pytest.raises(TmgError) as ei:
        check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(out)),
              ctx)
    assert ei.value.code == TMG_ERR_INVALID
    check(lib().tmg_sync(ctx), ctx)
    assert float(out.abs().max()) == 0.0  # nothing ran


def test_noalloc_rejects_oversized(ctx):
    # 16 kv heads x 8 queries x 74 splits x 130 floats > 4 MiB of partials.
    # The buffers are real and large enough, so even a wrongly accepted call
    # would stay in bounds.
    n_ctx, nq, nkv, d = 8192, 128, 16, 128
    q, k, v = inputs(n_ctx, nq, nkv, d, 9)
    out = torch.zeros(nq * d, device="cuda")
    with pytest.raises(TmgError) as ei:
        check(lib().tmg_op_attn_decode_noalloc(ctx, P(q), P(k), P(v), n_ctx, nq, nkv, d, P(out)),
              ctx)
    assert ei.value.code == TMG_ERR_CAPACITY
    assert "static scratch" in str(ei.value)
    check(lib().tmg_sync(ctx), ctx)
    assert float(out.abs().max()) == 0.0  # nothing ran
