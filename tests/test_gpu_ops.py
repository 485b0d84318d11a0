"""Op-level parity of the CUDA kernels (through the C ABI) with the CPU oracle.

Tolerances: the kernels compute in f32 but reassociate sums (warp shuffles,
split-K, online softmax), so a value may differ from the oracle's by a few
ulps of the sum of the absolute terms: |y - y_ref| <= 2e-6 * sum|x_i w_i|
(+ a tiny absolute floor).  RoPE is bit-exact (same table, same rounding);
argmax and top-k/top-p candidate selection are bit-exact on identical
logits; sampled probabilities agree within 1e-6 relative (exp rounding).
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


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def bf16(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def widen(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def bound(x, w):
    return 2e-6 * (np.abs(x) @ np.abs(widen(w)).T) + 1e-30


@pytest.mark.parametrize("N,K,M", [(3072, 2048, 1), (2048, 2048, 1), (2048, 8192, 1),
                                   (16384, 2048, 1), (4096, 14336, 1), (1792, 1024, 1),
                                   (17, 64, 1), (5, 4, 1), (300, 200, 3), (1000, 2048, 16),
                                   (128256, 2048, 1)])
def test_gemv(ctx, orc, N, K, M):
    rng = np.random.default_rng(N * 7 + K + M)
    w = bf16(rng.normal(0, 0.02, (N, K)))
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    wd, xd = dev(w.view(np.int16)), dev(x)
    yd = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    check(lib().tmg_op_gemv_bf16(ctx, P(xd), P(wd), N, K, M, P(yd)), ctx)
    y = yd.cpu().numpy()
    for m in range(M):
        ref = orc.matmul_w(x[m], w)
        assert np.all(np.abs(y[m] - ref) <= bound(x[m], w)), (m, np.max(np.abs(y[m] - ref)))


# (2048, 3072, 1024): 192-wide tiles, two rounds of the persistent grid (both
# TMEM accumulators in turn); (1000, 4100, 512): partial row and column tiles
# over several rounds
@pytest.mark.parametrize("T,N,K", [(37, 300, 256), (128, 3072, 2048), (1, 64, 64), (5, 9, 13),
                                   (2048, 3072, 1024), (1000, 4100, 512)])
def test_gemm_prefill(ctx, orc, T, N, K):
    rng = np.random.default_rng(T + N + K)
    w = bf16(rng.normal(0, 0.02, (N, K)))
    x = rng.normal(0, 1, (T, K)).astype(np.float32)
    yd = torch.zeros((T, N), dtype=torch.float32, device="cuda")
    xd, wd = dev(x), dev(w.view(np.int16))
    check(lib().tmg_op_gemm_bf16(ctx, P(xd), P(wd), N, K, T, P(yd)), ctx)
    y = yd.cpu().numpy()
    ref = orc.matmul_batch_w(x, w) if T >= 2 else orc.matmul_w(x[0], w)[None]
    assert np.all(np.abs(y - ref) <= bound(x, w))


def test_wmat_handle(ctx, orc):
    # WMat as a device handle (src/tensor.rs:198-206): upload once from host
    # memory, then matmul_w_into (M rows) and matmul_batch_w_into over it
    from tinyminigo_b200._lib import TmgError

    rng = np.random.default_rng(77)
    N, K = 1536, 2048
    w = bf16(rng.normal(0, 0.02, (N, K)))
    h = ctypes.c_void_p()
    check(lib().tmg_wmat_upload_bf16(ctx, w.ctypes.data_as(ctypes.c_void_p), N, K,
                                     ctypes.byref(h)), ctx)
    r, c = ctypes.c_int64(), ctypes.c_int64()
    check(lib().tmg_wmat_shape(h, ctypes.byref(r), ctypes.byref(c)))
    assert (r.value, c.value) == (N, K)
    w[:] = 0  # the handle holds its own copy
    w = bf16(np.random.default_rng(77).normal(0, 0.02, (N, K)))
    x = rng.normal(0, 1, (3, K)).astype(np.float32)
    xd = dev(x)
    yd = torch.zeros((3, N), dtype=torch.float32, device="cuda")
    check(lib().tmg_op_gemv_wmat(ctx, P(xd), h, 3, P(yd)), ctx)
    y = yd.cpu().numpy()
    for m in range(3):
        assert np.all(np.abs(y[m] - orc.matmul_w(x[m], w)) <= bound(x[m], w))
    T = 40
    xt = rng.normal(0, 1, (T, K)).astype(np.float32)
    xtd = dev(xt)
    ytd = torch.zeros((T, N), dtype=torch.float32, device="cuda")
    check(lib().tmg_op_gemm_wmat(ctx, P(xtd), h, T, P(ytd)), ctx)
    assert np.all(np.abs(ytd.cpu().numpy() - orc.matmul_batch_w(xt, w)) <= bound(xt, w))
    check(lib().tmg_wmat_free(h))
    with pytest.raises(TmgError):
        check(lib().tmg_wmat_upload_bf16(ctx, w.ctypes.data_as(ctypes.c_void_p), 0, K,
                                         ctypes.byref(h)), ctx)


@pytest.mark.parametrize("mode", [0, 1])
def test_rmsnorm(ctx, orc, mode):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (4, 2048)).astype(np.float32)
    w = rng.normal(1, 0.1, 2048).astype(np.float32)
    od = torch.zeros_like(dev(x))
    xd, wd = dev(x), dev(w)
    check(lib().tmg_op_rmsnorm(ctx, P(xd), P(wd), 1e-5, 2048, 4, mode, P(od)), ctx)
    ref = np.stack([orc.rms_norm(r, w, 1e-5) for r in x]) if mode == 0 else orc.rms_norm_batch(x, w, 1e-5)
    assert np.allclose(od.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("d,theta", [(16, 10000.0), (64, 500000.0), (128, 500000.0)])
def test_rope_bit_exact(ctx, orc, d, theta):
    rng = np.random.default_rng(d)
    heads, rows, pos0 = 3, 40, 33000
    x = rng.normal(0, 1, (rows, heads * d)).astype(np.float32)
    xd = dev(x)
    check(lib().tmg_op_rope(ctx, P(xd), rows, heads, d, pos0, theta), ctx)
    got = xd.cpu().numpy()
    for r in range(rows):
        assert np.array_equal(got[r], orc.rope_table_rotate(x[r], heads, d, pos0 + r, theta))


def test_swiglu(ctx, orc):
    rng = np.random.default_rng(4)
    g = rng.normal(0, 3, 10000).astype(np.float32)
    u = rng.normal(0, 1, 10000).astype(np.float32)
    od = torch.zeros(10000, dtype=torch.float32, device="cuda")
    gd, ud = dev(g), dev(u)
    check(lib().tmg_op_swiglu(ctx, P(gd), P(ud), 10000, P(od)), ctx)
    ref = np.array([orc.silu(float(a)) for a in g], np.float32) * u
    assert np.allclose(od.cpu().numpy(), ref, rtol=1e-6, atol=1e-30)


def attn_bound(q, keys, vals):
    return 1e-5 * (np.abs(vals).max() + 1e-6)


@pytest.mark.parametrize("n_ctx,nq,nkv,d", [(1, 4, 2, 16), (5, 4, 4, 64), (33, 32, 8, 64),
                                             (300, 32, 8, 64), (2000, 8, 2, 128),
                                             (4097, 4, 1, 64), (77, 12, 4, 32),
                                             (600, 16, 2, 64), (130, 16, 1, 64)])
def test_attn_decode(ctx, orc, n_ctx, nq, nkv, d):
    rng = np.random.default_rng(n_ctx + d)
    q = rng.normal(0, 1, nq * d).astype(np.float32)
    keys = rng.normal(0, 1, (n_ctx, nkv * d)).astype(np.float32)
    vals = rng.normal(0, 1, (n_ctx, nkv * d)).astype(np.float32)
    od = torch.zeros(nq * d, dtype=torch.float32, device="cuda")
    qd, kd, vd = dev(q), dev(keys), dev(vals)
    check(lib().tmg_op_attn_decode(ctx, P(qd), P(kd), P(vd), n_ctx, nq, nkv, d, P(od)), ctx)
    ref = orc.attention_batch(q, keys, vals, nq, nkv, d, n_ctx - 1)[0]
    assert np.max(np.abs(od.cpu().numpy() - ref)) < attn_bound(q, keys, vals)


# head dim 64 runs the register-tiled kernel (64-row blocks, 64-key tiles):
# partial row blocks, starts inside a key tile, one row, GQA groups of 1-8
@pytest.mark.parametrize("T,start,nq,nkv,d", [(1, 0, 4, 2, 16), (50, 0, 4, 2, 16),
                                               (50, 7, 32, 8, 64), (70, 3, 8, 2, 128),
                                               (200, 0, 32, 8, 64), (130, 61, 32, 8, 64),
                                               (1, 5, 4, 2, 64), (64, 0, 4, 4, 64),
                                               (257, 100, 16, 2, 64), (600, 1000, 8, 1, 64)])
def test_attn_prefill(ctx, orc, T, start, nq, nkv, d):
    rng = np.random.default_rng(T + start + d)
    q = rng.normal(0, 1, (T, nq * d)).astype(np.float32)
    keys = rng.normal(0, 1, (start + T, nkv * d)).astype(np.float32)
    vals = rng.normal(0, 1, (start + T, nkv * d)).astype(np.float32)
    od = torch.zeros((T, nq * d), dtype=torch.float32, device="cuda")
    qd, kd, vd = dev(q), dev(keys), dev(vals)
    check(lib().tmg_op_attn_prefill(ctx, P(qd), P(kd), P(vd), T, start, nq, nkv, d, P(od)), ctx)
    ref = orc.attention_batch(q, keys, vals, nq, nkv, d, start)
    assert np.max(np.abs(od.cpu().numpy() - ref)) < attn_bound(q, keys, vals)


def test_argmax_rules(ctx, orc):
    rows = [
        np.array([0.1, 3.0, 2.0], np.float32),
        np.array([2.0, 2.0], np.float32),  # tie -> lowest index
        np.array([np.nan, 1.0, np.nan], np.float32),  # NaN never wins
        np.array([-np.inf, -np.inf, -np.inf], np.float32),  # nothing wins -> 0
        np.array([-0.0, 0.0, -1.0], np.float32),
    ]
    for r in rows:
        out = torch.zeros(1, dtype=torch.int32, device="cuda")
        rd = dev(r)
        check(lib().tmg_op_argmax(ctx, P(rd), r.size, 1, P(out)), ctx)
        assert int(out.item()) == orc.argmax(r), r
    rng = np.random.default_rng(9)
    big = rng.normal(0, 1, (3, 128256)).astype(np.float32)
    big[1, 77] = big[1, 1000] = 50.0
    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    bd = dev(big)
    check(lib().tmg_op_argmax(ctx, P(bd), 128256, 3, P(out)), ctx)
    assert out.cpu().numpy().tolist() == [orc.argmax(r) for r in big]


def run_sample(ctx, logits, gen, T, k, p, pen, r):
    rows, V = logits.shape
    ld = dev(logits)
    gd = dev(np.asarray(gen, np.uint32).reshape(rows, -1).view(np.int32)) if len(gen) else None
    ud = dev(np.asarray(r, np.float32))
    nx = torch.zeros(rows, dtype=torch.int32, device="cuda")
    kk = max(k, 1)
    ci = torch.zeros((rows, kk), dtype=torch.int32, device="cuda")
    cp = torch.zeros((rows, kk), dtype=torch.float32, device="cuda")
    cut = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ng = len(gen) // rows if len(gen) else 0
    check(lib().tmg_op_sample(ctx, P(ld), V, rows, P(gd) if gd is not None else None, ng, T, k, p,
                              pen, P(ud), P(nx), P(ci), P(cp), P(cut)), ctx)
    return (nx.cpu().numpy().view(np.uint32), ci.cpu().numpy().view(np.uint32), cp.cpu().numpy(),
            cut.cpu().numpy(), ld.cpu().numpy())


@pytest.mark.parametrize("V,T,k,p,pen", [(128256, 0.8, 40, 0.95, 1.1), (128256, 1.0, 1, 1.0, 1.0),
                                         (32000, 0.5, 64, 0.5, 1.3), (1000, 1.2, 7, 1.0, 1.0),
                                         (128256, 0.8, 40, 0.95, 1.0)])
def test_sample_selection_bit_exact(ctx, orc, V, T, k, p, pen):
    rng = np.random.default_rng(V + k)
    rows = 3
    logits = (rng.normal(0, 1.5, (rows, V))).astype(np.float32)
    # ties across a slice boundary and inside the top-k
    logits[0, 5] = logits[0, 4100 % V] = logits[0, 90000 % V] = 9.0
    gen = rng.integers(0, V, (rows, 25)).astype(np.uint32)
    gen[:, 3] = gen[:, 0]  # repeated ids are penalised once
    gen[0, 1] = 5
    r = rng.random(rows).astype(np.float32)
    nx, ci, cp, cut, pen_logits = run_sample(ctx, logits, gen.reshape(-1), T, k, p, pen, r)
    for m in range(rows):
        ref_l = orc.apply_repetition_penalty(logits[m], gen[m], pen)
        assert np.array_equal(pen_logits[m], ref_l)
        idx, probs, c = orc.sample_select(ref_l, T, k, p)
        assert ci[m].tolist() == idx.tolist()
        assert int(cut[m]) == c
        assert np.allclose(cp[m], probs, rtol=1e-6, atol=0)
        assert int(nx[m]) == orc.sample(ref_l, T, k, p, float(r[m]))


def test_sample_greedy_with_penalty(ctx, orc):
    rng = np.random.default_rng(11)
    logits = rng.normal(0, 1, (2, 5000)).astype(np.float32)
    top = int(np.argmax(logits[0]))
    gen = np.array([[top, 3, 3], [1, 2, 3]], np.uint32)
    nx, _, _, _, _ = run_sample(ctx, logits, gen.reshape(-1), 0.0, 0, 1.0, 2.0, [0.5, 0.5])
    for m in range(2):
        ref_l = orc.apply_repetition_penalty(logits[m], gen[m], 2.0)
        assert int(nx[m]) == orc.argmax(ref_l)


def test_sample_reference_known_answers(ctx):
    # src/tensor.rs:1336-1364 on the device sampler
    l = np.array([[0.0, 5.0, 1.0, 4.0, 2.0]], np.float32)
    for r in np.linspace(0.0, 0.999, 25):
        nx, *_ = run_sample(ctx, l.copy(), [], 1.0, 2, 1.0, 1.0, [r])
        assert int(nx[0]) in (1, 3)
    l2 = np.array([[0.1, 0.2, 0.3, 0.4, 5.0]], np.float32)
    nx, *_ = run_sample(ctx, l2, [], 1.0, 4, 1.0, 1.0, [0.5])
    assert int(nx[0]) == 4


def test_sample_nan_is_an_error(ctx):
    l = np.ones((1, 300), np.float32)
    l[0, 7] = np.nan
    with pytest.raises(Exception, match="NaN"):
        run_sample(ctx, l, [], 1.0, 5, 1.0, 1.0, [0.3])
