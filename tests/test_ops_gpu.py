"""sm_100a kernels at sizes past the conformance cases: the 3xTF32 tcgen05 GEMM against a float64 reference with the
tolerance of ProjectAI.Tests/MatMulTests.cs:20-45 (rtol 1e-4, atol 1e-5), the fused extensions against the
reference's composed rules, and the bit-exact paths (gather, scatter-add, AdamW) against the oracle."""
import numpy as np
import pytest

from projectai_b200 import cabi

pytestmark = pytest.mark.gpu


def rnd(seed, *shape, scale=1.0):
    return (np.random.RandomState(seed).standard_normal(shape) * scale).astype(np.float32)


def assert_close(expected, got, rtol, atol, what):
    expected = np.asarray(expected, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64)
    assert expected.shape == got.shape, f"{what}: shape {got.shape} vs {expected.shape}"
    tol = atol + rtol * np.abs(expected)
    err = np.abs(expected - got)
    bad = np.argwhere(err > tol)
    assert bad.size == 0, f"{what}: {len(bad)} mismatches, first at {tuple(bad[0])}: {got[tuple(bad[0])]} vs {expected[tuple(bad[0])]}"


# ---------------------------------------------------------------- GEMM
@pytest.mark.parametrize("m,k,n,tb", [(257, 300, 129, False), (128, 64, 256, True), (1, 7, 3, False),
                                      (384, 5632, 512, True), (1000, 768, 2304, True), (300, 33, 1000, False)])
def test_matmul_matches_float64(cuda, m, k, n, tb):
    a = rnd(1, m, k)
    b = rnd(2, n, k) if tb else rnd(2, k, n)
    got = cuda.to_host(cuda.matmul(cuda.from_host(a), cuda.from_host(b), transpose_b=tb))
    ref = a.astype(np.float64) @ (b.astype(np.float64).T if tb else b.astype(np.float64))
    # |a|·|b| bounds the rounding of each dot product; the reference tolerance is relative to the result.
    scale = np.abs(a).astype(np.float64) @ (np.abs(b).T if tb else np.abs(b)).astype(np.float64)
    assert_close(ref, got, 1e-4, 1e-5 + 1e-6 * scale.max(), f"matmul {m}x{k}x{n} tb={tb}")


# Products the two-CTA kernel takes (more than one round of 128 x 256 tiles, no K split): K-major operands feed their
# raw fp32 tiles as hi through a tensor map and get a lo-only pack. Covered: a k tail (k = 100 reads zeros past the
# edge), row and column tails of the 256-row tiles, a column-slice view with a 16-byte aligned start (raw) and one
# with an unaligned start (packed hi and lo), and an MN-major B beside a raw A.
@pytest.mark.parametrize("m,k,n,tb,col0", [(2048, 100, 2048, True, 0), (1536, 256, 1000, True, 0),
                                           (2048, 768, 2048, True, 32), (2048, 768, 2048, True, 1),
                                           (2048, 256, 2048, False, 0)])
def test_matmul_pair_kernel_raw_operands(cuda, m, k, n, tb, col0):
    full = rnd(11, m, k + col0 + 8)
    a = full[:, col0:col0 + k]
    b = rnd(12, n, k) if tb else rnd(12, k, n)
    ta = cabi.slice_view(cuda.from_host(full), 1, col0, k)
    got = cuda.to_host(cuda.matmul(ta, cuda.from_host(b), transpose_b=tb))
    bt = b.astype(np.float64).T if tb else b.astype(np.float64)
    ref = a.astype(np.float64) @ bt
    scale = np.abs(a).astype(np.float64) @ np.abs(bt)
    assert_close(ref, got, 1e-4, 1e-5 + 1e-6 * scale.max(), f"pair matmul {m}x{k}x{n} tb={tb} col0={col0}")


def test_matmul_strided_operands_and_deep_k(cuda):
    # Weight-gradient shape: dW = dYᵀ·X with both operands as transposed views (MN-major), K = 8192 (split-K path).
    dy = rnd(3, 8192, 384, scale=0.05)
    x = rnd(4, 8192, 256)
    tdy, tx = cuda.from_host(dy), cuda.from_host(x)
    got = cuda.to_host(cuda.matmul(cabi.transpose(tdy, 0, 1), tx))
    ref = dy.astype(np.float64).T @ x.astype(np.float64)
    scale = np.abs(dy).astype(np.float64).T @ np.abs(x).astype(np.float64)
    assert_close(ref, got, 1e-4, 1e-6 * scale.max(), "dW = dYᵀ·X")


def test_matmul_batch_broadcast_gqa(cuda, oracle):
    a = rnd(5, 2, 4, 2, 33, 16)
    b = rnd(6, 2, 4, 1, 40, 16)
    got = cuda.to_host(cuda.matmul(cuda.from_host(a), cuda.from_host(b), transpose_b=True))
    exp = oracle.to_host(oracle.matmul(oracle.from_host(a), oracle.from_host(b), transpose_b=True))
    assert_close(exp, got, 1e-4, 1e-4, "gqa batch broadcast")


def test_matmul_offset_slice(cuda):
    a = rnd(7, 6, 130, 70)
    b = rnd(8, 70, 50)
    ta = cabi.slice_view(cuda.from_host(a), 0, 2, 3)
    got = cuda.to_host(cuda.matmul(ta, cuda.from_host(b)))
    ref = a[2:5].astype(np.float64) @ b.astype(np.float64)
    assert_close(ref, got, 1e-4, 1e-4, "sliced batch")


# ---------------------------------------------------------------- attention
def attention_ref(q, k, v, scale, pos_offset):
    """float64 statement of Modules.cs:169-203 and its gradient (GQA, causal)."""
    B, H, S, D = q.shape
    KVH, L = k.shape[1], k.shape[2]
    g = H // KVH
    q64, k64, v64 = (x.astype(np.float64) for x in (q, k, v))
    kk = np.repeat(k64, g, axis=1)
    vv = np.repeat(v64, g, axis=1)
    qs = q64 * scale
    s = qs @ np.swapaxes(kk, -1, -2)
    mask = np.arange(L)[None, :] <= (pos_offset + np.arange(S))[:, None]
    s = np.where(mask, s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o = p @ vv
    return o, p, qs, kk, vv


def attention_grads(q, k, v, do, scale, pos_offset):
    o, p, qs, kk, vv = attention_ref(q, k, v, scale, pos_offset)
    B, H, S, D = q.shape
    KVH = k.shape[1]
    g = H // KVH
    do64 = do.astype(np.float64)
    dv = np.swapaxes(p, -1, -2) @ do64
    dp = do64 @ np.swapaxes(vv, -1, -2)
    ds = p * (dp - (dp * p).sum(-1, keepdims=True))
    dq = (ds @ kk) * scale
    dk = np.swapaxes(ds, -1, -2) @ qs
    dk = dk.reshape(B, KVH, g, *dk.shape[2:]).sum(2)
    dv = dv.reshape(B, KVH, g, *dv.shape[2:]).sum(2)
    return o, dq, dk, dv


@pytest.mark.parametrize("B,H,KVH,S,L,D,off", [(2, 4, 2, 70, 70, 32, 0), (1, 2, 1, 1, 9, 16, 8), (1, 4, 4, 5, 12, 8, 7),
                                               (2, 12, 12, 130, 130, 64, 0), (1, 8, 2, 64, 64, 64, 0),
                                               # keys 164..299 are visible to no query: their dK/dV rows must be zeros
                                               (1, 2, 1, 64, 300, 64, 100)])
def test_sdpa_forward_backward(cuda, B, H, KVH, S, L, D, off):
    q = rnd(10, B, H, S, D)
    k = rnd(11, B, KVH, L, D)
    v = rnd(12, B, KVH, L, D)
    do = rnd(13, B, S, H, D)
    scale = 1.0 / np.sqrt(D)
    o_ref, dq_ref, dk_ref, dv_ref = attention_grads(q, k, v, np.swapaxes(do, 1, 2), scale, off)
    tq, tk, tv = cuda.from_host(q), cuda.from_host(k), cuda.from_host(v)
    out, lse = cuda.sdpa_fwd(tq, tk, tv, scale, True, off)
    got = cuda.to_host(out)  # [B,S,H,D]
    assert_close(np.swapaxes(o_ref, 1, 2), got, 1e-4, 1e-4, "sdpa out")
    dq, dk, dv = cuda.sdpa_bwd(tq, tk, tv, out, lse, cuda.from_host(do), scale, True, off)
    assert_close(dq_ref, cuda.to_host(dq), 1e-4, 1e-4, "dq")
    assert_close(dk_ref, cuda.to_host(dk), 1e-4, 1e-4, "dk")
    assert_close(dv_ref, cuda.to_host(dv), 1e-4, 1e-4, "dv")


def test_sdpa_strided_inputs(cuda):
    # q as the transposed view the model produces: [B,S,H,D] storage viewed as [B,H,S,D].
    B, S, H, D = 2, 40, 4, 32
    qs = rnd(20, B, S, H, D)
    k = rnd(21, B, H, S, D)
    v = rnd(22, B, H, S, D)
    tq = cabi.transpose(cuda.from_host(qs), 1, 2)
    out, _ = cuda.sdpa_fwd(tq, cuda.from_host(k), cuda.from_host(v), 0.2, True, 0)
    o_ref = attention_ref(np.swapaxes(qs, 1, 2), k, v, 0.2, 0)[0]
    assert_close(np.swapaxes(o_ref, 1, 2), cuda.to_host(out), 1e-4, 1e-4, "strided q")


# ---------------------------------------------------------------- fused row ops
def test_rmsnorm_backward(cuda):
    x = rnd(30, 67, 768)
    w = rnd(31, 768)
    g = rnd(32, 67, 768)
    eps = 1e-5
    x64, w64, g64 = (a.astype(np.float64) for a in (x, w, g))
    inv = 1 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + eps)
    y = x64 * inv * w64
    dot = (g64 * y).sum(-1, keepdims=True)
    dx_ref = inv * g64 * w64 - inv ** 2 / 768 * x64 * dot
    dw_ref = (g64 * x64 * inv).sum(0)
    dx, dw = cuda.rmsnorm_bwd(cuda.from_host(x), cuda.from_host(w), cuda.from_host(g), eps)
    assert_close(dx_ref, cuda.to_host(dx), 1e-4, 1e-4, "rmsnorm dx")
    assert_close(dw_ref, cuda.to_host(dw), 1e-4, 1e-4, "rmsnorm dw")


def test_silu_mul(cuda, oracle):
    gate = rnd(40, 33, 344)
    up = rnd(41, 33, 344)
    g = rnd(42, 33, 344)
    exp = oracle.to_host(oracle.mul(oracle.silu(oracle.from_host(gate)), oracle.from_host(up)))
    got = cuda.to_host(cuda.silu_mul_fwd(cuda.from_host(gate), cuda.from_host(up)))
    assert_close(exp, got, 1e-6, 1e-6, "silu_mul fwd")
    g64, a64, u64 = (x.astype(np.float64) for x in (g, gate, up))
    s = 1 / (1 + np.exp(-a64))
    dg_ref = g64 * u64 * (s + a64 * s - s * a64 * s)
    du_ref = g64 * a64 * s
    dg, du = cuda.silu_mul_bwd(cuda.from_host(gate), cuda.from_host(up), cuda.from_host(g))
    assert_close(dg_ref, cuda.to_host(dg), 1e-5, 1e-6, "silu_mul dgate")
    assert_close(du_ref, cuda.to_host(du), 1e-5, 1e-6, "silu_mul dup")


# (1000, 32000) and (300, 20000): more rows than SMs, so each CTA of the streaming kernel walks several rows with the
# next row's copy in flight; (150, 30002): a row length that is not a whole number of 16-byte units (register kernel).
@pytest.mark.parametrize("n,vocab", [(37, 256), (64, 32000), (9, 40000), (1000, 32000), (300, 20000), (150, 30002),
                                     (1, 32768), (200, 16388)])
def test_cross_entropy_fused(cuda, oracle, n, vocab):
    logits = rnd(50, n, vocab, scale=3.0)
    targets = np.random.RandomState(51).randint(0, vocab, size=n).astype(np.int32)
    targets[3:4] = -100
    targets[97::149] = -100  # ignored rows between streamed ones
    exp_loss = oracle.to_host(oracle.cross_entropy(oracle.from_host(logits), targets, -100))
    exp_grad = oracle.to_host(oracle.cross_entropy_grad(oracle.from_host(logits), targets, -100))
    loss, grad = cuda.cross_entropy_fused(cuda.from_host(logits), targets, -100, 1.0)
    assert_close(exp_loss, cuda.to_host(loss), 1e-5, 1e-6, "ce loss")
    assert_close(exp_grad, cuda.to_host(grad), 1e-4, 1e-7, "ce grad")
    assert_close(exp_loss, cuda.to_host(cuda.cross_entropy(cuda.from_host(logits), targets, -100)), 1e-5, 1e-6, "ce")
    assert_close(exp_grad, cuda.to_host(cuda.cross_entropy_grad(cuda.from_host(logits), targets, -100)), 1e-4, 1e-7, "ce grad")


def test_cross_entropy_every_row_ignored(cuda, oracle):
    """No counted row (CpuComputeBackend.cs:472, :480): the loss is 0 and the gradient all zeros, on the streaming
    path (rows of whole 16-byte units, more rows than SMs) as on the others."""
    for n, vocab in ((400, 32000), (5, 30002)):
        logits = rnd(54, n, vocab)
        targets = np.full(n, -100, np.int32)
        loss, grad = cuda.cross_entropy_fused(cuda.from_host(logits), targets, -100, 1.0)
        assert float(cuda.to_host(loss).reshape(-1)[0]) == 0.0
        assert not np.any(cuda.to_host(grad))
        assert float(oracle.to_host(oracle.cross_entropy(oracle.from_host(logits), targets, -100)).reshape(-1)[0]) == 0.0


def test_cross_entropy_streamed_rows_equal_register_rows(cuda):
    """Logits whose rows start on 16-byte boundaries take the streaming kernel (next row copied into shared memory
    while the current one is reduced); the same logits one float off that boundary take the register kernel. Both
    compute each row in the same order, so loss and gradient agree bit for bit."""
    n, vocab = 700, 32000
    logits = rnd(52, n, vocab, scale=3.0)
    targets = np.random.RandomState(53).randint(0, vocab, size=n).astype(np.int32)
    targets[5::151] = -100
    flat = np.concatenate([np.zeros(1, np.float32), logits.reshape(-1)])
    shifted = cabi.reshape(cabi.slice_view(cuda.from_host(flat), 0, 1, n * vocab), [n, vocab])
    loss_a, grad_a = cuda.cross_entropy_fused(cuda.from_host(logits), targets, -100, 1.0)
    loss_b, grad_b = cuda.cross_entropy_fused(shifted, targets, -100, 1.0)
    assert np.array_equal(cuda.to_host(loss_a).view(np.uint32), cuda.to_host(loss_b).view(np.uint32))
    assert np.array_equal(cuda.to_host(grad_a).view(np.uint32), cuda.to_host(grad_b).view(np.uint32))


# ---------------------------------------------------------------- bit-exact paths
def test_gather_scatter_bit_exact(cuda, oracle):
    rows = rnd(60, 500, 96)
    ids = np.random.RandomState(61).randint(0, 50, size=500).astype(np.int32)  # heavy repetition
    exp = oracle.to_host(oracle.scatter_add_rows(oracle.from_host(rows), ids, 50))
    got = cuda.to_host(cuda.scatter_add_rows(cuda.from_host(rows), ids, 50))
    assert np.array_equal(exp.view(np.uint32), got.view(np.uint32))
    table = rnd(62, 50, 96)
    exp = oracle.to_host(oracle.gather(oracle.from_host(table), ids))
    got = cuda.to_host(cuda.gather(cuda.from_host(table), ids))
    assert np.array_equal(exp, got)


def test_adamw_bit_exact_with_composed_reference(cuda, oracle):
    """The fused update equals the ~15 composed ops of Optimizers.cs:81-123 bit for bit."""
    n = 10007
    p, g = rnd(70, n), rnd(71, n, scale=0.1)
    m, v = rnd(72, n, scale=0.01), np.abs(rnd(73, n, scale=0.001))
    lr, b1, b2, eps, wd, t = 3e-4, 0.9, 0.95, 1e-8, 0.1, 3
    # composed on the oracle, exactly as Optimizers.cs does it
    o = oracle
    P, G, M, V = (o.from_host(x) for x in (p, g, m, v))
    m2 = o.add(o.mul_scalar(M, b1), o.mul_scalar(G, np.float32(1) - np.float32(b1)))
    v2 = o.add(o.mul_scalar(V, b2), o.mul_scalar(o.mul(G, G), np.float32(1) - np.float32(b2)))
    bc1 = np.float32(1) - np.power(np.float32(b1), np.float32(t), dtype=np.float32)
    bc2 = np.float32(1) - np.power(np.float32(b2), np.float32(t), dtype=np.float32)
    mhat = o.mul_scalar(m2, np.float32(1) / bc1)
    vhat = o.mul_scalar(v2, np.float32(1) / bc2)
    adaptive = o.div(mhat, o.add_scalar(o.sqrt(vhat), eps))
    delta = o.add(o.mul_scalar(adaptive, lr), o.mul_scalar(P, np.float32(lr) * np.float32(wd)))
    p_ref = o.to_host(o.sub(P, delta))
    c = cuda
    P2, G2, M2, V2 = (c.from_host(x) for x in (p, g, m, v))
    c.adamw_step(P2, G2, M2, V2, lr, b1, b2, eps, wd, t)
    assert np.array_equal(p_ref.view(np.uint32), c.to_host(P2).view(np.uint32))
    assert np.array_equal(o.to_host(m2).view(np.uint32), c.to_host(M2).view(np.uint32))
    assert np.array_equal(o.to_host(v2).view(np.uint32), c.to_host(V2).view(np.uint32))


def test_errors_match_reference_exceptions(cuda):
    t = cuda.from_host(rnd(80, 6, 4))
    with pytest.raises(cabi.OutOfRangeError):
        cuda.gather(t, [0, 6])
    with pytest.raises(cabi.OutOfRangeError):
        cuda.cross_entropy(t, [0, 1, 2, 3, 4, 9], -100)
    with pytest.raises(cabi.ArgumentError):
        cuda.matmul(t, cuda.from_host(rnd(81, 5, 3)))
    with pytest.raises(cabi.OutOfRangeError):
        cuda.sum(t, 2)


def test_scopes_free_and_keep_alive(cuda):
    base_in_use = cuda.memory_stats()[0]
    cuda.scope_begin()
    a = cuda.from_host(rnd(90, 1000))
    b = cuda.add_scalar(a, 1.0)
    cuda.keep_alive(b)
    cuda.scope_end()
    assert cuda.memory_stats()[0] > base_in_use  # b survived
    np.testing.assert_allclose(cuda.to_host(b), rnd(90, 1000) + 1, rtol=1e-6)
    with pytest.raises(cabi.InvalidOperationError):
        cuda.to_host(a)  # a was freed with its scope
    cuda.release(b)
    assert cuda.memory_stats()[0] == base_in_use
    assert cuda.check_device_error() == 0
