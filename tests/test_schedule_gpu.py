"""The persistent tensor-core kernels on their production schedule: every launch here hands each of the GPU's CTAs
several work items (at least 3 x the SM count), so a CTA walks a second, third, ... tile through the same TMEM
accumulator double buffer, the same running mbarrier phases and, for attention, the snake order over the
longest-first item list. The shapes are the 125M and 1B training shapes (linear layers, the tied LM head, weight
gradients through transposed views, causal GQA attention at seq 1024 and 2048).

References are float64, computed with torch on the same GPU (cuBLAS DGEMM and float64 elementwise ops):
* GEMM: |e - g| <= 1e-5 + 1e-6·max(|a|·|b|ᵀ) + 1e-4·|e|, the form of tests/test_ops_gpu.py (MatMulTests.cs:20-45,
  rtol 1e-4, atol 1e-5, widened by the rounding scale of K-long dot products);
* attention: |e - g| <= 1e-4 + 1e-4·|e| (AttentionTests.cs:83-141).
"""
import numpy as np
import pytest

from projectai_b200 import cabi
from test_ops_gpu import rnd

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev():
    return torch.device("cuda", 0)


def t64(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev(), torch.float64)


def check(expected, got, rtol, atol, what):
    """expected: float64 torch tensor on the GPU; got: numpy float32 from the backend."""
    g = t64(got)
    assert tuple(expected.shape) == tuple(g.shape), f"{what}: shape {tuple(g.shape)} vs {tuple(expected.shape)}"
    err = (expected - g).abs()
    bad = err > atol + rtol * expected.abs()
    n_bad = int(bad.sum())
    if n_bad:
        idx = tuple(int(i) for i in torch.nonzero(bad)[0])
        pytest.fail(f"{what}: {n_bad} of {expected.numel()} outside tolerance; first at {idx}: got {float(g[idx])} "
                    f"expected {float(expected[idx])} (worst |e-g| {float(err.max()):.3e})")


def sm_count():
    return torch.cuda.get_device_properties(0).multi_processor_count


# ---------------------------------------------------------------- GEMM: more tiles than CTAs
# (m, k, n, transpose_b, scale of a): 125M gate/up projection, 1B gate/up projection, the tied LM head at 125M, the
# down-projection input gradient dX = dY·W (B not transposed: an MN-major operand)
@pytest.mark.parametrize("m,k,n,tb", [(8192, 768, 2048, True), (8192, 2048, 5632, True), (8192, 768, 32000, True),
                                      (8192, 5632, 2048, False)])
def test_gemm_multi_tile_schedule(cuda, m, k, n, tb):
    tiles = -(-m // 128) * -(-n // 256)
    assert tiles >= 3 * sm_count(), "the case must give every CTA several tiles"
    a = rnd(101, m, k)
    b = rnd(102, n, k, scale=0.05) if tb else rnd(102, k, n, scale=0.05)
    got = cuda.to_host(cuda.matmul(cuda.from_host(a), cuda.from_host(b), transpose_b=tb))
    ta, tb64 = t64(a), t64(b)
    bt = tb64.T if tb else tb64
    ref = ta @ bt
    scale = float((ta.abs() @ bt.abs()).max())
    del ta, tb64, bt
    check(ref, got, 1e-4, 1e-5 + 1e-6 * scale, f"matmul {m}x{k}x{n} tb={tb}")


@pytest.mark.parametrize("m,k,n", [(5632, 8192, 2048), (2048, 8192, 2048)])
def test_gemm_weight_gradient_transposed_views(cuda, m, k, n):
    """dW = dYᵀ·X over the 8192 tokens of a step, both operands transposed views of row-major activations."""
    dy = rnd(103, k, m, scale=0.05)
    x = rnd(104, k, n)
    got = cuda.to_host(cuda.matmul(cabi.transpose(cuda.from_host(dy), 0, 1), cuda.from_host(x)))
    tdy, tx = t64(dy), t64(x)
    ref = tdy.T @ tx
    scale = float((tdy.abs().T @ tx.abs()).max())
    del tdy, tx
    check(ref, got, 1e-4, 1e-5 + 1e-6 * scale, f"dW {m}x{k}x{n}")


# ---------------------------------------------------------------- attention: more query tiles than CTAs
def attention_f64(q, k, v, do, scale, pos_offset):
    """float64 statement of Modules.cs:169-203 (GQA, causal) and its gradient, one batch element at a time.
    q [B,H,S,D], k/v [B,KVH,L,D], do [B,S,H,D]. Returns out [B,S,H,D], lse [B,H,S], dq, dk, dv."""
    B, H, S, D = q.shape
    KVH, L = k.shape[1], k.shape[2]
    g = H // KVH
    outs, lses, dqs, dks, dvs = [], [], [], [], []
    mask = torch.arange(L, device=dev())[None, :] <= (pos_offset + torch.arange(S, device=dev()))[:, None]
    for b in range(B):
        qb, kb, vb = t64(q[b]), t64(k[b]).repeat_interleave(g, 0), t64(v[b]).repeat_interleave(g, 0)
        dob = t64(do[b]).transpose(0, 1)  # [H,S,D]
        qs = qb * scale
        s = qs @ kb.transpose(-1, -2)
        s = torch.where(mask, s, torch.tensor(float("-inf"), device=dev(), dtype=torch.float64))
        mx = s.max(-1, keepdim=True).values
        e = torch.exp(s - mx)
        den = e.sum(-1, keepdim=True)
        p = e / den
        del e, s
        o = p @ vb
        lses.append((mx + torch.log(den))[..., 0])
        outs.append(o.transpose(0, 1))
        dvh = p.transpose(-1, -2) @ dob
        dp = dob @ vb.transpose(-1, -2)
        ds = p * (dp - (dp * p).sum(-1, keepdim=True))
        del dp, p
        dqs.append((ds @ kb) * scale)
        dkh = ds.transpose(-1, -2) @ qs
        del ds
        dks.append(dkh.reshape(KVH, g, L, D).sum(1))
        dvs.append(dvh.reshape(KVH, g, L, D).sum(1))
    return (torch.stack(outs), torch.stack(lses), torch.stack(dqs), torch.stack(dks), torch.stack(dvs))


# (B, H, KVH, S, L, pos_offset): the 125M attention (8 x 12 heads, seq 1024: 768 query tiles), the 1B attention
# (4 x 32 heads over 8 kv heads, seq 2048: 2048 query tiles), and a prefill over a cached prefix (keys beyond the
# queries, 3 x 128-query tiles per head)
@pytest.mark.parametrize("B,H,KVH,S,L,off", [(8, 12, 12, 1024, 1024, 0), (4, 32, 8, 2048, 2048, 0),
                                              (2, 32, 8, 384, 1408, 1024)])
def test_attention_multi_tile_schedule(cuda, B, H, KVH, S, L, off):
    D = 64
    items = B * H * -(-S // 128)
    assert items >= 3 * sm_count() or S < 512, "the case must give every CTA several query tiles"
    q, k, v = rnd(110, B, H, S, D), rnd(111, B, KVH, L, D), rnd(112, B, KVH, L, D)
    do = rnd(113, B, S, H, D)
    scale = 1.0 / np.sqrt(D)
    tq, tk, tv = cuda.from_host(q), cuda.from_host(k), cuda.from_host(v)
    out, lse = cuda.sdpa_fwd(tq, tk, tv, scale, True, off)
    dq, dk, dv = cuda.sdpa_bwd(tq, tk, tv, out, lse, cuda.from_host(do), scale, True, off)
    got = [cuda.to_host(t) for t in (out, lse, dq, dk, dv)]
    assert cuda.check_device_error() == 0
    ref = attention_f64(q, k, v, do, scale, off)
    for name, e, g in zip(("out", "lse", "dq", "dk", "dv"), ref, got):
        check(e, g, 1e-4, 1e-4, f"attention {name} B{B} H{H}/{KVH} S{S} L{L}")
