"""Decode-path kernels through the C ABI: the weight-streaming x·Wᵀ product for at most 32 rows (gemv.cu) and the
split-KV decode attention over views of a preallocated KV cache (attention_decode.cu), each against float64
statements of the reference ops with the tolerance of ProjectAI.Tests/MatMulTests.cs:20-45 (rtol 1e-4) and the
attention tests (AttentionTests.cs:83-141, 1e-4)."""
import numpy as np
import pytest

from projectai_b200 import cabi
from test_ops_gpu import assert_close, attention_ref, rnd

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,k,n", [(1, 2048, 2048), (1, 2048, 512), (2, 768, 1000), (3, 5632, 2048), (8, 2048, 777),
                                      (17, 2048, 5632), (32, 2048, 4000), (2, 130, 99), (5, 1, 3),
                                      # tensor-core range (5..32 rows): ragged n and k, split-K and single-split grids
                                      (5, 100, 130), (12, 2052, 1000), (16, 5632, 2048), (24, 2048, 512),
                                      (32, 2048, 32000), (32, 36, 129),
                                      # stream-K partition: CTAs that cover several whole tiles, and tiles split over
                                      # many CTAs (finished by the last to arrive)
                                      (32, 32, 100000), (20, 96, 50000), (7, 2048, 300), (32, 5632, 2048)])
def test_gemv_matches_float64(cuda, rows, k, n):
    x = rnd(30, rows, k)
    w = rnd(31, n, k, scale=0.02)
    got = cuda.to_host(cuda.matmul(cuda.from_host(x), cuda.from_host(w), transpose_b=True))
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    scale = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T
    assert_close(ref, got, 1e-4, 1e-6 * scale.max(), f"gemv {rows}x{k}x{n}")


def test_gemv_batched_and_sliced_rows(cuda):
    # the decode Linear shape: [batch, 1, d] · Wᵀ, with x a slice of a larger activation buffer
    xs = rnd(32, 32, 3, 1024)
    w = rnd(33, 640, 1024, scale=0.02)
    tx = cabi.slice_view(cuda.from_host(xs), 1, 2, 1)  # [32, 1, 1024], batch stride 3·1024
    got = cuda.to_host(cuda.matmul(tx, cuda.from_host(w), transpose_b=True))
    ref = xs[:, 2:3].astype(np.float64) @ w.astype(np.float64).T
    assert got.shape == (32, 1, 640)
    assert_close(ref, got, 1e-4, 1e-5, "batched gemv")
    # W as a row slice of a larger matrix (offset and row stride)
    wbig = rnd(34, 700, 1100, scale=0.02)
    tw = cabi.slice_view(cabi.slice_view(cuda.from_host(wbig), 0, 30, 640), 1, 4, 1024)
    got = cuda.to_host(cuda.matmul(cuda.from_host(xs[:, 0]), tw, transpose_b=True))
    ref = xs[:, 0].astype(np.float64) @ wbig[30:670, 4:1028].astype(np.float64).T
    assert_close(ref, got, 1e-4, 1e-5, "gemv on a weight slice")


def lse_ref(q, k, scale, pos_offset):
    B, H, S, D = q.shape
    g = H // k.shape[1]
    kk = np.repeat(k.astype(np.float64), g, axis=1)
    s = (q.astype(np.float64) * scale) @ np.swapaxes(kk, -1, -2)
    mask = np.arange(k.shape[2])[None, :] <= (pos_offset + np.arange(S))[:, None]
    s = np.where(mask, s, -np.inf)
    mx = s.max(-1, keepdims=True)
    return (mx + np.log(np.exp(s - mx).sum(-1, keepdims=True)))[..., 0]


@pytest.mark.parametrize("B,H,KVH,S,L", [(1, 32, 8, 1, 1), (1, 32, 8, 1, 100), (4, 32, 8, 1, 1000), (2, 16, 4, 3, 517),
                                         (3, 12, 12, 1, 2000), (1, 8, 1, 2, 64),
                                         # 64+ (batch, kv head) pairs: the streaming kernel, up to 16 query rows
                                         (8, 32, 8, 1, 1000), (16, 16, 4, 3, 517), (64, 8, 1, 2, 300), (32, 64, 4, 1, 2048)])
def test_decode_attention_over_cache_views(cuda, B, H, KVH, S, L):
    D, max_seq = 64, 2048
    q = rnd(40, B, H, S, D)
    kc = rnd(41, B, KVH, max_seq, D)
    vc = rnd(42, B, KVH, max_seq, D)
    off = L - S
    scale = 1.0 / np.sqrt(D)
    # the cache holds max_seq positions; attention sees the filled prefix as a strided view
    tk = cabi.slice_view(cuda.from_host(kc), 2, 0, L)
    tv = cabi.slice_view(cuda.from_host(vc), 2, 0, L)
    out, lse = cuda.sdpa_fwd(cuda.from_host(q), tk, tv, scale, True, off)
    k, v = kc[:, :, :L], vc[:, :, :L]
    o_ref = attention_ref(q, k, v, scale, off)[0]
    assert_close(np.swapaxes(o_ref, 1, 2), cuda.to_host(out), 1e-4, 1e-4, "decode attention out")
    assert_close(lse_ref(q, k, scale, off), cuda.to_host(lse), 1e-5, 1e-5, "decode attention lse")


# ---------------------------------------------------------------- decode steps replayed as a CUDA graph
from projectai_b200 import _paihost as H  # noqa: E402
import projectai_b200 as pai  # noqa: E402

GQA16 = dict(vocab_size=256, embedding_dim=128, layer_count=2, head_count=8, kv_head_count=2, ffn_hidden=344,
             max_sequence_length=64)   # head_dim 16, 4 query heads per kv head
HD64 = dict(vocab_size=300, embedding_dim=256, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=512,
            max_sequence_length=64)   # head_dim 64 (the compile-time head-dim kernel)


def _ids(seed, n, vocab):
    r = H.PcgRng(seed)
    return [int(r.next_u32() % vocab) for _ in range(n)]


@pytest.mark.parametrize("cfg,batch,fused", [(GQA16, 3, True), (HD64, 2, True), (HD64, 1, True), (GQA16, 7, True),
                                             (HD64, 20, True), (GQA16, 3, False), (HD64, 6, False),
                                             (GQA16, 32, True), (HD64, 32, False)])
def test_graph_decode_steps_match_eager_steps(cfg, batch, fused):
    """GraphDecoder (device ids/position, captured once, replayed) against LlamaModel.forward with the KV cache for the
    same tokens: logits within 1e-4·max|logit| (the decode attention splits the keys differently), greedy ids equal."""
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    m = H.LlamaModel(be, H.ModelConfig(**cfg), seed=3)
    vocab, plen, steps = cfg["vocab_size"], 5, 7
    prompt = np.array(_ids(5, batch * plen, vocab), np.float32).reshape(batch, plen)
    feed = [_ids(100 + s, batch, vocab) for s in range(steps)]
    eager_cache = H.KvCache(be, m, batch, cfg["max_sequence_length"])
    graph_cache = H.KvCache(be, m, batch, cfg["max_sequence_length"])
    with H.no_grad():
        m.forward(be.from_host(prompt), eager_cache)
        m.forward(be.from_host(prompt), graph_cache)
        dec = H.GraphDecoder(be, m, graph_cache, batch)
        dec.fused = fused
        for s, ids in enumerate(feed):
            e = be.to_host(m.forward(be.from_host(np.array(ids, np.float32).reshape(batch, 1)), eager_cache))
            g = be.to_host(dec.step(ids))
            assert g.shape == e.shape == (batch, 1, vocab)
            tol = 1e-4 * np.abs(e).max()
            assert np.abs(e - g).max() <= tol, f"step {s}: max |eager - graph| {np.abs(e - g).max():.3e} > {tol:.3e}"
            assert list(e[:, 0].argmax(-1)) == list(g[:, 0].argmax(-1))
        assert dec.captured
    assert graph_cache.length(0) == eager_cache.length(0) == plen + steps
    be.check_device_error()


@pytest.mark.parametrize("rows,n", [(32, 32000), (5, 1001), (1, 4), (3, 1)])
def test_device_argmax_follows_the_reference_rules(rows, n):
    """pai_argmax_rows against the host ArgMax (Sampling.cs:15-31): NaN skipped, ties to the lowest index, a row of
    NaN gives 0; on a dense [rows, n] tensor and on the last-position view of a [rows, 3, n] tensor."""
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    rs = np.random.RandomState(rows * 7 + n)
    x = rs.standard_normal((rows, 3, n)).astype(np.float32)
    last = x[:, 2]
    if n >= 4:
        last[0, rs.randint(0, n, size=max(1, n // 10))] = np.nan      # NaNs never win
        top = last[min(1, rows - 1)].max()
        last[min(1, rows - 1), [n - 1, n // 2]] = top + 1.0            # a tie: the lower index wins
        last[rows - 1, : n // 2] = -np.inf
    if rows >= 3:
        last[2, :] = np.nan                                            # no number: index 0
    expect = [H.argmax(last[r].copy()) for r in range(rows)]
    full = be.from_host(x)
    got_view = be.to_host(be.argmax_rows(full.slice(1, 2, 1)))  # [rows, 1, n], row stride 3·n
    got_dense = be.to_host(be.argmax_rows(be.from_host(np.ascontiguousarray(last))))
    assert [int(v) for v in got_view] == expect
    assert [int(v) for v in got_dense] == expect


def test_generate_replays_a_graph_with_the_eager_tokens(monkeypatch):
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    m = H.LlamaModel(be, H.ModelConfig(**GQA16), seed=4)
    prompt = _ids(9, 2 * 6, 256)
    with_graph = H.generate(be, m, prompt, 12, None, 2)
    monkeypatch.setenv("PAI_DECODE_GRAPH", "0")
    eager = H.generate(be, m, prompt, 12, None, 2)
    assert with_graph["graph"] and not eager["graph"]
    assert with_graph["tokens"] == eager["tokens"]
    monkeypatch.delenv("PAI_DECODE_GRAPH")
    a = H.generate(be, m, prompt, 12, H.TopKTopPSampler(2, 0.8, 40, 1.0), 2)
    b = H.generate(be, m, prompt, 12, H.TopKTopPSampler(2, 0.8, 40, 1.0), 2)
    assert a["tokens"] == b["tokens"]  # a fixed sampler seed reproduces the sequence through the replayed graph


def test_graph_decoder_rejects_bad_ids_and_overflow():
    cfg = dict(GQA16, max_sequence_length=8)
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    m = H.LlamaModel(be, H.ModelConfig(**cfg), seed=1)
    cache = H.KvCache(be, m, 1, 8)
    with H.no_grad():
        m.forward(be.from_host(np.zeros((1, 6), np.float32)), cache)
        dec = H.GraphDecoder(be, m, cache, 1)
        with pytest.raises(H.OutOfRangeError):
            dec.step([256])
        dec.step([1])
        dec.step([2])
        with pytest.raises(H.InvalidOperationError, match="overflow"):
            dec.step([3])
    be.check_device_error()


# ---------------------------------------------------------------- fused decode-step ops
@pytest.mark.parametrize("rows", [5, 32])
def test_linear_fused_at_the_1b_decode_shapes(rows):
    """The 1B decode step's products at batch 5 and 32: q/k/v side by side, SwiGLU gate/up with SiLU·mul, the down
    projection with the residual (k = 5632), against float64."""
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    rs = np.random.RandomState(40 + rows)
    x = rs.standard_normal((rows, 2048)).astype(np.float32)
    h = rs.standard_normal((rows, 5632)).astype(np.float32)
    w = lambda n, k: (rs.standard_normal((n, k)) * 0.02).astype(np.float32)
    wq, wk, wv, wg, wu, wd = w(2048, 2048), w(512, 2048), w(512, 2048), w(5632, 2048), w(5632, 2048), w(2048, 5632)
    res = rs.standard_normal((rows, 2048)).astype(np.float32)
    x64, h64 = x.astype(np.float64), h.astype(np.float64)
    tx = be.from_host(x)
    got = be.to_host(be.linear_fused(tx, [be.from_host(t) for t in (wq, wk, wv)], 0))
    exp = x64 @ np.concatenate([wq, wk, wv]).astype(np.float64).T
    bound = np.abs(x64) @ np.abs(np.concatenate([wq, wk, wv])).astype(np.float64).T
    assert np.abs(got - exp).max() <= 1e-5 * bound.max()
    got = be.to_host(be.linear_fused(tx, [be.from_host(wg), be.from_host(wu)], 2))
    g, u = x64 @ wg.astype(np.float64).T, x64 @ wu.astype(np.float64).T
    exp = g / (1 + np.exp(-g)) * u
    assert np.abs(got - exp).max() <= 1e-4 * np.abs(exp).max()
    got = be.to_host(be.linear_fused(be.from_host(h), [be.from_host(wd)], 1, be.from_host(res)))
    exp = res.astype(np.float64) + h64 @ wd.astype(np.float64).T
    bound = np.abs(h64) @ np.abs(wd).astype(np.float64).T
    assert np.abs(got - exp).max() <= 1e-5 * bound.max() + 1e-6 * np.abs(exp).max()
    be.check_device_error()


@pytest.mark.parametrize("rows", [1, 3, 8, 20, 32])
def test_linear_fused_modes_match_float64(rows):
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    rs = np.random.RandomState(rows)
    k = 2048
    x = rs.standard_normal((rows, k)).astype(np.float32)
    ws = [(rs.standard_normal((n, k)) * 0.02).astype(np.float32) for n in (512, 128, 128)]
    tx, tw = be.from_host(x), [be.from_host(w) for w in ws]
    x64 = x.astype(np.float64)
    bound = np.abs(x).astype(np.float64) @ np.abs(np.concatenate(ws)).astype(np.float64).T
    # mode 0: products side by side
    got = be.to_host(be.linear_fused(tx, tw, 0))
    exp = np.concatenate([x64 @ w.astype(np.float64).T for w in ws], axis=1)
    assert got.shape == (rows, 768)
    assert np.abs(got - exp).max() <= 1e-5 * bound.max()
    # mode 1: residual + x·W0ᵀ
    res = rs.standard_normal((rows, 512)).astype(np.float32)
    got = be.to_host(be.linear_fused(tx, [tw[0]], 1, be.from_host(res)))
    exp = res.astype(np.float64) + x64 @ ws[0].astype(np.float64).T
    assert np.abs(got - exp).max() <= 1e-5 * bound.max() + 1e-6 * np.abs(exp).max()
    # mode 2: SiLU(x·W1ᵀ)·(x·W2ᵀ)
    got = be.to_host(be.linear_fused(tx, [tw[1], tw[2]], 2))
    g, u = x64 @ ws[1].astype(np.float64).T, x64 @ ws[2].astype(np.float64).T
    exp = g / (1 + np.exp(-g)) * u
    assert np.abs(got - exp).max() <= 1e-4 * max(np.abs(exp).max(), 1e-3)
    with pytest.raises(H.ArgumentError):
        be.linear_fused(tx, [tw[0], tw[1]], 2)  # SiLU·mul needs two weights of one shape
    # split-K partials are added in a fixed order (the last CTA to arrive sums them by k): repeated calls agree bit for bit
    for mode, ws_, r_ in ((0, tw, None), (1, [tw[0]], be.from_host(res)), (2, [tw[1], tw[2]], None)):
        first = be.to_host(be.linear_fused(tx, ws_, mode, r_))
        for _ in range(3):
            assert np.array_equal(be.to_host(be.linear_fused(tx, ws_, mode, r_)), first)
    # with a norm weight: the same values as RmsNorm followed by the product (the normalised rows are bit-identical)
    nw = be.from_host((1 + 0.1 * rs.standard_normal(k)).astype(np.float32))
    fused = be.to_host(be.linear_fused(tx, tw, 0, None, nw, 1e-5))
    unfused = be.to_host(be.linear_fused(be.rms_norm(tx, nw, 1e-5), tw, 0))
    assert np.array_equal(fused, unfused) if rows < 5 else np.abs(fused - unfused).max() <= 1e-6 * np.abs(unfused).max()
    fused = be.to_host(be.linear_fused(tx, [tw[1], tw[2]], 2, None, nw, 1e-5))
    unfused = be.to_host(be.linear_fused(be.rms_norm(tx, nw, 1e-5), [tw[1], tw[2]], 2))
    assert np.array_equal(fused, unfused) if rows < 5 else np.abs(fused - unfused).max() <= 1e-6 * np.abs(unfused).max()
    be.check_device_error()


def test_rope_append_equals_rotary_at_and_kv_append():
    """Fused RoPE + cache append against the two separate position-on-device ops: bit-identical (same element ops).
    The strided q/k/v views of the fused q|k|v product are exercised by the graph decode tests above."""
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    rs = np.random.RandomState(3)
    B, Hh, KV, D, T, pos = 2, 8, 2, 64, 40, 17
    cos = be.from_host(rs.standard_normal((T, D)).astype(np.float32))
    sin = be.from_host(rs.standard_normal((T, D)).astype(np.float32))
    p = be.allocate([1])
    be.write(p, np.array([pos], np.float32))
    q = be.from_host(rs.standard_normal((B, Hh, 1, D)).astype(np.float32))
    k = be.from_host(rs.standard_normal((B, KV, 1, D)).astype(np.float32))
    v = be.from_host(rs.standard_normal((B, KV, 1, D)).astype(np.float32))
    kc1, vc1 = be.allocate([B, KV, T, D]), be.allocate([B, KV, T, D])
    kc2, vc2 = be.allocate([B, KV, T, D]), be.allocate([B, KV, T, D])
    qa = be.rope_append(q, k, v, cos, sin, kc1, vc1, p)
    qb = be.rotary_at(q, cos, sin, p)
    be.kv_append(be.rotary_at(k, cos, sin, p), v, kc2, vc2, p)
    assert np.array_equal(be.to_host(qa), be.to_host(qb))
    assert np.array_equal(be.to_host(kc1), be.to_host(kc2))
    assert np.array_equal(be.to_host(vc1), be.to_host(vc2))
    # RotaryEmbedding at position pos (CpuComputeBackend.cs:397-420), restated on the host
    c, s_ = be.to_host(cos)[pos], be.to_host(sin)[pos]
    qh = be.to_host(q)[:, :, 0]
    half = D // 2
    rot = np.concatenate([qh[..., :half] * c[:half] - qh[..., half:] * s_[:half],
                          qh[..., half:] * c[half:] + qh[..., :half] * s_[half:]], -1)
    np.testing.assert_allclose(be.to_host(qa)[:, :, 0], rot, rtol=1e-6, atol=1e-6)
    assert np.all(be.to_host(kc1)[:, :, :pos] == 0) and np.all(be.to_host(kc1)[:, :, pos + 1:] == 0)
    assert np.array_equal(be.to_host(vc1)[:, :, pos], be.to_host(v)[:, :, 0])
    be.check_device_error()


@pytest.mark.parametrize("B,NH,KV,D,T,pos", [(1, 32, 8, 64, 768, 517), (3, 8, 2, 16, 200, 130), (2, 16, 4, 64, 2048, 1500),
                                          (4, 8, 8, 32, 64, 0),
                                          # 64+ (batch, kv head) pairs: the streaming kernel (bulk-copied K/V ring)
                                          (16, 32, 8, 64, 768, 517), (32, 8, 2, 16, 100, 77), (8, 64, 8, 64, 2048, 1999),
                                          (64, 4, 1, 64, 40, 0)])
def test_attn_decode_step_equals_rope_append_then_sdpa_decode(B, NH, KV, D, T, pos):
    """The fused decode-step attention (RoPE + cache append + attention, cluster-merged key splits) against the two
    separate ops: bit-identical outputs and caches; and against float64 attention over the filled cache prefix."""
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    rs = np.random.RandomState(pos)
    cos = be.from_host(rs.standard_normal((T, D)).astype(np.float32))
    sin = be.from_host(rs.standard_normal((T, D)).astype(np.float32))
    p = be.allocate([1])
    be.write(p, np.array([pos], np.float32))
    q = be.from_host(rs.standard_normal((B, NH, 1, D)).astype(np.float32))
    k = be.from_host(rs.standard_normal((B, KV, 1, D)).astype(np.float32))
    v = be.from_host(rs.standard_normal((B, KV, 1, D)).astype(np.float32))
    prefix_k = rs.standard_normal((B, KV, T, D)).astype(np.float32)
    prefix_v = rs.standard_normal((B, KV, T, D)).astype(np.float32)
    kc1, vc1 = be.from_host(prefix_k), be.from_host(prefix_v)
    kc2, vc2 = be.from_host(prefix_k), be.from_host(prefix_v)
    scale = 1.0 / np.sqrt(D)
    fused = be.to_host(be.attn_decode_step(q, k, v, cos, sin, kc1, vc1, p, scale))
    qr = be.rope_append(q, k, v, cos, sin, kc2, vc2, p)
    two = be.to_host(be.sdpa_decode(qr, kc2, vc2, p, scale))
    assert np.array_equal(fused, two)
    assert np.array_equal(be.to_host(kc1), be.to_host(kc2)) and np.array_equal(be.to_host(vc1), be.to_host(vc2))
    kk, vv = be.to_host(kc1)[:, :, :pos + 1], be.to_host(vc1)[:, :, :pos + 1]
    o_ref = attention_ref(be.to_host(qr), kk, vv, scale, pos)[0]
    assert_close(np.swapaxes(o_ref, 1, 2), fused, 1e-4, 1e-4, "decode step attention")
    be.check_device_error()
