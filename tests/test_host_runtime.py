"""The C++ host runtime (tensor views, autograd, Llama modules, AdamW, trainer, samplers) run over the CPU oracle,
pinned by the known answers of the reference's own tests:

* PCG canonical vector and Gaussian moments — ProjectAI.Tests/FoundationTests.cs:38-58
* softmax / RMSNorm / RoPE values — TransformerOpsTests.cs:24-210
* embedding gradient 2/9 and 1/9, cross-entropy closed forms — EmbeddingLossTests.cs:44-93
* AdamW decoupled decay closed form, schedule override, per-parameter timestep — AdamWTests.cs:49-116
* checkpointed gradients == standard gradients — GradientCheckpointingTests.cs:16-54
* gradient accumulation == full batch — TrainingTests.cs:137-180
* KV-cache decode == full forward — LlamaModelTests.cs:26-54
* attention against a hand-rolled GQA reference — AttentionTests.cs:83-141
* greedy / top-k / top-p sampling — SamplingTests.cs:10-134
"""
import math

import numpy as np
import pytest

from conftest import ORACLE_LIB
from projectai_b200 import _paihost as H


@pytest.fixture()
def be():
    return H.Backend(str(ORACLE_LIB), "oracle_", 0)


def host(be, t):
    return be.to_host(t).reshape(-1)


# ---------------------------------------------------------------- RNG (FoundationTests.cs)
def test_pcg_canonical_vector():
    rng = H.PcgRng(42, 54)
    assert [rng.next_u32() for _ in range(6)] == [0xA15C02B7, 0x7B47F409, 0xBA1D3330, 0x83D2F293, 0xBFA4784B, 0xCBED606E]


def test_pcg_same_seed_reproduces_and_gaussian_moments():
    a, b = H.PcgRng(12345), H.PcgRng(12345)
    assert all(a.next_u32() == b.next_u32() for _ in range(100))
    r = H.PcgRng(2024)
    g = np.array([r.next_gaussian() for _ in range(200_000)], dtype=np.float64)
    assert abs(g.mean()) < 0.02 and abs(g.std() - 1) < 0.02
    f = H.PcgRng(3)
    assert all(0.0 <= f.next_float() < 1.0 for _ in range(1000))


# ---------------------------------------------------------------- transformer ops (TransformerOpsTests.cs)
def test_softmax_rmsnorm_rope_known_answers(be):
    y = host(be, be.softmax(be.from_host(np.array([1, 2, 3], np.float32)), 0))
    np.testing.assert_allclose(y, [0.09003057, 0.24472847, 0.66524096], atol=1e-4)
    y = host(be, be.softmax(be.from_host(np.array([80, 81, 82], np.float32)), 0))
    np.testing.assert_allclose(y, [0.09003057, 0.24472847, 0.66524096], atol=1e-4)
    x = be.from_host(np.array([[1, 2, 3, 4], [0, 0, 0, 0]], np.float32))
    w = be.from_host(np.array([2, 0.5, 1, 3], np.float32))
    inv = 1 / math.sqrt(7.5 + 1e-6)
    np.testing.assert_allclose(host(be, be.rms_norm(x, w, 1e-6)), [1 * inv * 2, 2 * inv * 0.5, 3 * inv, 4 * inv * 3, 0, 0, 0, 0], atol=1e-5)
    t0, t1 = 0.7, 1.3
    xr = be.from_host(np.array([[1, 2, 3, 4]], np.float32))
    c = be.from_host(np.array([[math.cos(t0), math.cos(t1), math.cos(t0), math.cos(t1)]], np.float32))
    s = be.from_host(np.array([[math.sin(t0), math.sin(t1), math.sin(t0), math.sin(t1)]], np.float32))
    y = host(be, be.rotary(xr, c, s))
    exp = [1 * math.cos(t0) - 3 * math.sin(t0), 2 * math.cos(t1) - 4 * math.sin(t1),
           3 * math.cos(t0) + 1 * math.sin(t0), 4 * math.cos(t1) + 2 * math.sin(t1)]
    np.testing.assert_allclose(y, exp, atol=1e-5)


# ---------------------------------------------------------------- embedding & loss (EmbeddingLossTests.cs)
def test_embedding_gradient_accumulates_repeats(be):
    cfg = H.ModelConfig(vocab_size=5, embedding_dim=4, layer_count=1, head_count=2, kv_head_count=2, ffn_hidden=8)
    m = H.LlamaModel(be, cfg, seed=1)
    ag = m.autograd
    w = dict(m.named_parameters())["embedding.weight"]
    rows = ag.embedding(w, [1, 1, 3])
    loss = ag.mean(rows)
    loss.backward()
    g = be.to_host(w.grad)
    n = 3 * 4
    assert np.all(g[[0, 2, 4]] == 0)
    np.testing.assert_allclose(g[1], 2 / n, rtol=1e-5)
    np.testing.assert_allclose(g[3], 1 / n, rtol=1e-5)


def test_cross_entropy_closed_forms(be):
    ag = H.Autograd(be)
    logits = be.from_host(np.array([[1, 2, 3], [1, 1, 1]], np.float32))
    r0 = -math.log(math.exp(3) / (math.exp(1) + math.exp(2) + math.exp(3)))
    r1 = -math.log(1 / 3)
    loss = H.cross_entropy_loss(ag, logits, be.from_host(np.array([2, 0], np.float32)))
    assert abs(host(be, loss)[0] - (r0 + r1) / 2) < 1e-4
    loss = H.cross_entropy_loss(ag, logits, be.from_host(np.array([2, 0], np.float32)), ignore_index=0)
    assert abs(host(be, loss)[0] - r0) < 1e-4
    with pytest.raises(H.OutOfRangeError):
        H.cross_entropy_loss(ag, logits, be.from_host(np.array([2, 7], np.float32)))


# ---------------------------------------------------------------- AdamW (AdamWTests.cs)
def test_adamw_decoupled_decay_and_schedule(be):
    p = be.from_host(np.array([1, 2, -3], np.float32))
    p.requires_grad = True
    p.grad = be.from_host(np.zeros(3, np.float32))
    opt = H.AdamW([p], be, lr=0.1, weight_decay=0.1)
    opt.step()
    np.testing.assert_allclose(host(be, p), np.array([1, 2, -3]) * (1 - 0.1 * 0.1), rtol=1e-5)
    q = be.from_host(np.array([1], np.float32))
    q.requires_grad = True
    q.grad = be.from_host(np.zeros(1, np.float32))
    opt2 = H.AdamW([q], be, lr=99.0, weight_decay=0.1)
    opt2.set_schedule(lambda step: 0.2)
    opt2.step()
    np.testing.assert_allclose(host(be, q), [1 - 0.2 * 0.1], rtol=1e-5)
    assert opt2.step_count == 1


def test_adamw_per_parameter_timestep(be):
    a = be.from_host(np.zeros(1, np.float32))
    b = be.from_host(np.zeros(1, np.float32))
    a.requires_grad = b.requires_grad = True
    opt = H.AdamW([a, b], be, lr=0.1, weight_decay=0.0)
    for _ in range(5):
        a.grad = be.from_host(np.ones(1, np.float32))
        b.grad = None
        opt.step()
    before = host(be, b)[0]
    a.grad = be.from_host(np.ones(1, np.float32))
    b.grad = be.from_host(np.ones(1, np.float32))
    opt.step()
    assert before == 0.0
    assert abs(host(be, b)[0] - before - (-0.1)) < 1e-2
    assert opt.state_t(b) == 1 and opt.state_t(a) == 6


# ---------------------------------------------------------------- model-level equivalences
def small_config(**kw):
    base = dict(vocab_size=16, embedding_dim=32, layer_count=3, head_count=4, kv_head_count=2, ffn_hidden=64,
                max_sequence_length=16)
    base.update(kw)
    return H.ModelConfig(**base)


def param_grads(be, model, ids, targets, checkpoint):
    for _, p in model.named_parameters():
        p.grad = None
    model.gradient_checkpointing = checkpoint
    ag = model.autograd
    logits = model.forward(be.from_host(ids))
    loss = H.cross_entropy_loss(ag, logits, be.from_host(targets))
    loss.backward()
    return {n: be.to_host(p.grad).copy() for n, p in model.named_parameters()}


def test_seeded_backward_equals_the_checkpoint_surrogate(be):
    """Autograd.Checkpoint seeds the recomputed segment's backward through Σ(recomputed ⊙ upstream)
    (Autograd.cs:143-144); the host runtime runs the walk from upstream directly. The leaf gradients agree bit for bit."""
    ag = H.Autograd(be)
    rs = np.random.RandomState(3)
    xs = rs.standard_normal((4, 6)).astype(np.float32)
    ws = rs.standard_normal((5, 6)).astype(np.float32)
    up = rs.standard_normal((4, 5)).astype(np.float32)

    def grads(seeded):
        x, w = be.from_host(xs), be.from_host(ws)
        x.requires_grad = w.requires_grad = True
        y = ag.silu(ag.matmul(x, w, True))
        u = be.from_host(up)
        if seeded:
            y.backward(u)
        else:
            ag.sum_all(ag.mul(y, u)).backward()
        return be.to_host(x.grad), be.to_host(w.grad)

    (sx, sw), (rx, rw) = grads(True), grads(False)
    assert np.array_equal(sx, rx) and np.array_equal(sw, rw)


def test_rope_on_the_sequence_major_layout_equals_the_head_major_rope(be):
    """RoPE on [b, s, heads, dh] with the tables broadcast over heads ([s, 1, dh]) gives, element for element, the
    values RotaryEmbedding gives on the head-major view [b, heads, s, dh] (RotaryEmbedding, Modules.cs:43-60)."""
    b, s, h, d = 2, 5, 3, 8
    rs = np.random.RandomState(4)
    x = rs.standard_normal((b, s, h, d)).astype(np.float32)
    cos = rs.standard_normal((s, d)).astype(np.float32)
    sin = rs.standard_normal((s, d)).astype(np.float32)
    tx = be.from_host(x)
    head_major = be.to_host(be.rotary(tx.transpose(1, 2), be.from_host(cos), be.from_host(sin)))
    seq_major = be.to_host(be.rotary(tx, be.from_host(cos.reshape(s, 1, d)), be.from_host(sin.reshape(s, 1, d))))
    assert np.array_equal(np.swapaxes(head_major, 1, 2), seq_major)


def test_checkpointed_gradients_match_standard(be):
    model = H.LlamaModel(be, small_config(), seed=0)
    ids = (np.arange(12) % 16).astype(np.float32).reshape(2, 6)
    targets = ((np.arange(12) * 7 + 3) % 16).astype(np.float32).reshape(2, 6)
    base = param_grads(be, model, ids, targets, False)
    ckpt = param_grads(be, model, ids, targets, True)
    assert base.keys() == ckpt.keys()
    for name, e in base.items():
        g = ckpt[name]
        assert np.all(np.abs(e - g) <= 1e-4 + 1e-4 * np.abs(e)), name


def test_gradient_accumulation_matches_full_batch(be):
    full = H.LlamaModel(be, small_config(vocab_size=259, layer_count=2), seed=5)
    acc = H.LlamaModel(be, small_config(vocab_size=259, layer_count=2), seed=5)
    rng = np.random.RandomState(11)
    ids = rng.randint(1, 259, size=(4, 8)).astype(np.float32)
    tg = rng.randint(1, 259, size=(4, 8)).astype(np.float32)
    loss = H.cross_entropy_loss(full.autograd, full.forward(be.from_host(ids)), be.from_host(tg))
    loss.backward()
    half = be.from_host(np.array([0.5], np.float32))
    for m in range(2):
        l = H.cross_entropy_loss(acc.autograd, acc.forward(be.from_host(ids[2 * m:2 * m + 2])), be.from_host(tg[2 * m:2 * m + 2]))
        acc.autograd.mul(l, half).backward()
    fp = dict(full.named_parameters())
    for name, p in acc.named_parameters():
        np.testing.assert_allclose(be.to_host(p.grad), be.to_host(fp[name].grad), atol=1e-4, err_msg=name)


def test_kv_cache_decode_matches_full_forward(be):
    cfg = small_config(vocab_size=8, layer_count=2, max_sequence_length=32)
    model = H.LlamaModel(be, cfg, seed=7)
    tokens = [1, 2, 3, 4, 5, 6]
    with H.no_grad():
        full = be.to_host(model.forward(be.from_host(np.array([tokens], np.float32))))[0, -1]
    out = H.generate(be, model, tokens[:1], 1)  # prefill of one token works
    assert len(out["tokens"]) == 1
    # incremental: the generate loop feeds its own argmax; teacher-force here through the same cache semantics
    from projectai_b200 import decode
    step_logits = decode.teacher_forced_last_logits(be, model, tokens)
    np.testing.assert_allclose(step_logits, full, atol=1e-3)


def test_attention_matches_hand_rolled_reference(be):
    for h, kvh, d in [(2, 1, 4), (4, 2, 8), (4, 1, 8)]:
        cfg = H.ModelConfig(vocab_size=16, embedding_dim=d, layer_count=1, head_count=h, kv_head_count=kvh, ffn_hidden=8,
                            max_sequence_length=16)
        m = H.LlamaModel(be, cfg, seed=9)
        names = dict(m.named_parameters())
        wq, wk, wv, wo = (be.to_host(names[f"block.0.attn.{n}.weight"]).astype(np.float64) for n in ("wq", "wk", "wv", "wo"))
        s, dh, g = 3, d // h, h // kvh
        x = np.random.RandomState(10).uniform(-1, 1, size=(s, d)).astype(np.float32)
        from projectai_b200 import decode
        got = decode.attention_layer_output(be, m, x)
        merged = np.zeros((s, h * dh))

        def rope(vec, pos):
            half = dh // 2
            y = np.empty(dh)
            for j in range(half):
                ang = pos * (1.0 / 10000 ** ((2 * j) / dh))
                y[j] = vec[j] * math.cos(ang) - vec[j + half] * math.sin(ang)
                y[j + half] = vec[j + half] * math.cos(ang) + vec[j] * math.sin(ang)
            return y
        for head in range(h):
            kv = head // g
            q = [rope(x[i] @ wq[head * dh:(head + 1) * dh].T, i) for i in range(s)]
            k = [rope(x[i] @ wk[kv * dh:(kv + 1) * dh].T, i) for i in range(s)]
            v = [x[i] @ wv[kv * dh:(kv + 1) * dh].T for i in range(s)]
            for i in range(s):
                sc = np.array([q[i] @ k[j] / math.sqrt(dh) for j in range(i + 1)])
                p = np.exp(sc - sc.max())
                p /= p.sum()
                merged[i, head * dh:(head + 1) * dh] = sum(p[j] * v[j] for j in range(i + 1))
        expected = merged @ wo.T
        np.testing.assert_allclose(got, expected, atol=1e-4)


# ---------------------------------------------------------------- samplers (SamplingTests.cs)
def test_samplers():
    assert H.argmax(np.array([0.1, 0.5, 0.3, -2], np.float32)) == 1
    assert H.argmax(np.array([0.5, 0.5, 0.1], np.float32)) == 0
    assert H.argmax(np.array([np.nan, 0.2, np.nan], np.float32)) == 1
    assert H.argmax(np.array([np.nan, np.nan], np.float32)) == 0
    s = H.TopKTopPSampler(1, temperature=0.0)
    assert all(s.sample(np.array([1, 2, 5, 0], np.float32)) == 2 for _ in range(20))
    s = H.TopKTopPSampler(42, temperature=1.0, top_k=2)
    assert {s.sample(np.array([1, 5, 3, 2, 4], np.float32)) for _ in range(500)} <= {1, 4}
    s = H.TopKTopPSampler(7, temperature=1.0, top_p=0.9)
    assert {s.sample(np.array([10, 9, 0, 0, 0], np.float32)) for _ in range(500)} <= {0, 1}
    s = H.TopKTopPSampler(3, temperature=1.0, top_p=0.3)
    assert all(s.sample(np.array([12, 0, 0, 0], np.float32)) == 0 for _ in range(100))
    a, b = H.TopKTopPSampler(5, 0.8, 40, 1.0), H.TopKTopPSampler(5, 0.8, 40, 1.0)
    logits = np.random.RandomState(0).standard_normal(256).astype(np.float32)
    assert [a.sample(logits) for _ in range(50)] == [b.sample(logits) for _ in range(50)]


def reference_topk_topp(logits, rng, temperature, top_k, top_p):
    """Sampling.cs:60-111 in float32 with the full descending sort (distinct logits, so the order is the argsort)."""
    x = logits.astype(np.float32)
    e = np.exp((x - x.max()) / np.float32(temperature)).astype(np.float32)
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    p = (e / s).astype(np.float32)
    order = sorted(range(len(p)), key=lambda i: (-p[i], i))
    keep = len(p) if top_k <= 0 else min(top_k, len(p))
    if top_p < 1:
        cum, kept = np.float32(0), 0
        for i in range(keep):
            cum = np.float32(cum + p[order[i]])
            kept += 1
            if cum >= np.float32(top_p):
                break
        keep = max(1, kept)
    total = np.float32(0)
    for i in range(keep):
        total = np.float32(total + p[order[i]])
    r = np.float32(np.float32(rng.next_u32() >> 8) * np.float32(1.0 / (1 << 24))) * total
    acc = np.float32(0)
    for i in range(keep):
        acc = np.float32(acc + p[order[i]])
        if r < acc:
            return order[i]
    return order[keep - 1]


def test_topk_partial_sort_and_batched_rows_match_the_reference_sampler():
    rs = np.random.RandomState(1)
    rows = np.stack([rs.permutation(2000).astype(np.float32) * 0.01 for _ in range(6)] +   # distinct logits per row
                    [rs.randint(0, 30, size=2000).astype(np.float32) * 0.1 for _ in range(4)])  # many exact ties
    for k, p in [(40, 1.0), (5, 0.9), (0, 0.5)]:
        s = H.TopKTopPSampler(9, 0.8, k, p)
        ref_rng = H.PcgRng(9)
        got = [s.sample(r) for r in rows]
        exp = [reference_topk_topp(r, ref_rng, 0.8, k, p) for r in rows]
        assert got == exp, (k, p)
        # the batched entry draws in row order: identical to row-by-row sample() calls
        a, b = H.TopKTopPSampler(21, 0.8, k, p), H.TopKTopPSampler(21, 0.8, k, p)
        assert a.sample_rows(rows) == [b.sample(r) for r in rows]


def test_scopes_release_intermediates(be):
    before = be.memory_stats()[0]
    be.begin_scope()
    x = be.from_host(np.ones(1000, np.float32))
    y = be.add_scalar(x, 1.0)
    be.keep_alive(y)
    be.end_scope()
    assert be.memory_stats()[0] > before
    with pytest.raises(H.InvalidOperationError):
        be.to_host(be.add(x, x))
    np.testing.assert_array_equal(be.to_host(y), np.full(1000, 2, np.float32))
    del y
    assert be.memory_stats()[0] == before


# ---------------------------------------------------------------- Trainer.Train (Training.cs:59-141)
def test_train_loop_draws_batches_like_next_batch_and_matches_manual_steps(be):
    """Trainer.train over host sequences: every step draws grad_accum micro-batches of batch_size rows with
    row = PcgRng(seed).NextUInt32() % count (NextBatch, Training.cs:122-141), inputs ids[:seq] and targets ids[1:seq+1],
    under the warmup+cosine schedule. The same draws fed to Trainer.step by hand give the same losses and weights, bit
    for bit; on_step sees each (step, loss); the report holds the per-step losses and the final step."""
    seq, batch, accum, steps = 8, 2, 2, 3
    data_rng = np.random.RandomState(3)
    seqs = [list(data_rng.randint(0, 259, size=seq + 1 + (i % 3))) for i in range(7)]

    def make():
        m = H.LlamaModel(be, small_config(vocab_size=259, layer_count=2), seed=5)
        tc = H.TrainingConfig(batch_size=batch, sequence_length=seq, learning_rate=1e-3, weight_decay=0.1, max_steps=steps,
                              grad_accum=accum, gradient_checkpointing=True, warmup_steps=1, seed=42,
                              checkpoint_directory="")
        return m, H.Trainer(be, m, tc, 0.9, 0.95)

    m1, t1 = make()
    seen = []
    report = t1.train([[int(v) for v in s] for s in seqs], on_step=lambda step, loss: seen.append((step, loss)))

    m2, t2 = make()
    rng = H.PcgRng(42)
    manual = []
    for _ in range(steps):
        ins, tgs = [], []
        for _ in range(accum):
            rows = [rng.next_u32() % len(seqs) for _ in range(batch)]
            ins.append(np.array([seqs[r][:seq] for r in rows], np.float32))
            tgs.append(np.array([seqs[r][1:seq + 1] for r in rows], np.float32))
        manual.append(t2.step(ins, tgs))
    assert report["final_step"] == steps
    assert np.array_equal(np.array(report["step_losses"], np.float32), np.array(manual, np.float32))
    assert seen == [(i + 1, l) for i, l in enumerate(report["step_losses"])]
    assert report["first_loss"] == report["step_losses"][0] and report["last_loss"] == report["step_losses"][-1]
    w2 = dict((n, be.to_host(p)) for n, p in m2.named_parameters())
    for n, p in m1.named_parameters():
        assert np.array_equal(be.to_host(p).view(np.uint32), w2[n].view(np.uint32)), n


def test_train_loop_rejects_empty_and_short_datasets(be):
    """Training.cs:66 (empty dataset: ArgumentException) and :131-133 (a drawn sequence shorter than seq + 1:
    InvalidOperationException with the reference's message)."""
    m = H.LlamaModel(be, small_config(vocab_size=259, layer_count=1), seed=1)
    tc = H.TrainingConfig(batch_size=1, sequence_length=8, max_steps=1, checkpoint_directory="")
    tr = H.Trainer(be, m, tc)
    with pytest.raises(H.ArgumentError, match="dataset is empty"):
        tr.train([])
    with pytest.raises(H.InvalidOperationError, match=r"dataset sequence 0 has length 5; need 9 for sequence length 8\."):
        tr.train([[1, 2, 3, 4, 5]])
