"""PAICKPT2 checkpoints and packed token datasets.

CPU: the oracle (oracle/formats.py) against known-answer bytes built by hand from the layout documented in
ProjectAI.Formats/Checkpoint.cs:11-16, its read checks (Checkpoint.cs:59-124) and the packed-dataset rules of
ProjectAI.Training/PackedBinDataset.cs and ProjectAI.Tests/PackedDatasetTests.cs (blocks of seq_len + 1 ids, trailing
remainder dropped, u16 when the vocabulary fits, a truncated shard rejected).

GPU: the native paths of project-ai_b200/csrc/io.cu through the C ABI — a saved file is byte-identical to the oracle's
for the same tensors (views, a scalar, a payload spanning several staging chunks), a save snapshots the tensors so
later device writes do not reach the file, a load reproduces the oracle's tensors and raises the reference's errors on
damaged files, and a dataset batch equals Trainer.NextBatch (Training.cs:122-141) bit for bit.
"""
import json
import struct
import sys

import numpy as np
import pytest

from conftest import ORACLE_LIB, ROOT

sys.path.insert(0, str(ROOT / "oracle"))
import formats as F  # noqa: E402  (the oracle, test infrastructure)

from projectai_b200 import cabi  # noqa: E402


def known_answer() -> bytes:
    """step 7, metadata "{}", "w" = [1, -2] and "s" = 0.5 (rank 0), written out field by field."""
    b = b"PAICKPT2" + struct.pack("<i", 7) + struct.pack("<i", 2) + b"{}" + struct.pack("<i", 2)
    b += struct.pack("<i", 1) + b"w" + struct.pack("<i", 1) + struct.pack("<i", 2) + struct.pack("<q", 8)
    b += struct.pack("<f", 1.0) + struct.pack("<f", -2.0)
    b += struct.pack("<i", 1) + b"s" + struct.pack("<i", 0) + struct.pack("<q", 4) + struct.pack("<f", 0.5)
    return b


# ---------------------------------------------------------------- oracle (CPU)
def test_oracle_checkpoint_matches_the_documented_layout(tmp_path):
    tensors = [("w", np.array([1.0, -2.0], np.float32)), ("s", np.array(0.5, np.float32))]
    assert F.checkpoint_bytes(7, tensors, "{}") == known_answer()
    p = tmp_path / "k.ckpt"
    p.write_bytes(known_answer())
    step, meta, back = F.load_checkpoint(p)
    assert (step, meta) == (7, "{}")
    assert [n for n, _ in back] == ["w", "s"] and back[1][1].shape == () and float(back[1][1]) == 0.5
    assert F.load_checkpoint(p, header_only=True)[:2] == (7, "{}")


def damaged_files(good: bytes):
    """(bytes, message fragment) pairs for each check of Checkpoint.Load (Checkpoint.cs:64-101)."""
    body = good[8:]
    meta_end = 8 + 8 + 2
    w_rank = meta_end + 4 + 4 + 1
    return [
        (b"PAICKPT1" + body, "bad magic"),
        (good[:12] + struct.pack("<i", -1) + good[16:], "bad metadata length (-1)"),
        (good[:12] + struct.pack("<i", (1 << 24) + 1) + good[16:], "bad metadata length"),
        (good[:meta_end] + struct.pack("<i", -3) + good[meta_end + 4:], "negative tensor count (-3)"),
        (good[:meta_end + 4] + struct.pack("<i", -1) + good[meta_end + 8:], "bad name length -1"),
        (good[:w_rank] + struct.pack("<i", 9) + good[w_rank + 4:], "invalid rank 9"),
        (good[:w_rank + 4] + struct.pack("<i", -2) + good[w_rank + 8:], "negative dimension -2"),
        (good[:w_rank + 8] + struct.pack("<q", 12) + good[w_rank + 16:], "payload length 12 != dims product"),
        (good[:-2], "is truncated"),
        (good[:14], "is truncated"),
    ]


def test_oracle_checkpoint_rejects_damaged_files(tmp_path):
    for i, (data, msg) in enumerate(damaged_files(known_answer())):
        p = tmp_path / f"bad{i}.ckpt"
        p.write_bytes(data)
        with pytest.raises(F.InvalidData, match=msg.replace("(", r"\(").replace(")", r"\)")):
            F.load_checkpoint(p)


def test_oracle_library_checkpoints_match_the_format_oracle(tmp_path):
    """The CPU oracle library's checkpoint entry points (used to run the host trainer's checkpoint flows on the CPU)
    write the bytes of the format restatement, views in logical row-major order, and read them back with its checks."""
    from projectai_b200 import _paihost as H

    be = H.Backend(str(ORACLE_LIB), "oracle_", 0)
    w = rnd(5, 6, 4)
    tensors = [("w", w), ("wT", np.ascontiguousarray(w.T)), ("s", np.array(2.5, np.float32)), ("e", np.zeros((0, 3), np.float32))]
    dev = be.from_host(w)
    items = [("w", dev), ("wT", dev.transpose(0, 1)), ("s", be.from_host(tensors[2][1])), ("e", be.allocate([0, 3]))]
    p = tmp_path / "o.ckpt"
    be.save_checkpoint(str(p), 7, items, "meta ✓")
    be.wait_checkpoint()
    assert p.read_bytes() == F.checkpoint_bytes(7, tensors, "meta ✓")
    step, meta, got = be.load_checkpoint(str(p))
    assert (step, meta) == (7, "meta ✓") and [n for n, _ in got] == [n for n, _ in tensors]
    for (n, t), (_, want) in zip(got, tensors):
        assert np.array_equal(be.to_host(t).reshape(want.shape), want), n
    for i, (data, msg) in enumerate(damaged_files(known_answer())):
        q = tmp_path / f"bad{i}.ckpt"
        q.write_bytes(data)
        with pytest.raises(H.InvalidDataError, match=msg.replace("(", r"\(").replace(")", r"\)")):
            be.load_checkpoint(str(q))


def test_oracle_packed_dataset_blocks_and_guards(tmp_path):
    ids = np.random.RandomState(3).randint(0, 259, size=16 * 17 + 5)
    m = F.pack_dataset(ids, 259, 16, tmp_path / "a")
    assert (m["Dtype"], m["BlockCount"], m["DroppedTokens"]) == ("u16", 16, 5)
    man, shard = F.read_manifest(tmp_path / "a")
    for b in (0, 7, 15):
        assert np.array_equal(F.get_sequence(man, shard, b), ids[b * 17:(b + 1) * 17])
    inp, tgt = F.next_batch(man, shard, [3, 0, 3])
    assert np.array_equal(inp[0], ids[51:67].astype(np.float32)) and np.array_equal(tgt[0], ids[52:68].astype(np.float32))
    with pytest.raises(IndexError):
        F.get_sequence(man, shard, 16)
    assert F.pack_dataset(ids, 70000, 16, tmp_path / "b")["Dtype"] == "u32"
    with open(shard, "r+b") as f:  # PackedDatasetTests.Open_RejectsTruncatedShard
        f.truncate(8)
    with pytest.raises(F.InvalidData, match="bytes but the manifest needs"):
        F.read_manifest(tmp_path / "a")
    with pytest.raises(FileNotFoundError):
        F.read_manifest(tmp_path / "missing")


# ---------------------------------------------------------------- native path (GPU)
def rnd(seed, *shape):
    return np.random.RandomState(seed).standard_normal(shape).astype(np.float32)


@pytest.mark.gpu
def test_saved_checkpoint_is_byte_identical_to_the_oracle(cuda, tmp_path):
    a, b, big = rnd(1, 33, 70), rnd(2, 5, 6, 7), rnd(3, 20_000_003)  # big spans three 32 MB staging chunks
    ta, tb, tbig = cuda.from_host(a), cuda.from_host(b), cuda.from_host(big)
    ts = cuda.from_host(np.array(0.25, np.float32), shape=())
    tt = cabi.transpose(ta, 0, 1)  # a strided view is written in its logical (row-major) order
    named = [("layers.0.w", ta), ("opt.m::layers.0.w", tt), ("b", tb), ("scalar", ts), ("big", tbig)]
    p = tmp_path / "s.ckpt"
    cuda.save_checkpoint(p, 42, named, '{"Config": 1}')
    cuda.wait_checkpoint()
    want = F.checkpoint_bytes(42, [("layers.0.w", a), ("opt.m::layers.0.w", a.T), ("b", b),
                                   ("scalar", np.array(0.25, np.float32)), ("big", big)], '{"Config": 1}')
    got = p.read_bytes()
    assert len(got) == len(want) and got == want


@pytest.mark.gpu
def test_save_snapshots_the_tensors_before_returning(cuda, tmp_path):
    x = rnd(4, 4_000_000)
    t = cuda.from_host(x)
    p = tmp_path / "snap.ckpt"
    cuda.save_checkpoint(p, 1, [("x", t)])
    cuda.copy(cuda.from_host(np.zeros_like(x)), t)  # queued after the snapshot, while the file is being written
    cuda.wait_checkpoint()
    assert np.array_equal(F.load_checkpoint(p)[2][0][1], x)
    assert np.array_equal(cuda.to_host(t), np.zeros_like(x))


@pytest.mark.gpu
def test_load_matches_the_oracle_and_raises_its_errors(cuda, tmp_path):
    tensors = [("w", rnd(5, 64, 48)), ("v", rnd(6, 9_000_001)), ("s", np.array(-1.5, np.float32)), ("e", np.zeros((0, 3), np.float32))]
    p = tmp_path / "l.ckpt"
    F.save_checkpoint(p, 9, tensors, "meta ✓")
    step, meta, got = cuda.load_checkpoint(p)
    assert (step, meta) == (9, "meta ✓") and list(got) == [n for n, _ in tensors]
    for name, arr in tensors:
        assert got[name].shape == arr.shape
        assert np.array_equal(cuda.to_host(got[name]), arr)
    assert cuda.read_checkpoint_metadata(p) == (9, "meta ✓")
    for i, (data, msg) in enumerate(damaged_files(known_answer())):
        q = tmp_path / f"bad{i}.ckpt"
        q.write_bytes(data)
        with pytest.raises(cabi.InvalidDataError, match=msg.replace("(", r"\(").replace(")", r"\)")):
            cuda.load_checkpoint(q)
    with pytest.raises(cabi.FileIOError):
        cuda.load_checkpoint(tmp_path / "absent.ckpt")
    with pytest.raises(cabi.FileIOError):
        cuda.save_checkpoint(tmp_path / "no" / "dir" / "x.ckpt", 0, [("w", cuda.from_host(tensors[0][1]))])


@pytest.mark.gpu
def test_load_reads_large_payloads_in_parts_and_reports_truncation_like_the_oracle(cuda, tmp_path):
    """Payloads of a whole 32 MB staging chunk and of a chunk and a bit load exactly (each chunk is read as up to four
    parts at once); a file cut inside the third part of a chunk reports the bytes up to the cut, as the reference's
    sequential reader does."""
    big = rnd(7, 8_388_608)              # 32 MB: one full chunk
    odd = rnd(8, 8_388_608 + 262_147)    # a full chunk, then 1 MB + 12 bytes
    p = tmp_path / "big.ckpt"
    F.save_checkpoint(p, 4, [("big", big), ("odd", odd)])
    _, _, got = cuda.load_checkpoint(p)
    assert np.array_equal(cuda.to_host(got["big"]), big) and np.array_equal(cuda.to_host(got["odd"]), odd)
    data = p.read_bytes()
    start = data.index(b"big") + 3 + 4 + 4 + 8  # name, rank, one dimension, payload length
    cut = tmp_path / "cut.ckpt"
    cut.write_bytes(data[:start + 20_000_000])
    with pytest.raises(F.InvalidData) as want:
        F.load_checkpoint(cut)
    assert "got 20000000" in str(want.value)
    with pytest.raises(cabi.InvalidDataError, match=r"expected 33554432 bytes, got 20000000\)"):
        cuda.load_checkpoint(cut)


@pytest.mark.gpu
@pytest.mark.parametrize("vocab", [259, 100_000])
def test_dataset_batch_equals_next_batch(cuda, tmp_path, vocab):
    seq = 64
    ids = np.random.RandomState(vocab).randint(0, vocab, size=40 * (seq + 1) + 11)
    m = F.pack_dataset(ids, vocab, seq, tmp_path)
    man, shard = F.read_manifest(tmp_path)
    cuda.dataset_open(shard, man["Dtype"], man["SequenceLength"], man["BlockCount"])
    for indices in ([0], [39, 3, 3, 17], list(range(40))):
        inp, tgt = cuda.dataset_batch(indices)
        want_i, want_t = F.next_batch(man, shard, indices)
        assert np.array_equal(cuda.to_host(inp), want_i) and np.array_equal(cuda.to_host(tgt), want_t)
    with pytest.raises(cabi.OutOfRangeError):
        cuda.dataset_batch([m["BlockCount"]])
    cuda.dataset_close()
    with pytest.raises(cabi.InvalidOperationError):
        cuda.dataset_batch([0])


@pytest.mark.gpu
def test_dataset_open_and_id_guards(cuda, tmp_path):
    seq = 8
    ids = np.arange(5 * (seq + 1), dtype=np.int64)
    F.pack_dataset(ids, 1 << 20, seq, tmp_path / "d")
    man, shard = F.read_manifest(tmp_path / "d")
    with pytest.raises(cabi.InvalidDataError, match="bytes but the manifest needs"):
        cuda.dataset_open(shard, "u32", seq, 6)
    with pytest.raises(cabi.InvalidDataError, match="unsupported dataset dtype"):
        cuda.dataset_open(shard, "u8", seq, 5)
    with pytest.raises(cabi.FileIOError):
        cuda.dataset_open(tmp_path / "none.bin", "u32", seq, 5)
    raw = np.fromfile(shard, dtype="<u4")
    raw[2 * (seq + 1) + 4] = 2**31  # above int32: GetSequence's checked cast throws
    raw.tofile(shard)
    cuda.dataset_open(shard, "u32", seq, 5)
    inp, _ = cuda.dataset_batch([1])
    assert np.array_equal(cuda.to_host(inp)[0], ids[9:17].astype(np.float32))
    with pytest.raises(cabi.OutOfRangeError, match="exceeds the int32 range"):
        cuda.dataset_batch([2])


@pytest.mark.gpu
def test_trainer_checkpoint_resume_and_dataset_batches(tmp_path):
    """The host trainer end to end: micro-batches from a packed dataset (device ids), two AdamW steps, a checkpoint
    in the reference's state layout (each parameter, then its opt.m:: / opt.v:: moments), restored into a model
    initialised from another seed; the restored weights and moments equal the saved ones exactly and the next step
    matches the uninterrupted run."""
    import projectai_b200 as pai
    from projectai_b200 import _paihost as H

    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    cfg = dict(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=344,
               max_sequence_length=64)
    seq = 32

    def trainer(seed):
        m = H.LlamaModel(be, H.ModelConfig(**cfg), seed=seed)
        tc = H.TrainingConfig(batch_size=2, sequence_length=seq, learning_rate=1e-3, weight_decay=0.1, max_steps=10,
                              gradient_checkpointing=True, warmup_steps=0)
        tr = H.Trainer(be, m, tc, 0.9, 0.95)
        tr.set_constant_lr(1e-3)
        return m, tr

    ids = np.random.RandomState(11).randint(0, 256, size=12 * (seq + 1))
    man = F.pack_dataset(ids, 256, seq, tmp_path / "ds")
    man, shard = F.read_manifest(tmp_path / "ds")
    be.dataset_open(str(shard), man["Dtype"], seq, man["BlockCount"])
    picks = [[0, 5], [7, 2], [11, 3]]

    def batch(i):
        inp, tgt = be.dataset_batch(picks[i])
        want_i, want_t = F.next_batch(man, shard, picks[i])
        assert np.array_equal(be.to_host(inp), want_i) and np.array_equal(be.to_host(tgt), want_t)
        return inp, tgt

    m1, t1 = trainer(0)
    for i in range(2):
        inp, tgt = batch(i)
        t1.step_tensors([inp], [tgt])
    path = tmp_path / "step-2.ckpt"
    t1.save_checkpoint(str(path), 2, '{"Config": "tiny"}')
    t1.wait_checkpoint()

    step, meta, saved = F.load_checkpoint(path)
    names = [n for n, _ in m1.named_parameters()]
    assert (step, meta) == (2, '{"Config": "tiny"}')
    assert [n for n, _ in saved] == [x for n in names for x in (n, f"opt.m::{n}", f"opt.v::{n}")]
    saved = dict(saved)
    for n, p in m1.named_parameters():
        assert np.array_equal(saved[n], be.to_host(p)), n

    m2, t2 = trainer(1)
    assert t2.restore(str(path)) == 2
    for n, p in m2.named_parameters():
        assert np.array_equal(be.to_host(p), saved[n]), n
    inp, tgt = batch(2)
    l1 = t1.step_tensors([inp], [tgt])
    l2 = t2.step_tensors([inp], [tgt])
    assert abs(l1 - l2) <= 1e-6 * abs(l1), (l1, l2)
    w1 = dict((n, be.to_host(p)) for n, p in m1.named_parameters())
    for n, p in m2.named_parameters():
        np.testing.assert_allclose(be.to_host(p), w1[n], rtol=1e-5, atol=1e-7, err_msg=n)
    be.dataset_close()

    bad = tmp_path / "missing.ckpt"
    F.save_checkpoint(bad, 1, [(n, saved[n]) for n in names[1:]])
    with pytest.raises(H.InvalidDataError, match="is missing parameter"):
        t2.restore(str(bad))


@pytest.mark.gpu
def test_train_loop_over_a_packed_dataset_writes_periodic_and_final_checkpoints(tmp_path):
    """Trainer.Train end to end on the CUDA library (Training.cs:59-120): batches drawn by NextBatch's rule from the
    open packed dataset, a checkpoint every 2 steps and a final one, named step-<n>.ckpt in the checkpoint directory.
    The final file holds the trained weights and moments exactly, and the step-2 file restores a trainer that then
    reproduces step 3's loss."""
    import projectai_b200 as pai
    from projectai_b200 import _paihost as H

    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    cfg = dict(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=344,
               max_sequence_length=64)
    seq = 32
    ids = np.random.RandomState(13).randint(0, 256, size=10 * (seq + 1))
    F.pack_dataset(ids, 256, seq, tmp_path / "ds")
    man, shard = F.read_manifest(tmp_path / "ds")
    be.dataset_open(str(shard), man["Dtype"], seq, man["BlockCount"])
    ckdir = tmp_path / "ck"

    def trainer(seed, steps):
        m = H.LlamaModel(be, H.ModelConfig(**cfg), seed=seed)
        tc = H.TrainingConfig(batch_size=2, sequence_length=seq, learning_rate=1e-3, weight_decay=0.1, max_steps=steps,
                              grad_accum=2, gradient_checkpointing=True, warmup_steps=1, seed=9,
                              checkpoint_every_steps=2, checkpoint_directory=str(ckdir))
        return m, H.Trainer(be, m, tc, 0.9, 0.95)

    m1, t1 = trainer(0, 3)
    report = t1.train(packed_blocks=man["BlockCount"])
    assert report["final_step"] == 3 and len(report["step_losses"]) == 3
    assert sorted(p.name for p in ckdir.iterdir()) == ["step-2.ckpt", "step-3.ckpt"]
    step, _, saved = F.load_checkpoint(ckdir / "step-3.ckpt")
    saved = dict(saved)
    assert step == 3
    for n, p in m1.named_parameters():
        assert np.array_equal(saved[n], be.to_host(p)), n
        assert f"opt.m::{n}" in saved and f"opt.v::{n}" in saved

    # resume from step 2: the rows of step 3 are the generator's draws after two steps of 2 x 2 rows
    m2, t2 = trainer(1, 3)
    assert t2.restore(str(ckdir / "step-2.ckpt")) == 2
    rng = H.PcgRng(9)
    for _ in range(2 * 2 * 2):
        rng.next_u32()
    batches = [be.dataset_batch([rng.next_u32() % man["BlockCount"] for _ in range(2)]) for _ in range(2)]
    l3 = t2.step_tensors([b[0] for b in batches], [b[1] for b in batches])
    assert abs(l3 - report["step_losses"][2]) <= 1e-6 * abs(l3), (l3, report["step_losses"][2])
    be.dataset_close()


# ---------------------------------------------------------------- self-describing model checkpoints (Checkpointing.cs)
def _meta_json(cfg_over=None, kind="bpe", dtype=0, tokenizer='{"merges":[]}'):
    cfg = {"VocabSize": 256, "EmbeddingDim": 128, "LayerCount": 2, "HeadCount": 4, "KvHeadCount": 2,
           "FeedForwardHiddenDim": 344, "MaxSequenceLength": 64, "RopeTheta": 10000, "NormEpsilon": 1E-05, "HeadDim": 32}
    cfg.update(cfg_over or {})
    d = {"Config": cfg, "Tokenizer": tokenizer, "ComputeDType": dtype}
    if kind is not None:
        d["TokenizerKind"] = kind
    return json.dumps(d)


def test_model_metadata_round_trip_and_peek_info(tmp_path):
    """The metadata record of Checkpointing.SaveModel (Checkpointing.cs:19, 22-36): ModelConfig under its C# property
    names in declaration order (HeadDim, computed, last), read back by PeekInfo from the header alone."""
    from projectai_b200 import _paihost as H
    from projectai_b200 import checkpointing as C

    cfg = H.ModelConfig(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=344,
                        max_sequence_length=64, rope_theta=500000.0, norm_eps=1e-6)
    j = C.config_to_json(cfg)
    assert list(j) == ["VocabSize", "EmbeddingDim", "LayerCount", "HeadCount", "KvHeadCount", "FeedForwardHiddenDim",
                       "MaxSequenceLength", "RopeTheta", "NormEpsilon", "HeadDim"]
    back = C.config_from_json(json.loads(json.dumps(j)))
    for a in ("vocab_size", "embedding_dim", "layer_count", "head_count", "kv_head_count", "ffn_hidden",
              "max_sequence_length", "rope_theta", "norm_eps", "head_dim"):
        assert getattr(back, a) == getattr(cfg, a), a

    p = tmp_path / "m.ckpt"
    F.save_checkpoint(p, 12, [("w", np.ones(3, np.float32))], _meta_json(kind="hf"))
    info = C.peek_info(p)
    assert (info.step, info.tokenizer_kind, info.compute_dtype) == (12, "hf", "F32")
    assert (info.config.embedding_dim, info.config.kv_head_count, info.config.head_dim) == (128, 2, 32)
    F.save_checkpoint(p, 3, [], _meta_json(kind=None, dtype=2))  # a file from before the kind tag: BPE
    info = C.peek_info(p)
    assert (info.tokenizer_kind, info.compute_dtype) == ("bpe", "BF16")
    assert C.read_metadata(p)[0] == 3


def test_model_load_refuses_what_the_reference_refuses(tmp_path):
    """LoadModel's checks (Checkpointing.cs:45-62) fire before any weight is read: a resume-only checkpoint (no
    metadata), unreadable metadata, an unknown tokenizer kind, an invalid config (ModelConfig.Validate), and, here, a
    model stored at another precision; the header checks are the reader's."""
    from projectai_b200 import _paihost as H
    from projectai_b200 import checkpointing as C

    p = tmp_path / "r.ckpt"
    F.save_checkpoint(p, 5, [("w", np.ones(3, np.float32))])
    with pytest.raises(H.InvalidDataError, match="has no model metadata; it cannot be loaded for inference"):
        C.load_model(None, p)
    with pytest.raises(H.InvalidDataError, match="has no model metadata; it cannot be described"):
        C.peek_info(p)
    F.save_checkpoint(p, 5, [], "{not json")
    with pytest.raises(H.InvalidDataError, match="unreadable model metadata"):
        C.load_model(None, p)
    F.save_checkpoint(p, 5, [], _meta_json(kind="sentencepiece"))
    with pytest.raises(H.InvalidDataError, match="unknown tokenizer kind 'sentencepiece'"):
        C.load_model(None, p)
    F.save_checkpoint(p, 5, [], _meta_json({"HeadCount": 3}))
    with pytest.raises(H.ArgumentError, match="must be divisible by"):
        C.load_model(None, p)
    F.save_checkpoint(p, 5, [], _meta_json(dtype=1))
    with pytest.raises(H.ArgumentError, match="F16 model"):
        C.load_model(None, p)
    p.write_bytes(b"NOTACKPT" + bytes(8))
    with pytest.raises(H.InvalidDataError, match=r"is not a ProjectAI checkpoint \(bad magic\)"):
        C.read_metadata(p)
    p.write_bytes(b"PAICKPT2" + struct.pack("<ii", 1, 40) + b"{}")
    with pytest.raises(H.InvalidDataError, match=r"truncated reading metadata \(expected 40 bytes, got 2\)"):
        C.read_metadata(p)


@pytest.mark.gpu
def test_save_model_then_load_model_rebuilds_the_trained_model(tmp_path):
    """SaveModel with the trainer's moments, then LoadModel into a model built from the stored config: the weights
    are the trained ones exactly and the logits match; the file carries the moments and the reference's metadata."""
    import projectai_b200 as pai
    from projectai_b200 import _paihost as H
    from projectai_b200 import checkpointing as C

    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
    cfg = H.ModelConfig(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=344,
                        max_sequence_length=64)
    m = H.LlamaModel(be, cfg, seed=3)
    tr = H.Trainer(be, m, H.TrainingConfig(batch_size=2, sequence_length=16, learning_rate=1e-3, max_steps=4,
                                           warmup_steps=0, checkpoint_directory=""), 0.9, 0.95)
    ids = np.random.RandomState(4).randint(0, 256, size=(2, 17)).astype(np.float32)
    tr.step([ids[:, :16].copy()], [ids[:, 1:].copy()])
    p = tmp_path / "model.ckpt"
    C.save_model(be, p, m, cfg, "bpe", '{"vocab":{}}', 1, trainer=tr)

    step, meta, saved = F.load_checkpoint(p)
    assert step == 1 and json.loads(meta)["Config"]["FeedForwardHiddenDim"] == 344
    assert any(n.startswith("opt.m::") for n, _ in saved)
    m2, cfg2, kind, tok, step2 = C.load_model(be, p)
    assert (kind, tok, step2, cfg2.layer_count) == ("bpe", '{"vocab":{}}', 1, 2)
    w = dict((n, be.to_host(t)) for n, t in m.named_parameters())
    for n, t in m2.named_parameters():
        assert np.array_equal(be.to_host(t), w[n]), n
    x = be.from_host(ids[:, :16].copy())
    assert np.array_equal(be.to_host(m.forward(x)), be.to_host(m2.forward(x)))


def test_train_loop_checkpoints_and_model_files_on_the_oracle(tmp_path):
    """The same flows on the CPU oracle library: Trainer.train writes step-2 and the final step-3 file, a trainer
    restored from step 2 reproduces step 3, and save_model / load_model rebuild the trained model exactly."""
    from projectai_b200 import _paihost as H
    from projectai_b200 import checkpointing as C

    be = H.Backend(str(ORACLE_LIB), "oracle_", 0)
    cfg = H.ModelConfig(vocab_size=64, embedding_dim=32, layer_count=2, head_count=4, kv_head_count=2, ffn_hidden=64,
                        max_sequence_length=16)
    seqs = [[int(v) for v in row] for row in np.random.RandomState(8).randint(0, 64, size=(6, 12))]
    ckdir = tmp_path / "ck"

    def trainer(seed):
        m = H.LlamaModel(be, cfg, seed=seed)
        tc = H.TrainingConfig(batch_size=2, sequence_length=8, learning_rate=1e-3, weight_decay=0.1, max_steps=3,
                              warmup_steps=1, seed=4, checkpoint_every_steps=2, checkpoint_directory=str(ckdir))
        return m, H.Trainer(be, m, tc, 0.9, 0.95)

    m1, t1 = trainer(0)
    report = t1.train(seqs)
    assert sorted(q.name for q in ckdir.iterdir()) == ["step-2.ckpt", "step-3.ckpt"]
    m2, t2 = trainer(1)
    assert t2.restore(str(ckdir / "step-2.ckpt")) == 2
    rng = H.PcgRng(4)
    for _ in range(2 * 2):
        rng.next_u32()
    rows = [rng.next_u32() % len(seqs) for _ in range(2)]
    l3 = t2.step([np.array([seqs[r][:8] for r in rows], np.float32)], [np.array([seqs[r][1:9] for r in rows], np.float32)])
    assert l3 == report["step_losses"][2]
    w1 = dict((n, be.to_host(p)) for n, p in m1.named_parameters())
    for n, p in m2.named_parameters():
        assert np.array_equal(be.to_host(p), w1[n]), n

    path = tmp_path / "model.ckpt"
    C.save_model(be, path, m1, cfg, "hf", '{"model":{}}', 3, trainer=t1)
    info = C.peek_info(path)
    assert (info.step, info.tokenizer_kind, info.config.ffn_hidden) == (3, "hf", 64)
    m3, cfg3, kind, tok, step = C.load_model(be, path)
    assert (kind, tok, step, cfg3.vocab_size) == ("hf", '{"model":{}}', 3, 64)
    for n, p in m3.named_parameters():
        assert np.array_equal(be.to_host(p), w1[n]), n
    with pytest.raises(H.InvalidDataError, match="has no model metadata"):
        C.load_model(be, ckdir / "step-3.ckpt")  # a resume checkpoint carries no model metadata


@pytest.mark.parametrize("vocab", [259, 100_000])
def test_train_loop_over_a_packed_dataset_on_the_oracle(tmp_path, vocab):
    """The oracle library's packed-dataset entry points give NextBatch's ids (u16 and u32 shards, against the numpy
    restatement), and Trainer.train over the open dataset equals Trainer.train over the same blocks as host sequences,
    bit for bit; a dataset whose sequence length differs from the trainer's is refused."""
    from projectai_b200 import _paihost as H

    be = H.Backend(str(ORACLE_LIB), "oracle_", 0)
    seq = 8
    ids = np.random.RandomState(9).randint(0, vocab, size=9 * (seq + 1) + 3)
    F.pack_dataset(ids, vocab, seq, tmp_path / "ds")
    man, shard = F.read_manifest(tmp_path / "ds")
    be.dataset_open(str(shard), man["Dtype"], seq, man["BlockCount"])
    inp, tgt = be.dataset_batch([4, 0, 8])
    want_i, want_t = F.next_batch(man, shard, [4, 0, 8])
    assert np.array_equal(be.to_host(inp), want_i) and np.array_equal(be.to_host(tgt), want_t)
    with pytest.raises(H.OutOfRangeError, match=r"index 9: valid range is \[0, 9\)"):
        be.dataset_batch([9])

    cfg = H.ModelConfig(vocab_size=vocab, embedding_dim=32, layer_count=1, head_count=4, kv_head_count=2, ffn_hidden=64,
                        max_sequence_length=16)

    def trainer(s=seq):
        m = H.LlamaModel(be, cfg, seed=2)
        tc = H.TrainingConfig(batch_size=2, sequence_length=s, learning_rate=1e-3, max_steps=2, grad_accum=2,
                              warmup_steps=0, seed=6, checkpoint_directory="")
        return m, H.Trainer(be, m, tc, 0.9, 0.95)

    m1, t1 = trainer()
    r1 = t1.train(packed_blocks=man["BlockCount"])
    blocks = [[int(v) for v in ids[b * (seq + 1):(b + 1) * (seq + 1)]] for b in range(man["BlockCount"])]
    m2, t2 = trainer()
    r2 = t2.train(blocks)
    assert r1["step_losses"] == r2["step_losses"]
    w2 = dict((n, be.to_host(p)) for n, p in m2.named_parameters())
    for n, p in m1.named_parameters():
        assert np.array_equal(be.to_host(p), w2[n]), n
    _, t3 = trainer(s=4)
    with pytest.raises(H.InvalidOperationError, match="holds sequences of length 8; the training sequence length is 4"):
        t3.train(packed_blocks=man["BlockCount"])
    be.dataset_close()
