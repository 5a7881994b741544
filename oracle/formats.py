"""CPU oracle for the training loop's file formats — TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module, as the checker of the native paths in project-ai_b200/csrc/io.cu; the product
never routes through it. It restates, in numpy and plain Python:

* the PAICKPT2 checkpoint writer and reader of ProjectAI.Formats/Checkpoint.cs:23-139 — the same little-endian layout
  (magic "PAICKPT2" | int32 step | int32 metaLen | metadata | int32 count | per tensor: int32 nameLen | name | int32 rank
  | rank x int32 dims | int64 byteLen | f32 payload) and the same validation order and messages on read;
* the packed token dataset: the shard writer of ProjectAI.Training/DatasetPacker.cs:40-98 (u16 when the vocabulary fits
  65536 ids, else u32; blocks of seq_len + 1 ids; the trailing remainder dropped), the manifest fields of
  ProjectAI.Training/DatasetManifest.cs:12-60, PackedBinDataset.Open/GetSequence (PackedBinDataset.cs:43-117), and the
  micro-batch construction of Trainer.NextBatch (ProjectAI.Training/Training.cs:122-141).

Parity is pinned by known-answer byte strings built from the documented layout in tests/test_formats.py, since the
reference's tests (ProjectAI.Tests/PackedDatasetTests.cs, CheckpointBackCompatTests.cs) check behaviour through the C#
types rather than committed golden files.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

MAGIC = b"PAICKPT2"


class InvalidData(ValueError):
    """InvalidDataException of the reference."""


# ---------------------------------------------------------------- checkpoints
def checkpoint_bytes(step: int, tensors, metadata: str = "") -> bytes:
    """Checkpoint.Save (Checkpoint.cs:23-57) as bytes: `tensors` is a sequence of (name, float32 array)."""
    out = bytearray(MAGIC)
    meta = metadata.encode("utf-8")
    out += struct.pack("<ii", int(step), len(meta)) + meta
    items = list(tensors)
    out += struct.pack("<i", len(items))
    for name, arr in items:
        a = np.array(arr, dtype=np.float32, order="C")  # keeps a 0-d (rank 0) array 0-d
        if a.size > 2**31 - 1:
            raise NotImplementedError(f"tensor '{name}' has {a.size} elements, exceeding this format's 2^31 limit.")
        nb = name.encode("utf-8")
        out += struct.pack("<i", len(nb)) + nb
        out += struct.pack("<i", a.ndim) + struct.pack(f"<{a.ndim}i", *a.shape)
        out += struct.pack("<q", a.size * 4) + a.astype("<f4").tobytes()
    return bytes(out)


def save_checkpoint(path, step: int, tensors, metadata: str = "") -> None:
    with open(path, "wb") as f:
        f.write(checkpoint_bytes(step, tensors, metadata))


def _reader(data: bytes, path: str):
    pos = [0]

    def take(n, what):
        chunk = data[pos[0]:pos[0] + n]
        if len(chunk) != n:
            raise InvalidData(f"'{path}' is truncated reading {what} (expected {n} bytes, got {len(chunk)}).")
        pos[0] += n
        return chunk

    def i32(what):
        return struct.unpack("<i", take(4, what))[0]

    return take, i32


def load_checkpoint(path, header_only: bool = False):
    """Checkpoint.Load / ReadMetadata (Checkpoint.cs:59-139): (step, metadata, [(name, array)])."""
    data = open(path, "rb").read()
    path = str(path)
    take, i32 = _reader(data, path)
    if data[:8] != MAGIC:
        raise InvalidData(f"'{path}' is not a ProjectAI checkpoint (bad magic).")
    take(8, "magic")
    step = i32("the step")
    meta_len = i32("the metadata length")
    if meta_len < 0 or meta_len > 1 << 24:
        raise InvalidData(f"'{path}' has a bad metadata length ({meta_len}).")
    meta = take(meta_len, "metadata").decode("utf-8")
    if header_only:
        return step, meta, []
    count = i32("the tensor count")
    if count < 0:
        raise InvalidData(f"'{path}' has a negative tensor count ({count}).")
    tensors = []
    for i in range(count):
        name_len = i32("a tensor name length")
        if name_len < 0 or name_len > 1 << 20:
            raise InvalidData(f"'{path}' tensor {i}: bad name length {name_len}.")
        name = take(name_len, f"tensor {i} name").decode("utf-8")
        rank = i32("a tensor rank")
        if rank < 0 or rank > 8:
            raise InvalidData(f"checkpoint tensor '{name}' has invalid rank {rank}.")
        dims = []
        for _ in range(rank):
            d = i32("a tensor dimension")
            if d < 0:
                raise InvalidData(f"checkpoint tensor '{name}' has a negative dimension {d}.")
            dims.append(d)
        expected = int(np.prod(dims, dtype=np.int64)) * 4 if dims else 4
        byte_len = struct.unpack("<q", take(8, "a payload length"))[0]
        if byte_len != expected or byte_len > 2**31 - 1:
            raise InvalidData(f"checkpoint tensor '{name}': payload length {byte_len} != dims product × 4 ({expected}).")
        payload = take(byte_len, f"tensor '{name}' payload")
        tensors.append((name, np.frombuffer(payload, dtype="<f4").reshape(dims).astype(np.float32)))
    return step, meta, tensors


# ---------------------------------------------------------------- packed token datasets
BIN_NAME = "tokens.bin"          # DatasetPacker.DefaultBinName
MANIFEST_NAME = "manifest.json"  # DatasetManifest.FileName


def pack_dataset(ids, vocab_size: int, seq_len: int, out_dir, tokenizer_kind: str = "bpe") -> dict:
    """DatasetPacker.Pack over an already-tokenized id stream: writes tokens.bin (u16 when the vocabulary fits 65536
    ids, else u32, little-endian) and manifest.json; returns the manifest."""
    ids = np.asarray(ids, dtype=np.int64)
    block = seq_len + 1
    blocks = len(ids) // block
    if blocks < 1:
        raise RuntimeError(f"corpus of {len(ids)} tokens is too short for one block of {block}.")
    dtype = "u16" if vocab_size <= 65536 else "u32"
    os.makedirs(out_dir, exist_ok=True)
    ids.astype("<u2" if dtype == "u16" else "<u4").tofile(os.path.join(out_dir, BIN_NAME))
    manifest = {"FormatVersion": 1, "TokenizerKind": tokenizer_kind, "TokenizerState": "", "TokenizerHash": "sha256:",
                "Dtype": dtype, "VocabSize": vocab_size, "SequenceLength": seq_len, "TotalTokens": int(len(ids)),
                "BlockCount": int(blocks), "DroppedTokens": int(len(ids) - blocks * block), "Shards": [BIN_NAME]}
    with open(os.path.join(out_dir, MANIFEST_NAME), "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def read_manifest(path) -> tuple:
    """DatasetManifest.TryResolvePath + FromJson + the checks of PackedBinDataset.Open (:55-83): (manifest, shard)."""
    path = str(path)
    mpath = os.path.join(path, MANIFEST_NAME) if os.path.isdir(path) else path
    if not os.path.isfile(mpath):
        raise FileNotFoundError(f"no '{MANIFEST_NAME}' found at '{path}'.")
    m = json.load(open(mpath))
    if m["Dtype"] not in ("u16", "u32"):
        raise InvalidData(f"unsupported dataset dtype '{m['Dtype']}'.")
    if m["SequenceLength"] < 1:
        raise InvalidData(f"manifest SequenceLength must be >= 1; got {m['SequenceLength']}.")
    if m["BlockCount"] < 1:
        raise InvalidData(f"manifest BlockCount must be >= 1; got {m['BlockCount']}.")
    if len(m["Shards"]) != 1:
        raise NotImplementedError(f"this build reads single-shard datasets; manifest lists {len(m['Shards'])} shards.")
    shard = os.path.join(os.path.dirname(mpath) or ".", m["Shards"][0])
    if not os.path.isfile(shard):
        raise FileNotFoundError(f"dataset shard '{shard}' (from manifest) not found.")
    width = 2 if m["Dtype"] == "u16" else 4
    needed = m["BlockCount"] * (m["SequenceLength"] + 1) * width
    if os.path.getsize(shard) < needed:
        raise InvalidData(f"dataset shard '{shard}' is {os.path.getsize(shard)} bytes but the manifest needs {needed} for "
                          f"{m['BlockCount']} blocks of {m['SequenceLength'] + 1} {m['Dtype']} ids.")
    return m, shard


def get_sequence(manifest: dict, shard, index: int) -> np.ndarray:
    """PackedBinDataset.GetSequence (:96-117): block `index` as int ids (u32 ids above int32 raise, its checked cast)."""
    if not 0 <= index < manifest["BlockCount"]:
        raise IndexError(f"valid range is [0, {manifest['BlockCount']}).")
    block = manifest["SequenceLength"] + 1
    dt = "<u2" if manifest["Dtype"] == "u16" else "<u4"
    raw = np.fromfile(shard, dtype=dt, count=block, offset=index * block * np.dtype(dt).itemsize)
    if raw.max(initial=0) > 2**31 - 1:
        raise OverflowError("id exceeds the int32 range.")
    return raw.astype(np.int64)


def next_batch(manifest: dict, shard, indices) -> tuple:
    """Trainer.NextBatch (Training.cs:122-141) for given block indices: float32 inputs and targets [B, S]."""
    s = manifest["SequenceLength"]
    inp = np.empty((len(indices), s), dtype=np.float32)
    tgt = np.empty((len(indices), s), dtype=np.float32)
    for r, idx in enumerate(indices):
        seq = get_sequence(manifest, shard, int(idx))
        inp[r] = seq[:s].astype(np.float32)
        tgt[r] = seq[1:s + 1].astype(np.float32)
    return inp, tgt
