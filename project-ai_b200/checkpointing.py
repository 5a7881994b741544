"""Self-describing model checkpoints: ``Checkpointing.SaveModel`` / ``LoadModel`` / ``PeekInfo``
(ProjectAI.Training/Checkpointing.cs:22-84) over the library's PAICKPT2 writer and reader.

The metadata string is the reference's JSON record ``Meta(Config, TokenizerKind, Tokenizer, ComputeDType)`` with the
``ModelConfig`` properties under their C# names (ProjectAI.Models/ModelConfig.cs:8-20), so a file written here loads
in the reference and the other way round. Tokenizers are outside this backend: the tokenizer kind ("bpe" or "hf") and
its JSON state travel through unchanged, for the caller to rebuild. The backend computes in F32, the reference's
default ``ComputeDType`` (0).
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

from . import _paihost as H

MAX_METADATA = 1 << 24  # Checkpoint.cs:70
F32 = 0  # DType.F32 (ProjectAI.Core/DType.cs)
_DTYPES = ["F32", "F16", "BF16", "I64", "I32", "U8", "Bool"]


def config_to_json(cfg) -> dict:
    """A ``ModelConfig`` as System.Text.Json writes the C# record: declared properties, then the computed HeadDim."""
    return {"VocabSize": cfg.vocab_size, "EmbeddingDim": cfg.embedding_dim, "LayerCount": cfg.layer_count,
            "HeadCount": cfg.head_count, "KvHeadCount": cfg.kv_head_count, "FeedForwardHiddenDim": cfg.ffn_hidden,
            "MaxSequenceLength": cfg.max_sequence_length, "RopeTheta": cfg.rope_theta, "NormEpsilon": cfg.norm_eps,
            "HeadDim": cfg.head_dim}


def config_from_json(d: dict):
    """The record back (``ModelConfig.Validate`` runs in the constructor and raises ``ArgumentError``). The defaults of
    the optional properties are the record's (ModelConfig.cs:16-18)."""
    try:
        return H.ModelConfig(vocab_size=int(d["VocabSize"]), embedding_dim=int(d["EmbeddingDim"]),
                             layer_count=int(d["LayerCount"]), head_count=int(d["HeadCount"]),
                             kv_head_count=int(d["KvHeadCount"]), ffn_hidden=int(d["FeedForwardHiddenDim"]),
                             max_sequence_length=int(d.get("MaxSequenceLength", 4096)),
                             rope_theta=float(d.get("RopeTheta", 10000.0)), norm_eps=float(d.get("NormEpsilon", 1e-5)))
    except (KeyError, TypeError, ValueError) as e:
        raise H.InvalidDataError(f"model metadata has an unreadable config ({type(e).__name__}: {e}).") from None


def read_metadata(path) -> tuple[int, str]:
    """``Checkpoint.ReadMetadata``: the step and the metadata string from the file's header, with the reader's checks
    and messages (magic, metadata length within 2^24, truncation); the payload is not touched."""
    p = str(path)
    try:
        f = open(p, "rb")
    except OSError as e:
        raise H.FileIOError(f"could not open '{p}': {e.strerror}") from None
    with f:
        head = f.read(16)
        if len(head) < 8 or head[:8] != b"PAICKPT2":
            raise H.InvalidDataError(f"'{p}' is not a ProjectAI checkpoint (bad magic).")
        if len(head) < 12:
            raise H.InvalidDataError(f"'{p}' is truncated reading the step.")
        if len(head) < 16:
            raise H.InvalidDataError(f"'{p}' is truncated reading the metadata length.")
        step, mlen = struct.unpack("<ii", head[8:16])
        if mlen < 0 or mlen > MAX_METADATA:
            raise H.InvalidDataError(f"'{p}' has a bad metadata length ({mlen}).")
        meta = f.read(mlen)
        if len(meta) != mlen:
            raise H.InvalidDataError(f"'{p}' is truncated reading metadata (expected {mlen} bytes, got {len(meta)}).")
    return step, meta.decode("utf-8", errors="replace")  # as Encoding.UTF8.GetString: invalid bytes become U+FFFD


def _meta(path, what: str) -> dict:
    _, text = read_metadata(path)
    if not text:
        raise H.InvalidDataError(f"checkpoint '{path}' has no model metadata; it cannot be {what} (was it saved by `train`?).")
    try:
        meta = json.loads(text)
    except ValueError:
        meta = None
    if not isinstance(meta, dict):
        raise H.InvalidDataError(f"checkpoint '{path}' has unreadable model metadata.")
    return meta


def _dtype(meta: dict, path) -> int:
    """ComputeDType as System.Text.Json writes the enum (a number), or by name; absent means F32."""
    v = meta.get("ComputeDType", F32)
    if isinstance(v, str) and v in _DTYPES:
        return _DTYPES.index(v)
    if isinstance(v, int) and not isinstance(v, bool):
        return v
    raise H.InvalidDataError(f"checkpoint '{path}' has an unreadable ComputeDType ({v!r}).")


def _dtype_name(dt: int) -> str:
    return _DTYPES[dt] if 0 <= dt < len(_DTYPES) else str(dt)


@dataclass
class CheckpointInfo:
    """``Checkpointing.CheckpointInfo``: what a catalog shows without loading weights."""
    config: object
    tokenizer_kind: str
    compute_dtype: str
    step: int


def peek_info(path) -> CheckpointInfo:
    """``Checkpointing.PeekInfo`` (Checkpointing.cs:72-80): config, tokenizer kind ("bpe" when the file predates the
    tag), precision and step from the header alone."""
    meta = _meta(path, "described")
    step, _ = read_metadata(path)
    kind = meta.get("TokenizerKind") or "bpe"
    return CheckpointInfo(config_from_json(meta.get("Config") or {}), kind, _dtype_name(_dtype(meta, path)), step)


def save_model(backend, path, model, config, tokenizer_kind: str, tokenizer_state: str, step: int, trainer=None,
               write: bool = True):
    """``Checkpointing.SaveModel`` (Checkpointing.cs:22-36): the weights, with the trainer's AdamW moments when a
    trainer is given (``EnumerateState``), and the config / tokenizer metadata. Returns once the file is complete, as
    the reference's synchronous save does (the library snapshots on the device and writes in the background).

    Data parallelism: one rank writes. With a ZeRO-1 trainer every rank must call this (the moment shards are
    gathered collectively) and the others pass ``write=False``; otherwise ranks with ``write=False`` return at once."""
    if tokenizer_kind not in ("bpe", "hf"):
        raise H.ArgumentError(f"can't persist tokenizer of kind '{tokenizer_kind}'.")
    metadata = json.dumps({"Config": config_to_json(config), "TokenizerKind": tokenizer_kind,
                           "Tokenizer": tokenizer_state, "ComputeDType": F32}, separators=(",", ":"))
    if trainer is not None:
        if not write and not trainer.zero1:
            return
        trainer.save_checkpoint(str(path) if write else "", step, metadata)
        trainer.wait_checkpoint()
    elif write:
        backend.save_checkpoint(str(path), step, model.named_parameters(), metadata)
        backend.wait_checkpoint()


def load_model(backend, path):
    """``Checkpointing.LoadModel`` (Checkpointing.cs:42-66): rebuilds the model from the stored config (parameters
    allocated without the initial draws, every one overwritten from the file; a missing or misshapen parameter raises
    ``InvalidDataError``) and returns ``(model, config, tokenizer_kind, tokenizer_state, step)``."""
    meta = _meta(path, "loaded for inference")
    dt = _dtype(meta, path)
    if dt != F32:
        raise H.ArgumentError(f"checkpoint '{path}' holds a {_dtype_name(dt)} model; this backend computes in F32.")
    kind = meta.get("TokenizerKind") or "bpe"
    if kind not in ("bpe", "hf"):
        raise H.InvalidDataError(f"checkpoint '{path}' has unknown tokenizer kind '{kind}'.")
    config = config_from_json(meta.get("Config") or {})
    model = H.LlamaModel(backend, config, seed=0, skip_init=True)
    step, _, tensors = backend.load_checkpoint(str(path))
    H.apply_weights(backend, model, tensors)
    return model, config, kind, meta.get("Tokenizer", ""), step
