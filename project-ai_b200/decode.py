"""Decode helpers over the host runtime: teacher-forced incremental decode through the KV cache (the per-token path of
ProjectAI.Training/Inference.cs:46-56) and single-layer attention, used to check decode against a full forward."""
from __future__ import annotations

import numpy as np

from . import _paihost as H


def teacher_forced_last_logits(be, model, tokens, max_sequence_length: int = 32) -> np.ndarray:
    """Feeds `tokens` one at a time through a fresh KV cache and returns the last step's logits row."""
    cache = H.KvCache(be, model, 1, max_sequence_length)
    last = None
    with H.no_grad():
        for t in tokens:
            logits = model.forward(be.from_host(np.array([[t]], np.float32)), cache)
            last = be.to_host(logits)[0, -1]
    return last


def teacher_forced_logits(be, model, prompt, continuation, max_sequence_length: int) -> np.ndarray:
    """Prefills `prompt`, then feeds `continuation` one token at a time; returns [len(continuation)+1, vocab] logits
    (the prefill's last row, then each step's row)."""
    cache = H.KvCache(be, model, 1, max_sequence_length)
    rows = []
    with H.no_grad():
        logits = model.forward(be.from_host(np.array([prompt], np.float32)), cache)
        rows.append(be.to_host(logits)[0, -1])
        for t in continuation:
            logits = model.forward(be.from_host(np.array([[t]], np.float32)), cache)
            rows.append(be.to_host(logits)[0, -1])
    return np.stack(rows)


def attention_layer_output(be, model, x: np.ndarray, layer: int = 0) -> np.ndarray:
    """Output of one Attention module on x [seq, dim] (batch 1), as Modules.cs:142-204 computes it."""
    with H.no_grad():
        out = model.attention(layer, be.from_host(x[None]))
    return be.to_host(out)[0]
