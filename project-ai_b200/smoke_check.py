"""One small training step on cuda:0 checked against the CPU oracle.

Tiny Llama config (vocab 256, d 128, 2 layers, 4 heads, FFN 344), batch 2 x seq 32, per-block recompute, one AdamW
step. The loss and every parameter gradient must match the oracle within 1e-4 relative (+1e-4 of the tensor's max).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from . import CUDA_LIB_PATH
from . import _paihost as H

ORACLE_LIB = Path(__file__).resolve().parent.parent / "oracle" / "build" / "liboracle.so"


def run() -> dict:
    cfg = H.ModelConfig(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=4, ffn_hidden=344,
                        max_sequence_length=64)
    r = H.PcgRng(1)
    ids = np.array([r.next_u32() % 256 for _ in range(2 * 33)], np.float32).reshape(2, 33)
    x, y = np.ascontiguousarray(ids[:, :32]), np.ascontiguousarray(ids[:, 1:])
    results = []
    for path, prefix in ((ORACLE_LIB, "oracle_"), (CUDA_LIB_PATH, "pai_")):
        be = H.Backend(str(path), prefix, 0)
        m = H.LlamaModel(be, cfg, seed=0)
        tc = H.TrainingConfig(batch_size=2, sequence_length=32, learning_rate=3e-4, weight_decay=0.1, max_steps=1,
                              gradient_checkpointing=True, warmup_steps=0)
        tr = H.Trainer(be, m, tc, 0.9, 0.95)
        loss = tr.step([x], [y])
        grads = {n: be.to_host(p.grad) for n, p in m.named_parameters()}
        if prefix == "pai_":
            be.check_device_error()
        results.append((loss, grads, be.name))
    (lo, go, _), (lc, gc, name) = results
    if not abs(lo - lc) <= 1e-4 * abs(lo):
        raise AssertionError(f"smoke: loss {lc} on {name} vs oracle {lo}")
    for n, e in go.items():
        g = gc[n]
        tol = 1e-4 * np.abs(e) + 1e-4 * np.abs(e).max()
        if not np.all(np.abs(e - g) <= tol):
            raise AssertionError(f"smoke: gradient {n} differs from the oracle")
    print(f"smoke ok on {name}: loss {lc:.6f} (oracle {lo:.6f}), {len(go)} gradients match")
    return {"loss": lc, "oracle_loss": lo}
