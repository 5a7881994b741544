"""Training-step benchmark of the B200 backend: train tokens/s (forward + per-block recompute + backward + AdamW).

One step = one pass of the reference trainer's step (ProjectAI.Training/Training.cs:87-113) through the host runtime
and the C ABI: forward with per-block gradient checkpointing, cross-entropy, backward with recompute, fused AdamW.
Workload at N=1 (and per GPU at N>1, weak scaling): ~1B Llama-style decoder, fp32 — vocab 32000, d_model 2048,
16 layers, 32 query heads over 8 KV heads (head_dim 64), SwiGLU FFN 5632, RMSNorm, RoPE base 10000, tied embeddings,
weights N(0, 0.02) from a seed; synthetic token ids uniform in [0, 32000) from PcgRng(rank*1000 + step), targets
shifted by one; seq 2048 x batch 4 per GPU. At N=1 the line also carries the same model without recompute (tokens/s
and peak memory), the ~125M config (vocab 32000, d_model 768, 12 layers, 12 heads, FFN 2048, seq 1024 x batch 8) as
an extra key, and KV-cache decode of the ~1B model.

value  — device-resident batches (uploaded before the timed region), timed with CUDA events on the library's stream.
mfu / hfu — model flops per token (3 x forward: linear layers, tied LM head, causal attention) and hardware flops per
         token (plus the recomputed block forwards) times tokens/s, over the 3xTF32 tensor ceiling.
e2e    — the same step through the public host-buffer entry (Trainer.step with host arrays: the ids H2D copy and the
         loss D2H read are inside the timed region).
roofline — the dominant kernel (the 3xTF32 tcgen05 GEMM): algorithmic 2·M·N·K flops per launch over its average
         event-timed duration inside the timed region, against the measured TF32 tensor peak / 3.
cpu_baseline / --impl reference — the CPU oracle (a C++ restatement of the reference CpuComputeBackend) running the
         same step on a bounded sample of the workload on this machine's host cores.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]; N>1 under torchrun.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
import __graft_entry__  # noqa: E402

pai = __graft_entry__.load_package()
from projectai_b200 import _paihost as H  # noqa: E402

ORACLE_LIB = ROOT / "oracle" / "build" / "liboracle.so"
METRIC = "train tokens/s (fwd+recompute+bwd+AdamW)"
CONFIGS = {
    "125m": dict(vocab_size=32000, embedding_dim=768, layer_count=12, head_count=12, kv_head_count=12, ffn_hidden=2048,
                 seq=1024, batch=8),
    "1b": dict(vocab_size=32000, embedding_dim=2048, layer_count=16, head_count=32, kv_head_count=8, ffn_hidden=5632,
               seq=2048, batch=4),
    "tiny": dict(vocab_size=256, embedding_dim=128, layer_count=2, head_count=4, kv_head_count=4, ffn_hidden=344,
                 seq=64, batch=4),
}


def model_config(c, max_seq):
    return H.ModelConfig(vocab_size=c["vocab_size"], embedding_dim=c["embedding_dim"], layer_count=c["layer_count"],
                         head_count=c["head_count"], kv_head_count=c["kv_head_count"], ffn_hidden=c["ffn_hidden"],
                         max_sequence_length=max_seq)


def param_count(c):
    d, f, v, h, kvh = c["embedding_dim"], c["ffn_hidden"], c["vocab_size"], c["head_count"], c["kv_head_count"]
    hd = d // h
    per_block = d * h * hd * 2 + d * kvh * hd * 2 + 3 * d * f + 2 * d
    return v * d + c["layer_count"] * per_block + d


def synthetic_batch(rank, step, batch, seq, vocab):
    r = H.PcgRng(rank * 1000 + step)
    ids = np.array([r.next_u32() % vocab for _ in range(batch * (seq + 1))], dtype=np.float32).reshape(batch, seq + 1)
    return np.ascontiguousarray(ids[:, :seq]), np.ascontiguousarray(ids[:, 1:])


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.file:
            return None
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def measured_tf32_peak(device):
    """Dense TF32 tensor-core peak measured with cuBLAS on this GPU (8192^3 fp32 GEMM with TF32 allowed, best of 10)."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device=f"cuda:{device}")
    b = torch.randn(n, n, device=f"cuda:{device}")
    for _ in range(3):
        a @ b
    best = 1e30
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        a @ b
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    torch.cuda.empty_cache()
    torch.backends.cuda.matmul.allow_tf32 = False
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def ncu_traffic():
    """Per-launch DRAM bytes of the GEMM kernel from the committed ncu summary, if one exists."""
    p = ROOT / "profiles" / "gemm_tcgen05_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


# Tokens per step of the bounded CPU samples (batch 1): the oracle's scalar loops take ~7 GFLOP per token of the
# ~1B model, and its composed AdamW makes ~20 passes over the 787 M parameters whatever the token count.
CPU_SAMPLE_SEQ = {"1b": 16, "125m": 64, "tiny": 64}
# The single-thread sample (the reference backend's loops on one core) is shorter to stay within ~10-30 s.
CPU_SAMPLE_SEQ_1THREAD = {"1b": 4, "125m": 16, "tiny": 64}


def flops_per_token(c, seq):
    """(model, hardware) flops per trained token. Forward: 2 flops per weight of the linear layers and the tied LM
    head, plus causal attention (QKᵀ and P·V over the (S+1)/2 keys a query sees on average: 2·(S+1)·d per layer).
    Model = 3 x forward (forward + backward); hardware adds the per-block recompute (the blocks' forward again)."""
    d, f, v, h, kvh, layers = (c["embedding_dim"], c["ffn_hidden"], c["vocab_size"], c["head_count"],
                               c["kv_head_count"], c["layer_count"])
    hd = d // h
    linear = 2 * d * h * hd + 2 * d * kvh * hd + 3 * d * f  # wq, wo, wk, wv, gate, up, down
    block = 2.0 * linear + 2.0 * (seq + 1) * h * hd
    fwd = layers * block + 2.0 * v * d
    return 3.0 * fwd, 3.0 * fwd + layers * block


def cpu_train_sample(cfg_name, seq, threads, steps=1, warmup=0):
    """Times the oracle (CPU restatement of the reference backend) on `steps` training steps of the full model at
    batch 1 x seq `seq` (a bounded sample of the workload), after `warmup` untimed steps. Returns (tokens/s, seconds)."""
    import ctypes
    ctypes.CDLL(str(ORACLE_LIB)).oracle_set_threads(threads)
    c = CONFIGS[cfg_name]
    seq = min(seq, c["seq"])
    be = H.Backend(str(ORACLE_LIB), "oracle_", 0)
    m = H.LlamaModel(be, model_config(c, seq), seed=0, init="normal0.02")
    tc = H.TrainingConfig(batch_size=1, sequence_length=seq, learning_rate=3e-4, weight_decay=0.1,
                          max_steps=steps + warmup + 10, gradient_checkpointing=True, warmup_steps=0)
    tr = H.Trainer(be, m, tc, 0.9, 0.95)
    for w in range(warmup):
        x, y = synthetic_batch(0, w, 1, seq, c["vocab_size"])
        tr.step([x], [y])
    t0 = time.perf_counter()
    for k in range(steps):
        x, y = synthetic_batch(0, warmup + k, 1, seq, c["vocab_size"])
        tr.step([x], [y])
    dt = time.perf_counter() - t0
    return seq * steps / dt, dt


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def decode_bench(local, cfg_name="1b", prompt_len=512, gen=256, batches=(1, 32)):
    """KV-cache decode on one GPU: the ~1B model with seeded N(0,0.02) weights, a prompt of `prompt_len` uniform
    random ids per sequence, `gen` new tokens per sequence, greedy and top-k 40 / temperature 0.8 sampling.

    tok/s follows the reference's bench (ProjectAI.Bench/BenchRunner.cs:110-122): generated tokens over the whole
    generate call (prefill + decode steps + host sampling), after one untimed warm-up call; the call is timed with CUDA
    events on the library's stream. decode_tok_s counts only the per-token steps after the prefill."""
    c = CONFIGS[cfg_name]
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", local)
    t0 = time.perf_counter()
    m = H.LlamaModel(be, model_config(c, prompt_len + gen), seed=0, init="normal0.02")
    init_s = time.perf_counter() - t0
    out = {"metric": "decode tok/s", "unit": "tokens/s",
           "config": {"workload": f"llama-{cfg_name} KV-cache decode", "prompt_len": prompt_len, "new_tokens": gen,
                      "params": param_count(c), "weights": "N(0,0.02) seeded", "prompt": "uniform random ids (PcgRng 7)"},
           "model_init_s": init_s}
    for b in batches:
        r = H.PcgRng(7)
        prompt = [int(r.next_u32() % c["vocab_size"]) for _ in range(b * prompt_len)]
        row = {}
        for mode in ("greedy", "topk40_t0.8"):
            sampler = None if mode == "greedy" else H.TopKTopPSampler(11, 0.8, 40, 1.0)
            H.generate(be, m, prompt, 4, sampler, b)  # warm-up (the reference's r == 0 run)
            be.timer_start()
            res = H.generate(be, m, prompt, gen, sampler, b)
            ms = be.timer_stop()
            n = len(res["tokens"])
            row[mode] = {"tok_s": n / (ms * 1e-3), "ms": ms, "generated": n, "prefill_ms": res["prefill_seconds"] * 1e3,
                         "decode_tok_s": b * (n // b - 1) / max(res["decode_seconds"], 1e-9)}
        out[f"batch{b}"] = row
    # per-kernel device time of one greedy generation per batch size: the weight-streaming products dominate (batch 1:
    # k_gemv_tn on the CUDA cores; batch 32: k_gemv_tc on the tensor cores)
    for b in batches:
        r = H.PcgRng(7)
        prompt = [int(r.next_u32() % c["vocab_size"]) for _ in range(b * prompt_len)]
        be.kernel_timing(True)
        be.timer_start()
        H.generate(be, m, prompt, 64, None, b)
        ms_timed = be.timer_stop()
        stats = {f: be.kernel_stats(f) for f in ("gemv", "attn_decode", "gemm", "attn_fwd")}
        be.kernel_timing(False)
        g_launches, g_ms, g_bytes = stats["gemv"]
        achieved = (g_bytes / max(g_launches, 1)) / ((g_ms / max(g_launches, 1)) * 1e-3) / 1e9 if g_ms else 0.0
        kernel = "k_gemv_tn (weight-streaming x·Wᵀ, CUDA cores)" if b <= 4 else "k_gemv_tc (weight-streaming x·Wᵀ, tcgen05 3xTF32)"
        sfx = "" if b == 1 else f"_batch{b}"
        out["roofline" + sfx] = {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                                 "frac": achieved / hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
                                 "launches": g_launches, "avg_launch_ms": g_ms / max(g_launches, 1),
                                 "sample": f"greedy batch {b}, prompt 512 + 64 new tokens (timed per call, x pack included; "
                                           "prefill GEMMs excluded: family gemm)"}
        out["kernels" + sfx] = {f: {"launches": v[0], "ms": v[1], "share": v[1] / ms_timed} for f, v in stats.items()}
    # whole decode steps against the HBM line: every weight and the cached K/V of every sequence are read once per
    # step (mean cache length over the run: prompt + half the new tokens)
    kv_row = 2 * c["kv_head_count"] * (c["embedding_dim"] // c["head_count"]) * 4 * c["layer_count"]
    out["step_roofline"] = {}
    for b in batches:
        tok_s = out[f"batch{b}"]["greedy"]["decode_tok_s"]
        step_s = b / tok_s
        bytes_step = 4.0 * param_count(c) + b * kv_row * (prompt_len + gen / 2)
        out["step_roofline"][f"batch{b}"] = {"bytes_per_step": bytes_step, "ms_per_step": step_s * 1e3,
                                             "achieved_GBps": bytes_step / step_s / 1e9,
                                             "frac": bytes_step / step_s / 1e9 / hbm}
    out["weights_gb_per_token"] = 4.0 * param_count(c) / 1e9
    out["hbm_ceiling_tok_s_batch1"] = hbm / (4.0 * param_count(c) / 1e9)
    del m
    be.sync()
    return out


def reference_arm(args):
    """The reference's CPU path on the host cores: the oracle port of CpuComputeBackend under the same host runtime,
    all threads, each step one full-model training step at batch 1 x seq CPU_SAMPLE_SEQ (a bounded sample: the
    workload's batch x seq per GPU would take hours per step on the CPU). The config block states that sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # under torchrun only rank 0 times the CPU reference
    c = CONFIGS[args.config]
    threads = os.cpu_count() or 1
    seq = min(args.cpu_sample_tokens or CPU_SAMPLE_SEQ[args.config], c["seq"])
    value, dt = cpu_train_sample(args.config, seq, threads, steps=args.steps, warmup=args.warmup)
    sample = (f"{args.config} model (all parameters, AdamW over all of them), per-block recompute, batch 1 x seq {seq} "
              f"per step; the GPU workload is batch {c['batch']} x seq {c['seq']} per GPU")
    cfg = workload_config(args.config, 1, True)
    cfg.update({"seq_len": seq, "batch_per_gpu": 1, "global_batch": 1, "parallelism": "cpu, one process",
                "sample_of": f"llama-{args.config} train step at batch {c['batch']} x seq {c['seq']} per GPU"})
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample,
                             "cpu": cpu_model()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def op_sweep(args):
    """Op-level sweep on one GPU (inputs N(0,1) fp32): each op timed with CUDA events on the library's stream after
    warm-up, reported against its roofline (tensor: measured TF32 / 3; HBM: measured copy bandwidth)."""
    from projectai_b200 import cabi
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    tf32 = measured_tf32_peak(0) if args.op not in ("gemm-only", "checkpoint") else 727.8
    lib = pai.cuda_library()
    be = cabi.NativeBackend(lib, 0)
    rng = np.random.RandomState(0)

    def scoped(fn):
        be.scope_begin()  # each call's outputs return to the cache, so the timed calls reuse warm blocks
        fn()
        be.scope_end()

    def timed(fn, reps):
        for _ in range(2):
            scoped(fn)
        be.timer_start()
        for _ in range(reps):
            scoped(fn)
        return be.timer_stop() / reps

    rows = []

    def emit(op, shape, ms, work, unit, peak):
        achieved = work / (ms * 1e-3) / (1e12 if unit == "TFLOP/s" else 1e9)
        rows.append({"op": op, "shape": shape, "ms": ms, "achieved": achieved, "unit": unit, "peak": peak,
                     "frac": achieved / peak})
        print(json.dumps(rows[-1]), flush=True)

    def randt(*shape):
        return be.from_host(rng.standard_normal(shape).astype(np.float32))

    gemm_shapes = [(m, k, k) for m in (2048, 8192) for k in (768, 2048, 5632)]
    if args.shape:
        gemm_shapes = [tuple(int(x) for x in args.shape.split(","))]
    if args.op in ("all", "gemm", "gemm-only"):
        for m, k, n in gemm_shapes:
            a, b = randt(m, k), randt(n, k)
            be.scope_begin()
            ms = timed(lambda: be.matmul(a, b, True), args.steps)
            be.scope_end()
            emit("matmul(3xTF32, transposeB)", [m, k, n], ms, 2.0 * m * n * k, "TFLOP/s", tf32 / 3)
            be.release(a)
            be.release(b)
    if args.op in ("all", "attention"):
        attn_shapes = [(4, 32, s_, 64) for s_ in (512, 2048, 4096)]
        if args.op == "attention" and args.shape:
            attn_shapes = [tuple(int(v) for v in args.shape.split(","))]
        for B, Hh, s, D in attn_shapes:
            q, k, v, do = randt(B, Hh, s, D), randt(B, Hh, s, D), randt(B, Hh, s, D), randt(B, s, Hh, D)
            fl = 2.0 * B * Hh * s * (s + 1) * D  # causal: 4·D per visible pair, s(s+1)/2 pairs
            be.scope_begin()
            ms = timed(lambda: be.sdpa_fwd(q, k, v, 0.125, True, 0), max(2, args.steps // 2))
            o, lse = be.sdpa_fwd(q, k, v, 0.125, True, 0)
            emit("attention fwd (causal)", [B, Hh, s, D], ms, fl, "TFLOP/s", tf32 / 3)
            ms = timed(lambda: be.sdpa_bwd(q, k, v, o, lse, do, 0.125, True, 0), max(2, args.steps // 2))
            emit("attention bwd (causal)", [B, Hh, s, D], ms, 2.5 * fl, "TFLOP/s", tf32 / 3)
            be.scope_end()
            for t in (q, k, v, do):
                be.release(t)
    if args.op in ("all", "decode", "decode-attn"):
        # 1B decode: every weight shape of a layer plus the LM head, x·Wᵀ for 1 and 32 rows; enough weight copies are
        # cycled that each timed call reads its W from HBM, not L2 (--shape rows,k,n: that product only)
        gemv_shapes = [((n, k), (1, 32)) for n, k in ((2048, 2048), (512, 2048), (5632, 2048), (2048, 5632), (32000, 2048))]
        if args.op == "decode" and args.shape:
            r0, k0, n0 = (int(v) for v in args.shape.split(","))
            gemv_shapes = [((n0, k0), (r0,))]
        for (n, k), row_counts in (gemv_shapes if args.op != "decode-attn" else []):
            copies = max(1, -(-300_000_000 // (n * k * 4)))
            ws = [randt(n, k) for _ in range(copies)]
            for rows_ in row_counts:
                x = randt(rows_, k)
                it = [0]

                def call():
                    it[0] = (it[0] + 1) % copies
                    be.matmul(x, ws[it[0]], True)
                reps = max(args.steps, 2 * copies)
                emit("gemv x·Wᵀ", [rows_, k, n], timed(call, reps), 4.0 * (n * k + rows_ * (n + k)), "GB/s", hbm)
                be.release(x)
            for t in ws:
                be.release(t)
        attn_batches = (1, 32)
        if args.op == "decode" and args.shape:
            attn_batches = ()
        elif args.op == "decode-attn" and args.shape:
            attn_batches = (int(args.shape),)
        for B in attn_batches:
            Hh, KV, D, L = 32, 8, 64, args.decode_cache_len
            q = randt(B, Hh, 1, D)
            kc, vc = randt(B, KV, L, D), randt(B, KV, L, D)
            be.scope_begin()
            ms = timed(lambda: be.sdpa_fwd(q, kc, vc, 0.125, True, L - 1), max(4, args.steps))
            be.scope_end()
            emit("decode attention (1 query, GQA 32/8)", [B, Hh, L, D], ms, 8.0 * B * KV * L * D, "GB/s", hbm)
            for t in (q, kc, vc):
                be.release(t)
    if args.op in ("all", "hbm"):
        x, w, g = randt(8192, 2048), randt(2048), randt(8192, 2048)
        cs, sn = randt(2048, 64), randt(2048, 64)
        xr = cabi.reshape(x, (4, 2048, 32, 64))
        be.scope_begin()
        emit("rmsnorm fwd", [8192, 2048], timed(lambda: be.rmsnorm(x, w, 1e-5), args.steps), 2 * 8192 * 2048 * 4, "GB/s", hbm)
        emit("rmsnorm bwd", [8192, 2048], timed(lambda: be.rmsnorm_bwd(x, w, g, 1e-5), args.steps), 3 * 8192 * 2048 * 4, "GB/s", hbm)
        xv = cabi.transpose(xr, 1, 2)
        emit("rope (strided q view)", [4, 32, 2048, 64], timed(lambda: be.rotary(xv, cs, sn), args.steps), 2 * 8192 * 2048 * 4, "GB/s", hbm)
        emit("swiglu silu(gate)*up", [8192, 2048], timed(lambda: be.silu_mul_fwd(x, g), args.steps), 3 * 8192 * 2048 * 4, "GB/s", hbm)
        emit("swiglu backward", [8192, 2048], timed(lambda: be.silu_mul_bwd(x, g, x), args.steps), 5 * 8192 * 2048 * 4, "GB/s", hbm)
        emit("residual add", [8192, 2048], timed(lambda: be.add(x, g), args.steps), 3 * 8192 * 2048 * 4, "GB/s", hbm)
        be.scope_end()
        logits = randt(8192, 32000)
        targets = rng.randint(0, 32000, size=8192).astype(np.int32)
        be.scope_begin()
        emit("cross-entropy loss+grad", [8192, 32000], timed(lambda: be.cross_entropy_fused(logits, targets), args.steps),
             2 * 8192 * 32000 * 4, "GB/s", hbm)
        be.scope_end()
        be.release(logits)
        n = args.adamw_elements
        p = be.allocate((n,))
        gg, mm, vv = be.allocate((n,)), be.allocate((n,)), be.allocate((n,))
        emit("adamw (fused, in place)", [n], timed(lambda: be.adamw_step(p, gg, mm, vv, 3e-4, 0.9, 0.95, 1e-8, 0.1, 1),
                                                  max(2, args.steps // 2)), 28.0 * n, "GB/s", hbm)
    if args.op == "checkpoint":
        checkpoint_io(be, args)
    be.close()


def checkpoint_io(be, args):
    """PAICKPT2 save and load of a 1B training state: every parameter of the 1B config (tied embedding, 16 blocks,
    final norm) with its two AdamW moments under the reference's names (Checkpointing.cs:103-115), 9.4 GB of fp32. The
    save's compute-stream cost (the device snapshot) is timed with CUDA events on the library's stream; the background
    file write and the load are timed on the host. The file goes to the system temporary directory and is removed."""
    import shutil
    c = CONFIGS["1b"]
    d, f, kv = c["embedding_dim"], c["ffn_hidden"], c["embedding_dim"] // c["head_count"] * c["kv_head_count"]
    shapes = [("embed.weight", (c["vocab_size"], d))]
    for i in range(c["layer_count"]):
        for nm, shp in (("attn_norm.weight", (d,)), ("attn.wq", (d, d)), ("attn.wk", (kv, d)), ("attn.wv", (kv, d)),
                        ("attn.wo", (d, d)), ("mlp_norm.weight", (d,)), ("mlp.gate", (f, d)), ("mlp.up", (f, d)),
                        ("mlp.down", (d, f))):
            shapes.append((f"blocks.{i}.{nm}", shp))
    shapes.append(("final_norm.weight", (d,)))
    named = []
    for nm, shp in shapes:
        named += [(nm, be.allocate(shp)), (f"opt.m::{nm}", be.allocate(shp)), (f"opt.v::{nm}", be.allocate(shp))]
    total = sum(int(np.prod(t.shape)) for _, t in named) * 4
    tmp = tempfile.mkdtemp(prefix="pai-ckpt-")
    try:
        for rnd in range(2):  # the second round is the one reported (pinned buffers and snapshot block warm)
            path = os.path.join(tmp, f"step-{rnd + 1}.ckpt")  # a new file per save, as the trainer names them
            if rnd:
                os.remove(os.path.join(tmp, "step-1.ckpt"))
            be.sync()
            be.timer_start()
            h0 = time.perf_counter()
            be.save_checkpoint(path, rnd + 1, named, '{"Config": "1b"}')
            h1 = time.perf_counter()
            stall_ms = be.timer_stop()
            be.wait_checkpoint()
            h2 = time.perf_counter()
        size = os.path.getsize(path)
        be.sync()
        l0 = time.perf_counter()
        be.scope_begin()
        step, _, loaded = be.load_checkpoint(path)
        be.sync()
        l1 = time.perf_counter()
        be.scope_end()
        line = {"op": "checkpoint save/load (PAICKPT2, 1B params + AdamW moments)", "tensors": len(named),
                "bytes": size, "state_bytes": total, "save_call_ms": (h1 - h0) * 1e3,
                "compute_stream_ms": stall_ms, "snapshot_GBps": total / (stall_ms * 1e-3) / 1e9,
                "write_s": h2 - h0, "write_GBps": size / (h2 - h0) / 1e9, "load_s": l1 - l0,
                "load_GBps": size / (l1 - l0) / 1e9, "loaded_tensors": len(loaded), "step": step}
        print(json.dumps(line), flush=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def workload_config(name, n, recompute=True, zero1=False):
    c = CONFIGS[name]
    mode = "per-block recompute" if recompute else "stored activations, no recompute"
    return {"workload": f"llama-{name} train step (fwd + {mode} + bwd + AdamW), fp32 semantics",
            "vocab": c["vocab_size"], "d_model": c["embedding_dim"], "layers": c["layer_count"], "heads": c["head_count"],
            "kv_heads": c["kv_head_count"], "ffn": c["ffn_hidden"], "seq_len": c["seq"], "batch_per_gpu": c["batch"],
            "global_batch": c["batch"] * n, "params": param_count(c),
            "parallelism": f"dp{n}" + (" zero1 (AdamW state sharded)" if zero1 else ""),
            "l2": "working set above L2 (weights alone 4 B x params), no flush needed"}


def device_resident_run(be, tr, rank, c, step0, steps):
    """Uploads `steps` synthetic batches, then times them through Trainer.step_tensors with CUDA events on the
    library's stream. Returns (ms, last loss)."""
    batches = []
    for k in range(steps):
        x, y = synthetic_batch(rank, step0 + k, c["batch"], c["seq"], c["vocab_size"])
        batches.append((be.from_host(x), be.from_host(y)))
    be.sync()
    be.timer_start()
    loss = None
    for x, y in batches:
        loss = tr.step_tensors([x], [y])
    return be.timer_stop(), loss


def side_runs(be, m, args, c, peak_tf32):
    """N=1 extras: the same model without per-block recompute (tokens/s and the allocator's peak), then the ~125M
    config. Each on device-resident batches after its own warm-up steps."""
    out = {}
    steps = max(3, min(args.steps, 10))
    tc = H.TrainingConfig(batch_size=c["batch"], sequence_length=c["seq"], learning_rate=3e-4, weight_decay=0.1,
                          max_steps=100, gradient_checkpointing=False, warmup_steps=0)
    tr = H.Trainer(be, m, tc, 0.9, 0.95)
    tr.set_constant_lr(3e-4)
    for w in range(2):
        x, y = synthetic_batch(0, 500 + w, c["batch"], c["seq"], c["vocab_size"])
        tr.step([x], [y])
    be.sync()
    be.reset_peak()
    ms, _ = device_resident_run(be, tr, 0, c, 600, steps)
    peak = be.memory_stats()[1]
    tokens = c["batch"] * c["seq"] * steps
    mf, _ = flops_per_token(c, c["seq"])
    out["no_recompute"] = {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms / steps, "steps": steps,
                           "peak_allocated_gb": peak / 1e9,
                           "mfu": mf * tokens / (ms * 1e-3) / 1e12 / (peak_tf32 / 3.0)}
    del tr
    be.sync()
    return out


def small_config_run(be, args, name, peak_tf32):
    """tokens/s of another config (per-block recompute) on device-resident batches, value only."""
    c = CONFIGS[name]
    m = H.LlamaModel(be, model_config(c, c["seq"]), seed=0, init="normal0.02")
    tc = H.TrainingConfig(batch_size=c["batch"], sequence_length=c["seq"], learning_rate=3e-4, weight_decay=0.1,
                          max_steps=100, gradient_checkpointing=True, warmup_steps=0)
    tr = H.Trainer(be, m, tc, 0.9, 0.95)
    tr.set_constant_lr(3e-4)
    for w in range(3):
        x, y = synthetic_batch(0, w, c["batch"], c["seq"], c["vocab_size"])
        tr.step([x], [y])
    steps = max(3, args.steps)
    be.reset_peak()
    ms, loss = device_resident_run(be, tr, 0, c, 3, steps)
    tokens = c["batch"] * c["seq"] * steps
    mf, hf = flops_per_token(c, c["seq"])
    res = {"workload": workload_config(name, 1)["workload"], "value": tokens / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms / steps, "steps": steps, "peak_allocated_gb": be.memory_stats()[1] / 1e9,
           "mfu": mf * tokens / (ms * 1e-3) / 1e12 / (peak_tf32 / 3.0),
           "hfu": hf * tokens / (ms * 1e-3) / 1e12 / (peak_tf32 / 3.0), "final_loss": loss}
    del tr, m
    be.sync()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--config", default="1b", choices=sorted(CONFIGS))
    ap.add_argument("--no-recompute", action="store_true")
    ap.add_argument("--zero1", action="store_true", help="N>1: shard the AdamW state over the ranks (ZeRO-1)")
    ap.add_argument("--cpu-sample-tokens", type=int, default=None,
                    help="tokens per CPU sample step (default: 16 for 1b, 64 for 125m and tiny)")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--skip-cpu-1thread", action="store_true", help="leave the single-thread CPU sample out")
    ap.add_argument("--skip-extra", action="store_true", help="leave the no-recompute and 125M runs out of the N=1 line")
    ap.add_argument("--op", default=None, choices=["all", "gemm", "gemm-only", "attention", "hbm", "decode", "decode-attn",
                                                   "checkpoint"],
                    help="op-level sweep instead of the training step")
    ap.add_argument("--shape", default=None, help="M,K,N for --op gemm; rows,K,N for --op decode; B,H,S,D for --op attention; "
                                                  "the batch for --op decode-attn")
    ap.add_argument("--adamw-elements", type=int, default=1_100_000_000, help="--op hbm: AdamW parameter count")
    ap.add_argument("--decode-cache-len", type=int, default=768, help="--op decode: cached positions for decode attention")
    ap.add_argument("--skip-decode", action="store_true", help="leave the ~1B decode measurement out of the N=1 line")
    ap.add_argument("--decode-only", action="store_true", help="print only the decode measurement")
    ap.add_argument("--decode-tokens", type=int, default=256)
    ap.add_argument("--decode-batches", default="1,32", help="--decode-only: batch sizes to generate at")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.op:
        return op_sweep(args)
    if args.decode_only:
        print(json.dumps(decode_bench(0, gen=args.decode_tokens, batches=tuple(int(v) for v in args.decode_batches.split(",")))),
              flush=True)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    c = CONFIGS[args.config]
    be = H.Backend(str(pai.CUDA_LIB_PATH), "pai_", local)
    if world > 1:
        uid = [be.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        be.nccl_init(uid[0], rank, world, 120000)

    peak_tf32 = measured_tf32_peak(local) if rank == 0 else None
    m = H.LlamaModel(be, model_config(c, c["seq"]), seed=0, init="normal0.02")
    tc = H.TrainingConfig(batch_size=c["batch"], sequence_length=c["seq"], learning_rate=3e-4, weight_decay=0.1,
                          max_steps=args.warmup + 2 * args.steps + 10, gradient_checkpointing=not args.no_recompute,
                          warmup_steps=0)
    tr = H.Trainer(be, m, tc, 0.9, 0.95)
    tr.set_constant_lr(3e-4)
    tr.zero1 = args.zero1 and world > 1

    def barrier():
        be.sync()
        if dist:
            dist.barrier()

    step = 0
    for _ in range(args.warmup):
        x, y = synthetic_batch(rank, step, c["batch"], c["seq"], c["vocab_size"])
        tr.step([x], [y])
        step += 1

    # ---- value: device-resident batches (uploaded before the timed region), no per-kernel instrumentation
    batches = []
    for k in range(args.steps):
        x, y = synthetic_batch(rank, step + k, c["batch"], c["seq"], c["vocab_size"])
        batches.append((be.from_host(x), be.from_host(y)))
    step += args.steps
    barrier()
    be.reset_peak()
    if world > 1:
        be.dp_stats()  # clears the warm-up steps' exposed all-reduce time
    launches0 = be.launch_count()
    losses = []
    with ClockSampler(local) as clocks:
        be.timer_start()
        for x, y in batches:
            losses.append(tr.step_tensors([x], [y]))
        ms = be.timer_stop()
    launches = be.launch_count() - launches0
    exposed_ms, exposed_steps = be.dp_stats() if world > 1 else (0.0, 0)
    mem_in_use, mem_peak, mem_reserved = be.memory_stats()
    be.check_device_error()
    barrier()

    # ---- per-kernel CUDA-event timing (the roofline's kernel durations), a separate pass over the same batches
    be.kernel_timing(True)
    be.timer_start()
    for x, y in batches:
        tr.step_tensors([x], [y])
    ms_timed = be.timer_stop()
    kstats = {f: be.kernel_stats(f) for f in ("gemm", "attn_fwd", "attn_bwd")}
    be.kernel_timing(False)
    barrier()
    del batches

    # ---- e2e: host buffers through the public step
    host_batches = [synthetic_batch(rank, step + k, c["batch"], c["seq"], c["vocab_size"]) for k in range(args.steps)]
    barrier()
    be.timer_start()
    for x, y in host_batches:
        losses.append(tr.step([x], [y]))
    ms_e2e = be.timer_stop()
    barrier()

    if dist:
        import torch
        t = torch.tensor([ms, ms_e2e, exposed_ms / max(exposed_steps, 1)], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e, exposed_per_step = t.tolist()

    tokens = c["batch"] * c["seq"] * world * args.steps
    value = tokens / (ms * 1e-3)
    e2e = tokens / (ms_e2e * 1e-3)
    line = None
    if rank == 0:
        g_launches, g_ms, g_flops = kstats["gemm"]
        avg_ms = g_ms / max(g_launches, 1)
        achieved = (g_flops / max(g_launches, 1)) / (avg_ms * 1e-3) / 1e12
        peak = peak_tf32 / 3.0
        traffic = ncu_traffic()
        # DRAM bytes of the captured GEMM launch, scaled to this step's average GEMM launch by algorithmic flops
        traffic_bytes = None
        if traffic and traffic.get("flops_per_launch"):
            traffic_bytes = traffic["bytes_per_launch"] * (g_flops / max(g_launches, 1)) / traffic["flops_per_launch"]
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "traffic": traffic_bytes,
                    "traffic_source": ("profiles/gemm_tcgen05_traffic.json: ncu dram__bytes_read+write of one "
                                       f"{traffic.get('shape')} launch, scaled by flops to the average launch")
                    if traffic else None,
                    "kernel": "k_gemm_tc (3xTF32 tcgen05)",
                    "peak_source": "measured on this GPU: cuBLAS TF32 GEMM (torch.matmul fp32, allow_tf32, 8192^3, best of 10)"
                                   f" = {peak_tf32:.1f} TFLOP/s, divided by 3 for 3xTF32",
                    "launches": g_launches, "avg_launch_ms": avg_ms,
                    "share_of_step": g_ms / ms_timed}
        kernels = {f: {"launches": v[0], "ms": v[1], "tflops": (v[2] / (v[1] * 1e-3) / 1e12) if v[1] else None,
                       "share_of_step": v[1] / ms_timed} for f, v in kstats.items()}
        mf, hf = flops_per_token(c, c["seq"])
        if args.no_recompute:
            hf = mf
        per_gpu = value / world
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (PcgRng token ids, N(0,0.02) weights)",
                "config": workload_config(args.config, world, not args.no_recompute, args.zero1 and world > 1),
                "roofline": roofline,
                "mfu": mf * per_gpu / 1e12 / peak, "hfu": hf * per_gpu / 1e12 / peak,
                "flops_per_token": {"model": mf, "hardware": hf,
                                    "note": "model = 3 x forward (linear layers, tied LM head, causal attention); "
                                            "hardware adds the recomputed block forwards; mfu/hfu are per GPU over "
                                            "the 3xTF32 ceiling (roofline.peak)"},
                "memory": {"peak_allocated_gb": mem_peak / 1e9, "reserved_gb": mem_reserved / 1e9,
                           "note": "device bytes held by tensors at the peak of the timed steps (weights, AdamW "
                                   "moments, gradients and activations), from the library's allocator"},
                "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 2 * c["batch"] * c["seq"] * 4,
                        "d2h_bytes_per_step": 4, "ms_per_step": ms_e2e / args.steps},
                "gpu_launches": launches, "kernels": kernels,
                "model_tflops_per_s": mf * per_gpu / 1e12,
                "recompute": not args.no_recompute, "final_loss": losses[-1],
                "clocks": clocks.summary(), "peak_tf32_tflops": peak_tf32}
        if world > 1:
            line["dp"] = {"exposed_allreduce_ms_per_step": exposed_per_step,
                          "exposed_share_of_step": exposed_per_step / (ms / args.steps),
                          "steps_counted": exposed_steps,
                          "note": "device time from the end of a step's backward (compute stream) to the end of its "
                                  "last NCCL all-reduce (communication stream), max over ranks; the per-block buckets "
                                  "before it overlap the backward"}
    del tr
    if rank == 0 and world == 1:
        if not args.skip_extra and not args.no_recompute:
            try:
                line.update(side_runs(be, m, args, c, peak_tf32))
                line["memory"]["no_recompute_peak_allocated_gb"] = line["no_recompute"]["peak_allocated_gb"]
            except Exception as e:  # the main line still prints; the failure is reported in its place
                line["no_recompute"] = {"error": f"{type(e).__name__}: {e}"}
        del m
        be.sync()
        if not args.skip_extra and args.config != "125m":
            try:
                line["extra_125m"] = small_config_run(be, args, "125m", peak_tf32)
            except Exception as e:
                line["extra_125m"] = {"error": f"{type(e).__name__}: {e}"}
        if not args.skip_decode:
            try:
                line["decode"] = decode_bench(local, gen=args.decode_tokens)
            except Exception as e:
                line["decode"] = {"error": f"{type(e).__name__}: {e}"}
        if not args.skip_cpu_baseline:
            threads = os.cpu_count() or 1
            seq = min(args.cpu_sample_tokens or CPU_SAMPLE_SEQ[args.config], c["seq"])
            v, dt = cpu_train_sample(args.config, seq, threads)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
                                    "sample": f"one training step of the {args.config} model (all parameters, AdamW "
                                              f"over all of them) at batch 1 x seq {seq} ({dt:.1f} s) on the CPU oracle"}
            if not args.skip_cpu_1thread:
                seq1 = min(CPU_SAMPLE_SEQ_1THREAD[args.config], c["seq"])
                v1, dt1 = cpu_train_sample(args.config, seq1, 1)
                line["cpu_baseline_1thread"] = {
                    "value": v1, "unit": "tokens/s", "cores": 1, "kind": "port", "cpu": cpu_model(),
                    "sample": f"one training step of the {args.config} model at batch 1 x seq {seq1} ({dt1:.1f} s) on "
                              f"the CPU oracle with one thread (the reference backend's loops, unparallelised)"}
    else:
        del m
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
