"""The C-ABI library loads and exports every entry point include/projectai_cuda.h declares (no device calls), and the
oracle library exports the contract ops under its own prefix."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import projectai_b200 as pai
from conftest import ORACLE_LIB, ROOT

HEADER = ROOT / "include" / "projectai_cuda.h"


def declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(pai_[a-z0-9_]+)\s*\(", text)))


def exported(lib: Path):
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_declares_the_contract():
    names = declared()
    for op in ["pai_add", "pai_matmul", "pai_softmax", "pai_rmsnorm", "pai_rotary", "pai_gather", "pai_scatter_add_rows",
               "pai_cross_entropy", "pai_cross_entropy_grad", "pai_cat", "pai_scope_begin", "pai_keep_alive",
               "pai_sdpa_fwd", "pai_sdpa_bwd", "pai_adamw_step", "pai_nccl_init", "pai_allreduce_bucket"]:
        assert op in names


def test_cuda_library_exports_every_declared_symbol():
    assert pai.CUDA_LIB_PATH.exists(), "build() has not produced the CUDA library"
    syms = exported(pai.CUDA_LIB_PATH)
    missing = [n for n in declared() if n not in syms]
    assert not missing, missing
    lib = ctypes.CDLL(str(pai.CUDA_LIB_PATH))  # loads without a GPU (no device call at load time)
    for n in declared():
        assert getattr(lib, n) is not None


def test_oracle_exports_contract_ops():
    syms = exported(ORACLE_LIB)
    for n in declared():
        op = n[len("pai_"):]
        if op in {"sdpa_fwd", "sdpa_bwd", "rmsnorm_bwd", "silu_mul_fwd", "silu_mul_bwd", "cross_entropy_fused", "adamw_step",
                  "nccl_unique_id", "nccl_init", "allreduce_bucket", "allreduce_wait", "nccl_abort", "dp_stats", "reduce_scatter_bucket", "allgather_bucket", "check_device_error",
                  "timer_start", "timer_stop", "launch_count", "kernel_timing", "kernel_stats", "rmsnorm_bwd_noalloc",
                  "write", "gather_dev", "rotary_at", "kv_append", "sdpa_decode", "graph_begin", "graph_end",
                  "graph_launch", "graph_destroy", "linear_fused", "rope_append", "attn_decode_step", "argmax_rows"}:
            continue  # fused extensions and diagnostics are CUDA-only
        if op.startswith(("ckpt_", "dataset_")):
            continue  # file I/O paths: their oracle is oracle/formats.py (tests/test_formats.py)
        assert "oracle_" + op in syms, op


def test_cuda_backend_fails_loudly_without_a_device():
    from conftest import HAS_GPU
    if HAS_GPU:
        pytest.skip("a device is present")
    from projectai_b200 import _paihost as H
    with pytest.raises(H.BackendError):
        H.Backend(str(pai.CUDA_LIB_PATH), "pai_", 0)
