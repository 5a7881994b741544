"""projectai_b200 — a B200-native (sm_100a) compute backend for project-ai's IComputeBackend seam.

* ``libprojectai_cuda.so`` (``lib/``) implements the C ABI of ``include/projectai_cuda.h``: every contract op and the
  fused extensions as hand-written sm_100a kernels, a stream-ordered caching allocator with scopes, and NCCL
  data parallelism.
* ``_paihost`` is the C++ host runtime that drives it the way the reference's C# host does: tensor views, the
  autograd tape, the Llama modules, AdamW, the trainer with per-block recompute, and KV-cache decode.

There is no CPU fallback: the entry points raise if the CUDA library or a CUDA device is missing.
"""
from __future__ import annotations

from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CUDA_LIB_PATH = PKG_DIR / "lib" / "libprojectai_cuda.so"

_cuda_library = None


def cuda_library():
    """The loaded CUDA backend library (``pai_`` entry points). Raises if it has not been built."""
    global _cuda_library
    if _cuda_library is None:
        if not CUDA_LIB_PATH.exists():
            raise RuntimeError(f"{CUDA_LIB_PATH} is missing: build it with __graft_entry__.build()")
        from .cabi import NativeLibrary

        _cuda_library = NativeLibrary(CUDA_LIB_PATH, "pai_")
    return _cuda_library


def cuda_backend(device: int = 0):
    """An op-level handle on one device (the C ABI through ctypes)."""
    from .cabi import NativeBackend

    return NativeBackend(cuda_library(), device)
