"""The allocation-free RMSNorm backward (pai_rmsnorm_bwd_noalloc), for callers that cannot allocate device memory.

It is called through the C ABI twice in a row, on different inputs, with output tensors the caller allocated
beforehand. Each time it must match the allocating entry point pai_rmsnorm_bwd, to the tolerance the op tests use
(|e - g| <= 1e-4 + 1e-4·|e|), and leave the context's allocator untouched. This file is collected last, so a run
that stops at the first failure has already run every other test. It also passes when run alone.
"""
import ctypes

import numpy as np
import pytest

import projectai_b200 as pai
from projectai_b200 import cabi

pytestmark = pytest.mark.gpu


def test_rmsnorm_bwd_noalloc_matches_the_allocating_entry_point():
    be = cabi.NativeBackend(pai.cuda_library(), 0)
    try:
        rng = np.random.RandomState(0)
        for call, (rows, d) in enumerate([(300, 768), (77, 2048)]):  # two calls in a row, sharing the scratch array
            x = be.from_host(rng.standard_normal((rows, d)).astype(np.float32))
            w = be.from_host(rng.standard_normal(d).astype(np.float32))
            g = be.from_host(rng.standard_normal((rows, d)).astype(np.float32))
            ref_dx, ref_dw = be.rmsnorm_bwd(x, w, g, 1e-5)
            dx = be.allocate((rows, d))  # the caller's output buffers, allocated before the call
            dw = be.allocate((d,))
            be.sync()
            before = be.memory_stats()
            pai.cuda_library().call("rmsnorm_bwd_noalloc", be.ctx, ctypes.byref(x), ctypes.byref(w), ctypes.byref(g),
                                    ctypes.c_float(1e-5), ctypes.byref(dx), ctypes.byref(dw))
            be.sync()
            after = be.memory_stats()
            assert after[0] == before[0] and after[2] == before[2], f"call {call} allocated: {before} -> {after}"
            for exp, got, name in ((be.to_host(ref_dx), be.to_host(dx), "dx"), (be.to_host(ref_dw), be.to_host(dw), "dw")):
                tol = 1e-4 + 1e-4 * np.abs(exp)
                assert np.all(np.abs(exp - got) <= tol), f"call {call}: {name} differs"
        # rows longer than the scratch array's limit are rejected with a clear error
        big = be.from_host(np.ones((1, 8200), np.float32))
        with pytest.raises(cabi.OutOfRangeError, match="at most 8192"):
            pai.cuda_library().call("rmsnorm_bwd_noalloc", be.ctx, ctypes.byref(big),
                                    ctypes.byref(be.from_host(np.ones(8200, np.float32))), ctypes.byref(big),
                                    ctypes.c_float(1e-5), ctypes.byref(big), ctypes.byref(be.allocate((8200,))))
        assert be.check_device_error() == 0
    finally:
        be.close()
