"""ctypes binding of the C ABI in ``include/projectai_cuda.h``.

``NativeBackend`` drives one library context through the same entry points a P/Invoke layer for
``ProjectAI.Core/IComputeBackend.cs`` binds: tensors are ``pai_tensor`` descriptors (storage base, element offset,
shape, element strides), every op returns a fresh contiguous tensor, and failures raise the exception class the
reference throws for the same condition (``ArgumentError`` ~ ArgumentException, ``OutOfRangeError`` ~
ArgumentOutOfRangeException, ``MemoryError`` for out-of-memory with the message containing "out of memory").

View helpers (``transpose``, ``slice``, ``broadcast_to``, ``reshape``) rewrite descriptors only, as the view
operations of ``ProjectAI.Core/Tensor.cs:75-168`` do.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint8, c_void_p
from pathlib import Path

import numpy as np

MAX_RANK = 8
F32 = 0


class PaiTensor(ctypes.Structure):
    _fields_ = [
        ("base", c_void_p),
        ("offset", c_int64),
        ("rank", c_int32),
        ("dtype", c_int32),
        ("dims", c_int32 * MAX_RANK),
        ("strides", c_int64 * MAX_RANK),
    ]

    @property
    def shape(self) -> tuple:
        return tuple(self.dims[i] for i in range(self.rank))

    @property
    def stride(self) -> tuple:
        return tuple(self.strides[i] for i in range(self.rank))

    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def copy_desc(self) -> "PaiTensor":
        t = PaiTensor()
        ctypes.memmove(ctypes.byref(t), ctypes.byref(self), ctypes.sizeof(PaiTensor))
        return t

    def is_contiguous(self) -> bool:
        acc = 1
        for d, s in reversed(list(zip(self.shape, self.stride))):
            if d == 1:
                continue
            if s != acc:
                return False
            acc *= d
        return True

    def __repr__(self) -> str:
        return f"PaiTensor(shape={self.shape}, strides={self.stride}, offset={self.offset})"


class BackendError(RuntimeError):
    pass


class ArgumentError(BackendError, ValueError):
    pass


class OutOfRangeError(ArgumentError, IndexError):
    pass


class InvalidOperationError(BackendError):
    pass


class DeviceTimeoutError(BackendError, TimeoutError):
    pass


class UnsupportedError(BackendError, NotImplementedError):
    pass


class FileIOError(BackendError, OSError):
    """IOException / FileNotFoundException: a checkpoint or dataset file could not be opened, read or written."""


class InvalidDataError(BackendError, ValueError):
    """InvalidDataException: a checkpoint or dataset file is malformed (ProjectAI.Formats/Checkpoint.cs:59-139)."""


_STATUS = {1: ArgumentError, 2: OutOfRangeError, 3: InvalidOperationError, 4: MemoryError, 5: BackendError,
           6: BackendError, 7: DeviceTimeoutError, 8: UnsupportedError, 9: FileIOError, 10: InvalidDataError}

T = POINTER(PaiTensor)
_I32P = POINTER(c_int32)
_SIGS = {
    "ctx_create": [c_int32, POINTER(c_void_p)],
    "ctx_destroy": [c_void_p],
    "sync": [c_void_p],
    "device_name": [c_void_p, c_char_p, c_int32],
    "alloc": [c_void_p, c_int32, _I32P, c_int32, T],
    "from_host": [c_void_p, POINTER(c_float), c_int64, c_int32, _I32P, c_int32, T],
    "to_host": [c_void_p, T, POINTER(c_float), c_int64],
    "copy": [c_void_p, T, T],
    "scope_begin": [c_void_p],
    "scope_end": [c_void_p],
    "keep_alive": [c_void_p, c_void_p],
    "release": [c_void_p, c_void_p],
    "finalize": [c_void_p, c_void_p],
    "memory_stats": [c_void_p, POINTER(c_int64), POINTER(c_int64), POINTER(c_int64)],
    "reset_peak": [c_void_p],
    "add": [c_void_p, T, T, T], "sub": [c_void_p, T, T, T], "mul": [c_void_p, T, T, T], "div": [c_void_p, T, T, T],
    "add_scalar": [c_void_p, T, c_float, T], "mul_scalar": [c_void_p, T, c_float, T],
    "sqrt": [c_void_p, T, T], "sigmoid": [c_void_p, T, T], "silu": [c_void_p, T, T],
    "matmul": [c_void_p, T, T, c_int32, T],
    "sum": [c_void_p, T, c_int32, c_int32, T], "mean": [c_void_p, T, c_int32, c_int32, T],
    "max": [c_void_p, T, c_int32, c_int32, T],
    "softmax": [c_void_p, T, c_int32, T],
    "rmsnorm": [c_void_p, T, T, c_float, T],
    "rotary": [c_void_p, T, T, T, T],
    "gather": [c_void_p, T, _I32P, c_int64, T],
    "scatter_add_rows": [c_void_p, T, _I32P, c_int64, c_int32, T],
    "cross_entropy": [c_void_p, T, _I32P, c_int64, c_int32, T],
    "cross_entropy_grad": [c_void_p, T, _I32P, c_int64, c_int32, T],
    "cat": [c_void_p, T, T, c_int32, T],
    "sdpa_fwd": [c_void_p, T, T, T, c_float, c_int32, c_int32, T, T],
    "sdpa_bwd": [c_void_p, T, T, T, T, T, T, c_float, c_int32, c_int32, T, T, T],
    "rmsnorm_bwd": [c_void_p, T, T, T, c_float, T, T],
    "silu_mul_fwd": [c_void_p, T, T, T],
    "silu_mul_bwd": [c_void_p, T, T, T, T, T],
    "cross_entropy_fused": [c_void_p, T, _I32P, c_int64, c_int32, c_float, T, T],
    "adamw_step": [c_void_p, T, T, T, T, c_float, c_float, c_float, c_float, c_float, c_int32, c_float],
    "nccl_unique_id": [POINTER(c_uint8)],
    "nccl_init": [c_void_p, POINTER(c_uint8), c_int32, c_int32, c_int32],
    "allreduce_bucket": [c_void_p, T, c_int32],
    "allreduce_wait": [c_void_p],
    "nccl_abort": [c_void_p],
    "check_device_error": [c_void_p, _I32P],
    "ckpt_save": [c_void_p, c_char_p, c_int32, c_char_p, c_int64, c_char_p, c_int64, T, c_int32],
    "ckpt_wait": [c_void_p],
    "ckpt_load": [c_void_p, c_char_p, c_int32, _I32P, POINTER(c_int64), _I32P],
    "ckpt_meta": [c_void_p, c_char_p, c_int64],
    "ckpt_tensor": [c_void_p, c_int32, c_char_p, c_int64, POINTER(c_int64), T],
    "ckpt_close": [c_void_p],
    "dataset_open": [c_void_p, c_char_p, c_int32, c_int32, c_int64],
    "dataset_batch": [c_void_p, POINTER(c_int64), c_int32, T, T],
    "dataset_close": [c_void_p],
    "rmsnorm_bwd_noalloc": [c_void_p, T, T, T, c_float, T, T],
    "timer_start": [c_void_p],
    "timer_stop": [c_void_p, POINTER(c_float)],
    "launch_count": [c_void_p, POINTER(c_int64)],
}


class NativeLibrary:
    """A loaded backend library whose entry points share one prefix (``pai_`` for the CUDA backend)."""

    def __init__(self, path: str | Path, prefix: str = "pai_"):
        self.path = str(path)
        self.prefix = prefix
        self.lib = ctypes.CDLL(self.path)
        self.fns = {}
        for name, args in _SIGS.items():
            f = getattr(self.lib, prefix + name, None)
            if f is None:
                continue
            f.argtypes = args
            f.restype = c_int32
            self.fns[name] = f
        err = getattr(self.lib, prefix + "last_error")
        err.argtypes = []
        err.restype = c_char_p
        self._err = err

    def has(self, name: str) -> bool:
        return name in self.fns

    def call(self, name: str, *args) -> None:
        f = self.fns.get(name)
        if f is None:
            raise UnsupportedError(f"{self.prefix}{name} is not provided by {self.path}")
        st = f(*args)
        if st != 0:
            msg = self._err().decode(errors="replace")
            raise _STATUS.get(st, BackendError)(msg)


def _dims(shape) -> ctypes.Array:
    arr = (c_int32 * MAX_RANK)()
    for i, d in enumerate(shape):
        arr[i] = int(d)
    return arr


def _ids(ids) -> tuple:
    a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    return a, a.ctypes.data_as(_I32P), a.size


class NativeBackend:
    """One context of a backend library; op names follow IComputeBackend (ProjectAI.Core/IComputeBackend.cs:9-96)."""

    def __init__(self, library: NativeLibrary, device: int = 0):
        self.library = library
        self.ctx = c_void_p()
        library.call("ctx_create", device, ctypes.byref(self.ctx))

    def close(self) -> None:
        if self.ctx:
            self.library.call("ctx_destroy", self.ctx)
            self.ctx = c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _c(self, name, *args):
        self.library.call(name, self.ctx, *args)

    @property
    def name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        self._c("device_name", buf, 256)
        return buf.value.decode()

    # --- allocation & transfer
    def allocate(self, shape) -> PaiTensor:
        out = PaiTensor()
        self._c("alloc", len(shape), _dims(shape), F32, ctypes.byref(out))
        return out

    def from_host(self, data, shape=None) -> PaiTensor:
        a = np.ascontiguousarray(np.asarray(data, dtype=np.float32))
        shape = a.shape if shape is None else tuple(shape)
        out = PaiTensor()
        self._c("from_host", a.ctypes.data_as(POINTER(c_float)), a.size, len(shape), _dims(shape), F32, ctypes.byref(out))
        return out

    def to_host(self, t: PaiTensor) -> np.ndarray:
        out = np.empty(t.shape, dtype=np.float32)
        self._c("to_host", ctypes.byref(t), out.ctypes.data_as(POINTER(c_float)), out.size)
        return out

    def copy(self, src: PaiTensor, dst: PaiTensor) -> None:
        self._c("copy", ctypes.byref(src), ctypes.byref(dst))

    def sync(self) -> None:
        self._c("sync")

    # --- scopes
    def scope_begin(self):
        self._c("scope_begin")

    def scope_end(self):
        self._c("scope_end")

    def keep_alive(self, t: PaiTensor):
        self._c("keep_alive", t.base)

    def release(self, t: PaiTensor):
        self._c("release", t.base)

    def memory_stats(self) -> tuple:
        a, b, c = c_int64(), c_int64(), c_int64()
        self._c("memory_stats", ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    # --- ops
    def _unary(self, name, x, *extra):
        out = PaiTensor()
        self._c(name, ctypes.byref(x), *extra, ctypes.byref(out))
        return out

    def _binary(self, name, a, b, *extra):
        out = PaiTensor()
        self._c(name, ctypes.byref(a), ctypes.byref(b), *extra, ctypes.byref(out))
        return out

    def add(self, a, b): return self._binary("add", a, b)
    def sub(self, a, b): return self._binary("sub", a, b)
    def mul(self, a, b): return self._binary("mul", a, b)
    def div(self, a, b): return self._binary("div", a, b)
    def add_scalar(self, a, s): return self._unary("add_scalar", a, c_float(s))
    def mul_scalar(self, a, s): return self._unary("mul_scalar", a, c_float(s))
    def sqrt(self, x): return self._unary("sqrt", x)
    def sigmoid(self, x): return self._unary("sigmoid", x)
    def silu(self, x): return self._unary("silu", x)
    def matmul(self, a, b, transpose_b=False): return self._binary("matmul", a, b, int(bool(transpose_b)))
    def sum(self, x, axis, keep_dims=False): return self._unary("sum", x, axis, int(keep_dims))
    def mean(self, x, axis, keep_dims=False): return self._unary("mean", x, axis, int(keep_dims))
    def max(self, x, axis, keep_dims=False): return self._unary("max", x, axis, int(keep_dims))
    def softmax(self, x, axis): return self._unary("softmax", x, axis)
    def rmsnorm(self, x, w, eps): return self._binary("rmsnorm", x, w, c_float(eps))

    def rotary(self, x, cos, sin):
        out = PaiTensor()
        self._c("rotary", ctypes.byref(x), ctypes.byref(cos), ctypes.byref(sin), ctypes.byref(out))
        return out

    def gather(self, table, ids):
        keep, p, n = _ids(ids)
        return self._unary("gather", table, p, n)

    def scatter_add_rows(self, rows, ids, row_count):
        keep, p, n = _ids(ids)
        return self._unary("scatter_add_rows", rows, p, n, row_count)

    def cross_entropy(self, logits, targets, ignore_index=-100):
        keep, p, n = _ids(targets)
        return self._unary("cross_entropy", logits, p, n, ignore_index)

    def cross_entropy_grad(self, logits, targets, ignore_index=-100):
        keep, p, n = _ids(targets)
        return self._unary("cross_entropy_grad", logits, p, n, ignore_index)

    def cross_entropy_fused(self, logits, targets, ignore_index=-100, grad_scale=1.0):
        keep, p, n = _ids(targets)
        loss, grad = PaiTensor(), PaiTensor()
        self._c("cross_entropy_fused", ctypes.byref(logits), p, n, ignore_index, c_float(grad_scale),
                ctypes.byref(loss), ctypes.byref(grad))
        return loss, grad

    def cat(self, a, b, axis): return self._binary("cat", a, b, axis)

    def sdpa_fwd(self, q, k, v, scale, causal=True, pos_offset=0):
        out, lse = PaiTensor(), PaiTensor()
        self._c("sdpa_fwd", ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), c_float(scale), int(causal), pos_offset,
                ctypes.byref(out), ctypes.byref(lse))
        return out, lse

    def sdpa_bwd(self, q, k, v, out, lse, dout, scale, causal=True, pos_offset=0):
        dq, dk, dv = PaiTensor(), PaiTensor(), PaiTensor()
        self._c("sdpa_bwd", ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(out), ctypes.byref(lse),
                ctypes.byref(dout), c_float(scale), int(causal), pos_offset, ctypes.byref(dq), ctypes.byref(dk),
                ctypes.byref(dv))
        return dq, dk, dv

    def rmsnorm_bwd(self, x, w, g, eps):
        dx, dw = PaiTensor(), PaiTensor()
        self._c("rmsnorm_bwd", ctypes.byref(x), ctypes.byref(w), ctypes.byref(g), c_float(eps), ctypes.byref(dx),
                ctypes.byref(dw))
        return dx, dw

    def silu_mul_fwd(self, gate, up): return self._binary("silu_mul_fwd", gate, up)

    def silu_mul_bwd(self, gate, up, g):
        dg, du = PaiTensor(), PaiTensor()
        self._c("silu_mul_bwd", ctypes.byref(gate), ctypes.byref(up), ctypes.byref(g), ctypes.byref(dg), ctypes.byref(du))
        return dg, du

    def adamw_step(self, p, g, m, v, lr, beta1, beta2, eps, weight_decay, t, grad_scale=1.0):
        self._c("adamw_step", ctypes.byref(p), ctypes.byref(g), ctypes.byref(m), ctypes.byref(v), c_float(lr),
                c_float(beta1), c_float(beta2), c_float(eps), c_float(weight_decay), int(t), c_float(grad_scale))

    def timer_start(self) -> None:
        self._c("timer_start")

    def timer_stop(self) -> float:
        ms = c_float()
        self._c("timer_stop", ctypes.byref(ms))
        return ms.value

    def check_device_error(self) -> int:
        code = c_int32()
        self._c("check_device_error", ctypes.byref(code))
        return code.value

    # --- checkpoints (ProjectAI.Formats/Checkpoint.cs) and packed datasets (ProjectAI.Training/PackedBinDataset.cs)
    def save_checkpoint(self, path, step: int, tensors, metadata: str = "") -> None:
        """Checkpoint.Save: `tensors` is a sequence of (name, PaiTensor). Returns once the tensors are snapshotted on
        the device; the file is written in the background until wait_checkpoint()."""
        items = list(tensors)
        names = b"".join(n.encode() + b"\0" for n, _ in items)
        arr = (PaiTensor * max(1, len(items)))(*[t for _, t in items])
        meta = metadata.encode()
        self._c("ckpt_save", str(path).encode(), int(step), meta, len(meta), names, len(names), arr, len(items))

    def wait_checkpoint(self) -> None:
        self._c("ckpt_wait")

    def _ckpt_header(self, path, header_only):
        step, mlen, count = c_int32(), c_int64(), c_int32()
        self._c("ckpt_load", str(path).encode(), int(header_only), ctypes.byref(step), ctypes.byref(mlen), ctypes.byref(count))
        buf = ctypes.create_string_buffer(max(1, mlen.value))
        self._c("ckpt_meta", buf, mlen.value)
        return step.value, buf.raw[:mlen.value].decode(), count.value

    def load_checkpoint(self, path) -> tuple:
        """Checkpoint.Load: (step, metadata, {name: PaiTensor}) with the tensors on the device in the current scope."""
        step, meta, count = self._ckpt_header(path, False)
        out = {}
        for i in range(count):
            nlen = c_int64()
            self._c("ckpt_tensor", i, None, 0, ctypes.byref(nlen), None)
            name = ctypes.create_string_buffer(max(1, nlen.value))
            t = PaiTensor()
            self._c("ckpt_tensor", i, name, nlen.value, None, ctypes.byref(t))
            out[name.raw[:nlen.value].decode()] = t
        self._c("ckpt_close")
        return step, meta, out

    def read_checkpoint_metadata(self, path) -> tuple:
        """Checkpoint.ReadMetadata: (step, metadata) from the header alone."""
        step, meta, _ = self._ckpt_header(path, True)
        self._c("ckpt_close")
        return step, meta

    def dataset_open(self, bin_path, dtype: str, seq_len: int, block_count: int) -> None:
        widths = {"u16": 2, "u32": 4}
        self._c("dataset_open", str(bin_path).encode(), widths.get(dtype, 0), int(seq_len), int(block_count))

    def dataset_batch(self, indices) -> tuple:
        """NextBatch over the given block indices: (inputs, targets) [len(indices), seq_len] F32 ids on the device."""
        idx = np.ascontiguousarray(np.asarray(indices, dtype=np.int64))
        inp, tgt = PaiTensor(), PaiTensor()
        self._c("dataset_batch", idx.ctypes.data_as(POINTER(c_int64)), idx.size, ctypes.byref(inp), ctypes.byref(tgt))
        return inp, tgt

    def dataset_close(self) -> None:
        self._c("dataset_close")


# --- view helpers (ProjectAI.Core/Tensor.cs:75-168): metadata only, storage shared
def transpose(t: PaiTensor, a0: int, a1: int) -> PaiTensor:
    r = t.copy_desc()
    r.dims[a0], r.dims[a1] = t.dims[a1], t.dims[a0]
    r.strides[a0], r.strides[a1] = t.strides[a1], t.strides[a0]
    return r


def slice_view(t: PaiTensor, axis: int, start: int, length: int) -> PaiTensor:
    if start < 0 or length < 0 or start + length > t.dims[axis]:
        raise OutOfRangeError(f"Slice [{start}, {start + length}) is out of range for axis {axis} (size {t.dims[axis]}).")
    r = t.copy_desc()
    r.dims[axis] = length
    r.offset = t.offset + start * t.strides[axis]
    return r


def broadcast_to(t: PaiTensor, shape) -> PaiTensor:
    shape = tuple(shape)
    lead = len(shape) - t.rank
    if lead < 0:
        raise ArgumentError(f"Cannot broadcast {t.shape} to fewer dimensions {shape}.")
    r = t.copy_desc()
    r.rank = len(shape)
    for i, d in enumerate(shape):
        r.dims[i] = d
        if i < lead:
            r.strides[i] = 0
            continue
        s = t.dims[i - lead]
        if s == d:
            r.strides[i] = t.strides[i - lead]
        elif s == 1:
            r.strides[i] = 0
        else:
            raise ArgumentError(f"Cannot broadcast {t.shape} to {shape}: axis {i} ({s} vs {d}).")
    return r


def reshape(t: PaiTensor, shape) -> PaiTensor:
    if not t.is_contiguous():
        raise InvalidOperationError("Reshape requires a contiguous tensor; materialize it first.")
    shape = tuple(int(d) for d in shape)
    n = 1
    for d in shape:
        n *= d
    if n != t.numel():
        raise ArgumentError(f"Cannot reshape {t.shape} to {shape}.")
    r = t.copy_desc()
    r.rank = len(shape)
    acc = 1
    for i in range(len(shape) - 1, -1, -1):
        r.dims[i] = shape[i]
        r.strides[i] = acc
        acc *= shape[i]
    return r
