"""Backend conformance: every IComputeBackend op on the CUDA library against the CPU oracle.

Restates the 30 op cases of ProjectAI.Tests/BackendConformanceTests.cs:60-113 (elementwise + broadcasting,
MatMul 2-D / batched / transposeB / GQA batch broadcast, reductions, transformer primitives, strided / sliced /
stride-0 views, Cat with a strided operand, Gather / ScatterAddRows / CrossEntropy), compared element-wise with
the reference's own tolerance |e − g| <= 1e-4 + 1e-4·|e| (BackendConformanceTests.cs:19-20,45-56).

Inputs are seeded uniform(-1, 1) draws, the same arrays fed to both sides (the reference draws from
System.Random; parity needs identical inputs on both sides, not .NET's stream).
"""
import numpy as np
import pytest

from projectai_b200 import cabi

ATOL = 1e-4
RTOL = 1e-4


def rand(seed, *dims):
    return np.random.RandomState(seed).uniform(-1, 1, size=dims).astype(np.float32)


def T(be, seed, *dims):
    return be.from_host(rand(seed, *dims), dims)


def TPos(be, seed, *dims):
    return be.from_host(np.abs(rand(seed, *dims)) + np.float32(0.1), dims)


def H(be, t):
    return be.to_host(t).reshape(-1)


CASES = {
    "Add": lambda be: H(be, be.add(T(be, 1, 2, 3, 4), T(be, 2, 2, 3, 4))),
    "Add[broadcast]": lambda be: H(be, be.add(T(be, 1, 2, 3, 4), T(be, 2, 4))),
    "Sub": lambda be: H(be, be.sub(T(be, 1, 2, 3, 4), T(be, 2, 2, 3, 4))),
    "Mul": lambda be: H(be, be.mul(T(be, 1, 2, 3, 4), T(be, 2, 2, 3, 4))),
    "Mul[broadcast]": lambda be: H(be, be.mul(T(be, 1, 2, 3, 4), T(be, 2, 1, 1, 4))),
    "Div": lambda be: H(be, be.div(T(be, 1, 2, 3, 4), TPos(be, 2, 2, 3, 4))),
    "AddScalar": lambda be: H(be, be.add_scalar(T(be, 1, 2, 3, 4), 0.75)),
    "MulScalar": lambda be: H(be, be.mul_scalar(T(be, 1, 2, 3, 4), -1.5)),
    "Sqrt": lambda be: H(be, be.sqrt(TPos(be, 1, 2, 3, 4))),
    "Sigmoid": lambda be: H(be, be.sigmoid(T(be, 1, 2, 3, 4))),
    "MatMul[2D]": lambda be: H(be, be.matmul(T(be, 1, 3, 4), T(be, 2, 4, 5))),
    "MatMul[batched]": lambda be: H(be, be.matmul(T(be, 1, 2, 3, 4), T(be, 2, 2, 4, 5))),
    "MatMul[transposeB]": lambda be: H(be, be.matmul(T(be, 1, 3, 4), T(be, 2, 5, 4), transpose_b=True)),
    "Sum[axis=-1]": lambda be: H(be, be.sum(T(be, 1, 2, 3, 4), -1)),
    "Sum[axis=0,keepDims]": lambda be: H(be, be.sum(T(be, 1, 2, 3, 4), 0, keep_dims=True)),
    "Mean[axis=-1]": lambda be: H(be, be.mean(T(be, 1, 2, 3, 4), -1)),
    "Max[axis=1]": lambda be: H(be, be.max(T(be, 1, 2, 3, 4), 1)),
    "Softmax[axis=-1]": lambda be: H(be, be.softmax(T(be, 1, 2, 3, 4), -1)),
    "RmsNorm": lambda be: H(be, be.rmsnorm(T(be, 1, 2, 3, 4), T(be, 9, 4), 1e-5)),
    "Silu": lambda be: H(be, be.silu(T(be, 1, 2, 3, 4))),
    "RotaryEmbedding": lambda be: H(be, be.rotary(T(be, 1, 1, 2, 3, 4), T(be, 2, 3, 4), T(be, 3, 3, 4))),
    "Softmax[transposed]": lambda be: H(be, be.softmax(cabi.transpose(T(be, 1, 3, 4), 0, 1), -1)),
    "Sum[sliced,offset]": lambda be: H(be, be.sum(cabi.slice_view(T(be, 1, 4, 5), 0, 1, 2), -1)),
    "Add[stride-0 broadcast view]": lambda be: H(be, be.add(T(be, 1, 2, 3, 4),
                                                            cabi.broadcast_to(T(be, 2, 1, 1, 4), (2, 3, 4)))),
    "MatMul[batch-broadcast,GQA]": lambda be: H(be, be.matmul(T(be, 1, 2, 2, 3, 4, 6), T(be, 2, 2, 2, 1, 5, 6),
                                                              transpose_b=True)),
    "Cat[axis=2]": lambda be: H(be, be.cat(T(be, 1, 2, 3, 4, 5), T(be, 2, 2, 3, 6, 5), 2)),
    "Cat[axis=-1]": lambda be: H(be, be.cat(T(be, 3, 2, 3, 4), T(be, 4, 2, 3, 6), -1)),
    "Cat[strided incoming]": lambda be: H(be, be.cat(T(be, 5, 2, 3, 4, 5), cabi.transpose(T(be, 6, 2, 6, 3, 5), 1, 2), 2)),
    "Gather": lambda be: H(be, be.gather(T(be, 1, 6, 4), [0, 2, 5, 2])),
    "ScatterAddRows": lambda be: H(be, be.scatter_add_rows(T(be, 1, 4, 4), [0, 2, 5, 2], 6)),
    "CrossEntropy": lambda be: H(be, be.cross_entropy(T(be, 1, 4, 5), [1, 3, 0, 2], -100)),
    "CrossEntropy[ignore]": lambda be: H(be, be.cross_entropy(T(be, 1, 4, 5), [1, -100, 0, 2], -100)),
    "CrossEntropyGrad": lambda be: H(be, be.cross_entropy_grad(T(be, 1, 4, 5), [1, -100, 0, 2], -100)),
}


def _numpy_reference(name):
    """Independent float64 numpy statement of each case, to check the oracle itself on CPU."""
    r = rand
    pos = lambda s, *d: np.abs(r(s, *d)).astype(np.float64) + np.float32(0.1)
    f = lambda s, *d: r(s, *d).astype(np.float64)

    def softmax(x, axis):
        e = np.exp(x - x.max(axis=axis, keepdims=True))
        return e / e.sum(axis=axis, keepdims=True)

    def rope(x, c, s):
        half = x.shape[-1] // 2
        rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
        return x * c + rot * s

    def ce(logits, targets, ignore):
        rows = [(i, t) for i, t in enumerate(targets) if t != ignore]
        lse = np.log(np.exp(logits - logits.max(1, keepdims=True)).sum(1)) + logits.max(1)
        return np.array([np.mean([lse[i] - logits[i, t] for i, t in rows])])

    def ce_grad(logits, targets, ignore):
        cnt = sum(1 for t in targets if t != ignore)
        g = softmax(logits, 1) / cnt
        for i, t in enumerate(targets):
            if t == ignore:
                g[i] = 0
            else:
                g[i, t] -= 1.0 / cnt
        return g

    table = {
        "Add": lambda: f(1, 2, 3, 4) + f(2, 2, 3, 4),
        "Add[broadcast]": lambda: f(1, 2, 3, 4) + f(2, 4),
        "Sub": lambda: f(1, 2, 3, 4) - f(2, 2, 3, 4),
        "Mul": lambda: f(1, 2, 3, 4) * f(2, 2, 3, 4),
        "Mul[broadcast]": lambda: f(1, 2, 3, 4) * f(2, 1, 1, 4),
        "Div": lambda: f(1, 2, 3, 4) / pos(2, 2, 3, 4),
        "AddScalar": lambda: f(1, 2, 3, 4) + 0.75,
        "MulScalar": lambda: f(1, 2, 3, 4) * -1.5,
        "Sqrt": lambda: np.sqrt(pos(1, 2, 3, 4)),
        "Sigmoid": lambda: 1 / (1 + np.exp(-f(1, 2, 3, 4))),
        "MatMul[2D]": lambda: f(1, 3, 4) @ f(2, 4, 5),
        "MatMul[batched]": lambda: f(1, 2, 3, 4) @ f(2, 2, 4, 5),
        "MatMul[transposeB]": lambda: f(1, 3, 4) @ f(2, 5, 4).T,
        "Sum[axis=-1]": lambda: f(1, 2, 3, 4).sum(-1),
        "Sum[axis=0,keepDims]": lambda: f(1, 2, 3, 4).sum(0, keepdims=True),
        "Mean[axis=-1]": lambda: f(1, 2, 3, 4).mean(-1),
        "Max[axis=1]": lambda: f(1, 2, 3, 4).max(1),
        "Softmax[axis=-1]": lambda: softmax(f(1, 2, 3, 4), -1),
        "RmsNorm": lambda: f(1, 2, 3, 4) / np.sqrt((f(1, 2, 3, 4) ** 2).mean(-1, keepdims=True) + 1e-5) * f(9, 4),
        "Silu": lambda: f(1, 2, 3, 4) / (1 + np.exp(-f(1, 2, 3, 4))),
        "RotaryEmbedding": lambda: rope(f(1, 1, 2, 3, 4), f(2, 3, 4), f(3, 3, 4)),
        "Softmax[transposed]": lambda: softmax(f(1, 3, 4).T, -1),
        "Sum[sliced,offset]": lambda: f(1, 4, 5)[1:3].sum(-1),
        "Add[stride-0 broadcast view]": lambda: f(1, 2, 3, 4) + f(2, 1, 1, 4),
        "MatMul[batch-broadcast,GQA]": lambda: f(1, 2, 2, 3, 4, 6) @ np.swapaxes(f(2, 2, 2, 1, 5, 6), -1, -2),
        "Cat[axis=2]": lambda: np.concatenate([f(1, 2, 3, 4, 5), f(2, 2, 3, 6, 5)], 2),
        "Cat[axis=-1]": lambda: np.concatenate([f(3, 2, 3, 4), f(4, 2, 3, 6)], -1),
        "Cat[strided incoming]": lambda: np.concatenate([f(5, 2, 3, 4, 5), np.swapaxes(f(6, 2, 6, 3, 5), 1, 2)], 2),
        "Gather": lambda: f(1, 6, 4)[[0, 2, 5, 2]],
        "ScatterAddRows": lambda: np.stack([f(1, 4, 4)[[i for i, t in enumerate([0, 2, 5, 2]) if t == row]].sum(0)
                                            for row in range(6)]),
        "CrossEntropy": lambda: ce(f(1, 4, 5), [1, 3, 0, 2], -100),
        "CrossEntropy[ignore]": lambda: ce(f(1, 4, 5), [1, -100, 0, 2], -100),
        "CrossEntropyGrad": lambda: ce_grad(f(1, 4, 5), [1, -100, 0, 2], -100),
    }
    return np.asarray(table[name](), dtype=np.float64).reshape(-1)


def assert_matches(expected, got, name, atol=ATOL, rtol=RTOL):
    assert got.shape == expected.shape, f"'{name}': length {got.shape} != oracle {expected.shape}"
    tol = atol + rtol * np.abs(expected)
    bad = np.nonzero(np.abs(expected - got) > tol)[0]
    assert bad.size == 0, f"'{name}' index {bad[0]}: {got[bad[0]]} vs oracle {expected[bad[0]]} (tol {tol[bad[0]]})"


def test_case_count():
    assert len(CASES) == 33  # 30 conformance cases + the three Cat cases of BackendConformanceTests.cs:100-104


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_numpy(oracle, name):
    """The oracle itself against an independent float64 statement of each op (CPU)."""
    assert_matches(_numpy_reference(name), CASES[name](oracle).astype(np.float64), name, atol=2e-6, rtol=2e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_cuda_matches_oracle(oracle, cuda, name):
    expected = CASES[name](oracle)
    got = CASES[name](cuda)
    assert_matches(expected, got, name)
