"""The oracle's restatements of the layers around the attention path, pinned
on the CPU against the reference test-suite's own expected values:
test/unit/ops/elementwise.cpp, ops/reduction.cpp, nn/mlp.cpp,
nn/mlp_forward.cpp (inputs and host formulas restated with numpy), with each
test's tolerance (testHelper/test.hpp:47-54 checkValue). Operators that are
exact in the reference's arithmetic are checked bit for bit against numpy
doing the same operations in the same element type."""
import numpy as np
import pytest

import oracle

TYPES = [np.float32, np.float64]


def check(value, expected, eps=1e-5, margin=1e-6):
    value, expected = np.asarray(value, np.float64), np.asarray(expected, np.float64)
    ok = (np.abs(value - expected) <= margin) | (np.abs(value - expected) <= eps * np.abs(expected))
    assert ok.all(), (value[~ok][:5], expected[~ok][:5])


def seq(shape, T):
    """elementwise.cpp:20-29: -3, -2.5, -2, ... in row-major order."""
    n = int(np.prod(shape))
    return (T(-3) + np.arange(n) * T(0.5)).astype(T).reshape(shape)


@pytest.mark.parametrize("T", TYPES)
def test_elementwise_reference_case(T):
    """elementwise.cpp:31-130, every operator of the chain."""
    a = seq((2, 4), T)
    b = (a + T(1)).astype(T)
    out = np.empty_like(a)
    check(oracle.binary(a, b, out, "add"), a + b)
    assert np.array_equal(oracle.binary(b, a, out, "sub"), b - a)
    assert np.array_equal(oracle.binary(a, b, out, "mul"), a * b)
    with np.errstate(divide="ignore"):  # a holds a 0: b / 0 = inf on both sides
        assert np.array_equal(oracle.binary(b, a, out, "div"), b / a)
    assert np.array_equal(oracle.unary(a, out, "scale", 3.0), a * T(3))
    check(oracle.binary(a, b, out, "axpy", 2.0), T(2) * a + b)
    bias = np.arange(4).astype(T)
    check(oracle.bias_add(a, bias, out), a + bias[None, :])
    eps = 1e-5 if T == np.float32 else 1e-9
    # padded views (row pitch 8): the transcendental chain ends in swiglu(x, x)
    store = np.zeros((2, 8), T)
    store[:, :4] = a
    pin = store[:, :4]
    pout = np.zeros((2, 8), T)[:, :4]
    oracle.unary(pin, pout, "exp")
    oracle.unary(pout, pout, "sqrt")
    oracle.unary(pout, pout, "rsqrt")
    oracle.binary(pin, pin, pout, "swiglu")
    sig = T(1) / (T(1) + np.exp(-a))
    check(pout, a * sig * a, eps, eps)


@pytest.mark.parametrize("T", TYPES)
@pytest.mark.parametrize("op,fn", [("relu", lambda x: np.where(x > 0, x, 0)),
                                   ("sigmoid", lambda x: 1 / (1 + np.exp(-x))),
                                   ("silu", lambda x: x / (1 + np.exp(-x))),
                                   ("exp", np.exp), ("sqrt", lambda x: np.sqrt(np.abs(x)))])
def test_activations_against_host_formulas(T, op, fn):
    x = seq((3, 7), T)
    if op == "sqrt":
        x = np.abs(x)
    got = oracle.unary(x, np.empty_like(x), op)
    eps = 1e-5 if T == np.float32 else 1e-12
    check(got, fn(x.astype(np.float64)), eps, eps)


@pytest.mark.parametrize("T", TYPES)
def test_gelu_against_erf_formula(T):
    """mlp_forward.cpp:30-31: 0.5 x (1 + erf(x / sqrt 2))."""
    import math
    x = seq((4, 5), T)
    got = oracle.unary(x, np.empty_like(x), "gelu")
    want = np.array([0.5 * v * (1 + math.erf(v * 0.70710678118654752440)) for v in x.ravel().astype(float)])
    eps = 1e-5 if T == np.float32 else 1e-12
    check(got.ravel(), want, eps, eps)


@pytest.mark.parametrize("T", TYPES)
def test_reduction_reference_case(T):
    """reduction.cpp:33-124: [2,3,4] = 1, 2, 3, ...; sum/mean/max/sumSquares
    over the fastest axis, dot over axis 1."""
    x = (np.arange(24) + 1).astype(T).reshape(2, 3, 4)
    eps = 1e-5 if T == np.float32 else 1e-12
    out = np.empty((2, 3, 1), T)
    check(oracle.reduce(x, out, "sum", 2), x.sum(2, keepdims=True), eps, eps)
    check(oracle.reduce(x, out, "mean", 2), x.mean(2, keepdims=True), eps, eps)
    assert np.array_equal(oracle.reduce(x, out, "max", 2), x.max(2, keepdims=True))
    check(oracle.reduce(x, out, "sum_squares", 2), (x * x).sum(2, keepdims=True), eps, eps)
    d = np.empty((2, 1, 4), T)
    check(oracle.reduce(x, d, "dot", 1, rhs=x), (x * x).sum(1, keepdims=True), eps, eps)


def test_reduction_empty_axis():
    """An axis of extent 0: sum 0, max lowest(), mean 0 / 0."""
    x = np.zeros((2, 0, 3), np.float32)
    out = np.empty((2, 1, 3), np.float32)
    assert np.all(oracle.reduce(x, out, "sum", 1) == 0)
    assert np.all(oracle.reduce(x, out, "max", 1) == np.finfo(np.float32).min)
    assert np.all(np.isnan(oracle.reduce(x, out, "mean", 1)))


@pytest.mark.parametrize("T", TYPES)
def test_masked_softmax_against_formula(T):
    """onAcc/internal/nn/softmax.hpp:76-116 with a -inf mask."""
    x = seq((2, 5), T)
    mask = np.where(np.arange(5) >= 3, -np.inf, 0).astype(T)[None, :].repeat(2, 0)
    got = oracle.masked_softmax(x, mask, np.empty_like(x), 1)
    v = x.astype(np.float64) + mask
    e = np.exp(v - v.max(1, keepdims=True))
    check(got, e / e.sum(1, keepdims=True), 1e-6, 1e-7)
    assert np.all(got[:, 3:] == 0)


def fill_det(shape, scale, shift, T):
    """mlp_forward.cpp:41-50: scale * (index + 1) + shift."""
    n = int(np.prod(shape))
    return (T(scale) * (np.arange(n) + 1).astype(T) + T(shift)).astype(T).reshape(shape)


@pytest.mark.parametrize("T", TYPES)
def test_mlp_forward_reference_cases(T):
    """mlp_forward.cpp:60-182: one layer (silu) and three layers (silu hidden,
    none last), host reference loops restated."""
    silu = lambda v: v / (T(1) + np.exp(-v))  # noqa: E731
    x = fill_det((2, 3), 0.3, -0.2, T)
    w = fill_det((3, 4), 0.11, -0.4, T)
    b = fill_det((4,), 0.07, 0.01, T)
    check(oracle.mlp_forward(x, [w], [b], "silu", "silu"), silu(x @ w + b))
    dims = (3, 5, 4, 2)
    x = fill_det((2, dims[0]), 0.2, -0.3, T)
    ws = [fill_det((dims[0], dims[1]), 0.09, -0.2, T), fill_det((dims[1], dims[2]), 0.07, -0.1, T),
          fill_det((dims[2], dims[3]), 0.05, -0.05, T)]
    bs = [fill_det((dims[1],), 0.03, 0.01, T), fill_det((dims[2],), 0.02, -0.01, T),
          fill_det((dims[3],), 0.01, 0.02, T)]
    h0 = silu(x @ ws[0] + bs[0])
    h1 = silu(h0 @ ws[1] + bs[1])
    check(oracle.mlp_forward(x, ws, bs, "silu", "none"), h1 @ ws[2] + bs[2])


@pytest.mark.parametrize("T", TYPES)
def test_gated_mlp_reference_case(T):
    """nn/mlp.cpp:20-68."""
    i, j = np.meshgrid(np.arange(4), np.arange(6), indexing="ij")
    x = np.ascontiguousarray((np.arange(4) + 1).astype(T)[None, :])
    wg = (T(0.05) * (i + j + 1)).astype(T)
    wu = (T(0.04) * (i + j + 1)).astype(T)
    i2, j2 = np.meshgrid(np.arange(6), np.arange(4), indexing="ij")
    wd = (T(0.03) * (i2 + j2 + 1)).astype(T)
    a = x @ wg
    b = x @ wu
    check(oracle.gated_mlp(x, wg, wu, wd), (a / (T(1) + np.exp(-a)) * b) @ wd)
