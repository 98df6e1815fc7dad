"""Elementwise ops, activations, reductions, maskedSoftmax and the MLP layers
on the GPU (onHost/ops/elementwise.hpp, onHost/ops/reduction.hpp,
onHost/nn/softmax.hpp:42-57, onHost/nn/mlp.hpp).

Three kinds of checks: the reference's own test cases with their known
answers and tolerances (test/unit/ops/elementwise.cpp, ops/reduction.cpp,
nn/mlp.cpp, nn/mlp_forward.cpp); parity with the CPU oracle on seeded inputs
(bit-exact where the arithmetic is exact, else within the stated tolerance),
on dense, misaligned and strided views; and the edge cases (empty tensors,
extent-1 axes, -inf masks, long rows).
"""
import math

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DT = [(torch.float32, np.float32), (torch.float64, np.float64)]
# exp / erf based results: the device math functions against the host's. The
# absolute part covers gelu's 1 + erf(x) cancellation for x << 0 (an ulp of
# erf near -1 times 0.5 |x|); the reference's own activation test allows
# 1e-5 / 1e-5 (f32) and 1e-9 / 1e-9 (f64), elementwise.cpp:121.
TRANS_TOL = {np.float32: dict(rtol=1e-5, atol=1e-6), np.float64: dict(rtol=1e-13, atol=1e-15)}
# softmax rows: sums formed in another order than the reference's loop
SOFTMAX_TOL = {np.float32: dict(rtol=1e-5, atol=1e-7), np.float64: dict(rtol=1e-11, atol=1e-300)}


@pytest.fixture(scope="module")
def ann():
    from tests.helpers import build_library
    build_library()
    import alpakann_b200 as a
    return a


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def check(value, expected, eps=1e-5, margin=1e-6):
    """checkValue (testHelper/test.hpp:47-54): Approx(expected).epsilon(eps).margin(margin)."""
    value, expected = np.asarray(value, np.float64), np.asarray(expected, np.float64)
    ok = (np.abs(value - expected) <= margin) | (np.abs(value - expected) <= eps * np.abs(expected))
    assert ok.all(), (value[~ok][:5], expected[~ok][:5])


def fill_sequence(shape, np_t):
    """elementwise.cpp:20-29: -3, -2.5, -2, ..."""
    n = int(np.prod(shape))
    return (np_t(-3) + np.arange(n) * np_t(0.5)).astype(np_t).reshape(shape)


# ---- reference test cases --------------------------------------------------------
@pytest.mark.parametrize("dtype,np_t", DT)
def test_reference_elementwise_case(ann, dtype, np_t):
    """elementwise.cpp:31-130."""
    ops = ann.onHost.ops
    q = None
    a = fill_sequence((2, 4), np_t)
    b = a + np_t(1)
    dA, dB = dev(a), dev(b)
    out = torch.empty_like(dA)
    ops.fill(q, None, out, 2.0)
    assert np.all(host(out) == 2)
    ops.copy(q, None, dA, out)
    assert np.array_equal(host(out), a)
    ops.add(q, None, dA, dB, out)
    check(host(out), a + b)
    ops.sub(q, None, dB, dA, out)
    ops.mul(q, None, dA, dB, out)
    ops.div(q, None, dB, dA, out)
    ops.scale(q, None, dA, 3.0, out)
    ops.axpy(q, None, 2.0, dA, dB, out)
    check(host(out), np_t(2) * a + b)
    bias = np.arange(4).astype(np_t)
    ops.biasAdd(q, None, dA, dev(bias), out)
    check(host(out), a + bias[None, :])
    ints = torch.empty((2, 4), dtype=torch.int32, device="cuda")
    ops.cast(q, None, dA, ints)
    assert np.array_equal(host(ints), a.astype(np.int32))
    # padded views, row pitch 8 (elementwise.cpp:95-129)
    store = torch.zeros(24, dtype=dtype, device="cuda")
    store_out = torch.zeros(24, dtype=dtype, device="cuda")
    pin = store.as_strided((2, 4), (8, 1))
    pout = store_out.as_strided((2, 4), (8, 1))
    pin.copy_(dev(a))
    ops.exp(q, None, pin, pout)
    ops.sqrt(q, None, pout, pout)
    ops.rsqrt(q, None, pout, pout)
    ops.relu(q, None, pin, pout)
    ops.sigmoid(q, None, pin, pout)
    ops.silu(q, None, pin, pout)
    ops.gelu(q, None, pin, pout)
    ops.swiglu(q, None, pin, pin, pout)
    eps = 1e-5 if np_t == np.float32 else 1e-9
    sig = np_t(1) / (np_t(1) + np.exp(-a))
    check(host(pout), a * sig * a, eps, eps)
    assert np.all(host(store_out).reshape(3, 8)[:2, 4:] == 0)  # padding untouched


@pytest.mark.parametrize("dtype,np_t", DT)
def test_reference_reduction_case(ann, dtype, np_t):
    """reduction.cpp:33-124: [2,3,4] = 1, 2, 3, ...; sum/mean/max/sumSquares
    over axis 2, dot over axis 1 of padded views."""
    ops = ann.onHost.ops
    x = (np.arange(24) + 1).astype(np_t).reshape(2, 3, 4)
    eps = 1e-5 if np_t == np.float32 else 1e-12
    out = torch.empty((2, 3, 1), dtype=dtype, device="cuda")
    d = dev(x)
    ops.reduceSum(None, None, d, out, 2)
    check(host(out), x.sum(2, keepdims=True), eps, eps)
    ops.reduceMean(None, None, d, out, 2)
    check(host(out), x.mean(2, keepdims=True), eps, eps)
    ops.reduceMax(None, None, d, out, 2)
    assert np.array_equal(host(out), x.max(2, keepdims=True))
    ops.reduceSumSquares(None, None, d, out, 2)
    check(host(out), (x * x).sum(2, keepdims=True), eps, eps)
    store = torch.zeros(48, dtype=dtype, device="cuda")
    lhs = store.as_strided((2, 3, 4), (24, 8, 1))
    lhs.copy_(d)
    rhs = torch.zeros(48, dtype=dtype, device="cuda").as_strided((2, 3, 4), (24, 8, 1))
    rhs.copy_(d)
    dot = torch.empty((2, 1, 4), dtype=dtype, device="cuda")
    ops.dot(None, None, lhs, rhs, dot, 1)
    check(host(dot), (x * x).sum(1, keepdims=True), eps, eps)
    assert ops.makeReducedExtents((2, 3, 4), 1) == (2, 1, 4)


@pytest.mark.parametrize("dtype,np_t", DT)
def test_reference_mlp_case(ann, dtype, np_t):
    """nn/mlp.cpp:20-68: the gated MLP on [1,4] x [4,6] -> [6,4]."""
    i, j = np.meshgrid(np.arange(4), np.arange(6), indexing="ij")
    x = (np.arange(4) + 1).astype(np_t)[None, :]
    wg = (np_t(0.05) * (i + j + 1)).astype(np_t)
    wu = (np_t(0.04) * (i + j + 1)).astype(np_t)
    i2, j2 = np.meshgrid(np.arange(6), np.arange(4), indexing="ij")
    wd = (np_t(0.03) * (i2 + j2 + 1)).astype(np_t)
    out = torch.empty((1, 4), dtype=dtype, device="cuda")
    ann.onHost.nn.mlp(None, None, dev(x), dev(wg), dev(wu), dev(wd), out)
    a = x @ wg
    b = x @ wu
    hidden = a / (np_t(1) + np.exp(-a)) * b
    check(host(out), hidden @ wd)


def fill_det(shape, scale, shift, np_t):
    """mlp_forward.cpp:41-50: scale * (index + 1) + shift."""
    n = int(np.prod(shape))
    return (np_t(scale) * (np.arange(n) + 1).astype(np_t) + np_t(shift)).astype(np_t).reshape(shape)


@pytest.mark.parametrize("dtype,np_t", DT)
def test_reference_mlp_forward_cases(ann, dtype, np_t):
    """mlp_forward.cpp:60-108 (one layer, silu) and :112-182 (three layers,
    silu hidden, none last), plus decodeLatent (:184-216)."""
    nn = ann.onHost.nn
    silu = lambda v: v / (np_t(1) + np.exp(-v))  # noqa: E731
    x = fill_det((2, 3), 0.3, -0.2, np_t)
    w = fill_det((3, 4), 0.11, -0.4, np_t)
    b = fill_det((4,), 0.07, 0.01, np_t)
    out = torch.empty((2, 4), dtype=dtype, device="cuda")
    nn.mlpForward(None, None, dev(x), [nn.WeightView(dev(w))], [nn.BiasView(dev(b))], nn.Activation.silu, out)
    check(host(out), silu(x @ w + b))

    dims = (3, 5, 4, 2)
    x = fill_det((2, dims[0]), 0.2, -0.3, np_t)
    ws = [fill_det((dims[0], dims[1]), 0.09, -0.2, np_t), fill_det((dims[1], dims[2]), 0.07, -0.1, np_t),
          fill_det((dims[2], dims[3]), 0.05, -0.05, np_t)]
    bs = [fill_det((dims[1],), 0.03, 0.01, np_t), fill_det((dims[2],), 0.02, -0.01, np_t),
          fill_det((dims[3],), 0.01, 0.02, np_t)]
    out = torch.empty((2, dims[3]), dtype=dtype, device="cuda")
    nn.mlpForward(None, None, dev(x), [dev(v) for v in ws], [dev(v) for v in bs], nn.Activation.silu,
                  nn.Activation.none, out)
    h0 = silu(x @ ws[0] + bs[0])
    h1 = silu(h0 @ ws[1] + bs[1])
    check(host(out), h1 @ ws[2] + bs[2])

    lat = fill_det((1, 3), 0.4, -0.6, np_t)
    w = fill_det((3, 5), 0.08, -0.3, np_t)
    out = torch.empty((1, 5), dtype=dtype, device="cuda")
    nn.decodeLatent(None, None, dev(lat), dev(w), out)
    check(host(out), lat @ w)


# ---- parity with the oracle --------------------------------------------------------
def views(t, kind):
    """dense, misaligned by one element (scalar path), transposed, sliced."""
    if kind == "dense":
        return t
    if kind == "offset":
        flat = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        v = flat[1:].view(t.shape)
        v.copy_(t)
        return v
    if kind == "transposed":
        return t.t().contiguous().t()
    big = torch.empty((t.shape[0], t.shape[1] + 7), dtype=t.dtype, device=t.device)
    v = big[:, 3:3 + t.shape[1]]
    v.copy_(t)
    return v


EXACT_UNARY = ["copy", "scale", "sqrt", "relu"]
TRANS_UNARY = ["exp", "rsqrt", "sigmoid", "silu", "gelu"]


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("kind", ["dense", "offset", "transposed", "sliced"])
def test_unary_parity(ann, dtype, np_t, kind):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((37, 1001)) * 3).astype(np_t)
    xs = np.abs(x) + np_t(0.01)
    for op in EXACT_UNARY + TRANS_UNARY:
        src = xs if op in ("sqrt", "rsqrt") else x
        want = oracle.unary(src, np.empty_like(src), op, 1.7)
        t_in = views(dev(src), kind)
        t_out = views(torch.zeros_like(dev(src)), kind)
        ann.onHost.ops.unaryOp(None, None, t_in, t_out, ann.onHost.ops.__dict__[op.upper()], 1.7)
        got = host(t_out)
        if op in EXACT_UNARY:
            assert np.array_equal(got, want), op
        else:
            np.testing.assert_allclose(got, want, **TRANS_TOL[np_t], err_msg=op)


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("kind", ["dense", "offset", "sliced"])
def test_binary_parity(ann, dtype, np_t, kind):
    rng = np.random.default_rng(2)
    l = (rng.standard_normal((129, 515)) * 2).astype(np_t)
    r = (rng.standard_normal((129, 515)) * 2 + 0.1).astype(np_t)
    for op in ["add", "sub", "mul", "div", "axpy", "swiglu"]:
        want = oracle.binary(l, r, np.empty_like(l), op, -0.75)
        out = views(torch.zeros_like(dev(l)), kind)
        ann.onHost.ops.binaryOp(None, None, views(dev(l), kind), views(dev(r), kind), out,
                                ann.onHost.ops.__dict__[op.upper()], -0.75)
        got = host(out)
        if op == "swiglu":
            np.testing.assert_allclose(got, want, **TRANS_TOL[np_t])
        else:
            assert np.array_equal(got, want), op


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("H", [512, 515])
@pytest.mark.parametrize("act", ["none", "relu", "silu", "gelu"])
def test_bias_activation_parity(ann, dtype, np_t, H, act):
    """One fused pass equals biasAdd then the activation in place."""
    from alpakann_b200 import _capi
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 33, H)).astype(np_t)
    b = rng.standard_normal(H).astype(np_t)
    want = oracle.bias_add(x, b, np.empty_like(x), act)
    dx, db = dev(x), dev(b)  # held: a view descriptor does not keep its tensor alive
    out = torch.empty_like(dx)
    code = ["none", "relu", "silu", "gelu"].index(act)
    _capi.check(getattr(_capi.lib, f"ann_bias_add_{'f32' if np_t == np.float32 else 'f64'}")(
        None, _capi.ref(dx), _capi.ref(db), code, _capi.ref(out)))
    got = host(out)
    if act in ("none", "relu"):
        assert np.array_equal(got, want)
    else:
        np.testing.assert_allclose(got, want, **TRANS_TOL[np_t])
    # strided input, bias with a stride
    xt = views(dev(x.reshape(99, H)), "sliced")
    bb = torch.zeros(2 * H, dtype=dtype, device="cuda")
    bb[::2] = dev(b)
    out2 = torch.empty((99, H), dtype=dtype, device="cuda")
    _capi.check(getattr(_capi.lib, f"ann_bias_add_{'f32' if np_t == np.float32 else 'f64'}")(
        None, _capi.ref(xt), _capi.ref(bb[::2]), code, _capi.ref(out2)))
    got2 = host(out2)
    if act in ("none", "relu"):
        assert np.array_equal(got2, want.reshape(99, H))
    else:
        np.testing.assert_allclose(got2, want.reshape(99, H), **TRANS_TOL[np_t])


@pytest.mark.parametrize("src,dst", [(torch.float32, torch.int32), (torch.float64, torch.float32),
                                     (torch.int32, torch.float64), (torch.uint32, torch.float32),
                                     (torch.int64, torch.float64), (torch.float32, torch.int64)])
def test_cast(ann, src, dst):
    rng = np.random.default_rng(4)
    a = (rng.standard_normal(1000) * 1000)
    if src in (torch.int32, torch.int64):
        t = torch.from_numpy(a.astype(np.int64)).to(src).cuda()
    elif src == torch.uint32:
        t = torch.from_numpy(np.abs(a).astype(np.uint32)).cuda()
    else:
        t = torch.from_numpy(a).to(src).cuda()
    out = torch.empty(1000, dtype=dst, device="cuda")
    ann.onHost.ops.cast(None, None, t, out)
    src_np = t.cpu().numpy()
    want = src_np.astype({torch.int32: np.int32, torch.int64: np.int64, torch.float32: np.float32,
                          torch.float64: np.float64}[dst])
    assert np.array_equal(host(out), want)


@pytest.mark.parametrize("dtype,value", [(torch.float32, -1.5), (torch.float64, 2.0 ** -40), (torch.int32, -7),
                                         (torch.uint32, 4000000000), (torch.int64, -(2 ** 40))])
def test_fill(ann, dtype, value):
    t = torch.zeros((17, 9), dtype=dtype, device="cuda")[:, 1:8]
    ann.onHost.ops.fill(None, None, t, value)
    got = host(t)
    assert np.all(got == np.array(value, dtype=got.dtype))
    full = host(t.as_strided((17, 9), (9, 1), t.storage_offset() - 1))
    assert np.all(full[:, 0] == 0) and np.all(full[:, 8] == 0)  # columns outside the view untouched


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("shape,axis", [((7, 33, 4099), 2), ((7, 33, 300), 2), ((7, 33, 5), 2), ((7, 33, 301), 1),
                                        ((4099, 3, 2), 0), ((1, 1, 1), 0), ((5, 0, 3), 1),
                                        ((3001, 4, 64), 0), ((1, 777, 128), 1), ((20000, 192), 0)])
def test_reduction_parity(ann, dtype, np_t, shape, axis):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(shape).astype(np_t)
    rshape = list(shape)
    rshape[axis] = 1
    eps = np.finfo(np_t).eps
    for op in ["sum", "max", "mean", "sum_squares", "dot"]:
        want = np.empty(rshape, np_t)
        y = rng.standard_normal(shape).astype(np_t)
        # Both sums carry rounding error up to about n * eps * sum |term|
        # (another order than the oracle's loop): bound the difference by
        # 4 eps sqrt(n) sum |term|, the statistical size of that error.
        terms = {"sum": x, "mean": x, "max": x, "sum_squares": x * x, "dot": x * y}[op].astype(np.float64)
        mag = np.abs(terms).sum(axis=axis, keepdims=True) / (max(shape[axis], 1) if op == "mean" else 1)
        bound = 4 * eps * math.sqrt(max(shape[axis], 1)) * mag + np.finfo(np_t).tiny
        oracle.reduce(x, want, op, axis, rhs=y if op == "dot" else None)
        out = torch.full(rshape, 123.0, dtype=dtype, device="cuda")
        o = ann.onHost.ops
        if op == "dot":
            o.dot(None, None, dev(x), dev(y), out, axis)
        else:
            o._reduce(None, {"sum": o.SUM, "max": o.MAX, "mean": o.MEAN, "sum_squares": o.SUM_SQUARES}[op],
                      dev(x), out, axis)
        got = host(out)
        if op == "max" or shape[axis] == 0:
            assert np.array_equal(got, want, equal_nan=True), op
        else:
            assert (np.abs(got.astype(np.float64) - want) <= bound).all(), op


@pytest.mark.parametrize("dtype,np_t", DT)
def test_column_reduction_padded_rows(ann, dtype, np_t):
    """Columns [:, :128] of a [600, 192] tensor reduced over axis 0 (row
    pitch 192, 16-byte aligned): the split-axis column path with a pitch
    wider than the run, for sum, max and dot."""
    rng = np.random.default_rng(12)
    big = rng.standard_normal((600, 192)).astype(np_t)
    other = rng.standard_normal((600, 192)).astype(np_t)
    x, y = big[:, :128], other[:, :128]
    dx, dy = dev(big)[:, :128], dev(other)[:, :128]
    o = ann.onHost.ops
    eps = np.finfo(np_t).eps
    for op in ["sum", "max", "dot"]:
        want = np.empty((1, 128), np_t)
        oracle.reduce(np.ascontiguousarray(x), want, op, 0, rhs=np.ascontiguousarray(y) if op == "dot" else None)
        out = torch.full((1, 128), 123.0, dtype=dtype, device="cuda")
        if op == "dot":
            o.dot(None, None, dx, dy, out, 0)
        elif op == "sum":
            o.reduceSum(None, None, dx, out, 0)
        else:
            o.reduceMax(None, None, dx, out, 0)
        got = host(out)
        if op == "max":
            assert np.array_equal(got, want), op
        else:
            terms = (x * y if op == "dot" else x).astype(np.float64)
            bound = 4 * eps * math.sqrt(600) * np.abs(terms).sum(0, keepdims=True)
            assert (np.abs(got.astype(np.float64) - want) <= bound).all(), op


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("shape,axis", [((2, 3, 17, 40), 3), ((2, 3, 5, 3000), 3), ((2, 40, 3, 5), 1)])
def test_masked_softmax_parity(ann, dtype, np_t, shape, axis):
    rng = np.random.default_rng(6)
    x = (rng.standard_normal(shape) * 4).astype(np_t)
    mask = np.where(rng.random(shape) < 0.3, -np.inf, rng.standard_normal(shape)).astype(np_t)
    # keep one finite entry per row
    idx = [slice(None)] * len(shape)
    idx[axis] = 0
    mask[tuple(idx)] = 0
    want = oracle.masked_softmax(x, mask, np.empty_like(x), axis)
    out = torch.empty_like(dev(x))
    ann.onHost.nn.maskedSoftmax(None, None, dev(x), dev(mask), out, axis)
    np.testing.assert_allclose(host(out), want, **SOFTMAX_TOL[np_t])


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("shape,axis,causal", [((1, 2, 9, 4096), 3, False), ((1, 2, 9, 4096), 3, True),
                                               ((1, 2, 3, 2051), 3, False), ((1, 2, 3, 2051), 3, True),
                                               ((1, 1, 2, 8192), 3, True), ((1, 1, 3000, 4), 2, False),
                                               ((1, 1, 3000, 4), 2, True), ((1, 2, 3, 9000), 3, True),
                                               ((1, 1, 3, 20000), 3, False), ((1, 1, 9001, 2), 2, True),
                                               ((1, 1, 2, 30001), 3, True)])
def test_long_softmax_rows(ann, dtype, np_t, shape, axis, causal):
    """Rows longer than 2048: in a CTA's registers up to 8192 elements, in
    shared memory up to 96 KB a row (36 KB, 72 KB and 80 KB rows here, past
    the 48 KB default), streamed beyond that; vectorised when the row is
    unit-stride and a multiple of 16 bytes, element-wise otherwise (2051,
    9001, 30001 and the axis-2 rows). Causal masks with the query axis before
    the key axis (queries 2, keys 3) and, for the axis-2 rows, the softmax
    axis as the query axis.

    The reference sums a row's exponentials one after another, so its own
    rounding error grows like sqrt(len) eps and scales the whole row by one
    factor; the relative tolerance grows with the row the same way (4 eps
    sqrt(len), at least the short-row tolerance), and in fp32 the GPU result
    must be no further from the softmax evaluated in fp64 than the oracle's."""
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(shape) * 6).astype(np_t)
    out = torch.empty_like(dev(x))

    def run_oracle(v):
        if causal:
            return oracle.causal_softmax(v, np.empty_like(v), axis, 2, 3)
        return oracle.softmax(v, np.empty_like(v), axis)

    want = run_oracle(x)
    if causal:
        ann.onHost.nn.causalSoftmax(None, None, dev(x), out, axis, 2, 3)
    else:
        ann.onHost.nn.softmax(None, None, dev(x), out, axis)
    got = host(out)
    tol = dict(SOFTMAX_TOL[np_t])
    tol["rtol"] = max(tol["rtol"], 4 * float(np.finfo(np_t).eps) * math.sqrt(shape[axis]))
    np.testing.assert_allclose(got, want, **tol)
    if np_t == np.float32:
        exact = run_oracle(x.astype(np.float64))
        assert np.abs(got - exact).max() <= np.abs(want - exact).max() * 1.5 + 1e-12


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("shape,kind", [((30001, 64), "softmax"), ((30001, 64), "masked"),
                                        ((1, 8, 1023, 1024), "causal"), ((3, 1, 700, 2048), "masked"),
                                        ((2, 1, 999, 4096), "causal"), ((400, 16384), "softmax"),
                                        ((300, 12000), "masked"), ((2, 1, 200, 16384), "causal")])
def test_softmax_many_rows(ann, dtype, np_t, shape, kind):
    """Many more rows than one pass of resident CTAs takes, so each CTA's ring
    of bulk copies wraps around several times, and a row count that leaves
    the last pass partly (or, for some CTAs, wholly) empty. Rows of 12000 and
    16384 take the whole-row bulk copies, two row stages in fp32 and one in
    fp64 (128 KiB rows), several rows a CTA. Relative tolerance scaled with
    the row as in test_long_softmax_rows."""
    tol = dict(SOFTMAX_TOL[np_t])
    tol["rtol"] = max(tol["rtol"], 4 * float(np.finfo(np_t).eps) * math.sqrt(shape[-1]))
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(shape) * 5).astype(np_t)
    out = torch.empty_like(dev(x))
    axis = len(shape) - 1
    if kind == "causal":
        want = oracle.causal_softmax(x, np.empty_like(x), axis, axis - 1, axis)
        ann.onHost.nn.causalSoftmax(None, None, dev(x), out, axis, axis - 1, axis)
    elif kind == "masked":
        mask = np.where(rng.random(shape) < 0.2, -np.inf, rng.standard_normal(shape)).astype(np_t)
        mask[..., 0] = 0
        want = oracle.masked_softmax(x, mask, np.empty_like(x), axis)
        ann.onHost.nn.maskedSoftmax(None, None, dev(x), dev(mask), out, axis)
    else:
        want = oracle.softmax(x, np.empty_like(x), axis)
        ann.onHost.nn.softmax(None, None, dev(x), out, axis)
    np.testing.assert_allclose(host(out), want, **tol)
    assert ann.take_device_error(torch.cuda.current_stream().cuda_stream) == 0  # no wait gave up


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("L", [256, 1024, 4096])
def test_softmax_rows_not_equally_spaced(ann, dtype, np_t, L):
    """Aligned rows whose starts are not equally spaced (the two outer axes
    of a [3, 5, 7, L] tensor swapped in the view): every row's offset is
    decoded from its index in the bulk-copy issuer and in the kernel; plain,
    causal and masked. Relative tolerance scaled with the row as in
    test_long_softmax_rows (the reference's sequential sum)."""
    tol = dict(SOFTMAX_TOL[np_t])
    tol["rtol"] = max(tol["rtol"], 4 * float(np.finfo(np_t).eps) * math.sqrt(L))
    rng = np.random.default_rng(13)
    base = (rng.standard_normal((3, 5, 7, L)) * 4).astype(np_t)
    x = base.transpose(1, 0, 2, 3)  # [5, 3, 7, L], outer strides not nested
    dx = dev(base).permute(1, 0, 2, 3)
    nn = ann.onHost.nn
    out = torch.empty(x.shape, dtype=dtype, device="cuda")
    nn.softmax(None, None, dx, out, 3)
    np.testing.assert_allclose(host(out), oracle.softmax(np.ascontiguousarray(x), np.empty(x.shape, np_t), 3),
                               **tol)
    nn.causalSoftmax(None, None, dx, out, 3, 2, 3)
    np.testing.assert_allclose(host(out), oracle.causal_softmax(np.ascontiguousarray(x), np.empty(x.shape, np_t), 3, 2,
                                                                3), **tol)
    mbase = np.where(rng.random((3, 5, 7, L)) < 0.25, -np.inf, rng.standard_normal((3, 5, 7, L))).astype(np_t)
    mbase[..., 0] = 0
    m = mbase.transpose(1, 0, 2, 3)
    nn.maskedSoftmax(None, None, dx, dev(mbase).permute(1, 0, 2, 3), out, 3)
    np.testing.assert_allclose(host(out), oracle.masked_softmax(np.ascontiguousarray(x), np.ascontiguousarray(m),
                                                                np.empty(x.shape, np_t), 3), **tol)
    assert ann.take_device_error(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("T", [64, 1024, 4096, 2051, 9000])
def test_causal_softmax_minus_inf_rows_match_reference(ann, dtype, np_t, T):
    """causalSoftmax on rows whose kept entries are all -inf (sum of exps 0):
    the reference gives 0/0 = NaN on kept entries and writes 0 on masked
    ones; a second row group mixes finite and -inf kept entries."""
    x = np.full((1, 2, 5, T), -np.inf, np_t)
    x[0, 1, :, ::3] = np.arange(len(range(0, T, 3)), dtype=np_t)[None, :] / np_t(7)
    want = oracle.causal_softmax(x, np.empty_like(x), 3, 2, 3)
    out = torch.empty_like(dev(x))
    ann.onHost.nn.causalSoftmax(None, None, dev(x), out, 3, 2, 3)
    got = host(out)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = ~np.isnan(want)
    np.testing.assert_allclose(got[fin], want[fin], **SOFTMAX_TOL[np_t])


def test_masked_softmax_all_masked_row_matches_reference(ann):
    """A row that is all -inf: max stays lowest(), every exp is 0, 0/0 = NaN
    (onAcc/internal/nn/softmax.hpp:90-113)."""
    x = np.zeros((1, 8), np.float32)
    mask = np.full((1, 8), -np.inf, np.float32)
    want = oracle.masked_softmax(x, mask, np.empty_like(x), 1)
    out = torch.empty((1, 8), device="cuda")
    ann.onHost.nn.maskedSoftmax(None, None, dev(x), dev(mask), out, 1)
    assert np.array_equal(np.isnan(host(out)), np.isnan(want)) and np.isnan(want).all()


@pytest.mark.parametrize("dtype,np_t", DT)
@pytest.mark.parametrize("layers", [1, 2, 3, 4])
def test_mlp_forward_parity(ann, dtype, np_t, layers):
    rng = np.random.default_rng(7 + layers)
    dims = [96, 256, 192, 128, 40][:layers + 1]
    x = rng.standard_normal((33, dims[0])).astype(np_t)
    ws = [(rng.standard_normal((dims[i], dims[i + 1])) / math.sqrt(dims[i])).astype(np_t) for i in range(layers)]
    bs = [rng.standard_normal(dims[i + 1]).astype(np_t) * np_t(0.1) for i in range(layers)]
    want = oracle.mlp_forward(x, ws, bs, "gelu", "silu")
    nn = ann.onHost.nn
    out = torch.empty((33, dims[-1]), dtype=dtype, device="cuda")
    dws, dbs = [dev(w) for w in ws], [dev(b) for b in bs]
    nn.mlpForward(None, None, dev(x), dws, dbs, nn.Activation.gelu, nn.Activation.silu, out)
    tol = dict(rtol=1e-4, atol=1e-5) if np_t == np.float32 else dict(rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(host(out), want, **tol)
    # caller workspace: same kernels, same result bit for bit
    need = nn.mlpForwardWorkspaceBytes(dev(x), dws, dbs, out)
    assert need == (min(layers - 1, 2) * 33 * max(dims[1:-1], default=0) * x.itemsize)
    ws_buf = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    out2 = torch.empty_like(out)
    nn.mlpForward(None, None, dev(x), dws, dbs, nn.Activation.gelu, nn.Activation.silu, out2, workspace=ws_buf)
    assert torch.equal(out, out2)


def test_mlp_forward_rejects(ann):
    from alpakann_b200._capi import AnnShapeError
    nn = ann.onHost.nn
    x = torch.zeros((4, 8), device="cuda")
    w0, w1 = torch.zeros((8, 16), device="cuda"), torch.zeros((15, 4), device="cuda")
    b0, b1 = torch.zeros(16, device="cuda"), torch.zeros(4, device="cuda")
    out = torch.zeros((4, 4), device="cuda")
    with pytest.raises(AnnShapeError, match="layer 1 weight expects in=15 but previous out=16"):
        nn.mlpForward(None, None, x, [w0, w1], [b0, b1], nn.Activation.relu, out)
    with pytest.raises(AnnShapeError, match="bias extent does not match"):
        nn.mlpForward(None, None, x, [w0], [b1], nn.Activation.relu, torch.zeros((4, 16), device="cuda"))
    with pytest.raises(AnnShapeError, match="output extent does not match batch x last-out"):
        nn.mlpForward(None, None, x, [w0], [b0], nn.Activation.relu, out)
    with pytest.raises(AnnShapeError, match="at least one layer"):
        nn.mlpForward(None, None, x, [], [], nn.Activation.relu, out)
    w1ok = torch.zeros((16, 4), device="cuda")
    small = torch.empty(8, dtype=torch.uint8, device="cuda")
    with pytest.raises(AnnShapeError, match="workspace"):
        nn.mlpForward(None, None, x, [w0, w1ok], [b0, b1], nn.Activation.relu, out, workspace=small)


@pytest.mark.parametrize("dtype,np_t", DT)
def test_gated_mlp_parity(ann, dtype, np_t):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((65, 128)).astype(np_t)
    wg = (rng.standard_normal((128, 344)) / math.sqrt(128)).astype(np_t)
    wu = (rng.standard_normal((128, 344)) / math.sqrt(128)).astype(np_t)
    wd = (rng.standard_normal((344, 96)) / math.sqrt(344)).astype(np_t)
    want = oracle.gated_mlp(x, wg, wu, wd)
    out = torch.empty((65, 96), dtype=dtype, device="cuda")
    ann.onHost.nn.mlp(None, None, dev(x), dev(wg), dev(wu), dev(wd), out)
    tol = dict(rtol=1e-4, atol=1e-5) if np_t == np.float32 else dict(rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(host(out), want, **tol)
    ws = torch.empty(2 * 65 * 344 * x.itemsize, dtype=torch.uint8, device="cuda")
    out2 = torch.empty_like(out)
    ann.onHost.nn.mlp(None, None, dev(x), dev(wg), dev(wu), dev(wd), out2, workspace=ws)
    assert torch.equal(out, out2)


def test_linear_bias_activation(ann):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((40, 64)).astype(np.float64)
    w = rng.standard_normal((64, 72)).astype(np.float64)
    b = rng.standard_normal(72).astype(np.float64)
    out = torch.empty((40, 72), dtype=torch.float64, device="cuda")
    nn = ann.onHost.nn
    nn.linearBias(None, None, dev(x), dev(w), dev(b), out)
    np.testing.assert_allclose(host(out), oracle.bias_add(oracle.gemm(x, w, np.empty((40, 72))), b,
                                                          np.empty((40, 72))), rtol=1e-12, atol=1e-12)
    nn.linearBias(None, None, dev(x), dev(w), dev(b), out, nn.Activation.relu)
    assert (host(out) >= 0).all()


def test_empty_and_mismatch(ann):
    from alpakann_b200._capi import AnnShapeError
    ops = ann.onHost.ops
    e = torch.empty((0, 5), device="cuda")
    ops.relu(None, None, e, e)
    ops.add(None, None, e, e, e)
    with pytest.raises(AnnShapeError, match="binaryOp shape mismatch"):
        ops.add(None, None, torch.zeros(3, device="cuda"), torch.zeros(4, device="cuda"), torch.zeros(3, device="cuda"))
    with pytest.raises(AnnShapeError, match="copy shape mismatch"):
        ops.copy(None, None, torch.zeros(3, device="cuda"), torch.zeros(4, device="cuda"))
    with pytest.raises(AnnShapeError, match="biasAdd expects a 1D bias view"):
        ops.biasAdd(None, None, torch.zeros((2, 3), device="cuda"), torch.zeros((1, 3), device="cuda"),
                    torch.zeros((2, 3), device="cuda"))
    with pytest.raises(AnnShapeError, match="reduceSum output extents mismatch"):
        ops.reduceSum(None, None, torch.zeros((2, 3), device="cuda"), torch.zeros((2, 3), device="cuda"), 1)
    with pytest.raises(AnnShapeError, match="reduceMax axis out of range"):
        ops.reduceMax(None, None, torch.zeros((2, 3), device="cuda"), torch.zeros((2, 1), device="cuda"), 2)
    with pytest.raises(AnnShapeError, match="maskedSoftmax shape mismatch"):
        ann.onHost.nn.maskedSoftmax(None, None, torch.zeros((2, 3), device="cuda"), torch.zeros((2, 4), device="cuda"),
                                    torch.zeros((2, 3), device="cuda"), 1)
