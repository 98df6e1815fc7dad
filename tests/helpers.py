"""Shared test helpers: golden fixtures, the reference's tolerance rule,
seeded inputs of the benchmark configurations."""
import json
import math
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_cases.json")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_library() -> str:
    """Builds (if stale) the CUDA library by loading alpakann_b200/build.py by
    path: importing the package would load the library before it is rebuilt."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ann_build", os.path.join(ROOT, "alpakann_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build()


def load_cases():
    with open(GOLDEN) as f:
        return json.load(f)["cases"]


def arr(d):
    return np.array(d["data"], dtype=d["dtype"]).reshape(d["shape"])


def approx_ok(actual, expected, eps, margin):
    """Catch::Approx(expected).epsilon(eps).margin(margin) == actual, element-wise
    (testHelper/test.hpp:47-54): |a-b| <= margin or |a-b| <= eps*|expected|."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    diff = np.abs(actual - expected)
    return (diff <= margin) | (diff <= eps * np.abs(expected))


def assert_approx(actual, expected, eps, margin, what=""):
    ok = approx_ok(actual, expected, eps, margin)
    if not ok.all():
        bad = np.argwhere(~ok)[:5]
        a = np.asarray(actual); e = np.asarray(expected)
        detail = ", ".join(f"{tuple(i)}: {a[tuple(i)]!r} vs {e[tuple(i)]!r}" for i in bad)
        raise AssertionError(f"{what}: {int((~ok).sum())} of {ok.size} elements outside tolerance: {detail}")


# Tolerance of the attention path against the oracle (fp32: 1e-4 relative,
# fp64: 1e-11 relative, the parity targets of this path), written as
# |a-b| <= rtol*|b| + atol with an absolute floor for values near zero.
TOL = {np.float32: (1e-4, 1e-5), np.float64: (1e-11, 1e-12)}


def tol_for(dtype):
    return TOL[np.dtype(dtype).type]


def assert_close(actual, expected, dtype, what=""):
    rtol, atol = tol_for(dtype)
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    err = np.abs(actual - expected)
    bound = rtol * np.abs(expected) + atol
    if not (err <= bound).all():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: max violation at {i}: {actual[i]!r} vs {expected[i]!r} "
                             f"(rtol {rtol}, atol {atol}, {int((err > bound).sum())} bad of {err.size})")


def assert_dot_close(actual, expected, absdot, K, dtype, what=""):
    """assert_close for contractions (sums of K products): on top of the
    tolerance, each output may differ by the dot-product rounding bound
    4 eps sqrt(K) sum|a b| (sum|a b| from the oracle on |a| and |b|), since sums
    that cancel to near 0 round differently in any two summation orders (the
    tensor-core kernels add in a different order from the reference's
    sequential loop)."""
    rtol, atol = tol_for(dtype)
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    err = np.abs(actual - expected)
    bound = rtol * np.abs(expected) + atol + 4 * np.finfo(dtype).eps * np.sqrt(K) * np.asarray(absdot, np.float64)
    if not (err <= bound).all():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: max violation at {i}: {actual[i]!r} vs {expected[i]!r} "
                             f"({int((err > bound).sum())} bad of {err.size})")


def rng(seed):
    return np.random.default_rng(seed)


def normal(g, shape, dtype, std=1.0):
    # N(0, std) drawn in float64, then cast, so every dtype sees the same draw.
    return (g.standard_normal(shape) * std).astype(dtype)


def rope_tables(positions, head_dim, theta, dtype):
    """cos/sin[position][pair] with angle = pos * theta^(-2*pair/D), built in fp64."""
    pos = np.arange(positions, dtype=np.float64)[:, None]
    pair = np.arange(head_dim // 2, dtype=np.float64)[None, :]
    ang = pos * np.power(theta, -2.0 * pair / head_dim)
    return np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)


def inv_sqrt(d):
    return 1.0 / math.sqrt(d)
