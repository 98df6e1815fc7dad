"""The CPU oracle against alpakaNN's own kernels, executed (CPU, no GPU).

oracle/_ref compiles the reference's device kernels
(include/alpaka/nn/onAcc/internal/nn/*.hpp) unmodified against a host-only
stand-in for the alpaka API (oracle/ref_harness) and runs them on the host.
The oracle restates the same kernels loop for loop, so on the same inputs the
two must agree BIT FOR BIT: attention scores / apply (both layouts, GQA),
rmsNorm (several ranks), RoPE (both layouts, position offsets), softmax and
causalSoftmax (every axis, Tq != Tk), maskedSoftmax and embeddingLookup, in
fp32 and fp64, plus the golden cases' own inputs. Skipped only where the
reference tree is absent and no prebuilt library exists."""
import numpy as np
import pytest

import oracle
from oracle import reference
from tests.helpers import arr, load_cases, normal, rng, rope_tables

pytestmark = pytest.mark.skipif(not reference.available(), reason="reference kernels not built (no reference tree)")

TYPES = [np.float32, np.float64]


def same(a, b):
    assert a.shape == b.shape
    assert np.array_equal(a, b, equal_nan=True), float(np.nanmax(np.abs(a.astype(np.float64) - b)))


@pytest.mark.parametrize("T", TYPES)
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("g", [1, 3])
def test_scores_and_apply(T, layout, g):
    G = rng(100 + 10 * layout + g)
    B, Tq, Tk, Hkv, D = 2, 19, 23, 2, 24
    Hq = Hkv * g
    q = normal(G, (B, Tq, Hq, D), T)
    kshape = (B, Tk, Hkv, D) if layout == 0 else (B, Hkv, Tk, D)
    k, v = normal(G, kshape, T), normal(G, kshape, T)
    s_o = oracle.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), T), g, layout)
    s_r = reference.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), T), g, layout)
    same(s_o, s_r)
    p = normal(G, (B, Hq, Tq, Tk), T)
    o_o = oracle.attention_apply(p, v, np.empty((B, Tq, Hq, D), T), g, layout)
    o_r = reference.attention_apply(p, v, np.empty((B, Tq, Hq, D), T), g, layout)
    same(o_o, o_r)


@pytest.mark.parametrize("T,eps", [(np.float32, 1e-6), (np.float32, 1e-5), (np.float64, 1e-12)])
@pytest.mark.parametrize("shape", [(7, 33), (3, 5, 64), (2, 3, 4, 16), (129,)])
def test_rms_norm(T, eps, shape):
    G = rng(len(shape) * 7 + shape[-1])
    x = normal(G, shape, T)
    w = (1.0 + normal(G, (shape[-1],), np.float64, 0.02)).astype(T)
    same(oracle.rms_norm(x, w, np.empty_like(x), T(eps)), reference.rms_norm(x, w, np.empty_like(x), T(eps)))


@pytest.mark.parametrize("T", TYPES)
@pytest.mark.parametrize("layout,offset", [(0, 0), (0, 17), (1, 0), (1, 5)])
def test_rope(T, layout, offset):
    G = rng(7 + layout + offset)
    B, Tt, H, D = 2, 9, 3, 16
    shape = (B, Tt, H, D) if layout == 0 else (B, H, Tt, D)
    x = normal(G, shape, T)
    cos, sin = rope_tables(Tt + offset, D, 1e4, T)
    same(oracle.rope(x, cos, sin, np.empty_like(x), layout, offset),
         reference.rope(x, cos, sin, np.empty_like(x), layout, offset))


@pytest.mark.parametrize("T", TYPES)
def test_softmax_every_axis_and_causal(T):
    G = rng(3)
    x = normal(G, (2, 3, 5, 7), T) * 4
    for axis in range(4):
        same(oracle.softmax(x, np.empty_like(x), axis), reference.softmax(x, np.empty_like(x), axis))
    # causal: the reference's generic rule idx[queryAxis] < idx[keyAxis] (top-left), any axes
    for axis, qa, ka in [(3, 2, 3), (2, 2, 3), (3, 1, 3), (1, 2, 1)]:
        same(oracle.causal_softmax(x, np.empty_like(x), axis, qa, ka),
             reference.causal_softmax(x, np.empty_like(x), axis, qa, ka))
    m = normal(G, x.shape, T)
    same(oracle.masked_softmax(x, m, np.empty_like(x), 3), reference.masked_softmax(x, m, np.empty_like(x), 3))


@pytest.mark.parametrize("T", TYPES)
def test_embedding(T):
    G = rng(11)
    table = normal(G, (50, 12), T)
    ids = G.integers(0, 50, size=17, dtype=np.uint32)
    same(oracle.embedding_lookup(ids, table, np.empty((17, 12), T)),
         reference.embedding_lookup(ids, table, np.empty((17, 12), T)))


def test_c1_block_op_by_op():
    """The c1 block (batch 1, seq 128, d_model 256, 4 heads x 64, fp32) from
    rmsNorm to attentionApply: every op, oracle == reference kernels."""
    T = np.float32
    G = rng(0x5EED + 1)
    x = normal(G, (128, 256), T)
    w = (1.0 + normal(G, (256,), np.float64, 0.02)).astype(T)
    y = oracle.rms_norm(x, w, np.empty_like(x), T(1e-6))
    same(y, reference.rms_norm(x, w, np.empty_like(x), T(1e-6)))
    q, k, v = (normal(G, (1, 128, 4, 64), T) for _ in range(3))
    cos, sin = rope_tables(128, 64, 1e4, T)
    rq = oracle.rope(q, cos, sin, np.empty_like(q))
    rk = oracle.rope(k, cos, sin, np.empty_like(k))
    same(rq, reference.rope(q, cos, sin, np.empty_like(q)))
    s = oracle.attention_scores(rq, rk, np.empty((1, 4, 128, 128), T))
    same(s, reference.attention_scores(rq, rk, np.empty((1, 4, 128, 128), T)))
    s *= T(0.125)
    p = oracle.causal_softmax(s, np.empty_like(s), 3, 2, 3)
    same(p, reference.causal_softmax(s, np.empty_like(s), 3, 2, 3))
    same(oracle.attention_apply(p, v, np.empty_like(q)), reference.attention_apply(p, v, np.empty_like(q)))


def test_golden_case_inputs():
    """Every golden case's inputs through both: scores, apply, softmax, rope,
    rmsNorm as the case names them."""
    n = 0
    for c in load_cases():
        op = c["op"]
        if op == "scores":
            q, k = arr(c["q"]), arr(c["k"])
            shape = tuple(arr(c["expected"]).shape)
            same(oracle.attention_scores(q, k, np.empty(shape, q.dtype), c["g"], c["layout"]),
                 reference.attention_scores(q, k, np.empty(shape, q.dtype), c["g"], c["layout"]))
            n += 1
        elif op == "apply":
            p, v = arr(c["probs"]), arr(c["v"])
            shape = tuple(arr(c["expected"]).shape)
            same(oracle.attention_apply(p, v, np.empty(shape, p.dtype), c["g"], c["layout"]),
                 reference.attention_apply(p, v, np.empty(shape, p.dtype), c["g"], c["layout"]))
            n += 1
    assert n > 0
