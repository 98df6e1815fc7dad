"""Pin the CPU oracle against the reference test-suite's known answers and
host-reference loops (tests/golden/reference_cases.json). CPU only."""
import numpy as np
import pytest

import oracle
from tests.helpers import arr, assert_approx, load_cases

CASES = load_cases()


def by_op(*ops):
    return [pytest.param(c, id=c["name"]) for c in CASES if c["op"] in ops]


def run_pipeline(c):
    q, k, v = arr(c["q"]), arr(c["k"]), arr(c["v"])
    T = q.dtype
    g, layout = c["g"], c["layout"]
    Tk = k.shape[1] if layout == 0 else k.shape[2]
    s = np.zeros((q.shape[0], q.shape[2], q.shape[1], Tk), T)
    oracle.attention_scores(q, k, s, g, layout)
    scores = s.copy()
    oracle.scale(s, T.type(c["scale"]), s)
    scaled = s.copy()
    p = np.zeros_like(s)
    if c["causal"]:
        oracle.causal_softmax(s, p, 3, 2, 3)
    else:
        oracle.softmax(s, p, 3)
    o = np.zeros(q.shape, T)
    oracle.attention_apply(p, v, o, g, layout)
    return scores, scaled, p, o


@pytest.mark.parametrize("c", by_op("pipeline"))
def test_pipeline(c):
    _, scaled, p, o = run_pipeline(c)
    # the reference test compares the scaled scores (scale is applied in place)
    assert_approx(scaled, arr(c["expected_scores"]), c["eps"], c["margin"], "scores")
    assert_approx(p, arr(c["expected_probs"]), c["eps"], c["margin"], "probs")
    assert_approx(o, arr(c["expected_out"]), c["eps"], c["margin"], "out")


@pytest.mark.parametrize("c", by_op("pipeline_finite"))
def test_determinism_finite(c):
    q, k, v = arr(c["q"]), arr(c["k"]), arr(c["v"])
    s = np.zeros(c["scores_shape"], q.dtype)
    oracle.attention_scores(q, k, s)
    p = np.zeros_like(s)
    oracle.softmax(s, p, 3)
    o = np.zeros_like(q)
    oracle.attention_apply(p, v, o)
    assert np.isfinite(s).all() and np.isfinite(o).all()
    s2 = np.zeros_like(s)
    oracle.attention_scores(q, k, s2)
    assert np.array_equal(s, s2)


@pytest.mark.parametrize("c", by_op("gqa"))
def test_gqa_known_answers(c):
    q, k, v = arr(c["q"]), arr(c["k"]), arr(c["v"])
    s = np.zeros((1, 4, 1, 1), q.dtype)
    oracle.attention_scores(q, k, s, c["g"], c["layout"])
    p = np.zeros_like(s)
    oracle.softmax(s, p, 3)
    o = np.zeros_like(q)
    oracle.attention_apply(p, v, o, c["g"], c["layout"])
    assert_approx(s, arr(c["expected_scores"]), c["eps"], c["margin"], "scores")
    assert_approx(o, arr(c["expected_out"]), c["eps"], c["margin"], "out")


@pytest.mark.parametrize("c", by_op("scores"))
def test_scores(c):
    q, k = arr(c["q"]), arr(c["k"])
    e = arr(c["expected"])
    s = np.full(e.shape, c["prefill_value"], q.dtype)
    oracle.attention_scores(q, k, s, c["g"], c["layout"])
    assert_approx(s, e, c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("apply"))
def test_apply(c):
    p, v = arr(c["probs"]), arr(c["v"])
    e = arr(c["expected"])
    o = np.full(e.shape, c["prefill_value"], p.dtype)
    oracle.attention_apply(p, v, o, c["g"], c["layout"])
    assert_approx(o, e, c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("softmax", "causal_softmax"))
def test_softmax(c):
    x = arr(c["x"])
    out = np.full_like(x, c["prefill_value"])
    if c["op"] == "softmax":
        oracle.softmax(x, out, c["axis"])
    else:
        oracle.causal_softmax(x, out, c["axis"], c["query_axis"], c["key_axis"])
    assert_approx(out, arr(c["expected"]), c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("softmax_stability"))
def test_softmax_stability(c):
    x = arr(c["x"])
    out = np.zeros_like(x)
    oracle.causal_softmax(x, out, 3, 2, 3)
    for z in c["zero_at"]:
        assert out[tuple(z)] == 0
    sums = [out[0, 0, 0, 0], out[0, 0, 1, :].sum(dtype=x.dtype)]
    assert_approx(np.array(sums), np.array(c["row_sums"]), c["eps"], c["margin"], "row sums")


@pytest.mark.parametrize("c", by_op("rope_qk"))
def test_rope(c):
    q, k, cos, sin = arr(c["q"]), arr(c["k"]), arr(c["cos"]), arr(c["sin"])
    oq, ok = np.zeros_like(q), np.zeros_like(k)
    oracle.rope(q, cos, sin, oq, c["layout"], c["position_offset"])
    oracle.rope(k, cos, sin, ok, c["layout"], c["position_offset"])
    assert_approx(oq, arr(c["expected_q"]), c["eps"], c["margin"], "q")
    assert_approx(ok, arr(c["expected_k"]), c["eps"], c["margin"], "k")


@pytest.mark.parametrize("c", by_op("qkv_rope"))
def test_qkv_rope(c):
    x, cos, sin = arr(c["x"]), arr(c["cos"]), arr(c["sin"])
    t, h, d = c["tokens"], c["heads"], c["head_dim"]
    outs = []
    for w in ("wq", "wk", "wv"):
        o = np.zeros((t, h * d), x.dtype)
        oracle.gemm(x, arr(c[w]), o)
        outs.append(o)
    q4 = outs[0].reshape(1, t, h, d)
    k4 = outs[1].reshape(1, t, h, d)
    rq, rk = np.zeros_like(q4), np.zeros_like(k4)
    oracle.rope(q4, cos, sin, rq)
    oracle.rope(k4, cos, sin, rk)
    assert_approx(rq.reshape(t, h * d), arr(c["expected_q"]), c["eps"], c["margin"], "q")
    assert_approx(rk.reshape(t, h * d), arr(c["expected_k"]), c["eps"], c["margin"], "k")
    assert_approx(outs[2], arr(c["expected_v"]), c["eps"], c["margin"], "v")


@pytest.mark.parametrize("c", by_op("rms_norm"))
def test_rms_norm(c):
    x, w = arr(c["x"]), arr(c["w"])
    out = np.zeros_like(x)
    oracle.rms_norm(x, w, out, x.dtype.type(c["epsilon"]))
    assert_approx(out, arr(c["expected"]), c["eps"], c["margin"], "rmsNorm")


@pytest.mark.parametrize("c", by_op("embedding"))
def test_embedding(c):
    table, ids = arr(c["table"]), arr(c["ids"])
    view = table[:, c["col_offset"]:c["col_offset"] + c["hidden"]]  # strided subview, no copy
    out = np.zeros((ids.shape[0], c["hidden"]), table.dtype)
    oracle.embedding_lookup(ids, view, out)
    assert np.array_equal(out, arr(c["expected"]))


def test_attention_rows_matches_per_op_pipeline():
    """The sampled-row pipeline equals the full per-op pipeline on those rows."""
    g = np.random.default_rng(7)
    for T in (np.float32, np.float64):
        q = g.standard_normal((2, 9, 4, 8)).astype(T)
        k = g.standard_normal((2, 2, 9, 8)).astype(T)   # BHTD, 2 kv heads (g = 2)
        v = g.standard_normal((2, 2, 9, 8)).astype(T)
        for causal in (False, True):
            s = np.zeros((2, 4, 9, 9), T)
            oracle.attention_scores(q, k, s, 2, 1)
            oracle.scale(s, T(0.3), s)
            p = np.zeros_like(s)
            (oracle.causal_softmax(s, p, 3, 2, 3) if causal else oracle.softmax(s, p, 3))
            o = np.zeros_like(q)
            oracle.attention_apply(p, v, o, 2, 1)
            rows = np.array([[0, 0, 0], [1, 8, 3], [0, 4, 2], [1, 3, 1]], np.int64)
            got = oracle.attention_rows(q, k, v, rows, T(0.3), 2, 1, causal)
            want = np.stack([o[b, i, h] for b, i, h in rows])
            assert np.array_equal(got, want)
