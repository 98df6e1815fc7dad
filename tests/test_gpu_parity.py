"""Parity of the CUDA path with the CPU oracle on seeded inputs shaped like the
benchmark configurations, plus the edge cases of the reference's semantics.

Tolerances: integer/byte work (embedding gather) and uncontracted element-wise
work (RoPE, scale) are compared bit for bit; reductions within
|a-b| <= rtol*|b| + atol with (rtol, atol) = (1e-4, 1e-5) for fp32 and
(1e-11, 1e-12) for fp64 (tests/helpers.py TOL)."""
import math

import numpy as np
import pytest

import oracle
from tests.helpers import assert_close, assert_dot_close, normal, rng, rope_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ann():
    import alpakann_b200
    return alpakann_b200


def dev(a):
    import torch
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy()).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def empty(shape, dtype):
    import torch
    return torch.full(shape, float("nan"), dtype=torch.float32 if dtype == np.float32 else torch.float64,
                      device="cuda")


# ---------------------------------------------------------------- c1 / c4 ---
@pytest.mark.parametrize("T", [np.float32, np.float64])
def test_prefill_block_small(ann, T):
    """c1 (fp32) and a reduced c4 (fp64): embedding -> rmsNorm -> qkv -> rope ->
    scores -> scale -> causalSoftmax -> apply, every op against the oracle on
    the SAME inputs (the GPU's previous output), so errors never compound."""
    nn, ops = ann.onHost.nn, ann.onHost.ops
    g = rng(0x5EED + 1)
    B, Tt, dm, H, D, vocab = 1, 128, 256, 4, 64, 1024
    eps = 1e-6 if T == np.float32 else 1e-12
    ids = g.integers(0, vocab, size=B * Tt, dtype=np.uint32)
    table = normal(g, (vocab, dm), T)
    w = (1.0 + normal(g, (dm,), np.float64, 0.02)).astype(T)
    wq, wk, wv = (normal(g, (dm, H * D), T, 1.0 / math.sqrt(dm)) for _ in range(3))
    cos, sin = rope_tables(Tt, D, 1e4, T)
    q = ann.Queue()

    x = empty((B * Tt, dm), T)
    nn.embeddingLookup(q, None, dev(ids), dev(table), x)
    hx = host(x)
    assert np.array_equal(hx, table[ids])  # bit-exact gather

    y = empty((B * Tt, dm), T)
    nn.rmsNorm(q, None, x, dev(w), y, eps)
    ref = np.empty_like(hx)
    oracle.rms_norm(hx, w, ref, T(eps))
    hy = host(y)
    assert_close(hy, ref, T, "rmsNorm")

    Q2, K2, V2 = (empty((B * Tt, H * D), T) for _ in range(3))
    nn.qkvProjection(q, dev(hy), dev(wq), dev(wk), dev(wv), Q2, K2, V2)
    for name, t, wt in (("Q", Q2, wq), ("K", K2, wk), ("V", V2, wv)):
        r = np.empty((B * Tt, H * D), T)
        oracle.gemm(hy, wt, r)
        rt, at = (1e-4, 1e-5) if T == np.float32 else (1e-11, 1e-12)
        got = host(t)
        # cuBLAS and the sequential host sum order differ: compare relative to the row scale
        scale_ = np.abs(hy).max() * np.abs(wt).max() * dm
        assert np.abs(got - r).max() <= rt * scale_ + at, f"qkvProjection {name}"

    Q4, K4 = Q2.view(B, Tt, H, D), K2.view(B, Tt, H, D)
    hq, hk = host(Q4), host(K4)
    nn.ropeInPlace(q, None, Q4, K4, dev(cos), dev(sin))
    rq, rk = np.empty_like(hq), np.empty_like(hk)
    oracle.rope(hq, cos, sin, rq)
    oracle.rope(hk, cos, sin, rk)
    assert np.array_equal(host(Q4), rq) and np.array_equal(host(K4), rk)  # bit-exact rotation

    V4 = V2.view(B, Tt, H, D)
    s = empty((B, H, Tt, Tt), T)
    nn.attentionScores(q, None, Q4, K4, s)
    rs = np.empty((B, H, Tt, Tt), T)
    oracle.attention_scores(rq, rk, rs)
    hs = host(s)
    absdot = oracle.attention_scores(np.abs(rq), np.abs(rk), np.empty_like(rs))
    assert_dot_close(hs, rs, absdot, D, T, "scores")

    scale = T(1.0 / math.sqrt(D))
    ops.scale(q, None, s, scale, s)
    ss = np.empty_like(hs)
    oracle.scale(hs, scale, ss)
    assert np.array_equal(host(s), ss)  # bit-exact scale

    p = empty((B, H, Tt, Tt), T)
    nn.causalSoftmax(q, None, s, p, 3, 2, 3)
    rp = np.empty_like(ss)
    oracle.causal_softmax(ss, rp, 3, 2, 3)
    hp = host(p)
    assert_close(hp, rp, T, "causalSoftmax")
    assert (hp[..., np.triu_indices(Tt, 1)[0], np.triu_indices(Tt, 1)[1]] == 0).all()

    o = empty((B, Tt, H, D), T)
    nn.attentionApply(q, None, p, V4, o)
    ro = np.empty((B, Tt, H, D), T)
    hv = host(V4)
    oracle.attention_apply(hp, hv, ro)
    absdot = oracle.attention_apply(np.abs(hp), np.abs(hv), np.empty_like(ro))
    assert_dot_close(host(o), ro, absdot, Tt, T, "attentionApply")


# -------------------------------------------------------------------- c2 ---
def _decode_inputs(T, B, Tk, Hq, Hkv, D, seed, layout=1):
    g = rng(seed)
    q = normal(g, (B, 1, Hq, D), T)
    shape = (B, Hkv, Tk, D) if layout == 1 else (B, Tk, Hkv, D)
    return q, normal(g, shape, T), normal(g, shape, T)


def test_decode_c2_per_op_and_fused(ann):
    """c2: batch 8, 1 query, cache 2048, 32 heads x 128, fp32, BHTD cache.
    RoPE at position 2048 on Q and the new K row, then the per-op pipeline and
    the fused kernel, both against the oracle pipeline."""
    nn, ops = ann.onHost.nn, ann.onHost.ops
    T, B, Tk, H, D = np.float32, 8, 2048, 32, 128
    q, k, v = _decode_inputs(T, B, Tk, H, H, D, 0x5EED + 2)
    knew = normal(rng(99), (B, 1, H, D), T)
    cos, sin = rope_tables(Tk + 1, D, 1e4, T)
    queue = ann.Queue()
    dq, dkn = dev(q), dev(knew)
    nn.ropeInPlace(queue, None, dq, dkn, dev(cos), dev(sin), ann.RopeLayout.BTHD, Tk)
    rq, rkn = np.empty_like(q), np.empty_like(knew)
    oracle.rope(q, cos, sin, rq, 0, Tk)
    oracle.rope(knew, cos, sin, rkn, 0, Tk)
    assert np.array_equal(host(dq), rq) and np.array_equal(host(dkn), rkn)

    scale = T(1.0 / math.sqrt(D))
    rs = np.empty((B, H, 1, Tk), T)
    oracle.attention_scores(rq, k, rs, 1, 1)
    oracle.scale(rs, scale, rs)
    rp = np.empty_like(rs)
    oracle.softmax(rs, rp, 3)
    ro = np.empty((B, 1, H, D), T)
    oracle.attention_apply(rp, v, ro, 1, 1)

    dk, dv = dev(k), dev(v)
    s, p, o = empty((B, H, 1, Tk), T), empty((B, H, 1, Tk), T), empty((B, 1, H, D), T)
    nn.attentionScores(queue, None, dq, dk, s, 1, ann.AttentionKvLayout.BHTD)
    ops.scale(queue, None, s, scale, s)
    nn.softmax(queue, None, s, p, 3)
    nn.attentionApply(queue, None, p, dv, o, 1, ann.AttentionKvLayout.BHTD)
    abs_s = oracle.attention_scores(np.abs(rq), np.abs(k), np.empty_like(rs), 1, 1) * scale
    abs_o = oracle.attention_apply(np.abs(rp), np.abs(v), np.empty_like(ro), 1, 1)
    assert_dot_close(host(s), rs, abs_s, D, T, "scores*scale")
    assert_close(host(p), rp, T, "softmax")
    assert_dot_close(host(o), ro, abs_o, Tk, T, "per-op out")

    of = empty((B, 1, H, D), T)
    nn.attentionDecode(queue, None, dq, dk, dv, of, scale, 1, ann.AttentionKvLayout.BHTD)
    assert_close(host(of), ro, T, "fused decode out")
    # repeated calls are deterministic
    of2 = empty((B, 1, H, D), T)
    nn.attentionDecode(queue, None, dq, dk, dv, of2, scale, 1, ann.AttentionKvLayout.BHTD)
    assert np.array_equal(host(of), host(of2))
    assert queue.take_device_error() == 0


@pytest.mark.parametrize("T,D", [(np.float32, 64), (np.float32, 128), (np.float32, 256), (np.float64, 64),
                                 (np.float64, 128)])
@pytest.mark.parametrize("Tk", [1, 31, 33, 1000, 2049, 5000])
def test_decode_fused_shapes(ann, T, D, Tk):
    """Ragged key counts (partial tiles, one key, several splits), all head
    sizes, fp32 and fp64, against the oracle pipeline."""
    B, H = 2, 4
    q, k, v = _decode_inputs(T, B, Tk, H, H, D, 1000 + Tk + D)
    scale = T(1.0 / math.sqrt(D))
    rows = np.array([[b, 0, h] for b in range(B) for h in range(H)], np.int64)
    ref = oracle.attention_rows(q, k, v, rows, scale, 1, 1, False).reshape(B, 1, H, D)
    o = empty((B, 1, H, D), T)
    ann.onHost.nn.attentionDecode(ann.Queue(), None, dev(q), dev(k), dev(v), o, scale, 1,
                                  ann.AttentionKvLayout.BHTD)
    assert_close(host(o), ref, T, f"decode D={D} Tk={Tk}")


@pytest.mark.parametrize("layout", [0, 1])
def test_decode_fused_gqa_layouts_multiquery(ann, layout):
    """GQA (g = 4), BTHD and BHTD caches, several query tokens per sequence
    (each a non-causal row over the whole cache), strided output view."""
    import torch
    T, B, Tq, Hq, Hkv, D, Tk = np.float32, 3, 2, 8, 2, 128, 700
    g = rng(7 + layout)
    q = normal(g, (B, Tq, Hq, D), T)
    shape = (B, Hkv, Tk, D) if layout == 1 else (B, Tk, Hkv, D)
    k, v = normal(g, shape, T), normal(g, shape, T)
    scale = T(0.0883883)
    rows = np.array([[b, t, h] for b in range(B) for t in range(Tq) for h in range(Hq)], np.int64)
    ref = oracle.attention_rows(q, k, v, rows, scale, 4, layout, False).reshape(B, Tq, Hq, D)
    big = torch.zeros((B, Tq, Hq, 2 * D), dtype=torch.float32, device="cuda")
    o = big[..., D:]  # non-contiguous output rows
    ann.onHost.nn.attentionDecode(ann.Queue(), None, dev(q), dev(k), dev(v), o, scale, 4, layout)
    assert_close(host(o), ref, T, "decode gqa")
    assert (host(big[..., :D]) == 0).all()


def test_decode_empty_cache_gives_zeros(ann):
    T, B, H, D = np.float32, 1, 2, 64
    q = normal(rng(3), (B, 1, H, D), T)
    k = np.zeros((B, H, 0, D), T)
    o = empty((B, 1, H, D), T)
    import torch
    ann.onHost.nn.attentionDecode(ann.Queue(), None, dev(q), torch.zeros((B, H, 0, D), device="cuda"),
                                  torch.zeros((B, H, 0, D), device="cuda"), o, 0.125, 1, 1)
    # attentionApply over zero keys sums nothing
    assert (host(o) == 0).all()
    del k


# --------------------------------------------------------- softmax axes ---
@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("axis,qa,ka", [(3, 2, 3), (2, 3, 2), (2, 2, 3), (1, 2, 3), (3, 3, 3)])
def test_causal_softmax_generic_axes(ann, T, axis, qa, ka):
    """The mask rule probe[queryAxis] < probe[keyAxis] for any axis choice,
    including rows that are entirely masked (written as zeros)."""
    x = normal(rng(axis * 10 + qa + ka), (2, 3, 37, 41), T) * T(4)
    ref = np.empty_like(x)
    oracle.causal_softmax(x, ref, axis, qa, ka)
    out = empty(x.shape, T)
    ann.onHost.nn.causalSoftmax(ann.Queue(), None, dev(x), out, axis, qa, ka)
    assert_close(host(out), ref, T, "causalSoftmax")


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("L", [1, 5, 1024, 1025, 4096, 32768])
def test_softmax_row_lengths(ann, T, L):
    x = normal(rng(L), (2, 3, L), T) * T(3)
    ref = np.empty_like(x)
    oracle.softmax(x, ref, 2)
    out = empty(x.shape, T)
    ann.onHost.nn.softmax(ann.Queue(), None, dev(x), out, 2)
    assert_close(host(out), ref, T, "softmax")


@pytest.mark.parametrize("T,L,rows", [(np.float32, 32768, 700), (np.float64, 16384, 5), (np.float32, 20000, 3)])
@pytest.mark.parametrize("kind", ["softmax", "causal", "masked"])
def test_softmax_long_rows_on_clusters(ann, T, L, rows, kind):
    """Rows of 64 to 224 KB: a quarter of each row per CTA of a four-CTA
    cluster, the row max and sum combined through distributed shared memory.
    700 rows of 32768 are more rows than resident clusters (each cluster walks
    several); causal rows keep a prefix (query axis 1 against the key axis);
    maskedSoftmax doubles the bytes a row."""
    g = rng(L + rows)
    x = normal(g, (rows, 1, L), T) * T(4)
    ref = np.empty_like(x)
    out = empty(x.shape, T)
    nn = ann.onHost.nn
    if kind == "softmax":
        oracle.softmax(x, ref, 2)
        nn.softmax(ann.Queue(), None, dev(x), out, 2)
    elif kind == "causal":  # query index = row (axis 0), key = axis 2: keeps [0, row]
        oracle.causal_softmax(x, ref, 2, 0, 2)
        nn.causalSoftmax(ann.Queue(), None, dev(x), out, 2, 0, 2)
    else:
        m = normal(g, x.shape, T)
        oracle.masked_softmax(x, m, ref, 2)
        nn.maskedSoftmax(ann.Queue(), None, dev(x), dev(m), out, 2)
    assert_close(host(out), ref, T, kind)


# ----------------------------------------------------- rms / embedding ---
@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("shape", [(3, 5), (4, 256), (2, 3, 1024), (5, 4096), (3, 8192), (2, 1027)])
def test_rms_norm_shapes(ann, T, shape):
    g = rng(sum(shape))
    x = normal(g, shape, T)
    w = (1.0 + normal(g, (shape[-1],), np.float64, 0.02)).astype(T)
    eps = 1e-5
    ref = np.empty_like(x)
    oracle.rms_norm(x, w, ref, T(eps))
    out = empty(shape, T)
    ann.onHost.nn.rmsNorm(ann.Queue(), None, dev(x), dev(w), out, eps)
    assert_close(host(out), ref, T, "rmsNorm")


def test_rms_norm_strided_rows(ann):
    import torch
    T = np.float32
    x = normal(rng(5), (6, 2 * 300), T)
    xs = x[:, ::2]
    w = np.ones(300, T)
    ref = np.empty((6, 300), T)
    oracle.rms_norm(np.ascontiguousarray(xs), w, ref, T(1e-6))
    dx = dev(x)[:, ::2]
    out = torch.empty((6, 300), dtype=torch.float32, device="cuda")
    ann.onHost.nn.rmsNorm(ann.Queue(), None, dx, dev(w), out, 1e-6)
    assert_close(host(out), ref, T, "rmsNorm strided")


@pytest.mark.parametrize("T", [np.float32, np.float64])
def test_embedding_gather_bitexact_and_bad_ids(ann, T):
    g = rng(11)
    table = normal(g, (1024, 256), T)
    ids = g.integers(0, 1024, size=300, dtype=np.uint32)
    out = empty((300, 256), T)
    queue = ann.Queue()
    ann.onHost.nn.embeddingLookup(queue, None, dev(ids), dev(table), out)
    assert np.array_equal(host(out), table[ids])
    assert queue.take_device_error() == 0
    ids[7] = 1024  # out of range: zero row and a device error bit instead of an out-of-bounds read
    ann.onHost.nn.embeddingLookup(queue, None, dev(ids), dev(table), out)
    h = host(out)
    assert (h[7] == 0).all() and np.array_equal(np.delete(h, 7, 0), np.delete(table[ids.clip(0, 1023)], 7, 0))
    assert queue.take_device_error() & 0x1
    assert queue.take_device_error() == 0


@pytest.mark.parametrize("T", [np.float32, np.float64])
def test_rope_bhtd_and_offsets(ann, T):
    """RoPE on a BHTD tensor at a position offset, out of place and in place,
    bit-exact against the oracle."""
    import torch
    g = rng(21)
    x = normal(g, (2, 3, 17, 64), T)
    cos, sin = rope_tables(40, 64, 5e5, T)
    ref = np.empty_like(x)
    oracle.rope(x, cos, sin, ref, 1, 23)
    out = empty(x.shape, T)
    ann.onHost.nn.rope(ann.Queue(), None, dev(x), dev(cos), dev(sin), out, ann.RopeLayout.BHTD, 23)
    assert np.array_equal(host(out), ref)
    dx = dev(x)
    ann.onHost.nn.ropeInPlace(ann.Queue(), None, dx, dev(cos), dev(sin), ann.RopeLayout.BHTD, 23)
    assert np.array_equal(host(dx), ref)
    # non-contiguous head vectors take the scalar path, same bits
    big = torch.zeros((2, 3, 17, 128), dtype=dx.dtype, device="cuda")
    big[..., ::2] = dev(x)
    sub = big[..., ::2]
    ann.onHost.nn.ropeInPlace(ann.Queue(), None, sub, dev(cos), dev(sin), ann.RopeLayout.BHTD, 23)
    assert np.array_equal(host(sub), ref)


@pytest.mark.parametrize("T", [np.float32, np.float64])
def test_scores_apply_gqa_bthd_ragged(ann, T):
    """Per-op scores/apply with GQA (g = 3), ragged tile edges, both layouts."""
    g = rng(31)
    B, Tq, Tk, Hq, Hkv, D = 2, 67, 45, 6, 2, 40
    q = normal(g, (B, Tq, Hq, D), T)
    for layout in (0, 1):
        kshape = (B, Tk, Hkv, D) if layout == 0 else (B, Hkv, Tk, D)
        k, v = normal(g, kshape, T), normal(g, kshape, T)
        rs = np.empty((B, Hq, Tq, Tk), T)
        oracle.attention_scores(q, k, rs, 3, layout)
        s = empty(rs.shape, T)
        ann.onHost.nn.attentionScores(ann.Queue(), None, dev(q), dev(k), s, 3, layout)
        assert_close(host(s), rs, T, "scores")
        p = normal(g, rs.shape, T)
        ro = np.empty((B, Tq, Hq, D), T)
        oracle.attention_apply(p, v, ro, 3, layout)
        o = empty(ro.shape, T)
        ann.onHost.nn.attentionApply(ann.Queue(), None, dev(p), dev(v), o, 3, layout)
        assert_close(host(o), ro, T, "apply")


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("case", ["scores_bthd", "scores_bhtd_gqa", "apply_bthd", "apply_bhtd_gqa"])
def test_scores_apply_wide_tiles(ann, case, T):
    """fp32 scores / apply at sizes that fill the GPU, so they run on the
    128-column tiles (8 x 8 outputs a thread for scores, 4 x 8 for apply):
    ragged edges, GQA, both K/V layouts, against the oracle. Sums of
    hundreds of products can cancel to near 0, where FMA and the oracle's
    separate multiply-add round differently; each output may differ by the
    dot-product rounding bound 4 eps sqrt(K) sum|a b| on top of the usual
    tolerance (sum|a b| from the oracle on |a| and |b|). fp64 runs on the
    FP64 tensor-core tiles (64 x 64, mma.sync m16n8k4) at smaller sizes."""
    g = rng(41)
    layout = 1 if "bhtd" in case else 0
    gq = 2 if "gqa" in case else 1
    # fp32: D = 72 and Tk = 612 take the 16-byte-load variant, D = 70 and
    # Tk = 611 the scalar-load one
    if T == np.float64:
        if case.startswith("scores"):
            B, Tq, Tk, Hq, D = 2, 301, 277, 4, (64 if gq > 1 else 37)
        else:
            B, Tq, Tk, Hq, D = 2, 290, (256 if gq > 1 else 283), 4, 64
    elif case.startswith("scores"):
        B, Tq, Tk, Hq, D = 1, 1100, 1037, 8, (72 if gq > 1 else 70)
    else:
        B, Tq, Tk, Hq, D = 1, 700, (612 if gq > 1 else 611), 48, 128
    Hkv = Hq // gq
    kshape = (B, Tk, Hkv, D) if layout == 0 else (B, Hkv, Tk, D)
    if case.startswith("scores"):
        q, k = normal(g, (B, Tq, Hq, D), T), normal(g, kshape, T)
        want = oracle.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), T), gq, layout)
        s = empty(want.shape, T)
        ann.onHost.nn.attentionScores(ann.Queue(), None, dev(q), dev(k), s, gq, layout)
        got, K = host(s), D
        absdot = oracle.attention_scores(np.abs(q), np.abs(k), np.empty_like(want), gq, layout)
    else:
        p, v = normal(g, (B, Hq, Tq, Tk), T), normal(g, kshape, T)
        want = oracle.attention_apply(p, v, np.empty((B, Tq, Hq, D), T), gq, layout)
        o = empty(want.shape, T)
        ann.onHost.nn.attentionApply(ann.Queue(), None, dev(p), dev(v), o, gq, layout)
        got, K = host(o), Tk
        absdot = oracle.attention_apply(np.abs(p), np.abs(v), np.empty_like(want), gq, layout)
    rtol, atol = (1e-4, 1e-5) if T == np.float32 else (1e-11, 1e-12)
    err = np.abs(got.astype(np.float64) - want)
    bound = rtol * np.abs(want.astype(np.float64)) + atol + 4 * np.finfo(T).eps * np.sqrt(K) * absdot
    assert (err <= bound).all(), (case, float((err - bound).max()), int((err > bound).sum()))


@pytest.mark.parametrize("T,D", [(np.float32, 128), (np.float64, 64)])
@pytest.mark.parametrize("splits", [1, 2, 5, 8, 16])
def test_decode_forced_cluster_sizes(ann, monkeypatch, T, D, splits):
    """Every cluster size up to the non-portable 16, and one CTA walking many
    2048-key sub-chunks (online rescale), on scores with a wide dynamic range."""
    B, H, Tk = 1, 3, 9000
    g = rng(splits * 7 + D)
    q = normal(g, (B, 1, H, D), T) * T(3)
    k, v = normal(g, (B, H, Tk, D), T), normal(g, (B, H, Tk, D), T)
    scale = T(1.0 / math.sqrt(D))
    rows = np.array([[0, 0, h] for h in range(H)], np.int64)
    ref = oracle.attention_rows(q, k, v, rows, scale, 1, 1, False).reshape(B, 1, H, D)
    monkeypatch.setenv("ANN_DECODE_SPLITS", str(splits))
    o = empty((B, 1, H, D), T)
    queue = ann.Queue()
    ann.onHost.nn.attentionDecode(queue, None, dev(q), dev(k), dev(v), o, scale, 1, ann.AttentionKvLayout.BHTD)
    assert_close(host(o), ref, T, f"decode splits={splits}")
    assert queue.take_device_error() == 0


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("case", ["reassembly", "sliced", "odd_rows"])
def test_scale_strided_views_bitexact(ann, T, case):
    """ops::scale on strided views (the row path for unit-stride inner runs and the
    generic element path), bit for bit against the same product in numpy."""
    import torch
    g = rng(17)
    s = T(0.5) if case != "reassembly" else T(1.0)
    if case == "reassembly":   # rank-major gather [G,B,T,Hl,D] -> BTHD [B,T,G,Hl,D]
        x = normal(g, (4, 3, 5, 2, 64), T)
        src = dev(x).permute(1, 2, 0, 3, 4)
        out = torch.full((3, 5, 4, 2, 64), float("nan"), dtype=src.dtype, device="cuda")
        ref = (x.transpose(1, 2, 0, 3, 4) * s).astype(T)
    elif case == "sliced":     # every other row of a matrix into a column-sliced output
        x = normal(g, (40, 96), T)
        src = dev(x)[::2, 8:72]
        big = torch.full((20, 80), float("nan"), dtype=src.dtype, device="cuda")
        out = big[:, 4:68]
        ref = (x[::2, 8:72] * s).astype(T)
    else:                      # rows of 3 elements: not a whole 16-byte vector, generic path
        x = normal(g, (7, 9, 3), T)
        src = dev(x).permute(1, 0, 2)
        out = torch.full((9, 7, 3), float("nan"), dtype=src.dtype, device="cuda")
        ref = (x.transpose(1, 0, 2) * s).astype(T)
    ann.onHost.ops.scale(ann.Queue(), None, src, s, out)
    assert np.array_equal(host(out), ref)



@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("H", [256, 2048, 300])
def test_embedding_rms_norm_fused_equals_two_launches(ann, T, H):
    """Fused gather + rmsNorm = embeddingLookup then rmsNorm, bit for bit (row
    lengths for the warp path, the CTA path and the unvectorised path); an id out
    of range gives a zero row and the token-id error bit."""
    g = rng(23)
    table = normal(g, (1024, H), T)
    w = (1 + 0.02 * normal(g, (H,), T)).astype(T)
    ids = g.integers(0, 1024, size=77, dtype=np.uint32)
    queue = ann.Queue()
    hidden, two, fused = empty((77, H), T), empty((77, H), T), empty((77, H), T)
    ann.onHost.nn.embeddingLookup(queue, None, dev(ids), dev(table), hidden)
    ann.onHost.nn.rmsNorm(queue, None, hidden, dev(w), two, 1e-6)
    ann.onHost.nn.embeddingRmsNorm(queue, None, dev(ids), dev(table), dev(w), fused, 1e-6)
    assert np.array_equal(host(fused), host(two))
    ref = np.empty((77, H), T)
    oracle.rms_norm(np.ascontiguousarray(table[ids]), w, ref, T(1e-6))
    assert_close(host(fused), ref, T, "embeddingRmsNorm")
    assert queue.take_device_error() == 0
    ids[5] = 4096
    ann.onHost.nn.embeddingRmsNorm(queue, None, dev(ids), dev(table), dev(w), fused, 1e-6)
    h = host(fused)
    assert (h[5] == 0).all() and np.array_equal(np.delete(h, 5, 0), np.delete(host(two), 5, 0))
    assert queue.take_device_error() & 0x1



@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("rope", [False, True])
def test_kv_cache_append(ann, T, rope):
    """New rows land at [position, position + Tn) of a layer of an LBHTD cache,
    everything else untouched; with RoPE tables K equals ropeInPlace + append and
    the oracle's rope (onAcc/internal/nn/rope.hpp:35-46), bit for bit, and V is
    copied as is."""
    import torch
    g = rng(31)
    L, B, Hkv, Tcap, D, Tn, pos = 2, 3, 4, 40, 64, 5, 17
    cache_k = normal(g, (L, B, Hkv, Tcap, D), T)
    cache_v = normal(g, (L, B, Hkv, Tcap, D), T)
    kn, vn = normal(g, (B, Tn, Hkv, D), T), normal(g, (B, Tn, Hkv, D), T)
    ck, cv = dev(cache_k), dev(cache_v)
    cos, sin = rope_tables(Tcap, D, 1e4, T)
    queue = ann.Queue()
    if rope:
        ann.onHost.nn.kvCacheAppend(queue, None, dev(kn), dev(vn), ck[1], cv[1], pos, dev(cos), dev(sin))
        kr = dev(kn)
        ann.onHost.nn.ropeInPlace(queue, None, kr, dev(cos), dev(sin), ann.RopeLayout.BTHD, pos)
        want_k = host(kr)
        oracle_k = oracle.rope(kn, cos, sin, np.empty_like(kn), 0, pos)
        assert np.array_equal(want_k, oracle_k)
    else:
        ann.onHost.nn.kvCacheAppend(queue, None, dev(kn), dev(vn), ck[1], cv[1], pos)
        want_k = kn
    hk, hv = host(ck), host(cv)
    ek, ev = cache_k.copy(), cache_v.copy()
    ek[1, :, :, pos:pos + Tn] = want_k.transpose(0, 2, 1, 3)
    ev[1, :, :, pos:pos + Tn] = vn.transpose(0, 2, 1, 3)
    assert np.array_equal(hk, ek) and np.array_equal(hv, ev)


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("in_place", [False, True])
def test_output_projection_residual(ann, T, in_place):
    """output = residual + input . Wo against an fp64 product, at the GEMM tolerance."""
    import torch
    g = rng(37)
    N, K, M = 70, 256, 192
    x, w, r = normal(g, (N, K), T), (normal(g, (K, M), T) / np.sqrt(K)).astype(T), normal(g, (N, M), T)
    ref = r.astype(np.float64) + x.astype(np.float64) @ w.astype(np.float64)
    dr = dev(r)
    out = dr if in_place else empty((N, M), T)
    ann.onHost.nn.outputProjectionResidual(ann.Queue(), dev(x), dev(w), dr, out)
    rtol, atol = (1e-4, 1e-4) if T == np.float32 else (1e-11, 1e-11)
    assert np.allclose(host(out), ref, rtol=rtol, atol=atol)
