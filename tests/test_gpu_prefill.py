"""Fused prefill attention against the oracle's per-op pipeline
(scores -> scale -> causalSoftmax / softmax -> apply): full comparison where
the oracle finishes in seconds, sampled rows at the full configuration
sizes. Tolerances as in tests/helpers.py TOL (fp32 1e-4 rel + 1e-5 abs,
fp64 1e-11 rel + 1e-12 abs)."""
import math

import numpy as np
import pytest

import oracle
from tests.helpers import assert_close, normal, rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ann():
    import alpakann_b200
    return alpakann_b200


@pytest.fixture(params=["tensor", "tensor-1sm", "fma"], autouse=True)
def kernel(request, monkeypatch):
    """fp32 runs on the tcgen05 3xTF32 kernel on SM pairs by default;
    ANN_PREFILL_TC_PAIR=0 keeps it on one SM per CTA, ANN_PREFILL_FMA=1
    selects the FMA kernel (fp64 runs on the FP64 tensor cores, or on DFMA
    with ANN_PREFILL_FMA=1)."""
    monkeypatch.delenv("ANN_PREFILL_FMA", raising=False)
    monkeypatch.delenv("ANN_PREFILL_TC_PAIR", raising=False)
    if request.param == "fma":
        monkeypatch.setenv("ANN_PREFILL_FMA", "1")
    elif request.param == "tensor-1sm":
        monkeypatch.setenv("ANN_PREFILL_TC_PAIR", "0")
    return request.param


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def empty(shape, T):
    import torch
    return torch.full(shape, float("nan"), dtype=torch.float32 if T == np.float32 else torch.float64, device="cuda")


def oracle_pipeline(q, k, v, scale, g, layout, causal):
    T = q.dtype.type
    B, Tq, Hq, D = q.shape
    Tk = k.shape[1] if layout == 0 else k.shape[2]
    s = np.empty((B, Hq, Tq, Tk), q.dtype)
    oracle.attention_scores(q, k, s, g, layout)
    oracle.scale(s, T(scale), s)
    p = np.empty_like(s)
    if causal:
        oracle.causal_softmax(s, p, 3, 2, 3)
    else:
        oracle.softmax(s, p, 3)
    o = np.empty_like(q)
    oracle.attention_apply(p, v, o, g, layout)
    return o


def run(ann, q, k, v, scale, g, layout, causal):
    o = empty(q.shape, q.dtype.type)
    queue = ann.Queue()
    ann.onHost.nn.attentionPrefill(queue, None, dev(q), dev(k), dev(v), o, scale, g, layout, causal)
    got = host(o)
    assert queue.take_device_error() == 0
    return got


@pytest.mark.parametrize("T", [np.float32, np.float64])
def test_prefill_c1_full(ann, T):
    """c1 shape (batch 1, seq 128, 4 heads x 64), causal, scale 1/8."""
    g = rng(0x5EED + 11)
    q, k, v = (normal(g, (1, 128, 4, 64), T) for _ in range(3))
    ref = oracle_pipeline(q, k, v, 0.125, 1, 0, True)
    assert_close(run(ann, q, k, v, 0.125, 1, 0, True), ref, T, "prefill c1")


@pytest.mark.parametrize("T,D", [(np.float32, 64), (np.float32, 128), (np.float64, 64), (np.float64, 128)])
@pytest.mark.parametrize("Tq,Tk,causal", [(1, 1, True), (100, 100, True), (130, 130, True), (50, 130, True),
                                          (130, 50, True), (77, 200, False), (64, 64, True)])
def test_prefill_shapes(ann, T, D, Tq, Tk, causal):
    """Ragged tiles, Tq != Tk with the reference's top-left mask, non-causal."""
    g = rng(Tq * 1000 + Tk + D)
    q = normal(g, (2, Tq, 3, D), T)
    k, v = normal(g, (2, Tk, 3, D), T), normal(g, (2, Tk, 3, D), T)
    sc = 1.0 / math.sqrt(D)
    ref = oracle_pipeline(q, k, v, sc, 1, 0, causal)
    assert_close(run(ann, q, k, v, sc, 1, 0, causal), ref, T, f"prefill Tq={Tq} Tk={Tk} causal={causal}")


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("layout", [0, 1])
def test_prefill_gqa_layouts(ann, T, layout):
    g = rng(40 + layout)
    B, Tt, Hq, Hkv, D = 2, 150, 8, 2, 64
    q = normal(g, (B, Tt, Hq, D), T)
    shape = (B, Tt, Hkv, D) if layout == 0 else (B, Hkv, Tt, D)
    k, v = normal(g, shape, T), normal(g, shape, T)
    ref = oracle_pipeline(q, k, v, 0.125, 4, layout, True)
    assert_close(run(ann, q, k, v, 0.125, 4, layout, True), ref, T, "prefill gqa")


@pytest.mark.parametrize("T", [np.float32, np.float64])
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_kv_cache_views(ann, T, D):
    """K / V as views into a larger BHTD cache: heads 1..2 of 4, the first Tk of
    Tcap positions (the layout of a KV cache with spare capacity). The fp32 path
    reads them through TMA tensor maps with these strides."""
    import torch
    g = rng(77 + D)
    B, Tq, Tk, Tcap, Hq = 2, 150, 150, 203, 2
    q = normal(g, (B, Tq, Hq, D), T)
    kc, vc = normal(g, (B, 4, Tcap, D), T), normal(g, (B, 4, Tcap, D), T)
    k, v = kc[:, 1:3, :Tk], vc[:, 1:3, :Tk]
    sc = 1.0 / math.sqrt(D)
    ref = oracle_pipeline(q, np.ascontiguousarray(k), np.ascontiguousarray(v), sc, 1, 1, True)
    o = empty(q.shape, T)
    queue = ann.Queue()
    kd, vd = dev(kc), dev(vc)
    ann.onHost.nn.attentionPrefill(queue, None, dev(q), kd[:, 1:3, :Tk], vd[:, 1:3, :Tk], o, sc, 1, 1, True)
    assert_close(host(o), ref, T, "prefill over cache views")
    assert queue.take_device_error() == 0


@pytest.mark.parametrize("shape", [(2, 1000, 3, 128), (1, 300, 2, 64)])
def test_prefill_alternating_tile_order_same_bits(ann, monkeypatch, shape):
    """ANN_PREFILL_ALTERNATE=1: the fp32 pair kernel takes its query tiles in
    the order heaviest, lightest, second heaviest, ... (the order it uses for
    multicast outputs with few waves of work); every tile is computed exactly
    as before, so the output is bit-identical to the default order."""
    B, Tt, H, D = shape
    g = rng(Tt + D)
    q, k, v = (normal(g, (B, Tt, H, D), np.float32) for _ in range(3))
    sc = 1.0 / math.sqrt(D)
    monkeypatch.setenv("ANN_PREFILL_ALTERNATE", "0")
    base = run(ann, q, k, v, sc, 1, 0, True)
    monkeypatch.setenv("ANN_PREFILL_ALTERNATE", "1")
    alt = run(ann, q, k, v, sc, 1, 0, True)
    assert np.array_equal(base, alt)
    assert_close(alt, oracle_pipeline(q, k, v, sc, 1, 0, True), np.float32, "prefill, alternating order")


def _sampled(ann, T, B, Tt, H, D, seed, nrows=24):
    import torch
    dt = torch.float32 if T == np.float32 else torch.float64
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, Tt, H, D), generator=gen, dtype=dt, device="cuda")
    k = torch.randn((B, Tt, H, D), generator=gen, dtype=dt, device="cuda")
    v = torch.randn((B, Tt, H, D), generator=gen, dtype=dt, device="cuda")
    o = torch.full_like(q, float("nan"))
    sc = 1.0 / math.sqrt(D)
    queue = ann.Queue()
    ann.onHost.nn.attentionPrefill(queue, None, q, k, v, o, sc, 1, 0, True)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(o).all())
    g = np.random.default_rng(seed)
    rows = [(0, 0, 0), (B - 1, Tt - 1, H - 1), (0, 63, 1), (0, 64, 1)]
    rows += [(int(g.integers(B)), int(g.integers(Tt)), int(g.integers(H))) for _ in range(nrows - len(rows))]
    for b, i, h in rows:
        qh = q[b:b + 1, i:i + 1, h:h + 1].cpu().numpy()
        kh = k[b:b + 1, :i + 1, h:h + 1].cpu().numpy()  # causal: keys 0..i
        vh = v[b:b + 1, :i + 1, h:h + 1].cpu().numpy()
        ref = oracle.attention_rows(qh, kh, vh, np.array([[0, 0, 0]], np.int64), T(sc), 1, 0, False)[0]
        assert_close(o[b, i, h].cpu().numpy(), ref, T, f"row {(b, i, h)}")
    assert queue.take_device_error() == 0


def test_prefill_c4_fp64_sampled(ann):
    """c4: batch 2, seq 1024, 16 heads x 64, fp64, causal."""
    _sampled(ann, np.float64, 2, 1024, 16, 64, 4)


def test_prefill_fp64_long_grid_sampled(ann):
    """fp64 D = 64 on a grid long enough for the 16-key-tile variant (2048 CTAs)."""
    _sampled(ann, np.float64, 4, 2048, 16, 64, 5)


def test_prefill_c3_fp32_sampled(ann):
    """c3: batch 4, seq 4096, 32 heads x 128, fp32, causal."""
    _sampled(ann, np.float32, 4, 4096, 32, 128, 3)


@pytest.mark.parametrize("splits", ["1", "2", "4"])
@pytest.mark.parametrize("shape,causal", [((1, 333, 2, 64), True), ((2, 160, 3, 128), True),
                                          ((1, 100, 2, 64), False), ((1, 40, 2, 64), True)])
def test_prefill_f64_key_splits(ann, monkeypatch, kernel, splits, shape, causal):
    """fp64 on the FP64 tensor cores with the key range of every query tile split
    over a cluster of 1, 2 or 4 CTAs (merged through distributed shared memory
    with the log-sum-exp rule): ragged query and key tiles, splits with no keys
    (40 rows: two 32-key tiles over four CTAs), causal and not, against the
    oracle. The split count a head-sharded rank picks on its own is one of these."""
    if kernel != "tensor":
        pytest.skip("the split is a property of the fp64 tensor-core kernel")
    monkeypatch.setenv("ANN_PREFILL_F64_SPLITS", splits)
    T = np.float64
    B, Tt, H, D = shape
    g = rng(Tt * 7 + D + int(splits))
    q, k, v = (normal(g, (B, Tt, H, D), T) for _ in range(3))
    if not causal:
        k, v = (normal(g, (B, Tt + 37, H, D), T) for _ in range(2))
    scale = 1.0 / math.sqrt(D)
    want = oracle_pipeline(q, k, v, scale, 1, 0, causal)
    got = run(ann, q, k, v, scale, 1, 0, causal)
    assert_close(got, want, T, f"fp64 prefill, {splits} key splits")
