"""The drop-in attentionScores / attentionApply (fp32) on the tensor cores
(tcgen05 3xTF32 on SM pairs, csrc/attention_tc.cu) against the oracle's
restatement of onAcc/internal/nn/attention.hpp:15-68.

Shapes cover what the kernels tile: head dims 64 and 128, query counts that
are not multiples of the 256-row pair tile, key counts that are multiples of 4
but not of the 128-key tile / 32-key chunk, several key chunks per work unit,
GQA, both K/V layouts, strided (padded) rows of the output, and the split of
the key range of attentionApply in two halves (small grids). Outputs outside
the view stay untouched. The FP32-pipe kernels that serve the other shapes are
forced with ANN_ATTENTION_OPS_SIMT=1 on the same inputs.

Tolerance: |got - want| <= rtol |want| + atol + 4 eps sqrt(K) sum|a b|, the
dot-product rounding bound on top of (1e-4, 1e-5) (sums of many products can
cancel to near 0, where any two summation orders differ), with sum|a b| from
the oracle on |a| and |b|."""
import numpy as np
import pytest

import oracle
from tests.helpers import normal, rng

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ann():
    from tests.helpers import build_library
    build_library()
    import alpakann_b200
    return alpakann_b200


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def check(got, want, absdot, K):
    err = np.abs(got.astype(np.float64) - want)
    bound = 1e-4 * np.abs(want.astype(np.float64)) + 1e-5 + 4 * np.finfo(np.float32).eps * np.sqrt(K) * absdot
    assert (err <= bound).all(), (float((err - bound).max()), int((err > bound).sum()))


SCORES = [  # B, Tq, Tk, Hq, Hkv, D, layout
    (1, 300, 388, 3, 3, 64, 0),     # one 256-row tile + a ragged one, ragged last key tile
    (2, 256, 1280, 4, 2, 128, 1),   # GQA, BHTD, 10 key tiles (several per work unit)
    (1, 97, 4, 2, 1, 128, 0),       # a single 4-key tile, most rows past Tq
    (1, 513, 2052, 2, 2, 64, 1),    # three row tiles, 17 key tiles
]


@pytest.mark.parametrize("case", SCORES)
def test_scores_tensor_cores(ann, case):
    import torch
    B, Tq, Tk, Hq, Hkv, D, layout = case
    g = rng(sum(case))
    gq = Hq // Hkv
    q = normal(g, (B, Tq, Hq, D), np.float32)
    kshape = (B, Tk, Hkv, D) if layout == 0 else (B, Hkv, Tk, D)
    k = normal(g, kshape, np.float32)
    want = oracle.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), np.float32), gq, layout)
    absdot = oracle.attention_scores(np.abs(q), np.abs(k), np.empty_like(want), gq, layout)
    # S rows padded by 8 floats: the pad must stay untouched
    big = torch.full((B, Hq, Tq, Tk + 8), float("nan"), device="cuda")
    s = big[..., :Tk]
    queue = ann.Queue()
    ann.onHost.nn.attentionScores(queue, None, dev(q), dev(k), s, gq, layout)
    hb = host(big)
    check(hb[..., :Tk], want, absdot, D)
    assert np.isnan(hb[..., Tk:]).all()
    assert queue.take_device_error() == 0


APPLY = [  # B, Tq, Tk, Hq, Hkv, D, layout
    (1, 300, 388, 3, 3, 64, 0),     # ragged rows and keys (12.1 chunks of 32)
    (2, 256, 1024, 4, 2, 128, 1),   # GQA, BHTD; small grid: the key range splits in two
    (1, 70, 4, 2, 2, 128, 0),       # one 4-key chunk
    (4, 600, 2048, 8, 8, 64, 1),    # 96 pair tiles x 64 chunks
]


@pytest.mark.parametrize("case", APPLY)
def test_apply_tensor_cores(ann, case):
    import torch
    B, Tq, Tk, Hq, Hkv, D, layout = case
    g = rng(sum(case) + 1)
    gq = Hq // Hkv
    p = normal(g, (B, Hq, Tq, Tk), np.float32)
    kshape = (B, Tk, Hkv, D) if layout == 0 else (B, Hkv, Tk, D)
    v = normal(g, kshape, np.float32)
    want = oracle.attention_apply(p, v, np.empty((B, Tq, Hq, D), np.float32), gq, layout)
    absdot = oracle.attention_apply(np.abs(p), np.abs(v), np.empty_like(want), gq, layout)
    queue = ann.Queue()
    o = torch.full((B, Tq, Hq, D), float("nan"), device="cuda")
    ann.onHost.nn.attentionApply(queue, None, dev(p), dev(v), o, gq, layout)
    check(host(o), want, absdot, Tk)
    # a strided output (rows padded): no split, the pad stays untouched
    big = torch.full((B, Tq, Hq, D + 4), float("nan"), device="cuda")
    ann.onHost.nn.attentionApply(queue, None, dev(p), dev(v), big[..., :D], gq, layout)
    hb = host(big)
    check(hb[..., :D], want, absdot, Tk)
    assert np.isnan(hb[..., D:]).all()
    assert queue.take_device_error() == 0


def test_scores_over_cache_view(ann):
    """K as a view into a larger BHTD cache (heads 1..2 of 3, the first Tk of
    Tcap positions): the K tiles come through a TMA tensor map with the cache's
    strides."""
    import torch
    B, Tq, Tk, Tcap, Hq, D = 2, 270, 300, 333, 2, 128
    g = rng(13)
    q = normal(g, (B, Tq, Hq, D), np.float32)
    kc = normal(g, (B, 3, Tcap, D), np.float32)
    k = np.ascontiguousarray(kc[:, 1:3, :Tk])
    want = oracle.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), np.float32), 1, 1)
    absdot = oracle.attention_scores(np.abs(q), np.abs(k), np.empty_like(want), 1, 1)
    s = torch.full((B, Hq, Tq, Tk), float("nan"), device="cuda")
    queue = ann.Queue()
    ann.onHost.nn.attentionScores(queue, None, dev(q), dev(kc)[:, 1:3, :Tk], s, 1, 1)
    check(host(s), want, absdot, D)
    assert queue.take_device_error() == 0


def test_apply_strided_probs(ann):
    """P as a view with padded rows (row pitch Tk + 12 floats, NaN in the pad):
    each row's bulk copy starts at its own pitch and takes Tk keys only."""
    import torch
    B, Tq, Tk, Hq, D = 2, 200, 324, 2, 64
    g = rng(11)
    p = normal(g, (B, Hq, Tq, Tk), np.float32)
    v = normal(g, (B, Tk, Hq, D), np.float32)
    want = oracle.attention_apply(p, v, np.empty((B, Tq, Hq, D), np.float32), 1, 0)
    absdot = oracle.attention_apply(np.abs(p), np.abs(v), np.empty_like(want), 1, 0)
    big = torch.full((B, Hq, Tq, Tk + 12), float("nan"), device="cuda")
    big[..., :Tk] = dev(p)
    o = torch.full((B, Tq, Hq, D), float("nan"), device="cuda")
    queue = ann.Queue()
    ann.onHost.nn.attentionApply(queue, None, big[..., :Tk], dev(v), o)
    check(host(o), want, absdot, Tk)
    assert queue.take_device_error() == 0


def test_apply_split_is_deterministic(ann):
    """The two halves of the key range add into the output in either order:
    repeated calls give identical bits."""
    import torch
    g = rng(5)
    B, Tq, Tk, Hq, D = 1, 512, 4096, 2, 128
    p = dev(normal(g, (B, Hq, Tq, Tk), np.float32))
    v = dev(normal(g, (B, Tk, Hq, D), np.float32))
    outs = []
    for _ in range(3):
        o = torch.empty((B, Tq, Hq, D), device="cuda")
        ann.onHost.nn.attentionApply(ann.Queue(), None, p, v, o)
        outs.append(host(o))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_fp32_pipe_kernels_still_match(ann, monkeypatch):
    """ANN_ATTENTION_OPS_SIMT=1 routes the same shapes to the FP32-pipe tiles."""
    import torch
    monkeypatch.setenv("ANN_ATTENTION_OPS_SIMT", "1")
    g = rng(9)
    B, Tq, Tk, Hq, D = 1, 300, 388, 3, 64
    q, k = normal(g, (B, Tq, Hq, D), np.float32), normal(g, (B, Tk, Hq, D), np.float32)
    want = oracle.attention_scores(q, k, np.empty((B, Hq, Tq, Tk), np.float32), 1, 0)
    absdot = oracle.attention_scores(np.abs(q), np.abs(k), np.empty_like(want), 1, 0)
    s = torch.empty((B, Hq, Tq, Tk), device="cuda")
    ann.onHost.nn.attentionScores(ann.Queue(), None, dev(q), dev(k), s)
    check(host(s), want, absdot, D)
