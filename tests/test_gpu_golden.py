"""The reference test-suite's hot-path cases (tests/golden), run through the
drop-in API on the GPU, with each test's own tolerance."""
import numpy as np
import pytest

from tests.helpers import arr, assert_approx, load_cases

pytestmark = pytest.mark.gpu

CASES = load_cases()


def by_op(*ops):
    return [pytest.param(c, id=c["name"]) for c in CASES if c["op"] in ops]


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
    return t.cpu().numpy()


@pytest.mark.parametrize("c", by_op("pipeline"))
def test_pipeline(ann, c):
    import torch
    nn, ops = ann.onHost.nn, ann.onHost.ops
    q, k, v = dev(arr(c["q"])), dev(arr(c["k"])), dev(arr(c["v"]))
    T = q.dtype
    Tk = k.shape[1] if c["layout"] == 0 else k.shape[2]
    scores = torch.empty((q.shape[0], q.shape[2], q.shape[1], Tk), dtype=T, device="cuda")
    probs = torch.empty_like(scores)
    out = torch.empty_like(q)
    queue = ann.Queue()
    nn.attentionScores(queue, None, q, k, scores, c["g"], c["layout"])
    ops.scale(queue, None, scores, c["scale"], scores)
    if c["causal"]:
        nn.causalSoftmax(queue, None, scores, probs, 3, 2, 3)
    else:
        nn.softmax(queue, None, scores, probs, 3)
    nn.attentionApply(queue, None, probs, v, out, c["g"], c["layout"])
    assert_approx(host(scores), arr(c["expected_scores"]), c["eps"], c["margin"], "scores")
    assert_approx(host(probs), arr(c["expected_probs"]), c["eps"], c["margin"], "probs")
    assert_approx(host(out), arr(c["expected_out"]), c["eps"], c["margin"], "out")
    if not c["causal"] and k.shape[3] in (64, 128):
        pass  # fused decode is covered by test_gpu_parity with supported head sizes


@pytest.mark.parametrize("c", by_op("pipeline_finite"))
def test_determinism_finite(ann, c):
    import torch
    nn = ann.onHost.nn
    q, k, v = dev(arr(c["q"])), dev(arr(c["k"])), dev(arr(c["v"]))
    s = torch.empty(c["scores_shape"], dtype=q.dtype, device="cuda")
    p, o = torch.empty_like(s), torch.empty_like(q)
    queue = ann.Queue()
    nn.attentionScores(queue, None, q, k, s)
    nn.softmax(queue, None, s, p, 3)
    nn.attentionApply(queue, None, p, v, o)
    s1, o1 = host(s), host(o)
    assert np.isfinite(s1).all() and np.isfinite(o1).all()
    nn.attentionScores(queue, None, q, k, s)
    nn.softmax(queue, None, s, p, 3)
    nn.attentionApply(queue, None, p, v, o)
    assert np.array_equal(s1, host(s)) and np.array_equal(o1, host(o))


@pytest.mark.parametrize("c", by_op("gqa"))
def test_gqa_known_answers(ann, c):
    import torch
    nn = ann.onHost.nn
    q, k, v = dev(arr(c["q"])), dev(arr(c["k"])), dev(arr(c["v"]))
    s = torch.empty((1, 4, 1, 1), dtype=q.dtype, device="cuda")
    p, o = torch.empty_like(s), torch.empty_like(q)
    queue = ann.Queue()
    nn.attentionScores(queue, None, q, k, s, 2, ann.AttentionKvLayout.BTHD)
    nn.softmax(queue, None, s, p, 3)
    nn.attentionApply(queue, None, p, v, o, 2, ann.AttentionKvLayout.BTHD)
    assert_approx(host(s), arr(c["expected_scores"]), c["eps"], c["margin"], "scores")
    assert_approx(host(o), arr(c["expected_out"]), c["eps"], c["margin"], "out")


@pytest.mark.parametrize("c", by_op("scores"))
def test_scores(ann, c):
    import torch
    e = arr(c["expected"])
    s = torch.full(e.shape, c["prefill_value"], dtype=dev(e).dtype, device="cuda")
    ann.onHost.nn.attentionScores(ann.Queue(), None, dev(arr(c["q"])), dev(arr(c["k"])), s, c["g"], c["layout"])
    assert_approx(host(s), e, c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("apply"))
def test_apply(ann, c):
    import torch
    e = arr(c["expected"])
    o = torch.full(e.shape, c["prefill_value"], dtype=dev(e).dtype, device="cuda")
    ann.onHost.nn.attentionApply(ann.Queue(), None, dev(arr(c["probs"])), dev(arr(c["v"])), o, c["g"], c["layout"])
    assert_approx(host(o), e, c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("softmax", "causal_softmax"))
def test_softmax(ann, c):
    import torch
    x = dev(arr(c["x"]))
    out = torch.full_like(x, c["prefill_value"])
    if c["op"] == "softmax":
        ann.onHost.nn.softmax(ann.Queue(), None, x, out, c["axis"])
    else:
        ann.onHost.nn.causalSoftmax(ann.Queue(), None, x, out, c["axis"], c["query_axis"], c["key_axis"])
    assert_approx(host(out), arr(c["expected"]), c["eps"], c["margin"], c["name"])


@pytest.mark.parametrize("c", by_op("softmax_stability"))
def test_softmax_stability(ann, c):
    import torch
    x = dev(arr(c["x"]))
    out = torch.empty_like(x)
    ann.onHost.nn.causalSoftmax(ann.Queue(), None, x, out, 3, 2, 3)
    o = host(out)
    for z in c["zero_at"]:
        assert o[tuple(z)] == 0
    sums = np.array([o[0, 0, 0, 0], o[0, 0, 1, :].sum(dtype=o.dtype)])
    assert_approx(sums, np.array(c["row_sums"]), c["eps"], c["margin"], "row sums")


@pytest.mark.parametrize("c", by_op("rope_qk"))
def test_rope(ann, c):
    import torch
    q, k, cs, sn = dev(arr(c["q"])), dev(arr(c["k"])), dev(arr(c["cos"])), dev(arr(c["sin"]))
    oq, ok = torch.empty_like(q), torch.empty_like(k)
    ann.onHost.nn.rope(ann.Queue(), None, q, k, cs, sn, oq, ok)
    assert_approx(host(oq), arr(c["expected_q"]), c["eps"], c["margin"], "q")
    assert_approx(host(ok), arr(c["expected_k"]), c["eps"], c["margin"], "k")
    # in place, both tensors in one launch
    ann.onHost.nn.ropeInPlace(ann.Queue(), None, q, k, cs, sn)
    assert np.array_equal(host(q), host(oq)) and np.array_equal(host(k), host(ok))


@pytest.mark.parametrize("c", by_op("qkv_rope"))
def test_qkv_rope(ann, c):
    import torch
    nn = ann.onHost.nn
    x = dev(arr(c["x"]))
    t, h, d = c["tokens"], c["heads"], c["head_dim"]
    # flat buffers viewed 2-D for the projection and 4-D for RoPE (attention.cpp:941-953)
    flats = [torch.empty(t * h * d, dtype=x.dtype, device="cuda") for _ in range(3)]
    q2, k2, v2 = (f.view(t, h * d) for f in flats)
    nn.qkvProjection(ann.Queue(), x, dev(arr(c["wq"])), dev(arr(c["wk"])), dev(arr(c["wv"])), q2, k2, v2)
    q4, k4 = flats[0].view(1, t, h, d), flats[1].view(1, t, h, d)
    nn.ropeInPlace(ann.Queue(), None, q4, k4, dev(arr(c["cos"])), dev(arr(c["sin"])))
    assert_approx(host(q2), arr(c["expected_q"]), c["eps"], c["margin"], "q")
    assert_approx(host(k2), arr(c["expected_k"]), c["eps"], c["margin"], "k")
    assert_approx(host(v2), arr(c["expected_v"]), c["eps"], c["margin"], "v")


@pytest.mark.parametrize("c", by_op("rms_norm"))
def test_rms_norm(ann, c):
    import torch
    x = dev(arr(c["x"]))
    out = torch.empty_like(x)
    ann.onHost.nn.rmsNorm(ann.Queue(), None, x, dev(arr(c["w"])), out, c["epsilon"])
    assert_approx(host(out), arr(c["expected"]), c["eps"], c["margin"], "rmsNorm")


@pytest.mark.parametrize("c", by_op("embedding"))
def test_embedding(ann, c):
    import torch
    storage = dev(arr(c["table"]))
    table = storage[:, c["col_offset"]:c["col_offset"] + c["hidden"]]  # device subview with row pitch
    ids = dev(arr(c["ids"]))
    out = torch.empty((ids.shape[0], c["hidden"]), dtype=storage.dtype, device="cuda")
    ann.onHost.nn.embeddingLookup(ann.Queue(), None, ids, table, out)
    assert np.array_equal(host(out), arr(c["expected"]))


@pytest.mark.parametrize("c", by_op("embedding_validation"))
def test_embedding_validation(ann, c):
    import torch
    T = torch.float32 if c["name"].endswith("f32") else torch.float64
    ids = torch.zeros(c["ids_shape"], dtype=torch.int32, device="cuda")
    table = torch.ones(c["table_shape"], dtype=T, device="cuda")
    ok = torch.empty(c["valid_out"], dtype=T, device="cuda")
    ann.onHost.nn.embeddingLookup(ann.Queue(), None, ids, table, ok)  # REQUIRE_NOTHROW
    torch.cuda.synchronize()
    for shape in c["invalid_outs"]:
        with pytest.raises(ValueError):
            ann.onHost.nn.embeddingLookup(ann.Queue(), None, ids, table,
                                          torch.empty(shape, dtype=T, device="cuda"))
