"""Generate tests/golden/reference_cases.json from the reference's own tests.

Every case below restates one hot-path test of alpakaNN's test suite
(test/unit/nn/{attention,softmax,rope,rms_norm,embedding}.cpp): the same
input fill formulas, and expected values computed by the test's own host
loops (not by the kernels), in the test's element type with the test's
operation order. Literal known answers from the tests are stored as given.
The tolerance each test uses (testHelper/test.hpp:47-54, Catch::Approx with
epsilon/margin) travels with each case.

The reference cannot be compiled here (alpaka3 is fetched over the network at
configure time), so these fixtures are how the CPU oracle is pinned: the
oracle restates the onAcc kernels, these restate the tests' host references,
and tests/test_oracle_golden.py checks one against the other.

Run: python tests/golden/make_golden.py   (deterministic; no randomness)
"""
import json
import math
import os

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_cases.json")


def fill4d(shape, base, T):
    # test/unit/nn/attention.cpp:24-28: base + T(101*i0 + 17*i1 + 7*i2 + 3*i3)
    a = np.empty(shape, dtype=T)
    for idx in np.ndindex(*shape):
        a[idx] = T(base) + T(idx[0] * 101 + idx[1] * 17 + idx[2] * 7 + idx[3] * 3)
    return a


def ref_scores(q, k, g, layout, T):
    # attention.cpp:30-66 referenceScoresBTHD / referenceScoresBHTD
    B, Tq, Hq, D = q.shape
    Tk = k.shape[1] if layout == 0 else k.shape[2]
    s = np.empty((B, Hq, Tq, Tk), dtype=T)
    for b, h, i, j in np.ndindex(B, Hq, Tq, Tk):
        kvh = h // g
        acc = T(0)
        for d in range(D):
            kk = k[b, j, kvh, d] if layout == 0 else k[b, kvh, j, d]
            acc = T(acc + T(q[b, i, h, d] * kk))
        s[b, h, i, j] = acc
    return s


def ref_apply(p, v, g, layout, T):
    # attention.cpp:68-106 referenceApplyBHTD / referenceApplyBTHD
    B, Hq, Tq, Tk = p.shape
    D = v.shape[3]
    o = np.empty((B, Tq, Hq, D), dtype=T)
    for b, i, h, d in np.ndindex(B, Tq, Hq, D):
        kvh = h // g
        acc = T(0)
        for j in range(Tk):
            vv = v[b, j, kvh, d] if layout == 0 else v[b, kvh, j, d]
            acc = T(acc + T(p[b, h, i, j] * vv))
        o[b, i, h, d] = acc
    return o


def ref_scale(s, f, T):
    # attention.cpp:108-113 scaleTensor
    out = s.copy()
    for idx in np.ndindex(*s.shape):
        out[idx] = T(s[idx] * T(f))
    return out


def ref_softmax(x, causal, T):
    # attention.cpp:115-174 and softmax.cpp:20-83 (max from -inf, exp, /= sum)
    out = np.empty_like(x)
    B, H, Q, K = x.shape
    for b, h, q in np.ndindex(B, H, Q):
        last = q if causal else K - 1
        m = T(-np.inf)
        for k in range(last + 1):
            m = max(m, x[b, h, q, k])
        s = T(0)
        for k in range(K):
            if causal and k > q:
                out[b, h, q, k] = T(0)
                continue
            e = T(np.exp(T(x[b, h, q, k] - m)))
            out[b, h, q, k] = e
            s = T(s + e)
        for k in range(last + 1):
            out[b, h, q, k] = T(out[b, h, q, k] / s)
    return out


def arr(a):
    return {"dtype": str(a.dtype), "shape": list(a.shape), "data": [float(x) if a.dtype.kind == "f" else int(x)
                                                                    for x in a.reshape(-1)]}


def cases_for(T):
    tn = "f32" if T == np.float32 else "f64"
    out = []

    # attention.cpp:179-217 -- determinism/finiteness
    shape = (1, 2, 1, 2)
    q = np.empty(shape, T); k = np.empty(shape, T); v = np.empty(shape, T)
    for idx in np.ndindex(*shape):
        q[idx] = T(idx[1] + idx[3] + 1)
        k[idx] = T(idx[1] + idx[3] + 2)
        v[idx] = T(idx[1] * 2 + idx[3] + 1)
    out.append({"name": f"attention_determinism_{tn}", "op": "pipeline_finite", "source": "nn/attention.cpp:179-236",
                "q": arr(q), "k": arr(k), "v": arr(v), "scores_shape": [1, 1, 2, 2]})

    # attention.cpp:240-309 -- grouped query heads, literal known answers
    q = np.zeros((1, 1, 4, 2), T)
    for h in range(4):
        q[0, 0, h, 0] = T(h + 1); q[0, 0, h, 1] = T(h + 2)
    k = np.array([[[[1, 2], [3, 4]]]], T)
    v = np.array([[[[10, 20], [30, 40]]]], T)
    out.append({"name": f"attention_gqa_{tn}", "op": "gqa", "source": "nn/attention.cpp:240-309",
                "q": arr(q), "k": arr(k), "v": arr(v), "g": 2, "layout": 0,
                "expected_scores": arr(np.array([5, 8, 25, 32], T).reshape(1, 4, 1, 1)),
                "expected_out": arr(np.array([10, 20, 10, 20, 30, 40, 30, 40], T).reshape(1, 1, 4, 2)),
                "eps": 1e-5, "margin": 1e-6})

    # attention.cpp:332-364 -- scores, prefill BTHD
    q = fill4d((1, 4, 4, 4), 0.25, T); k = fill4d((1, 4, 4, 4), -0.5, T)
    out.append({"name": f"scores_prefill_{tn}", "op": "scores", "source": "nn/attention.cpp:332-364",
                "q": arr(q), "k": arr(k), "g": 1, "layout": 0, "prefill_value": -999.0,
                "expected": arr(ref_scores(q, k, 1, 0, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:390-423 -- scores, decode BHTD
    q = fill4d((1, 1, 4, 4), 0.75, T); k = fill4d((1, 4, 5, 4), -0.125, T)
    out.append({"name": f"scores_decode_{tn}", "op": "scores", "source": "nn/attention.cpp:390-423",
                "q": arr(q), "k": arr(k), "g": 1, "layout": 1, "prefill_value": -777.0,
                "expected": arr(ref_scores(q, k, 1, 1, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:448-491 -- apply, decode BHTD
    probs = np.zeros((1, 4, 1, 5), T)
    for h in range(4):
        norm = T(0)
        for key in range(5):
            val = T((h + 1) * (key + 2)); probs[0, h, 0, key] = val; norm = T(norm + val)
        for key in range(5):
            probs[0, h, 0, key] = T(probs[0, h, 0, key] / norm)
    values = fill4d((1, 4, 5, 4), 1.25, T)
    out.append({"name": f"apply_decode_{tn}", "op": "apply", "source": "nn/attention.cpp:448-491",
                "probs": arr(probs), "v": arr(values), "g": 1, "layout": 1, "prefill_value": -555.0,
                "expected": arr(ref_apply(probs, values, 1, 1, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:517-563 -- apply, prefill BTHD with causal probabilities
    probs = np.zeros((1, 4, 4, 4), T)
    for qq in range(4):
        for h in range(4):
            norm = T(0)
            for key in range(4):
                val = T((qq + 1) * (h + 2) * (key + 1)) if key <= qq else T(0)
                probs[0, h, qq, key] = val; norm = T(norm + val)
            for key in range(4):
                probs[0, h, qq, key] = T(probs[0, h, qq, key] / norm) if norm > T(0) else T(0)
    values = fill4d((1, 4, 4, 4), 1.0, T)
    out.append({"name": f"apply_prefill_{tn}", "op": "apply", "source": "nn/attention.cpp:517-563",
                "probs": arr(probs), "v": arr(values), "g": 1, "layout": 0, "prefill_value": -444.0,
                "expected": arr(ref_apply(probs, values, 1, 0, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:591-651 -- prefill pipeline: scores -> scale 0.5 -> causalSoftmax -> apply (BTHD)
    q = fill4d((1, 4, 4, 4), 0.125, T); k = fill4d((1, 4, 4, 4), -0.25, T); v = fill4d((1, 4, 4, 4), 0.5, T)
    es = ref_scale(ref_scores(q, k, 1, 0, T), 0.5, T)
    ep = ref_softmax(es, True, T)
    out.append({"name": f"pipeline_prefill_{tn}", "op": "pipeline", "source": "nn/attention.cpp:591-651",
                "q": arr(q), "k": arr(k), "v": arr(v), "g": 1, "layout": 0, "scale": 0.5, "causal": True,
                "expected_scores": arr(es), "expected_probs": arr(ep),
                "expected_out": arr(ref_apply(ep, v, 1, 0, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:674-734 -- decode pipeline: scores(BHTD) -> scale 0.5 -> softmax -> apply
    q = fill4d((1, 1, 4, 4), 0.375, T); k = fill4d((1, 4, 5, 4), -0.0625, T); v = fill4d((1, 4, 5, 4), 0.875, T)
    es = ref_scale(ref_scores(q, k, 1, 1, T), 0.5, T)
    ep = ref_softmax(es, False, T)
    out.append({"name": f"pipeline_decode_{tn}", "op": "pipeline", "source": "nn/attention.cpp:674-734",
                "q": arr(q), "k": arr(k), "v": arr(v), "g": 1, "layout": 1, "scale": 0.5, "causal": False,
                "expected_scores": arr(es), "expected_probs": arr(ep),
                "expected_out": arr(ref_apply(ep, v, 1, 1, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:757-835 -- explicit BTHD -> BHTD cache assembly, then the decode pipeline
    q = fill4d((1, 1, 4, 4), 0.375, T)
    kt = fill4d((1, 5, 4, 4), -0.0625, T); vt = fill4d((1, 5, 4, 4), 0.875, T)
    kb = np.ascontiguousarray(kt.transpose(0, 2, 1, 3)); vb = np.ascontiguousarray(vt.transpose(0, 2, 1, 3))
    es = ref_scale(ref_scores(q, kb, 1, 1, T), 0.5, T)
    ep = ref_softmax(es, False, T)
    out.append({"name": f"pipeline_bhtd_assembly_{tn}", "op": "pipeline", "source": "nn/attention.cpp:757-835",
                "q": arr(q), "k": arr(kb), "v": arr(vb), "g": 1, "layout": 1, "scale": 0.5, "causal": False,
                "expected_scores": arr(es), "expected_probs": arr(ep),
                "expected_out": arr(ref_apply(ep, vb, 1, 1, T)), "eps": 1e-5, "margin": 1e-5})

    # attention.cpp:852-975 -- qkvProjection + ropeInPlace(q, k) with flat buffers viewed 2-D and 4-D
    tokens, heads, hd = 3, 1, 4
    hidden, pairs = heads * hd, hd // 2
    x = np.empty((tokens, hidden), T)
    for r, c in np.ndindex(tokens, hidden):
        x[r, c] = T(T(-0.25) + T(T(r * 13 + c * 3) * T(0.05)))
    wq = np.empty((hidden, hidden), T); wk = np.empty_like(wq); wv = np.empty_like(wq)
    for r, c in np.ndindex(hidden, hidden):
        flat = T(r * hidden + c)
        wq[r, c] = T(T(-0.1) + T(flat * T(0.01)))
        wk[r, c] = T(T(0.2) - T(flat * T(0.007)))
        wv[r, c] = T(T(-0.05) + T(flat * T(0.009)))

    def proj(w):
        e = np.empty((tokens, hidden), T)
        for r, c in np.ndindex(tokens, hidden):
            acc = T(0)
            for inner in range(hidden):
                acc = T(acc + T(x[r, inner] * w[inner, c]))
            e[r, c] = acc
        return e

    cos = np.empty((tokens, pairs), T); sin = np.empty((tokens, pairs), T)
    for pos, pr in np.ndindex(tokens, pairs):
        ang = T(T(T(pos + 1) * T(0.25)) * T(pr + 1))
        cos[pos, pr] = T(math.cos(float(ang))) if T == np.float64 else np.float32(np.cos(ang))
        sin[pos, pr] = T(math.sin(float(ang))) if T == np.float64 else np.float32(np.sin(ang))

    def rope2d(pm):
        e = np.empty_like(pm)
        for t, pr in np.ndindex(tokens, pairs):
            c, s = cos[t, pr], sin[t, pr]
            x0, x1 = pm[t, 2 * pr], pm[t, 2 * pr + 1]
            e[t, 2 * pr] = T(T(x0 * c) - T(x1 * s))
            e[t, 2 * pr + 1] = T(T(x0 * s) + T(x1 * c))
        return e

    rq, rk, rv = proj(wq), proj(wk), proj(wv)
    out.append({"name": f"qkv_rope_{tn}", "op": "qkv_rope", "source": "nn/attention.cpp:852-975",
                "x": arr(x), "wq": arr(wq), "wk": arr(wk), "wv": arr(wv), "cos": arr(cos), "sin": arr(sin),
                "tokens": tokens, "heads": heads, "head_dim": hd,
                "expected_q": arr(rope2d(rq)), "expected_k": arr(rope2d(rk)), "expected_v": arr(rv),
                "eps": 1e-5, "margin": 1e-5})

    # softmax.cpp:88-114 -- stability with large logits, causal; literal properties
    x = np.array([1000, 1001, 999, -1, 0, 1], T).reshape(1, 1, 2, 3)
    out.append({"name": f"softmax_stability_{tn}", "op": "softmax_stability", "source": "nn/softmax.cpp:88-114",
                "x": arr(x), "zero_at": [[0, 0, 0, 1], [0, 0, 0, 2]], "row_sums": [1.0, 1.0],
                "eps": 1e-5, "margin": 1e-6})

    # softmax.cpp:116-139 -- causalSoftmax, prefill shape
    x = np.empty((1, 4, 4, 4), T)
    for idx in np.ndindex(*x.shape):
        x[idx] = T(T(idx[0] * 97 + idx[1] * 23 + idx[2] * 11 + idx[3] * 5) * T(0.03125))
    out.append({"name": f"causal_softmax_prefill_{tn}", "op": "causal_softmax", "source": "nn/softmax.cpp:116-139",
                "x": arr(x), "axis": 3, "query_axis": 2, "key_axis": 3, "prefill_value": -123.0,
                "expected": arr(ref_softmax(x, True, T)), "eps": 1e-5, "margin": 1e-5})

    # softmax.cpp:141-165 -- softmax, decode shape
    x = np.empty((1, 4, 1, 6), T)
    for idx in np.ndindex(*x.shape):
        x[idx] = T(T(T(idx[0] * 97 + idx[1] * 29 + idx[2] * 13 + idx[3] * 3) * T(0.0625)) - T(0.5))
    out.append({"name": f"softmax_decode_{tn}", "op": "softmax", "source": "nn/softmax.cpp:141-165",
                "x": arr(x), "axis": 3, "prefill_value": -321.0,
                "expected": arr(ref_softmax(x, False, T)), "eps": 1e-5, "margin": 1e-5})

    # rope.cpp:20-82 -- pairwise rotation known answer (q checked by the test; k by the same formula)
    q = np.empty((1, 2, 1, 4), T)
    for idx in np.ndindex(*q.shape):
        q[idx] = T(idx[1] * 10 + idx[3] + 1)
    k = (q + T(1)).astype(T)
    cos = np.empty((2, 2), T); sin = np.empty((2, 2), T)
    for pos, pr in np.ndindex(2, 2):
        ang = T(T(pos + pr + 1) * T(0.25))
        cos[pos, pr] = T(math.cos(float(ang))) if T == np.float64 else np.float32(np.cos(ang))
        sin[pos, pr] = T(math.sin(float(ang))) if T == np.float64 else np.float32(np.sin(ang))

    def rope4(a):
        e = np.empty_like(a)
        for t, pr in np.ndindex(a.shape[1], 2):
            for h in range(a.shape[2]):
                c, s = cos[t, pr], sin[t, pr]
                x0, x1 = a[0, t, h, 2 * pr], a[0, t, h, 2 * pr + 1]
                e[0, t, h, 2 * pr] = T(T(x0 * c) - T(x1 * s))
                e[0, t, h, 2 * pr + 1] = T(T(x0 * s) + T(x1 * c))
        return e

    tol = 1e-5 if T == np.float32 else 1e-12
    out.append({"name": f"rope_pairwise_{tn}", "op": "rope_qk", "source": "nn/rope.cpp:20-82",
                "q": arr(q), "k": arr(k), "cos": arr(cos), "sin": arr(sin), "layout": 0, "position_offset": 0,
                "expected_q": arr(rope4(q)), "expected_k": arr(rope4(k)), "eps": tol, "margin": tol})

    # rope.cpp:105-146 -- q and k with different head counts (the test checks finiteness)
    q = np.empty((1, 2, 2, 4), T); k = np.empty((1, 2, 1, 4), T)
    for idx in np.ndindex(*q.shape):
        q[idx] = T(idx[1] * 100 + idx[2] * 10 + idx[3] + 1)
    for idx in np.ndindex(*k.shape):
        k[idx] = T(idx[1] * 100 + idx[3] + 2)
    for pos, pr in np.ndindex(2, 2):
        ang = T(T(pos + pr + 1) * T(0.2))
        cos[pos, pr] = T(math.cos(float(ang))) if T == np.float64 else np.float32(np.cos(ang))
        sin[pos, pr] = T(math.sin(float(ang))) if T == np.float64 else np.float32(np.sin(ang))
    out.append({"name": f"rope_gqa_heads_{tn}", "op": "rope_qk", "source": "nn/rope.cpp:105-146",
                "q": arr(q), "k": arr(k), "cos": arr(cos.copy()), "sin": arr(sin.copy()), "layout": 0,
                "position_offset": 0, "expected_q": arr(rope4(q)), "expected_k": arr(rope4(k)),
                "eps": tol, "margin": tol})

    # rms_norm.cpp:18-48 -- [2,4], eps 1e-5, x * (1/sqrt(mean + eps)) * w
    x = np.empty((2, 4), T)
    for r, c in np.ndindex(2, 4):
        x[r, c] = T(r * 4 + c + 1)
    w = np.array([T(T(0.5) + T(i)) for i in range(4)], T)
    e = np.empty_like(x)
    for r in range(2):
        ss = T(0)
        for c in range(4):
            ss = T(ss + T(x[r, c] * x[r, c]))
        inv = T(T(1) / T(np.sqrt(T(T(ss / T(4)) + T(1e-5)))))
        for c in range(4):
            e[r, c] = T(T(x[r, c] * inv) * w[c])
    out.append({"name": f"rms_norm_{tn}", "op": "rms_norm", "source": "nn/rms_norm.cpp:18-48",
                "x": arr(x), "w": arr(w), "epsilon": 1e-5, "expected": arr(e), "eps": 1e-5, "margin": 1e-6})

    # embedding.cpp:20-53 -- gather
    table = np.empty((4, 3), T)
    for r, c in np.ndindex(4, 3):
        table[r, c] = T(r * 10 + c)
    ids = np.array([3, 0, 2, 1, 3], np.uint32)
    out.append({"name": f"embedding_gather_{tn}", "op": "embedding", "source": "nn/embedding.cpp:20-53",
                "table": arr(table), "ids": arr(ids), "col_offset": 0, "hidden": 3,
                "expected": arr(table[ids]), "eps": 1e-5, "margin": 1e-6})

    # embedding.cpp:55-95 -- non-contiguous subview of a wider storage (pitch 5, column offset 2)
    storage = np.empty((3, 5), T)
    for r, c in np.ndindex(3, 5):
        storage[r, c] = T(r * 10 + c)
    ids = np.array([2, 0, 1, 2], np.uint32)
    out.append({"name": f"embedding_subview_{tn}", "op": "embedding", "source": "nn/embedding.cpp:55-95",
                "table": arr(storage), "ids": arr(ids), "col_offset": 2, "hidden": 2,
                "expected": arr(storage[:, 2:4][ids]), "eps": 1e-5, "margin": 1e-6})

    # embedding.cpp:134-170 -- shape and rank validation (throws std::invalid_argument)
    out.append({"name": f"embedding_validation_{tn}", "op": "embedding_validation",
                "source": "nn/embedding.cpp:134-170", "ids_shape": [2], "table_shape": [3, 4],
                "valid_out": [2, 4], "invalid_outs": [[3, 4], [2, 5], [2, 4, 1]]})
    return out


def main():
    cases = cases_for(np.float32) + cases_for(np.float64)
    with open(OUT, "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "cases": cases}, f, indent=None, separators=(",", ":"))
        f.write("\n")
    print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
    main()
