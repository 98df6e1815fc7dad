"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects on the host exactly the shapes on which the
reference throws std::invalid_argument (no compute call is made: every call
here fails validation before anything is enqueued)."""
import ctypes
import os
import re

import numpy as np
import pytest

from tests.helpers import load_cases

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def capi():
    from tests.helpers import build_library
    build_library()
    from alpakann_b200 import _capi
    return _capi


def header_symbols():
    syms = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            syms |= set(re.findall(r"\b(ann_\w+)\s*\(", text))
    return syms


def test_exports_every_declared_symbol(capi):
    syms = header_symbols()
    assert len(syms) >= 27
    for s in sorted(syms):
        assert hasattr(capi.lib, s), f"{s} declared in include/ but not exported"
    # the ctypes table covers exactly the declared API
    assert syms == set(capi.SIGNATURES), sorted(syms ^ set(capi.SIGNATURES))


def test_version_and_error_string(capi):
    assert capi.lib.ann_version() == 100
    assert isinstance(capi.lib.ann_last_error(), bytes)


def _call_einval(capi, fn, *args):
    rc = fn(None, *args)
    assert rc == capi.ANN_EINVAL, capi.lib.ann_last_error()
    return capi.lib.ann_last_error().decode()


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_embedding_validation(capi, sfx, T):
    # nn/embedding.cpp:134-170: wrong rows, wrong cols, wrong rank all throw
    case = [c for c in load_cases() if c["op"] == "embedding_validation"][0]
    ids = np.zeros(case["ids_shape"], np.uint32)
    table = np.ones(case["table_shape"], T)
    f = getattr(capi.lib, f"ann_embedding_lookup_{sfx}")
    for shape in case["invalid_outs"]:
        out = np.zeros(shape, T)
        msg = _call_einval(capi, f, capi.ref(ids), capi.ref(table), capi.ref(out))
        assert "embeddingLookup" in msg
    # 2-D ids
    msg = _call_einval(capi, f, capi.ref(np.zeros((2, 1), np.uint32)), capi.ref(table),
                       capi.ref(np.zeros((2, 4), T)))
    assert msg == "embeddingLookup expects 1D ids and 2D embedding/output."


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_rms_norm_validation(capi, sfx, T):
    f = getattr(capi.lib, f"ann_rms_norm_{sfx}")
    x = np.ones((2, 4), T)
    assert _call_einval(capi, f, capi.ref(x), capi.ref(np.ones(4, T)), capi.ref(np.ones((2, 5), T)),
                        1e-5) == "rmsNorm shape mismatch."
    assert _call_einval(capi, f, capi.ref(x), capi.ref(np.ones(3, T)), capi.ref(np.ones((2, 4), T)),
                        1e-5) == "rmsNorm expects a 1D weight matching the last axis."
    assert _call_einval(capi, f, capi.ref(x), capi.ref(np.ones((1, 4), T)), capi.ref(np.ones((2, 4), T)),
                        1e-5) == "rmsNorm expects a 1D weight matching the last axis."


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_rope_validation(capi, sfx, T):
    # validateRopeShape, onHost/nn/rope.hpp:21-46
    f = getattr(capi.lib, f"ann_rope_{sfx}")
    x = np.ones((1, 3, 2, 4), T)
    c = np.ones((3, 2), T)
    r = capi.ref
    assert _call_einval(capi, f, r(x), r(c), r(c), r(np.ones((1, 3, 2, 6), T)), 0, 0) == "rope shape mismatch."
    odd = np.ones((1, 3, 2, 3), T)
    assert _call_einval(capi, f, r(odd), r(c), r(c), r(odd), 0, 0) == "rope requires an even head dimension."
    assert _call_einval(capi, f, r(x), r(c), r(np.ones((4, 2), T)), r(x), 0, 0) == \
        "rope cosine/sine table shape mismatch."
    c3 = np.ones((3, 3), T)
    assert _call_einval(capi, f, r(x), r(c3), r(c3), r(x), 0, 0) == "rope table pair count mismatch."
    assert _call_einval(capi, f, r(x), r(c), r(c), r(x), 0, 1) == "rope table does not cover requested positions."
    # BHTD: coverage is checked on the token axis (axis 2)
    xb = np.ones((1, 2, 4, 4), T)
    assert _call_einval(capi, f, r(xb), r(c), r(c), r(xb), 1, 0) == \
        "rope table does not cover requested positions."
    fi = getattr(capi.lib, f"ann_rope_inplace_{sfx}")
    kbad = np.ones((1, 4, 1, 4), T)  # 4 tokens, table covers 3
    assert _call_einval(capi, fi, r(x), r(kbad), r(c), r(c), 0, 0) == \
        "rope table does not cover requested positions."


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_attention_validation(capi, sfx, T):
    r = capi.ref
    q = np.ones((1, 4, 4, 4), T)
    s = np.ones((1, 4, 4, 4), T)
    fs = getattr(capi.lib, f"ann_attention_scores_{sfx}")
    fa = getattr(capi.lib, f"ann_attention_apply_{sfx}")
    # attention.hpp:64-65 / :93-94
    assert _call_einval(capi, fs, r(q), r(q), r(s), 0, 0) == "attentionScores requires queriesPerKvGroup > 0."
    assert _call_einval(capi, fa, r(s), r(q), r(q), 0, 0) == "attentionApply requires queriesPerKvGroup > 0."
    # reads the reference would make out of bounds
    assert "do not cover" in _call_einval(capi, fs, r(q), r(np.ones((1, 3, 4, 4), T)), r(s), 1, 0)
    assert "do not cover" in _call_einval(capi, fa, r(s), r(np.ones((1, 3, 4, 4), T)), r(q), 1, 0)


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_softmax_and_scale_validation(capi, sfx, T):
    r = capi.ref
    x = np.ones((1, 4, 4, 4), T)
    y = np.ones((1, 4, 4, 5), T)
    assert _call_einval(capi, getattr(capi.lib, f"ann_softmax_{sfx}"), r(x), r(y), 3) == "softmax shape mismatch."
    assert _call_einval(capi, getattr(capi.lib, f"ann_causal_softmax_{sfx}"), r(x), r(y), 3, 2, 3) == \
        "softmax shape mismatch."
    assert "axis out of range" in _call_einval(capi, getattr(capi.lib, f"ann_softmax_{sfx}"), r(x), r(x), 4)
    assert _call_einval(capi, getattr(capi.lib, f"ann_scale_{sfx}"), r(x), 0.5, r(y)) == "scale shape mismatch."


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_gemm_and_decode_validation(capi, sfx, T):
    r = capi.ref
    a = np.ones((3, 4), T)
    assert _call_einval(capi, getattr(capi.lib, f"ann_gemm_{sfx}"), r(a), r(np.ones((5, 2), T)),
                        r(np.ones((3, 2), T))) == "gemm shape mismatch."
    fd = getattr(capi.lib, f"ann_attention_decode_{sfx}")
    q = np.ones((2, 1, 4, 64), T)
    kv = np.ones((2, 4, 16, 64), T)
    assert "queriesPerKvGroup > 0" in _call_einval(capi, fd, r(q), r(kv), r(kv), r(q), 0.1, 0, 1)
    assert "extents of Q" in _call_einval(capi, fd, r(q), r(kv), r(kv), r(np.ones((2, 1, 4, 32), T)), 0.1, 1, 1)
    kv3 = np.ones((3, 4, 16, 64), T)  # batch 3 against Q's batch 2
    assert "does not match" in _call_einval(capi, fd, r(q), r(kv3), r(kv3), r(q), 0.1, 1, 1)
    kvd = np.ones((2, 4, 16, 64), T)
    assert "K and V extents differ" in _call_einval(capi, fd, r(q), r(kvd), r(np.ones((2, 4, 15, 64), T)), r(q),
                                                    0.1, 1, 1)


def test_view_descriptor_rejects_bad_pitch(capi):
    v = capi.AnnView()
    x = np.ones(8, np.float32)
    v.data = x.ctypes.data
    v.rank = 1
    v.extents[0] = 4
    v.pitches[0] = 6  # not a multiple of 4 bytes
    w = np.ones(4, np.float32)
    rc = capi.lib.ann_scale_f32(None, ctypes.byref(v), 1.0, capi.ref(w))
    assert rc == capi.ANN_EINVAL
    assert b"pitch" in capi.lib.ann_last_error()


@pytest.mark.parametrize("sfx,T", [("f32", np.float32), ("f64", np.float64)])
def test_prefill_validation(capi, sfx, T):
    r = capi.ref
    fp = getattr(capi.lib, f"ann_attention_prefill_{sfx}")
    q = np.ones((1, 8, 4, 64), T)
    kv = np.ones((1, 8, 4, 64), T)
    assert "queriesPerKvGroup > 0" in _call_einval(capi, fp, r(q), r(kv), r(kv), r(q), 0.1, 0, 0, 1)
    assert "invalid kv layout" in _call_einval(capi, fp, r(q), r(kv), r(kv), r(q), 0.1, 1, 2, 1)
    assert "extents of Q" in _call_einval(capi, fp, r(q), r(kv), r(kv), r(np.ones((1, 8, 4, 32), T)), 0.1, 1, 0, 1)
    assert "does not match" in _call_einval(capi, fp, r(q), r(np.ones((1, 8, 4, 32), T)),
                                            r(np.ones((1, 8, 4, 32), T)), r(q), 0.1, 1, 0, 1)



def test_comm_argument_validation():
    """ann_comm_* reject bad arguments on the host, before NCCL is touched."""
    import ctypes

    from alpakann_b200 import _capi
    lib = _capi.lib
    uid = (ctypes.c_char * _capi.COMM_ID_BYTES)()
    h = ctypes.c_void_p()
    assert lib.ann_comm_init(ctypes.byref(h), 0, 0, ctypes.byref(uid), 10.0) == _capi.ANN_EINVAL
    assert lib.ann_comm_init(ctypes.byref(h), 2, 2, ctypes.byref(uid), 10.0) == _capi.ANN_EINVAL
    assert lib.ann_comm_init(ctypes.byref(h), 2, -1, ctypes.byref(uid), 10.0) == _capi.ANN_EINVAL
    assert lib.ann_comm_init(ctypes.byref(h), 2, 0, ctypes.byref(uid), 0.0) == _capi.ANN_EINVAL
    assert lib.ann_comm_init(None, 2, 0, ctypes.byref(uid), 10.0) == _capi.ANN_EINVAL
    assert lib.ann_comm_unique_id(None) == _capi.ANN_EINVAL
    assert lib.ann_comm_allgather(None, None, None, None, 16) == _capi.ANN_EINVAL
    assert b"null communicator" in lib.ann_last_error()
    assert lib.ann_comm_size(None, None, None) == _capi.ANN_EINVAL
    assert lib.ann_comm_destroy(None) == _capi.ANN_OK
    assert lib.ann_comm_abort(None) == _capi.ANN_OK



def test_embedding_rms_norm_validation():
    """The fused call throws on the conditions of embeddingLookup and rmsNorm."""
    import numpy as np

    from alpakann_b200 import _capi
    lib = _capi.lib
    ids = np.zeros(4, np.uint32)
    table = np.zeros((8, 16), np.float32)
    w = np.zeros(16, np.float32)
    R = _capi.ref
    assert lib.ann_embedding_rms_norm_f32(None, R(ids), R(table), R(w), R(np.zeros((4, 8), np.float32)),
                                          1e-6) == _capi.ANN_EINVAL
    assert lib.ann_embedding_rms_norm_f32(None, R(ids), R(table), R(np.zeros(8, np.float32)),
                                          R(np.zeros((4, 16), np.float32)), 1e-6) == _capi.ANN_EINVAL
    assert lib.ann_embedding_rms_norm_f32(None, R(ids.reshape(2, 2)), R(table), R(w),
                                          R(np.zeros((4, 16), np.float32)), 1e-6) == _capi.ANN_EINVAL



def test_kv_cache_append_and_residual_validation():
    """Shape checks of the KV-cache append and the residual projection, before any launch."""
    import numpy as np

    from alpakann_b200 import _capi
    lib, R = _capi.lib, _capi.ref
    kn = np.zeros((2, 3, 4, 8), np.float32)
    kc = np.zeros((2, 4, 10, 8), np.float32)
    assert lib.ann_kv_cache_append_f32(None, R(kn), R(kn), R(kc), R(kc), None, None, 8) == _capi.ANN_EINVAL
    assert b"capacity" in lib.ann_last_error()
    bad = np.zeros((2, 5, 10, 8), np.float32)  # kv heads differ
    assert lib.ann_kv_cache_append_f32(None, R(kn), R(kn), R(bad), R(bad), None, None, 0) == _capi.ANN_EINVAL
    tab = np.zeros((16, 4), np.float32)
    assert lib.ann_kv_cache_append_f32(None, R(kn), R(kn), R(kc), R(kc), R(tab), None, 0) == _capi.ANN_EINVAL
    x, w = np.zeros((4, 8), np.float32), np.zeros((8, 6), np.float32)
    assert lib.ann_output_projection_residual_f32(None, R(x), R(w), R(np.zeros((4, 5), np.float32)),
                                                  R(np.zeros((4, 6), np.float32))) == _capi.ANN_EINVAL


def test_selftest_limit_validated(capi):
    """The wait self-test refuses limits above 2 s before launching anything."""
    rc = capi.lib.ann_selftest_wait(None, 0, 3_000_000_000)
    assert rc == capi.ANN_EINVAL and "2 s" in capi.lib.ann_last_error().decode()
