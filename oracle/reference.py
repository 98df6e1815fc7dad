"""alpakaNN's own device kernels run on the host -- TEST INFRASTRUCTURE ONLY.

ctypes binding of oracle/_ref/libann_ref.so (oracle/build_ref.py): the
reference's AttentionScoresKernel, AttentionApplyKernel,
EmbeddingLookupKernel, RmsNormKernel, RopeSingleKernel, SoftmaxKernel and
MaskedSoftmaxKernel (include/alpaka/nn/onAcc/internal/nn/*.hpp), compiled
unmodified against a host-only stand-in for the alpaka API. The tests use it
to pin the CPU oracle (a restatement of the same kernels) to the reference's
own code. available() is False when the library can be neither found nor
built (no reference tree).
"""
import ctypes

import numpy as np

from . import build_ref as _build
from . import view
from . import OView

_lib = None


def available() -> bool:
    try:
        return lib() is not None
    except OSError:
        return False


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        if path is None:
            return None
        _lib = ctypes.CDLL(path)
        P = ctypes.POINTER(OView)
        u32 = ctypes.c_uint32
        for sfx, ct in (("f32", ctypes.c_float), ("f64", ctypes.c_double)):
            getattr(_lib, f"ref_attention_scores_{sfx}").argtypes = [P, P, P, u32, ctypes.c_int]
            getattr(_lib, f"ref_attention_apply_{sfx}").argtypes = [P, P, P, u32, ctypes.c_int]
            getattr(_lib, f"ref_embedding_lookup_{sfx}").argtypes = [P, P, P]
            getattr(_lib, f"ref_rms_norm_{sfx}").argtypes = [P, P, P, ct]
            getattr(_lib, f"ref_rope_{sfx}").argtypes = [P, P, P, P, ctypes.c_int, u32]
            getattr(_lib, f"ref_softmax_{sfx}").argtypes = [P, P, u32, ctypes.c_int, u32, u32]
            getattr(_lib, f"ref_masked_softmax_{sfx}").argtypes = [P, P, P, u32]
            for name in ("attention_scores", "attention_apply", "embedding_lookup", "rope"):
                getattr(_lib, f"ref_{name}_{sfx}").restype = None
    return _lib


def _sfx(a):
    return {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64"}[a.dtype]


def _call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc not in (None, 0):
        raise ValueError(f"{name}: unsupported rank")


def attention_scores(q, k, s, g=1, layout=0):
    _call(f"ref_attention_scores_{_sfx(q)}", view(q), view(k), view(s), g, layout)
    return s


def attention_apply(p, v, o, g=1, layout=0):
    _call(f"ref_attention_apply_{_sfx(p)}", view(p), view(v), view(o), g, layout)
    return o


def embedding_lookup(ids, table, out):
    _call(f"ref_embedding_lookup_{_sfx(table)}", view(ids), view(table), view(out))
    return out


def rms_norm(x, w, out, eps):
    _call(f"ref_rms_norm_{_sfx(x)}", view(x), view(w), view(out), eps)
    return out


def rope(x, cos, sin, out, layout=0, position_offset=0):
    _call(f"ref_rope_{_sfx(x)}", view(x), view(cos), view(sin), view(out), layout, position_offset)
    return out


def softmax(x, out, axis):
    _call(f"ref_softmax_{_sfx(x)}", view(x), view(out), axis, 0, 0, 0)
    return out


def causal_softmax(x, out, axis, query_axis, key_axis):
    _call(f"ref_softmax_{_sfx(x)}", view(x), view(out), axis, 1, query_axis, key_axis)
    return out


def masked_softmax(x, mask, out, axis):
    _call(f"ref_masked_softmax_{_sfx(x)}", view(x), view(mask), view(out), axis)
    return out
