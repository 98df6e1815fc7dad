"""CPU oracle for the alpakaNN attention path -- TEST INFRASTRUCTURE ONLY.

ctypes binding of oracle/ann_oracle.cpp, a plain C++/OpenMP restatement of
the reference's per-element alpaka kernels. Only tests, the smoke check and
bench.py's CPU-baseline leg use it, always as the checker or as the timed CPU
baseline, never as a product code path.

Arrays are numpy arrays with arbitrary (positive) strides; a view descriptor
with byte pitches is built from each array, as ann_view is for device memory.
"""
import ctypes
import os

import numpy as np

from . import build as _build

MAX_RANK = 8


class OView(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("rank", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("extents", ctypes.c_int64 * MAX_RANK), ("pitches", ctypes.c_int64 * MAX_RANK)]


def view(a: np.ndarray) -> OView:
    v = OView()
    v.data = a.ctypes.data
    v.rank = a.ndim
    for i in range(a.ndim):
        v.extents[i] = a.shape[i]
        v.pitches[i] = a.strides[i]
    return v


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = ctypes.CDLL(path)
        P = ctypes.POINTER(OView)
        for sfx, ct in (("f32", ctypes.c_float), ("f64", ctypes.c_double)):
            getattr(_lib, f"oracle_embedding_lookup_{sfx}").argtypes = [P, P, P]
            getattr(_lib, f"oracle_rms_norm_{sfx}").argtypes = [P, P, P, ct]
            getattr(_lib, f"oracle_rope_{sfx}").argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_uint32]
            getattr(_lib, f"oracle_attention_scores_{sfx}").argtypes = [P, P, P, ctypes.c_uint32, ctypes.c_int]
            getattr(_lib, f"oracle_attention_apply_{sfx}").argtypes = [P, P, P, ctypes.c_uint32, ctypes.c_int]
            getattr(_lib, f"oracle_scale_{sfx}").argtypes = [P, ct, P]
            getattr(_lib, f"oracle_softmax_{sfx}").argtypes = [P, P, ctypes.c_uint32, ctypes.c_int,
                                                                ctypes.c_uint32, ctypes.c_uint32]
            getattr(_lib, f"oracle_gemm_{sfx}").argtypes = [P, P, P]
            getattr(_lib, f"oracle_attention_rows_{sfx}").argtypes = [
                P, P, P, ctypes.c_void_p, ctypes.c_int64, ct, ctypes.c_uint32, ctypes.c_int, ctypes.c_int,
                ctypes.c_void_p]
        _lib.oracle_set_threads.argtypes = [ctypes.c_int]
        _lib.oracle_max_threads.restype = ctypes.c_int
    return _lib


def _sfx(a):
    if a.dtype == np.float32:
        return "f32"
    if a.dtype == np.float64:
        return "f64"
    raise TypeError(f"oracle supports float32/float64, got {a.dtype}")


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return lib().oracle_max_threads()


def embedding_lookup(ids, table, out):
    assert ids.dtype == np.uint32
    getattr(lib(), f"oracle_embedding_lookup_{_sfx(table)}")(view(ids), view(table), view(out))
    return out


def rms_norm(x, w, out, eps):
    getattr(lib(), f"oracle_rms_norm_{_sfx(x)}")(view(x), view(w), view(out), eps)
    return out


def rope(x, cos, sin, out, layout=0, position_offset=0):
    getattr(lib(), f"oracle_rope_{_sfx(x)}")(view(x), view(cos), view(sin), view(out), layout, position_offset)
    return out


def attention_scores(q, k, s, g=1, layout=0):
    getattr(lib(), f"oracle_attention_scores_{_sfx(q)}")(view(q), view(k), view(s), g, layout)
    return s


def attention_apply(p, v, o, g=1, layout=0):
    getattr(lib(), f"oracle_attention_apply_{_sfx(p)}")(view(p), view(v), view(o), g, layout)
    return o


def scale(x, scalar, out):
    getattr(lib(), f"oracle_scale_{_sfx(x)}")(view(x), scalar, view(out))
    return out


def softmax(x, out, axis):
    getattr(lib(), f"oracle_softmax_{_sfx(x)}")(view(x), view(out), axis, 0, 0, 0)
    return out


def causal_softmax(x, out, axis, query_axis, key_axis):
    getattr(lib(), f"oracle_softmax_{_sfx(x)}")(view(x), view(out), axis, 1, query_axis, key_axis)
    return out


def gemm(a, b, c):
    getattr(lib(), f"oracle_gemm_{_sfx(a)}")(view(a), view(b), view(c))
    return c


def attention_rows(q, k, v, rows, scale_value, g=1, layout=0, causal=False):
    """Pipeline scores -> scale -> (causal) softmax -> apply for selected
    query rows. rows: int64 array [n, 3] of (b, i, hq). Returns [n, D]."""
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((rows.shape[0], q.shape[3]), dtype=q.dtype)
    getattr(lib(), f"oracle_attention_rows_{_sfx(q)}")(
        view(q), view(k), view(v), rows.ctypes.data, rows.shape[0], scale_value, g, layout, int(causal),
        out.ctypes.data)
    return out


def library_path() -> str:
    return _build.OUT if os.path.exists(_build.OUT) else _build.build()
