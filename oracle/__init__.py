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
            getattr(_lib, f"oracle_masked_softmax_{sfx}").argtypes = [P, P, P, ctypes.c_uint32]
            getattr(_lib, f"oracle_unary_{sfx}").argtypes = [P, P, ctypes.c_int, ct]
            getattr(_lib, f"oracle_binary_{sfx}").argtypes = [P, P, P, ctypes.c_int, ct]
            getattr(_lib, f"oracle_bias_add_{sfx}").argtypes = [P, P, P, ctypes.c_int]
            getattr(_lib, f"oracle_reduce_{sfx}").argtypes = [P, P, P, ctypes.c_int, ctypes.c_uint32]
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


def masked_softmax(x, mask, out, axis):
    """onAcc/internal/nn/softmax.hpp:76-116."""
    getattr(lib(), f"oracle_masked_softmax_{_sfx(x)}")(view(x), view(mask), view(out), axis)
    return out


# operator codes of include/ann_b200.h (ANN_UNARY_*, ANN_BINARY_*, ANN_ACT_*, ANN_REDUCE_*)
UNARY = {"copy": 0, "scale": 1, "exp": 2, "sqrt": 3, "rsqrt": 4, "relu": 5, "sigmoid": 6, "silu": 7, "gelu": 8}
BINARY = {"add": 0, "sub": 1, "mul": 2, "div": 3, "axpy": 4, "swiglu": 5}
ACT = {"none": 0, "relu": 1, "silu": 2, "gelu": 3}
REDUCE = {"sum": 0, "max": 1, "mean": 2, "sum_squares": 3, "dot": 4}


def unary(x, out, op, scalar=0.0):
    """onHost/ops/elementwise.hpp:15-178, one operator per element."""
    getattr(lib(), f"oracle_unary_{_sfx(x)}")(view(x), view(out), UNARY[op], scalar)
    return out


def binary(lhs, rhs, out, op, alpha=0.0):
    getattr(lib(), f"oracle_binary_{_sfx(lhs)}")(view(lhs), view(rhs), view(out), BINARY[op], alpha)
    return out


def bias_add(x, bias, out, act="none"):
    """biasAdd (elementwise.hpp:216-228), then the activation as a second pass."""
    getattr(lib(), f"oracle_bias_add_{_sfx(x)}")(view(x), view(bias), view(out), ACT[act])
    return out


def reduce(x, out, op, axis, rhs=None):
    """reduction.hpp:52-114: ascending loop over the axis per output."""
    r = view(rhs) if rhs is not None else None
    getattr(lib(), f"oracle_reduce_{_sfx(x)}")(view(x), ctypes.byref(r) if r is not None else None, view(out),
                                               REDUCE[op], axis)
    return out


def mlp_forward(x, weights, biases, hidden_act, last_act):
    """mlpForward (onHost/nn/mlp.hpp:150-218): per layer gemm, biasAdd, then the
    activation; hidden_act on every layer but the last."""
    h = np.ascontiguousarray(x)
    for i, (w, b) in enumerate(zip(weights, biases)):
        out = np.empty((h.shape[0], w.shape[1]), h.dtype)
        gemm(h, w, out)
        bias_add(out, b, out, last_act if i + 1 == len(weights) else hidden_act)
        h = out
    return h


def gated_mlp(x, wg, wu, wd):
    """mlp (onHost/nn/mlp.hpp:307-337): swiglu(x.Wg, x.Wu) . Wd."""
    g = np.empty((x.shape[0], wg.shape[1]), x.dtype)
    u = np.empty_like(g)
    gemm(x, wg, g)
    gemm(x, wu, u)
    h = binary(g, u, np.empty_like(g), "swiglu")
    out = np.empty((x.shape[0], wd.shape[1]), x.dtype)
    return gemm(h, wd, out)
