"""ctypes binding of the ann_b200 C ABI (include/ann_b200.h).

The shared library is built in-tree by alpakann_b200/build.py. Importing this
module without it raises ImportError: there is no CPU fallback.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libann_b200.so")

ANN_OK, ANN_EINVAL, ANN_ECUDA, ANN_ENOTSUP, ANN_EDEVICE, ANN_ENCCL, ANN_EIO = 0, 1, 2, 3, 4, 5, 6
COMM_ID_BYTES = 128
ANN_DEVERR_TOKEN_ID, ANN_DEVERR_WAIT_TIMEOUT = 0x1, 0x2
MAX_RANK = 8


class AnnView(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("rank", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("extents", ctypes.c_int64 * MAX_RANK), ("pitches", ctypes.c_int64 * MAX_RANK)]


class AnnTensorSpec(ctypes.Structure):
    """ann_tensor_spec: TensorSpec of onHost/core/binary.hpp:33-39."""
    _fields_ = [("name", ctypes.c_char_p), ("offset_bytes", ctypes.c_uint64), ("count", ctypes.c_uint64),
                ("shape", ctypes.POINTER(ctypes.c_uint64)), ("shape_rank", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


if not os.path.exists(LIB_PATH):
    raise ImportError(f"alpakann_b200: {LIB_PATH} is missing; build it with `python alpakann_b200/build.py`")

lib = ctypes.CDLL(LIB_PATH)

_P = ctypes.POINTER(AnnView)
_S = ctypes.c_void_p
_u32, _i32 = ctypes.c_uint32, ctypes.c_int32
_f = {"f32": ctypes.c_float, "f64": ctypes.c_double}

# Every exported entry point and its argument types. The symbol test checks
# this table against include/ann_b200.h.
_C = ctypes.c_void_p  # ann_comm
_ID = ctypes.c_char * COMM_ID_BYTES
SIGNATURES = {
    "ann_version": ([], ctypes.c_int),
    "ann_last_error": ([], ctypes.c_char_p),
    "ann_take_device_error": ([_S, ctypes.POINTER(_u32)], ctypes.c_int),
    "ann_selftest_wait": ([_S, _i32, ctypes.c_uint64], ctypes.c_int),
    "ann_comm_unique_id": ([ctypes.POINTER(_ID)], ctypes.c_int),
    "ann_comm_init": ([ctypes.POINTER(_C), _i32, _i32, ctypes.POINTER(_ID), ctypes.c_double], ctypes.c_int),
    "ann_comm_size": ([_C, ctypes.POINTER(_i32), ctypes.POINTER(_i32)], ctypes.c_int),
    "ann_comm_allgather": ([_C, _S, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
    "ann_comm_destroy": ([_C], ctypes.c_int),
    "ann_comm_abort": ([_C], ctypes.c_int),
    "ann_cast": ([_S, _P, _i32, _P, _i32], ctypes.c_int),
    "ann_mlp_static_scratch": ([_S, _i32, _P, _P, _P, _P, _P], ctypes.c_int),
    "ann_fill": ([_S, _P, _i32, ctypes.c_void_p], ctypes.c_int),
    "ann_mlp_forward_workspace_bytes": ([_P, _i32, _P, _P, _P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64)],
                                        ctypes.c_int),
    "ann_signal_barrier": ([_S, ctypes.c_void_p, ctypes.c_void_p, _i32, _i32, _u32, ctypes.c_uint64],
                           ctypes.c_int),
    "ann_signal_barrier_dev": ([_S, ctypes.c_void_p, ctypes.c_void_p, _i32, _i32, ctypes.c_void_p, ctypes.c_uint64],
                               ctypes.c_int),
    "ann_sha256_file": ([ctypes.c_char_p, ctypes.c_char_p], ctypes.c_int),
    "ann_sha256_bytes": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p], ctypes.c_int),
    "ann_load_binary_tensor": ([_S, ctypes.c_char_p, ctypes.POINTER(AnnTensorSpec), ctypes.c_size_t,
                                ctypes.c_char_p, ctypes.c_void_p], ctypes.c_int),
    "ann_load_binary_tensor_box": ([_S, ctypes.c_char_p, ctypes.POINTER(AnnTensorSpec), ctypes.c_size_t,
                                    ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64], ctypes.c_int),
}
for _sfx, _ft in _f.items():
    SIGNATURES.update({
        f"ann_embedding_lookup_{_sfx}": ([_S, _P, _P, _P], ctypes.c_int),
        f"ann_rms_norm_{_sfx}": ([_S, _P, _P, _P, _ft], ctypes.c_int),
        f"ann_embedding_rms_norm_{_sfx}": ([_S, _P, _P, _P, _P, _ft], ctypes.c_int),
        f"ann_rope_{_sfx}": ([_S, _P, _P, _P, _P, _i32, _u32], ctypes.c_int),
        f"ann_rope_inplace_{_sfx}": ([_S, _P, _P, _P, _P, _i32, _u32], ctypes.c_int),
        f"ann_attention_scores_{_sfx}": ([_S, _P, _P, _P, _u32, _i32], ctypes.c_int),
        f"ann_scale_{_sfx}": ([_S, _P, _ft, _P], ctypes.c_int),
        f"ann_softmax_{_sfx}": ([_S, _P, _P, _u32], ctypes.c_int),
        f"ann_causal_softmax_{_sfx}": ([_S, _P, _P, _u32, _u32, _u32], ctypes.c_int),
        f"ann_attention_apply_{_sfx}": ([_S, _P, _P, _P, _u32, _i32], ctypes.c_int),
        f"ann_gemm_{_sfx}": ([_S, _P, _P, _P], ctypes.c_int),
        f"ann_qkv_projection_{_sfx}": ([_S, _P, _P, _P, _P, _P, _P, _P], ctypes.c_int),
        f"ann_output_projection_residual_{_sfx}": ([_S, _P, _P, _P, _P], ctypes.c_int),
        f"ann_kv_cache_append_{_sfx}": ([_S, _P, _P, _P, _P, _P, _P, _u32], ctypes.c_int),
        f"ann_masked_softmax_{_sfx}": ([_S, _P, _P, _P, _u32], ctypes.c_int),
        f"ann_unary_{_sfx}": ([_S, _i32, _P, _P, _ft], ctypes.c_int),
        f"ann_binary_{_sfx}": ([_S, _i32, _P, _P, _P, _ft], ctypes.c_int),
        f"ann_bias_add_{_sfx}": ([_S, _P, _P, _i32, _P], ctypes.c_int),
        f"ann_reduce_{_sfx}": ([_S, _i32, _P, _P, _u32], ctypes.c_int),
        f"ann_dot_{_sfx}": ([_S, _P, _P, _P, _u32], ctypes.c_int),
        f"ann_linear_bias_{_sfx}": ([_S, _P, _P, _P, _i32, _P], ctypes.c_int),
        f"ann_mlp_forward_{_sfx}": ([_S, _P, _i32, _P, _P, _i32, _i32, _P, ctypes.c_void_p, ctypes.c_uint64],
                                    ctypes.c_int),
        f"ann_mlp_{_sfx}": ([_S, _P, _P, _P, _P, _P, ctypes.c_void_p, ctypes.c_uint64], ctypes.c_int),
        f"ann_attention_decode_{_sfx}": ([_S, _P, _P, _P, _P, _ft, _u32, _i32], ctypes.c_int),
        f"ann_attention_prefill_{_sfx}": ([_S, _P, _P, _P, _P, _ft, _u32, _i32, _i32], ctypes.c_int),
        f"ann_attention_decode_mirror_{_sfx}": ([_S, _P, _P, _P, _P, ctypes.c_void_p, _ft, _u32, _i32], ctypes.c_int),
        f"ann_attention_prefill_mirror_{_sfx}": ([_S, _P, _P, _P, _P, ctypes.c_void_p, _ft, _u32, _i32, _i32],
                                                 ctypes.c_int),
    })

for _name, (_args, _res) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res


class AnnError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


class AnnShapeError(AnnError, ValueError):
    """ANN_EINVAL: the reference throws std::invalid_argument here."""


class AnnNotSupported(AnnError, NotImplementedError):
    """ANN_ENOTSUP."""


class AnnIOError(AnnError):
    """ANN_EIO: a file could not be opened / read, or its digest did not match
    (std::runtime_error in the reference)."""


class AnnCommError(AnnError):
    """ANN_ENCCL: NCCL failed, or a rank did not join / finish within the deadline."""


def check(rc: int) -> None:
    if rc == ANN_OK:
        return
    msg = lib.ann_last_error().decode(errors="replace")
    if rc == ANN_EINVAL:
        raise AnnShapeError(rc, msg)
    if rc == ANN_ENOTSUP:
        raise AnnNotSupported(rc, msg)
    if rc == ANN_ENCCL:
        raise AnnCommError(rc, msg)
    if rc == ANN_EIO:
        raise AnnIOError(rc, msg)
    raise AnnError(rc, msg)


def view(t) -> AnnView:
    """ann_view of a torch tensor (device memory) or numpy array: extents and
    byte pitches taken from its shape and strides, no copy."""
    v = AnnView()
    if isinstance(t, np.ndarray):
        v.data = t.ctypes.data
        shape, pitches = t.shape, t.strides
    else:
        v.data = t.data_ptr()
        es = t.element_size()
        shape, pitches = tuple(t.shape), tuple(s * es for s in t.stride())
    if len(shape) > MAX_RANK:
        raise ValueError(f"rank {len(shape)} exceeds {MAX_RANK}")
    v.rank = len(shape)
    for i, (e, p) in enumerate(zip(shape, pitches)):
        v.extents[i] = e
        v.pitches[i] = p
    return v


def ref(t):
    return ctypes.byref(view(t))


def take_device_error(stream_handle: int) -> int:
    bits = _u32(0)
    check(lib.ann_take_device_error(stream_handle, ctypes.byref(bits)))
    return bits.value
