"""Dispatch helpers shared by onHost.nn and onHost.ops."""
import os
import sys

import torch

from .. import _capi
from .._capi import check, lib, ref

_SFX = {torch.float32: "f32", torch.float64: "f64"}


def suffix(*tensors) -> str:
    """Element type of the call (the reference's T_Type template argument):
    every floating tensor must share it."""
    dt = None
    for t in tensors:
        if t is None:
            continue
        if t.dtype not in _SFX:
            raise TypeError(f"alpakann_b200 supports float32 and float64 tensors, got {t.dtype}")
        if dt is None:
            dt = t.dtype
        elif t.dtype != dt:
            raise TypeError(f"mixed element types {dt} and {t.dtype} in one call")
    return _SFX[dt]


def fn(name: str, sfx: str):
    return getattr(lib, f"ann_{name}_{sfx}")


def handle(queue) -> int:
    if queue is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(queue, int):
        return queue
    if hasattr(queue, "handle"):
        return queue.handle
    return queue.cuda_stream  # torch.cuda.Stream


def trace_enabled() -> bool:
    """ALPAKANN_DEBUG_ATTENTION_TRACE: non-empty and not starting with '0'
    (onHost/nn/attention.hpp:24-28)."""
    env = os.environ.get("ALPAKANN_DEBUG_ATTENTION_TRACE")
    return bool(env) and env[0] != "0"


def trace(msg: str) -> None:
    if trace_enabled():
        print(msg, file=sys.stderr)


def ext(t) -> str:
    return "{" + ", ".join(str(int(e)) for e in t.shape) + "}"


def gemm(queue, A, B, C):
    """onHost::gemm (onHost/matrix/gemm.hpp:28-33): C = A * B, row-major,
    float/double, on cuBLAS."""
    sfx = suffix(A, B, C)
    check(fn("gemm", sfx)(handle(queue), ref(A), ref(B), ref(C)))


__all__ = ["suffix", "fn", "handle", "trace", "ext", "gemm", "_capi"]
