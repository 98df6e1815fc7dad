"""alpaka::nn::onHost core: flat model artifacts (onHost/core/binary.hpp).

TensorSpec (:33-39), sha256File (:212-232) and loadBinaryTensor (:234-323),
plus loadBinaryTensorBox, which loads one rank's rectangle of a row-major
weight for head sharding (no reference counterpart: the reference loads
whole tensors only).
"""
import ctypes
import os
from dataclasses import dataclass, field
from typing import Sequence, Tuple

import torch

from .._capi import AnnTensorSpec, check, lib

_ELEM = {torch.float32: 4, torch.float64: 8}


@dataclass
class TensorSpec:
    """One tensor of a ".bin" artifact: payload at ``offsetBytes``, ``count``
    elements, informational row-major ``shape``."""
    name: str
    offsetBytes: int
    count: int
    shape: Sequence[int] = field(default_factory=tuple)


def _spec(spec: TensorSpec):
    shape = (ctypes.c_uint64 * max(1, len(spec.shape)))(*[int(e) for e in spec.shape])
    s = AnnTensorSpec()
    name = spec.name.encode()
    s.name = name
    s.offset_bytes = int(spec.offsetBytes)
    s.count = int(spec.count)
    s.shape = ctypes.cast(shape, ctypes.POINTER(ctypes.c_uint64)) if len(spec.shape) else None
    s.shape_rank = len(spec.shape)
    return s, (shape, name)  # keep the buffers alive with the struct


def _path(path) -> bytes:
    return os.fsencode(path)


def sha256File(path) -> str:
    """SHA-256 of the file as 64 lowercase hex digits; AnnIOError (a
    RuntimeError) if it cannot be opened or read."""
    out = ctypes.create_string_buffer(65)
    check(lib.ann_sha256_file(_path(path), out))
    return out.value.decode()


def sha256Bytes(data: bytes) -> str:
    out = ctypes.create_string_buffer(65)
    check(lib.ann_sha256_bytes(data, len(data), out))
    return out.value.decode()


def _dtype(dtype):
    if dtype not in _ELEM:
        raise TypeError("alpaka::nn::onHost::loadBinaryTensor supports only float32 and float64 tensors.")
    return _ELEM[dtype]


def _target(queue, device):
    """(stream handle, device) of a load: a torch.cuda.Stream carries its
    device; otherwise the given or current device and its current stream."""
    if isinstance(queue, torch.cuda.Stream):
        return queue.cuda_stream, queue.device
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if queue is None:
        return torch.cuda.current_stream(dev).cuda_stream, dev
    return (queue if isinstance(queue, int) else queue.handle), dev


def loadBinaryTensor(queue, path, spec: TensorSpec, expectedSha256: str = "", dtype=torch.float32,
                     device=None) -> torch.Tensor:
    """loadBinaryTensor<T>: a new 1-D device tensor of ``spec.count`` elements
    (dtype float32 or float64 is the reference's T_Type). Every check of the
    reference runs, digest included, before the tensor is allocated:
    AnnShapeError (ValueError) for the layout, AnnIOError for file errors and
    a digest mismatch. The copy is enqueued on ``queue``; synchronise it
    before reading the tensor elsewhere."""
    es = _dtype(dtype)
    s, keep = _spec(spec)
    p = _path(path)
    sha = expectedSha256.encode()
    check(lib.ann_load_binary_tensor(None, p, ctypes.byref(s), es, sha, None))  # checks only
    stream, dev = _target(queue, device)
    with torch.cuda.device(dev):
        out = torch.empty(int(spec.count), dtype=dtype, device=dev)
        check(lib.ann_load_binary_tensor(stream, p, ctypes.byref(s), es, b"", out.data_ptr()))
    if isinstance(queue, torch.cuda.Stream):
        out.record_stream(queue)
    return out


def loadBinaryTensorBox(queue, path, spec: TensorSpec, rows: Tuple[int, int], cols: Tuple[int, int],
                        expectedSha256: str = "", dtype=torch.float32, device=None) -> torch.Tensor:
    """Rows ``[rows[0], rows[0]+rows[1])`` x columns ``[cols[0], cols[0]+cols[1])``
    of a tensor stored row-major as ``[shape[0], count/shape[0]]``, as a new
    dense ``[rows[1], cols[1]]`` device tensor: one rank's column-parallel
    (Wq/Wk/Wv) or row-parallel (Wo) shard, read without the other ranks'
    columns."""
    es = _dtype(dtype)
    s, keep = _spec(spec)
    p = _path(path)
    sha = expectedSha256.encode()
    r0, nr = (int(v) for v in rows)
    c0, nc = (int(v) for v in cols)
    check(lib.ann_load_binary_tensor_box(None, p, ctypes.byref(s), es, sha, r0, nr, c0, nc, None, nc * es))
    stream, dev = _target(queue, device)
    with torch.cuda.device(dev):
        out = torch.empty((nr, nc), dtype=dtype, device=dev)
        check(lib.ann_load_binary_tensor_box(stream, p, ctypes.byref(s), es, b"", r0, nr, c0, nc, out.data_ptr(),
                                             nc * es))
    if isinstance(queue, torch.cuda.Stream):
        out.record_stream(queue)
    return out


__all__ = ["TensorSpec", "sha256File", "sha256Bytes", "loadBinaryTensor", "loadBinaryTensorBox"]
