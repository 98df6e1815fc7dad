"""alpaka::nn::onHost::ops -- elementwise ops, activations and axis
reductions (reference: onHost/ops/elementwise.hpp, onHost/ops/reduction.hpp).

Same names and argument order as the reference; T_Type comes from the
tensors' dtype (float32 / float64). Shape errors raise AnnShapeError (a
ValueError) with the reference's message. `exec` is accepted and ignored.
In-place calls (input is output) are allowed.
"""
import ctypes

import torch

from .._capi import check, lib, ref
from ._common import fn, handle, suffix

# unaryOp / binaryOp operator codes (include/ann_b200.h)
COPY, SCALE, EXP, SQRT, RSQRT, RELU, SIGMOID, SILU, GELU = range(9)
ADD, SUB, MUL, DIV, AXPY, SWIGLU = range(6)
SUM, MAX, MEAN, SUM_SQUARES, DOT = range(5)
_DTYPE = {torch.float32: 0, torch.float64: 1, torch.int32: 2, torch.uint32: 3, torch.int64: 4}
_CT = {0: ctypes.c_float, 1: ctypes.c_double, 2: ctypes.c_int32, 3: ctypes.c_uint32, 4: ctypes.c_int64}


def _unary(queue, op, input, output, scalar=0.0):
    check(fn("unary", suffix(input, output))(handle(queue), op, ref(input), ref(output), float(scalar)))


def _binary(queue, op, lhs, rhs, output, alpha=0.0):
    check(fn("binary", suffix(lhs, rhs, output))(handle(queue), op, ref(lhs), ref(rhs), ref(output), float(alpha)))


def fill(queue, exec, out, value):
    """elementwise.hpp:250-254: every element of out = value (out's type)."""
    if out.dtype not in _DTYPE:
        raise TypeError(f"fill: unsupported element type {out.dtype}")
    code = _DTYPE[out.dtype]
    v = _CT[code](value)
    check(lib.ann_fill(handle(queue), ref(out), code, ctypes.byref(v)))


def copy(queue, exec, input, output):
    _unary(queue, COPY, input, output)


def scale(queue, exec, input, scalar, output):
    """out = in * scalar (elementwise.hpp:326-330)."""
    check(fn("scale", suffix(input, output))(handle(queue), ref(input), float(scalar), ref(output)))


def add(queue, exec, lhs, rhs, out):
    _binary(queue, ADD, lhs, rhs, out)


def sub(queue, exec, lhs, rhs, out):
    _binary(queue, SUB, lhs, rhs, out)


def mul(queue, exec, lhs, rhs, out):
    _binary(queue, MUL, lhs, rhs, out)


def div(queue, exec, lhs, rhs, out):
    _binary(queue, DIV, lhs, rhs, out)


def axpy(queue, exec, alpha, x, y, out):
    """out = alpha * x + y (elementwise.hpp:332-336)."""
    _binary(queue, AXPY, x, y, out, alpha)


def swiglu(queue, exec, lhs, rhs, out):
    """out = lhs * sigmoid(lhs) * rhs (elementwise.hpp:410-414)."""
    _binary(queue, SWIGLU, lhs, rhs, out)


def biasAdd(queue, exec, input, bias, out):
    """out[..., h] = input[..., h] + bias[h] (elementwise.hpp:338-353)."""
    check(fn("bias_add", suffix(input, bias, out))(handle(queue), ref(input), ref(bias), 0, ref(out)))


def cast(queue, exec, input, out):
    """ops::cast<T_Out> (elementwise.hpp:355-361): T_Out is out's dtype."""
    if input.dtype not in _DTYPE or out.dtype not in _DTYPE:
        raise TypeError(f"cast: unsupported element types {input.dtype} -> {out.dtype}")
    check(lib.ann_cast(handle(queue), ref(input), _DTYPE[input.dtype], ref(out), _DTYPE[out.dtype]))


def exp(queue, exec, input, out):
    _unary(queue, EXP, input, out)


def sqrt(queue, exec, input, out):
    _unary(queue, SQRT, input, out)


def rsqrt(queue, exec, input, out):
    _unary(queue, RSQRT, input, out)


def relu(queue, exec, input, out):
    _unary(queue, RELU, input, out)


def sigmoid(queue, exec, input, out):
    _unary(queue, SIGMOID, input, out)


def silu(queue, exec, input, out):
    _unary(queue, SILU, input, out)


def gelu(queue, exec, input, out):
    _unary(queue, GELU, input, out)


def unaryOp(queue, exec, input, out, op, scalar=0.0):
    """ops::unaryOp with one of the operator codes above."""
    _unary(queue, op, input, out, scalar)


def binaryOp(queue, exec, lhs, rhs, out, op, alpha=0.0):
    """ops::binaryOp with one of the operator codes above."""
    _binary(queue, op, lhs, rhs, out, alpha)


def _reduce(queue, op, input, out, axis):
    check(fn("reduce", suffix(input, out))(handle(queue), op, ref(input), ref(out), int(axis)))


def reduceSum(queue, exec, input, out, axis):
    _reduce(queue, SUM, input, out, axis)


def reduceMax(queue, exec, input, out, axis):
    _reduce(queue, MAX, input, out, axis)


def reduceMean(queue, exec, input, out, axis):
    _reduce(queue, MEAN, input, out, axis)


def reduceSumSquares(queue, exec, input, out, axis):
    _reduce(queue, SUM_SQUARES, input, out, axis)


def dot(queue, exec, lhs, rhs, out, axis):
    check(fn("dot", suffix(lhs, rhs, out))(handle(queue), ref(lhs), ref(rhs), ref(out), int(axis)))


def makeReducedExtents(extents, axis):
    """reduction.hpp:285-288: the extents with extent 1 on `axis`."""
    e = list(extents)
    e[axis] = 1
    return tuple(e)
