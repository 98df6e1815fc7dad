"""alpaka::nn::onHost::ops -- the elementwise glue on the attention path
(reference: onHost/ops/elementwise.hpp:330-334)."""
from .._capi import check, ref
from ._common import fn, handle, suffix


def scale(queue, exec, input, scalar, output):
    """out = in * scalar; in-place (input is output) allowed."""
    check(fn("scale", suffix(input, output))(handle(queue), ref(input), float(scalar), ref(output)))
