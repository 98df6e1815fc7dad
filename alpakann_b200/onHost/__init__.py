"""alpaka::nn::onHost -- host API of the attention path (reference:
include/alpaka/nn/onHost/). Sub-namespaces nn and ops, plus gemm
(onHost/matrix/gemm.hpp:28-33)."""
from . import nn, ops
from ._common import gemm

__all__ = ["nn", "ops", "gemm"]
