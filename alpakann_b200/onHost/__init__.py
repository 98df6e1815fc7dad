"""alpaka::nn::onHost -- host API of the attention path (reference:
include/alpaka/nn/onHost/). Sub-namespaces nn and ops, plus gemm
(onHost/matrix/gemm.hpp:28-33) and the model-artifact loader of
onHost/core/binary.hpp (TensorSpec, sha256File, loadBinaryTensor)."""
from . import core, nn, ops
from ._common import gemm
from .core import TensorSpec, loadBinaryTensor, loadBinaryTensorBox, sha256File

__all__ = ["core", "nn", "ops", "gemm", "TensorSpec", "sha256File", "loadBinaryTensor", "loadBinaryTensorBox"]
