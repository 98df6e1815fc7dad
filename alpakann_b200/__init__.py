"""alpakann_b200 -- B200-native drop-in for alpakaNN's attention path.

The path embeddingLookup -> rmsNorm -> qkvProjection -> ropeInPlace ->
attentionScores -> scale -> (causal)softmax -> attentionApply runs on
hand-written sm_100a CUDA kernels behind the C ABI in include/ann_b200.h.
This package mirrors the reference's host namespace alpaka::nn::onHost:

    from alpakann_b200 import onHost, Queue, AttentionKvLayout
    onHost.nn.attentionScores(queue, exec, Q, K, scores, 1, AttentionKvLayout.BTHD)

Tensors are torch CUDA tensors (any strides); `queue` wraps a CUDA stream and
`exec` is accepted and ignored, as the alpaka executor has no meaning here.
"""
import enum

from . import _capi
from ._capi import AnnError, AnnNotSupported, AnnShapeError, take_device_error

__version__ = "0.1.0"


class AttentionKvLayout(enum.IntEnum):
    """alpaka::nn::AttentionKvLayout (nn/attention.hpp:10-14)."""
    BTHD = 0
    BHTD = 1


class RopeLayout(enum.IntEnum):
    """alpaka::nn::RopeLayout (nn/rope.hpp:10-14)."""
    BTHD = 0
    BHTD = 1


class Queue:
    """In-order queue = one CUDA stream (alpaka's queue.enqueue order).

    Queue() uses torch's current stream of the current device; Queue(stream)
    wraps a torch.cuda.Stream or a raw cudaStream_t handle (int)."""

    def __init__(self, stream=None):
        import torch
        if stream is None:
            stream = torch.cuda.current_stream()
        self.stream = stream
        self.handle = stream if isinstance(stream, int) else stream.cuda_stream

    def wait(self):
        """alpaka::onHost::wait(queue)."""
        import torch
        if isinstance(self.stream, int):
            torch.cuda.synchronize()
        else:
            self.stream.synchronize()

    def take_device_error(self) -> int:
        return take_device_error(self.handle)


def library_path() -> str:
    return _capi.LIB_PATH


from . import onHost  # noqa: E402

__all__ = ["onHost", "Queue", "AttentionKvLayout", "RopeLayout", "AnnError", "AnnShapeError", "AnnNotSupported",
           "library_path"]
