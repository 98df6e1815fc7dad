"""Outputs that every rank of the node holds, written through NVLink multicast.

The head-sharded path's gather without a collective (include/ann_b200.h,
"multicast ("mirror") outputs"): the full output tensor lives in memory that
every rank has bound to ONE NVLink multicast object, here torch symmetric
memory (plumbing only: it allocates, maps the peers' copies and creates the
multicast object). Each rank's decode / prefill kernel stores its head slice
through the multicast address, so the switch writes it into every rank's
copy while the kernel runs; one signal barrier (ann_signal_barrier_dev, its
epoch kept in device memory so that a CUDA graph can replay it) after the
kernel tells every rank that all slices have landed.

MirrorBuffer.available() says whether this node can do it (NVSwitch
multicast needs driver and fabric support); the sharded steps fall back to the
NCCL all-gather when it cannot.
"""
import ctypes

import torch

from ._capi import check, lib


def _group_name(group):
    import torch.distributed as dist
    g = group if group is not None else dist.group.WORLD
    return g.group_name


class MirrorBuffer:
    """One tensor of `shape` on every rank, bound to one multicast object, plus
    the signal words of the barrier that publishes it."""

    def __init__(self, shape, dtype, group=None, timeout_s: float = 5.0):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        name = _group_name(group)
        self.tensor = symm.empty(tuple(shape), dtype=dtype, device="cuda")
        self._h = symm.rendezvous(self.tensor, name)
        mc = int(self._h.multicast_ptr)
        if mc == 0:
            raise RuntimeError("no NVLink multicast object for this buffer (multicast not supported here)")
        base = int(self._h.buffer_ptrs[self.rank])
        self._mc = mc + (self.tensor.data_ptr() - base)
        # barrier signals: nranks words per rank, zero before the first barrier
        self._sig = symm.empty((max(self.world, 1),), dtype=torch.int32, device="cuda")
        self._sig.zero_()
        self._hs = symm.rendezvous(self._sig, name)
        off = self._sig.data_ptr() - int(self._hs.buffer_ptrs[self.rank])
        ptrs = [int(p) + off for p in self._hs.buffer_ptrs]
        self._peer_sig = torch.tensor(ptrs, dtype=torch.int64, device="cuda")
        self._epoch_word = torch.zeros((1,), dtype=torch.int32, device="cuda")  # this rank's last epoch
        self.timeout_ns = int(timeout_s * 1e9)
        torch.cuda.synchronize()
        dist.barrier(group)  # every rank's signals are zero before anyone signals

    @staticmethod
    def available(group=None) -> bool:
        """Whether the CUDA driver and fabric of this node support multicast objects."""
        try:
            from torch._C._autograd import DeviceType
            from torch._C._distributed_c10d import _SymmetricMemory
            return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, torch.cuda.current_device()))
        except Exception:
            return False

    def mirror_of(self, view: torch.Tensor) -> int:
        """Multicast address of the first element of `view`, a view into this buffer."""
        off = view.data_ptr() - self.tensor.data_ptr()
        nbytes = self.tensor.numel() * self.tensor.element_size()
        if not 0 <= off < max(nbytes, 1):
            raise ValueError("view is not inside this buffer")
        return self._mc + off

    @property
    def epoch_word(self) -> int:
        """Device address of this rank's epoch word (every barrier on these
        signals, from Python or the C++ header, advances it on the device)."""
        return self._epoch_word.data_ptr()

    def barrier(self, queue):
        """Enqueue the barrier on `queue` (every rank, same order): afterwards every
        rank's copy holds all ranks' stores made through the multicast address.
        Capturable in a CUDA graph: the epoch advances on the device."""
        check(lib.ann_signal_barrier_dev(queue.handle, ctypes.c_void_p(self._sig.data_ptr()),
                                         ctypes.c_void_p(self._peer_sig.data_ptr()), self.world, self.rank,
                                         ctypes.c_void_p(self.epoch_word), self.timeout_ns))


__all__ = ["MirrorBuffer"]
