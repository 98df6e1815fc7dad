"""The node's NCCL communicator through the C ABI (ann_comm_*): rendezvous id,
deadline-bounded join, rank-major all-gather on a library queue, teardown.

The head-sharded path uses it for the re-assembly of per-rank output slabs, so
the data-path collective is this library's own NCCL call; torch.distributed is
only one possible carrier of the 128-byte rendezvous id (any key-value store
with set/get works, e.g. the TCPStore torchrun provides).
"""
import ctypes

from . import _capi
from ._capi import COMM_ID_BYTES, check, lib


def unique_id() -> bytes:
    """A new rendezvous id; rank 0 creates it and hands it to the other ranks."""
    buf = (ctypes.c_char * COMM_ID_BYTES)()
    check(lib.ann_comm_unique_id(ctypes.byref(buf)))
    return bytes(buf.raw)


class Comm:
    """One rank of the communicator, on the current CUDA device."""

    def __init__(self, nranks: int, rank: int, uid: bytes, timeout_s: float = 60.0):
        if len(uid) != COMM_ID_BYTES:
            raise ValueError(f"rendezvous id must be {COMM_ID_BYTES} bytes")
        buf = (ctypes.c_char * COMM_ID_BYTES).from_buffer_copy(uid)
        self._h = ctypes.c_void_p()
        check(lib.ann_comm_init(ctypes.byref(self._h), nranks, rank, ctypes.byref(buf), float(timeout_s)))
        self.nranks, self.rank = nranks, rank

    @classmethod
    def from_store(cls, store, nranks: int, rank: int, timeout_s: float = 60.0, key: str = "ann_comm_id"):
        """Rendezvous through a key-value store (set/get of bytes)."""
        if rank == 0:
            uid = unique_id()
            store.set(key, uid)
        else:
            uid = bytes(store.get(key))
        return cls(nranks, rank, uid, timeout_s)

    @classmethod
    def from_torch(cls, group=None, timeout_s: float = 60.0):
        """Rendezvous over an initialised torch.distributed process group (the id
        travels with broadcast_object_list from rank 0)."""
        import torch.distributed as dist
        rank, nranks = dist.get_rank(group), dist.get_world_size(group)
        box = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        return cls(nranks, rank, box[0], timeout_s)

    def all_gather(self, queue, send, recv):
        """recv[r] = send of rank r, enqueued on `queue`. send: a contiguous
        tensor; recv: contiguous with nranks times its bytes."""
        nbytes = send.numel() * send.element_size()
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("all_gather needs contiguous tensors")
        if recv.numel() * recv.element_size() != self.nranks * nbytes:
            raise ValueError(f"receive buffer must hold {self.nranks} x {nbytes} bytes")
        check(lib.ann_comm_allgather(self._h, queue.handle, send.data_ptr(), recv.data_ptr(), nbytes))

    def close(self):
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib.ann_comm_destroy(h))

    def abort(self):
        if self._h:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib.ann_comm_abort(h))

    def __del__(self):
        try:
            self.abort()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


__all__ = ["Comm", "unique_id", "_capi"]
