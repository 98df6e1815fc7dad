"""Head-sharded decode and prefill attention across the GPUs of one node.

Attention heads are independent (the reference kernels read only query head hq
and KV head hq / g: onAcc/internal/nn/attention.hpp:28-36, 57-64), so rank r of
G owns query heads [r*H/G, (r+1)*H/G) and the matching KV heads, and keeps only
those heads of the KV cache. A decode step on every rank is

    ropeInPlace(Q_r, Knew_r) -> fused decode attention over its cache slice
    -> all-gather of the per-rank outputs -> re-assembly into BTHD [B,T,H,D]

The all-gather (this library's NCCL communicator, alpakann_b200.comm.Comm,
enqueued on the step's own queue) concatenates rank-major ([G][B,T,H/G,D]);
the re-assembly is a strided copy into the [B,T,G,H/G,D] view of the output
(one CUDA kernel of this library: ops::scale by 1 with strided views).

Prefill does the same per batch index: the fused causal prefill of batch b
on this rank's heads, then an asynchronous all-gather of that [T,H/G,D] slab
while batch b+1 computes, then re-assembly. (Chunks along T are not possible:
the reference's top-left causal mask has no query offset.)

Where the node supports NVLink multicast (NVSwitch NVLS), both steps gather
without a collective instead (gather='multicast', alpakann_b200.mirror): the
output lives in memory every rank has bound to one multicast object, each
rank's kernel stores its heads through the multicast address into every
rank's copy while it computes, and one signal barrier per step publishes
them. No re-assembly pass: the stores land at their BTHD positions.
"""
from dataclasses import dataclass
from datetime import timedelta

import torch


class ShardingError(RuntimeError):
    """A rank did not join, or left before a collective finished, within the deadline."""


def join(rank: int, world: int, backend: str = "nccl", timeout_s: float = 60.0, device=None):
    """Join the node's process group with a deadline: a rank that never joins,
    or a collective that a peer never enters, ends in ShardingError (or the
    backend's own timeout error) instead of waiting for good. Rendezvous is
    read from MASTER_ADDR / MASTER_PORT."""
    import torch.distributed as dist

    kw = dict(backend=backend, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    if device is not None:
        kw["device_id"] = device
    try:
        dist.init_process_group(**kw)
    except Exception as e:  # store / rendezvous timeout
        raise ShardingError(f"rank {rank} of {world}: process group not complete within {timeout_s} s ({e})") from e


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    heads: int          # query heads in total
    kv_heads: int       # KV heads in total

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"bad rank {self.rank} of world {self.world}")
        if self.heads % self.world or self.kv_heads % self.world:
            raise ValueError(f"{self.heads} query / {self.kv_heads} kv heads do not shard over {self.world} ranks")
        if self.heads % self.kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")

    @property
    def local_heads(self) -> int:
        return self.heads // self.world

    @property
    def local_kv_heads(self) -> int:
        return self.kv_heads // self.world

    @property
    def head_slice(self) -> slice:
        return slice(self.rank * self.local_heads, (self.rank + 1) * self.local_heads)

    @property
    def kv_head_slice(self) -> slice:
        return slice(self.rank * self.local_kv_heads, (self.rank + 1) * self.local_kv_heads)


def gathered_buffer(shard: HeadShard, B: int, T: int, D: int, dtype, device) -> torch.Tensor:
    """Receive buffer of the all-gather, rank-major [G, B, T, H/G, D]."""
    return torch.empty((shard.world, B, T, shard.local_heads, D), dtype=dtype, device=device)


def reassembly_views(gathered: torch.Tensor, out: torch.Tensor):
    """(src, dst) strided views such that copying src into dst turns the
    rank-major gather into BTHD: dst[b, t, r, h, d] = gathered[r, b, t, h, d]."""
    G, B, T, Hl, D = gathered.shape
    if tuple(out.shape) != (B, T, G * Hl, D) or not out.is_contiguous():
        raise ValueError(f"output must be a contiguous [{B}, {T}, {G * Hl}, {D}] tensor")
    return gathered.permute(1, 2, 0, 3, 4), out.view(B, T, G, Hl, D)


def _mirror_or_none(shape, dtype, gather_requested: str):
    """A MirrorBuffer for 'multicast' / 'auto'; for 'auto' every rank agrees on the
    outcome (one all-reduce), and a failure anywhere means the NCCL gather on every
    rank. None when the NCCL gather is to be used."""
    import torch.distributed as dist

    from .mirror import MirrorBuffer
    if gather_requested == "multicast":
        return MirrorBuffer(shape, dtype)
    buf, ok = None, 1
    try:
        buf = MirrorBuffer(shape, dtype)
    except Exception:  # no multicast object on this node after all
        ok = 0
    flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return buf if int(flag) == 1 else None


def choose_gather(gather: str, world: int) -> str:
    """'multicast' (outputs stored through an NVLink multicast address inside the
    kernel, then a signal barrier), 'nccl' (all-gather + re-assembly) or, for
    'auto', multicast where the node supports it."""
    if world == 1:
        return "none"
    if gather == "auto":
        from .mirror import MirrorBuffer
        return "multicast" if MirrorBuffer.available() else "nccl"
    if gather not in ("multicast", "nccl"):
        raise ValueError(f"unknown gather {gather!r}")
    return gather


class HeadShardedDecode:
    """One decode step of the head-sharded path on this rank. `comm` is the
    node's communicator (alpakann_b200.comm.Comm), used by the NCCL gather;
    world 1 needs none. gather: 'auto' | 'multicast' | 'nccl' (choose_gather)."""

    def __init__(self, shard: HeadShard, B: int, D: int, dtype=torch.float32, device="cuda", comm=None,
                 gather: str = "auto"):
        self.gather = choose_gather(gather, shard.world)
        if self.gather == "nccl" and comm is None:
            raise ValueError("a sharded step over several ranks needs a Comm")
        self.shard, self.B, self.D, self.comm = shard, B, D, comm
        self.gathered = None
        if self.gather == "multicast":
            self.mirror = _mirror_or_none((B, 1, shard.heads, D), dtype, gather)
            if self.mirror is None:
                if comm is None:
                    raise ValueError("no multicast on this node, and the NCCL gather needs a Comm")
                self.gather = "nccl"
        if self.gather == "multicast":
            self.out = self.mirror.tensor
            self.out_local = self.out[:, :, shard.head_slice, :]  # this rank's heads of every copy
            self._out_mc = self.mirror.mirror_of(self.out_local)
            return
        self.out_local = torch.empty((B, 1, shard.local_heads, D), dtype=dtype, device=device)
        self.out = torch.empty((B, 1, shard.heads, D), dtype=dtype, device=device)
        self.gathered = gathered_buffer(shard, B, 1, D, dtype, device) if shard.world > 1 else None
        if self.gathered is not None:
            self._src, self._dst = reassembly_views(self.gathered, self.out)

    def step(self, queue, q, knew, k_cache, v_cache, cos, sin, position, scale):
        """q, knew: [B,1,H/G,D] of this rank (rotated in place); k_cache,
        v_cache: [B, H/G, Tk, D] of this rank. Returns the full [B,1,H,D]."""
        from . import AttentionKvLayout, RopeLayout, onHost
        g = self.shard.heads // self.shard.kv_heads
        onHost.nn.ropeInPlace(queue, None, q, knew, cos, sin, RopeLayout.BTHD, position)
        if self.shard.world == 1:
            onHost.nn.attentionDecode(queue, None, q, k_cache, v_cache, self.out, scale, g, AttentionKvLayout.BHTD)
            return self.out
        if self.gather == "multicast":
            onHost.nn.attentionDecodeMirror(queue, None, q, k_cache, v_cache, self.out_local, self._out_mc, scale, g,
                                            AttentionKvLayout.BHTD)
            self.mirror.barrier(queue)
            return self.out
        onHost.nn.attentionDecode(queue, None, q, k_cache, v_cache, self.out_local, scale, g,
                                  AttentionKvLayout.BHTD)
        self.comm.all_gather(queue, self.out_local, self.gathered)
        onHost.ops.scale(queue, None, self._src, 1.0, self._dst)
        return self.out


class HeadShardedPrefill:
    """Fused causal prefill of this rank's heads, gathered into the full BTHD
    output. Batch index b is one chunk on its own side stream: prefill(b), then
    its all-gather on the communicator's stream (gathers keep one order on every
    rank), then its re-assembly; the chunks' prefills run side by side while
    finished chunks are gathered, and the caller's queue waits for every chunk
    at the end. `comm` as in HeadShardedDecode."""

    def __init__(self, shard: HeadShard, B: int, T: int, D: int, dtype=torch.float32, device="cuda", comm=None,
                 streams: int = 4, gather: str = "auto"):
        self.gather = choose_gather(gather, shard.world)
        if self.gather == "nccl" and comm is None:
            raise ValueError("a sharded prefill over several ranks needs a Comm")
        self.shard, self.B, self.T, self.D, self.comm = shard, B, T, D, comm
        if self.gather == "multicast":
            self.mirror = _mirror_or_none((B, T, shard.heads, D), dtype, gather)
            if self.mirror is None:
                if comm is None:
                    raise ValueError("no multicast on this node, and the NCCL gather needs a Comm")
                self.gather = "nccl"
        if self.gather == "multicast":
            self.out = self.mirror.tensor
            self.out_local = self.out[:, :, shard.head_slice, :]
            self._out_mc = self.mirror.mirror_of(self.out_local)
            return
        self.out = torch.empty((B, T, shard.heads, D), dtype=dtype, device=device)
        if shard.world > 1:
            self.out_local = torch.empty((B, T, shard.local_heads, D), dtype=dtype, device=device)
            # one receive slab per batch index so that gathers in flight never share a buffer
            self.gathered = torch.empty((B, shard.world, 1, T, shard.local_heads, D), dtype=dtype, device=device)
            self._views = [reassembly_views(self.gathered[b], self.out[b:b + 1]) for b in range(B)]
            self._side = [torch.cuda.Stream(device=device) for _ in range(max(1, min(streams, B)))]
            self._comm_stream = torch.cuda.Stream(device=device)

    def run(self, queue, q, k, v, scale, kv_layout=None, causal=True):
        """q: [B,T,H/G,D], k/v: [B,Tk,H_kv/G,D] (BTHD) or [B,H_kv/G,Tk,D] (BHTD)
        of this rank. Returns the full [B,T,H,D] output (ready in `queue` order)."""
        from . import AttentionKvLayout, Queue, onHost
        layout = AttentionKvLayout.BTHD if kv_layout is None else kv_layout
        g = self.shard.heads // self.shard.kv_heads
        if self.shard.world == 1:
            onHost.nn.attentionPrefill(queue, None, q, k, v, self.out, scale, g, layout, causal)
            return self.out
        if self.gather == "multicast":  # every rank's heads land in every copy inside the kernel
            onHost.nn.attentionPrefillMirror(queue, None, q, k, v, self.out_local, self._out_mc, scale, g, layout,
                                             causal)
            self.mirror.barrier(queue)
            return self.out
        caller = queue.stream if not isinstance(queue.stream, int) else torch.cuda.ExternalStream(queue.stream)
        comm_q = Queue(self._comm_stream)
        inputs_ready = torch.cuda.Event()
        inputs_ready.record(caller)
        chunk_done = []
        for b in range(self.B):
            side = self._side[b % len(self._side)]
            sq = Queue(side)
            side.wait_event(inputs_ready)
            onHost.nn.attentionPrefill(sq, None, q[b:b + 1], k[b:b + 1], v[b:b + 1], self.out_local[b:b + 1],
                                       scale, g, layout, causal)
            computed = torch.cuda.Event()
            computed.record(side)
            self._comm_stream.wait_event(computed)
            self.comm.all_gather(comm_q, self.out_local[b:b + 1], self.gathered[b])
            gathered = torch.cuda.Event()
            gathered.record(self._comm_stream)
            side.wait_event(gathered)
            src, dst = self._views[b]
            onHost.ops.scale(sq, None, src, 1.0, dst)
            done = torch.cuda.Event()
            done.record(side)
            chunk_done.append(done)
        for done in chunk_done:
            caller.wait_event(done)
        return self.out
