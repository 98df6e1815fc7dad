"""Head-sharded decode and prefill attention across the GPUs of one node.

Attention heads are independent (the reference kernels read only query head hq
and KV head hq / g: onAcc/internal/nn/attention.hpp:28-36, 57-64), so rank r of
G owns query heads [r*H/G, (r+1)*H/G) and the matching KV heads, and keeps only
those heads of the KV cache. A decode step on every rank is

    ropeInPlace(Q_r, Knew_r) -> fused decode attention over its cache slice
    -> all-gather of the per-rank outputs -> re-assembly into BTHD [B,T,H,D]

The all-gather concatenates rank-major ([G][B,T,H/G,D]); the re-assembly is a
strided copy into the [B,T,G,H/G,D] view of the output (one CUDA kernel of
this library: ops::scale by 1 with strided views).

Prefill does the same per batch index: the fused causal prefill of batch b
on this rank's heads, then an asynchronous all-gather of that [T,H/G,D] slab
while batch b+1 computes, then re-assembly. (Chunks along T are not possible:
the reference's top-left causal mask has no query offset.)
"""
from dataclasses import dataclass
from datetime import timedelta

import torch


class ShardingError(RuntimeError):
    """A rank did not join, or left before a collective finished, within the deadline."""


def _check_queue(queue):
    """torch.distributed orders a collective after torch's current stream, so the
    kernels before it must run there too."""
    handle = torch.cuda.current_stream().cuda_stream
    if queue.handle != handle:
        raise ValueError("the sharded path needs a Queue on torch's current stream (ann.Queue())")


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


class HeadShardedDecode:
    """One decode step of the head-sharded path on this rank. `group` is a
    torch.distributed process group (NCCL on GPUs); world 1 needs none."""

    def __init__(self, shard: HeadShard, B: int, D: int, dtype=torch.float32, device="cuda", group=None):
        self.shard, self.B, self.D, self.group = shard, B, D, group
        self.out_local = torch.empty((B, 1, shard.local_heads, D), dtype=dtype, device=device)
        self.out = torch.empty((B, 1, shard.heads, D), dtype=dtype, device=device)
        self.gathered = gathered_buffer(shard, B, 1, D, dtype, device) if shard.world > 1 else None
        if self.gathered is not None:
            self._src, self._dst = reassembly_views(self.gathered, self.out)

    def step(self, queue, q, knew, k_cache, v_cache, cos, sin, position, scale):
        """q, knew: [B,1,H/G,D] of this rank (rotated in place); k_cache,
        v_cache: [B, H/G, Tk, D] of this rank. Returns the full [B,1,H,D]."""
        import torch.distributed as dist

        from . import AttentionKvLayout, RopeLayout, onHost
        if self.shard.world > 1:
            _check_queue(queue)
        g = self.shard.heads // self.shard.kv_heads
        onHost.nn.ropeInPlace(queue, None, q, knew, cos, sin, RopeLayout.BTHD, position)
        if self.shard.world == 1:
            onHost.nn.attentionDecode(queue, None, q, k_cache, v_cache, self.out, scale, g, AttentionKvLayout.BHTD)
            return self.out
        onHost.nn.attentionDecode(queue, None, q, k_cache, v_cache, self.out_local, scale, g,
                                  AttentionKvLayout.BHTD)
        dist.all_gather_into_tensor(self.gathered, self.out_local, group=self.group)
        onHost.ops.scale(queue, None, self._src, 1.0, self._dst)
        return self.out


class HeadShardedPrefill:
    """Fused causal prefill of this rank's heads, gathered into the full BTHD
    output. Batch index b is one chunk on its own side stream: prefill(b) ->
    all-gather(b) (NCCL, ordered after prefill(b) only) -> re-assembly(b), so the
    chunks' prefills run side by side and fill the GPU while finished chunks are
    gathered; the caller's stream waits for every chunk at the end. `group` as
    in HeadShardedDecode."""

    def __init__(self, shard: HeadShard, B: int, T: int, D: int, dtype=torch.float32, device="cuda", group=None,
                 streams: int = 4):
        self.shard, self.B, self.T, self.D, self.group = shard, B, T, D, group
        self.out = torch.empty((B, T, shard.heads, D), dtype=dtype, device=device)
        if shard.world > 1:
            self.out_local = torch.empty((B, T, shard.local_heads, D), dtype=dtype, device=device)
            # one receive slab per batch index so that gathers in flight never share a buffer
            self.gathered = torch.empty((B, shard.world, 1, T, shard.local_heads, D), dtype=dtype, device=device)
            self._views = [reassembly_views(self.gathered[b], self.out[b:b + 1]) for b in range(B)]
            self._streams = [torch.cuda.Stream(device=device) for _ in range(max(1, min(streams, B)))]

    def run(self, queue, q, k, v, scale, kv_layout=None, causal=True):
        """q: [B,T,H/G,D], k/v: [B,Tk,H_kv/G,D] (BTHD) or [B,H_kv/G,Tk,D] (BHTD)
        of this rank. Returns the full [B,T,H,D] output (ready on the caller's stream)."""
        import torch.distributed as dist

        from . import AttentionKvLayout, Queue, onHost
        layout = AttentionKvLayout.BTHD if kv_layout is None else kv_layout
        g = self.shard.heads // self.shard.kv_heads
        if self.shard.world == 1:
            onHost.nn.attentionPrefill(queue, None, q, k, v, self.out, scale, g, layout, causal)
            return self.out
        _check_queue(queue)
        main = torch.cuda.current_stream()
        inputs_ready = torch.cuda.Event()
        inputs_ready.record(main)
        chunk_done = []
        for b in range(self.B):  # every rank issues the gathers in the same order
            side = self._streams[b % len(self._streams)]
            with torch.cuda.stream(side):
                side.wait_event(inputs_ready)
                sq = Queue(side)
                onHost.nn.attentionPrefill(sq, None, q[b:b + 1], k[b:b + 1], v[b:b + 1], self.out_local[b:b + 1],
                                           scale, g, layout, causal)
                work = dist.all_gather_into_tensor(self.gathered[b], self.out_local[b:b + 1], group=self.group,
                                                   async_op=True)
                work.wait()  # the side stream (not the host) waits for the gather
                src, dst = self._views[b]
                onHost.ops.scale(sq, None, src, 1.0, dst)
                done = torch.cuda.Event()
                done.record(side)
                chunk_done.append(done)
        for done in chunk_done:
            main.wait_event(done)
        return self.out
