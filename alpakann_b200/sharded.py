"""Head-sharded decode attention across the GPUs of one node.

Attention heads are independent (the reference kernels read only query head hq
and KV head hq / g: onAcc/internal/nn/attention.hpp:28-36, 57-64), so rank r of
G owns query heads [r*H/G, (r+1)*H/G) and the matching KV heads, and keeps only
those heads of the KV cache. A decode step on every rank is

    ropeInPlace(Q_r, Knew_r) -> fused decode attention over its cache slice
    -> all-gather of the per-rank outputs -> re-assembly into BTHD [B,T,H,D]

The all-gather concatenates rank-major ([G][B,T,H/G,D]); the re-assembly is a
strided copy into the [B,T,G,H/G,D] view of the output (one CUDA kernel of
this library: ops::scale by 1 with strided views).
"""
from dataclasses import dataclass

import torch


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
