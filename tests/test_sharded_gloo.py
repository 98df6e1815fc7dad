"""Host logic of the head-sharded decode path on CPU ranks (gloo): head
partition, rank-major all-gather and re-assembly into BTHD must reproduce the
unsharded result exactly. The per-rank attention here is a torch fp64
restatement (the GPU kernels are covered by the -m gpu tests)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from alpakann_b200.sharded import HeadShard, gathered_buffer, reassembly_views


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attention(q, k, v, g, scale):
    # q [B,1,H,D], k/v [B,Hkv,Tk,D] -> out [B,1,H,D]; query head h reads kv head h // g
    kk = k.repeat_interleave(g, dim=1)
    vv = v.repeat_interleave(g, dim=1)
    s = torch.einsum("bthd,bhkd->bhtk", q, kk) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhtk,bhkd->bthd", p, vv)


def _worker(rank, world, port, B, H, Hkv, Tk, D, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(0)
        q = torch.randn(B, 1, H, D, generator=gen, dtype=torch.float64)
        k = torch.randn(B, Hkv, Tk, D, generator=gen, dtype=torch.float64)
        v = torch.randn(B, Hkv, Tk, D, generator=gen, dtype=torch.float64)
        shard = HeadShard(rank, world, H, Hkv)
        local = _attention(q[:, :, shard.head_slice], k[:, shard.kv_head_slice], v[:, shard.kv_head_slice],
                           H // Hkv, 0.125)
        gathered = gathered_buffer(shard, B, 1, D, torch.float64, "cpu")
        dist.all_gather(list(gathered.unbind(0)), local.contiguous())  # rank-major, as all_gather_into_tensor
        out = torch.empty(B, 1, H, D, dtype=torch.float64)
        src, dst = reassembly_views(gathered, out)
        dst.copy_(src)
        full = _attention(q, k, v, H // Hkv, 0.125)
        result[rank] = bool(torch.equal(out, full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,H,Hkv", [(2, 8, 8), (4, 8, 4), (2, 6, 2)])
def test_head_sharded_gather_reassembles_bthd(world, H, Hkv):
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), 3, H, Hkv, 40, 16, result), nprocs=world, join=True,
                       start_method="spawn")
    assert dict(result) == {r: True for r in range(world)}


def test_shard_validation():
    with pytest.raises(ValueError):
        HeadShard(0, 3, 32, 32)       # 32 heads over 3 ranks
    with pytest.raises(ValueError):
        HeadShard(2, 2, 32, 32)       # rank out of range
    with pytest.raises(ValueError):
        HeadShard(0, 2, 8, 3)         # query heads not a multiple of kv heads
    s = HeadShard(3, 8, 64, 64)
    assert (s.local_heads, s.head_slice) == (8, slice(24, 32))
    g = gathered_buffer(s, 2, 1, 4, torch.float32, "cpu")
    with pytest.raises(ValueError):
        reassembly_views(g, torch.empty(2, 1, 63, 4))
