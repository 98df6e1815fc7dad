"""Host logic of the head-sharded decode path on CPU ranks (gloo): head
partition, rank-major all-gather and re-assembly into BTHD must reproduce the
unsharded result exactly. The per-rank attention here is a torch fp64
restatement (the GPU kernels are covered by the -m gpu tests)."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from alpakann_b200.sharded import HeadShard, ShardingError, gathered_buffer, join, reassembly_views


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


def _absent_peer_worker(rank, world, port, result):
    """Rank 1 never joins; rank 0's join must end at its deadline."""
    if rank == 1:
        return
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.monotonic()
    try:
        join(rank, world, "gloo", timeout_s=3.0)
        result[rank] = ("joined", time.monotonic() - t0)
        import torch.distributed as dist
        dist.destroy_process_group()
    except ShardingError:
        result[rank] = ("ShardingError", time.monotonic() - t0)


def test_rank_that_never_joins_ends_in_an_error():
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    mp.start_processes(_absent_peer_worker, args=(2, _free_port(), result), nprocs=2, join=True,
                       start_method="spawn")
    kind, seconds = result[0]
    assert kind == "ShardingError"
    assert seconds < 60


def _leaving_peer_worker(rank, world, port, result):
    """Both ranks join; rank 1 leaves before the all-gather of a step. Rank 0's
    all-gather must fail (peer gone or process-group timeout), not wait for good."""
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    join(rank, world, "gloo", timeout_s=5.0)
    if rank == 1:
        os._exit(0)  # leaves between steps, without a clean shutdown
    shard = HeadShard(rank, world, 4, 4)
    gathered = gathered_buffer(shard, 1, 1, 8, torch.float32, "cpu")
    t0 = time.monotonic()
    try:
        dist.all_gather(list(gathered.unbind(0)), torch.zeros(1, 1, 2, 8))
        result[rank] = ("completed", time.monotonic() - t0)
    except Exception as e:  # gloo reports the closed connection or its timeout
        result[rank] = (type(e).__name__, time.monotonic() - t0)
    os._exit(0)


def test_rank_that_leaves_before_the_gather_ends_in_an_error():
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    ctx = mp.start_processes(_leaving_peer_worker, args=(2, _free_port(), result), nprocs=2, join=False,
                             start_method="spawn")
    deadline = time.monotonic() + 120
    while 0 not in result and time.monotonic() < deadline:
        time.sleep(0.2)
    for p in ctx.processes:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    kind, seconds = result[0]
    assert kind != "completed"
    assert seconds < 60
