"""The node's communicator (ann_comm_*, NCCL) and head sharding across GPUs.

On one GPU: a 1-rank communicator gathers exactly, and a rank whose peer never
joins ends in ANN_ENCCL at its deadline (host-side bootstrap wait; no kernel
runs). On two GPUs: the gathered decode and prefill outputs equal the 1-GPU
outputs bit for bit, through the NCCL all-gather and through the multicast
stores (alpakann_b200.mirror) -- the same kernels run the same per-head
arithmetic, and the decode split and the fp64 prefill's key split are pinned
(ANN_DECODE_SPLITS, ANN_PREFILL_F64_SPLITS) so that both runs sum every row in
the same order. The signal barrier's bounded wait runs
out on one GPU when no rank signals (no multicast, no peer memory)."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _two_gpus():
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result, gather):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), ANN_DECODE_SPLITS="2",
                      ANN_PREFILL_F64_SPLITS="2")
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    import alpakann_b200 as ann
    from alpakann_b200.comm import Comm
    from alpakann_b200.sharded import HeadShard, HeadShardedDecode, HeadShardedPrefill, join
    join(rank, world, "nccl", timeout_s=60, device=torch.device("cuda", rank))
    comm = Comm.from_torch(timeout_s=60)
    try:
        gen = torch.Generator().manual_seed(2024)
        res = {}
        # ---- decode, GQA (8 query heads over 4 KV heads), BHTD cache, RoPE at position Tk
        B, H, Hkv, Tk, D = 3, 8, 4, 700, 128
        q, knew = (torch.randn(B, 1, H, D, generator=gen) for _ in range(2))
        k, v = (torch.randn(B, Hkv, Tk, D, generator=gen) for _ in range(2))
        ang = np.arange(Tk + 1)[:, None] * np.power(1e4, -2.0 * np.arange(D // 2) / D)[None]
        cos = torch.from_numpy(np.cos(ang)).float().cuda()
        sin = torch.from_numpy(np.sin(ang)).float().cuda()
        sc = 1.0 / math.sqrt(D)
        shard = HeadShard(rank, world, H, Hkv)
        hs, ks = shard.head_slice, shard.kv_head_slice
        dec = HeadShardedDecode(shard, B, D, torch.float32, "cuda", comm, gather=gather)
        res["gather"] = dec.gather
        got = None
        for _ in range(2):  # twice: the second step's barrier runs on the next epoch
            got = dec.step(ann.Queue(), q[:, :, hs].contiguous().cuda(), knew[:, :, hs].contiguous().cuda(),
                           k[:, ks].contiguous().cuda(), v[:, ks].contiguous().cuda(), cos, sin, Tk, sc).cpu()
        one = HeadShardedDecode(HeadShard(0, 1, H, Hkv), B, D, torch.float32, "cuda")
        ref = one.step(ann.Queue(), q.cuda(), knew.cuda(), k.cuda(), v.cuda(), cos, sin, Tk, sc).cpu()
        res["decode"] = bool(torch.equal(got, ref))
        # ---- causal prefill, fp32 (tensor cores) and fp64 (DFMA), BTHD
        for name, dt, (B, T, H, D) in (("prefill_f32", torch.float32, (2, 300, 4, 128)),
                                       ("prefill_f64", torch.float64, (2, 200, 4, 64))):
            q, k, v = (torch.randn(B, T, H, D, generator=gen, dtype=dt) for _ in range(3))
            shard = HeadShard(rank, world, H, H)
            hs = shard.head_slice
            sp = HeadShardedPrefill(shard, B, T, D, dt, "cuda", comm, gather=gather)
            sc = 1.0 / math.sqrt(D)
            got = sp.run(ann.Queue(), *(x[:, :, hs].contiguous().cuda() for x in (q, k, v)), sc).cpu()
            ref = torch.empty(B, T, H, D, dtype=dt, device="cuda")
            ann.onHost.nn.attentionPrefill(ann.Queue(), None, q.cuda(), k.cuda(), v.cuda(), ref, sc, 1, 0, True)
            res[name] = bool(torch.equal(got, ref.cpu()))
        torch.cuda.synchronize()
        res["device_error"] = ann.Queue().take_device_error()
        result[rank] = res
    finally:
        torch.cuda.synchronize()
        dist.barrier()  # no rank leaves while another may still store into its memory
        comm.close()
        dist.destroy_process_group()


def test_comm_single_rank_gathers_exactly():
    import alpakann_b200 as ann
    from alpakann_b200.comm import Comm, unique_id
    x = torch.randn(3, 5, 7, device="cuda")
    y = torch.full((1, 3, 5, 7), float("nan"), device="cuda")
    with Comm(1, 0, unique_id(), timeout_s=30) as comm:
        assert (comm.nranks, comm.rank) == (1, 0)
        comm.all_gather(ann.Queue(), x, y)
        torch.cuda.synchronize()
    assert torch.equal(y[0], x)


def _absent_peer(result):
    import time
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from alpakann_b200._capi import AnnCommError
    from alpakann_b200.comm import Comm, unique_id
    torch.cuda.set_device(0)
    t0 = time.monotonic()
    try:
        Comm(2, 0, unique_id(), timeout_s=3.0)  # rank 1 never joins
        result["outcome"] = ("joined", time.monotonic() - t0)
    except AnnCommError as e:
        result["outcome"] = ("ANN_ENCCL", time.monotonic() - t0, str(e))


def test_comm_rank_that_never_joins_ends_in_enccl():
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    p = mp.get_context("spawn").Process(target=_absent_peer, args=(result,))
    p.start()
    p.join(timeout=120)
    if p.is_alive():
        p.kill()
    kind, seconds = result["outcome"][:2]
    assert kind == "ANN_ENCCL"
    assert seconds < 60


def _multicast_available():
    if not _two_gpus():
        return False
    from alpakann_b200.mirror import MirrorBuffer
    return MirrorBuffer.available()


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["nccl", "multicast"])
def test_two_gpu_head_sharding_equals_one_gpu(gather):
    """Both gathers: the NCCL all-gather + re-assembly, and the multicast
    stores from inside the kernels + signal barrier (where the node has NVLink
    multicast)."""
    if gather == "multicast" and not _multicast_available():
        pytest.skip("no NVLink multicast on this node")
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), result, gather), nprocs=2, join=True, start_method="spawn")
    want = {"decode": True, "prefill_f32": True, "prefill_f64": True, "device_error": 0, "gather": gather}
    assert dict(result) == {0: want, 1: want}
