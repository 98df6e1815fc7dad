"""Benchmark of the attention decode step (one JSON line on rank 0).

Headline workload (c5): batch 16, one query token per sequence, KV cache of
32768 tokens, 64 heads x head_dim 128, fp32, BHTD cache (32 GiB of K+V). Each
step rotates Q and the new K row with RoPE (theta 5e5) at position 32768 and
runs fused decode attention (scores -> scale 1/sqrt(128) -> softmax -> apply)
over the cache. With N GPUs the heads are sharded (64/N per GPU, each GPU
holds only its heads' cache) and the per-head outputs are all-gathered (NCCL)
and re-assembled into [B,1,H,D] on every rank: total work is fixed, so the
scaling is strong. The same line carries, under "extra", the smaller decode
workload c2 (batch 8, cache 2048, 32 heads x 128) measured the same way.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c5|c2] [--no-extra]

--impl reference times the CPU oracle (the reference's per-element host
algorithm restated in C++/OpenMP; the reference itself cannot be built
here) on a bounded sample of the same workload, on rank 0.
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "c2": dict(B=8, Tk=2048, H=32, D=128, theta=1e4,
               desc="decode: batch 8, 1 query token, KV cache 2048, 32 heads x 128, fp32, BHTD, RoPE 1e4 at pos 2048"),
    "c5": dict(B=16, Tk=32768, H=64, D=128, theta=5e5,
               desc="decode: batch 16, 1 query token, KV cache 32768, 64 heads x 128 (d_model 8192), fp32, BHTD, "
                    "RoPE 5e5 at pos 32768"),
}
L2_BYTES = 126 * 1024 * 1024


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=3000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="c5")
    p.add_argument("--no-extra", action="store_true", help="skip the secondary c2 measurement")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU-baseline sample")
    p.add_argument("--prefill-only", metavar="B,T,H,D[,f64]", default=None,
                   help="run only the fused causal prefill on this shape (--steps launches) and print its time; "
                        "the small case the prefill ncu captures use")
    p.add_argument("--ops", action="store_true",
                   help="measure only the HBM-bound ops (elementwise, bias+activation, reductions, maskedSoftmax) "
                        "and the MLP layers on 1 GiB operands; one JSON line per op")
    p.add_argument("--ops-elems", type=int, default=1 << 28,
                   help="elements per operand of --ops (default 2^28 = 1 GiB of float32); a smaller value also skips "
                        "the MLP lines (the small case ncu captures use)")
    p.add_argument("--loader", metavar="MIB", type=int, default=None,
                   help="measure only the model-artifact loader on a MIB-sized float32 file (page-cached): "
                        "sha256File, loadBinaryTensor, a 1/8 column shard, against pinned and pageable copies")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tf32_peak():
    """Dense tf32 tensor TFLOP/s: half the measured bf16 burst rate (B200 runs
    kind::tf32 at half the kind::f16 rate), else half the 1.59 PFLOP/s fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]) / 2, "measured bf16 / 2"
    except Exception:
        return 1590.0 / 2, "fallback bf16 / 2"


def ncu_traffic(workload):
    """DRAM bytes per decode launch (1 GPU) from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", f"decode_{workload}_ncu.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi sampler (200 ms) for the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.samples = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self, t0, t1):
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        inside = [s for ts, s in self.samples if t0 - 0.2 <= ts <= t1 + 0.2]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in inside:
            try:
                sm.append(float(s[1]))
                mx.append(float(s[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, s[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU ---
class CpuSample:
    """The oracle's per-op decode pipeline (RoPE on Q and the new K row,
    attentionScores, scale, softmax, attentionApply) on `batches` x `heads`
    of the workload, inputs prepared once."""

    def __init__(self, w, batches, heads):
        import numpy as np

        import oracle
        self.oracle = oracle
        B, Tk, H, D = w["B"], w["Tk"], w["H"], w["D"]
        g = np.random.default_rng(0)
        self.q = g.standard_normal((batches, 1, heads, D)).astype(np.float32)
        self.kn = g.standard_normal((batches, 1, heads, D)).astype(np.float32)
        self.k = g.standard_normal((batches, heads, Tk, D)).astype(np.float32)
        self.v = g.standard_normal((batches, heads, Tk, D)).astype(np.float32)
        ang = np.arange(Tk + 1, dtype=np.float64)[:, None] * np.power(w["theta"], -2.0 * np.arange(D // 2) / D)[None]
        self.cos, self.sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        self.s = np.empty((batches, heads, 1, Tk), np.float32)
        self.p = np.empty_like(self.s)
        self.o = np.empty_like(self.q)
        self.rq, self.rk = np.empty_like(self.q), np.empty_like(self.kn)
        self.scale = np.float32(1.0 / math.sqrt(D))
        self.Tk = Tk
        self.frac = (batches * heads) / (B * H)
        self.desc = f"{batches} sequence(s) x {heads} head(s) of {B}x{H} per step, scaled by {1 / self.frac:g}"

    def step(self):
        o = self.oracle
        o.rope(self.q, self.cos, self.sin, self.rq, 0, self.Tk)
        o.rope(self.kn, self.cos, self.sin, self.rk, 0, self.Tk)
        o.attention_scores(self.rq, self.k, self.s, 1, 1)
        o.scale(self.s, self.scale, self.s)
        o.softmax(self.s, self.p, 3)
        o.attention_apply(self.p, self.v, self.o, 1, 1)

    def time_full_steps(self, seconds=None, steps=None):
        """Seconds per FULL workload step, from timing the sample."""
        reps, t0 = 0, time.perf_counter()
        while (steps is not None and reps < steps) or (seconds is not None and
                                                       (reps == 0 or time.perf_counter() - t0 < seconds)):
            self.step()
            reps += 1
        return (time.perf_counter() - t0) / reps / self.frac, reps


def cpu_sample_for(w):
    # c2: one sequence x all heads (1/8 of a step); c5: one sequence x one head (1/1024)
    return CpuSample(w, 1, w["H"]) if w["Tk"] <= 4096 else CpuSample(w, 1, 1)


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    oracle.set_threads(os.cpu_count() or 1)
    smp = cpu_sample_for(w)
    for _ in range(args.warmup):
        smp.step()
    step, _ = smp.time_full_steps(steps=args.steps)
    value = w["B"] / step
    line = {"impl": "reference", "metric": "decode attn tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w["desc"], "batch": w["B"], "kv_len": w["Tk"], "heads": w["H"],
                       "head_dim": w["D"]},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                             "sample": smp.desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU ---
class DecodeBench:
    """Inputs and the two step flavours (device-resident and end-to-end) of
    the head-sharded decode workload on this rank."""

    def __init__(self, w, rank, world, comm):
        import numpy as np
        import torch

        import alpakann_b200 as ann
        from alpakann_b200 import _capi
        from alpakann_b200.sharded import HeadShard, HeadShardedDecode
        self.torch, self.capi, self.w = torch, _capi, w
        self.world = world
        B, Tk, H, D = w["B"], w["Tk"], w["H"], w["D"]
        self.shard = HeadShard(rank, world, H, H)
        Hl = self.shard.local_heads
        f32 = torch.float32
        gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
        self.kv_bytes = 2 * B * Hl * Tk * D * 4
        self.copies = max(1, math.ceil(3 * L2_BYTES / self.kv_bytes))  # rotate caches: every step reads cold HBM
        self.caches = [(torch.randn((B, Hl, Tk, D), generator=gen, dtype=f32, device="cuda"),
                        torch.randn((B, Hl, Tk, D), generator=gen, dtype=f32, device="cuda"))
                       for _ in range(self.copies)]
        self.q = torch.randn((B, 1, Hl, D), generator=gen, dtype=f32, device="cuda")
        self.knew = torch.randn((B, 1, Hl, D), generator=gen, dtype=f32, device="cuda")
        ang = np.arange(Tk + 1, dtype=np.float64)[:, None] * np.power(w["theta"], -2.0 * np.arange(D // 2) / D)[None]
        self.cos = torch.from_numpy(np.cos(ang)).to(f32).cuda()
        self.sin = torch.from_numpy(np.sin(ang)).to(f32).cuda()
        self.scale = 1.0 / math.sqrt(D)
        self.sharded = HeadShardedDecode(self.shard, B, D, f32, "cuda", comm)
        self.comm = comm
        self.stream = torch.cuda.current_stream()
        self.queue = ann.Queue(self.stream)
        # descriptors built once: the device-timed loop only issues C-ABI calls
        V = _capi.view
        self.vq, self.vkn, self.vcos, self.vsin = V(self.q), V(self.knew), V(self.cos), V(self.sin)
        self.vout = V(self.sharded.out if world == 1 else self.sharded.out_local)
        self.vkv = [(V(k), V(v)) for k, v in self.caches]
        if world > 1:
            self.vsrc, self.vdst = V(self.sharded._src), V(self.sharded._dst)
        self.launches_per_step = 2 if world == 1 else 3  # rope, decode (+ re-assembly); NCCL's own kernel not counted
        self.gather_bytes = self.sharded.out_local.numel() * 4
        # pinned host buffers of the end-to-end step
        self.hq = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
        self.hk = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
        self.hout = torch.empty((B, 1, H, D), dtype=f32).pin_memory()

    def step(self, i, ev=None):
        lib, R, sh, chk = self.capi.lib, ctypes.byref, self.stream.cuda_stream, self.capi.check
        chk(lib.ann_rope_inplace_f32(sh, R(self.vq), R(self.vkn), R(self.vcos), R(self.vsin), 0, self.w["Tk"]))
        vk, vv = self.vkv[i % self.copies]
        if ev is not None:
            ev[0].record(self.stream)
        chk(lib.ann_attention_decode_f32(sh, R(self.vq), R(vk), R(vv), R(self.vout), self.scale, 1, 1))
        if ev is not None:
            ev[1].record(self.stream)
        if self.world > 1:  # this library's NCCL all-gather, then the re-assembly kernel
            chk(lib.ann_comm_allgather(self.comm._h, sh, self.sharded.out_local.data_ptr(),
                                       self.sharded.gathered.data_ptr(), self.gather_bytes))
            chk(lib.ann_scale_f32(sh, R(self.vsrc), 1.0, R(self.vdst)))

    def e2e_step(self, i):
        """Through the public Python API, with the step's inputs copied from
        pinned host memory and the full output read back."""
        self.q.copy_(self.hq, non_blocking=True)
        self.knew.copy_(self.hk, non_blocking=True)
        k, v = self.caches[i % self.copies]
        out = self.sharded.step(self.queue, self.q, self.knew, k, v, self.cos, self.sin, self.w["Tk"], self.scale)
        self.hout.copy_(out, non_blocking=True)

    def release(self):
        self.caches.clear()
        self.vkv.clear()
        self.torch.cuda.empty_cache()


def barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(values, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t]


def measure(bench, steps, warmup, world, rank, with_clocks):
    import torch
    for i in range(warmup):
        bench.step(i)
    barrier(world)
    clocks = Clocks() if (with_clocks and rank == 0) else None
    if clocks:
        time.sleep(0.5)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    t_wall0 = time.time()
    start.record(bench.stream)
    for i in range(steps):
        bench.step(i, kev[i])
    end.record(bench.stream)
    barrier(world)
    t_wall1 = time.time()
    elapsed = start.elapsed_time(end) / 1e3
    kernel_s = sum(a.elapsed_time(b) for a, b in kev) / 1e3 / steps
    clk = clocks.stop(t_wall0, t_wall1) if clocks else None

    e2e_steps = max(1, min(steps, 1000))
    for i in range(min(warmup, 5)):
        bench.e2e_step(i)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(bench.stream)
    for i in range(e2e_steps):
        bench.e2e_step(i)
    e1.record(bench.stream)
    barrier(world)
    e2e_s = e0.elapsed_time(e1) / 1e3 / e2e_steps
    elapsed, kernel_s, e2e_s = max_over_ranks([elapsed, kernel_s, e2e_s], world)
    return elapsed, kernel_s, e2e_s, e2e_steps, clk


PREFILL = {
    "c3": dict(B=4, T=4096, H=32, D=128, dtype="f32",
               desc="prefill: batch 4, seq 4096, 32 heads x 128, fp32, causal, scale 1/sqrt(128)"),
    "c4": dict(B=2, T=1024, H=16, D=64, dtype="f64",
               desc="prefill: batch 2, seq 1024, 16 heads x 64, fp64, causal, scale 1/8"),
}


def measure_prefill(name, world, rank, comm, reps=10):
    """Fused causal prefill of this rank's heads (heads sharded over ranks) and,
    for N > 1, the all-gather of the outputs into BTHD (batch b gathered while
    batch b + 1 computes), timed with CUDA events; TFLOP/s counts QK^T + PV over
    the causal half including the diagonal, 4*B*H*D*T(T+1)/2, for the whole job."""
    import torch

    import alpakann_b200 as ann
    from alpakann_b200.sharded import HeadShard, HeadShardedPrefill
    p = PREFILL[name]
    B, T, H, D = p["B"], p["T"], p["H"], p["D"]
    dt = torch.float32 if p["dtype"] == "f32" else torch.float64
    Hl = H // world
    gen = torch.Generator(device="cuda").manual_seed(77 + rank)
    q, k, v = (torch.randn((B, T, Hl, D), generator=gen, dtype=dt, device="cuda") for _ in range(3))
    queue = ann.Queue()
    sc = 1.0 / math.sqrt(D)
    sharded = HeadShardedPrefill(HeadShard(rank, world, H, H), B, T, D, dt, "cuda", comm)
    for _ in range(2):
        sharded.run(queue, q, k, v, sc)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        sharded.run(queue, q, k, v, sc)
    e1.record()
    barrier(world)
    t = max_over_ranks([e0.elapsed_time(e1) / 1e3 / reps], world)[0]
    flops = 4 * B * H * D * T * (T + 1) / 2
    del q, k, v, sharded
    torch.cuda.empty_cache()
    res = {"workload": p["desc"], "ms": t * 1e3, "tflops": flops / t / 1e12, "tokens_per_s": B * T / t,
           "dtype": p["dtype"], "gathered": world > 1}
    if p["dtype"] == "f32":
        # 3xTF32: every useful flop costs three tf32 tensor flops
        pk, kind = tf32_peak()
        pair = os.environ.get("ANN_PREFILL_TC_PAIR", "1")[:1] != "0"
        name = (f"prefill_pair_kernel<{D}> (tcgen05 cta_group::2 on SM pairs, 3xTF32)" if pair
                else f"prefill_tc_kernel<{D}> (tcgen05 3xTF32)")
        res.update(kernel=name, tf32_peak_tflops=pk, tf32_peak_kind=kind,
                   frac_of_3xtf32_peak=3 * res["tflops"] / world / pk)
    else:
        pk = fp64_gemm_tflops()
        res.update(kernel=f"prefill_f64_kernel<{D}> (FP64 tensor cores, mma.sync m16n8k4)", fp64_peak_tflops=pk,
                   fp64_peak_kind="cuBLAS DGEMM 4096^3, measured in this run",
                   frac_of_fp64_peak=res["tflops"] / world / pk)
    return res


def fp64_gemm_tflops():
    """Dense fp64 TFLOP/s of cuBLAS DGEMM (torch.matmul, 4096^3, best of 5): the
    fp64 counterpart of the measured bf16 GEMM peak, measured in this run."""
    import torch
    n = 4096
    a, b = (torch.randn(n, n, dtype=torch.float64, device="cuda") for _ in range(2))
    for _ in range(2):
        torch.matmul(a, b)
    best = float("inf")
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) / 1e3)
    del a, b
    return 2.0 * n ** 3 / best / 1e12


def prefill_only(args):
    """--prefill-only B,T,H,D[,f64]: causal prefill launches on one GPU, CUDA-event timed."""
    import torch

    import alpakann_b200 as ann
    f = args.prefill_only.split(",")
    B, T, H, D = (int(x) for x in f[:4])
    dt = torch.float64 if len(f) > 4 and f[4] == "f64" else torch.float32
    gen = torch.Generator(device="cuda").manual_seed(77)
    q, k, v = (torch.randn((B, T, H, D), generator=gen, dtype=dt, device="cuda") for _ in range(3))
    o = torch.empty_like(q)
    queue = ann.Queue()
    sc = 1.0 / math.sqrt(D)
    for _ in range(args.warmup):
        ann.onHost.nn.attentionPrefill(queue, None, q, k, v, o, sc, 1, 0, True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ann.onHost.nn.attentionPrefill(queue, None, q, k, v, o, sc, 1, 0, True)
    e1.record()
    torch.cuda.synchronize()
    if queue.take_device_error() != 0:
        raise SystemExit("prefill reported a device error")
    t = e0.elapsed_time(e1) / 1e3 / max(args.steps, 1)
    flops = 4 * B * H * D * T * (T + 1) / 2
    print(json.dumps({"prefill": args.prefill_only, "launches": args.steps, "ms": t * 1e3,
                      "tflops": flops / t / 1e12}), flush=True)


def ops_only(args):
    """--ops: device time per launch (CUDA events, median of --steps after
    --warmup, operands larger than L2) and algorithmic bytes / time against
    the measured HBM copy peak, for the ops of onHost/ops and onHost/nn/mlp.hpp."""
    import torch

    import alpakann_b200 as ann
    ops, nn = ann.onHost.ops, ann.onHost.nn
    peak, kind = peaks()
    torch.manual_seed(0)
    dev = "cuda"
    f32 = torch.float32
    G = max(args.ops_elems // (1 << 21), 1) << 21  # elements per operand, a multiple of 4096 * 512
    R = G // 4096
    a = torch.randn(G, device=dev)
    b = torch.randn(G, device=dev)
    o = torch.empty(G, device=dev)
    rows = a.view(R, 4096)
    bias = torch.randn(4096, device=dev)
    red_rows = torch.empty((R, 1), device=dev)
    red_cols = torch.empty((1, 4096), device=dev)
    S = G // 2 // (1024 * 1024)  # softmax rows of 1024: half of an operand
    sm_in = a[:S << 20].view(S, 1, 1024, 1024)
    sm_mask = b[:S << 20].view(S, 1, 1024, 1024)
    sm_out = o[:S << 20].view(S, 1, 1024, 1024)

    def timed(fn, reps=max(args.steps, 5), warm=max(args.warmup, 3)):
        """Mean device time of `reps` back-to-back launches between two
        events, so the host's launch work overlaps the previous kernel
        instead of being counted as device time."""
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps

    cases = [
        ("add", 3 * 4 * G, lambda: ops.add(None, None, a, b, o)),
        ("axpy", 3 * 4 * G, lambda: ops.axpy(None, None, 0.5, a, b, o)),
        ("silu", 2 * 4 * G, lambda: ops.silu(None, None, a, o)),
        ("gelu", 2 * 4 * G, lambda: ops.gelu(None, None, a, o)),
        ("swiglu", 3 * 4 * G, lambda: ops.swiglu(None, None, a, b, o)),
        (f"biasAdd+silu [{R},4096]", 2 * 4 * G,
         lambda: ann._capi.check(ann._capi.lib.ann_bias_add_f32(
             None, ann._capi.ref(rows), ann._capi.ref(bias), 2, ann._capi.ref(o.view(R, 4096))))),
        (f"reduceSum axis 1 [{R},4096]", 4 * G, lambda: ops.reduceSum(None, None, rows, red_rows, 1)),
        (f"reduceSum axis 0 [{R},4096]", 4 * G, lambda: ops.reduceSum(None, None, rows, red_cols, 0)),
        (f"maskedSoftmax [{S},1,1024,1024]", 3 * 4 * (S << 20),
         lambda: nn.maskedSoftmax(None, None, sm_in, sm_mask, sm_out, 3)),
        (f"softmax [{S},1,1024,1024]", 2 * 4 * (S << 20), lambda: nn.softmax(None, None, sm_in, sm_out, 3)),
    ]
    if S >= 16:  # rows of 4096 (one CTA's registers) and 16384 (one CTA's shared memory)
        S4, S16 = S // 4, S // 16
        r4_in, r4_out = a[:S4 << 22].view(S4, 1, 1024, 4096), o[:S4 << 22].view(S4, 1, 1024, 4096)
        r16_in, r16_out = a[:S16 << 24].view(S16, 1, 1024, 16384), o[:S16 << 24].view(S16, 1, 1024, 16384)
        cases.append((f"causalSoftmax [{S4},1,1024,4096]", 2 * 4 * (S4 << 22),
                      lambda: nn.causalSoftmax(None, None, r4_in, r4_out, 3, 2, 3)))
        cases.append((f"softmax [{S16},1,1024,16384]", 2 * 4 * (S16 << 24),
                      lambda: nn.softmax(None, None, r16_in, r16_out, 3)))
    if S >= 64:  # decode-shaped rows of 32768 keys (128 KiB, streamed): c5's softmax, twice over
        r32_in, r32_out = a[:1 << 26].view(32, 64, 1, 32768), o[:1 << 26].view(32, 64, 1, 32768)
        cases.append(("softmax [32,64,1,32768]", 2 * 4 * (1 << 26), lambda: nn.softmax(None, None, r32_in, r32_out, 3)))
    # the attention path's own HBM-bound calls: embeddingLookup, rmsNorm, the
    # two fused into one launch, ropeInPlace on Q and K, ops::scale
    H = 4096
    ntok = R // 2  # gathered rows: half of a [R, 4096] table
    table = a.view(R, H)
    ids = torch.randint(0, R, (ntok,), device=dev, dtype=torch.int32)
    emb_out = o[:ntok * H].view(ntok, H)
    norm_w = torch.rand(H, device=dev) + 0.5
    heads, hd = 32, 128
    T = G // 2 // (heads * hd)  # Q and K: half of an operand each
    rq, rk = a[:G // 2].view(1, T, heads, hd), b[:G // 2].view(1, T, heads, hd)
    ang = torch.arange(T, device=dev, dtype=torch.float64)[:, None] * torch.pow(
        10000.0, -2.0 * torch.arange(hd // 2, device=dev, dtype=torch.float64) / hd)[None, :]
    cos_t, sin_t = torch.cos(ang).float(), torch.sin(ang).float()
    cases += [
        (f"embeddingLookup [{ntok}] of [{R},{H}]", 2 * 4 * ntok * H + 4 * ntok,
         lambda: nn.embeddingLookup(None, None, ids, table, emb_out)),
        (f"rmsNorm [{R},{H}]", 2 * 4 * G, lambda: nn.rmsNorm(None, None, rows, norm_w, o.view(R, H), 1e-5)),
        (f"embeddingLookup+rmsNorm [{ntok}] of [{R},{H}]", 2 * 4 * ntok * H + 4 * ntok,
         lambda: nn.embeddingRmsNorm(None, None, ids, table, norm_w, emb_out, 1e-5)),
        (f"ropeInPlace Q,K [1,{T},{heads},{hd}]", 2 * 2 * 4 * (G // 2) + 2 * 4 * T * (hd // 2),
         lambda: nn.ropeInPlace(None, None, rq, rk, cos_t, sin_t)),
        ("scale", 2 * 4 * G, lambda: ops.scale(None, None, a, 0.5, o)),
    ]
    for name, nbytes, fn in cases:
        t = timed(fn)
        print(json.dumps({"op": name, "dtype": "f32", "ms": round(t * 1e3, 4), "GBps": round(nbytes / t / 1e9, 1),
                          "frac_of_hbm_peak": round(nbytes / t / 1e9 / peak, 3), "peak_GBps": peak,
                          "peak_kind": kind, "bytes_per_launch": nbytes}), flush=True)
    # the drop-in attentionScores / attentionApply (scores materialised, as the
    # reference does): one c3-like slice, B 1, T 4096, 8 heads of 128, fp32,
    # against the nominal FP32 SIMT peak (148 SMs x 128 lanes x 2 x 1965 MHz);
    # a fixed shape (512 MiB of scores) whatever --ops-elems is
    Tq, Hs, Dh = 4096, 8, 128
    q4 = torch.randn((1, Tq, Hs, Dh), device=dev)
    k4 = torch.randn((1, Tq, Hs, Dh), device=dev)
    s4 = torch.empty((1, Hs, Tq, Tq), device=dev)
    o4 = torch.empty((1, Tq, Hs, Dh), device=dev)
    simt_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    flops = 2 * Hs * Tq * Tq * Dh
    for name, fn in ((f"attentionScores Q,K [1,{Tq},{Hs},{Dh}] -> S [1,{Hs},{Tq},{Tq}]",
                      lambda: nn.attentionScores(None, None, q4, k4, s4)),
                     (f"attentionApply P [1,{Hs},{Tq},{Tq}], V [1,{Tq},{Hs},{Dh}]",
                      lambda: nn.attentionApply(None, None, s4, k4, o4))):
        t = timed(fn, reps=5, warm=2)
        print(json.dumps({"op": name, "dtype": "f32", "ms": round(t * 1e3, 3), "TFLOPs": round(flops / t / 1e12, 2),
                          "frac_of_fp32_simt_nominal": round(flops / t / 1e12 / simt_peak, 3)}), flush=True)
    del q4, k4, s4, o4
    # the same two ops in fp64 at the c4 prefill shape (B 2, T 1024, 16 heads
    # of 64), against the DGEMM rate cuBLAS reaches on this GPU
    Tq, Hs, Dh = 1024, 16, 64
    q4 = torch.randn((2, Tq, Hs, Dh), device=dev, dtype=torch.float64)
    k4 = torch.randn((2, Tq, Hs, Dh), device=dev, dtype=torch.float64)
    s4 = torch.empty((2, Hs, Tq, Tq), device=dev, dtype=torch.float64)
    o4 = torch.empty((2, Tq, Hs, Dh), device=dev, dtype=torch.float64)
    ga, gb = torch.randn((4096, 4096), device=dev, dtype=torch.float64), torch.randn((4096, 4096), device=dev,
                                                                                   dtype=torch.float64)
    dgemm = 2 * 4096 ** 3 / timed(lambda: torch.mm(ga, gb), reps=3, warm=1) / 1e12
    del ga, gb
    flops = 2 * 2 * Hs * Tq * Tq * Dh
    for name, fn in ((f"attentionScores Q,K [2,{Tq},{Hs},{Dh}] -> S [2,{Hs},{Tq},{Tq}] f64",
                      lambda: nn.attentionScores(None, None, q4, k4, s4)),
                     (f"attentionApply P [2,{Hs},{Tq},{Tq}], V [2,{Tq},{Hs},{Dh}] f64",
                      lambda: nn.attentionApply(None, None, s4, k4, o4))):
        t = timed(fn, reps=5, warm=2)
        print(json.dumps({"op": name, "dtype": "f64", "ms": round(t * 1e3, 4), "TFLOPs": round(flops / t / 1e12, 2),
                          "frac_of_cublas_dgemm": round(flops / t / 1e12 / dgemm, 3),
                          "cublas_dgemm_tflops": round(dgemm, 1)}), flush=True)
    del q4, k4, s4, o4
    del a, b, o
    torch.cuda.empty_cache()
    if args.ops_elems != 1 << 28:
        return
    # the gated MLP and a 3-layer mlpForward at decoder-like shapes: cuBLAS
    # GEMMs plus this library's fused passes
    M, K, F = 4096, 4096, 14336
    x = torch.randn((M, K), device=dev) / 8
    wg, wu = torch.randn((K, F), device=dev) / 64, torch.randn((K, F), device=dev) / 64
    wd = torch.randn((F, K), device=dev) / 120
    out = torch.empty((M, K), device=dev)
    ws = torch.empty(2 * M * F * 4, dtype=torch.uint8, device=dev)
    t = timed(lambda: nn.mlp(None, None, x, wg, wu, wd, out, workspace=ws), reps=5, warm=2)
    flops = 2 * M * K * F * 3
    t_sw = timed(lambda: ops.swiglu(None, None, ws.view(f32)[:M * F], ws.view(f32)[M * F:], ws.view(f32)[:M * F]))
    print(json.dumps({"op": f"mlp (gated) x[{M},{K}] W[{K},{F}]", "dtype": "f32", "ms": round(t * 1e3, 3),
                      "TFLOPs": round(flops / t / 1e12, 1), "swiglu_pass_ms": round(t_sw * 1e3, 3),
                      "swiglu_share": round(t_sw / t, 3)}), flush=True)


def loader_only(args):
    """--loader MIB: GB/s of the artifact loader (onHost/core/binary.hpp) with
    the file in the page cache. Denominators measured in the same run: a
    pinned host->device copy (the copy-engine ceiling) and the reference's
    route (whole tensor read into one pageable host buffer, then copied)."""
    import tempfile
    import time

    import numpy as np
    import torch

    from alpakann_b200.onHost import core
    mib = args.loader
    n = (mib << 20) // 4
    rows, cols = 4096, n // 4096
    n = rows * cols
    nbytes = n * 4
    d = tempfile.mkdtemp(prefix="ann_loader_")
    path = os.path.join(d, "w.bin")
    rng = np.random.default_rng(1)
    rng.standard_normal(n, dtype=np.float32).tofile(path)
    spec = core.TensorSpec("w", 0, n, (rows, cols))
    torch.cuda.init()
    reps = max(args.steps, 1)

    def timed(fn):
        fn()  # warm: page cache, staging buffers, allocator
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            best = min(best, time.perf_counter() - t0)
        return best

    try:
        t_sha = timed(lambda: core.sha256File(path))
        out = {}
        t_load = timed(lambda: out.__setitem__("w", core.loadBinaryTensor(None, path, spec)))
        shard_cols = cols // 8
        t_box = timed(lambda: out.__setitem__("b", core.loadBinaryTensorBox(None, path, spec, (0, rows),
                                                                             (3 * shard_cols, shard_cols))))
        host_pinned = torch.empty(n, dtype=torch.float32, pin_memory=True)
        dev = torch.empty(n, dtype=torch.float32, device="cuda")
        t_h2d = timed(lambda: dev.copy_(host_pinned, non_blocking=True))

        def reference_route():
            host = np.fromfile(path, dtype=np.float32, count=n)  # one pageable host buffer
            dev.copy_(torch.from_numpy(host))
        t_ref = timed(reference_route)
        ok = torch.equal(out["w"].view(rows, cols)[:, 3 * shard_cols:4 * shard_cols], out["b"])
    finally:
        os.remove(path)
        os.rmdir(d)
    gbs = lambda b, t: round(b / t / 1e9, 2)  # noqa: E731
    print(json.dumps({
        "loader": {"file_mib": mib, "shape": [rows, cols], "dtype": "f32", "reps": reps, "timing": "best of reps, "
                   "wall clock around the call plus a device synchronize"},
        "sha256File_GBps": gbs(nbytes, t_sha),
        "loadBinaryTensor_GBps": gbs(nbytes, t_load),
        "box_1of8_columns_GBps": gbs(nbytes // 8, t_box),
        "pinned_h2d_GBps": gbs(nbytes, t_h2d),
        "reference_route_GBps": gbs(nbytes, t_ref),
        "load_frac_of_pinned_h2d": round(t_h2d / t_load, 3),
        "box_equals_slice": bool(ok)}), flush=True)


def main():
    args = parse()
    if args.ops:
        ops_only(args)
        return
    if args.loader:
        loader_only(args)
        return
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
        return
    if args.prefill_only:
        prefill_only(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    comm = None
    if world > 1:  # torch.distributed: rendezvous, barriers, max over ranks; the data path uses comm
        from alpakann_b200.comm import Comm
        from alpakann_b200.sharded import join
        join(rank, world, "nccl", timeout_s=120, device=torch.device("cuda", local))
        comm = Comm.from_torch(timeout_s=120)
    peak, peak_kind = peaks()

    def run(wl, steps, warmup, with_clocks):
        bench = DecodeBench(WORKLOADS[wl], rank, world, comm)
        elapsed, kernel_s, e2e_s, e2e_steps, clk = measure(bench, steps, warmup, world, rank, with_clocks)
        ww = WORKLOADS[wl]
        B, Tk, H, D = ww["B"], ww["Tk"], ww["H"], ww["D"]
        Hl = H // world
        alg = 2 * B * Hl * Tk * D * 4 + 2 * B * Hl * D * 4  # per launch per GPU: K+V read, Q read, O write
        res = dict(value=B * steps / elapsed, ms_per_step=elapsed / steps * 1e3, kernel_us=kernel_s * 1e6,
                   achieved=alg / kernel_s / 1e9, e2e=B / e2e_s, e2e_steps=e2e_steps, clk=clk,
                   copies=bench.copies, kv_mib=bench.kv_bytes / 2**20, launches=bench.launches_per_step * steps,
                   h2d=2 * B * Hl * D * 4 * world, d2h=B * H * D * 4 * world, alg=alg)
        bench.release()
        return res

    main_res = run(args.workload, args.steps, args.warmup, True)
    extra = {}
    if not args.no_extra:
        other = "c2" if args.workload == "c5" else "c5"
        o = run(other, max(10, args.steps if other == "c2" else args.steps // 16), args.warmup, False)
        extra[other] = {"workload": WORKLOADS[other]["desc"], "value": o["value"], "unit": "tokens/s",
                        "ms_per_step": o["ms_per_step"], "kernel_us": o["kernel_us"],
                        "achieved_gbs": o["achieved"], "frac": o["achieved"] / peak, "e2e": o["e2e"]}
        for name in ("c3", "c4"):
            extra[f"{name}_prefill"] = measure_prefill(name, world, rank, comm)

    if rank == 0:
        r = main_res
        cpu = None
        if world == 1:
            import oracle
            smp = cpu_sample_for(w)
            smp.step()
            cpu_step, reps = smp.time_full_steps(seconds=args.cpu_seconds)
            cpu = {"value": w["B"] / cpu_step, "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                   "sample": f"{smp.desc}; {reps} reps"}
        line = {
            "metric": "decode attn tokens/s", "value": r["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w["desc"], "batch": w["B"], "kv_len": w["Tk"], "heads": w["H"],
                       "head_dim": w["D"],
                       "parallelism": f"head-sharded x{world}" + (" + NCCL all-gather" if world > 1 else ""),
                       "l2": f"inputs larger than L2: {r['copies']} KV cache cop{'y' if r['copies'] == 1 else 'ies'} "
                             f"of {r['kv_mib']:.0f} MiB per GPU, rotated per step"},
            "roofline": {"bound": "hbm", "achieved": r["achieved"], "peak": peak, "unit": "GB/s",
                         "frac": r["achieved"] / peak,
                         "traffic": ncu_traffic(args.workload) if world == 1 else None,
                         "peak_kind": peak_kind, "kernel": "decode_kernel<float,128>",
                         "kernel_us": r["kernel_us"], "alg_bytes_per_launch": r["alg"],
                         "frac_of_8TBs_nominal": r["achieved"] / 8000.0},
            "cpu_baseline": cpu,
            "e2e": {"value": r["e2e"], "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"], "steps": r["e2e_steps"]},
            "gpu_launches": r["launches"],
            "clocks": r["clk"],
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
