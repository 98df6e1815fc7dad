"""Benchmark of the attention decode step (one JSON line on rank 0).

Workload (default): batch 8, one query token per sequence, KV cache of 2048
tokens, 32 heads x head_dim 128, fp32, BHTD cache; each step rotates Q and the
new K row with RoPE (theta 1e4) at position 2048 and runs fused decode
attention (scores -> scale 1/sqrt(128) -> softmax -> apply) over the cache.
With N GPUs the heads are sharded (32/N per GPU) and the per-head outputs are
all-gathered and re-assembled into [B,1,H,D] on every rank.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c2|c5]

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
               desc="decode: batch 16, 1 query token, KV cache 32768, 64 heads x 128, fp32, BHTD, RoPE 5e5 at "
                    "pos 32768"),
}
L2_BYTES = 126 * 1024 * 1024


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    p.add_argument("--steps", type=int, default=5000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU-baseline sample")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(workload):
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
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
        self.window = None
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

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        t0, t1 = self.window
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


def rope_tables(positions, D, theta, torch, dtype):
    import numpy as np
    pos = np.arange(positions, dtype=np.float64)[:, None]
    ang = pos * np.power(theta, -2.0 * np.arange(D // 2, dtype=np.float64) / D)[None, :]
    return (torch.from_numpy(np.cos(ang)).to(dtype).cuda(), torch.from_numpy(np.sin(ang)).to(dtype).cuda())


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


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    oracle.set_threads(os.cpu_count() or 1)
    # one sequence x all heads per step (1/B of the work) keeps --steps K bounded
    smp = CpuSample(w, 1, w["H"])
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
def main():
    args = parse()
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
        return
    import torch
    import torch.distributed as dist

    import alpakann_b200 as ann
    from alpakann_b200 import _capi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=120))
    B, Tk, H, D = w["B"], w["Tk"], w["H"], w["D"]
    if H % world:
        raise SystemExit(f"{H} heads do not shard over {world} GPUs")
    Hl = H // world
    f32 = torch.float32
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    kv_bytes = 2 * B * Hl * Tk * D * 4
    copies = max(1, math.ceil(3 * L2_BYTES / kv_bytes))  # rotate caches so each step reads cold HBM
    caches = [(torch.randn((B, Hl, Tk, D), generator=gen, dtype=f32, device="cuda"),
               torch.randn((B, Hl, Tk, D), generator=gen, dtype=f32, device="cuda")) for _ in range(copies)]
    q = torch.randn((B, 1, Hl, D), generator=gen, dtype=f32, device="cuda")
    knew = torch.randn((B, 1, Hl, D), generator=gen, dtype=f32, device="cuda")
    out = torch.empty((B, 1, Hl, D), dtype=f32, device="cuda")
    cos, sin = rope_tables(Tk + 1, D, w["theta"], torch, f32)
    full = torch.empty((B, 1, H, D), dtype=f32, device="cuda")
    gathered = torch.empty((world, B, 1, Hl, D), dtype=f32, device="cuda") if world > 1 else None
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    lib = _capi.lib

    # Descriptors built once: the timed loop only issues C-ABI calls.
    V = _capi.view
    vq, vkn, vout, vcos, vsin = V(q), V(knew), V(out), V(cos), V(sin)
    vkv = [(V(k), V(v)) for k, v in caches]
    if world > 1:
        # re-assembly: gathered[r, b, 0, h, d] -> full[b, 0, r*Hl + h, d] (a strided copy = scale by 1)
        vsrc = V(gathered.permute(1, 2, 0, 3, 4))
        vdst = V(full.view(B, 1, world, Hl, D))
    R = ctypes.byref

    def step(i, ev=None):
        _capi.check(lib.ann_rope_inplace_f32(sh, R(vq), R(vkn), R(vcos), R(vsin), 0, Tk))
        vk, vv = vkv[i % copies]
        if ev is not None:
            ev[0].record(stream)
        _capi.check(lib.ann_attention_decode_f32(sh, R(vq), R(vk), R(vv), R(vout), scale, 1, 1))
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)
            _capi.check(lib.ann_scale_f32(sh, R(vsrc), 1.0, R(vdst)))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        step(i)
    barrier()
    clocks = Clocks() if rank == 0 else None
    time.sleep(0.5 if clocks else 0)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t_wall0 = time.time()
    start.record(stream)
    for i in range(args.steps):
        step(i, kev[i])
    end.record(stream)
    barrier()
    t_wall1 = time.time()
    if clocks:
        clocks.mark(t_wall0, t_wall1)
    elapsed = start.elapsed_time(end) / 1e3
    kernel_s = sum(a.elapsed_time(b) for a, b in kev) / 1e3 / args.steps
    t = torch.tensor([elapsed, kernel_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed, kernel_s = float(t[0]), float(t[1])
    clk = clocks.stop() if clocks else None

    # ---- end to end through the public API with host buffers ----
    hq = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
    hk = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
    hout = torch.empty((B, 1, H, D), dtype=f32).pin_memory()
    nn = ann.onHost.nn
    queue = ann.Queue(stream)
    e2e_steps = min(args.steps, 2000)

    def e2e_step(i):
        q.copy_(hq, non_blocking=True)
        knew.copy_(hk, non_blocking=True)
        nn.ropeInPlace(queue, None, q, knew, cos, sin, ann.RopeLayout.BTHD, Tk)
        k, v = caches[i % copies]
        nn.attentionDecode(queue, None, q, k, v, out, scale, 1, ann.AttentionKvLayout.BHTD)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)
            ann.onHost.ops.scale(queue, None, gathered.permute(1, 2, 0, 3, 4), 1.0, full.view(B, 1, world, Hl, D))
            hout.copy_(full, non_blocking=True)
        else:
            hout.copy_(out, non_blocking=True)

    for i in range(min(args.warmup, 10)):
        e2e_step(i)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(stream)
    barrier()
    te = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te[0]) / e2e_steps

    if rank == 0:
        peak, peak_kind = peaks()
        alg_bytes = 2 * B * Hl * Tk * D * 4 + 2 * B * Hl * D * 4  # K+V + Q read + O write, per launch per GPU
        achieved = alg_bytes / kernel_s / 1e9
        traffic = ncu_traffic(args.workload) if world == 1 else None
        cpu = None
        if world == 1:
            import oracle
            smp = CpuSample(w, 1, w["H"])
            smp.step()
            cpu_step, reps = smp.time_full_steps(seconds=args.cpu_seconds)
            cpu = {"value": B / cpu_step, "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                   "sample": f"{smp.desc}; {reps} reps"}
        line = {
            "metric": "decode attn tokens/s", "value": B * args.steps / elapsed, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w["desc"], "batch": B, "kv_len": Tk, "heads": H, "head_dim": D,
                       "parallelism": f"head-sharded x{world}" + (" + NCCL all-gather" if world > 1 else ""),
                       "l2": f"inputs larger than L2: {copies} KV cache copies of {kv_bytes / 2**20:.0f} MiB per GPU "
                             f"rotated per step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "decode_kernel<float,128>", "kernel_us": kernel_s * 1e6,
                         "frac_of_8TBs_nominal": achieved / 8000.0},
            "cpu_baseline": cpu,
            "e2e": {"value": B / e2e_s, "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * B * Hl * D * 4 * world, "d2h_bytes_per_step": B * H * D * 4 * world,
                    "steps": e2e_steps},
            "gpu_launches": args.steps * (2 if world == 1 else 3),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
