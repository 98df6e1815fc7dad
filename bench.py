"""Benchmark of the attention decode step (one JSON line on rank 0).

Headline workload (c5): batch 16, one query token per sequence, KV cache of
32768 tokens, 64 heads x head_dim 128, fp32, BHTD cache (32 GiB of K+V). Each
step normalises the step's hidden states (rmsNorm), rotates Q and the new K
row with RoPE (theta 5e5) at position 32768 and runs fused decode attention
(scores -> scale 1/sqrt(128) -> softmax -> apply) over the cache. With N GPUs
the heads are sharded (64/N per GPU, each GPU holds only its heads' cache)
and every rank's decode kernel stores its heads into every rank's full
[B,1,H,D] output through NVLink multicast, then one signal barrier (NCCL
all-gather + re-assembly where the node has no multicast): total work is
fixed, so the scaling is strong. The timed steps are replays of the step
captured in a CUDA graph (the launched step is reported beside it). The same
line carries, under "extra", the smaller decode workload c2 (batch 8, cache
2048, 32 heads x 128) measured the same way, and the c3 / c4 prefills.

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
    p.add_argument("--decode-only", metavar="B,Tk,H,D", default=None,
                   help="run only the fused decode kernel on this BHTD cache shape (--steps launches, fp32) and print "
                        "its time; the small case the decode ncu captures use")
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


def tf32_peak(sustained=False):
    """Dense tf32 tensor TFLOP/s: half the measured bf16 rate (B200 runs
    kind::tf32 at half the kind::f16 rate), burst (a kernel timed alone) or
    sustained (seconds of back-to-back GEMMs under the 1 kW power cap), else
    half the fallback (1.59 PFLOP/s burst, 1.4 sustained)."""
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)[key]) / 2, f"measured {key} / 2"
    except Exception:
        return (1400.0 if sustained else 1590.0) / 2, "fallback bf16 / 2"


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
    """nvidia-smi sampler (every 50 ms) of the GPUs this run uses, started
    before the timed region; stop() keeps the samples taken inside it."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.samples = []
        self.gpus = gpu_ids
        sel = ["-i", ",".join(gpu_ids)] if gpu_ids else []
        try:
            self.proc = subprocess.Popen(["nvidia-smi"] + sel + [f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        inside = [s for ts, s in self.samples if t0 <= ts <= t1]
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
                "reasons": sorted(reasons), "samples": len(sm), "gpus": len(self.gpus) if self.gpus else "all",
                "window_s": round(t1 - t0, 3), "interval_ms": 50}


def gpu_ids(world):
    """nvidia-smi ids (UUIDs) of the GPUs of every rank, if nvidia-smi accepts them."""
    import torch
    import torch.distributed as dist
    uuid = "GPU-" + str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
    ids = [uuid]
    if world > 1:
        ids = [None] * world
        dist.all_gather_object(ids, uuid)
    try:
        r = subprocess.run(["nvidia-smi", "-i", ",".join(ids), "--query-gpu=index", "--format=csv,noheader"],
                           capture_output=True, text=True, timeout=20)
        if r.returncode == 0 and len(r.stdout.split()) == len(ids):
            return ids
    except (OSError, subprocess.TimeoutExpired):
        pass
    return None


# ------------------------------------------------------------------ CPU ---
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class CpuSample:
    """The oracle's per-op decode pipeline (RoPE on Q and the new K row,
    attentionScores, scale, softmax, attentionApply) for ONE sequence of the
    batch with all of its heads, inputs prepared once. One sample step decodes
    one token; its K/V (2 GiB for the 32768-key cache) stream from DRAM on
    every step, as the full batch would."""

    def __init__(self, w):
        import numpy as np

        import oracle
        self.oracle = oracle
        B, Tk, H, D = w["B"], w["Tk"], w["H"], w["D"]
        g = np.random.default_rng(0)
        f32 = np.float32
        self.q = g.standard_normal((1, 1, H, D), dtype=f32)
        self.kn = g.standard_normal((1, 1, H, D), dtype=f32)
        # K / V: N(0,1) draws for 4 heads, repeated over the others (the timed
        # loops do not depend on the values; every head still has its own
        # memory, so the whole sample streams from DRAM)
        self.k = np.empty((1, H, Tk, D), f32)
        self.v = np.empty((1, H, Tk, D), f32)
        base = min(H, 4)
        kb, vb = (g.standard_normal((base, Tk, D), dtype=f32) for _ in range(2))
        for h in range(H):
            self.k[0, h] = kb[h % base]
            self.v[0, h] = vb[h % base]
        ang = np.arange(Tk + 1, dtype=np.float64)[:, None] * np.power(w["theta"], -2.0 * np.arange(D // 2) / D)[None]
        self.cos, self.sin = np.cos(ang).astype(f32), np.sin(ang).astype(f32)
        self.s = np.empty((1, H, 1, Tk), f32)
        self.p = np.empty_like(self.s)
        self.o = np.empty_like(self.q)
        self.rq, self.rk = np.empty_like(self.q), np.empty_like(self.kn)
        self.scale = f32(1.0 / math.sqrt(D))
        self.Tk = Tk
        self.kv_mib = 2 * self.k.nbytes / 2**20
        self.desc = (f"one step = 1 of the {B} sequences with all {H} heads ({self.kv_mib:.0f} MiB of K/V streamed "
                     f"from DRAM), the oracle's per-element loops on {{cores}} OpenMP threads; tokens/s = sequences/s")

    def step(self):
        o = self.oracle
        o.rope(self.q, self.cos, self.sin, self.rq, 0, self.Tk)
        o.rope(self.kn, self.cos, self.sin, self.rk, 0, self.Tk)
        o.attention_scores(self.rq, self.k, self.s, 1, 1)
        o.scale(self.s, self.scale, self.s)
        o.softmax(self.s, self.p, 3)
        o.attention_apply(self.p, self.v, self.o, 1, 1)

    def time_steps(self, seconds=None, steps=None):
        """Seconds per sample step (one token)."""
        reps, t0 = 0, time.perf_counter()
        while (steps is not None and reps < steps) or (seconds is not None and
                                                       (reps == 0 or time.perf_counter() - t0 < seconds)):
            self.step()
            reps += 1
        return (time.perf_counter() - t0) / reps, reps


def decode_config(w):
    """The `config` both arms print (identical, so the two lines compare)."""
    return {"workload": w["desc"], "batch": w["B"], "kv_len": w["Tk"], "heads": w["H"], "head_dim": w["D"],
            "l2": "every step streams a K/V working set larger than the last-level cache (GPU: the KV cache, "
                  "rotated over copies when a shard is smaller than 3x L2; CPU: one sequence's K/V, 2 GiB at "
                  "32768 keys)"}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    cores = host_cores()
    oracle.set_threads(cores)
    smp = CpuSample(w)
    for _ in range(args.warmup):
        smp.step()
    step, _ = smp.time_steps(steps=args.steps)
    value = 1.0 / step  # one token per sample step
    line = {"impl": "reference", "metric": "decode attn tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_config(w),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                             "sample": smp.desc.format(cores=oracle.max_threads())},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU ---
class DecodeE2E(ctypes.Structure):
    """struct DecodeE2E of tests/cpp/decode_e2e.cpp (the step through the C++ drop-in header)."""
    _fields_ = [("B", ctypes.c_int32), ("Hl", ctypes.c_int32), ("H", ctypes.c_int32), ("Tk", ctypes.c_int32),
                ("D", ctypes.c_int32), ("dm", ctypes.c_int32), ("eps", ctypes.c_float), ("scale", ctypes.c_float),
                ("position", ctypes.c_uint32),
                ("h_q", ctypes.c_void_p), ("h_knew", ctypes.c_void_p), ("h_hidden", ctypes.c_void_p),
                ("h_out", ctypes.c_void_p), ("q", ctypes.c_void_p), ("knew", ctypes.c_void_p),
                ("hidden", ctypes.c_void_p), ("normed", ctypes.c_void_p), ("norm_w", ctypes.c_void_p),
                ("cos_t", ctypes.c_void_p), ("sin_t", ctypes.c_void_p), ("k_caches", ctypes.c_void_p),
                ("v_caches", ctypes.c_void_p), ("n_caches", ctypes.c_int32), ("out", ctypes.c_void_p),
                ("head0", ctypes.c_int32), ("out_mirror", ctypes.c_void_p), ("signals", ctypes.c_void_p),
                ("peer_signals", ctypes.c_void_p), ("nranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("epoch_word", ctypes.c_void_p), ("timeout_ns", ctypes.c_uint64)]


def e2e_library():
    """tests/cpp/_build/libdecode_e2e.so (built by tests/cpp/build.py), or None."""
    path = os.path.join(ROOT, "tests", "cpp", "_build", "libdecode_e2e.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    lib.decode_e2e_run.argtypes = [ctypes.POINTER(DecodeE2E), ctypes.c_int, ctypes.c_void_p,
                                   ctypes.POINTER(ctypes.c_float)]
    lib.decode_e2e_error.restype = ctypes.c_char_p
    return lib


class DecodeBench:
    """Inputs and the two step flavours (device-resident and end-to-end) of
    the head-sharded decode workload on this rank."""

    def __init__(self, w, rank, world, comm):
        import numpy as np
        import torch

        import alpakann_b200 as ann
        from alpakann_b200 import _capi
        from alpakann_b200.sharded import HeadShard, HeadShardedDecode
        self.torch, self.capi, self.w, self.ann = torch, _capi, w, ann
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
        # the path starts with rmsNorm of the step's hidden states [B, d_model]
        # (eps 1e-5, weight 1 + N(0, 0.02)), replicated on every rank
        dm = H * D
        self.hidden = torch.randn((B, dm), generator=gen, dtype=f32, device="cuda")
        self.norm_w = 1.0 + 0.02 * torch.randn((dm,), generator=gen, dtype=f32, device="cuda")
        self.normed = torch.empty_like(self.hidden)
        self.eps = 1e-5
        self.sharded = HeadShardedDecode(self.shard, B, D, f32, "cuda", comm)
        self.comm = comm
        self.stream = torch.cuda.current_stream()
        self.queue = ann.Queue(self.stream)
        # descriptors built once: the device-timed loop only issues C-ABI calls
        V = _capi.view
        self.vq, self.vkn, self.vcos, self.vsin = V(self.q), V(self.knew), V(self.cos), V(self.sin)
        self.vh, self.vw, self.vn = V(self.hidden), V(self.norm_w), V(self.normed)
        self.vout = V(self.sharded.out if world == 1 else self.sharded.out_local)
        self.vkv = [(V(k), V(v)) for k, v in self.caches]
        self.gather = self.sharded.gather
        if self.gather == "nccl":
            self.vsrc, self.vdst = V(self.sharded._src), V(self.sharded._dst)
        # rmsNorm, rope, decode (+ re-assembly after NCCL, whose own kernel is not
        # counted; or the signal barrier after the multicast stores)
        self.launches_per_step = 3 if world == 1 else 4
        self.gather_bytes = self.sharded.out_local.numel() * 4
        # pinned host buffers of the end-to-end step
        self.hq = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
        self.hk = torch.randn((B, 1, Hl, D), dtype=f32).pin_memory()
        self.hh = torch.randn((B, dm), dtype=f32).pin_memory()
        self.hout = torch.empty((B, 1, H, D), dtype=f32).pin_memory()
        self.h2d_bytes = (self.hq.numel() + self.hk.numel() + self.hh.numel()) * 4
        self.d2h_bytes = self.hout.numel() * 4

    def step(self, i, ev=None):
        lib, R, sh, chk = self.capi.lib, ctypes.byref, self.stream.cuda_stream, self.capi.check
        chk(lib.ann_rms_norm_f32(sh, R(self.vh), R(self.vw), R(self.vn), self.eps))
        chk(lib.ann_rope_inplace_f32(sh, R(self.vq), R(self.vkn), R(self.vcos), R(self.vsin), 0, self.w["Tk"]))
        vk, vv = self.vkv[i % self.copies]
        if ev is not None:
            ev[0].record(self.stream)
        if self.gather == "multicast":  # every rank's heads go to every rank's copy from inside the kernel
            chk(lib.ann_attention_decode_mirror_f32(sh, R(self.vq), R(vk), R(vv), R(self.vout),
                                                    ctypes.c_void_p(self.sharded._out_mc), self.scale, 1, 1))
        else:
            chk(lib.ann_attention_decode_f32(sh, R(self.vq), R(vk), R(vv), R(self.vout), self.scale, 1, 1))
        if ev is not None:
            ev[1].record(self.stream)
        if self.gather == "multicast":
            self.sharded.mirror.barrier(self.queue)
        elif self.gather == "nccl":  # this library's NCCL all-gather, then the re-assembly kernel
            chk(lib.ann_comm_allgather(self.comm._h, sh, self.sharded.out_local.data_ptr(),
                                       self.sharded.gathered.data_ptr(), self.gather_bytes))
            chk(lib.ann_scale_f32(sh, R(self.vsrc), 1.0, R(self.vdst)))

    def capture_graphs(self):
        """The device-resident step captured in CUDA graphs, one per cache copy
        (rmsNorm, RoPE, decode and, across ranks, the multicast stores and the
        signal barrier, whose epoch lives in device memory so that every replay
        is a new epoch), on a stream of their own: (graphs, stream), or None
        for the NCCL gather (not captured) or where capture fails."""
        torch = self.torch
        if self.gather == "nccl":
            return None
        s = torch.cuda.Stream()
        s.wait_stream(self.stream)
        saved = self.stream, self.queue
        self.stream, self.queue = s, self.ann.Queue(s)
        graphs = []
        try:
            for i in range(self.copies):  # uncaptured warm-up on the capturing stream
                self.step(i)
            s.synchronize()
            for i in range(self.copies):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    self.step(i)
                graphs.append(g)
        except Exception as e:  # noqa: BLE001 -- report and time the launched step instead
            print(f"graph capture failed, timing launched steps: {e}", file=sys.stderr)
            torch.cuda.synchronize()
            return None
        finally:
            self.stream, self.queue = saved
        return graphs, s

    def cpp_e2e_setup(self):
        """The DecodeE2E record for the C++ step (None where it does not apply:
        no library, or the NCCL gather, which the C++ step does not run)."""
        lib = e2e_library()
        if lib is None or self.gather == "nccl":
            return None
        w, sh = self.w, self.sharded
        st = DecodeE2E()
        st.B, st.Hl, st.H, st.Tk, st.D, st.dm = w["B"], self.shard.local_heads, w["H"], w["Tk"], w["D"], w["H"] * w["D"]
        st.eps, st.scale, st.position = self.eps, self.scale, w["Tk"]
        st.h_q, st.h_knew, st.h_hidden, st.h_out = (t.data_ptr() for t in (self.hq, self.hk, self.hh, self.hout))
        st.q, st.knew, st.hidden, st.normed = (t.data_ptr() for t in (self.q, self.knew, self.hidden, self.normed))
        st.norm_w, st.cos_t, st.sin_t = self.norm_w.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr()
        self._kp = (ctypes.c_void_p * self.copies)(*[k.data_ptr() for k, _ in self.caches])
        self._vp = (ctypes.c_void_p * self.copies)(*[v.data_ptr() for _, v in self.caches])
        st.k_caches, st.v_caches = ctypes.cast(self._kp, ctypes.c_void_p), ctypes.cast(self._vp, ctypes.c_void_p)
        st.n_caches = self.copies
        st.out = sh.out.data_ptr()
        st.head0 = self.shard.head_slice.start if self.world > 1 else 0
        st.nranks, st.rank = self.world, self.shard.rank
        if self.gather == "multicast":
            m = sh.mirror
            st.out_mirror, st.signals, st.peer_signals = sh._out_mc, m._sig.data_ptr(), m._peer_sig.data_ptr()
            st.epoch_word, st.timeout_ns = m.epoch_word, m.timeout_ns
        self._e2e_lib, self._e2e = lib, st
        return st

    def cpp_e2e(self, steps):
        """`steps` decode steps through the C++ drop-in header with host buffers;
        returns the device seconds between events around them."""
        st = self._e2e
        ms = ctypes.c_float(0)
        rc = self._e2e_lib.decode_e2e_run(ctypes.byref(st), steps, ctypes.c_void_p(self.stream.cuda_stream),
                                          ctypes.byref(ms))
        if rc != 0:
            raise RuntimeError("C++ decode step: " + self._e2e_lib.decode_e2e_error().decode())
        return ms.value / 1e3

    def e2e_step(self, i):
        """Through the public Python API, with the step's inputs copied from
        pinned host memory and the full output read back."""
        self.q.copy_(self.hq, non_blocking=True)
        self.knew.copy_(self.hk, non_blocking=True)
        self.hidden.copy_(self.hh, non_blocking=True)
        self.ann.onHost.nn.rmsNorm(self.queue, None, self.hidden, self.norm_w, self.normed, self.eps)
        k, v = self.caches[i % self.copies]
        out = self.sharded.step(self.queue, self.q, self.knew, k, v, self.cos, self.sin, self.w["Tk"], self.scale)
        self.hout.copy_(out, non_blocking=True)

    def check_parity(self, seqs=2):
        """One step, then the gathered output of `seqs` sequences (all heads of
        every rank) against an fp64 recomputation on the device of each
        rank's own heads (rotated q, that rank's K/V cache), and the rmsNorm
        output against an fp64 recomputation. Tolerance |a-b| <= 1e-4|b| + 1e-5.
        Returns the worst error over ranks, as a fraction of the tolerance."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        self.e2e_step(0)
        torch.cuda.synchronize()
        out = self.hout.clone()
        k, v = self.caches[0]
        f64 = torch.float64
        B = self.w["B"]
        sel = [0, B - 1][:seqs]
        q = self.q[sel].to(f64)  # [s, 1, Hl, D], rotated in place by the step
        ref = []
        for j, b in enumerate(sel):
            s_ = torch.einsum("hd,htd->ht", q[j, 0], k[b].to(f64)) * self.scale
            p_ = torch.softmax(s_, dim=-1)
            ref.append(torch.einsum("ht,htd->hd", p_, v[b].to(f64)))
        ref = torch.stack(ref)[:, None]  # [s, 1, Hl, D]
        if self.world > 1:
            parts = [torch.empty_like(ref) for _ in range(self.world)]
            dist.all_gather(parts, ref.contiguous())
            ref = torch.cat(parts, dim=2)
        got = out[sel].to(f64).cuda()
        worst = float(((got - ref).abs() / (1e-4 * ref.abs() + 1e-5)).max())
        x = self.hh.to(f64).cuda()
        nref = x * torch.rsqrt((x * x).mean(dim=1, keepdim=True) + self.eps) * self.norm_w.to(f64)
        worst_n = float(((self.normed.to(f64) - nref).abs() / (1e-4 * nref.abs() + 1e-5)).max())
        t = torch.tensor([worst, worst_n], dtype=f64, device="cuda")
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return {"ok": bool(t[0] <= 1.0 and t[1] <= 1.0), "decode_err_over_tol": float(t[0]),
                "rmsnorm_err_over_tol": float(t[1]),
                "sample": f"{len(sel)} of {B} sequences x all {self.w['H']} heads of the gathered output and the "
                          f"rmsNorm output, vs fp64 recomputation on each head's own rank; "
                          f"tolerance |a-b| <= 1e-4 |b| + 1e-5"}

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


def measure(bench, steps, warmup, world, rank, clock_ids, min_region_s=1.0, max_repeats=60):
    """W warm-up steps; then three repetitions of `steps` launched steps with
    CUDA events around every decode launch (the kernel's time for the
    roofline, and the launched step's time); then the timed loop of EXACTLY
    `steps` steps, the step replayed from a CUDA graph (launched where it
    cannot be captured), each repetition bracketed by a barrier and a device
    synchronize on both sides, repeated until the repetitions add up to about
    `min_region_s` (so that the clock sampler sees the GPUs busy). Device time
    per repetition = CUDA events on the stream the steps run on, max over
    ranks; the reported time is the median repetition."""
    import torch
    for i in range(warmup):
        bench.step(i)
    barrier(world)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launched, kernel_s = [], []
    for _ in range(3):
        barrier(world)
        start.record(bench.stream)
        for i in range(steps):
            bench.step(i, kev[i])
        end.record(bench.stream)
        barrier(world)
        el, ks = max_over_ranks([start.elapsed_time(end) / 1e3,
                                 sum(a.elapsed_time(b) for a, b in kev) / 1e3 / steps], world)
        launched.append(el)
        kernel_s.append(ks)
    captured = bench.capture_graphs()
    ok = max_over_ranks([0.0 if captured is not None else 1.0], world)[0] == 0.0  # all ranks replay, or none
    graphs, gs = captured if (ok and captured is not None) else (None, bench.stream)
    if graphs is not None:
        gs.wait_stream(bench.stream)
        with torch.cuda.stream(gs):
            for i in range(warmup):
                graphs[i % len(graphs)].replay()
    barrier(world)
    clocks = Clocks(clock_ids) if (clock_ids is not None and rank == 0) else None
    reps = []
    t_wall0 = time.time()
    repeats = max_repeats
    r = 0
    while r < repeats:
        barrier(world)
        start.record(gs)
        if graphs is not None:
            with torch.cuda.stream(gs):
                for i in range(steps):
                    graphs[i % len(graphs)].replay()
        else:
            for i in range(steps):
                bench.step(i)
        end.record(gs)
        barrier(world)
        el = max_over_ranks([start.elapsed_time(end) / 1e3], world)[0]
        reps.append(el)
        if r == 0:  # every rank takes the same repeat count
            repeats = int(max(1, min(max_repeats, math.ceil(min_region_s / max(el, 1e-6)))))
        r += 1
    t_wall1 = time.time()
    clk = clocks.stop(t_wall0, t_wall1) if clocks else None
    bench.stream.wait_stream(gs)
    elapsed = statistics.median(reps)
    kernel = statistics.median(kernel_s)
    launched_el = statistics.median(launched)
    if graphs is not None:
        torch.cuda.synchronize()
        del graphs

    # end to end: through the C++ drop-in header (alpaka::nn::onHost) with host
    # buffers where its step applies, else through the Python mirror of the API
    e2e_steps = max(1, min(steps, 1000))
    cpp = bench.cpp_e2e_setup() is not None
    if cpp:
        bench.cpp_e2e(min(warmup, 5) or 1)
        barrier(world)
        e2e_s = bench.cpp_e2e(e2e_steps) / e2e_steps
        barrier(world)
    else:
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
    e2e_s = max_over_ranks([e2e_s], world)[0]
    api = ("C++ alpaka::nn::onHost header (tests/cpp/decode_e2e.cpp)" if cpp else
           "Python mirror of alpaka::nn::onHost (alpakann_b200.onHost)")
    return elapsed, kernel, e2e_s, e2e_steps, clk, len(reps), (min(reps), max(reps)), api, launched_el, ok


GATHER_DESC = {"none": "", "nccl": " + NCCL all-gather + re-assembly",
               "multicast": " + NVLink multicast stores of every rank's heads from inside the kernel + signal barrier"}
GATHER_STEP = {"none": "", "nccl": " -> NCCL all-gather -> re-assembly into BTHD",
               "multicast": " (its output stores reach every rank's copy through NVSwitch multicast) -> signal barrier"}


PREFILL = {
    "c3": dict(B=4, T=4096, H=32, D=128, dtype="f32",
               desc="prefill: batch 4, seq 4096, 32 heads x 128, fp32, causal, scale 1/sqrt(128)"),
    "c4": dict(B=2, T=1024, H=16, D=64, dtype="f64",
               desc="prefill: batch 2, seq 1024, 16 heads x 64, fp64, causal, scale 1/8"),
}


def measure_prefill(name, world, rank, comm, clock_ids=None, reps=10, sustained_s=1.0, max_repeats=1000):
    """Fused causal prefill of this rank's heads (heads sharded over ranks) and,
    for N > 1, the gather of the outputs into every rank's BTHD output, timed
    with CUDA events; TFLOP/s counts QK^T + PV over the causal half including
    the diagonal, 4*B*H*D*T(T+1)/2, for the whole job. Two timings: `reps`
    launches after the parity check (a burst, the figure the line's ms /
    tflops report), then repetitions of `reps` launches for about
    `sustained_s` seconds with the clock sampler running (median repetition,
    max over ranks), the regime of a long prefill under the power cap."""
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
    out = sharded.run(queue, q, k, v, sc)
    parity = prefill_parity(out, q, k, v, sc, rank, world)
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
    clocks = Clocks(clock_ids) if (clock_ids is not None and rank == 0) else None
    t_wall0 = time.time()
    sus, repeats, r = [], max_repeats, 0
    while r < repeats:
        barrier(world)
        e0.record()
        for _ in range(reps):
            sharded.run(queue, q, k, v, sc)
        e1.record()
        barrier(world)
        el = max_over_ranks([e0.elapsed_time(e1) / 1e3 / reps], world)[0]
        sus.append(el)
        if r == 0:  # every rank takes the same repeat count
            repeats = int(max(1, min(max_repeats, math.ceil(sustained_s / max(el * reps, 1e-6)))))
        r += 1
    t_wall1 = time.time()
    clk = clocks.stop(t_wall0, t_wall1) if clocks else None
    ts = statistics.median(sus)
    sustained = {"ms": ts * 1e3, "tflops": flops / ts / 1e12, "repeats": len(sus), "launches_each": reps,
                 "seconds": round(t_wall1 - t_wall0, 3), "clocks": clk}
    gather = sharded.gather
    del q, k, v, out, sharded
    torch.cuda.empty_cache()
    res = {"workload": p["desc"], "ms": t * 1e3, "tflops": flops / t / 1e12, "tokens_per_s": B * T / t,
           "dtype": p["dtype"], "gathered": world > 1, "parallelism": f"head-sharded x{world}"
           + GATHER_DESC[gather].replace("decode", "prefill"), "parity": parity}
    if p["dtype"] == "f32":
        # 3xTF32: every useful flop costs three tf32 tensor flops
        pk, kind = tf32_peak()
        pair = os.environ.get("ANN_PREFILL_TC_PAIR", "1")[:1] != "0"
        name = (f"prefill_pair_kernel<{D}> (tcgen05 cta_group::2 on SM pairs, 3xTF32)" if pair
                else f"prefill_tc_kernel<{D}> (tcgen05 3xTF32)")
        pks, kinds = tf32_peak(sustained=True)
        sustained.update(tf32_peak_tflops=pks, tf32_peak_kind=kinds,
                         frac_of_3xtf32_sustained_peak=3 * sustained["tflops"] / world / pks)
        res.update(kernel=name, tf32_peak_tflops=pk, tf32_peak_kind=kind,
                   frac_of_3xtf32_peak=3 * res["tflops"] / world / pk, sustained=sustained)
    else:
        pk = fp64_gemm_tflops()
        res.update(kernel=f"prefill_f64_kernel<{D}> (FP64 tensor cores, mma.sync m16n8k4)", fp64_peak_tflops=pk,
                   fp64_peak_kind="cuBLAS DGEMM 4096^3, measured in this run",
                   frac_of_fp64_peak=res["tflops"] / world / pk, sustained=sustained)
    if world > 1:
        # fused compute + collective: the target time of a rank is the slower of
        # its useful flops at the compute ceiling and the bytes of the output that
        # must reach it over NVLink (every other rank's heads) at the measured
        # peer-copy rate of this pool, 770 GB/s per direction
        elem = 4 if p["dtype"] == "f32" else 8
        ingress = (world - 1) / world * B * T * H * D * elem
        ceiling = pk / 3 if p["dtype"] == "f32" else pk
        t_compute = flops / world / (ceiling * 1e12)
        t_link = ingress / 770e9
        target = max(t_compute, t_link)
        res["fused_roofline"] = {"target_ms": target * 1e3, "bound": "nvlink" if t_link >= t_compute else "compute",
                                 "compute_ms": t_compute * 1e3, "nvlink_ms": t_link * 1e3,
                                 "nvlink_bytes_per_gpu": ingress, "link_gbs": 770.0, "frac": target / t}
    return res


def measure_prefill_block(world, rank, comm, reps=5):
    """The c3 block as the path runs it (test/unit/nn/attention.cpp:856-974
    composes it): hidden states [B*T, d_model] -> rmsNorm (eps 1e-6, weight
    1 + N(0, 0.02)) -> qkvProjection (cuBLAS fp32 GEMMs, weights
    N(0, 1/sqrt(d_model)); column-parallel: this rank's heads' columns) ->
    ropeInPlace(Q, K) (theta 1e4) -> fused causal prefill of this rank's heads
    -> gather into every rank's BTHD output. CUDA events around each stage
    (max over ranks of the means); the attention TFLOP/s of the line's
    c3_prefill counts the attention stage alone."""
    import numpy as np
    import torch

    import alpakann_b200 as ann
    from alpakann_b200.sharded import HeadShard, HeadShardedPrefill
    B, T, H, D = 4, 4096, 32, 128
    dm, Hl, N = H * D, H // world, 4 * 4096
    gen = torch.Generator(device="cuda").manual_seed(99)
    x = torch.randn((N, dm), generator=gen, device="cuda")
    w = 1.0 + 0.02 * torch.randn((dm,), generator=gen, device="cuda")
    Ws = [torch.randn((dm, Hl * D), generator=gen, device="cuda") / math.sqrt(dm) for _ in range(3)]
    y = torch.empty_like(x)
    Q, K, V = (torch.empty((N, Hl * D), device="cuda") for _ in range(3))
    ang = np.arange(T, dtype=np.float64)[:, None] * np.power(1e4, -2.0 * np.arange(D // 2) / D)[None]
    cos, sin = torch.from_numpy(np.cos(ang)).float().cuda(), torch.from_numpy(np.sin(ang)).float().cuda()
    sharded = HeadShardedPrefill(HeadShard(rank, world, H, H), B, T, D, torch.float32, "cuda", comm)
    queue = ann.Queue()
    nn = ann.onHost.nn
    q4, k4, v4 = (t.view(B, T, Hl, D) for t in (Q, K, V))
    stages = ["rmsNorm", "qkvProjection", "ropeInPlace", "attention + gather"]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(stages) + 1)]
    acc = [0.0] * len(stages)

    def block(timed):
        if timed:
            ev[0].record()
        nn.rmsNorm(queue, None, x, w, y, 1e-6)
        if timed:
            ev[1].record()
        nn.qkvProjection(queue, y, Ws[0], Ws[1], Ws[2], Q, K, V)
        if timed:
            ev[2].record()
        nn.ropeInPlace(queue, None, q4, k4, cos, sin)
        if timed:
            ev[3].record()
        sharded.run(queue, q4, k4, v4, 1.0 / math.sqrt(D))
        if timed:
            ev[4].record()

    block(False)
    barrier(world)
    for _ in range(reps):
        block(True)
        torch.cuda.synchronize()
        for i in range(len(stages)):
            acc[i] += ev[i].elapsed_time(ev[i + 1]) / reps
    acc = max_over_ranks(acc, world)
    del x, y, Q, K, V, Ws, sharded
    torch.cuda.empty_cache()
    return {"workload": "prefill block: hidden [16384, 4096] -> rmsNorm -> qkvProjection -> ropeInPlace -> causal "
                        "attention [4, 4096, 32 x 128], fp32", "ms": sum(acc),
            "stages_ms": {n: round(t, 4) for n, t in zip(stages, acc)},
            "tokens_per_s": N / (sum(acc) / 1e3), "qkv": "cuBLAS fp32 GEMMs, column-parallel over the ranks"}


def prefill_parity(out, q, k, v, scale, rank, world, rows=(0, 1, 777, -1)):
    """The gathered prefill output at a few query rows of every batch and head
    against an fp64 recomputation on the device by the rank that owns the head
    (causal, top-left mask). Tolerance |a-b| <= rtol |b| + atol with the fp32
    (1e-4, 1e-5) or fp64 (1e-11, 1e-12) pair; returns the worst error as a
    fraction of the tolerance, max over ranks."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    f64 = torch.float64
    B, T, Hl, D = q.shape
    rtol, atol = (1e-4, 1e-5) if q.dtype == torch.float32 else (1e-11, 1e-12)
    idx = sorted({r % T for r in rows})
    ref = torch.empty((B, len(idx), Hl, D), dtype=f64, device="cuda")
    for j, i in enumerate(idx):
        qi = q[:, i].to(f64)                                   # [B, Hl, D]
        s_ = torch.einsum("bhd,bthd->bht", qi, k[:, :i + 1].to(f64)) * scale
        ref[:, j] = torch.einsum("bht,bthd->bhd", torch.softmax(s_, -1), v[:, :i + 1].to(f64))
    if world > 1:
        parts = [torch.empty_like(ref) for _ in range(world)]
        dist.all_gather(parts, ref)
        ref = torch.cat(parts, dim=2)
    got = out[:, idx].to(f64)
    worst = ((got - ref).abs() / (rtol * ref.abs() + atol)).max()
    if world > 1:
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    w = float(worst)
    return {"ok": w <= 1.0, "err_over_tol": w,
            "sample": f"query rows {idx} of every batch and all heads of the gathered output vs fp64 recomputation "
                      f"on each head's own rank; tolerance |a-b| <= {rtol:g} |b| + {atol:g}"}


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


def decode_only(args):
    """--decode-only B,Tk,H,D: fused decode launches on one GPU, CUDA-event timed."""
    import torch

    import alpakann_b200 as ann
    B, Tk, H, D = (int(x) for x in args.decode_only.split(","))
    gen = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn((B, 1, H, D), generator=gen, device="cuda")
    k, v = (torch.randn((B, H, Tk, D), generator=gen, device="cuda") for _ in range(2))
    o = torch.empty_like(q)
    queue = ann.Queue()
    lay = ann.AttentionKvLayout.BHTD
    for _ in range(args.warmup):
        ann.onHost.nn.attentionDecode(queue, None, q, k, v, o, None, 1, lay)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ann.onHost.nn.attentionDecode(queue, None, q, k, v, o, None, 1, lay)
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / max(args.steps, 1)
    alg = 2 * B * H * Tk * D * 4 + 2 * B * H * D * 4
    print(json.dumps({"decode": args.decode_only, "launches": args.steps, "us": t * 1e6, "alg_bytes": alg,
                      "GBps": alg / t / 1e9}), flush=True)


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
    # reference does): one c3-like slice, B 1, T 4096, 8 heads of 128, fp32 on
    # the tensor cores (3xTF32: three tf32 MMAs per useful product), against the
    # 3xTF32 ceiling = measured tf32 rate / 3; a fixed shape (512 MiB of
    # scores) whatever --ops-elems is
    Tq, Hs, Dh = 4096, 8, 128
    q4 = torch.randn((1, Tq, Hs, Dh), device=dev)
    k4 = torch.randn((1, Tq, Hs, Dh), device=dev)
    s4 = torch.empty((1, Hs, Tq, Tq), device=dev)
    o4 = torch.empty((1, Tq, Hs, Dh), device=dev)
    tf32, tf32_kind = tf32_peak()
    ceiling = tf32 / 3
    flops = 2 * Hs * Tq * Tq * Dh
    for name, fn in ((f"attentionScores Q,K [1,{Tq},{Hs},{Dh}] -> S [1,{Hs},{Tq},{Tq}]",
                      lambda: nn.attentionScores(None, None, q4, k4, s4)),
                     (f"attentionApply P [1,{Hs},{Tq},{Tq}], V [1,{Tq},{Hs},{Dh}]",
                      lambda: nn.attentionApply(None, None, s4, k4, o4))):
        t = timed(fn, reps=5, warm=2)
        print(json.dumps({"op": name, "dtype": "f32", "ms": round(t * 1e3, 3), "TFLOPs": round(flops / t / 1e12, 2),
                          "frac_of_3xtf32_ceiling": round(flops / t / 1e12 / ceiling, 3),
                          "ceiling_tflops": round(ceiling, 1), "ceiling_kind": tf32_kind + ", / 3"}), flush=True)
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
    if args.decode_only:
        decode_only(args)
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
    clock_ids = gpu_ids(world)

    def run(wl, steps, warmup, with_clocks, check=False):
        bench = DecodeBench(WORKLOADS[wl], rank, world, comm)
        parity = bench.check_parity() if check else None
        elapsed, kernel_s, e2e_s, e2e_steps, clk, nrep, spread, api, launched_el, graphed = measure(
            bench, steps, warmup, world, rank, clock_ids if with_clocks else None)
        ww = WORKLOADS[wl]
        B, Tk, H, D = ww["B"], ww["Tk"], ww["H"], ww["D"]
        Hl = H // world
        alg = 2 * B * Hl * Tk * D * 4 + 2 * B * Hl * D * 4  # per launch per GPU: K+V read, Q read, O write
        launched = {"value": B * steps / launched_el, "ms_per_step": launched_el / steps * 1e3,
                    "unit": "tokens/s", "how": "the same steps launched one call at a time (median of 3 repetitions)"}
        res = dict(value=B * steps / elapsed, ms_per_step=elapsed / steps * 1e3, kernel_us=kernel_s * 1e6,
                   achieved=alg / kernel_s / 1e9, e2e=B / e2e_s, e2e_steps=e2e_steps, clk=clk,
                   copies=bench.copies, kv_mib=bench.kv_bytes / 2**20, launches=bench.launches_per_step * steps,
                   h2d=bench.h2d_bytes, d2h=bench.d2h_bytes, alg=alg, parity=parity, repeats=nrep,
                   rep_ms=[x / steps * 1e3 for x in spread], gather=bench.gather, api=api, launched=launched,
                   graphed=graphed)
        bench.release()
        return res

    main_res = run(args.workload, args.steps, args.warmup, True, check=True)
    extra = {}
    if not args.no_extra:
        other = "c2" if args.workload == "c5" else "c5"
        o = run(other, max(10, args.steps if other == "c2" else args.steps // 16), args.warmup, False, check=True)
        extra[other] = {"workload": WORKLOADS[other]["desc"], "value": o["value"], "unit": "tokens/s",
                        "ms_per_step": o["ms_per_step"], "kernel_us": o["kernel_us"],
                        "achieved_gbs": o["achieved"], "frac": o["achieved"] / peak, "e2e": o["e2e"],
                        "parity": o["parity"], "step_replayed_from_cuda_graph": o["graphed"],
                        "launched": o["launched"]}
        for name in ("c3", "c4"):
            extra[f"{name}_prefill"] = measure_prefill(name, world, rank, comm, clock_ids)
        extra["c3_block"] = measure_prefill_block(world, rank, comm)

    if rank == 0:
        r = main_res
        cpu = None
        if world == 1:
            import oracle
            oracle.set_threads(host_cores())
            smp = CpuSample(w)
            smp.step()
            cpu_step, reps = smp.time_steps(seconds=args.cpu_seconds)
            cpu = {"value": 1.0 / cpu_step, "unit": "tokens/s", "cores": oracle.max_threads(), "kind": "port",
                   "sample": smp.desc.format(cores=oracle.max_threads()) + f"; {reps} steps"}
        line = {
            "metric": "decode attn tokens/s", "value": r["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_config(w),
            "parallelism": f"head-sharded x{world}" + GATHER_DESC[r["gather"]],
            "step": "rmsNorm [B, d_model] -> ropeInPlace(Q, new K row) -> fused decode over this rank's KV cache"
                    + GATHER_STEP[r["gather"]],
            "timing": {"repeats": r["repeats"], "each": f"{args.steps} steps between barriers + synchronize",
                       "steps_run_as": ("replays of the step captured in a CUDA graph (rmsNorm, RoPE, decode"
                                        + (", multicast stores, signal barrier" if world > 1 else "") + ")"
                                        if r["graphed"] else "launched steps"),
                       "reported": "median repetition (max over ranks)", "min_max_ms_per_step": r["rep_ms"],
                       "kv_cache_copies": r["copies"], "kv_mib_per_gpu": r["kv_mib"]},
            "parity": r["parity"],
            "roofline": {"bound": "hbm", "achieved": r["achieved"], "peak": peak, "unit": "GB/s",
                         "frac": r["achieved"] / peak,
                         "traffic": ncu_traffic(args.workload) if world == 1 else None,
                         "peak_kind": peak_kind, "kernel": "decode_kernel<float,128>",
                         "kernel_us": r["kernel_us"], "alg_bytes_per_launch": r["alg"],
                         "frac_of_8TBs_nominal": r["achieved"] / 8000.0},
            "cpu_baseline": cpu,
            "e2e": {"value": r["e2e"], "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"], "steps": r["e2e_steps"], "api": r["api"]},
            "gpu_launches": r["launches"] * r["repeats"],
            "launched": r["launched"],
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
