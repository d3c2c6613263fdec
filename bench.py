#!/usr/bin/env python
"""Benchmark of the B200 affine INT8 quantized linear (batch-1 streaming chunks).

Workload (one "step"): one 60 s stream at batch 1 -- 54 chunks of 1120 ms --
through the quantized linears of all 24 FastConformer blocks (M = 14 frames
after 8x subsampling, d_model 1024, ff 4096), bf16 activations, INT8 weights
with group 64 and bf16 scale/bias, random init N(0, 0.02) quantised on the
device, 24 distinct weight sets (~640 MB, far larger than the 126 MB L2,
re-read by every chunk).  Per block, in data-dependency order: FFN1 up
(+SiLU) 1024->4096, FFN1 down 4096->1024, fused q|k|v 1024->3072, out
1024->1024, conv pointwise-1 1024->2048, pointwise-2 1024->1024, FFN2 up
(+SiLU), FFN2 down.  (The relative-position projection is not per chunk: its
input table is constant, so the encoder projects it once when its weights are
bound.)  The non-linear ops between the linears (attention core, GLU,
depthwise conv, LayerNorm) are not part of this workload; their inputs are
stood in by the producing linear's output of the same shape, so every launch
depends on the previous one as in the encoder.

metric: GB/s of algorithmic bytes (N*K weight bytes + 4*N*K/g scale/bias bytes
+ 2*M*K activation bytes + 2*M*N output bytes per linear) / device time.

The line also carries:
  linear   -- config 1: the single 4096x1024 linear at M = 14 over 40 distinct
              weight copies, launched back to back on one stream and as four
              independent streams, plus a sweep of N that separates K1's
              streaming rate from its fixed cost per launch;
  batched  -- the same 24 blocks at M = 896 (64 streams' chunks stacked: the
              tensor-core GEMM) and the FFN-up GEMM alone;
  encoder  -- the full streaming encoder + RNNT greedy decode at 64 streams
              per GPU for a 60 s stream (54 chunks), the encoder alone, and
              one stream.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank holds a full weight replica and runs its
own streams (no data-path collective; a barrier and a max-reduction of the
timings are the only communication).  --impl reference times the CPU
restatement of the reference's quantized_matmul (the oracle, OpenMP C, all
host cores) on the same 24-block workload with the same metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "catcher-tippi_b200"))

METRIC = "INT8 qlinear HBM GB/s (M=14) & encoder audio-sec/sec at 1/2/4/8 B200"
UNIT = "GB/s"
GROUP = 64
M_FRAMES = 14
N_BLOCKS = 24
ENCODER_LAYERS = 24
CHUNKS_PER_STEP = 54  # a 60 s stream: ceil(60 / 1.12) chunks

# name, N, K, rows, act, input (name of a producer or "x0")
BLOCK = [
    ("ffn1_up", 4096, 1024, M_FRAMES, "silu", "x0"),
    ("ffn1_down", 1024, 4096, M_FRAMES, "none", "ffn1_up"),
    ("qkv", 3072, 1024, M_FRAMES, "none", "ffn1_down"),
    ("out", 1024, 1024, M_FRAMES, "none", "qkv"),
    ("pw1", 2048, 1024, M_FRAMES, "none", "out"),
    ("pw2", 1024, 1024, M_FRAMES, "none", "pw1"),
    ("ffn2_up", 4096, 1024, M_FRAMES, "silu", "pw2"),
    ("ffn2_down", 1024, 4096, M_FRAMES, "none", "ffn2_up"),
]


def linear_bytes(n: int, k: int, m: int, g: int = GROUP) -> int:
    return n * k + 4 * n * k // g + 2 * m * k + 2 * m * n


def block_bytes(rows: int = M_FRAMES) -> int:
    return sum(linear_bytes(n, k, rows) for _, n, k, _, _, _ in BLOCK)


CHUNK_BYTES = N_BLOCKS * block_bytes()
LAUNCHES_PER_CHUNK = N_BLOCKS * len(BLOCK)
WORKLOAD = ("quantized linears of the 24-block FastConformer encoder at batch 1 (M=14), one 60 s "
            "stream = 54 chunks of 1120 ms per step, bf16, INT8 group 64, 24 distinct weight sets")


def set_blocks(n: int) -> None:
    """Fewer blocks for small profiling captures (the workload line says so)."""
    global N_BLOCKS, CHUNK_BYTES, LAUNCHES_PER_CHUNK, WORKLOAD
    N_BLOCKS = n
    CHUNK_BYTES = N_BLOCKS * block_bytes()
    LAUNCHES_PER_CHUNK = N_BLOCKS * len(BLOCK)
    WORKLOAD = WORKLOAD.replace("24-block", f"{n}-block").replace("24 distinct", f"{n} distinct")


# DRAM bytes (read + write) per algorithmic byte of K1, from one ncu capture of
# the 4096x1024 linear at M = 14 (4.515 MB for 4.600 MB algorithmic); traffic
# grows with the bytes a launch streams, so it is scaled to the average launch.
K1_TRAFFIC_PER_ALGO_BYTE = 4.5146e6 / 4599808


def _peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def measured_peak() -> tuple[float, str]:
    p = _peaks()
    return (float(p["hbm_gbs"]), "measured") if "hbm_gbs" in p else (6650.0, "fallback")


def measured_tensor_peak(sustained: bool = True) -> tuple[float, str]:
    p = _peaks()
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    if key in p:
        return float(p[key]), "measured"
    return (1400.0 if sustained else 1590.0), "fallback"


def max_over_ranks(dist, ms: float, device: str = "cuda") -> float:
    """The slowest rank's device time: every rank passes its own, all get the
    maximum (one all-reduce, taken by every rank in the same order)."""
    if dist is None:
        return ms
    import torch
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weak_scaling_value(world: int, units_per_rank: float, ms: float) -> float:
    """Whole-job throughput of a weak-scaling run: every rank processed the
    same units (bytes, audio seconds) and the job took the slowest rank's
    time, so value = world * units / max time."""
    return world * units_per_rank / (ms * 1e-3)


def host_threads() -> int:
    """Host cores this process may run on (the cgroup / affinity set)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------- clocks


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- GPU arm


class EncoderLinears:
    """Weights and activation buffers of the 24-block linear chain on one GPU.
    rows = 14 is one stream's chunk; rows = 896 stacks 64 streams' chunks."""

    def __init__(self, torch, cq, device: int, seed: int = 0, rows: int = M_FRAMES):
        self.torch, self.cq = torch, cq
        dev = torch.device("cuda", device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.layers = []  # [block][i] -> QuantizedLinear
        for _ in range(N_BLOCKS):
            blk = []
            for _, n, k, _, _, _ in BLOCK:
                w = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32) * 0.02
                q, s, b = cq.quantize(w, GROUP, "bf16")
                layer = cq.QuantizedLinear.from_device(q, s, b, None, GROUP, "bf16", device)
                layer.reserve(rows)  # batched-path workspace, before graph capture
                blk.append(layer)
                del w, q, s, b
            self.layers.append(blk)
        torch.cuda.synchronize()
        bf = torch.bfloat16
        self.rows = rows
        self.spec = [(nm, n, k, rows, act, src) for nm, n, k, _, act, src in BLOCK]
        self.x0 = torch.randn((rows, 1024), generator=gen, device=dev).to(bf)
        self.out = {name: torch.empty((rows, n), dtype=bf, device=dev)
                    for name, n, _, _, _, _ in self.spec}
        self.final = self.out["ffn2_down"]
        fn = cq.lib().cq_linear_forward_ex
        self._fn = fn
        self._calls = None

    def steps(self):
        """(layer, x, y, act, rows) of every linear of one chunk, in launch order."""
        out = []
        for b, blk in enumerate(self.layers):
            for layer, (name, n, k, m, act, src) in zip(blk, self.spec):
                if src == "x0":
                    x = self.x0 if b == 0 else self.out["ffn2_down"]
                else:
                    x = self.out[src]
                out.append((layer, x, self.out[name], act, m))
        return out

    def launch_chunk(self, stream_ptr: int) -> None:
        """All 24 blocks' linears, each consuming its producer's output, as
        C-ABI calls (cq_linear_forward_ex) with their argument tuples built
        once."""
        if self._calls is None or self._calls[0] != stream_ptr:
            acts = self.cq.ACTS
            self._calls = (stream_ptr, [
                (layer._h, ctypes.c_void_p(x.data_ptr()), x.stride(0), m,
                 ctypes.c_void_p(y.data_ptr()), y.stride(0), acts[act], ctypes.c_void_p(stream_ptr))
                for layer, x, y, act, m in self.steps()])
        fn = self._fn
        bad = 0
        for args in self._calls[1]:
            bad |= fn(*args)
        if bad:
            raise RuntimeError("cq_linear_forward_ex failed: " + self.cq.last_error())

    def launch_step(self, stream_ptr: int, chunks: int = 1) -> None:
        for _ in range(chunks):
            self.launch_chunk(stream_ptr)


class SingleLinear:
    """Config 1: x bf16 [14, K] . W[N, K]^T, group 64, over `copies` distinct
    weight copies (together larger than L2); every launch reads the same x and
    writes its own output."""

    def __init__(self, torch, cq, device: int, n: int = 4096, k: int = 1024, copies: int = 40,
                 seed: int = 0):
        dev = torch.device("cuda", device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.torch, self.cq, self.N, self.K, self.copies = torch, cq, n, k, copies
        self.layers = []
        for _ in range(copies):
            w = torch.randn((n, k), generator=gen, device=dev) * 0.02
            q, s, b = cq.quantize(w, GROUP, "bf16")
            self.layers.append(cq.QuantizedLinear.from_device(q, s, b, None, GROUP, "bf16", device))
            del w, q, s, b
        self.x0 = torch.randn((M_FRAMES, k), generator=gen, device=dev).to(torch.bfloat16)
        self.ys = [torch.empty((M_FRAMES, n), dtype=torch.bfloat16, device=dev)
                   for _ in range(copies)]
        self.final = self.ys[-1]
        self.bytes = linear_bytes(n, k, M_FRAMES)

    def launch_step(self, stream_ptr: int, branches=None) -> None:
        """One stream (branches None) or round-robin over the given streams."""
        for i, layer in enumerate(self.layers):
            sp = stream_ptr if branches is None else branches[i % len(branches)]
            layer.forward_raw(self.x0.data_ptr(), self.K, M_FRAMES, self.ys[i].data_ptr(), self.N,
                              "none", sp)


def capture(torch, fn, stream, branches: int = 0):
    """A CUDA graph of fn(stream_ptr) (or fn(stream_ptr, [branch stream ptrs])
    forked over `branches` side streams and joined again)."""
    with torch.cuda.stream(stream):
        if branches:
            side = [torch.cuda.Stream() for _ in range(branches)]
            fn(stream.cuda_stream, [s.cuda_stream for s in side])  # eager warm-up
        else:
            fn(stream.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        if branches:
            fork = torch.cuda.Event()
            fork.record(stream)
            for s in side:
                s.wait_event(fork)
            fn(stream.cuda_stream, [s.cuda_stream for s in side])
            for s in side:
                join = torch.cuda.Event()
                join.record(s)
                stream.wait_event(join)
        else:
            fn(stream.cuda_stream)
    torch.cuda.synchronize()
    return g


def time_replays(torch, g, steps: int, warmup: int, dist) -> float:
    """Device time of `steps` back-to-back replays (max over ranks), in ms."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    torch.cuda.nvtx.range_push("timed")  # profilers can select the timed launches
    s.record(cur)
    for _ in range(steps):
        g.replay()
    e.record(cur)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, s.elapsed_time(e))
    if dist:
        dist.barrier()
    return ms


def hbm_roofline(bytes_per_launch: float, launch_us: float, kernel: str, note: str) -> dict:
    peak, kind = measured_peak()
    achieved = bytes_per_launch / (launch_us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_kind": f"{kind} copy bandwidth",
            "traffic": round(K1_TRAFFIC_PER_ALGO_BYTE * bytes_per_launch),
            "traffic_note": "DRAM read+write bytes per launch, scaled from the ncu capture of "
                            "the 4096x1024 linear (0.981 of algorithmic)",
            "kernel": kernel, "avg_launch_us": round(launch_us, 3), "note": note}


def linear_object(torch, cq, args, local_rank: int, dist) -> dict:
    """Config 1 (the 4096x1024 linear at M = 14) and K1's streaming sweep."""
    res = {"workload": ("single INT8 affine quantized linear x bf16 [14,1024] . W[4096,1024]^T, "
                        "group 64, 40 distinct weight copies (184 MB, larger than L2) per step"),
           "metric": "GB/s", "bytes_per_launch": linear_bytes(4096, 1024, M_FRAMES)}
    lin = SingleLinear(torch, cq, local_rank)
    stream = torch.cuda.Stream()
    steps = max(args.steps, 20)
    for key, branches in (("serial", 0), ("concurrent", 4)):
        g = capture(torch, lin.launch_step, stream, branches)
        ms = time_replays(torch, g, steps, args.warmup, dist) / steps
        us = ms * 1e3 / lin.copies
        res[key] = {
            "value": round(lin.copies * lin.bytes / (ms * 1e-3) / 1e9, 2), "us_per_linear": round(us, 3),
            "how": ("40 launches back to back on one stream (programmatic dependent launch)"
                    if not branches else
                    "the 40 independent launches spread over 4 streams of one graph "
                    "(fork / join), so launches overlap")}
        del g
    res["roofline"] = hbm_roofline(lin.bytes, res["concurrent"]["us_per_linear"], "qgemv_kernel (K1)",
                                   "per-linear time of the concurrent launches")
    del lin
    # streaming sweep: per-launch time against bytes, serial launches over
    # enough distinct copies to exceed L2 twice
    pts = []
    for n in (4096, 16384, 65536):
        b = linear_bytes(n, 1024, M_FRAMES)
        copies = max(3, -(-260_000_000 // b))
        lin = SingleLinear(torch, cq, local_rank, n=n, copies=copies, seed=n)
        g = capture(torch, lin.launch_step, stream)
        ms = time_replays(torch, g, max(10, steps // 2), args.warmup, dist)
        pts.append((b, ms * 1e3 / max(10, steps // 2) / copies))
        del g, lin
    xs, ys = [p[0] for p in pts], [p[1] for p in pts]
    xm, ym = sum(xs) / len(xs), sum(ys) / len(ys)
    slope = sum((x - xm) * (y - ym) for x, y in zip(xs, ys)) / sum((x - xm) ** 2 for x in xs)
    peak, kind = measured_peak()
    stream_gbs = 1e-3 / slope if slope > 0 else None  # bytes per us -> GB/s
    res["sweep"] = {
        "points": [{"N": n, "bytes": b, "us_per_launch": round(t, 3), "GB_per_s": round(b / t / 1e3, 1)}
                   for n, (b, t) in zip((4096, 16384, 65536), pts)],
        "streaming_GB_per_s": round(stream_gbs, 1) if stream_gbs else None,
        "streaming_frac": round(stream_gbs / peak, 4) if stream_gbs else None,
        "fixed_us_per_launch": round(ym - slope * xm, 3),
        "how": "K = 1024, M = 14, serial launches; least-squares line through (bytes, us): the "
               "slope is K1's streaming rate, the intercept its fixed cost per launch"}
    return res


def batched_object(torch, cq, args, local_rank: int, dist) -> dict:
    """The 24 blocks at M = 896 (64 streams' chunks stacked: K2) and the FFN-up
    GEMM alone."""
    rows = 64 * M_FRAMES
    enc = EncoderLinears(torch, cq, local_rank, rows=rows)
    stream = torch.cuda.Stream()
    g = capture(torch, enc.launch_step, stream)
    steps = max(args.steps, 20)
    ms = time_replays(torch, g, steps, args.warmup, dist) / steps
    flops = N_BLOCKS * sum(2 * rows * n * k for _, n, k, _, _, _ in BLOCK)
    tpeak, tkind = measured_tensor_peak(sustained=True)
    tf = flops / (ms * 1e-3) / 1e12
    res = {"workload": ("quantized linears of the 24-block FastConformer encoder for one chunk of "
                        "64 concurrent streams (M=896 rows per linear), bf16, INT8 group 64"),
           "ms_per_chunk": round(ms, 4), "tflops": round(tf, 2),
           "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": tpeak, "unit": "TFLOP/s",
                        "frac": round(tf / tpeak, 4), "peak_kind": f"{tkind} dense bf16 (sustained)",
                        "kernel": "qgemm_kernel (K2) + activation prepass",
                        "note": "all 192 linears of the chunk, one CUDA graph"}}
    del g, enc
    # FFN up alone: 32 distinct weight copies (145 MB) back to back
    copies = 32
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    layers = []
    for _ in range(copies):
        w = torch.randn((4096, 1024), generator=gen, device="cuda") * 0.02
        q, s, b = cq.quantize(w, GROUP, "bf16")
        L = cq.QuantizedLinear.from_device(q, s, b, None, GROUP, "bf16", local_rank)
        L.reserve(rows)
        layers.append(L)
    x = torch.randn((rows, 1024), generator=gen, device="cuda").to(torch.bfloat16)
    y = torch.empty((rows, 4096), dtype=torch.bfloat16, device="cuda")

    def run(sp):
        for L in layers:
            L.forward_raw(x.data_ptr(), 1024, rows, y.data_ptr(), 4096, "silu", sp)

    g = capture(torch, run, stream)
    ms = time_replays(torch, g, steps, args.warmup, dist) / steps / copies
    bpeak, bkind = measured_tensor_peak(sustained=False)
    tf = 2 * rows * 4096 * 1024 / (ms * 1e-3) / 1e12
    res["ffn_up"] = {"shape": "M=896 x N=4096 x K=1024, SiLU epilogue", "us_per_call": round(ms * 1e3, 3),
                     "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": bpeak,
                                  "unit": "TFLOP/s", "frac": round(tf / bpeak, 4),
                                  "peak_kind": f"{bkind} dense bf16 (burst)",
                                  "kernel": "qgemm_kernel (K2) + activation prepass",
                                  "note": "32 distinct weight copies (145 MB) back to back"}}
    del g
    # the GEMM alone: activations already in the tensor-core format (what the
    # encoder's LayerNorm hands FFN-up), converted once outside the graph
    x16, rs = layers[0].prescale_activations(x)
    fn = cq.lib().cq_linear_forward_prescaled
    silu = cq.ACTS["silu"]

    def run_pre(sp):
        for L in layers:
            if fn(L._h, ctypes.c_void_p(x16.data_ptr()), ctypes.c_void_p(rs.data_ptr()), rows,
                  ctypes.c_void_p(y.data_ptr()), 4096, silu, ctypes.c_void_p(sp)):
                raise RuntimeError("cq_linear_forward_prescaled failed: " + cq.last_error())

    g = capture(torch, run_pre, stream)
    ms = time_replays(torch, g, steps, args.warmup, dist) / steps / copies
    tf = 2 * rows * 4096 * 1024 / (ms * 1e-3) / 1e12
    res["ffn_up"]["gemm_only"] = {
        "us_per_call": round(ms * 1e3, 3),
        "roofline": {"bound": "tensor", "achieved": round(tf, 2), "peak": bpeak, "unit": "TFLOP/s",
                     "frac": round(tf / bpeak, 4), "peak_kind": f"{bkind} dense bf16 (burst)",
                     "kernel": "qgemm_kernel (K2)",
                     "note": "cq_linear_forward_prescaled on activations converted once "
                             "(cq_linear_prescale_activations), 32 distinct weight copies"}}
    del g, layers
    return res


CHUNK_MEL = 112          # log-mel frames per chunk (lookahead 13: 8 * (13 + 1))
CHUNK_AUDIO_S = 1.12     # 112 frames at the 10 ms hop
ENC_STREAMS = 64         # concurrent streams per GPU (64 x 14 = 896 rows per linear)


def encoder_flops_per_chunk(streams: int) -> int:
    """Algorithmic FLOPs (2 * rows * N * K) of every quantized linear in one
    chunk of `streams` streams: 24 blocks, subsampling and prompt projector.
    (The position projection is made once per state, not per chunk.)"""
    q = 14
    block = (2 * 4096 * 1024 * 2 + 3072 * 1024 + 1024 * 1024 + 2048 * 1024 + 1024 * 1024)
    f = streams * q * block * ENCODER_LAYERS
    f += streams * (28 * 33 * 256 * 256 + 14 * 17 * 256 * 256 + q * 4352 * 1024)
    f += streams * q * (1152 * 2048 + 2048 * 1024)
    return 2 * f


# Programmatic dependent launch of the (encoder, RNNT) states when the two run
# pipelined on one GPU.  Measured at 64 streams: both off 9.29 ms per chunk,
# both on 9.55, one of them on 9.60-9.66 -- early-launched CTAs waiting on
# their stream hold SM room the other stream could use.  Alone, each state
# keeps PDL on (the encoder 6.03 vs 6.12 ms, the RNNT 4.10 vs 4.86 ms).
PIPELINE_PDL = (False, False)


def bench_encoder(torch, cq, args, world: int, local_rank: int, dist, streams: int,
                  chunks: int, with_e2e: bool = True, with_rnnt: bool = False) -> dict:
    """Streaming encoder (subsampling + 24 FastConformer blocks + prompt
    projector) over `streams` lock-step streams, one 112-frame chunk per step,
    through the C ABI (cq_encoder_encode_chunk replays one CUDA graph per
    chunk).  With `with_rnnt`, every chunk's encoder output is also decoded by
    the batched RNNT greedy decoder (cq_rnnt_decode_chunk), pipelined on a
    second CUDA stream: RNNT of chunk c overlaps the encoder of chunk c + 1."""
    from nemotron_cuda.encoder import Encoder
    enc = Encoder.random(None, seed=7, dtype="bf16", device=local_rank)
    st = enc.state(streams, CHUNK_MEL)
    if with_rnnt:
        st.set_pdl(PIPELINE_PDL[0])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11 + local_rank)
    mel = torch.randn((streams, CHUNK_MEL, 128), generator=gen, device="cuda")
    outs = [st.encode_chunk(mel)]  # first chunk (eager; later chunks replay a graph)
    frames = outs[0].shape[0] // streams
    s_enc = torch.cuda.Stream()
    # e2e input: each stream's 1.12 s window of 16 kHz PCM as the chunk
    # scheduler cuts it (18320 samples, uncentered -> 112 frames), through the
    # GPU log-mel frontend (cq_logmel_extract) into the encoder's input
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron(device=local_rank)
    pcm_samples = CHUNK_MEL * 160 + 400
    assert fe.frames(pcm_samples, False) == CHUNK_MEL
    pcm = torch.randn((streams, pcm_samples), generator=gen, device="cuda") * 0.1
    host_pcm = torch.empty((streams, pcm_samples), dtype=torch.float32).pin_memory()
    host_pcm.copy_(pcm.cpu())
    rn = rst = None
    if with_rnnt:
        from nemotron_cuda.rnnt import Rnnt
        outs.append(torch.empty_like(outs[0]))
        rn = Rnnt.random(None, seed=13, dtype="bf16", device=local_rank)
        rst = rn.state(streams, frames)
        rst.set_pdl(PIPELINE_PDL[1])
        # the decoder's short dependent launches are the critical path: give them
        # priority over the encoder's GEMMs when both have CTAs waiting for SMs
        lo, hi = torch.cuda.Stream.priority_range() if hasattr(torch.cuda.Stream, "priority_range") \
            else (0, -1)
        s_dec = torch.cuda.Stream(priority=min(lo, hi))
        tok = [torch.empty((streams, rst.capacity), dtype=torch.int32, device="cuda") for _ in range(2)]
        tfr = [torch.empty_like(t) for t in tok]
        cnt = [torch.empty((streams,), dtype=torch.int32, device="cuda") for _ in range(2)]
        host_tok = torch.empty((streams, rst.capacity), dtype=torch.int32).pin_memory()
        host_cnt = torch.empty((streams,), dtype=torch.int32).pin_memory()
        enc_done = [torch.cuda.Event() for _ in range(2)]
        dec_done = [torch.cuda.Event() for _ in range(2)]
    host_out = torch.empty(tuple(outs[0].shape), dtype=outs[0].dtype).pin_memory()
    torch.cuda.synchronize()

    def run(n: int, e2e: bool) -> None:
        for i in range(n):
            b = i % 2 if with_rnnt else 0
            with torch.cuda.stream(s_enc):
                if e2e:
                    pcm.copy_(host_pcm, non_blocking=True)
                    fe.extract_raw(pcm, pcm_samples, False, mel, stream=s_enc)
                if with_rnnt:
                    s_enc.wait_event(dec_done[b])  # the decoder has read this buffer
                st.encode_chunk(mel, outs[b], stream=s_enc)
                if e2e and not with_rnnt:
                    host_out.copy_(outs[b], non_blocking=True)
                if with_rnnt:
                    enc_done[b].record(s_enc)
            if with_rnnt:
                with torch.cuda.stream(s_dec):
                    s_dec.wait_event(enc_done[b])
                    rst.decode_chunk_raw(outs[b], frames, tok[b], tfr[b], cnt[b], stream=s_dec)
                    if e2e:
                        host_cnt.copy_(cnt[b], non_blocking=True)
                        host_tok.copy_(tok[b], non_blocking=True)
                    dec_done[b].record(s_dec)

    def timed(e2e: bool) -> float:
        run(args.warmup, e2e)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")  # profilers can select the timed launches
        s.record(s_enc)
        if with_rnnt:
            s_dec.wait_stream(s_enc)
        run(chunks, e2e)
        if with_rnnt:
            s_enc.wait_stream(s_dec)
        e.record(s_enc)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        return max_over_ranks(dist, ms)

    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = timed(False)
    clock_info = clocks.stop()
    ms_e2e = timed(True) if with_e2e else None
    kernels = st.kernels_per_chunk + (rst.kernels_per_chunk if with_rnnt else 0)
    status = cq.device_status(local_rank)
    if status != 0:
        raise RuntimeError(f"device watchdog reported status {status}")
    per_chunk = ms / chunks
    audio = streams * CHUNK_AUDIO_S * chunks  # per rank
    flops = encoder_flops_per_chunk(streams)
    tpeak, tkind = measured_tensor_peak()
    tflops = flops / (per_chunk * 1e-3) / 1e12
    what = ("streaming FastConformer encoder (Conv2D subsampling, 24 blocks d=1024 ff=4096 8 heads, "
            "attention window 56+14 frames, conv kernel 9 cache, prompt projector)")
    if with_rnnt:
        what += (" + batched RNNT greedy decode (2-layer LSTM 640, joint 640 -> vocab 1025, at most "
                 "10 symbols per frame; random weights emit the maximum), RNNT of chunk c pipelined "
                 "with the encoder of chunk c+1 on a second CUDA stream")
    res = {
        "metric": "encoder audio-sec/sec", "value": round(weak_scaling_value(world, audio, ms), 1),
        "unit": "audio-s/s", "streams_per_gpu": streams, "chunks": chunks,
        "ms_per_chunk": round(per_chunk, 4), "chunk_audio_s": CHUNK_AUDIO_S,
        "workload": (f"{what}; {streams} lock-step streams per GPU, 112 log-mel frames x 128 bins "
                     f"per chunk, random-init INT8 group 64 bf16"),
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": tpeak,
                     "unit": "TFLOP/s", "frac": round(tflops / tpeak, 4),
                     "peak_kind": f"{tkind} dense bf16 (sustained)",
                     "note": "encoder linear FLOPs of the whole chunk / chunk time (lower bound "
                             "on the GEMMs' own rate)"},
        "clocks": clock_info,
        "gpu_launches": kernels * chunks, "kernels_per_chunk": kernels,
    }
    if ms_e2e is not None:
        res["e2e"] = {"value": round(weak_scaling_value(world, audio, ms_e2e), 1), "unit": "audio-s/s",
                      "h2d_bytes_per_step": host_pcm.numel() * 4,
                      "d2h_bytes_per_step": (host_tok.numel() + host_cnt.numel()) * 4
                      if with_rnnt else host_out.numel() * 2,
                      "path": "pinned host PCM (18320 samples per stream) -> device, "
                              "cq_logmel_extract, cq_encoder_encode_chunk"
                              + (", cq_rnnt_decode_chunk, token ids and counts" if with_rnnt
                                 else ", encoder output") +
                              " -> pinned host, every chunk inside the timed region"}
    del st, enc, rst, rn, fe
    return res


def bench_rnnt(torch, cq, args, world: int, local_rank: int, dist, streams: int) -> dict:
    """Batched RNNT greedy decode alone (cq_rnnt_decode_chunk): one step = one
    chunk of 14 encoder frames for every stream, the encoder output a fixed
    random bf16 tensor (random weights emit the maximum of 10 symbols per
    frame); e2e adds the pinned-host copy of the encoder output and the token
    read-back to every step."""
    from nemotron_cuda.rnnt import Rnnt
    frames = 14
    rn = Rnnt.random(None, seed=13, dtype="bf16", device=local_rank)
    st = rn.state(streams, frames)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(17 + local_rank)
    enc = (torch.randn((streams * frames, 1024), generator=gen, device="cuda") * 0.5) \
        .to(torch.bfloat16)
    host_enc = torch.empty((streams * frames, 1024), dtype=torch.bfloat16).pin_memory()
    host_enc.copy_(enc.cpu())
    tok = torch.empty((streams, st.capacity), dtype=torch.int32, device="cuda")
    tfr, cnt = torch.empty_like(tok), torch.empty((streams,), dtype=torch.int32, device="cuda")
    host_tok = torch.empty((streams, st.capacity), dtype=torch.int32).pin_memory()
    host_cnt = torch.empty((streams,), dtype=torch.int32).pin_memory()
    s = torch.cuda.Stream()

    def run(n: int, e2e: bool) -> None:
        with torch.cuda.stream(s):
            for _ in range(n):
                if e2e:
                    enc.copy_(host_enc, non_blocking=True)
                st.decode_chunk_raw(enc, frames, tok, tfr, cnt, stream=s)
                if e2e:
                    host_cnt.copy_(cnt, non_blocking=True)
                    host_tok.copy_(tok, non_blocking=True)

    def timed(e2e: bool) -> float:
        run(args.warmup, e2e)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        run(args.steps, e2e)
        e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        return max_over_ranks(dist, ms)

    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = timed(False)
    clock_info = clocks.stop()
    ms_e2e = timed(True)
    status = cq.device_status(local_rank)
    if status != 0:
        raise RuntimeError(f"device watchdog reported status {status}")
    audio = streams * CHUNK_AUDIO_S * args.steps  # per rank
    res = {
        "metric": "RNNT decode audio-sec/sec", "value": round(weak_scaling_value(world, audio, ms), 1),
        "unit": "audio-s/s", "ms_per_chunk": round(ms / args.steps, 4),
        "symbols_per_stream_per_chunk": round(float(cnt.float().mean().item()), 1),
        "workload": (f"batched RNNT greedy decode (2-layer LSTM 640, joint 640 -> vocab 1025, at "
                     f"most 10 symbols per frame), {streams} lock-step streams per GPU, 14 encoder "
                     f"frames (1.12 s) per chunk, random-init INT8 group 64 bf16"),
        "clocks": clock_info, "gpu_launches": st.kernels_per_chunk * args.steps,
        "e2e": {"value": round(weak_scaling_value(world, audio, ms_e2e), 1), "unit": "audio-s/s",
                "h2d_bytes_per_step": host_enc.numel() * 2,
                "d2h_bytes_per_step": (host_tok.numel() + host_cnt.numel()) * 4,
                "path": "pinned host encoder output -> device, cq_rnnt_decode_chunk, token ids "
                        "and counts -> pinned host, every chunk inside the timed region"},
    }
    del st, rn
    return res


def bench_logmel(torch, cq, args, world: int, local_rank: int, dist, streams: int) -> dict:
    """GPU log-mel frontend alone (cq_logmel_extract): one step = the uncentered
    18320-sample window of every stream (112 frames x 128 mel bins, one 1.12 s
    chunk of the streaming scheduler); e2e adds the pinned-host PCM copy and
    the feature read-back to every step."""
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron(device=local_rank)
    samples = 112 * 160 + 400
    gen = torch.Generator(device="cuda")
    gen.manual_seed(23 + local_rank)
    audio = torch.randn((streams, samples), generator=gen, device="cuda") * 0.1
    frames = fe.frames(samples, False)
    out = torch.empty((streams, frames, 128), device="cuda")
    host_audio = torch.empty((streams, samples), dtype=torch.float32).pin_memory()
    host_audio.copy_(audio.cpu())
    host_out = torch.empty((streams, frames, 128), dtype=torch.float32).pin_memory()
    s = torch.cuda.Stream()

    def run(n: int, e2e: bool) -> None:
        with torch.cuda.stream(s):
            for _ in range(n):
                if e2e:
                    audio.copy_(host_audio, non_blocking=True)
                fe.extract_raw(audio, samples, False, out, stream=s)
                if e2e:
                    host_out.copy_(out, non_blocking=True)

    def timed(e2e: bool) -> float:
        run(args.warmup, e2e)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        run(args.steps, e2e)
        e1.record(s)
        torch.cuda.synchronize()
        return max_over_ranks(dist, e0.elapsed_time(e1))

    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = timed(False)
    clock_info = clocks.stop()
    ms_e2e = timed(True)
    status = cq.device_status(local_rank)
    if status != 0:
        raise RuntimeError(f"device watchdog reported status {status}")
    audio_s = streams * CHUNK_AUDIO_S * args.steps  # per rank
    step_bytes = streams * samples * 4 + streams * frames * 128 * 4
    peak, peak_kind = measured_peak()
    achieved = step_bytes / (ms / args.steps * 1e-3) / 1e9
    res = {
        "metric": "log-mel frontend audio-sec/sec", "value": round(weak_scaling_value(world, audio_s, ms), 1),
        "unit": "audio-s/s", "ms_per_chunk": round(ms / args.steps, 4),
        "workload": (f"log-mel frontend (preemphasis 0.97, Hann 400 in n_fft 512, f64 FFT, 128 Slaney "
                     f"mel bins, ln) of {streams} uncentered 18320-sample windows per step"),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} copy bandwidth",
                     "note": "PCM in + features out per step / step time", "traffic": None},
        "clocks": clock_info, "gpu_launches": args.steps,
        "e2e": {"value": round(weak_scaling_value(world, audio_s, ms_e2e), 1), "unit": "audio-s/s",
                "h2d_bytes_per_step": host_audio.numel() * 4, "d2h_bytes_per_step": host_out.numel() * 4,
                "path": "pinned host PCM -> device, cq_logmel_extract, features -> pinned host, every "
                        "step inside the timed region"},
    }
    del fe
    return res


def cpu_encoder_baseline(target_s: float = 8.0, with_rnnt: bool = True) -> dict:
    """The CPU restatement of the encoder (oracle/encoder_oracle.py, numpy +
    the OpenMP C linear) and, with `with_rnnt`, of the RNNT greedy decoder
    (oracle/rnnt_oracle.py) on one stream: a bounded sample of chunks."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import encoder_oracle as eo
    import oracle
    import rnnt_oracle as ro
    oracle.set_threads(host_threads())
    cfg = eo.EncoderConfig()
    enc = eo.Encoder(cfg, eo.random_params(cfg, 3, "bf16"), "bf16")
    cache = enc.new_cache()
    dec = dstate = None
    if with_rnnt:
        rcfg = ro.RnntConfig()
        dec = ro.RnntDecoder(rcfg, ro.random_params(rcfg, 4, "bf16"), "bf16")
        dstate = dec.new_state()
    rng = np.random.default_rng(0)
    mel = rng.standard_normal((CHUNK_MEL, 128)).astype(np.float32)

    def chunk():
        y = enc.encode_chunk(mel, 101, cache)
        if dec is not None:
            dec.decode_frames(y, dstate)

    chunk()  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        chunk()
        n += 1
        if time.perf_counter() - t0 >= target_s and n >= 2:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n * CHUNK_AUDIO_S / dt, 3), "unit": "audio-s/s",
            "cores": oracle.max_threads(), "kind": "port",
            "sample": f"{n} chunks of one stream (112 mel frames each), {dt:.1f} s, numpy + OpenMP "
                      f"C restatement of the streaming encoder"
                      + (" and the RNNT greedy decoder" if with_rnnt else "") + " (oracle/)"}


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import nemotron_cuda as cq
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "encoder":
        res = bench_encoder(torch, cq, args, world, local_rank, dist, args.streams, args.steps,
                            with_rnnt=not args.no_rnnt)
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        line = {"metric": METRIC, "value": res["value"], "unit": res["unit"], "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_chunk"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init INT8 weights quantised on device; log-mel ~ N(0,1))",
                "config": {"workload": res["workload"], "group_size": GROUP,
                           "streams_per_gpu": args.streams,
                           "parallelism": f"dp{world} (replicated weights, independent streams)",
                           "l2": "inputs larger than L2 (640 MB of weights per chunk)"},
                "e2e": res["e2e"], "roofline": res["roofline"], "clocks": res["clocks"],
                "gpu_launches": res["gpu_launches"]}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_encoder_baseline(args.cpu_seconds, not args.no_rnnt)
        return line
    if args.workload == "logmel":
        res = bench_logmel(torch, cq, args, world, local_rank, dist, args.streams)
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        return {"metric": res["metric"], "value": res["value"], "unit": res["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": res["ms_per_chunk"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (PCM ~ N(0, 0.01))",
                "config": {"workload": res["workload"], "streams_per_gpu": args.streams,
                           "parallelism": f"dp{world} (independent streams)",
                           "l2": "inputs smaller than L2 (8.4 MB per step at 64 streams)"},
                "e2e": res["e2e"], "roofline": res["roofline"], "clocks": res["clocks"],
                "gpu_launches": res["gpu_launches"]}
    if args.workload == "rnnt":
        res = bench_rnnt(torch, cq, args, world, local_rank, dist, args.streams)
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        return {"metric": res["metric"], "value": res["value"], "unit": res["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": res["ms_per_chunk"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init INT8 weights; encoder output ~ N(0, 0.25))",
                "config": {"workload": res["workload"], "group_size": GROUP,
                           "streams_per_gpu": args.streams,
                           "symbols_per_stream_per_chunk": res["symbols_per_stream_per_chunk"],
                           "parallelism": f"dp{world} (replicated weights, independent streams)",
                           "l2": "weights (7.6 MB) L2-resident; every step reads them again"},
                "e2e": res["e2e"], "clocks": res["clocks"], "gpu_launches": res["gpu_launches"]}
    if args.workload == "linear" and args.linear_n:
        # one N alone, serial launches (for profiling captures of K1 at large N)
        b = linear_bytes(args.linear_n, 1024, M_FRAMES)
        copies = max(3, -(-260_000_000 // b))
        lin = SingleLinear(torch, cq, local_rank, n=args.linear_n, copies=copies)
        g = capture(torch, lin.launch_step, torch.cuda.Stream())
        ms = time_replays(torch, g, args.steps, args.warmup, dist)
        us = ms * 1e3 / args.steps / copies
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        return {"metric": "INT8 qlinear HBM GB/s (M=14)", "value": round(b / us / 1e3, 2),
                "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"x bf16 [14,1024] . W[{args.linear_n},1024]^T, group 64, "
                                       f"{copies} distinct weight copies, serial launches"},
                "roofline": hbm_roofline(b, us, "qgemv_kernel (K1)", "serial launches"),
                "gpu_launches": copies * args.steps}
    if args.workload == "linear":
        res = linear_object(torch, cq, args, local_rank, dist)
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        best = res["concurrent"]
        return {"metric": "INT8 qlinear HBM GB/s (M=14)", "value": best["value"], "unit": UNIT,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(best["us_per_linear"] * 40 / 1e3, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init INT8 weights N(0,0.02) quantised on device)",
                "config": {"workload": res["workload"], "group_size": GROUP,
                           "l2": "inputs larger than L2 (184 MB of distinct weights per step)"},
                "roofline": res["roofline"], "linear": res, "gpu_launches": 40 * args.steps}
    if args.workload == "batched":
        res = batched_object(torch, cq, args, local_rank, dist)
        if dist:
            dist.destroy_process_group()
        if rank != 0:
            return None
        return {"metric": "INT8 qlinear TFLOP/s (M=896)", "value": res["tflops"], "unit": "TFLOP/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": res["ms_per_chunk"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": res["workload"], "group_size": GROUP,
                           "l2": "inputs larger than L2 (640 MB of weights per step)"},
                "roofline": res["roofline"], "batched": res}

    # ---- default: the batch-1 chain, one 60 s stream (54 chunks) per step
    enc = EncoderLinears(torch, cq, local_rank)
    chunks = args.chunks_per_step
    step_bytes, launches = CHUNK_BYTES * chunks, LAUNCHES_PER_CHUNK * chunks
    stream = torch.cuda.Stream()
    graph = capture(torch, lambda sp: enc.launch_step(sp, chunks), stream)

    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = time_replays(torch, graph, args.steps, args.warmup, dist)
    clock_info = clocks.stop()
    del graph

    # end to end: every chunk copies its input from pinned host memory, calls
    # the C ABI once per linear (no graph: the host cost of each call is in
    # the timed region) and reads the chunk's output back to pinned memory
    host_in = torch.empty((M_FRAMES, 1024), dtype=torch.bfloat16).pin_memory()
    host_in.copy_(enc.x0.cpu())
    host_out = torch.empty((M_FRAMES, 1024), dtype=torch.bfloat16).pin_memory()

    def e2e_steps(n: int) -> None:
        with torch.cuda.stream(stream):
            for _ in range(n * chunks):
                enc.x0.copy_(host_in, non_blocking=True)
                enc.launch_chunk(stream.cuda_stream)
                host_out.copy_(enc.final, non_blocking=True)

    e2e_steps(args.warmup)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(dist, e0.elapsed_time(e1))
    status = cq.device_status(local_rank)
    del enc

    linear = batched = encoder = None
    if not args.no_extras:
        linear = linear_object(torch, cq, args, local_rank, dist)
        batched = batched_object(torch, cq, args, local_rank, dist)
    if not args.no_encoder:
        encoder = bench_encoder(torch, cq, args, world, local_rank, dist, ENC_STREAMS,
                                args.encoder_chunks, with_rnnt=True)
        for key, streams in (("encoder_only", ENC_STREAMS), ("batch1", 1)):
            sub = bench_encoder(torch, cq, args, world, local_rank, dist, streams,
                                args.encoder_chunks, with_e2e=False)
            sub.pop("clocks", None)
            encoder[key] = sub
    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return None
    if status != 0:
        raise RuntimeError(f"device watchdog reported status {status}")
    ms_step = ms / args.steps
    value = weak_scaling_value(world, step_bytes, ms_step) / 1e9
    value_e2e = weak_scaling_value(world, step_bytes, ms_e2e / args.steps) / 1e9
    per_launch_us = ms_step * 1e3 / launches
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init INT8 weights N(0,0.02) quantised on device; bf16 x ~ N(0,1))",
        "config": {"workload": WORKLOAD, "group_size": GROUP, "rows": M_FRAMES,
                   "chunks_per_step": chunks, "bytes_per_chunk_per_gpu": CHUNK_BYTES,
                   "launches_per_chunk": LAUNCHES_PER_CHUNK,
                   "l2": "inputs larger than L2 (every chunk re-reads 640 MB of distinct weights)",
                   "parallelism": f"dp{world} (replicated weights, independent streams)",
                   "graph": "one CUDA graph per step (54 chunks x 192 linears), programmatic "
                            "dependent launch edges"},
        "e2e": {"value": round(value_e2e, 2), "unit": UNIT,
                "h2d_bytes_per_step": host_in.numel() * 2 * chunks,
                "d2h_bytes_per_step": host_out.numel() * 2 * chunks,
                "path": "per chunk: pinned host input -> device, one C-ABI cq_linear_forward_ex call "
                        "per linear (eager, no graph), output -> pinned host; all inside the timed "
                        "region"},
        "gpu_launches": launches * args.steps,
        "roofline": hbm_roofline(step_bytes / launches, per_launch_us, "qgemv_kernel (K1)",
                                 "the dependent batch-1 chain: average bytes and device time per "
                                 "linear"),
        "clocks": clock_info,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(target_s=args.cpu_seconds)
    if linear is not None:
        line["linear"] = linear
        line["batched"] = batched
    if encoder is not None:
        if world == 1 and not args.no_cpu_baseline:
            encoder["cpu_baseline"] = cpu_encoder_baseline(args.cpu_seconds)
        line["encoder"] = encoder
    return line


# ----------------------------------------------------------------- CPU arms


class OracleChain:
    """The 24-block chain on the host for the CPU restatement: every block's
    weights drawn N(0, 0.02) and quantised by the oracle's quantiser (the same
    algorithm, bit for bit, as the device quantiser of the GPU arm), bf16."""

    def __init__(self, seed: int = 1, blocks: int | None = None):
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        self.oracle = oracle
        oracle.set_threads(host_threads())
        rng = np.random.default_rng(seed)
        self.blocks = []
        for _ in range(N_BLOCKS if blocks is None else blocks):
            blk = []
            for _, n, k, _, _, _ in BLOCK:
                w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
                blk.append(oracle.quantize(w, GROUP, "bf16"))
            self.blocks.append(blk)
        self.x0 = oracle.to_t(rng.standard_normal((M_FRAMES, 1024)).astype(np.float32), "bf16")
        self.bytes = len(self.blocks) * block_bytes()

    def run_chunk(self) -> None:
        O = self.oracle
        outs = {}
        for b, blk in enumerate(self.blocks):
            for (q, s, sb), (name, n, k, m, act, src) in zip(blk, BLOCK):
                x = (self.x0 if b == 0 else outs["ffn2_down"]) if src == "x0" else outs[src]
                outs[name] = O.qmatmul(x, q, s, sb, GROUP, "bf16", None, act)


def cpu_baseline(target_s: float = 12.0) -> dict:
    ob = OracleChain()
    ob.run_chunk()  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        ob.run_chunk()
        n += 1
        if time.perf_counter() - t0 >= target_s and n >= 2:
            break
    dt = time.perf_counter() - t0
    return {"value": round(n * ob.bytes / dt / 1e9, 3), "unit": UNIT,
            "cores": ob.oracle.max_threads(), "kind": "port",
            "sample": f"{n} chunks of the 24-block chain (192 linears, M=14, 640 MB of weights), "
                      f"{dt:.1f} s, OpenMP C restatement of quantized_matmul (oracle/)"}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    ob = OracleChain()
    for _ in range(args.warmup):
        ob.run_chunk()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ob.run_chunk()
    dt = time.perf_counter() - t0
    value = args.steps * ob.bytes / dt / 1e9
    enc = None if args.no_encoder else cpu_encoder_baseline(args.cpu_seconds)
    cores = ob.oracle.max_threads()
    return {
        "encoder": enc,
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init INT8 weights N(0,0.02); bf16 x ~ N(0,1))", "impl": "reference",
        "config": {"workload": WORKLOAD, "group_size": GROUP, "rows": M_FRAMES,
                   "chunks_per_step": args.chunks_per_step, "bytes_per_chunk_per_gpu": CHUNK_BYTES,
                   "launches_per_chunk": LAUNCHES_PER_CHUNK,
                   "l2": "inputs larger than L2 (every chunk re-reads 640 MB of distinct weights)",
                   "parallelism": f"dp{args.gpus} (replicated weights, independent streams)",
                   "graph": "one CUDA graph per step (54 chunks x 192 linears), programmatic "
                            "dependent launch edges"},
        "sample": "each step is one chunk of the 24-block chain (1/54 of the GPU arm's step; the "
                  "metric is a rate, so the values compare)",
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{args.steps} chunks of the 24-block chain (192 linears, M=14, "
                                   f"640 MB of weights), {dt:.1f} s, OpenMP C restatement of MLX "
                                   f"quantized_matmul (oracle/) on {cores} host threads; MLX itself "
                                   f"cannot run on this host"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> None:
    # stdout carries exactly one JSON line (rank 0); anything else that a
    # library prints (NCCL's banner, warnings) goes to stderr
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["block", "linear", "batched", "encoder", "rnnt", "logmel"],
                    default="block",
                    help="block: the 24-block M=14 linear chain, one 60 s stream per step "
                         "(default; the line also carries the 'linear', 'batched' and 'encoder' "
                         "objects); linear: config 1 alone (one 4096x1024 linear, serial and "
                         "concurrent launches, N sweep); batched: the 24-block chain at M=896 "
                         "(64 streams, tensor-core path) and the FFN-up GEMM; encoder: the full "
                         "streaming encoder alone (value in audio-s/s); rnnt: the batched RNNT "
                         "greedy decoder alone; logmel: the GPU log-mel frontend alone")
    ap.add_argument("--streams", type=int, default=ENC_STREAMS,
                    help="streams per GPU of the encoder, rnnt and logmel workloads")
    ap.add_argument("--chunks-per-step", type=int, default=CHUNKS_PER_STEP,
                    help="chunks of the batch-1 chain per step (54: one 60 s stream)")
    ap.add_argument("--encoder-chunks", type=int, default=CHUNKS_PER_STEP,
                    help="timed chunks of the encoder measurement in the default run (54: a "
                         "60 s stream per stream)")
    ap.add_argument("--no-encoder", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default run without the 'linear' and 'batched' objects")
    ap.add_argument("--blocks", type=int, default=N_BLOCKS,
                    help="FastConformer blocks in the linear workloads (24 in the encoder; "
                         "fewer only for small profiling captures)")
    ap.add_argument("--linear-n", type=int, default=0,
                    help="linear workload: only serial launches of x[14,1024] . W[N,1024]^T "
                         "(profiling captures of K1 at large N)")
    ap.add_argument("--no-rnnt", action="store_true",
                    help="encoder workload without the RNNT decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    args = ap.parse_args()
    if args.blocks != N_BLOCKS:
        set_blocks(args.blocks)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    line = run_reference(args, rank) if args.impl == "reference" else run_ours(
        args, rank, world, local_rank)
    if line is not None:
        json_out.write(json.dumps(line) + "\n")
        json_out.flush()


if __name__ == "__main__":
    main()
