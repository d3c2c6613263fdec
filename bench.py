#!/usr/bin/env python
"""Benchmark of the B200 affine INT8 quantized linear (batch-1 streaming chunk).

Workload (one "step"): the quantized linears of all 24 FastConformer blocks
for one 1120 ms chunk at batch 1 (M = 14 frames after 8x subsampling,
d_model 1024, ff 4096), bf16 activations, INT8 weights with group 64 and bf16
scale/bias, random init N(0, 0.02) quantised on the device, 24 distinct weight
sets (~640 MB, far larger than the 126 MB L2).  Per block, in data-dependency
order: FFN1 up (+SiLU) 1024->4096, FFN1 down 4096->1024, fused q|k|v
1024->3072, pos-proj 1024->1024 over 2*70-1 = 139 rows, out 1024->1024,
conv pointwise-1 1024->2048, pointwise-2 1024->1024, FFN2 up (+SiLU), FFN2
down.  The non-linear ops between them (attention core, GLU, depthwise conv,
LayerNorm) are not part of this workload; their inputs are stood in by the
producing linear's output of the same shape, so every launch depends on the
previous one as in the encoder.

metric: GB/s of algorithmic bytes (N*K weight bytes + 4*N*K/g scale/bias bytes
+ 2*M*K activation bytes + 2*M*N output bytes per linear) / device time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: every rank holds a full weight replica and runs its
own stream's chunks (no data-path collective; a barrier and a max-reduction of
the timings are the only communication).  --impl reference times the CPU
restatement of the reference's quantized_matmul (the oracle, OpenMP C) on the
host cores with the same metric.
"""
from __future__ import annotations

import argparse
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
POS_ROWS = 139

# name, N, K, rows, act, input (name of a producer or "x0" / "pe"), input columns used
BLOCK = [
    ("ffn1_up", 4096, 1024, M_FRAMES, "silu", "x0"),
    ("ffn1_down", 1024, 4096, M_FRAMES, "none", "ffn1_up"),
    ("qkv", 3072, 1024, M_FRAMES, "none", "ffn1_down"),
    ("pos", 1024, 1024, POS_ROWS, "none", "pe"),
    ("out", 1024, 1024, M_FRAMES, "none", "qkv"),
    ("pw1", 2048, 1024, M_FRAMES, "none", "out"),
    ("pw2", 1024, 1024, M_FRAMES, "none", "pw1"),
    ("ffn2_up", 4096, 1024, M_FRAMES, "silu", "pw2"),
    ("ffn2_down", 1024, 4096, M_FRAMES, "none", "ffn2_up"),
]


def linear_bytes(n: int, k: int, m: int, g: int = GROUP) -> int:
    return n * k + 4 * n * k // g + 2 * m * k + 2 * m * n


BLOCK_BYTES = sum(linear_bytes(n, k, m) for _, n, k, m, _, _ in BLOCK)
STEP_BYTES = N_BLOCKS * BLOCK_BYTES
LAUNCHES_PER_STEP = N_BLOCKS * len(BLOCK)
WORKLOAD = ("quantized linears of the 24-block FastConformer encoder for one 1120 ms chunk "
            "at batch 1 (M=14; pos-proj M=139), bf16, INT8 group 64, 24 distinct weight sets")


def set_blocks(n: int) -> None:
    """Fewer blocks for small profiling captures (the workload line says so)."""
    global N_BLOCKS, STEP_BYTES, LAUNCHES_PER_STEP, WORKLOAD
    N_BLOCKS = n
    STEP_BYTES = N_BLOCKS * BLOCK_BYTES
    LAUNCHES_PER_STEP = N_BLOCKS * len(BLOCK)
    WORKLOAD = WORKLOAD.replace("24-block", f"{n}-block").replace("24 distinct", f"{n} distinct")


# DRAM bytes (read + write) per algorithmic byte of K1, from one ncu capture of
# the 4096x1024 linear at M = 14 (4.531 MB for 4.600 MB algorithmic); traffic
# grows with the bytes a launch streams, so it is scaled to the average launch.
K1_TRAFFIC_PER_ALGO_BYTE = 4.5312e6 / 4599808
# The same ratio for the persistent chain kernel (qchain_kernel), from one ncu
# capture of a 2-block chain; 1.0 until that capture is summarised.
CHAIN_TRAFFIC_PER_ALGO_BYTE = 1.0


def measured_tensor_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 1400.0, "fallback"


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


def measured_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


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
    rows = 14 is one stream's chunk; rows = 896 stacks 64 streams' chunks (the
    pos-proj input is shared by all streams and keeps its 139 rows)."""

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
        self.spec = [(nm, n, k, rows if m == M_FRAMES else m, act, src)
                     for nm, n, k, m, act, src in BLOCK]
        self.x0 = torch.randn((rows, 1024), generator=gen, device=dev).to(bf)
        self.pe = torch.randn((POS_ROWS, 1024), generator=gen, device=dev).to(bf)
        # the batch-1 chain keeps every block's outputs (no buffer reuse, so the
        # persistent chain needs no completion waits); the batched workload
        # reuses one set
        sets = N_BLOCKS if rows == M_FRAMES else 1
        self.outs = [{name: torch.empty((m, n), dtype=bf, device=dev)
                      for name, n, _, m, _, _ in self.spec} for _ in range(sets)]
        self.out = self.outs[-1]

    def steps(self):
        """(layer, x, y, act, rows) of every linear, in launch order."""
        out = []
        for b, blk in enumerate(self.layers):
            cur = self.outs[b % len(self.outs)]
            prev = self.outs[(b - 1) % len(self.outs)]
            for layer, (name, n, k, m, act, src) in zip(blk, self.spec):
                if src == "x0":
                    x = self.x0 if b == 0 else prev["ffn2_down"]
                elif src == "pe":
                    x = self.pe
                else:
                    x = cur[src]
                out.append((layer, x, cur[name], act, m))
        return out

    def use_chain(self) -> None:
        """Run every step as one persistent launch (include/cqchain.h)."""
        self.chain = self.cq.LinearChain(self.steps())

    def launch_step(self, stream_ptr: int) -> None:
        """All 24 blocks' linears, each consuming its producer's output."""
        if getattr(self, "chain", None) is not None:
            self.chain.run_raw(stream_ptr)
            return
        for layer, x, y, act, m in self.steps():
            layer.forward_raw(x.data_ptr(), x.stride(0), m, y.data_ptr(), y.stride(0), act,
                              stream_ptr)


class SingleLinear:
    """Back-to-back independent launches of the single-linear workload:
    x bf16 [14, 1024] . W[4096, 1024]^T, group 64, over 40 distinct weight
    copies (~184 MB, larger than L2); every launch reads the same x."""

    COPIES = 40
    N, K = 4096, 1024

    def __init__(self, torch, cq, device: int, seed: int = 0):
        dev = torch.device("cuda", device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.layers = []
        for _ in range(self.COPIES):
            w = torch.randn((self.N, self.K), generator=gen, device=dev) * 0.02
            q, s, b = cq.quantize(w, GROUP, "bf16")
            self.layers.append(cq.QuantizedLinear.from_device(q, s, b, None, GROUP, "bf16", device))
            del w, q, s, b
        self.x0 = torch.randn((M_FRAMES, self.K), generator=gen, device=dev).to(torch.bfloat16)
        self.ys = [torch.empty((M_FRAMES, self.N), dtype=torch.bfloat16, device=dev)
                   for _ in range(2)]
        self.final = self.ys[(self.COPIES - 1) % 2]

    def launch_step(self, stream_ptr: int) -> None:
        for i, layer in enumerate(self.layers):
            y = self.ys[i % 2]
            layer.forward_raw(self.x0.data_ptr(), self.K, M_FRAMES, y.data_ptr(), self.N, "none",
                              stream_ptr)


BATCH_ROWS = 64 * M_FRAMES  # 64 concurrent streams' chunks stacked per linear
BATCHED_WORKLOAD = ("quantized linears of the 24-block FastConformer encoder for one 1120 ms chunk "
                    "of 64 concurrent streams (M=896 rows per linear; pos-proj M=139), bf16, INT8 "
                    "group 64, 24 distinct weight sets")
LINEAR_BYTES = linear_bytes(SingleLinear.N, SingleLinear.K, M_FRAMES)
LINEAR_WORKLOAD = ("single INT8 affine quantized linear x bf16 [14,1024] . W[4096,1024]^T, "
                   "group 64, 40 independent back-to-back launches over distinct weight copies")


CHUNK_MEL = 112          # log-mel frames per chunk (lookahead 13: 8 * (13 + 1))
CHUNK_AUDIO_S = 1.12     # 112 frames at the 10 ms hop
ENC_STREAMS = 64         # concurrent streams per GPU (64 x 14 = 896 rows per linear)


def encoder_flops_per_chunk(streams: int) -> int:
    """Algorithmic FLOPs (2 * rows * N * K) of every quantized linear in one
    chunk of `streams` streams: 24 blocks, subsampling and prompt projector.
    The position projection (83 rows) is shared by the streams of a state."""
    q = 14
    block = (2 * 4096 * 1024 * 2 + 3072 * 1024 + 1024 * 1024 + 2048 * 1024 + 1024 * 1024)
    f = streams * q * block * ENCODER_LAYERS
    f += (56 + 14 + 14 - 1) * 1024 * 1024 * ENCODER_LAYERS  # relative_k_proj
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
        s.record(s_enc)
        if with_rnnt:
            s_dec.wait_stream(s_enc)
        run(chunks, e2e)
        if with_rnnt:
            s_enc.wait_stream(s_dec)
        e.record(s_enc)
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
    step_flops = None
    if args.workload == "linear":
        enc = SingleLinear(torch, cq, local_rank)
        step_bytes, launches, workload = LINEAR_BYTES * SingleLinear.COPIES, SingleLinear.COPIES, LINEAR_WORKLOAD
        in_shape = (M_FRAMES, SingleLinear.K)
    elif args.workload == "batched":
        enc = EncoderLinears(torch, cq, local_rank, rows=BATCH_ROWS)
        step_bytes = N_BLOCKS * sum(linear_bytes(n, k, m) for _, n, k, m, _, _ in enc.spec)
        step_flops = N_BLOCKS * sum(2 * m * n * k for _, n, k, m, _, _ in enc.spec)
        launches, workload = LAUNCHES_PER_STEP, BATCHED_WORKLOAD
        in_shape = (BATCH_ROWS, 1024)
    else:
        enc = EncoderLinears(torch, cq, local_rank)
        step_bytes, launches, workload = STEP_BYTES, LAUNCHES_PER_STEP, WORKLOAD
        in_shape = (M_FRAMES, 1024)
        if args.chain:
            enc.use_chain()
            launches = 1

    # eager warm-up (sets kernel attributes before capture), then capture.
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        enc.launch_step(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        enc.launch_step(stream.cuda_stream)
    # end-to-end graph: pinned host input -> device, chain, device -> pinned host
    final = enc.final if args.workload == "linear" else enc.out["ffn2_down"]
    host_in = torch.empty(in_shape, dtype=torch.bfloat16).pin_memory()
    host_in.copy_(enc.x0.cpu())
    host_out = torch.empty(tuple(final.shape), dtype=torch.bfloat16).pin_memory()
    graph_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_e2e, stream=stream):
        enc.x0.copy_(host_in, non_blocking=True)
        enc.launch_step(stream.cuda_stream)
        host_out.copy_(final, non_blocking=True)
    torch.cuda.synchronize()

    def timed(g) -> float:
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream()
        s.record(cur)
        for _ in range(args.steps):
            g.replay()
        e.record(cur)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        ms = max_over_ranks(dist, ms)
        if dist:
            dist.barrier()
        return ms

    clocks = ClockSampler(local_rank)
    clocks.start()
    ms = timed(graph)
    clock_info = clocks.stop()
    ms_e2e = timed(graph_e2e)
    status = cq.device_status(local_rank)

    del graph, graph_e2e
    encoder = None
    if args.workload == "block" and not args.no_encoder:
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
    peak, peak_kind = measured_peak()
    per_launch_us = ms_step * 1e3 / launches
    achieved = (step_bytes / launches) / (per_launch_us * 1e-6) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} copy bandwidth",
                "traffic": round(K1_TRAFFIC_PER_ALGO_BYTE * step_bytes / launches),
                "traffic_note": "bytes per launch, scaled from the ncu capture of the 4096x1024 "
                                "linear (dram read+write / algorithmic = 0.985)",
                "kernel": "qgemv_kernel (K1)", "avg_launch_us": round(per_launch_us, 3)}
    chained = getattr(enc, "chain", None) is not None
    if chained:
        roofline.update({
            "traffic": round(CHAIN_TRAFFIC_PER_ALGO_BYTE * step_bytes),
            "traffic_note": "bytes per launch, scaled by blocks from the ncu capture of a "
                            "2-block chain (dram read+write / algorithmic bytes)",
            "kernel": "qchain_kernel (persistent linear chain, one launch per step)"})
    if step_flops is not None:
        tpeak, tkind = measured_tensor_peak()
        tflops = step_flops / (ms_step * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(tflops, 2), "peak": tpeak,
                    "unit": "TFLOP/s", "frac": round(tflops / tpeak, 4),
                    "peak_kind": f"{tkind} dense bf16 (sustained: a step is a long run)",
                    "traffic": None, "kernel": "qgemm_kernel (K2)",
                    "avg_launch_us": round(per_launch_us, 3)}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init INT8 weights N(0,0.02) quantised on device; bf16 x ~ N(0,1))",
        "config": {"workload": workload, "group_size": GROUP, "rows": M_FRAMES,
                   "bytes_per_step_per_gpu": step_bytes, "launches_per_step": launches,
                   "l2": "inputs larger than L2 (distinct weights per step exceed 126 MB)",
                   "parallelism": f"dp{world} (replicated weights, independent streams)",
                   "graph": ("one CUDA graph per step holding one persistent cooperative "
                             "launch of all 216 linears" if chained else
                             "one CUDA graph per step, programmatic dependent launch edges")},
        "e2e": {"value": round(value_e2e, 2), "unit": UNIT,
                "h2d_bytes_per_step": host_in.numel() * 2,
                "d2h_bytes_per_step": host_out.numel() * 2,
                "path": ("C-ABI cq_linear_chain_run" if chained else
                         "C-ABI cq_linear_forward_ex calls") +
                        " captured in a CUDA graph with the pinned-host input copy and output "
                        "read inside the timed region"},
        "gpu_launches": launches * args.steps,
        "roofline": roofline,
        "clocks": clock_info,
    }
    if step_flops is not None:
        line["tflops"] = round(step_flops / (ms_step * 1e-3) / 1e12 * world, 2)
    if world == 1 and not args.no_cpu_baseline and args.workload != "batched":
        line["cpu_baseline"] = cpu_baseline(target_s=args.cpu_seconds, workload=args.workload)
    if encoder is not None:
        if world == 1 and not args.no_cpu_baseline:
            encoder["cpu_baseline"] = cpu_encoder_baseline(args.cpu_seconds)
        line["encoder"] = encoder
    return line


# ----------------------------------------------------------------- CPU arms


class OracleBlocks:
    """Host copies of a few blocks' packed weights for the CPU restatement
    (workload "linear": each block is the single 4096x1024 linear)."""

    def __init__(self, n_blocks: int, seed: int = 1, workload: str = "block"):
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        self.oracle = oracle
        rng = np.random.default_rng(seed)
        self.spec = BLOCK if workload == "block" else [
            ("linear", SingleLinear.N, SingleLinear.K, M_FRAMES, "none", "x0")]
        self.bytes = sum(linear_bytes(n, k, m) for _, n, k, m, _, _ in self.spec)
        self.blocks = []
        for _ in range(n_blocks):
            blk = []
            for _, n, k, m, act, _ in self.spec:
                q = rng.integers(0, 256, size=(n, k), dtype=np.uint8).view(np.uint32)
                s = oracle.to_t((rng.random((n, k // GROUP)) * 1e-3).astype(np.float32), "bf16")
                b = oracle.to_t((rng.random((n, k // GROUP)) * -0.1).astype(np.float32), "bf16")
                blk.append((q, s, b))
            self.blocks.append(blk)
        self.x = {name: oracle.to_t(rng.standard_normal((m, k)).astype(np.float32), "bf16")
                  for name, n, k, m, _, _ in self.spec}

    def run_block(self, i: int) -> None:
        for (q, s, b), (name, n, k, m, act, _) in zip(self.blocks[i % len(self.blocks)], self.spec):
            self.oracle.qmatmul(self.x[name], q, s, b, GROUP, "bf16", None, act)


def cpu_baseline(target_s: float = 12.0, workload: str = "block") -> dict:
    ob = OracleBlocks(4 if workload == "block" else 40, workload=workload)
    ob.run_block(0)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        ob.run_block(n)
        n += 1
        if time.perf_counter() - t0 >= target_s and n >= 2:
            break
    dt = time.perf_counter() - t0
    what = ("blocks x 9 linears (M=14, pos M=139) rotating over 4 weight sets"
            if workload == "block" else "4096x1024 linears (M=14) rotating over 40 weight sets")
    return {"value": round(n * ob.bytes / dt / 1e9, 3), "unit": UNIT,
            "cores": ob.oracle.max_threads(), "kind": "port",
            "sample": f"{n} {what}, {dt:.1f} s, OpenMP C restatement of quantized_matmul "
                      f"(oracle/)"}


def run_reference(args, rank: int) -> dict | None:
    if rank != 0:
        return None
    ob = OracleBlocks(4 if args.workload == "block" else 40, workload=args.workload)
    reps = 1 if args.workload == "block" else SingleLinear.COPIES
    for i in range(args.warmup):
        ob.run_block(i)
    t0 = time.perf_counter()
    for i in range(args.steps * reps):
        ob.run_block(i)
    dt = time.perf_counter() - t0
    value = args.steps * reps * ob.bytes / dt / 1e9
    enc = None if args.no_encoder else cpu_encoder_baseline(args.cpu_seconds)
    return {
        "encoder": enc,
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD if args.workload == "block" else LINEAR_WORKLOAD,
                   "group_size": GROUP, "rows": M_FRAMES,
                   "step": ("one block's 9 linears (1/24 of the GPU arm's step; same metric)"
                            if args.workload == "block" else "40 linears, as the GPU arm")},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": ob.oracle.max_threads(),
                         "kind": "port",
                         "sample": "OpenMP C restatement of MLX quantized_matmul (oracle/); "
                                   "MLX itself cannot run on this host"},
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
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["block", "linear", "batched", "encoder", "rnnt", "logmel"],
                    default="block",
                    help="block: the 24-block M=14 linear chain (default, plus the full "
                         "encoder at 64 streams and at 1 stream as the line's 'encoder' "
                         "object); linear: one 4096x1024 linear, independent back-to-back "
                         "launches; batched: the 24-block chain at M=896 (64 streams), "
                         "tensor-core path; encoder: the full streaming encoder alone "
                         "(value in audio-s/s); rnnt: the batched RNNT greedy decoder alone; "
                         "logmel: the GPU log-mel frontend alone")
    ap.add_argument("--streams", type=int, default=ENC_STREAMS,
                    help="streams per GPU of the encoder, rnnt and logmel workloads")
    ap.add_argument("--encoder-chunks", type=int, default=20,
                    help="timed chunks of the encoder measurement in the default run")
    ap.add_argument("--no-encoder", action="store_true")
    ap.add_argument("--blocks", type=int, default=N_BLOCKS,
                    help="FastConformer blocks in the linear workloads (24 in the encoder; "
                         "fewer only for small profiling captures)")
    ap.add_argument("--chain", action="store_true",
                    help="block workload: the persistent linear chain (one launch per step) "
                         "instead of one K1 launch per linear")
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
