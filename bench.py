#!/usr/bin/env python3
"""Benchmark: FlowLM frames/s on B200 (the batched FlowLM configuration).

Workload (one "step"): 256 independent Pocket-TTS-shaped FlowLM streams
(6 layers, d 1024, 16 heads × 64, FFN 4096, Q8_0 weights; flow head
1024→512→32, one LSD step), each starting from its own 64-position
prefilled KV cache (seed i), run for 512 autoregressive frames: every
frame is flowLM.step + flowHead.sample for all streams with the latent
fed back on the device. Synthetic seeded weights and inputs (no network,
the reference ships no weights). Metric: stream-frames per second, whole
job (all GPUs).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

`value` times K steps with the noise already in HBM (CUDA events on the
library's stream, barrier + synchronize around the K steps, max over
ranks); `e2e` times the public per-frame C-ABI call (grx_streams_step)
with pinned host buffers, i.e. the host→device noise copy and the
device→host latent/eos/scaled copies of every frame inside the timed
region. `roofline` is the attention kernel (the dominant one: it streams
the float32 KV caches) measured live from its own %globaltimer span in
every launch of the timed steps. `cpu_baseline` is the reference's
algorithm (the C++ restatement in oracle/, the reference being Go, which
this image cannot build) on this box's host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS = ROOT / "MEASURED_PEAKS.json"
METRIC = "FlowLM frames/s (stream-frames per second, whole job)"
UNIT = "frames/s"
TRAFFIC_PER_ALGO = 143.51e6 / 139.79e6  # k_attn DRAM bytes / algorithmic bytes, measured (ncu)
C0_FRAMES = 256  # one stream, 256 frames from a 64-position prefill
# DRAM bytes per frame of the persistent one-stream kernel, from one ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum = 774.2 MB for a
# launch of 16 frames that starts from a cold L2).
C0_TRAFFIC_PER_FRAME = 774.2e6 / 16


def peaks():
    try:
        p = json.loads(PEAKS.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (the recipe's clocks line)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.lines = device, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_workload(n, seed0=1, prefill=64, layers=6, d=1024):
    """Per-stream voices [layers][2][prefill][d] of N(0,1), seeds seed0..seed0+n-1."""
    from gorelaxor_b200 import synth

    cfg = synth.FlowLMConfig()
    vs = []
    for i in range(n):
        v = synth.voice_tensors(cfg, prefill, seed0 + i)
        vs.append(np.stack([np.stack([v[f"voice.{l}.k"], v[f"voice.{l}.v"]]) for l in range(layers)]))
    return cfg, vs


def sample_prefill(run_frames, frames, prefill=64):
    """The prefill length at which `frames` sampled frames attend, on
    average, as many keys as the `run_frames` frames of a run from `prefill`
    positions do (frame f attends prefill + f + 1 keys)."""
    return max(1, prefill + run_frames // 2 - frames // 2)


class CpuFlowLM:
    """The reference's algorithm on the host: the oracle's fast mode (the
    reference's SIMD kernels restated in their lane order, bit-identical to
    the exact restatement; AVX-512 VNNI int8 tiles where the processor has
    them), built once and warmed up before anything is timed."""

    def __init__(self, cfg, tensors):
        from oracle import oracle as orc

        self.cfg, self.orc = cfg, orc
        self.om = orc.FlowLM(cfg, tensors)
        with orc.fast_mode() as fm:
            self.kind = {2: "AVX-512 VNNI", 1: "AVX2", 0: "scalar"}[fm.kind]
        self.sample(1, 2, 8, 1)  # packs the weight panels

    def sample(self, streams, frames, prefill, threads):
        """`streams` independent streams × `frames` frames from `prefill`
        positions on `threads` threads (one stream per thread; a single
        stream splits its products over them). Returns frames/s and the
        wall time of the timed frames."""
        from gorelaxor_b200 import synth

        cfg = self.cfg
        _, vs = make_workload(streams, prefill=prefill)
        sts = [self.om.stream(kv) for kv in vs]
        del vs
        noise = np.stack([synth.noise_frames(1 + i, frames, cfg.ldim, cfg.temperature) for i in range(streams)], axis=1)
        with self.orc.fast_mode():
            t0 = time.perf_counter()
            self.om.run(sts, noise, threads=threads)
            dt = time.perf_counter() - t0
        return streams * frames / dt, dt


def cpu_sample(cfg, tensors, streams, frames, threads, run_frames=512, cpu=None):
    """C1's CPU baseline: `streams` streams × `frames` frames at the run's
    mean key count, one stream per thread. Returns frames/s, the wall time
    and the prefill used."""
    cpu = cpu or CpuFlowLM(cfg, tensors)
    pre = sample_prefill(run_frames, frames)
    cpu.sample(min(streams, threads), 2, pre, threads)  # warm-up at the same shape
    v, dt = cpu.sample(streams, frames, pre, threads)
    return v, dt, pre


def run_reference(args, rank, world):
    """--impl reference: the reference's algorithm on the host cores."""
    if rank != 0:
        return
    from gorelaxor_b200 import synth

    cores = os.cpu_count() or 1
    if args.workload == "tdt":
        cfg = synth.TDTConfig()
        tensors = synth.tdt_tensors(cfg, 0)
        streams, frames = min(args.batch, cores), 100
        tdt_cpu_sample(cfg, tensors, streams, 10, cores)
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = tdt_cpu_sample(cfg, tensors, streams, frames, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        sample = f"{streams} streams x {frames} encoder frames per step, {cores} threads"
        print(json.dumps({
            "impl": "reference", "metric": TDT_METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"C3 TDT decode, {args.batch} streams x {args.frames} frames (sampled)",
                       "global_batch": args.batch, "frames": args.frames, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    if args.workload == "whisper":
        cfg = synth.WhisperConfig()
        tensors = synth.whisper_tensors(cfg, 0)
        words = synth.whisper_words(cfg)
        streams, steps = min(args.batch, cores), 8
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = whisper_cpu_sample(cfg, tensors, words, streams, steps, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        sample = f"{streams} streams x {steps} tokens per step incl. cross K/V and prompt, {cores} threads"
        print(json.dumps({
            "impl": "reference", "metric": WHISPER_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0->f16/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"C2 Whisper, {args.batch} streams x {args.frames} tokens (sampled)",
                       "global_batch": args.batch, "tokens": args.frames, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    if args.workload == "fconf":
        fc = fconf_config()
        tensors = synth.fconf_tensors(fc, 0)
        utts = min(args.batch, cores)
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = fconf_cpu_sample(fc, tensors, utts, args.frames, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        print(json.dumps({
            "impl": "reference", "metric": FCONF_METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"Parakeet TDT 0.6B encoder, {args.batch} utterances x {args.frames} frames "
                                   f"(sampled)", "global_batch": args.batch, "frames": args.frames,
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": utts, "kind": "port",
                             "sample": f"{utts} utterances, one per thread: the subsampling alone and with 1 of "
                                       f"the {fc.layers} blocks, scaled to all blocks"},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    if args.workload == "whisper_encoder":
        cfg = synth.WhisperConfig()
        tensors = synth.whisper_tensors(cfg, 0)
        tensors.update(synth.whisper_encoder_tensors(cfg, 0))
        words = synth.whisper_words(cfg)
        windows = min(args.batch, cores)
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = wenc_cpu_sample(cfg, tensors, words, windows, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        sample = (f"{windows} windows, one per thread: conv front end alone and with 1 of the {cfg.n_audio_layer} "
                  f"blocks, scaled to a whole window; cross K/V prep not included")
        print(json.dumps({
            "impl": "reference", "metric": WENC_METRIC, "value": value, "unit": "windows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f16/Q8_0 weights widened)",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"Whisper base.en encoder + cross K/V, {args.batch} windows (sampled)",
                       "global_batch": args.batch, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "windows/s", "cores": windows, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "windows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    if args.workload == "mimi_encoder":
        mc = mimi_config()
        tensors = synth.mimi_tensors(mc, 32, 0, encoder=True)
        clips, frames = min(args.batch, cores), 12
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = menc_cpu_sample(mc, tensors, clips, frames, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        print(json.dumps({
            "impl": "reference", "metric": MENC_METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"Mimi encode, {args.batch} clips x {args.frames} frames (sampled)",
                       "global_batch": args.batch, "frames": args.frames, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": clips, "kind": "port",
                             "sample": f"{clips} clips x {frames} frames (one piece) per step, one clip per thread"},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    if args.workload == "mimi":
        mc = mimi_config()
        tensors = synth.mimi_tensors(mc, 32, 0)
        streams, frames = min(args.batch, cores), 8
        vals, times = [], []
        for _ in range(args.steps):
            v, dt = mimi_cpu_sample(mc, tensors, streams, frames, cores)
            vals.append(v)
            times.append(dt)
        value = float(np.mean(vals))
        sample = f"{streams} streams x {frames} latents from a fresh state per step, {min(cores, streams)} threads"
        print(json.dumps({
            "impl": "reference", "metric": MIMI_METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": f"Mimi decode, {args.batch} streams x {args.frames} latents (sampled)",
                       "global_batch": args.batch, "frames": args.frames, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "frames/s", "cores": min(cores, streams), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    cfg = synth.FlowLMConfig()
    tensors = synth.flowlm_tensors(cfg, 0)
    cpu = CpuFlowLM(cfg, tensors)
    streams, frames = min(args.batch, cores), 8
    pre = sample_prefill(args.frames, frames)
    for _ in range(args.warmup):
        cpu.sample(streams, 2, pre, cores)
    vals, times = [], []
    for _ in range(args.steps):
        v, dt = cpu.sample(streams, frames, pre, cores)
        vals.append(v)
        times.append(dt)
    value = float(np.mean(vals))
    sample = (f"{streams} streams x {frames} frames per step from {pre}-position prefills (the run's mean of "
              f"{64 + (args.frames + 1) / 2:.1f} keys), one stream per thread, {cores} threads, {cpu.kind} kernels")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/f32",
            "data": "synthetic (seeded; the reference ships no weights)",
            "config": {"workload": "C1 FlowLM, 256 streams x 512 frames (sampled)", "global_batch": args.batch,
                       "frames": args.frames, "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    # C0 (one stream, batch 1): the stream's products split over every thread.
    c0_frames = 32
    c0_pre = sample_prefill(C0_FRAMES, c0_frames)
    cpu.sample(1, 4, c0_pre, cores)
    c0v, c0dt = cpu.sample(1, c0_frames, c0_pre, cores)
    line["c0"] = {"value": c0v, "unit": UNIT, "us_per_frame": 1e6 / c0v, "cores": cores,
                  "sample": f"1 stream x {c0_frames} frames from a {c0_pre}-position prefill, {cores} threads"}
    print(json.dumps(line), flush=True)


TDT_METRIC = "TDT encoder frames/s (stream-frames decoded per second, whole job)"


def tdt_cpu_sample(cfg, tensors, streams, frames, threads):
    """The oracle's Decode on `threads` host threads: `streams` fresh streams
    of `frames` encoder frames. Returns frames/s and the wall time."""
    from gorelaxor_b200 import synth
    from oracle import oracle as orc

    om = orc.TDT(cfg, tensors)
    enc = np.stack([synth.encoder_frames(1 + i, frames, cfg.D) for i in range(streams)])
    with orc.fast_mode():
        t0 = time.perf_counter()
        om.run(enc, 16 * frames + 1024, threads)
        dt = time.perf_counter() - t0
    return streams * frames / dt, dt


def run_tdt(args, rank, world, local):
    """--workload tdt: the Parakeet-TDT-shaped decode loop (C3): `batch`
    streams per GPU of `frames` N(0,1) encoder frames (640 wide); one step =
    Model.Decode of every stream (encoder projection + the greedy loop)."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    B, T = args.batch, args.frames
    cfg = synth.TDTConfig()
    tensors = synth.tdt_tensors(cfg, 0)
    model = g.TDT(synth.tdt_gguf(cfg, tensors), device=local)
    mine = partition(B * world, world, rank)
    enc = np.stack([synth.encoder_frames(1 + s, T, cfg.D) for s in mine])
    cap = 16 * T + 1024
    b = g.TDTBatch(model, B, T, cap)
    Ts = [T] * B
    d_enc = torch.from_numpy(enc).cuda()
    d_tok = torch.empty((B, cap, 4), dtype=torch.int32, device="cuda")
    d_cnt = torch.empty(B, dtype=torch.int32, device="cuda")
    ext = torch.cuda.ExternalStream(b.cuda_stream())

    def one():
        b.reset()
        b.decode_device(d_enc.data_ptr(), Ts, d_tok.data_ptr(), d_cnt.data_ptr())

    for _ in range(args.warmup):
        one()
    clocks = Clocks(local)
    l0, i0 = b.launches(), b.iterations()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks.start()
    ms = []
    for _ in range(args.steps):
        b.reset()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        b.decode_device(d_enc.data_ptr(), Ts, d_tok.data_ptr(), d_cnt.data_ptr())
        e1.record(ext)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches, iters = b.launches() - l0, b.iterations() - i0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * T * world / (total_ms / 1000)
    tokens = int(d_cnt.sum().item())
    stream_iters = b.stream_iterations()
    step_s = total_ms / args.steps / 1000
    # The reference's bytes (conformer/rnnt.go:111-173, each stream on its own):
    # the encoder projection's Q8_0 weight and the stream's encoder rows, per
    # iteration jPred + jOut, per emission the two LSTM layers (Wx, Wh).
    q8 = lambda r, c: r * c * 34 // 32
    per_iter = q8(cfg.J, cfg.H) + q8(cfg.V + len(cfg.durations), cfg.J)
    per_emit = cfg.layers * 2 * q8(4 * cfg.H, cfg.H)
    ref_bytes = B * (q8(cfg.J, cfg.D) + T * cfg.D * 4) + stream_iters * per_iter + (tokens + B) * per_emit
    # What the batched loop must move through HBM per step: the encoder rows,
    # the projection written once and read by the joint (one row per stream
    # iteration), the decoder's 8.1 MB of weights once; the rest stays in L2.
    dev_bytes = B * T * cfg.D * 4 + B * T * cfg.J * 4 + stream_iters * cfg.J * 4 + \
        q8(cfg.J, cfg.D) + per_iter + per_emit
    hbm, peak_kind = peaks()

    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(enc).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            b.reset()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            toks, counts = b.decode(pin, Ts)
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * T * world / (emax / 1000), "unit": "frames/s",
               "h2d_bytes_per_step": enc.nbytes, "d2h_bytes_per_step": B * cap * 16 + B * 4,
               "note": "grx_tdt_decode: encoder output H2D from pinned memory, tokens and counts D2H"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        streams, frames = min(B, cores), 100
        v, dt = tdt_cpu_sample(cfg, tensors, streams, frames, cores)
        cpu = {"value": v, "unit": "frames/s", "cores": cores, "kind": "port",
               "sample": f"{streams} streams x {frames} encoder frames ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": TDT_METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded Q8_0 decoder, N(0,1) encoder output; the reference ships no weights)",
        "config": {"workload": f"C3 TDT decode: {B} streams x {T} encoder frames per GPU", "global_batch": B * world,
                   "frames": T, "parallelism": f"streams partitioned, {world} GPU(s), no collective",
                   "l2": "encoder output 245 MB per GPU, larger than L2"},
        "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck,
        "loop": {"rounds_per_step": iters / args.steps, "stream_iterations_last_step": stream_iters,
                 "tokens_last_step": tokens},
        "roofline": {"bound": "latency/L2", "kernel": "whole decode", "achieved": dev_bytes / step_s / 1e9,
                     "peak": hbm, "unit": "GB/s", "frac": dev_bytes / step_s / 1e9 / hbm, "peak_kind": peak_kind,
                     "traffic": None,
                     "reference_bytes_per_s_gbs": ref_bytes / step_s / 1e9,
                     "note": "achieved = the bytes the batched loop must move through HBM per step (encoder rows, "
                             "the projection written and read back, the weights once) over the step time; the "
                             "decoder's 8.1 MB of Q8_0 weights stay in L2 and every round is a handful of dependent "
                             "launches, so the loop is bound by latency, not HBM. reference_bytes_per_s_gbs counts "
                             "what the reference reads per stream (per iteration jPred+jOut, per emission the "
                             "LSTM, per stream the projection), served here from L2 and shared by the streams"},
    }
    print(json.dumps(line), flush=True)


MIMI_METRIC = "Mimi frames/s (latent frames decoded to 1920-sample audio frames per second, whole job)"


def mimi_config():
    """Pocket TTS's Mimi decoder shape: d 512, 8 heads × 64, FFN 2048, 2
    layers, a 250-position window, 2 rows per latent, SEANet ratios
    (8, 6, 5, 4) with 64 filters: 1920 samples per latent at 24 kHz."""
    from gorelaxor_b200 import synth

    return synth.MimiConfig(d=512, heads=8, ff=2048, layers=2, context=250, upsample=2, ratios=(8, 6, 5, 4), nf=64)


def mimi_latents(streams, frames, ldim=32, seed0=1):
    """[frames][streams][ldim] scaled latents, N(0,1), stream i seeded seed0 + i."""
    return np.stack([np.random.default_rng(seed0 + i).normal(0, 1, (frames, ldim)).astype(np.float32)
                     for i in range(streams)], axis=1)


def mimi_cpu_sample(mc, tensors, streams, frames, threads):
    """The oracle's decoder on host threads: `streams` fresh states ×
    `frames` latents, one thread per stream (ctypes drops the GIL)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc

    om = orc.Mimi(mc, tensors, 32)
    lat = mimi_latents(streams, frames)
    sts = [om.state() for _ in range(streams)]

    def one(i):
        for f in range(frames):
            om.decode(sts[i], lat[f, i])

    with orc.fast_mode():
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=min(threads, streams)) as ex:
            list(ex.map(one, range(streams)))
        dt = time.perf_counter() - t0
    return streams * frames / dt, dt


def run_mimi(args, rank, world, local):
    """--workload mimi: Pocket TTS's Mimi decoder (the next stage of the
    FlowLM loop): `batch` streams per GPU, each decoding `frames` latents in
    order with its streaming state; one step = every stream's frames from a
    fresh state."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    B, F = args.batch, args.frames
    mc = mimi_config()
    tensors = synth.mimi_tensors(mc, 32, 0)
    gm = g.Mimi(synth.flowlm_gguf(synth.FlowLMConfig(), tensors, mimi=mc), device=local)
    mine = partition(B * world, world, rank)
    lat = mimi_latents(len(mine), F, seed0=1 + mine.start)
    s = g.MimiStreams(gm, B, F)
    d_lat = torch.from_numpy(lat).cuda()
    d_pcm = torch.empty((F, B, gm.frame), dtype=torch.float32, device="cuda")
    ext = torch.cuda.ExternalStream(s.cuda_stream())

    def one():
        s.reset()
        s.decode_device(F, d_lat.data_ptr(), d_pcm.data_ptr())

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    l0 = s.launches()
    if dist:
        dist.barrier()
    clocks.start()
    ms = []
    for _ in range(args.steps):
        s.reset()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        s.decode_device(F, d_lat.data_ptr(), d_pcm.data_ptr())
        e1.record(ext)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches = s.launches() - l0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * F * world / (total_ms / 1000)

    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(lat).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            s.reset()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for f in range(F):
                s.decode(pin[f])
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * F * world / (emax / 1000), "unit": "frames/s",
               "h2d_bytes_per_step": int(lat.nbytes), "d2h_bytes_per_step": int(F * B * gm.frame * 4),
               "note": "grx_mimi_decode per frame: latents H2D from pinned memory, samples D2H"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        streams, frames = min(B, cores), 8
        v, dt = mimi_cpu_sample(mc, tensors, streams, frames, cores)
        cpu = {"value": v, "unit": "frames/s", "cores": min(cores, streams), "kind": "port",
               "sample": f"{streams} streams x {frames} latents from a fresh state ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": MIMI_METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded Q8_0/f32 decoder in the converter's types, N(0,1) latents)",
        "config": {"workload": f"Mimi decode: {B} streams x {F} latents per GPU", "global_batch": B * world,
                   "frames": F, "parallelism": f"streams partitioned, {world} GPU(s), no collective",
                   "l2": f"activations {B * 5} MB per GPU per frame, larger than L2"},
        "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck,
    }
    print(json.dumps(line), flush=True)


MENC_METRIC = "Mimi encoder frames/s (1920-sample 24 kHz audio frames encoded to latents per second, whole job)"


def menc_clips(clips, samples, seed0=1):
    """[clips][samples] clip audio, N(0, 0.3), clip i seeded seed0 + i."""
    return np.stack([np.random.default_rng(seed0 + i).normal(0, 0.3, samples).astype(np.float32)
                     for i in range(clips)])


def menc_cpu_sample(mc, tensors, clips, frames, threads):
    """The oracle's cloneCond encoding on host threads, one clip of `frames`
    frames per thread. Returns (frames/s, wall seconds)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc

    om = orc.Mimi(mc, tensors, 32)
    x = menc_clips(clips, frames * mc.frame)
    with orc.fast_mode():
        om.clone_latents(x[0][: mc.frame])  # warm-up
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=min(threads, clips)) as ex:
            list(ex.map(om.clone_latents, list(x)))
        dt = time.perf_counter() - t0
    return clips * frames / dt, dt


def run_mimi_encoder(args, rank, world, local):
    """--workload mimi_encoder: Pocket TTS's Mimi encoder as voice cloning
    runs it (cloneCond, voice.go:113-124): `batch` clips per GPU of `frames`
    1920-sample frames each, encoded together, each from a fresh state; one
    step = every clip."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    B, F = args.batch, args.frames
    mc = mimi_config()
    tensors = synth.mimi_tensors(mc, 32, 0, encoder=True)
    gm = g.Mimi(synth.flowlm_gguf(synth.FlowLMConfig(), tensors, mimi=mc), device=local)
    mine = partition(B * world, world, rank)
    samples = F * gm.frame
    x = menc_clips(len(mine), samples, seed0=1 + mine.start)
    enc = g.MimiEncoder(gm, B, samples)
    d_x = torch.from_numpy(x).cuda()
    d_lat = torch.empty((B, F, gm.ldim), dtype=torch.float32, device="cuda")
    ext = torch.cuda.ExternalStream(enc.cuda_stream())
    for _ in range(args.warmup):
        enc.encode_device(samples, d_x.data_ptr(), d_lat.data_ptr())
        enc.sync()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    l0 = enc.launches()
    if dist:
        dist.barrier()
    clocks.start()
    ms = []
    for _ in range(args.steps):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        enc.encode_device(samples, d_x.data_ptr(), d_lat.data_ptr())
        e1.record(ext)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches = enc.launches() - l0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * F * world / (total_ms / 1000)
    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(x).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            enc.encode(pin)
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * F * world / (emax / 1000), "unit": "frames/s",
               "h2d_bytes_per_step": int(x.nbytes), "d2h_bytes_per_step": int(B * F * gm.ldim * 4),
               "note": "grx_mimi_encode: clips H2D, latents D2H (device buffers allocated per call)"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        clips, frames = min(B, cores), 12
        v, dt = menc_cpu_sample(mc, tensors, clips, frames, cores)
        cpu = {"value": v, "unit": "frames/s", "cores": clips, "kind": "port",
               "sample": f"{clips} clips x {frames} frames (one piece), one clip per thread ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": MENC_METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded Q8_0/f32 encoder in the converter's types, N(0, 0.3) audio)",
        "config": {"workload": f"Mimi encode (voice cloning): {B} clips x {F} frames ({F * 0.08:.1f} s) per GPU",
                   "global_batch": B * world, "frames": F,
                   "parallelism": f"clips partitioned, {world} GPU(s), no collective",
                   "l2": f"activations {B * 23} MB per GPU per piece at the sample rate, larger than L2"},
        "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck}), flush=True)


WENC_METRIC = "Whisper encoder windows/s (30 s log-mel windows encoded, cross K/V included, whole job)"


def wenc_cpu_sample(cfg, tensors, words, windows, threads):
    """The oracle's encoder on host threads, one window per thread: the
    conv front end alone and with one block, scaled to conv + all blocks.
    Returns (windows/s, wall seconds of the sample)."""
    from concurrent.futures import ThreadPoolExecutor

    from gorelaxor_b200 import synth
    from oracle import oracle as orc

    om = orc.Whisper(cfg, tensors, words)
    mels = [synth.whisper_mel(1 + i, cfg) for i in range(windows)]

    def timed(blocks):
        with orc.fast_mode():
            t0 = time.perf_counter()
            with ThreadPoolExecutor(max_workers=min(threads, windows)) as ex:
                list(ex.map(lambda m: om.encode(m, blocks), mels))
            return time.perf_counter() - t0

    t_front, t_one = timed(0), timed(1)
    per_window = t_front + cfg.n_audio_layer * (t_one - t_front)
    return windows / per_window, t_front + t_one


def run_whisper_encoder(args, rank, world, local):
    """--workload whisper_encoder: base.en's audio encoder (conv front end,
    6 blocks of 512 × 8 heads over 1500 positions, final LayerNorm) and the
    decoder layers' cross K/V, for `batch` windows per GPU; one step =
    grx_whisper_encode_device of every window."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    B = args.batch
    cfg = synth.WhisperConfig()
    tensors = synth.whisper_tensors(cfg, 0)
    tensors.update(synth.whisper_encoder_tensors(cfg, 0))
    words = synth.whisper_words(cfg)
    model = g.Whisper(synth.whisper_ggml(cfg, tensors, words), device=local)
    mine = partition(B * world, world, rank)
    mel = np.stack([synth.whisper_mel(1 + s, cfg) for s in mine])
    b = g.WhisperBatch(model, B)
    d_mel = torch.from_numpy(mel).cuda()
    ext = torch.cuda.ExternalStream(b.cuda_stream())
    for _ in range(args.warmup):
        b.encode_device(d_mel.data_ptr())
    clocks = Clocks(local)
    l0 = b.launches()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks.start()
    ms = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        b.encode_device(d_mel.data_ptr())
        e1.record(ext)
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches = b.launches() - l0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * world / (total_ms / 1000)
    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(mel).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            b.encode(pin)
            out = b.encoder_out()
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * world / (emax / 1000), "unit": "windows/s",
               "h2d_bytes_per_step": int(mel.nbytes), "d2h_bytes_per_step": int(out.nbytes),
               "note": "grx_whisper_encode (log-mel from pinned memory, cross K/V prep included), then the "
                       "encoder output read back with grx_whisper_encoder_out"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        windows = min(B, cores)
        v, dt = wenc_cpu_sample(cfg, tensors, words, windows, cores)
        cpu = {"value": v, "unit": "windows/s", "cores": windows, "kind": "port",
               "sample": f"{windows} windows, one per thread: conv front end alone and with 1 of the "
                         f"{cfg.n_audio_layer} blocks, scaled to a whole window; cross K/V prep not included ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    flop = 2 * (3000 * 240 * 512 + 1500 * 1536 * 512 + cfg.n_audio_layer * (
        4 * 1500 * 512 * 512 + 2 * 1500 * 512 * 2048 + 2 * 8 * 1500 * 1500 * 64) + cfg.n_text_layer * 2 * 1500 * 512 * 512)
    print(json.dumps({
        "metric": WENC_METRIC, "value": value, "unit": "windows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (f16/Q8_0 weights widened)",
        "data": "synthetic (seeded weights in whisper.cpp's types, N(-0.3, 0.5) log-mel windows)",
        "config": {"workload": f"Whisper base.en encoder + cross K/V: {B} windows per GPU", "global_batch": B * world,
                   "parallelism": f"windows partitioned, {world} GPU(s), no collective",
                   "l2": "activations and scores well above L2 per window"},
        "fp32_tflops": flop * value / world / 1e12,
        "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck}), flush=True)


FCONF_METRIC = "FastConformer encoder frames/s (80 ms encoder frames per second, whole job)"


def fconf_config():
    """Parakeet TDT 0.6B's encoder shape: d 1024, 8 heads × 128, 24 layers,
    d_ff 4096, 256 subsampling channels, 128 mels, kernel 9."""
    from gorelaxor_b200 import synth

    return synth.FConfConfig(d=1024, heads=8, layers=24, dff=4096, sub_c=256, n_mels=128)


def fconf_cpu_sample(fc, tensors, utts, frames, threads):
    """The oracle's encoder on host threads, one utterance per thread: the
    subsampling alone and with one block, scaled to all blocks. Returns
    (encoder frames/s, wall seconds)."""
    from concurrent.futures import ThreadPoolExecutor

    from gorelaxor_b200 import synth
    from oracle import oracle as orc

    oc = orc.FConf(fc, tensors)
    mels = [synth.fconf_mel(1 + i, fc.n_mels, frames) for i in range(utts)]

    def timed(blocks):
        with orc.fast_mode():
            t0 = time.perf_counter()
            with ThreadPoolExecutor(max_workers=min(threads, utts)) as ex:
                rows = list(ex.map(lambda m: oc.encode(m, None, blocks).shape[0], mels))
            return time.perf_counter() - t0, rows[0]

    (t0, T), (t1, _) = timed(0), timed(1)
    per_utt = t0 + fc.layers * (t1 - t0)
    return utts * T / per_utt, t0 + t1


def run_fconf(args, rank, world, local):
    """--workload fconf: Parakeet TDT 0.6B's FastConformer encoder on
    `batch` utterances of `frames` 10 ms log-mel frames per GPU (one
    grx_fconf_encode_device call each); one step = every utterance."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    B, Fr = args.batch, args.frames
    fc = fconf_config()
    tensors = synth.fconf_tensors(fc, 0)
    gm = g.FConf(synth.fconf_gguf(fc, tensors), device=local)
    mine = partition(B * world, world, rank)
    mel = np.stack([synth.fconf_mel(1 + s, fc.n_mels, Fr) for s in mine])
    d_mel = torch.from_numpy(mel).cuda()
    t = Fr
    for _ in range(3):
        t = (t - 1) // 2 + 1
    T = t
    d_out = torch.empty((B, T, fc.d), dtype=torch.float32, device="cuda")
    ext = torch.cuda.ExternalStream(gm.cuda_stream())

    def one():
        for i in range(B):
            gm.encode_device(d_mel[i].data_ptr(), Fr, Fr, d_out[i].data_ptr())

    for _ in range(args.warmup):
        one()
    gm.sync()
    clocks = Clocks(local)
    l0 = gm.launches()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks.start()
    ms = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        one()
        e1.record(ext)
        gm.sync()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches = gm.launches() - l0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * T * world / (total_ms / 1000)
    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(mel).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for i in range(B):
                out = gm.encode(pin[i])
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * T * world / (emax / 1000), "unit": "frames/s",
               "h2d_bytes_per_step": int(mel.nbytes), "d2h_bytes_per_step": int(B * out.nbytes),
               "note": "grx_fconf_encode per utterance: log-mel in from pinned memory, the encoder rows read back"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        utts = min(B, cores)
        v, dt = fconf_cpu_sample(fc, tensors, utts, Fr, cores)
        cpu = {"value": v, "unit": "frames/s", "cores": utts, "kind": "port",
               "sample": f"{utts} utterances of {Fr} frames, one per thread: the subsampling alone and with 1 of "
                         f"the {fc.layers} blocks, scaled to all blocks ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": FCONF_METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded Q8_0 matrices, float16 1x1 convolutions as the converter keeps them, N(0,1) "
                "log-mel)",
        "config": {"workload": f"Parakeet TDT 0.6B encoder: {B} utterances x {Fr} frames ({T} encoder frames) per GPU",
                   "global_batch": B * world, "frames": Fr,
                   "parallelism": f"utterances partitioned, {world} GPU(s), no collective",
                   "l2": "weights 650 MB, larger than L2"},
        "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck}), flush=True)


WHISPER_METRIC = "Whisper tokens/s (greedy decode tokens per second, whole job)"


def whisper_cpu_sample(cfg, tensors, words, streams, steps, threads):
    """The oracle's window (cross K/V, 4-token prompt, greedy steps) for
    `streams` streams on `threads` host threads: tokens/s and wall time."""
    from gorelaxor_b200 import synth
    from oracle import oracle as orc

    om = orc.Whisper(cfg, tensors, words)
    enc = np.stack([synth.whisper_encoder_out(1 + i, cfg) for i in range(streams)])
    prompt = [50360, 100, 200, 50257]
    with orc.fast_mode():
        t0 = time.perf_counter()
        om.run(enc, prompt, 3, steps, threads)
        dt = time.perf_counter() - t0
    return streams * steps / dt, dt


def run_whisper(args, rank, world, local):
    """--workload whisper: the base.en-shaped decoder (C2): `batch` streams
    per GPU, each with its own N(0,1) encoder output, a 4-token prompt and
    `frames` greedy tokens. A step = the prompt and the token loop of every
    stream; the window's cross K/V prep is timed apart."""
    import torch

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth
    from gorelaxor_b200.dist import max_over_ranks, partition

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    B, T = args.batch, args.frames
    cfg = synth.WhisperConfig()
    tensors = synth.whisper_tensors(cfg, 0)
    words = synth.whisper_words(cfg)
    model = g.Whisper(synth.whisper_ggml(cfg, tensors, words), device=local)
    mine = partition(B * world, world, rank)
    enc = np.stack([synth.whisper_encoder_out(1 + s, cfg) for s in mine])
    b = g.WhisperBatch(model, B)
    d_enc = torch.from_numpy(enc).cuda()
    d_tok = torch.empty((T, B, 4), dtype=torch.int32, device="cuda")
    ext = torch.cuda.ExternalStream(b.cuda_stream())
    prompt = [model.prev, 100, 200, model.sot]

    def one():
        b.set_audio_device(d_enc.data_ptr())
        b.prompt(prompt, 3)
        b.run_device(T, d_tok.data_ptr())
        b.sync()

    for _ in range(args.warmup):
        one()
    clocks = Clocks(local)
    l0 = b.launches()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks.start()
    ms, kv_ms = [], []
    for _ in range(args.steps):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(ext)
        b.set_audio_device(d_enc.data_ptr())
        e1.record(ext)
        b.prompt(prompt, 3)
        b.run_device(T, d_tok.data_ptr())
        e2.record(ext)
        b.sync()
        kv_ms.append(e0.elapsed_time(e1))
        ms.append(e1.elapsed_time(e2))
    ck = clocks.stop()
    launches = b.launches() - l0
    total_ms = max_over_ranks(float(np.sum(ms)), device="cuda")
    value = args.steps * B * T * world / (total_ms / 1000)
    # Algorithmic bytes of a step: per decoded token row the decoder's Q8_0
    # weights once (51.6 MB, the logits product included), and per stream the
    # cross K/V (36.9 MB) and the self K/V rows 0..pos; the prompt pass as one
    # more token.
    st_, L_ = cfg.n_state, cfg.n_text_layer
    wbytes = synth.whisper_q8_bytes(cfg)
    xkv = L_ * 2 * cfg.n_audio_ctx * st_ * 4
    nks = len(prompt) + np.arange(T + 1)
    step_bytes = float(np.sum(wbytes + B * (xkv + L_ * 2 * st_ * 4 * nks)))
    hbm, peak_kind = peaks()
    achieved = step_bytes / (total_ms / args.steps / 1000) / 1e9
    roof = {"bound": "hbm", "kernel": "whole decode step", "achieved": achieved, "peak": hbm, "unit": "GB/s",
            "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": None,
            "bytes_per_token": step_bytes / (B * (T + 1)),
            "note": "algorithmic bytes per step (the decoder's Q8_0 weights once per token row, each stream's cross "
                    "K/V and self K/V rows per token) over the step's device time"}

    e2e = None
    if args.e2e_steps > 0:
        pin = torch.from_numpy(enc).pin_memory().numpy()
        em = []
        for _ in range(args.e2e_steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            b.set_audio(pin)
            b.prompt(prompt, 3)
            b.run(T)
            em.append((time.perf_counter() - t0) * 1000)
        emax = max_over_ranks(float(np.sum(em)), device="cuda")
        e2e = {"value": args.e2e_steps * B * T * world / (emax / 1000), "unit": "tokens/s",
               "h2d_bytes_per_step": enc.nbytes + 4 * B * len(prompt), "d2h_bytes_per_step": T * B * 16 + 4 * B,
               "note": "grx_whisper_set_audio (encoder output from pinned memory, cross K/V prep included), "
                       "grx_whisper_prompt, grx_whisper_run with the tokens read back"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        streams, steps = min(B, cores), 8
        v, dt = whisper_cpu_sample(cfg, tensors, words, streams, steps, cores)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"{streams} streams x {steps} tokens incl. cross K/V and prompt ({dt:.1f} s wall)"}
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": WHISPER_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q8_0->f16/f32",
        "data": "synthetic (seeded Q8_0 decoder, N(0,1) encoder output; the reference ships no weights)",
        "config": {"workload": f"C2 Whisper base.en decoder: {B} streams x {T} greedy tokens from a 4-token prompt",
                   "global_batch": B * world, "tokens": T,
                   "parallelism": f"streams partitioned, {world} GPU(s), no collective",
                   "l2": "cross K/V 36.9 MB per stream (1.2 GB at 32), larger than L2"},
        "cross_kv_ms_per_step": float(np.mean(kv_ms)),
        "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="grx", choices=["grx", "reference"])
    ap.add_argument("--workload", default="flowlm",
                    choices=["flowlm", "tdt", "whisper", "mimi", "mimi_encoder", "whisper_encoder", "fconf"])
    ap.add_argument("--batch", type=int, default=None, help="streams per GPU (flowlm 256, tdt 128)")
    ap.add_argument("--frames", type=int, default=None, help="frames per stream (flowlm 512, tdt 750)")
    ap.add_argument("--e2e-steps", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    args.batch = args.batch or {"flowlm": 256, "tdt": 128, "whisper": 32, "mimi": 256, "mimi_encoder": 16,
                                "whisper_encoder": 8, "fconf": 4}[args.workload]
    args.frames = args.frames or {"flowlm": 512, "tdt": 750, "whisper": 224, "mimi": 32, "mimi_encoder": 125,
                                  "whisper_encoder": 1, "fconf": 3000}[args.workload]
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "tdt":
        return run_tdt(args, rank, world, local)
    if args.workload == "whisper":
        return run_whisper(args, rank, world, local)
    if args.workload == "mimi":
        return run_mimi(args, rank, world, local)
    if args.workload == "mimi_encoder":
        return run_mimi_encoder(args, rank, world, local)
    if args.workload == "whisper_encoder":
        return run_whisper_encoder(args, rank, world, local)
    if args.workload == "fconf":
        return run_fconf(args, rank, world, local)

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # each rank builds its 256 voices (3.2 GB of caches) before the first
        # barrier; with eight ranks on one host that can take minutes
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    import gorelaxor_b200 as g
    from gorelaxor_b200 import synth

    B, F = args.batch, args.frames
    cfg = synth.FlowLMConfig()
    tensors = synth.flowlm_tensors(cfg, 0)
    model = g.FlowLM(synth.flowlm_gguf(cfg, tensors), device=local)
    from gorelaxor_b200.dist import max_over_ranks, partition

    mine = partition(B * world, world, rank)  # this rank's streams of the job (no collective on the step)
    _, kvs = make_workload(len(mine), seed0=1 + mine.start)
    st = g.Streams(model, [model.voice(kv) for kv in kvs], F)
    del kvs
    noise = np.stack([synth.noise_frames(1 + s, F, cfg.ldim, cfg.temperature) for s in mine], axis=1)
    d_noise = torch.from_numpy(noise).cuda()
    d_lat = torch.empty_like(d_noise)
    d_eos = torch.empty((F, B), device="cuda")
    P = st.parts()
    d_ts = torch.empty((F, cfg.layers, P, 2), dtype=torch.int64, device="cuda")
    ext = torch.cuda.ExternalStream(st.cuda_stream())  # the library's stream: events go there

    def one_step(timed_ts=False):
        st.reset()
        if timed_ts:
            d_ts[..., 0] = -1
            d_ts[..., 1] = 0
            torch.cuda.synchronize()
            st.run_device_timed(F, d_noise.data_ptr(), d_lat.data_ptr(), d_eos.data_ptr(), d_ts.data_ptr())
        else:
            st.run_device(F, d_noise.data_ptr(), d_lat.data_ptr(), d_eos.data_ptr())

    for _ in range(args.warmup):
        one_step()
    st.sync()

    # ---- timed: K steps, device-resident inputs ----
    clocks = Clocks(local)
    launches0 = st.launches()
    attn_ns, attn_bytes = [], []
    step_ms = []
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks.start()
    evs = []
    for _ in range(args.steps):
        # reset and the timestamp preset happen before the step's start event
        st.reset()
        d_ts[..., 0] = -1
        d_ts[..., 1] = 0
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        st.run_device_timed(F, d_noise.data_ptr(), d_lat.data_ptr(), d_eos.data_ptr(), d_ts.data_ptr())
        e1.record(ext)
        st.sync()
        evs.append((e0, e1))
        ts = d_ts.cpu().numpy().view(np.uint64)
        attn_ns.append((ts[..., 1] - ts[..., 0]).astype(np.float64))
    step_ms = [a.elapsed_time(b) for a, b in evs]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ck = clocks.stop()
    launches = st.launches() - launches0
    total_ms = max_over_ranks(float(np.sum(step_ms)), device="cuda")
    frames_total = args.steps * B * F * world
    value = frames_total / (total_ms / 1000)

    # attention roofline: algorithmic bytes per launch / its own span
    H, d = cfg.heads, cfg.d
    nk = 64 + np.arange(F) + 1
    per_launch = B * (H * (nk * 64 * 4 * 2 + 64 * 4) + d * 1 + d // 32 * 8)  # K+V reads, q, Q8 out (s,s)
    per_launch = np.repeat(per_launch[:, None], cfg.layers, axis=1).astype(np.float64)
    durs = np.stack(attn_ns)  # [steps][F][L][parts]
    achieved = float(per_launch.sum() * args.steps / durs.sum())  # B/ns = GB/s
    attn_share = float(durs.sum() / 1e6 / np.sum(step_ms) / P)  # of each part's timeline, this rank
    hbm, peak_kind = peaks()
    # DRAM bytes per launch: one ncu capture at 66 keys (256 streams, frame 1,
    # layers 0-1: read+write 143.51 MB against 139.79 MB algorithmic) scaled
    # to every launch by its algorithmic bytes (the K/V rows dominate both).
    traffic = float(per_launch.mean()) * TRAFFIC_PER_ALGO

    # ---- e2e: the public per-frame call with pinned host buffers ----
    e2e = None
    if args.e2e_steps > 0:
        pin_noise = torch.from_numpy(noise).pin_memory().numpy()
        outs = [torch.empty((B, cfg.ldim), pin_memory=True).numpy() for _ in range(2)]
        pe = torch.empty(B, pin_memory=True).numpy()
        e2e_ms = []
        for _ in range(args.e2e_steps):
            st.reset()
            torch.cuda.synchronize()
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            for f in range(F):
                lat, eos, sc, _ = st_step(st, pin_noise[f], outs[0], pe, outs[1])
            t1 = time.perf_counter()
            e2e_ms.append((t1 - t0) * 1000)
        em = max_over_ranks(float(np.sum(e2e_ms)), device="cuda")
        e2e = {"value": args.e2e_steps * B * F * world / (em / 1000), "unit": UNIT,
               "h2d_bytes_per_step": F * B * cfg.ldim * 4,
               "d2h_bytes_per_step": F * B * (2 * cfg.ldim + 1) * 4,
               "note": "grx_streams_step per frame: noise H2D, latent+scaled+eos D2H, host-synchronous"}

    # ---- C0: one stream, on this rank's GPU ----
    c0 = run_c0(g, model, cfg, local, args.warmup, max(3, args.steps // 4)) if world == 1 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        streams, frames = min(64, cores), 8
        cpu_h = CpuFlowLM(cfg, tensors)
        v, dt, pre = cpu_sample(cfg, tensors, streams, frames, cores, run_frames=F, cpu=cpu_h)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{streams} streams x {frames} frames from {pre}-position prefills (the run's mean key "
                         f"count), one stream per thread, {cpu_h.kind} kernels ({dt:.1f} s wall, after a warm-up)"}
        if c0 is not None:
            c0_frames = 32
            pre0 = sample_prefill(C0_FRAMES, c0_frames)
            cpu_h.sample(1, 4, pre0, cores)
            v0, _ = cpu_h.sample(1, c0_frames, pre0, cores)
            c0["cpu_baseline"] = {"value": v0, "unit": UNIT, "cores": cores, "kind": "port",
                                  "sample": f"1 stream x {c0_frames} frames from a {pre0}-position prefill, its "
                                            f"products split over {cores} threads, {cpu_h.kind} kernels"}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/f32",
        "data": "synthetic (seeded Q8_0 weights and N(0,1) prefills; the reference ships no weights)",
        "config": {"workload": "C1 FlowLM batched: 256 streams x 512 frames per GPU from 64-position prefills",
                   "global_batch": B * world, "frames": F, "prefill": 64, "model": "Pocket-TTS-shaped FlowLM",
                   "parallelism": f"streams partitioned, {world} GPU(s), no collective",
                   "l2": "inputs larger than L2 (KV caches 7.3 GB per GPU)"},
        "e2e": e2e,
        "roofline": {"bound": "hbm", "kernel": "k_attn", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": traffic,
                     "traffic_unit": "bytes per launch (ncu dram read+write at 66 keys, scaled by key rows)",
                     "share": attn_share,
                     "note": "algorithmic bytes per launch (K,V rows 0..pos of every head + q + Q8 output) over the "
                             "kernel's own first-CTA-start to last-CTA-end span, every launch of the timed steps"},
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
        "clocks": ck,
        "c0": c0,
    }
    print(json.dumps(line), flush=True)


def c0_bytes_per_frame(cfg, nk):
    """SURVEY-style algorithmic bytes of one batch-1 frame attending nk keys:
    the transformer's and flow head's weights once (Q8_0 at 34/32 bytes per
    value, float32 at 4), lm.input and the EOS row, and the K/V rows read."""
    d, ff, L, fd, ld = cfg.d, cfg.ff, cfg.layers, cfg.flow_dim, cfg.ldim
    q8 = L * (3 * d * d + d * d + ff * d + d * ff)
    q8 += fd * d + cfg.flow_depth * (3 * fd * fd + 2 * fd * fd) + 2 * fd * fd
    f32 = fd * ld + ld * fd + d * ld + d
    return q8 * 34 // 32 + f32 * 4 + L * 2 * d * 4 * nk


def run_c0(g, model, cfg, local, warmup, steps):
    """one stream from a 64-position prefill, 256 frames
    per step, the latent fed back on the device. `value` is device-timed with
    the noise resident in HBM (L2 flushed before each step); `e2e` is the
    public per-frame call with pinned host buffers."""
    import torch

    F = C0_FRAMES
    _, kvs = make_workload(1, seed0=1)
    st = g.Streams(model, [model.voice(kvs[0])], F)
    from gorelaxor_b200 import synth

    noise = synth.noise_frames(1, F, cfg.ldim, cfg.temperature)[:, None, :].copy()
    d_noise = torch.from_numpy(noise).cuda()
    d_lat = torch.empty_like(d_noise)
    d_eos = torch.empty((F, 1), device="cuda")
    ext = torch.cuda.ExternalStream(st.cuda_stream())
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB, twice the L2
    for _ in range(warmup):
        st.reset()
        st.run_device(F, d_noise.data_ptr(), d_lat.data_ptr(), d_eos.data_ptr())
    st.sync()
    clocks = Clocks(local)
    clocks.start()
    l0 = st.launches()
    ms = []
    for _ in range(steps):
        st.reset()
        flush.fill_(1.0)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        st.run_device(F, d_noise.data_ptr(), d_lat.data_ptr(), d_eos.data_ptr())
        e1.record(ext)
        st.sync()
        ms.append(e0.elapsed_time(e1))
    ck = clocks.stop()
    launches = st.launches() - l0
    t = float(np.mean(ms))
    nk = 64 + np.arange(F) + 1
    per_step = float(sum(c0_bytes_per_frame(cfg, int(k)) for k in nk))
    hbm, peak_kind = peaks()
    achieved = per_step / (t / 1000) / 1e9
    # e2e: grx_streams_step per frame, pinned host noise in, latent/scaled/eos out
    pin_noise = torch.from_numpy(noise).pin_memory().numpy()
    outs = [torch.empty((1, cfg.ldim), pin_memory=True).numpy() for _ in range(2)]
    pe = torch.empty(1, pin_memory=True).numpy()
    st.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for f in range(F):
        st_step(st, pin_noise[f], outs[0], pe, outs[1])
    e2e_s = time.perf_counter() - t0
    return {
        "workload": f"C0 FlowLM batch 1: 1 stream x {F} frames from a 64-position prefill",
        "value": F / (t / 1000), "unit": UNIT, "us_per_frame": 1000 * t / F, "steps": steps, "warmup": warmup,
        "e2e": {"value": F / e2e_s, "unit": UNIT, "h2d_bytes_per_step": F * cfg.ldim * 4,
                "d2h_bytes_per_step": F * (2 * cfg.ldim + 1) * 4,
                "note": "grx_streams_step per frame, host-synchronous"},
        "roofline": {"bound": "hbm", "kernel": "whole frame", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_kind": peak_kind, "bytes_per_frame_mean": per_step / F,
                     "traffic": C0_TRAFFIC_PER_FRAME,
                     "traffic_unit": "bytes per frame (ncu dram read+write of one k_frame1 launch of 16 frames "
                                     "from a cold L2, divided by 16)",
                     "limiter": "latency of the frame's dependency chain: 35 grid barriers and the steps between "
                                "them (ncu: warps stalled at barriers 13.2 per issued instruction, DRAM 2.6 % busy)",
                     "note": "algorithmic bytes per frame (Q8_0 weights of the transformer and flow head, float32 "
                             "rows, K/V rows 0..pos) over the frame's device time; the 82.9 MB of weights fit in "
                             "the 126 MB L2, which is flushed before each step but not between the frames of a "
                             "step, so later frames read weights largely from L2"},
        "gpu_launches": int(launches), "clocks": ck,
    }


def st_step(st, noise_row, lat_out, eos_out, sc_out):
    """grx_streams_step into caller-owned (pinned) host buffers."""
    import gorelaxor_b200 as g

    g._check(g.lib().grx_streams_step(st._h, g._ptr(noise_row), None, g._ptr(eos_out), g._ptr(lat_out),
                                      g._ptr(sc_out)))
    return lat_out, eos_out, sc_out, None


if __name__ == "__main__":
    main()
