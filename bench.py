#!/usr/bin/env python3
"""Benchmark driver (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload codec|qlinear|frontend] [--clips B] [--seconds S]

Workloads
  codec    (default) the headline metric "x-realtime encode+decode per GPU at
           q=12 stereo": one step = encode + decode of B independent 30 s 44.1 kHz
           joint-stereo clips (cfg0 settings: q=12, --batch_size 3) per GPU,
           through the library's batched C ABI.  `value` is measured with PCM
           resident in HBM (tsac_cuda_encode_batch_device /
           tsac_cuda_decode_batch_device); `e2e` through the host-buffer API
           (CudaAnalyzer.encode_batch / decode_batch: PCM H2D, streams and
           decoded PCM D2H inside the timed region; min(K, 2) steps).  Clips:
           synthetic.music_like with seeds rank*100000 + i; weights: seeded
           package 0.  Default B = 64 clips per GPU, so an 8-GPU step codes
           exactly cfg4's box batch of 512 clips (the decoder's Transformer
           steps are latency-bound, so throughput grows with the batch).  The
           timed steps sit in the NVTX range "timed".
  qlinear  cfg1 quantized-linear microbench (aggregate HBM GB/s).
  frontend encoder front end only (padding, DAC analysis, RVQ) of B clips per
           GPU: the exact-order analysis convolutions in isolation, for
           profiling.
  synthesis  DAC decoder only (RVQ reconstruction + tensor-core synthesis) of
           --frames latent frames of one stereo window batch (profiling).
  decode   Transformer decode steps + range decoding of B clips of S seconds
           (encoded once, untimed), for profiling the decode loop.

Multi-GPU: one process per GPU (torchrun); each rank codes its own clips
(clips shard with no data-path collective: "scaling": "weak"); the timed region
is bracketed by a barrier + cuda synchronize and the max over ranks is taken.
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import multiprocessing as mp
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tsac-metal_b200"))

L2_BYTES = 126 * 1024 * 1024
CLIP_SECONDS = 30.0
QLINEAR_SHAPES = [(1024, 1024), (1024, 4096), (4096, 1024)]
QLINEAR_MS = [1, 3, 16, 64, 256]
SM_COUNT = 148


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "sm_max_mhz": data.get("sm_max_mhz", 1965.0), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, torch):
        props = torch.cuda.get_device_properties(torch.cuda.current_device())
        uuid = getattr(props, "uuid", None)
        self.select = f"--id=GPU-{uuid}" if uuid else f"--id={torch.cuda.current_device()}"
        self.samples = []
        self.proc = None
        self.active = False

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", self.select, f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and self.active:
                self.samples.append(parts)

    def stop(self):
        self.active = False
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        mx = [v for v in (num(s[2]) for s in self.samples) if v is not None]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def event_pair(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def max_over_ranks(value, world, torch, dist):
    """Slowest rank's time: every rank takes this collective at the same point."""
    if world == 1:
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_streams(streams, world, rank, torch, dist):
    """All ranks' encoded streams, gathered to every rank over the process
    group (NCCL on GPUs: the only collective on the data path, used to collect
    results); returns the list of all streams in rank order on rank 0, else None.
    Each rank sends one byte tensor of its length-prefixed streams."""
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    payload = b"".join(len(x).to_bytes(8, "little") + bytes(x) for x in streams)
    size = torch.tensor([len(payload)], device=device, dtype=torch.int64)
    sizes = [torch.zeros_like(size) for _ in range(world)]
    dist.all_gather(sizes, size)
    longest = int(max(int(x.item()) for x in sizes))
    buf = torch.zeros(longest, dtype=torch.uint8, device=device)
    if payload:
        buf[: len(payload)] = torch.frombuffer(bytearray(payload), dtype=torch.uint8).to(device)
    parts = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    if rank != 0:
        return None
    out = []
    for n, part in zip(sizes, parts):
        raw = part[: int(n.item())].cpu().numpy().tobytes()
        at = 0
        while at < len(raw):
            length = int.from_bytes(raw[at: at + 8], "little")
            out.append(raw[at + 8: at + 8 + length])
            at += 8 + length
    return out


def golden_streams():
    """sha256 of the reference's stream per PCM seed (30 s stereo, q=12, batch
    3): the cfg0 golden (seed 0) and the cfg4 box-batch goldens, all made by
    tests/golden/make_golden.py running the reference scalar path."""
    out = {}
    cfg0 = ROOT / "tests" / "golden" / "cfg0_stereo_30s.json"
    if cfg0.exists():
        out[0] = json.loads(cfg0.read_text())["stream_sha256"]
    for path in sorted((ROOT / "tests" / "golden" / "cfg4").glob("seed_*.json")):
        record = json.loads(path.read_text())
        out[int(record["pcm_seed"])] = record["stream_sha256"]
    return out


def parity_counts(streams, seeds, goldens):
    """(checked, matched): streams whose seed has a reference golden, and how
    many of them are byte-identical to it."""
    checked = matched = 0
    for stream, seed in zip(streams, seeds):
        if seed in goldens:
            checked += 1
            matched += hashlib.sha256(bytes(stream)).hexdigest() == goldens[seed]
    return checked, matched


def sum_over_ranks(values, world, torch, dist):
    """Element-wise sum of small integer counters over ranks (every rank calls it)."""
    if world == 1:
        return list(values)
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor(list(values), device=device, dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [int(x) for x in t.tolist()]


def clip_seeds(rank, clips):
    """PCM seeds of one rank's clips: disjoint across ranks (clip sharding with
    no data-path exchange); rank 0's clip 0 is the cfg0 clip (seed 0)."""
    return [rank * 100000 + i for i in range(clips)]


def host_thread_share(world):
    """Host threads one rank may use for range coding: with several ranks on
    one host, an even share of the CPUs this process may run on (the decode
    loop's workers spin between steps, so oversubscribing the host would slow
    every rank); alone, 0 = the library's automatic choice."""
    local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    if local <= 1:
        return 0
    try:
        cpus = len(os.sched_getaffinity(0))
    except AttributeError:
        cpus = os.cpu_count() or 1
    return max(1, cpus // local)


def whole_job_rate(units_per_rank, world, elapsed_ms_max):
    """Units all ranks processed / the slowest rank's time (units per second)."""
    return units_per_rank * world / (elapsed_ms_max / 1e3)


def launch_count():
    """Kernels the library has launched so far in this process (graph replays
    add their kernel nodes)."""
    import tsac_cuda
    fn = tsac_cuda.library().tsac_cuda_launch_count
    fn.restype = ctypes.c_uint64
    return int(fn())


def kernel_stats():
    import tsac_cuda
    lib = tsac_cuda.library()
    out = ctypes.c_void_p()
    tsac_cuda.check(lib.tsac_cuda_kernel_stats(ctypes.byref(out)))
    text = ctypes.cast(out, ctypes.c_char_p).value.decode()
    lib.tsac_cuda_free(out)
    return json.loads(text)


def fp32_issue_peak(torch):
    """FMUL+FADD issue rate of this GPU (the exact convolution's instruction
    pair) from the library's probe kernel, with the SM clock sampled meanwhile."""
    import tsac_cuda
    lib = tsac_cuda.library()
    rate, ms = ctypes.c_double(), ctypes.c_double()
    clocks = ClockSampler(torch).start()
    clocks.active = True
    status = 0
    for _ in range(3):
        status |= lib.tsac_cuda_fp32_issue_rate(200000, ctypes.byref(rate), ctypes.byref(ms),
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    clocks.active = False
    clocks.stop()
    if status != 0:
        return None
    info = clocks.summary()
    return {"tops": round(rate.value / 1e12, 2), "launch_ms": round(ms.value, 2),
            "sm_mhz": info.get("sm_mhz"),
            "nominal_at_that_clock": round(SM_COUNT * 128 * (info.get("sm_mhz") or 1965.0) * 1e6 / 1e12, 2)}


# -------------------------------------------------------------------- codec --
def codec_workload(args, rank, world, torch, dist):
    import synthetic
    import tsac_cuda

    dev = torch.device("cuda", torch.cuda.current_device())
    clips = args.clips
    opts = tsac_cuda.EncodeOptions(method="normal", codebooks=12, entropy_batch=3)
    host = [synthetic.music_like(seed, args.seconds, 2) for seed in clip_seeds(rank, clips)]
    device_pcm = [torch.from_numpy(p).to(dev) for p in host]
    analyzer = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), torch.cuda.current_device())
    threads = host_thread_share(world)
    analyzer.set_host_threads(threads)
    streams = tsac_cuda.encode_batch_device(analyzer, device_pcm, opts)
    outs = []
    for s in streams:
        ch, spc, _ = tsac_cuda.stream_info(s)
        outs.append(torch.empty((spc, ch), dtype=torch.float32, device=dev))

    def step():
        s = tsac_cuda.encode_batch_device(analyzer, device_pcm, opts)
        tsac_cuda.decode_batch_device(analyzer, s, outs)
        return s

    clocks = ClockSampler(torch).start()
    for _ in range(args.warmup):
        streams = step()
    # Parity: every clip of every rank whose seed has a reference golden
    # (cfg0 = rank 0's clip 0, cfg4's box-batch goldens) is byte-compared.
    seeds = clip_seeds(rank, clips)
    goldens = golden_streams() if args.seconds == CLIP_SECONDS else {}
    parity_checked, parity_matched = sum_over_ranks(parity_counts(streams, seeds, goldens), world,
                                                    torch, dist)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    tsac_cuda.library().tsac_cuda_kernel_timing(1)
    start, end = event_pair(torch)
    torch.cuda.synchronize()
    clocks.active = True
    launches_before = launch_count()
    torch.cuda.nvtx.range_push("timed")  # lets an ncu launch list select the timed steps
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clocks.active = False
    launches = launch_count() - launches_before
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world, torch, dist)
    stats = kernel_stats()
    tsac_cuda.library().tsac_cuda_kernel_timing(0)
    value = whole_job_rate(clips * args.seconds * args.steps, world, elapsed_ms)

    # e2e: the host-buffer API, PCM H2D and PCM/streams D2H inside the region.
    if world > 1:
        dist.barrier()
    s2, e2 = event_pair(torch)
    torch.cuda.synchronize()
    s2.record()
    h2d = d2h = 0
    e2e_steps = min(args.steps, 2)
    gathered = None
    for _ in range(e2e_steps):
        st = analyzer.encode_batch(host, opts)
        decoded = analyzer.decode_batch(st)
        if world > 1:
            gathered = gather_streams(st, world, rank, torch, dist)
        h2d = sum(p.nbytes for p in host)
        d2h = sum(d.samples.nbytes for d in decoded) + sum(len(x) for x in st)
    e2.record()
    torch.cuda.synchronize()
    clocks.stop()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2), world, torch, dist)
    e2e_value = whole_job_rate(clips * args.seconds * e2e_steps, world, e2e_ms)
    # The streams rank 0 gathered (all ranks' clips, rank-major) against the goldens.
    gathered_parity = None
    if gathered is not None:
        all_seeds = [s for r in range(world) for s in clip_seeds(r, clips)]
        gathered_parity = dict(zip(("checked", "matched"), parity_counts(gathered, all_seeds, goldens)))

    # Roofline of the dominant kernel family, from the live CUDA-event timing.
    peaks = measured_peaks()
    dominant = max(stats.items(), key=lambda kv: kv[1]["ms"])
    name, d = dominant
    clock_info = clocks.summary()
    sm_mhz = clock_info.get("sm_mhz") or peaks["sm_max_mhz"]
    if name == "conv_tc":
        # 3xTF32 tcgen05 convolutions: useful FLOPs (one multiply-add per
        # product); the kernel issues three TF32 MMAs per product and TF32
        # runs at half the bf16 rate, so the ceiling is bf16 peak / 6.
        achieved = d["work"] / (d["ms"] / 1e3) / 1e12
        peak = peaks["bf16_tflops"] / 6
        roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 2),
                    "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                    "kernel": name, "peak_source": peaks["source"] + " bf16 / 6 (3xTF32)"}
    elif name.startswith("conv"):
        # Exact-order convolutions issue one FP32 multiply and one add per MAC
        # on the CUDA cores.  Peak: the FMUL+FADD issue rate measured on this
        # GPU by the library's probe (tsac_cuda_fp32_issue_rate), beside the
        # nominal 148 SMs x 128 lanes x median SM clock.
        # traffic: DRAM bytes per MAC of the committed ncu capture of this
        # kernel (bench.py --workload frontend --seconds 4, a 128 -> 128 7-tap
        # layer: 45.8 MB read + 2.5 MB written for 10.10 G MAC; the rest of the
        # output was still in L2 when the launch ended), scaled to the mean
        # launch here by its MACs (streaming activations: bytes grow with MACs).
        achieved = d["work"] / (d["ms"] / 1e3) / 1e12
        nominal = SM_COUNT * 128 * sm_mhz * 1e6 / 1e12
        probe = fp32_issue_peak(torch)
        peak = probe["tops"] if probe else nominal
        traffic = None
        if name == "conv_exact":
            traffic = round((45.8e6 + 2.5e6) / 10.10e9 * (d["work"] / 2) / d["launches"])
        roofline = {"bound": "fp32", "achieved": round(achieved, 2), "peak": round(peak, 2),
                    "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                    "traffic_source": "ncu capture of a smaller launch, scaled by MACs" if traffic else None,
                    "kernel": name,
                    "peak_source": ("measured FMUL+FADD issue rate (tsac_cuda_fp32_issue_rate)" if probe
                                    else f"nominal FP32 issue at median SM clock {sm_mhz} MHz"),
                    "fp32_probe": probe, "nominal_peak": round(nominal, 2),
                    "frac_of_nominal": round(achieved / nominal, 4),
                    "work_per_launch": d["work"] / d["launches"],
                    "avg_launch_ms": d["ms"] / d["launches"]}
    else:
        achieved = d["work"] / (d["ms"] / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                    "kernel": name, "peak_source": peaks["source"]}
    shares = {k: round(v["ms"] / sum(x["ms"] for x in stats.values()), 4) for k, v in stats.items()}
    return {
        "metric": "x-realtime encode+decode (30 s 44.1 kHz joint stereo, q=12, batch 3)",
        "value": round(value, 2),
        "unit": "x realtime",
        "ms_per_step": round(elapsed_ms / args.steps, 2),
        "dtype": "f32+int8 (exact reference arithmetic)",
        "config": {"workload": "cfg0/cfg4: encode+decode of 30 s stereo clips", "clips_per_gpu": clips,
                   "codebooks": 12, "entropy_batch": 3, "seconds_per_clip": args.seconds,
                   "l2": "working set (PCM, activations) far larger than L2 each step",
                   "host_threads_per_rank": threads or "auto",
                   "parity_streams_checked": parity_checked,
                   "parity_streams_matched": parity_matched,
                   "parity_gathered_streams": gathered_parity},
        "roofline": roofline,
        "kernel_time_shares": shares,
        "qlinear": qlinear_summary(torch) if rank == 0 else None,
        "gpu_launches": launches,
        "launches_before_timed": launches_before,
        "clocks": clock_info,
        "e2e": {"value": round(e2e_value, 2), "unit": "x realtime", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "streams_gathered_on_rank0": len(gathered) if gathered is not None else None},
    }


# Reference scalar path (oracle/_ref: the reference's ScalarAnalyzer code
# compiled from its own sources), timed on the host cores.  Each worker process
# prepares the five models once (ref_session_create: exactly the models
# ScalarAnalyzer::encode/decode build inside every call) before timing, so the
# timed region holds coding only.
_REF = {}


def _reference_worker_init():
    import tsac_cuda
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libtsac_ref.so"))
    lib.ref_last_error.restype = ctypes.c_char_p
    handle = ctypes.c_void_p()
    if lib.ref_session_create(str(tsac_cuda.seeded_package(0)).encode(), 2, 12, ctypes.byref(handle)) != 0:
        raise RuntimeError(lib.ref_last_error().decode())
    _REF["lib"], _REF["session"] = lib, handle


def _reference_clip(job):
    """One reference encode (q=12, batch 3) + decode of a stereo clip; returns
    (status, seconds)."""
    import synthetic
    seed, seconds = job
    lib, session = _REF["lib"], _REF["session"]
    pcm = synthetic.music_like(seed, seconds, 2)
    out = ctypes.POINTER(ctypes.c_uint8)()
    n = ctypes.c_size_t()
    t0 = time.time()
    rc = lib.ref_session_encode(session, pcm.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(2),
                                ctypes.c_size_t(pcm.shape[0]), 1, 3, ctypes.byref(out), ctypes.byref(n))
    if rc != 0:
        return rc, time.time() - t0
    stream = bytes(out[: n.value])
    lib.ref_free(out)
    pcm_out = ctypes.POINTER(ctypes.c_float)()
    ns, nc = ctypes.c_size_t(), ctypes.c_uint()
    rc = lib.ref_session_decode(session, stream, ctypes.c_size_t(len(stream)), ctypes.byref(pcm_out),
                                ctypes.byref(ns), ctypes.byref(nc))
    if rc == 0:
        lib.ref_free(pcm_out)
    return rc, time.time() - t0


# The reference codes ~0.006 s of audio per second per core, the same at
# 0.1 s, 0.5 s, 1 s and 30 s clips (measured), so short clips sample its rate
# faithfully; a 30 s clip would take ~80 min per core.
REFERENCE_ARM_SECONDS = 0.5     # --impl reference: ~80 s per step
BASELINE_SAMPLE_SECONDS = 0.1   # cpu_baseline inside our arm: ~16 s


def codec_cpu(steps: int, seconds: float):
    """Reference scalar path on all host cores: per step, one clip of `seconds`
    per core, as independent processes (each with models prepared before timing)."""
    cores = min(os.cpu_count() or 1, 32)
    ctx = mp.get_context("spawn")
    walls = []
    with ctx.Pool(cores, initializer=_reference_worker_init) as pool:
        pool.map(_reference_clip, [(999, 0.02)] * cores)  # every worker prepared and warm
        for step in range(steps):
            t0 = time.time()
            results = pool.map(_reference_clip, [(1000 + step * cores + i, seconds) for i in range(cores)])
            walls.append(time.time() - t0)
            if any(rc for rc, _ in results):
                raise RuntimeError("reference encode/decode failed")
    wall = sum(walls)
    value = cores * seconds * len(walls) / wall
    return {"value": round(value, 5), "unit": "x realtime", "cores": cores, "kind": "reference",
            "sample": f"{len(walls)} step(s) x {cores} processes, each the reference ScalarAnalyzer "
                      f"path encode+decode of one {seconds} s stereo clip (q=12, batch 3), models "
                      f"prepared before timing; {wall:.1f} s wall"}


def frontend_workload(args, rank, world, torch, dist):
    """Encoder front end only (padding, DAC analysis, RVQ) of B clips per GPU:
    the exact-order analysis convolutions in isolation (profiling workload)."""
    import synthetic
    import tsac_cuda

    opts = tsac_cuda.EncodeOptions(method="fast", codebooks=12)
    host = [synthetic.music_like(rank * 100000 + i, args.seconds, 2) for i in range(args.clips)]
    analyzer = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), torch.cuda.current_device())
    for _ in range(args.warmup):
        for p in host:
            analyzer.analyze_tokens(p, opts)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    tsac_cuda.library().tsac_cuda_kernel_timing(1)
    start, end = event_pair(torch)
    launches_before = launch_count()
    start.record()
    for _ in range(args.steps):
        for p in host:
            analyzer.analyze_tokens(p, opts)
    end.record()
    torch.cuda.synchronize()
    launches = launch_count() - launches_before
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world, torch, dist)
    stats = kernel_stats()
    tsac_cuda.library().tsac_cuda_kernel_timing(0)
    conv = stats["conv_exact"]
    peaks = measured_peaks()
    achieved = conv["work"] / (conv["ms"] / 1e3) / 1e12
    peak = SM_COUNT * 128 * peaks["sm_max_mhz"] * 1e6 / 1e12
    return {
        "metric": "x-realtime encoder front end (DAC analysis + RVQ)",
        "value": round(args.clips * args.seconds * args.steps * world / (elapsed_ms / 1e3), 2),
        "unit": "x realtime", "ms_per_step": round(elapsed_ms / args.steps, 2),
        "dtype": "f32 (exact reference order)",
        "config": {"workload": "encoder front end", "clips_per_gpu": args.clips,
                   "seconds_per_clip": args.seconds},
        "roofline": {"bound": "fp32", "achieved": round(achieved, 2), "peak": round(peak, 2),
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "kernel": "conv_exact", "peak_source": "nominal FP32 issue at max SM clock"},
        "gpu_launches": launches,
        "e2e": None,
    }


def profile_workload(args, rank, world, torch, dist):
    """Small single-family workloads for ncu captures: the timed steps sit in
    the NVTX range "timed"; the line reports per-family kernel time."""
    import synthetic
    import tsac_cuda

    analyzer = tsac_cuda.CudaAnalyzer(tsac_cuda.seeded_package(0), torch.cuda.current_device())
    if args.workload == "synthesis":
        tokens = np.random.default_rng(1).integers(0, 1024, (args.frames, 12)).astype(np.uint16)
        latent = analyzer.rvq_decode(2, 12, tokens)
        audio_seconds = args.frames * 512 / 44100

        def step():
            analyzer.dac_synthesis(2, latent)
    else:
        opts = tsac_cuda.EncodeOptions(method="normal", codebooks=12, entropy_batch=3)
        pcms = [synthetic.music_like(rank * 100000 + i, args.seconds, 2) for i in range(args.clips)]
        streams = analyzer.encode_batch(pcms, opts)
        audio_seconds = args.clips * args.seconds

        def step():
            analyzer.decode_batch(streams)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    tsac_cuda.library().tsac_cuda_kernel_timing(1)
    launches_before = launch_count()
    start, end = event_pair(torch)
    torch.cuda.nvtx.range_push("timed")
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    elapsed_ms = start.elapsed_time(end)
    stats = kernel_stats()
    tsac_cuda.library().tsac_cuda_kernel_timing(0)
    analyzer.close()
    total = sum(v["ms"] for v in stats.values()) or 1.0
    return {"metric": f"x-realtime ({args.workload} only; profiling workload)",
            "value": round(audio_seconds * args.steps / (elapsed_ms / 1e3), 2), "unit": "x realtime",
            "ms_per_step": round(elapsed_ms / args.steps, 3), "dtype": "f32+int8",
            "config": {"workload": args.workload, "frames": args.frames, "clips": args.clips,
                       "seconds": args.seconds},
            "kernel_ms": {k: round(v["ms"], 3) for k, v in stats.items()},
            "kernel_time_shares": {k: round(v["ms"] / total, 4) for k, v in stats.items()},
            "gpu_launches": launch_count() - launches_before, "e2e": None}


# ------------------------------------------------------------------ qlinear --
def qlinear_bytes(k, n, m):
    """Algorithmic bytes of one call (cfg1 formula)."""
    return n * k + 4 * n * k // 256 + 4 * n + m * k + 2 * m * k // 256 + 2 * m * n


def _bf16(x):
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def qlinear_workload(args, rank, world, torch, dist):
    """cfg1: for each weight shape, a pool of distinct weight matrices larger
    than 2x L2 is cycled through (every call reads its weights from HBM); for
    each M the pool's calls are captured in one CUDA graph, and the timed
    replay gives the per-call time.  GB/s = algorithmic bytes per call / time.
    A step replays all 15 (shape, M) graphs once."""
    import tsac_cuda

    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(1 + rank)
    scratch = torch.empty(tsac_cuda.qlinear_scratch_bytes(256, 4096), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    graphs, calls, pool_bytes = {}, {}, 0
    keep = []  # every tensor a captured graph reads stays alive while the graphs do
    for k, n in QLINEAR_SHAPES:
        pool = max(2, -(-2 * L2_BYTES // (n * k)))
        weights = [(torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev),
                    (torch.rand((k // 256, n), device=dev) * 1.5 + 0.5) / 127) for _ in range(pool)]
        pool_bytes += pool * (n * k + 4 * n * k // 256)
        bias = torch.zeros(n, device=dev)
        for m in QLINEAR_MS:
            x = torch.from_numpy(_bf16(rng.standard_normal((m, k)).astype(np.float32)).view(np.int16)).to(dev)
            y = torch.empty((m, n), dtype=torch.int16, device=dev)
            tsac_cuda.qlinear(weights[0][0], weights[0][1], bias, x, y, scratch, error_word=err)  # lazy init
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for w, ws in weights:
                    tsac_cuda.qlinear(w, ws, bias, x, y, scratch, error_word=err)
            graphs[(k, n, m)] = g
            calls[(k, n, m)] = pool
            keep += [x, y]
        keep += [weights, bias]
    clocks = ClockSampler(torch).start()
    for _ in range(args.warmup):
        for g in graphs.values():
            g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    per_case = {key: 0.0 for key in graphs}
    marks = []
    clocks.active = True
    start, end = event_pair(torch)
    start.record(stream)
    for _ in range(args.steps):
        for key, g in graphs.items():
            e0, e1 = event_pair(torch)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            marks.append((key, e0, e1))
    end.record(stream)
    torch.cuda.synchronize()
    clocks.active = False
    clocks.stop()
    for key, e0, e1 in marks:
        per_case[key] += e0.elapsed_time(e1)
    elapsed_ms = max_over_ranks(start.elapsed_time(end), world, torch, dist)
    assert int(err.item()) == 0
    step_bytes = sum(qlinear_bytes(k, n, m) * calls[(k, n, m)] for (k, n, m) in graphs)
    value = step_bytes * args.steps * world / (elapsed_ms / 1e3) / 1e9
    sweep = {f"K{k}_N{n}_M{m}": round(qlinear_bytes(k, n, m) * calls[(k, n, m)] * args.steps
                                      / (per_case[(k, n, m)] / 1e3) / 1e9, 1)
             for (k, n, m) in graphs}
    dom_key = (1024, 4096, 3)
    dom_ms = per_case[dom_key] / (args.steps * calls[dom_key])
    dom_gbs = qlinear_bytes(*dom_key) / (dom_ms / 1e3) / 1e9
    peaks = measured_peaks()
    return {
        "metric": "qlinear HBM GB/s (cfg1 aggregate)", "value": round(value, 1), "unit": "GB/s",
        "ms_per_step": round(elapsed_ms / args.steps, 4), "dtype": "int8",
        "config": {"workload": "cfg1 quantized-linear microbench", "shapes": QLINEAR_SHAPES,
                   "M": QLINEAR_MS, "weights_pool_bytes": pool_bytes,
                   "calls_per_step": sum(calls.values()),
                   "l2": "each shape cycles through > 2x L2 of distinct weights (HBM-resident)"},
        "sweep_gbs": sweep,
        "roofline": {"bound": "hbm", "achieved": round(dom_gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(dom_gbs / peaks["hbm_gbs"], 4), "traffic": None,
                     "kernel": "qlinear K=1024 N=4096 M=3 (quantize + matmul, graph-replayed)",
                     "avg_call_ms": round(dom_ms, 5), "peak_source": peaks["source"]},
        "gpu_launches": 2 * sum(calls.values()) * args.steps,
        "clocks": clocks.summary(),
        "e2e": None,
    }


def qlinear_summary(torch, steps=20):
    """cfg1 (the metric's "qlinear HBM GB/s") measured beside the codec step,
    as --workload qlinear measures it: aggregate and per-shape GB/s of
    algorithmic bytes with every call's weights read from HBM."""
    class Args:
        pass
    a = Args()
    a.steps, a.warmup = steps, 3
    r = qlinear_workload(a, 0, 1, torch, None)
    return {"aggregate_gbs": r["value"], "unit": "GB/s",
            "frac_of_hbm": round(r["value"] / measured_peaks()["hbm_gbs"], 4),
            "per_shape_gbs": r["sweep_gbs"], "roofline": r["roofline"], "ms_per_step": r["ms_per_step"],
            "steps": steps, "clocks": r["clocks"], "config": r["config"]}


# --------------------------------------------------------------------- main --
def main():
    import faulthandler
    faulthandler.enable()  # a crash in native code still prints the Python stack
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=["codec", "qlinear", "frontend", "synthesis", "decode"],
                        default="codec")
    parser.add_argument("--frames", type=int, default=172, help="latent frames (synthesis workload)")
    parser.add_argument("--clips", type=int, default=64, help="clips per GPU per step (8 x 64 = cfg4's 512)")
    parser.add_argument("--seconds", type=float, default=CLIP_SECONDS,
                        help="clip length (30 s is the benchmark; shorter for profiling runs)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    common = {"n_gpus": world, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "data": "synthetic (seeded music-like PCM; seeded random-init weights)"}
    if args.impl == "reference":
        if rank == 0:
            steps_run = max(1, min(args.steps, 2))
            cpu = codec_cpu(steps_run, REFERENCE_ARM_SECONDS)
            line = {"impl": "reference",
                    "metric": "x-realtime encode+decode (30 s 44.1 kHz joint stereo, q=12, batch 3)",
                    "value": cpu["value"], "unit": "x realtime", **common,
                    "steps": steps_run, "steps_requested": args.steps, "warmup": 0,
                    "dtype": "f32+int8 (exact reference arithmetic)",
                    "config": {"workload": "cfg0/cfg4: encode+decode of stereo clips (q=12, batch 3)",
                               "codebooks": 12, "entropy_batch": 3,
                               "reference_sample": f"{REFERENCE_ARM_SECONDS} s clips, one per host core "
                                                   "per step (a 30 s clip takes ~80 min per core)"},
                    "cpu_baseline": cpu,
                    "e2e": {"value": cpu["value"], "unit": "x realtime", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return
    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    if args.workload == "codec":
        result = codec_workload(args, rank, world, torch, dist)
    elif args.workload == "frontend":
        result = frontend_workload(args, rank, world, torch, dist)
    elif args.workload in ("synthesis", "decode"):
        result = profile_workload(args, rank, world, torch, dist)
    else:
        result = qlinear_workload(args, rank, world, torch, dist)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = (codec_cpu(1, BASELINE_SAMPLE_SECONDS)
                                      if args.workload == "codec" else None)
        line = {"metric": result.pop("metric"), "value": result.pop("value"),
                "unit": result.pop("unit"), **common, **result}
        line["config"]["parallelism"] = (f"clip sharding over {world} GPU(s); no collective in the "
                                         "compute path; streams gathered to rank 0 over NCCL in e2e"
                                         if world > 1 else "1 GPU")
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
