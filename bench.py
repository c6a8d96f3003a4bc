#!/usr/bin/env python3
"""Benchmark driver (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload codec|qlinear]

Workloads
  qlinear  BASELINE cfg1: the quantized-linear microbench.  One step runs all
           15 (shape, M) cases — (K,N) in {(1024,1024),(1024,4096),(4096,1024)}
           x M in {1,3,16,64,256} — each on a distinct weight matrix drawn from
           a pool larger than 2x L2, so weights stream from HBM.  Metric:
           aggregate algorithmic HBM GB/s.
  codec    BASELINE cfg0/cfg4: full encode+decode round trip of 30 s 44.1 kHz
           joint-stereo clips at q=12, batch 3 (x-realtime).  (Enabled once
           the whole-codec path is present in the library.)

Multi-GPU: one process per GPU (torchrun); each rank runs its own replica of
the workload (clips shard with no data-path collective: "scaling": "weak");
the timed region is bracketed by a barrier + cuda synchronize and the max
over ranks is reported.
"""
from __future__ import annotations

import argparse
import ctypes
import json
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
QLINEAR_SHAPES = [(1024, 1024), (1024, 4096), (4096, 1024)]
QLINEAR_MS = [1, 3, 16, 64, 256]


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def qlinear_bytes(k, n, m):
    """Algorithmic bytes of one call (cfg1 formula)."""
    return n * k + 4 * n * k // 256 + 4 * n + m * k + 2 * m * k // 256 + 2 * m * n


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ------------------------------------------------------------------ qlinear --
def qlinear_workload(args, rank, world, torch, dist):
    import tsac_cuda

    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(1 + rank)
    per_step_weight = sum(n * k for k, n in QLINEAR_SHAPES) * len(QLINEAR_MS)
    pool_steps = max(2, -(-2 * L2_BYTES // per_step_weight))
    cases = []  # per pool slot: list of (k, n, m, tensors...)
    for slot in range(pool_steps):
        row = []
        for k, n in QLINEAR_SHAPES:
            for m in QLINEAR_MS:
                w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
                s = (torch.rand((k // 256, n), device=dev) * 1.5 + 0.5) / 127
                b = torch.zeros(n, device=dev)
                x = torch.from_numpy(
                    _bf16(rng.standard_normal((m, k)).astype(np.float32)).view(np.int16)).to(dev)
                y = torch.empty((m, n), dtype=torch.int16, device=dev)
                row.append((k, n, m, w, s, b, x, y))
        cases.append(row)
    scratch = torch.empty(tsac_cuda.qlinear_scratch_bytes(256, 4096), dtype=torch.uint8,
                          device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    per_case_ms = {}

    def step(i, record=None):
        for c, (k, n, m, w, s, b, x, y) in enumerate(cases[i % pool_steps]):
            if record is not None:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            tsac_cuda.qlinear(w, s, b, x, y, scratch, error_word=err)
            if record is not None:
                e1.record(stream)
                record.append((k, n, m, e0, e1))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    records = []
    with ClockSampler(torch.cuda.current_device()) as clocks:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            step(args.warmup + i, records)
        end.record(stream)
        torch.cuda.synchronize()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    assert int(err.item()) == 0
    step_bytes = sum(qlinear_bytes(k, n, m) for k, n in QLINEAR_SHAPES for m in QLINEAR_MS)
    total_bytes = step_bytes * args.steps * world
    value = total_bytes / (elapsed_ms / 1e3) / 1e9
    for k, n, m, e0, e1 in records:
        per_case_ms.setdefault((k, n, m), []).append(e0.elapsed_time(e1))
    sweep = {f"K{k}_N{n}_M{m}": round(qlinear_bytes(k, n, m) / (statistics.mean(v) / 1e3) / 1e9, 1)
             for (k, n, m), v in per_case_ms.items()}
    # Dominant kernel for the roofline: the decode-shaped GEMV call, M=3 on K=N=1024.
    dom = per_case_ms[(1024, 4096, 3)]
    dom_gbs = qlinear_bytes(1024, 4096, 3) / (statistics.mean(dom) / 1e3) / 1e9
    peaks = measured_peaks()
    e2e = qlinear_e2e(args, cases, scratch, err, torch, tsac_cuda)
    return {
        "metric": "qlinear HBM GB/s (cfg1 aggregate)",
        "value": round(value, 1),
        "unit": "GB/s",
        "ms_per_step": round(elapsed_ms / args.steps, 4),
        "dtype": "int8",
        "config": {"workload": "cfg1 quantized-linear microbench", "shapes": QLINEAR_SHAPES,
                   "M": QLINEAR_MS, "weights_pool_bytes": per_step_weight * pool_steps,
                   "l2": "weights cycle through a pool > 2x L2 (HBM-resident)"},
        "sweep_gbs": sweep,
        "roofline": {"bound": "hbm", "achieved": round(dom_gbs, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(dom_gbs / peaks["hbm_gbs"], 4),
                     "traffic": None, "kernel": "qlinear K=1024 N=4096 M=3",
                     "peak_source": peaks["source"]},
        "gpu_launches": 2 * len(QLINEAR_SHAPES) * len(QLINEAR_MS) * args.steps,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }


def qlinear_e2e(args, cases, scratch, err, torch, tsac_cuda):
    """Same workload through the C ABI with host buffers: H2D x, compute, D2H y."""
    row = cases[0]
    host_x = [torch.from_numpy(c[6].cpu().numpy()).pin_memory() for c in row]
    host_y = [torch.empty(tuple(c[7].shape), dtype=torch.int16).pin_memory() for c in row]
    stream = torch.cuda.current_stream()
    h2d = sum(c[6].numel() * 2 for c in row)
    d2h = sum(c[7].numel() * 2 for c in row)

    def step():
        for (k, n, m, w, s, b, x, y), hx, hy in zip(row, host_x, host_y):
            x.copy_(hx, non_blocking=True)
            tsac_cuda.qlinear(w, s, b, x, y, scratch, error_word=err)
            hy.copy_(y, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    step_bytes = sum(qlinear_bytes(k, n, m) for k, n in QLINEAR_SHAPES for m in QLINEAR_MS)
    return {"value": round(step_bytes * args.steps / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "note": "weights resident (model state); activations H2D and outputs D2H each step"}


def qlinear_cpu(threads: int, budget_s: float = 12.0):
    """Reference scalar packed linear (oracle/_ref) on host cores, all cfg1 cases."""
    sys.path.insert(0, str(ROOT / "tests"))
    from concurrent.futures import ThreadPoolExecutor

    lib_path = ROOT / "oracle" / "_ref" / "libtsac_ref.so"
    kind = "reference"
    if lib_path.exists():
        lib = ctypes.CDLL(str(lib_path))
        fn = lib.ref_packed_linear
    else:
        lib = ctypes.CDLL(str(ROOT / "oracle" / "liboracle.so"))
        fn = lib.oracle_linear
        kind = "port"
    rng = np.random.default_rng(7)
    data = []
    for k, n in QLINEAR_SHAPES:
        for m in QLINEAR_MS:
            w = rng.integers(-127, 128, (n, k), dtype=np.int8)
            s = (rng.uniform(0.5, 2, (k // 256, n)) / 127).astype(np.float32)
            b = np.zeros(n, np.float32)
            x = _bf16(rng.standard_normal((m, k)).astype(np.float32))
            y = np.zeros((m, n), np.uint16)
            data.append((k, n, m, w, s, b, x, y))

    def one(case):
        k, n, m, w, s, b, x, y = case
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        fn(p(w), p(s), p(b), ctypes.c_size_t(k), ctypes.c_size_t(n), p(x), ctypes.c_size_t(m), p(y))
        return qlinear_bytes(k, n, m)

    total_bytes, t0 = 0, time.time()
    passes = 0
    with ThreadPoolExecutor(threads) as pool:
        while time.time() - t0 < budget_s or passes == 0:
            total_bytes += sum(pool.map(one, data))
            passes += 1
    elapsed = time.time() - t0
    return {"value": round(total_bytes / elapsed / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": kind,
            "sample": f"{passes} pass(es) over the 15 cfg1 cases, {threads} threads, {elapsed:.1f} s"}


def _bf16(x):
    b = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


# --------------------------------------------------------------------- main --
def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=["qlinear"], default="qlinear")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    common = {"n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
              "data": "synthetic"}
    if args.impl == "reference":
        if rank == 0:
            cpu = qlinear_cpu(os.cpu_count() or 1)
            line = {"impl": "reference", "metric": "qlinear HBM GB/s (cfg1 aggregate)",
                    "value": cpu["value"], "unit": "GB/s", **common, "dtype": "int8",
                    "config": {"workload": "cfg1 quantized-linear microbench",
                               "shapes": QLINEAR_SHAPES, "M": QLINEAR_MS},
                    "cpu_baseline": cpu,
                    "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return
    import torch

    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    result = qlinear_workload(args, rank, world, torch, dist)
    if rank == 0:
        result["cpu_baseline"] = qlinear_cpu(os.cpu_count() or 1, budget_s=10.0)
        line = {**{"metric": result.pop("metric"), "value": result.pop("value"),
                   "unit": result.pop("unit")}, **common, **result}
        line["config"]["parallelism"] = f"replicas x{world}"
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
