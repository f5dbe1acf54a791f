"""Shared benchmark harness: device timing, JSONL records, roofline fractions.

Records follow the reference's JSONL benchmark schema (name, device,
world_size, rank, iters, warmup, size, median/p90/min/max ms, baseline_* and
ratio_to_*; reference ``benchmarks/common.py:90-170``) and add what a
multi-GPU B200 measurement needs: ``max_over_ranks_ms`` (the per-iteration
median taken as the maximum over ranks), ``tflops`` / ``gbs`` and
``roofline_frac`` against the measured peaks of the machine
(``MEASURED_PEAKS.json`` at the repository root, when present).

Timing: CUDA events on the launching stream after warm-up, one event pair per
iteration, a barrier and a device synchronize around the timed block.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from contextlib import nullcontext

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                  "nvlink_gbs": 770.0, "source": "fallback"}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    out = dict(FALLBACK_PEAKS)
    try:
        with open(path) as f:
            measured = json.load(f)
        out.update({k: measured[k] for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained") if k in measured})
        out["source"] = "measured"
    except (OSError, ValueError):
        pass
    return out


def parser(description):
    p = argparse.ArgumentParser(description=description)
    p.add_argument("--device", choices=("cpu", "cuda"), default="cuda" if torch.cuda.is_available() else "cpu")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--output", default=None, help="append JSONL records to this file")
    p.add_argument("--size", choices=("small", "medium", "large"), default="small")
    return p


def init_distributed(device):
    if dist.is_initialized():
        return
    if "RANK" not in os.environ:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    if device.type == "cuda":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group("nccl" if device.type == "cuda" else "gloo")


def rank():
    return dist.get_rank() if dist.is_initialized() else 0


def world_size():
    return dist.get_world_size() if dist.is_initialized() else 1


def sync(device):
    if dist.is_initialized():
        dist.barrier()
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def _max_over_ranks(value, device):
    if not dist.is_initialized() or world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_call(fn, *, warmup, iters, device, grad=False):
    """Per-iteration device times in ms (CUDA events) or host times on CPU."""
    ctx = nullcontext() if grad else torch.no_grad()
    with ctx:
        for _ in range(warmup):
            fn()
        sync(device)
        times = []
        for _ in range(iters):
            if device.type == "cuda":
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                fn()
                end.record()
                torch.cuda.synchronize(device)
                times.append(start.elapsed_time(end))
            else:
                t0 = time.perf_counter()
                fn()
                times.append((time.perf_counter() - t0) * 1e3)
        sync(device)
    return times


def percentile(values, frac):
    values = sorted(values)
    return values[min(len(values) - 1, max(0, round((len(values) - 1) * frac)))] if values else 0.0


class Writer:
    def __init__(self, output=None):
        self.output = output

    def write(self, record):
        if rank() != 0:
            return
        line = json.dumps(record, sort_keys=True)
        print(line, flush=True)
        if self.output:
            with open(self.output, "a", encoding="utf-8") as f:
                f.write(line + "\n")


def benchmark(name, fn, *, args, device, writer, flops=None, bytes_moved=None, extra=None, baselines=None,
              grad=False, peak_key="bf16_tflops"):
    times = time_call(fn, warmup=args.warmup, iters=args.iters, device=device, grad=grad)
    med = statistics.median(times)
    worst = _max_over_ranks(med, device)
    record = {"name": name, "device": str(device), "world_size": world_size(), "rank": rank(),
              "iters": args.iters, "warmup": args.warmup, "size": args.size,
              "median_ms": med, "p90_ms": percentile(times, 0.9), "min_ms": min(times), "max_ms": max(times),
              "max_over_ranks_ms": worst}
    pk = peaks()
    if flops:
        record["tflops"] = flops / (worst / 1e3) / 1e12
        record["roofline_frac"] = record["tflops"] / pk[peak_key]
        record["roofline_of"] = f"{pk['source']} {peak_key}"
    elif bytes_moved:
        record["gbs"] = bytes_moved / (worst / 1e3) / 1e9
        record["roofline_frac"] = record["gbs"] / pk["hbm_gbs"]
        record["roofline_of"] = f"{pk['source']} hbm_gbs"
    if extra:
        record.update(extra)
    for key, value in (baselines or {}).items():
        record[f"baseline_{key}_ms"] = value
        if value:
            record[f"ratio_to_{key}"] = worst / value
    writer.write(record)
    return record


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi (every 100 ms) and
    keeps the samples that arrive during the timed region (host-stamped on
    arrival).  Started before the warm-up so the sampler is running when the
    timed region begins; a region shorter than the interval keeps the sample
    nearest to it."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = set(devices)
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001 - clocks are best-effort metadata
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line))

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        self.proc.stdout.close()
        rows = []
        for stamp, line in self.lines:
            cols = [c.strip() for c in line.split(",")]
            if len(cols) < 9 or not cols[0].isdigit() or int(cols[0]) not in self.devices:
                continue
            try:
                rows.append((stamp, float(cols[1]), float(cols[2]), cols[5:9]))
            except ValueError:
                continue
        t0, t1 = self.t0 or 0.0, self.t1 or time.time()
        inside = [r for r in rows if t0 <= r[0] <= t1 + 0.1]
        if not inside and rows:
            mid = 0.5 * (t0 + t1)
            nearest = min(abs(r[0] - mid) for r in rows)
            inside = [r for r in rows if abs(r[0] - mid) == nearest]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = {name for r in inside for name, value in zip(names, r[3]) if value.lower() == "active"}
        sm = sorted(r[1] for r in inside)
        out = {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(r[2] for r in inside) if inside else None,
               "reasons": sorted(reasons), "samples": len(sm)}
        keep = os.environ.get("EINSHARD_CLOCKS_DIR")
        if keep:
            with open(os.path.join(keep, f"einshard_clocks_{os.getpid()}.csv"), "w") as f:
                f.writelines(f"{stamp:.3f},{line}" for stamp, line in self.lines)
        return out


def visible_gpu_indices(world):
    """nvidia-smi indices of this job's GPUs (CUDA_VISIBLE_DEVICES when it lists indices)."""
    listed = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    if listed and all(v.isdigit() for v in listed):
        return [int(v) for v in listed[:world]]
    return list(range(world))
