"""Device timing and clock sampling for benchmarks.

* ``DeviceTimer``: CUDA events on the launching stream, bracketed by a barrier and ``torch.cuda.synchronize()`` on
  both sides; multi-rank results are reduced as the MAX over ranks.
* ``ClockSampler``: runs ``nvidia-smi --query-gpu=... -lms 200`` during the timed region (read-only queries) and
  summarises the SM clock under load and any throttle reasons that were active.
"""

from __future__ import annotations

import csv
import io
import os
import statistics
import subprocess
import tempfile
from typing import Optional

import torch
import torch.distributed as dist

_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
          "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
          "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def max_over_ranks(value: float) -> float:
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([value], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return value


class DeviceTimer:
    """``with DeviceTimer() as t: ...`` then ``t.ms`` (max over ranks)."""

    def __enter__(self):
        barrier()
        torch.cuda.synchronize()
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)
        self.start.record()
        return self

    def __exit__(self, *exc):
        self.end.record()
        torch.cuda.synchronize()
        barrier()
        self.local_ms = self.start.elapsed_time(self.end)
        self.ms = max_over_ranks(self.local_ms)
        return False


class ClockSampler:
    def __init__(self, gpu_index: Optional[int] = None, interval_ms: int = 200) -> None:
        self.gpu_index = gpu_index
        self.interval_ms = interval_ms
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            cmd = ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits", f"-lms", str(self.interval_ms)]
            if self.gpu_index is not None:
                cmd += ["-i", str(self.gpu_index)]
            self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        self.file.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.file.read())) if len(r) >= 10]
        try:
            os.unlink(self.file.name)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x.strip())
            except ValueError:
                return None

        loaded = [r for r in rows if (num(r[4]) or 0) > 50] or rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        reasons = set()
        for r in loaded:
            for name, value in zip(_REASONS, r[6:10]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(loaded[0][2]),
                "power_w_max": max((num(r[3]) or 0) for r in loaded),
                "samples": len(loaded),
                "reasons": sorted(reasons)}
