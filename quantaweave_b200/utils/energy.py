"""GPU energy and electricity-cost tracking for training runs (reference ``src/energy_tracking.py``).

Energy sources, first that answers wins:

1. NVML's cumulative energy counter (``nvmlDeviceGetTotalEnergyConsumption``, millijoules) for the current CUDA
   device: read-only, available on B200;
2. a sysfs hwmon ``energy*_input`` sensor labelled ``card`` (microjoules), the reference's source.

Every field is best-effort: with no sensor ``sample()`` returns ``{}``. Cumulative kWh resumes from the last
``energy_kwh_cumulative`` written to the metrics file.
"""

from __future__ import annotations

import glob
import json
import time
from pathlib import Path
from typing import Callable, Optional

JOULES_PER_KWH = 3.6e6


def _hwmon_card_energy_uj() -> Optional[int]:
    for hwmon in glob.glob("/sys/class/hwmon/hwmon*") + glob.glob("/sys/class/drm/card*/device/hwmon/hwmon*"):
        for entry in glob.glob(f"{hwmon}/energy*_input"):
            try:
                if Path(entry.replace("_input", "_label")).read_text().strip() != "card":
                    continue
                return int(Path(entry).read_text().strip())
            except OSError:
                continue
    return None


def _nvml_reader() -> Optional[Callable[[], Optional[int]]]:
    try:
        import pynvml
        import torch

        if not torch.cuda.is_available():
            return None
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        pynvml.nvmlDeviceGetTotalEnergyConsumption(handle)
    except Exception:  # noqa: BLE001 - no NVML, no device, or no counter
        return None

    def read() -> Optional[int]:
        try:
            return int(pynvml.nvmlDeviceGetTotalEnergyConsumption(handle)) * 1000  # mJ -> uJ
        except Exception:  # noqa: BLE001
            return None

    return read


def _last_logged_kwh(path: Path) -> float:
    try:
        with path.open("rb") as handle:
            handle.seek(0, 2)
            size = handle.tell()
            handle.seek(max(0, size - 8192))
            lines = handle.read().splitlines()
        for line in reversed(lines):
            if not line.strip():
                continue
            record = json.loads(line)
            return float(record.get("energy_kwh_cumulative", 0.0))
    except (OSError, ValueError):
        pass
    return 0.0


class PowerCostTracker:
    """Call ``sample()`` at each metrics log and merge the returned dict into the record."""

    def __init__(self, rate_usd_per_kwh: Optional[float], resume_from: Optional[Path] = None,
                 reader: Optional[Callable[[], Optional[int]]] = None) -> None:
        self.rate = rate_usd_per_kwh
        self.energy_kwh = _last_logged_kwh(Path(resume_from)) if resume_from and Path(resume_from).exists() else 0.0
        self._read = reader or _nvml_reader() or _hwmon_card_energy_uj
        self._last_uj = self._read()
        self._last_time = time.perf_counter()
        self.available = self._last_uj is not None

    def sample(self) -> dict:
        if not self.available:
            return {}
        now = time.perf_counter()
        current = self._read()
        dt = now - self._last_time
        self._last_time = now
        watts = None
        if current is not None and self._last_uj is not None and dt > 0:
            delta = current - self._last_uj
            if delta >= 0:
                watts = delta / 1e6 / dt
                self.energy_kwh += delta / 1e6 / JOULES_PER_KWH
        if current is not None:
            self._last_uj = current
        record = {"gpu_power_watts": watts, "energy_kwh_cumulative": self.energy_kwh}
        if self.rate is not None:
            record["cost_usd_cumulative"] = self.energy_kwh * self.rate
        return record
