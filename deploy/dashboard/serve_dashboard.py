"""Dependency-free live viewer for training runs with a system-telemetry tab.

    python deploy/dashboard/serve_dashboard.py --runs-dir artifacts/outputs --port 8090

Feature parity with the reference ``deploy/dashboard/serve_dashboard.py`` (``discover_runs``, procfs CPU/RAM,
hardware telemetry, ``SystemMonitor`` sampling thread, ``make_handler`` routes, ``--bind-interface``): it serves
``index.html``, the list of runs under ``--runs-dir`` (newest ``metrics.jsonl`` first, i.e. the active run), one run's
metrics rows, and a live telemetry feed. GPU telemetry on a B200 node comes from NVML (utilisation, HBM used,
power, SM clock and its throttle reasons, temperature) for every GPU. Everything is read-only: NVML is only queried.
"""

from __future__ import annotations

import argparse
import http.server
import json
import re
import socketserver
import subprocess
import threading
import time
from pathlib import Path
from urllib.parse import parse_qs, urlparse

DASHBOARD_DIR = Path(__file__).resolve().parent


def resolve_interface_ip(interface: str) -> str:
    """IPv4 address of a named interface (e.g. a VPN tunnel), so the dashboard listens only there."""
    try:
        out = subprocess.run(["ip", "-4", "-o", "addr", "show", "dev", interface], capture_output=True, text=True,
                             timeout=5, check=True).stdout
    except (subprocess.CalledProcessError, FileNotFoundError) as error:
        raise SystemExit(f"--bind-interface {interface}: could not query it ({error})")
    match = re.search(r"inet (\d+\.\d+\.\d+\.\d+)", out)
    if not match:
        raise SystemExit(f"--bind-interface {interface}: no IPv4 address on that interface")
    return match.group(1)


def discover_runs(runs_dir: Path) -> list[dict]:
    runs = []
    for path in Path(runs_dir).glob("*/metrics.jsonl") if Path(runs_dir).is_dir() else []:
        try:
            st = path.stat()
        except OSError:
            continue
        runs.append({"name": path.parent.name, "mtime": st.st_mtime, "size": st.st_size})
    return sorted(runs, key=lambda r: r["mtime"], reverse=True)


def read_metrics(runs_dir: Path, name: str, tail: int = 5000) -> list[dict]:
    if "/" in name or name.startswith("."):
        raise ValueError("bad run name")
    path = Path(runs_dir) / name / "metrics.jsonl"
    rows = []
    for line in path.read_text().splitlines()[-tail:]:
        try:
            rows.append(json.loads(line))
        except json.JSONDecodeError:
            continue  # a row being written right now
    return rows


def read_proc_stat() -> dict[str, int]:
    with open("/proc/stat") as fh:
        fields = [int(x) for x in fh.readline().split()[1:9]]
    return dict(zip(("user", "nice", "system", "idle", "iowait", "irq", "softirq", "steal"), fields))


def read_meminfo() -> dict[str, int]:
    out = {}
    with open("/proc/meminfo") as fh:
        for line in fh:
            key, _, rest = line.partition(":")
            out[key] = int(rest.split()[0]) * 1024
    return out


def read_gpus() -> list[dict]:
    """One record per GPU from NVML (read-only queries); [] when NVML is unavailable."""
    try:
        import pynvml
    except ImportError:
        return []
    try:
        pynvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver on this host
        return []
    gpus = []
    try:
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            util = pynvml.nvmlDeviceGetUtilizationRates(h)
            mem = pynvml.nvmlDeviceGetMemoryInfo(h)
            gpus.append({"index": i, "name": pynvml.nvmlDeviceGetName(h), "util": util.gpu, "mem_util": util.memory,
                         "mem_used": mem.used, "mem_total": mem.total,
                         "power_w": pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0,
                         "sm_mhz": pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                         "sm_max_mhz": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM),
                         "throttle": pynvml.nvmlDeviceGetCurrentClocksEventReasons(h),
                         "temp_c": pynvml.nvmlDeviceGetTemperature(h, pynvml.NVML_TEMPERATURE_GPU)})
    except Exception as error:  # noqa: BLE001
        gpus.append({"error": str(error)})
    finally:
        pynvml.nvmlShutdown()
    return gpus


class SystemMonitor:
    """Samples CPU %, memory and GPU telemetry once per ``interval`` seconds in a daemon thread."""

    def __init__(self, interval: float = 1.0, history: int = 300) -> None:
        self.interval, self.history = interval, history
        self.samples: list[dict] = []
        self.lock = threading.Lock()
        self._previous = read_proc_stat()
        self._stop = threading.Event()
        self.thread = threading.Thread(target=self._run, daemon=True)

    def start(self) -> "SystemMonitor":
        self.thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()

    def sample(self) -> dict:
        now = read_proc_stat()
        delta = {k: now[k] - self._previous.get(k, 0) for k in now}
        self._previous = now
        busy = sum(v for k, v in delta.items() if k not in ("idle", "iowait"))
        total = sum(delta.values()) or 1
        mem = read_meminfo()
        return {"time": time.time(), "cpu_percent": 100.0 * busy / total,
                "mem_used": mem.get("MemTotal", 0) - mem.get("MemAvailable", 0), "mem_total": mem.get("MemTotal", 0),
                "gpus": read_gpus()}

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            record = self.sample()
            with self.lock:
                self.samples = (self.samples + [record])[-self.history:]

    def snapshot(self) -> list[dict]:
        with self.lock:
            return list(self.samples)


def make_handler(runs_dir: Path, monitor: SystemMonitor):
    class Handler(http.server.BaseHTTPRequestHandler):
        def _send(self, status: int, body: bytes, kind: str) -> None:
            self.send_response(status)
            self.send_header("Content-Type", kind)
            self.send_header("Cache-Control", "no-store")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def _json(self, payload, status: int = 200) -> None:
            self._send(status, json.dumps(payload).encode(), "application/json")

        def do_GET(self) -> None:  # noqa: N802
            url = urlparse(self.path)
            if url.path in ("/", "/index.html"):
                return self._send(200, (DASHBOARD_DIR / "index.html").read_bytes(), "text/html; charset=utf-8")
            if url.path == "/api/runs":
                return self._json(discover_runs(runs_dir))
            if url.path == "/api/metrics":
                runs = discover_runs(runs_dir)
                name = parse_qs(url.query).get("run", [runs[0]["name"] if runs else ""])[0]
                try:
                    return self._json({"run": name, "rows": read_metrics(runs_dir, name)})
                except (OSError, ValueError) as error:
                    return self._json({"error": str(error)}, 404)
            if url.path == "/api/system":
                return self._json(monitor.snapshot())
            return self._json({"error": "not found"}, 404)

        def log_message(self, *_args) -> None:
            pass

    return Handler


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--runs-dir", type=Path, default=Path("artifacts/outputs"))
    p.add_argument("--host", default="127.0.0.1")
    p.add_argument("--bind-interface", help="listen only on this interface's IPv4 address (e.g. a VPN tunnel)")
    p.add_argument("--port", type=int, default=8090)
    args = p.parse_args(argv)
    host = resolve_interface_ip(args.bind_interface) if args.bind_interface else args.host
    monitor = SystemMonitor().start()
    socketserver.ThreadingTCPServer.allow_reuse_address = True
    with socketserver.ThreadingTCPServer((host, args.port), make_handler(args.runs_dir, monitor)) as httpd:
        print(f"dashboard on http://{host}:{args.port} (runs under {args.runs_dir})")
        httpd.serve_forever()


if __name__ == "__main__":
    main()
