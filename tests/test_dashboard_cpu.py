"""Dashboard server routes (reference test: tests/test_dashboard.py)."""

import importlib.util
import json
import socketserver
import threading
import urllib.request
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _module():
    spec = importlib.util.spec_from_file_location("serve_dashboard", ROOT / "deploy/dashboard/serve_dashboard.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_dashboard_routes(tmp_path):
    mod = _module()
    for name, rows in (("old", 2), ("new", 3)):
        (tmp_path / name).mkdir()
        (tmp_path / name / "metrics.jsonl").write_text(
            "".join(json.dumps({"step": i, "loss": 5.0 - i}) + "\n" for i in range(rows)) + '{"partial')
    import os
    import time

    os.utime(tmp_path / "old" / "metrics.jsonl", (time.time() - 100, time.time() - 100))
    assert [r["name"] for r in mod.discover_runs(tmp_path)] == ["new", "old"]
    monitor = mod.SystemMonitor(interval=0.05)
    monitor.samples = [monitor.sample()]
    server = socketserver.ThreadingTCPServer(("127.0.0.1", 0), mod.make_handler(tmp_path, monitor))
    port = server.server_address[1]
    threading.Thread(target=server.serve_forever, daemon=True).start()
    try:
        get = lambda p: urllib.request.urlopen(f"http://127.0.0.1:{port}{p}").read()  # noqa: E731
        assert b"QuantaWeave" in get("/")
        data = json.loads(get("/api/metrics"))
        assert data["run"] == "new" and len(data["rows"]) == 3
        assert len(json.loads(get("/api/metrics?run=old"))["rows"]) == 2
        system = json.loads(get("/api/system"))
        assert system[0]["cpu_percent"] >= 0 and system[0]["mem_total"] > 0
        try:
            get("/api/metrics?run=../etc")
            raise AssertionError("path traversal accepted")
        except urllib.error.HTTPError as error:
            assert error.code == 404
    finally:
        server.shutdown()
        server.server_close()
