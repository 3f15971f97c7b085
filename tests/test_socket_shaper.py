"""The LD_PRELOAD socket shaper limits local TCP throughput and shares one bucket across processes."""

from __future__ import annotations

import json
import os
import platform
import socket
import subprocess
import sys
import textwrap
import threading
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SHAPER = ROOT / "infra" / "socket_shaper.so"

pytestmark = pytest.mark.skipif(platform.system() != "Linux", reason="Linux-only LD_PRELOAD shaper")

TRANSFER = textwrap.dedent("""
    import json, socket, threading, time
    TOTAL = 8 * 1024 * 1024
    payload = b"x" * (1 << 20)
    srv = socket.socket(); srv.bind(("127.0.0.1", 0)); srv.listen(1)
    port = srv.getsockname()[1]
    def serve():
        conn, _ = srv.accept(); got = 0
        while got < TOTAL:
            chunk = conn.recv(1 << 20)
            if not chunk: break
            got += len(chunk)
        conn.close()
    t = threading.Thread(target=serve, daemon=True); t.start()
    cli = socket.socket(); cli.connect(("127.0.0.1", port))
    t0 = time.perf_counter(); sent = 0
    while sent < TOTAL:
        cli.sendall(payload[: min(len(payload), TOTAL - sent)]); sent += min(len(payload), TOTAL - sent)
    cli.shutdown(socket.SHUT_WR); t.join()
    dt = time.perf_counter() - t0
    print(json.dumps({"seconds": dt, "mbps": TOTAL * 8 / (dt * 1e6)}))
""")

CLIENT = textwrap.dedent("""
    import socket, sys
    total, host, port = int(sys.argv[1]), sys.argv[2], int(sys.argv[3])
    payload = b"x" * (1 << 20); c = socket.socket(); c.connect((host, port)); sent = 0
    while sent < total:
        n = min(len(payload), total - sent); c.sendall(payload[:n]); sent += n
    c.shutdown(socket.SHUT_WR); c.close()
""")


@pytest.fixture(scope="module")
def shaper() -> Path:
    subprocess.run([sys.executable, str(ROOT / "infra" / "build_socket_shaper.py")], check=True, cwd=ROOT)
    assert SHAPER.exists()
    return SHAPER


def _env(so: Path, bw: str, burst: str, shared: str | None = None, stats: Path | None = None) -> dict:
    env = dict(os.environ)
    env.update(LD_PRELOAD=str(so), ZERO_SOCKET_SHAPER_BW_GBPS=bw, ZERO_SOCKET_SHAPER_LATENCY_MS="0",
               ZERO_SOCKET_SHAPER_BURST_BYTES=burst)
    env.pop("ZERO_SOCKET_SHAPER_SHARED_NAME", None)
    if shared:
        env["ZERO_SOCKET_SHAPER_SHARED_NAME"] = shared
    if stats:
        env["ZERO_SOCKET_SHAPER_STATS_DIR"] = str(stats)
    return env


def test_shaper_limits_throughput_and_writes_stats(shaper: Path, tmp_path: Path) -> None:
    plain = json.loads(subprocess.run([sys.executable, "-c", TRANSFER], check=True, capture_output=True,
                                      text=True).stdout)
    stats = tmp_path / "stats"
    stats.mkdir()
    shaped = json.loads(subprocess.run([sys.executable, "-c", TRANSFER], check=True, capture_output=True, text=True,
                                       env=_env(shaper, "0.1", "65536", stats=stats)).stdout)
    assert shaped["seconds"] > plain["seconds"]
    assert shaped["mbps"] < 140.0  # 0.1 Gbit/s = 100 Mbit/s plus one burst
    files = list(stats.glob("socket_shaper_*.json"))
    assert files
    record = json.loads(files[0].read_text())
    assert record["total_shaped_calls"] > 0 and record["total_shaped_bytes"] > 0
    assert record["total_bandwidth_sleep_s"] > 0.0


def _two_clients(shaper: Path, name_a: str, name_b: str) -> float:
    total = 4 * 1024 * 1024
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(2)
    host, port = srv.getsockname()

    def drain(conn):
        got = 0
        while got < total:
            chunk = conn.recv(1 << 20)
            if not chunk:
                break
            got += len(chunk)
        conn.close()

    readers = []

    def accept():
        for _ in range(2):
            conn, _ = srv.accept()
            th = threading.Thread(target=drain, args=(conn,), daemon=True)
            th.start()
            readers.append(th)

    acc = threading.Thread(target=accept, daemon=True)
    acc.start()
    t0 = time.perf_counter()
    procs = [subprocess.Popen([sys.executable, "-c", CLIENT, str(total), host, str(port)],
                              env=_env(shaper, "0.1", "32768", shared=name)) for name in (name_a, name_b)]
    for p in procs:
        assert p.wait(timeout=60) == 0
    acc.join(timeout=30)
    for th in readers:
        th.join(timeout=30)
    srv.close()
    return time.perf_counter() - t0


def test_shared_bucket_is_one_link_for_all_processes(shaper: Path) -> None:
    tag = str(os.getpid())
    independent = _two_clients(shaper, f"zb_shaper_a_{tag}", f"zb_shaper_b_{tag}")
    shared = _two_clients(shaper, f"zb_shaper_s_{tag}", f"zb_shaper_s_{tag}")
    assert shared > 1.4 * independent
