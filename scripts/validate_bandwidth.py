"""Check that a bandwidth limit is really applied before trusting a bandwidth sweep.

Subcommands:

* ``check``    - TCP reachability of host:port and the routed egress device,
* ``server``   - an iperf3 server,
* ``validate`` - iperf3 throughput without and with ``infra/throttle.sh`` (tc tbf) shaping on a device;
                 passes when shaped / baseline <= ``--max-shaped-ratio``.  tc is removed again on exit,
                 SIGINT and SIGTERM,
* ``socket``   - the LD_PRELOAD shaper (``infra/socket_shaper.so``) on loopback: a local TCP transfer
                 without and with ``ZERO_SOCKET_SHAPER_BW_GBPS``; passes when the shaped rate is within
                 ``--tolerance`` of the requested one.  Needs no root, no iperf3 and no second host.

Every subcommand prints (and optionally writes) one JSON record; exit code 0 = pass, 2 = fail.
The first three mirror the reference's ``scripts/validate_bandwidth.py``.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import signal
import socket
import subprocess
import sys
import textwrap
from pathlib import Path
from typing import Dict, List, Optional

ROOT = Path(__file__).resolve().parents[1]
THROTTLE = ROOT / "infra" / "throttle.sh"
_tc_device: Optional[str] = None

TRANSFER = textwrap.dedent("""
    import json, socket, sys, threading, time
    total = int(sys.argv[1]); payload = b"x" * (1 << 20)
    srv = socket.socket(); srv.bind(("127.0.0.1", 0)); srv.listen(1)
    def drain():
        c, _ = srv.accept(); got = 0
        while got < total:
            b = c.recv(1 << 20)
            if not b: break
            got += len(b)
        c.close()
    t = threading.Thread(target=drain); t.start()
    cli = socket.socket(); cli.connect(srv.getsockname()); t0 = time.perf_counter(); sent = 0
    while sent < total:
        n = min(len(payload), total - sent); cli.sendall(payload[:n]); sent += n
    cli.shutdown(socket.SHUT_WR); t.join(); dt = time.perf_counter() - t0
    print(json.dumps({"seconds": dt, "gbps": total * 8 / dt / 1e9}))
""")


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Validate bandwidth shaping (tc + iperf3, or the LD_PRELOAD socket shaper)")
    sub = p.add_subparsers(dest="command", required=True)
    c = sub.add_parser("check", help="Check TCP reachability to a host and port")
    c.add_argument("--target-host", required=True)
    c.add_argument("--port", type=int, default=5201)
    c.add_argument("--connect-timeout-s", type=float, default=5.0)
    c.add_argument("--json-output", default="")
    s = sub.add_parser("server", help="Run an iperf3 server")
    s.add_argument("--bind", default="0.0.0.0")
    s.add_argument("--port", type=int, default=5201)
    s.add_argument("--one-off", action="store_true")
    v = sub.add_parser("validate", help="Measure baseline and tc-shaped throughput with iperf3")
    v.add_argument("--target-host", required=True)
    v.add_argument("--port", type=int, default=5201)
    v.add_argument("--device", required=True)
    v.add_argument("--rate", required=True, help="tc rate, e.g. 10gbit or 500mbit")
    v.add_argument("--burst", default="1mb")
    v.add_argument("--latency", default="10ms")
    v.add_argument("--duration-s", type=int, default=5)
    v.add_argument("--connect-timeout-s", type=float, default=5.0)
    v.add_argument("--iperf-timeout-s", type=int, default=20)
    v.add_argument("--baseline-runs", type=int, default=1)
    v.add_argument("--shaped-runs", type=int, default=1)
    v.add_argument("--max-shaped-ratio", type=float, default=0.8)
    v.add_argument("--allow-route-mismatch", action="store_true")
    v.add_argument("--json-output", default="")
    k = sub.add_parser("socket", help="Measure the LD_PRELOAD socket shaper on loopback")
    k.add_argument("--bw-gbps", type=float, default=0.2)
    k.add_argument("--bytes", type=int, default=16 << 20)
    k.add_argument("--burst-bytes", type=int, default=262144)
    k.add_argument("--tolerance", type=float, default=0.3, help="allowed relative deviation from --bw-gbps")
    k.add_argument("--json-output", default="")
    return p.parse_args(argv)


def _emit(path: str, record: Dict[str, object]) -> None:
    print(json.dumps(record, indent=2))
    if path:
        Path(path).parent.mkdir(parents=True, exist_ok=True)
        Path(path).write_text(json.dumps(record, indent=2) + "\n")


def _route_device(host: str) -> str:
    out = subprocess.run(["ip", "route", "get", host], check=True, text=True, capture_output=True).stdout.split()
    if "dev" not in out:
        raise RuntimeError(f"could not determine the route device for {host!r}")
    return out[out.index("dev") + 1]


def _connect(host: str, port: int, timeout: float) -> Dict[str, object]:
    rec = {"target_host": host, "port": port, "timeout_s": timeout, "routed_device": _route_device(host)}
    try:
        with socket.create_connection((host, port), timeout=timeout):
            pass
        rec.update(connectable=True, error=None)
    except OSError as exc:
        rec.update(connectable=False, error=f"{type(exc).__name__}: {exc}")
    return rec


def _iperf_bps(host: str, port: int, seconds: int, timeout: int) -> float:
    try:
        done = subprocess.run(["iperf3", "-c", host, "-p", str(port), "-t", str(seconds), "-J"], check=True, text=True,
                              capture_output=True, timeout=timeout)
    except subprocess.TimeoutExpired as exc:
        raise RuntimeError(f"iperf3 client timed out after {timeout}s ({host}:{port})") from exc
    except subprocess.CalledProcessError as exc:
        raise RuntimeError(f"iperf3 client failed for {host}:{port}: {(exc.stderr or exc.stdout or '').strip()}") from exc
    end = json.loads(done.stdout).get("end", {})
    summary = end.get("sum_received") or end.get("sum_sent") or {}
    if "bits_per_second" not in summary:
        raise RuntimeError("iperf3 JSON did not contain a summary throughput")
    return float(summary["bits_per_second"])


def _clear_tc(device: str) -> None:
    subprocess.run([str(THROTTLE), "delete", device], check=False, capture_output=True, text=True)


def _on_signal(signum, _frame) -> None:
    global _tc_device
    if _tc_device is not None:
        _clear_tc(_tc_device)
        _tc_device = None
    raise SystemExit(128 + signum)


def run_validate(a: argparse.Namespace) -> int:
    global _tc_device
    for tool in ("iperf3", "ip"):
        if shutil.which(tool) is None:
            raise FileNotFoundError(f"required command not found: {tool}")
    signal.signal(signal.SIGINT, _on_signal)
    signal.signal(signal.SIGTERM, _on_signal)
    routed = _route_device(a.target_host)
    if routed != a.device and not a.allow_route_mismatch:
        raise RuntimeError(f"route to {a.target_host} uses {routed}, not {a.device} (use --allow-route-mismatch)")
    pre = _connect(a.target_host, a.port, a.connect_timeout_s)
    if not pre["connectable"]:
        raise RuntimeError(f"TCP preflight failed: {pre['error']}")
    base = [_iperf_bps(a.target_host, a.port, a.duration_s, a.iperf_timeout_s) for _ in range(a.baseline_runs)]
    try:
        _tc_device = a.device
        subprocess.run([str(THROTTLE), "apply", a.device, a.rate, a.burst, a.latency], check=True, capture_output=True,
                       text=True)
        shaped = [_iperf_bps(a.target_host, a.port, a.duration_s, a.iperf_timeout_s) for _ in range(a.shaped_runs)]
    finally:
        _clear_tc(a.device)
        _tc_device = None
    b, s = sum(base) / len(base), sum(shaped) / len(shaped)
    ratio = s / b if b > 0 else float("inf")
    rec = {"target_host": a.target_host, "port": a.port, "requested_device": a.device, "routed_device": routed,
           "rate": a.rate, "burst": a.burst, "latency": a.latency, "duration_s": a.duration_s,
           "baseline_runs_bps": base, "shaped_runs_bps": shaped, "baseline_mean_gbps": b / 1e9,
           "shaped_mean_gbps": s / 1e9, "shaped_ratio": ratio, "max_shaped_ratio": a.max_shaped_ratio,
           "passed": ratio <= a.max_shaped_ratio}
    _emit(a.json_output, rec)
    return 0 if rec["passed"] else 2


def _transfer(nbytes: int, env: Dict[str, str]) -> Dict[str, float]:
    out = subprocess.run([sys.executable, "-c", TRANSFER, str(nbytes)], check=True, text=True, capture_output=True,
                         env=env, timeout=600).stdout
    return json.loads(out.strip().splitlines()[-1])


def run_socket(a: argparse.Namespace) -> int:
    so = ROOT / "infra" / "socket_shaper.so"
    subprocess.run([sys.executable, str(ROOT / "infra" / "build_socket_shaper.py")], check=True, cwd=ROOT,
                   capture_output=True)
    plain = _transfer(a.bytes, dict(os.environ))
    env = dict(os.environ, LD_PRELOAD=str(so), ZERO_SOCKET_SHAPER_BW_GBPS=str(a.bw_gbps),
               ZERO_SOCKET_SHAPER_BURST_BYTES=str(a.burst_bytes), ZERO_SOCKET_SHAPER_LATENCY_MS="0")
    shaped = _transfer(a.bytes, env)
    dev = abs(shaped["gbps"] - a.bw_gbps) / a.bw_gbps
    rec = {"mode": "socket_shaper_loopback", "requested_gbps": a.bw_gbps, "unshaped_gbps": plain["gbps"],
           "shaped_gbps": shaped["gbps"], "relative_deviation": dev, "tolerance": a.tolerance,
           "bytes": a.bytes, "passed": dev <= a.tolerance}
    _emit(a.json_output, rec)
    return 0 if rec["passed"] else 2


def main(argv: Optional[List[str]] = None) -> int:
    a = parse_args(argv)
    try:
        if a.command == "check":
            if shutil.which("ip") is None:
                raise FileNotFoundError("required command not found: ip")
            rec = _connect(a.target_host, a.port, a.connect_timeout_s)
            _emit(a.json_output, rec)
            return 0 if rec["connectable"] else 2
        if a.command == "server":
            cmd = ["iperf3", "-s", "-B", a.bind, "-p", str(a.port)] + (["-1"] if a.one_off else [])
            subprocess.run(cmd, check=True)
            return 0
        if a.command == "validate":
            return run_validate(a)
        return run_socket(a)
    except Exception as exc:
        if getattr(a, "json_output", ""):
            Path(a.json_output).write_text(json.dumps({"passed": False, "error": f"{type(exc).__name__}: {exc}"}) + "\n")
        raise


if __name__ == "__main__":
    raise SystemExit(main())
