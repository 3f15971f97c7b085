#!/usr/bin/env bash
# Egress bandwidth limit with a tc token-bucket filter.
#   infra/throttle.sh apply <device> <rate> [burst] [latency]   e.g. apply eth0 10gbit 1mb 10ms
#   infra/throttle.sh delete <device>
#   infra/throttle.sh status <device>
# Needs root (or sudo) for tc.
set -euo pipefail
run_tc() { if [[ "$(id -u)" -eq 0 ]]; then tc "$@"; else sudo tc "$@"; fi; }
cmd="${1:-}"; shift || true
case "$cmd" in
  apply)
    dev="${1:?device}"; rate="${2:?rate}"; burst="${3:-1mb}"; latency="${4:-10ms}"
    run_tc qdisc replace dev "$dev" root tbf rate "$rate" burst "$burst" latency "$latency"
    run_tc qdisc show dev "$dev" ;;
  delete)
    dev="${1:?device}"
    run_tc qdisc del dev "$dev" root 2>/dev/null || true ;;
  status)
    dev="${1:?device}"
    run_tc qdisc show dev "$dev" ;;
  *)
    echo "usage: $0 apply <device> <rate> [burst] [latency] | delete <device> | status <device>" >&2
    exit 1 ;;
esac
