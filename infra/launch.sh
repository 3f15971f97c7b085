#!/usr/bin/env bash
# torchrun wrapper: infra/launch.sh <nproc_per_node> [train_zero.py args...]
# Multi-node: NNODES, NODE_RANK, MASTER_ADDR (default 127.0.0.1) and MASTER_PORT (default 29500).
set -euo pipefail
here="$(cd "$(dirname "$0")/.." && pwd)"
nproc="${1:?nproc_per_node}"; shift
exec python -m torch.distributed.run \
  --nnodes "${NNODES:-1}" --node_rank "${NODE_RANK:-0}" --nproc_per_node "$nproc" \
  --master_addr "${MASTER_ADDR:-127.0.0.1}" --master_port "${MASTER_PORT:-29500}" \
  "$here/train_zero.py" "$@"
