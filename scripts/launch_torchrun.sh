#!/usr/bin/env bash
# torchrun launcher for scripts/run_distributed.py (reference scripts/launch_torchrun.sh).
#
#   scripts/launch_torchrun.sh --config configs/bench_onetrans_v6_b200.yaml --gpus 8 \
#       [--nnodes 2 --node-rank 0 --master-addr 10.0.0.1] [--] <extra run_distributed.py flags>
#
# Single node by default (rendezvous on 127.0.0.1). Multi-node: the same
# command on every node with its --node-rank and the rank-0 node's address.
# NCCL settings come from the environment (NCCL_DEBUG, NCCL_NVLS_ENABLE,
# NCCL_IB_HCA, ...); PD_ATTN_TC_FWD / PD_ATTN_TC_BWD / PD_KERNELS select kernels.
set -euo pipefail

CONFIG=""
GPUS=8
NNODES=1
NODE_RANK=0
MASTER_ADDR="127.0.0.1"
MASTER_PORT=29500
TIMEOUT_S=0
EXTRA=()
while [[ $# -gt 0 ]]; do
  case "$1" in
    --config) CONFIG="$2"; shift 2 ;;
    --gpus) GPUS="$2"; shift 2 ;;
    --nnodes) NNODES="$2"; shift 2 ;;
    --node-rank) NODE_RANK="$2"; shift 2 ;;
    --master-addr) MASTER_ADDR="$2"; shift 2 ;;
    --master-port) MASTER_PORT="$2"; shift 2 ;;
    --timeout) TIMEOUT_S="$2"; shift 2 ;;
    --) shift; EXTRA+=("$@"); break ;;
    *) EXTRA+=("$1"); shift ;;
  esac
done
if [[ -z "$CONFIG" ]]; then
  echo "usage: $0 --config <yaml> [--gpus N] [--nnodes N --node-rank R --master-addr A] [-- flags]" >&2
  exit 2
fi
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
CMD=(python -m torch.distributed.run --nnodes="$NNODES" --node-rank="$NODE_RANK" --nproc-per-node="$GPUS"
     --master-addr="$MASTER_ADDR" --master-port="$MASTER_PORT"
     "$HERE/run_distributed.py" --config "$CONFIG" "${EXTRA[@]}")
echo "[launch] ${CMD[*]}"
if [[ "$TIMEOUT_S" -gt 0 ]]; then
  exec timeout -k 60 "$TIMEOUT_S" "${CMD[@]}"
fi
exec "${CMD[@]}"
