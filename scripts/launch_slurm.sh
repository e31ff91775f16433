#!/usr/bin/env bash
# Submit a multi-node training job to Slurm: one srun task per node, each
# starting torchrun with one rank per GPU, every rank running
# scripts/run_distributed.py (reference scripts/launch_slurm.sh).
#
#   scripts/launch_slurm.sh --config configs/bench_onetrans_v6_b200.yaml --nnodes 2 \
#       --run-name v6_2n --partition b200 [--max-steps 1000] [--skip-eval] [--dry-run]
#
# Rendezvous: the first host of the allocation is the torchrun master; with
# --nccl-if the master address is that host's IPv4 on the named interface and
# NCCL / Gloo bootstrap over it. Inside a node the ranks talk over NVLink /
# NVSwitch (NVLS when NCCL enables it); across nodes over InfiniBand
# (--ib-hca picks the HCAs). --dry-run prints the generated batch script and
# submits nothing. Logs go to <results-dir>/<run-name>/logs.
set -euo pipefail

HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
PROJECT="$(dirname "$HERE")"
MODE=bare
# shellcheck source=scripts/slurm_common.sh
source "$HERE/slurm_common.sh"
slurm_main "$@"
