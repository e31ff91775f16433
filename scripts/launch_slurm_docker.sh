#!/usr/bin/env bash
# Slurm launcher that runs each node's torchrun inside a container
# (reference scripts/launch_slurm_docker.sh). Same flags as
# scripts/launch_slurm.sh, plus:
#
#   --image IMG          container image (default: $PD_DOCKER_IMAGE or nvcr.io/nvidia/pytorch:25.04-py3)
#   --submit sbatch|srun sbatch queues a batch script (default); srun runs in
#                        the foreground on an allocation (needs --reservation
#                        or an existing allocation)
#
# The project directory is bind-mounted at the same path, so the in-tree
# extension .so files built on the host are the ones the ranks load. The
# container gets every GPU of the node, the host network (NCCL's NVLink / IB
# transports and the torchrun rendezvous), the host IPC namespace (CUDA IPC
# peer handles between ranks) and unlimited locked memory (IB registration).
set -euo pipefail

HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
PROJECT="$(dirname "$HERE")"
MODE=docker
# shellcheck source=scripts/slurm_common.sh
source "$HERE/slurm_common.sh"
slurm_main "$@"
