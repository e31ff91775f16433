# Shared body of scripts/launch_slurm.sh and scripts/launch_slurm_docker.sh
# (sourced; the caller sets HERE, PROJECT and MODE=bare|docker).
#
# Flags follow the reference launchers (scripts/launch_slurm.sh:20-60,
# scripts/launch_slurm_docker.sh:28-120 of the reference project); the
# AMD-only switches (AINIC / RCCL plugin, hipBLASLt tuning files, CK wheels,
# platform probing) have no counterpart on B200 and are not accepted.

slurm_usage() {
  cat >&2 <<'EOF'
usage: launch_slurm[_docker].sh --config <yaml> [options] [-- <extra run_distributed.py flags>]
  --nnodes N            nodes (default 1)            --gpus N           GPUs per node (default 8)
  --max-steps N         0 = the config's epochs      --run-name NAME    (default dist_slurm)
  --results-dir DIR     (default results)            --dense-strategy   ddp | fsdp | zero2 | dmp (default ddp)
  --data-root DIR       dataset root override        --log-interval N   (default 1000)
  --partition P         --time HH:MM:SS (12:00:00)   --job-name NAME    --account A
  --nodelist L          --dependency D               --reservation R    --qos Q
  --nccl-if IF          bootstrap / socket interface --ib-hca LIST      NCCL_IB_HCA for inter-node
  --rdzv-port P         torchrun master port (29500)
  --skip-eval           --pipeline                   --trace [--trace-steps S --trace-warmup W
                        --trace-active A --trace-ranks R]
  --attention-impl I    --comm peer|nccl             --kernels native|eager   --resume PATH|latest
  --hbm-cap-gb G        --ddr-cap-gb G               per-rank planner capacities
  --python PY           interpreter on the nodes (bare mode; default python3)
  --image IMG           container image (docker mode)
  --submit sbatch|srun  queue a batch job, or run it in the foreground through salloc
  --dry-run             print the generated batch script and exit
EOF
}

slurm_main() {
  local NNODES=1 GPUS=8 CONFIG="" DATA_ROOT="" MAX_STEPS=0 RUN_NAME="dist_slurm" RESULTS_DIR="results"
  local DENSE_STRATEGY="ddp" PARTITION="" TIME="12:00:00" JOB_NAME="dlrm_b200" LOG_INTERVAL=1000
  local NCCL_IF="" IB_HCA="" NODELIST="" DEPENDENCY="" RESERVATION="" QOS="" ACCOUNT="" RDZV_PORT=29500
  local HBM_CAP_GB="" DDR_CAP_GB="" SUBMIT="sbatch" DRY_RUN=0 PY="python3"
  local IMAGE="${PD_DOCKER_IMAGE:-nvcr.io/nvidia/pytorch:25.04-py3}"
  local -a RUN_ARGS=() EXTRA=()
  while [[ $# -gt 0 ]]; do
    case "$1" in
      --nnodes|--nodes)  NNODES="$2"; shift 2 ;;
      --gpus)            GPUS="$2"; shift 2 ;;
      --config)          CONFIG="$2"; shift 2 ;;
      --data-root)       DATA_ROOT="$2"; shift 2 ;;
      --max-steps)       MAX_STEPS="$2"; shift 2 ;;
      --run-name)        RUN_NAME="$2"; shift 2 ;;
      --results-dir)     RESULTS_DIR="$2"; shift 2 ;;
      --dense-strategy)  DENSE_STRATEGY="$2"; shift 2 ;;
      --partition)       PARTITION="$2"; shift 2 ;;
      --time)            TIME="$2"; shift 2 ;;
      --job-name)        JOB_NAME="$2"; shift 2 ;;
      --account)         ACCOUNT="$2"; shift 2 ;;
      --log-interval)    LOG_INTERVAL="$2"; shift 2 ;;
      --nccl-if)         NCCL_IF="$2"; shift 2 ;;
      --ib-hca)          IB_HCA="$2"; shift 2 ;;
      --nodelist)        NODELIST="$2"; shift 2 ;;
      --dependency)      DEPENDENCY="$2"; shift 2 ;;
      --reservation)     RESERVATION="$2"; shift 2 ;;
      --qos)             QOS="$2"; shift 2 ;;
      --rdzv-port)       RDZV_PORT="$2"; shift 2 ;;
      --hbm-cap-gb)      HBM_CAP_GB="$2"; shift 2 ;;
      --ddr-cap-gb)      DDR_CAP_GB="$2"; shift 2 ;;
      --python)          PY="$2"; shift 2 ;;
      --image)           IMAGE="$2"; shift 2 ;;
      --submit)          SUBMIT="$2"; shift 2 ;;
      --dry-run)         DRY_RUN=1; shift ;;
      --skip-eval|--trace|--pipeline) RUN_ARGS+=("$1"); shift ;;
      --trace-steps|--trace-warmup|--trace-active|--trace-ranks|--attention-impl|--attn-impl|--comm|--kernels|--resume)
        local f="$1"; [[ "$f" == "--attn-impl" ]] && f="--attention-impl"
        RUN_ARGS+=("$f" "$2"); shift 2 ;;
      -h|--help)         slurm_usage; return 0 ;;
      --)                shift; EXTRA+=("$@"); break ;;
      *) echo "unknown flag: $1" >&2; slurm_usage; return 2 ;;
    esac
  done

  [[ -n "$CONFIG" ]] || { echo "--config is required" >&2; slurm_usage; return 2; }
  [[ "$NNODES" =~ ^[1-9][0-9]*$ && "$GPUS" =~ ^[1-9][0-9]*$ ]] || { echo "--nnodes/--gpus must be positive integers" >&2; return 2; }
  [[ "$MAX_STEPS" =~ ^[0-9]+$ && "$RDZV_PORT" =~ ^[0-9]+$ ]] || { echo "--max-steps/--rdzv-port must be integers" >&2; return 2; }
  case "$DENSE_STRATEGY" in ddp|fsdp|zero2|dmp) ;; *) echo "--dense-strategy must be ddp, fsdp, zero2 or dmp" >&2; return 2 ;; esac
  case "$SUBMIT" in sbatch|srun) ;; *) echo "--submit must be sbatch or srun" >&2; return 2 ;; esac
  local cfg_abs="$CONFIG"
  [[ "$cfg_abs" == /* ]] || cfg_abs="$PROJECT/$CONFIG"
  [[ -f "$cfg_abs" ]] || { echo "config not found: $CONFIG" >&2; return 2; }

  local LOG_DIR="$RESULTS_DIR"
  [[ "$LOG_DIR" == /* ]] || LOG_DIR="$PROJECT/$LOG_DIR"
  LOG_DIR="$LOG_DIR/$RUN_NAME/logs"

  local -a ARGS=(--config "$cfg_abs" --dense-strategy "$DENSE_STRATEGY" --run-name "$RUN_NAME"
                 --results-dir "$RESULTS_DIR" --log-interval "$LOG_INTERVAL")
  [[ "$MAX_STEPS" -gt 0 ]] && ARGS+=(--max-steps "$MAX_STEPS")
  [[ -n "$DATA_ROOT" ]] && ARGS+=(--data-root "$DATA_ROOT")
  ARGS+=("${RUN_ARGS[@]}" "${EXTRA[@]}")

  local torchrun
  torchrun="-m torch.distributed.run --nnodes=\$SLURM_NNODES --node-rank=\$SLURM_NODEID --nproc-per-node=$GPUS"
  torchrun+=" --master-addr=\$MASTER_ADDR --master-port=\$MASTER_PORT $(printf '%q' "$PROJECT/scripts/run_distributed.py")"
  torchrun+=" $(printf '%q ' "${ARGS[@]}")"

  local node_cmd
  if [[ "$MODE" == docker ]]; then
    # every exported variable the ranks read is forwarded by name
    node_cmd="docker run --rm --name pd_\${SLURM_JOB_ID}_\${SLURM_NODEID} --gpus all --network host --ipc host"
    node_cmd+=" --ulimit memlock=-1 --ulimit stack=67108864 --shm-size 64g --cap-add IPC_LOCK"
    node_cmd+=" \$( [[ -d /dev/infiniband ]] && echo --device=/dev/infiniband )"
    node_cmd+=" -v $(printf '%q' "$PROJECT"):$(printf '%q' "$PROJECT") -w $(printf '%q' "$PROJECT")"
    node_cmd+=" \$(for v in \$PD_FORWARD_ENV; do printf -- '-e %s ' \"\$v\"; done)"
    node_cmd+=" $(printf '%q' "$IMAGE") python $torchrun"
  else
    node_cmd="cd $(printf '%q' "$PROJECT") && exec $(printf '%q' "$PY") $torchrun"
  fi

  local script
  script="$(slurm_render)"
  if [[ "$DRY_RUN" -eq 1 ]]; then
    printf '%s\n' "$script"
    return 0
  fi
  mkdir -p "$LOG_DIR"
  local file="$LOG_DIR/${JOB_NAME}_submit_$(date +%Y%m%d_%H%M%S).sh"
  printf '%s\n' "$script" > "$file"
  chmod +x "$file"
  echo "[launch] batch script: $file"
  if [[ "$SUBMIT" == sbatch ]]; then
    sbatch "$file"
  else
    # foreground: salloc takes the allocation and runs the same script on this host
    local -a alloc=(--nodes="$NNODES" --ntasks-per-node=1 --gpus-per-node="$GPUS" --exclusive --time="$TIME"
                    --job-name="$JOB_NAME")
    [[ -n "$PARTITION" ]] && alloc+=(--partition="$PARTITION")
    [[ -n "$NODELIST" ]] && alloc+=(--nodelist="$NODELIST")
    [[ -n "$RESERVATION" ]] && alloc+=(--reservation="$RESERVATION")
    [[ -n "$QOS" ]] && alloc+=(--qos="$QOS")
    [[ -n "$ACCOUNT" ]] && alloc+=(--account="$ACCOUNT")
    salloc "${alloc[@]}" bash "$file"
  fi
}

# The batch script: Slurm header, rendezvous and NCCL environment, then one
# srun task per node running node_cmd. Reads the caller's locals.
slurm_render() {
  echo "#!/usr/bin/env bash"
  echo "#SBATCH --job-name=$JOB_NAME"
  echo "#SBATCH --nodes=$NNODES"
  echo "#SBATCH --ntasks-per-node=1"
  echo "#SBATCH --gpus-per-node=$GPUS"
  echo "#SBATCH --exclusive"
  echo "#SBATCH --time=$TIME"
  echo "#SBATCH --output=$LOG_DIR/%x_%j.out"
  [[ -n "$PARTITION" ]] && echo "#SBATCH --partition=$PARTITION"
  [[ -n "$NODELIST" ]] && echo "#SBATCH --nodelist=$NODELIST"
  [[ -n "$DEPENDENCY" ]] && echo "#SBATCH --dependency=$DEPENDENCY"
  [[ -n "$RESERVATION" ]] && echo "#SBATCH --reservation=$RESERVATION"
  [[ -n "$QOS" ]] && echo "#SBATCH --qos=$QOS"
  [[ -n "$ACCOUNT" ]] && echo "#SBATCH --account=$ACCOUNT"
  echo "set -euo pipefail"
  echo "MASTER_HOST=\$(scontrol show hostnames \"\$SLURM_JOB_NODELIST\" | head -n 1)"
  if [[ -n "$NCCL_IF" ]]; then
    echo "MASTER_ADDR=\$(srun --nodes=1 --ntasks=1 --nodelist=\"\$MASTER_HOST\" ip -4 -o addr show dev $(printf '%q' "$NCCL_IF") | awk '{split(\$4, a, \"/\"); print a[1]; exit}')"
    echo "export NCCL_SOCKET_IFNAME=$(printf '%q' "$NCCL_IF") GLOO_SOCKET_IFNAME=$(printf '%q' "$NCCL_IF")"
  else
    echo "MASTER_ADDR=\$MASTER_HOST"
  fi
  echo "export MASTER_ADDR MASTER_PORT=$RDZV_PORT"
  echo "export NCCL_DEBUG=\${NCCL_DEBUG:-WARN} PYTHONUNBUFFERED=1 OMP_NUM_THREADS=\${OMP_NUM_THREADS:-8}"
  [[ -n "$IB_HCA" ]] && echo "export NCCL_IB_HCA=$(printf '%q' "$IB_HCA")"
  [[ -n "$HBM_CAP_GB" ]] && echo "export PRIMUS_TORCHREC_HBM_CAP_GB=$(printf '%q' "$HBM_CAP_GB")"
  [[ -n "$DDR_CAP_GB" ]] && echo "export PRIMUS_TORCHREC_DDR_CAP_GB=$(printf '%q' "$DDR_CAP_GB")"
  # the submitting shell's framework and NCCL switches travel with the job
  local v
  # (not CUDA_VISIBLE_DEVICES and the like: each node sees its own GPUs)
  for v in $(compgen -e | grep -E '^(PD_|NCCL_|TORCH_NCCL_)' | grep -vE '^(PD_DOCKER_IMAGE|NCCL_VERSION)$' || true); do
    echo "export $v=$(printf '%q' "${!v}")"
  done
  if [[ "$MODE" == docker ]]; then
    echo "export PD_FORWARD_ENV=\"\$(compgen -e | grep -E '^(PD_|NCCL_|TORCH_NCCL_|GLOO_|MASTER_|SLURM_|OMP_|PYTHON|PRIMUS_)' | tr '\n' ' ')\""
  fi
  echo "echo \"[launch] \$SLURM_NNODES nodes x $GPUS GPUs, master \$MASTER_ADDR:\$MASTER_PORT\""
  echo "srun --ntasks-per-node=1 --kill-on-bad-exit=1 bash -c $(printf '%q' "$node_cmd")"
}
