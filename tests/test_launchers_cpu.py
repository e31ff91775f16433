"""The Slurm launchers (scripts/launch_slurm.sh, scripts/launch_slurm_docker.sh)
render a batch script that is valid bash and starts one torchrun per node
with the requested ranks, rendezvous and run_distributed.py flags. Checked
with --dry-run (nothing is submitted)."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CFG = "configs/bench_onetrans_v6_b200.yaml"

pytestmark = pytest.mark.skipif(shutil.which("bash") is None, reason="needs bash")


def _render(script, *args, env=None):
    e = {k: v for k, v in os.environ.items() if not k.startswith(("PD_", "NCCL_"))}
    e.update(env or {})
    r = subprocess.run(["bash", str(ROOT / "scripts" / script), "--config", CFG, "--dry-run", *args],
                       capture_output=True, text=True, env=e, cwd=ROOT)
    return r


@pytest.mark.parametrize("script", ["launch_slurm.sh", "launch_slurm_docker.sh"])
def test_dry_run_renders_valid_batch_script(script, tmp_path):
    r = _render(script, "--nnodes", "2", "--gpus", "4", "--partition", "b200", "--nccl-if", "ib0",
                "--max-steps", "50", "--skip-eval", "--trace", "--trace-ranks", "all", "--", "--comm", "nccl",
                env={"PD_ATTN_TC_FWD": "1", "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr
    text = r.stdout
    f = tmp_path / "job.sh"
    f.write_text(text)
    assert subprocess.run(["bash", "-n", str(f)]).returncode == 0
    for line in ["#SBATCH --nodes=2", "#SBATCH --gpus-per-node=4", "#SBATCH --ntasks-per-node=1",
                 "#SBATCH --partition=b200", "export NCCL_SOCKET_IFNAME=ib0", "export PD_ATTN_TC_FWD=1"]:
        assert line in text, line
    assert "CUDA_VISIBLE_DEVICES" not in text            # each node keeps its own GPUs
    srun = [ln for ln in text.splitlines() if ln.startswith("srun --ntasks-per-node=1")]
    assert len(srun) == 1
    # the node command, as the node's bash will see it
    node_cmd = subprocess.run(["bash", "-c", srun[0].replace("srun --ntasks-per-node=1 --kill-on-bad-exit=1 bash -c ",
                                                             "printf '%s' ", 1)],
                              capture_output=True, text=True).stdout
    for part in ["--nproc-per-node=4", "--nnodes=$SLURM_NNODES", "--node-rank=$SLURM_NODEID",
                 "--master-addr=$MASTER_ADDR", "scripts/run_distributed.py", "--max-steps 50", "--skip-eval",
                 "--trace-ranks all", "--comm nccl", "--dense-strategy ddp"]:
        assert part in node_cmd, part
    if script == "launch_slurm_docker.sh":
        assert "docker run" in node_cmd and "--gpus all" in node_cmd and "--ipc host" in node_cmd


@pytest.mark.parametrize("args,msg", [(["--config", "missing.yaml"], "config not found"),
                                      (["--nnodes", "0"], "positive integers"),
                                      (["--dense-strategy", "zero"], "ddp, fsdp, zero2 or dmp"),
                                      (["--bogus"], "unknown flag")])
def test_bad_arguments_exit_2(args, msg):
    r = _render("launch_slurm.sh", *args)
    assert r.returncode == 2 and msg in r.stderr
