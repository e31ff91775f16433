"""A failing argument check in the native extensions raises RuntimeError with
its message. (Messages assembled from several parts crashed the process with
SIGSEGV in the nvcc-compiled sources; they are now formatted into one string,
PD_CHECK in csrc/common.cuh.) Each case runs in a child process, so a crash
fails the test instead of ending the run. CPU only: the checks fire before any
device work."""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

CASES = {
    "too_many_tables": """
import torch, primus_dlrm_b200._C as C
n = 40
w = [torch.zeros(4, 128) for _ in range(n)]
p = [torch.zeros(1, dtype=torch.int64) for _ in range(n)]
C.emb_keys([torch.zeros(4, dtype=torch.int64)], [torch.zeros(4, 128)], torch.zeros(1, 4, dtype=torch.int64),
           [torch.zeros(0, dtype=torch.int64)], w, p, torch.zeros(n, 6, dtype=torch.int64), 128)
""",
    "gemm_operand": """
import torch, primus_dlrm_b200._gemm as G
G.tc_gemm(torch.zeros(1, 4, 8), torch.zeros(1, 64, 8), torch.zeros(1, 4, 64), err=torch.zeros(1, dtype=torch.int32))
""",
    "attention_operand": """
import torch, primus_dlrm_b200._gemm as G
G.fmha_fwd(torch.zeros(1, 4, 2, 32), torch.zeros(1, 4, 2, 32), torch.zeros(1, 4, 2, 32), 0.1)
""",
}


def _built(name: str) -> bool:
    return any((ROOT / "primus_dlrm_b200").glob(f"{name}.*.so"))


@pytest.mark.parametrize("case", sorted(CASES))
def test_failing_check_raises(case):
    if not (_built("_C") and _built("_gemm")):
        pytest.skip("extensions not built")
    code = "import sys\nsys.path.insert(0, %r)\ntry:\n" % str(ROOT)
    code += "".join("    " + line + "\n" for line in CASES[case].strip().splitlines())
    code += "except RuntimeError as e:\n    print('RAISED', str(e)[:200])\n"
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"child died (rc {r.returncode}): {r.stderr[-500:]}"
    assert "RAISED" in r.stdout, r.stdout + r.stderr[-500:]
