"""Expert parallelism across the GPUs of one machine: tests/ep_check.py under torchrun, one rank per GPU (skipped with fewer
than two GPUs visible)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_expert_parallel_parity_across_gpus():
    import torch
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("fewer than two GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533", os.path.join(ROOT, "tests", "ep_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env={**os.environ, "NCCL_NVLS_ENABLE": "0"})
    print(r.stdout[-2000:])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "parity over" in r.stdout and "ok" in r.stdout
