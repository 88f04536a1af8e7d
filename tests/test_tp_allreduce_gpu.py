"""Row-parallel projection + all-reduce over peer memory on 2..8 GPUs (skipped with fewer
than two).  Each rank is its own process on its own GPU (ranks that wait on one another
never share a GPU); NVLS is off in NCCL, whose all-reduce is only the reference here."""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_row_parallel_linear_peer_allreduce(ranks):
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr=127.0.0.1", f"--master-port={29600 + ranks}",
           str(ROOT / "tests" / "tp_allreduce_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(": OK") == ranks, r.stdout
