"""The column-sharded GEMM on 2 GPUs (torchrun, one rank per GPU): the all-gather
fused into the GEMM epilogue (P2P stores over NVLink) and the NCCL variant, each
rank's gathered C checked against the oracle.  Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_sharded_gemm_two_ranks():
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(here, "mp_sharded_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "failures=0" in res.stdout
