"""Tile-sharded training step on 2 GPUs (NCCL) vs the single-GPU step.

Runs tests/multigpu_check.py under torchrun with two processes; skipped when
fewer than two GPUs are visible (the CPU gloo test covers the exchange logic).
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("exchange", ["nccl", "peers", "rgb", "route", "route-peer"])
def test_two_gpu_sharded_step_matches_single_gpu(exchange):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MSPLAT_EXCHANGE=exchange)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29555",
           os.path.join(HERE, "multigpu_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=360)
    assert r.returncode == 0 and "MULTIGPU OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
