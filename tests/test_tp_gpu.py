"""Tensor-parallel decode (column-sharded linears, NCCL all-gathers): the
sharded engine on 2 GPUs must reproduce the single-GPU engine bit for bit.
Runs tests/tp_worker.py as two ranks; skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_matches_single_gpu(tmp_path):
    env = dict(os.environ, BNN_TP_MODEL=str(tmp_path / "tp_model.gguf"), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29513",
           str(ROOT / "tests" / "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    assert "TP OK 2" in r.stdout
