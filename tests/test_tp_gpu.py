"""Tensor-parallel decode (column-sharded linears, NCCL all-gathers): the
sharded engine on 2 and 4 GPUs must reproduce the single-GPU engine bit for
bit (whose one-row steps run as the persistent step kernel). Runs
tests/tp_worker.py as one rank per GPU; skipped with fewer GPUs."""
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


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_matches_single_gpu(tmp_path, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, BNN_TP_MODEL=str(tmp_path / "tp_model.gguf"), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(29513 + 10 * world),
           str(ROOT / "tests" / "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=360)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    assert f"TP OK {world}" in r.stdout
