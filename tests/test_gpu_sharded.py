"""Tensor-parallel decode on 2 GPUs (B200, NVLink): greedy ids (and routed
experts) equal the reference executor's on the golden checkpoints, and the
one-shot NVLink sum (pyrite_cuda_allreduce_sum) equals NCCL's allreduce.
Needs at least two GPUs; runs tests/sharded_worker.py under torchrun."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("golden", ["llama_tiny.json", "moe_tiny.json", "c1_small.json"])
def test_two_gpu_sharded_decode_matches_reference(cuda_device, golden):
    if _gpus() < 2:
        pytest.skip("tensor-parallel decode needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", str(ROOT / "tests" / "sharded_worker.py"),
           str(ROOT / "tests" / "golden" / golden)]
    res = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    out = json.loads(lines[-1])
    assert out["ids_match"] and out["routed_match"] in (None, True), out


def test_two_gpu_nvlink_allreduce_equals_nccl(cuda_device):
    if _gpus() < 2:
        pytest.skip("the allreduce needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29534", str(ROOT / "tests" / "sharded_worker.py"), "allreduce"]
    res = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env, cwd=ROOT)
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    out = json.loads(lines[-1])
    assert out["allreduce_ok"], out
