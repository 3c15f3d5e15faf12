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


def test_nvlink_allreduce_wait_gives_up_and_reports(cuda_device):
    """Failure detection on one GPU, without a fault: a sum over two ranks
    whose second rank never raises its flag (its buffer is a second local
    allocation nothing writes) waits its bounded 5 s, sets status bit 0,
    leaves `inout` untouched and returns; the context stays usable."""
    import ctypes

    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    n = 256
    size = int(lib.pyrite_cuda_allreduce_buffer_size(n))
    bufs, handle = [], (ctypes.c_ubyte * 64)()
    for _ in range(2):
        p = ctypes.c_void_p()
        assert lib.pyrite_cuda_ipc_buffer_create(size, ctypes.byref(p), handle) == 0
        bufs.append(p.value)
    peers = torch.tensor(bufs, dtype=torch.int64, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    part = torch.ones(n, device="cuda")
    out = torch.full((n,), 3.0, device="cuda")
    K.status()  # start clean
    assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), n, peers.data_ptr(), size, 2, 0, epoch.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert K.status() & 1  # the wait gave up (and the bit is cleared again)
    assert bool((out == 3.0).all())
    assert int(epoch.item()) == 1
    # the context still runs work
    assert float((part * 2).sum().item()) == 2 * n
    for p in bufs:
        assert lib.pyrite_cuda_ipc_buffer_close(p, 1) == 0
    # argument checks: n not a multiple of 4, rank outside the world
    s = torch.cuda.current_stream().cuda_stream
    assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), 6, peers.data_ptr(), size, 2, 0, epoch.data_ptr(),
                                         s) == -3
    assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), n, peers.data_ptr(), size, 2, 2, epoch.data_ptr(),
                                         s) == -3
    # n beyond what the buffers were created for
    assert lib.pyrite_cuda_allreduce_sum(part.data_ptr(), out.data_ptr(), 2 * n, peers.data_ptr(), size, 2, 0,
                                         epoch.data_ptr(), s) == -3
