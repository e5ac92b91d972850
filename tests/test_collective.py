"""The NVLS gradient all-reduce and the fused exchange-and-Adam step on two GPUs (one process
each) against NCCL's all-reduce (and the single-GPU Adam after it): with two ranks each
element's sum is one fp32 addition, so the sums agree exactly; the updated parameters agree to a
few ulp (the Adam arithmetic may contract into FMAs differently in the two kernels)."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.gpu
def test_nvls_allreduce_matches_nccl_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_DEBUG="WARN")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29581",
           str(ROOT / "tests" / "_nvls_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=env)
    out = res.stdout + res.stderr
    if "unavailable" in out:
        pytest.skip("no NVLink multicast on this fabric")
    assert res.returncode == 0, out[-3000:]
    for r in range(2):  # each rank reports on a line of its own
        assert f"rank {r} mismatches 0" in out, out[-3000:]


@pytest.mark.gpu
def test_nvls_adam_matches_allreduce_then_adam_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_DEBUG="WARN")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29582",
           str(ROOT / "tests" / "_nvls_adam_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=env)
    out = res.stdout + res.stderr
    if "unavailable" in out:
        pytest.skip("no NVLink multicast on this fabric")
    assert res.returncode == 0, out[-3000:]
    for r in range(2):  # each rank reports on a line of its own
        assert f"rank {r} mismatches 0" in out, out[-3000:]
