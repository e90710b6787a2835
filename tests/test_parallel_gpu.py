"""Ulysses sequence parallelism on real GPUs over NCCL (needs 2 or more GPUs; skipped on one).

Runs tests/sp_worker.py under torchrun on 2 GPUs: a 2-block engine whose tokens are sharded over the ranks must
produce exactly the single-GPU engine's output, bit for bit, over three forwards.  The exchanges run inside the
producing kernels over CUDA IPC peer memory (the qkv GEMM writes the receivers' layout, pushed in contiguous
blocks; the attention kernel stores each token's rows to its owner); attention runs per rank on its heads, dense
and under a block-sparse mask; activation scales are all-reduced.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mask", [False, True], ids=["dense", "block_sparse"])
def test_ulysses_engine_bitwise_equals_single_gpu(mask):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", SP_MASK="1" if mask else "0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), str(ROOT / "tests" / "sp_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    line = next(l for l in out.splitlines() if l.startswith("RESULT"))
    assert "bitwise=True" in line and "status=0" in line and f"mask={mask}" in line, line
