"""The NVFP4 quantisers compute scale = e4m3(amax / 6) and its reciprocal without IEEE divisions
(csrc/common.cuh div6_rn, e4m3_rcp).  tests/cuda/quant_exact_check.cu compares both with CUDA's correctly rounded
division over every non-negative finite fp32 and every scale byte; this test builds and runs it on the GPU."""

from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_division_free_scale_helpers_match_ieee_division(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "quant_exact_check"
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    f"-I{ROOT / 'minimax-h3-tensorfold-rtx_b200' / 'csrc'}", f"-I{ROOT / 'include'}",
                    "--expt-relaxed-constexpr", "-o", str(exe), str(ROOT / "tests" / "cuda" / "quant_exact_check.cu")],
                   check=True, capture_output=True, text=True, timeout=300)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    got = {k: int(v) for k, v in re.findall(r"(mismatch_[\w^-]+)=(\d+)", r.stdout)}
    # x / 6 may differ from the IEEE quotient only below 2^-10, where the e4m3 scale rounds to the same byte
    assert got["mismatch_ge_2^-10"] == 0 and got["mismatch_e4m3"] == 0, r.stdout
    assert got["mismatch_rcp"] == 0, r.stdout
