"""Shared helpers of the GPU parity tests (seeded inputs, numpy <-> torch)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import nvfp4 as ON


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def bf16_array(shape, seed, scale=1.0, outliers=True) -> np.ndarray:
    """N(0, scale) bf16 values with 1% of the last-dim channels x20 (BASELINE's activation distribution)."""

    rs = np.random.RandomState(seed)
    x = (rs.randn(*shape) * scale).astype(np.float32)
    if outliers and shape[-1] >= 100:
        ch = rs.permutation(shape[-1])[: shape[-1] // 100]
        x[..., ch] *= 20
    return ON.bf16_round(x)


def to_dev(a: np.ndarray, dtype=torch.bfloat16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().view(torch.uint8).cpu().numpy()


def device_ok():
    from tfvideo import native
    torch.cuda.synchronize()
    assert native.device_status(reset=True) == 0
