"""Seeded synthetic inputs with BASELINE.json's shapes and value distributions, made on the device.

BASELINE's configs name no dataset: activations are N(0, 1) bf16 with 1% of the channels scaled x 20 (outliers),
weights N(0, 0.02), and attention inputs are q / k / v after QK-RMSNorm (unit RMS per head row).  The benchmark and
the full-shape parity tests draw their inputs here, so that both see the same distributions; everything is generated
on the GPU from a seed (tens of GB of host randn would dominate a run otherwise).
"""

from __future__ import annotations

import torch


def dev_activations(M: int, K: int, seed: int) -> torch.Tensor:
    """bf16 [M, K]: N(0, 1) with K // 100 channels (a seeded draw) multiplied by 20."""

    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=g, device="cuda")
    ch = torch.randperm(K, generator=torch.Generator().manual_seed(seed + 1))[: K // 100].cuda()
    x[:, ch] *= 20
    return x.to(torch.bfloat16)


def dev_weight(N: int, K: int, seed: int) -> torch.Tensor:
    """bf16 [N, K] ~ N(0, 0.02)."""

    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)


def dev_qkv(S: int, H: int, seed: int, head_dim: int = 128) -> torch.Tensor:
    """bf16 [S, 3, H, head_dim]: q, k, v rows of unit RMS (QK-RMSNorm's output with unit weights); k carries a seeded
    per-(head, channel) offset, the kind of channel bias the FP8 recipe's K-mean smoothing removes."""

    g = torch.Generator(device="cuda").manual_seed(seed)
    t = torch.randn(S, 3, H, head_dim, generator=g, device="cuda")
    t = t / t.pow(2).mean(-1, keepdim=True).sqrt()
    t[:, 1] += torch.randn(H, head_dim, generator=g, device="cuda")
    return t.to(torch.bfloat16)
