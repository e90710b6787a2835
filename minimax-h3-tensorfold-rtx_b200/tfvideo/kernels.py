"""Fused elementwise kernels of a MiniMax H3 block on B200 (libh3b200): each reads its input once, writes once.

Same interface as tfvideo/kernels.py of the reference (:31, :56, :76): ``idx`` (int32 [S]) is each row's
modulation row and ``mod`` (fp32 [R, 6, D]) holds shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp.
fp32 inside, bf16 out.  ``gelu_tanh`` is the FFN activation of BASELINE's H3-shaped configs.
"""

from __future__ import annotations

import torch

from . import native as N


def _check_rows(x: torch.Tensor, name: str) -> None:
    if x.dim() != 2 or x.dtype != torch.bfloat16 or x.stride(1) != 1:
        raise ValueError(f"{name}: expected a row-major bf16 [S, D] tensor, got {tuple(x.shape)} {x.dtype}")


def norm_mod(x: torch.Tensor, w: torch.Tensor, mod: torch.Tensor, part: int, idx: torch.Tensor, eps: float,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm(x) * w * (1 + scale) + shift for x [S, D] bf16; ``part`` 0 = attention (chunks 0, 1), 1 = MLP (3, 4)."""

    _check_rows(x, "norm_mod")
    out = torch.empty_like(x) if out is None else out
    N.norm_mod(x, w.float().contiguous(), mod.float().contiguous(), idx.to(torch.int32).contiguous(), part, eps,
               out=out)
    return out


def gate_add(x: torch.Tensor, y: torch.Tensor, mod: torch.Tensor, part: int, idx: torch.Tensor) -> torch.Tensor:
    """x += y * gate in place (x, y [S, D] bf16); ``part`` 0 = gate_msa (chunk 2), 1 = gate_mlp (chunk 5)."""

    _check_rows(x, "gate_add")
    _check_rows(y, "gate_add")
    N.gate_add(x, y, mod.float().contiguous(), idx.to(torch.int32).contiguous(), part)
    return x


def swiglu(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[M, 2F] = [gate | up] bf16 -> silu(gate) * up, [M, F] bf16."""

    _check_rows(gu, "swiglu")
    M, F2 = gu.shape
    out = torch.empty((M, F2 // 2), dtype=torch.bfloat16, device=gu.device) if out is None else out
    N.act(gu, out, N.ACT_SWIGLU)
    return out


def gelu_tanh(u: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[M, F] bf16 -> gelu(u, approximate="tanh"), [M, F] bf16."""

    _check_rows(u, "gelu_tanh")
    out = torch.empty_like(u) if out is None else out
    N.act(u, out, N.ACT_GELU)
    return out
