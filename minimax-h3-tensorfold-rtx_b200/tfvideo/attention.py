"""Attention backends for the full (non-causal) packed sequence: q, k, v [1, H, S, D] bf16 (strided views are fine,
last dim contiguous) -> [1, H, S, D].  Same registry as tfvideo/attention.py of the reference (:44-54).

fp8            libh3b200's tcgen05 FP8 flash attention (Q/K FP8 per row / per 128-key block with K smoothed, P and V
               FP8); the default.  Its output is a [1, H, S, D] view of token-major [S, H, D] memory, which is what
               the block's out-projection reads.
sdpa / cudnn   PyTorch's bf16 backends, kept as the reference's comparison points (not the fast path).
The reference's ``int8`` (comfy-kitchen) and ``fp4`` (Triton, sm_120) backends have no B200 build; asking for them
raises ValueError, like any unknown name.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import native as N

HEAD_DIM = 128


def sdpa_flash(q, k, v):
    with sdpa_kernel([SDPBackend.FLASH_ATTENTION, SDPBackend.CUDNN_ATTENTION, SDPBackend.EFFICIENT_ATTENTION],
                     set_priority=True):
        return F.scaled_dot_product_attention(q, k, v)


def sdpa_cudnn(q, k, v):
    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION],
                     set_priority=True):
        return F.scaled_dot_product_attention(q, k, v)


def _workspace(S: int, H: int, device) -> torch.Tensor:
    n = N.attn_workspace_bytes(S, H)
    return torch.empty(n + 1024, dtype=torch.uint8, device=device)


def aligned_workspace(buf: torch.Tensor) -> torch.Tensor:
    off = (-buf.data_ptr()) % 1024
    return buf[off:]


def fp8_tokens(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, S: int, H: int, ld: int, hstride: int,
               out: torch.Tensor, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Low-level form: element (t, h, d) of q / k / v at base + t * ld + h * hstride + d; out [S, H * 128] bf16."""

    ws = aligned_workspace(_workspace(S, H, q.device) if workspace is None else workspace)
    N.attn_fp8(q, k, v, ld, hstride, S, H, out, out.stride(0), ws)
    return out


def fp8(q, k, v):
    _, H, S, D = q.shape
    if D != HEAD_DIM or not (q.stride(3) == k.stride(3) == v.stride(3) == 1):
        raise ValueError("fp8 attention: head_dim 128 with a contiguous last dim")
    if not (q.stride(1) == k.stride(1) == v.stride(1) and q.stride(2) == k.stride(2) == v.stride(2)):
        q, k, v = (t.contiguous() for t in (q, k, v))
    out = torch.empty((S, H * D), dtype=torch.bfloat16, device=q.device)
    fp8_tokens(q, k, v, S, H, q.stride(2), q.stride(1), out)
    return out.view(1, S, H, D).transpose(1, 2)


BACKENDS = {"sdpa": sdpa_flash, "cudnn": sdpa_cudnn, "fp8": fp8}
BENCH: dict = {}
DEFAULT = "fp8"


def get(name: str):
    if name == "auto":
        name = DEFAULT
    if name not in BACKENDS:
        raise ValueError(f"attention backend {name!r}: one of {', '.join(['auto', *BACKENDS])}")
    return BACKENDS[name]
