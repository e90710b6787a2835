"""Attention backends for the full (non-causal) packed sequence: q, k, v [1, H, S, D] bf16 (strided views are fine,
last dim contiguous) -> [1, H, S, D].  Same registry as tfvideo/attention.py of the reference (:44-54).

fp8            libh3b200's tcgen05 FP8 flash attention (Q/K FP8 per row / per 128-key block with K smoothed, P and V
               FP8); the default.  Its output is a [1, H, S, D] view of token-major [S, H, D] memory, which is what
               the block's out-projection reads.
fp8_sparse(m)  the same kernel under a block-sparse mask ``m`` (a TileMask: per 128-token query tile, the 128-token KV
               tiles it attends to).  ``TileMask.block_sparse`` builds the seeded mask of BASELINE's sharded config
               (25% of tiles per query row, diagonal and text tiles always kept).
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


TILE = 128


class TileMask:
    """Block-sparse attention mask on 128 x 128 tiles, shared by all heads: query tile r (tokens 128 r .. 128 r + 127)
    attends to the KV tiles kv_idx[kv_ptr[r] : kv_ptr[r + 1]].  Held on the device as int32 CSR (the C ABI's form)."""

    def __init__(self, lists, S: int, device="cuda"):
        nt = (S + TILE - 1) // TILE
        if len(lists) != nt:
            raise ValueError(f"TileMask: {len(lists)} rows for {nt} query tiles")
        ptr, idx = [0], []
        for row in lists:
            row = sorted(set(int(c) for c in row))
            if row and (row[0] < 0 or row[-1] >= nt):
                raise ValueError(f"TileMask: KV tile out of range [0, {nt})")
            idx.extend(row)
            ptr.append(len(idx))
        self.S, self.tiles = S, nt
        self.lists = [sorted(set(int(c) for c in row)) for row in lists]
        self.kv_ptr = torch.tensor(ptr, dtype=torch.int32, device=device)
        self.kv_idx = torch.tensor(idx if idx else [0], dtype=torch.int32, device=device)
        self.kept = len(idx)

    @property
    def density(self) -> float:
        return self.kept / float(self.tiles * self.tiles)

    @classmethod
    def block_sparse(cls, S: int, keep: float = 0.25, text_tokens: int = 512, seed: int = 4, device="cuda"):
        """Seeded mask: every query tile keeps its diagonal tile and the text tiles (the first ``text_tokens``
        tokens), then further KV tiles drawn without replacement until ``keep`` of its row is kept."""

        nt = (S + TILE - 1) // TILE
        per_row = max(1, int(round(keep * nt)))
        text = list(range(min(nt, (text_tokens + TILE - 1) // TILE)))
        g = torch.Generator().manual_seed(seed)
        lists = []
        for r in range(nt):
            row = set(text) | {r}
            order = torch.randperm(nt, generator=g).tolist()
            for c in order:
                if len(row) >= per_row:
                    break
                row.add(c)
            lists.append(sorted(row))
        return cls(lists, S, device)


def fp8_tokens(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, S: int, H: int, ld: int, hstride: int,
               out: torch.Tensor, workspace: torch.Tensor | None = None, mask: TileMask | None = None) -> torch.Tensor:
    """Low-level form: element (t, h, d) of q / k / v at base + t * ld + h * hstride + d; out [S, H * 128] bf16.
    ``mask`` (a TileMask for this S) selects the block-sparse kernel."""

    ws = aligned_workspace(_workspace(S, H, q.device) if workspace is None else workspace)
    if mask is None:
        N.attn_fp8(q, k, v, ld, hstride, S, H, out, out.stride(0), ws)
    else:
        if mask.S != S:
            raise ValueError(f"TileMask built for S={mask.S}, attention has S={S}")
        N.attn_fp8_sparse(q, k, v, ld, hstride, S, H, mask.kv_ptr, mask.kv_idx, out, out.stride(0), ws)
    return out


def fp8(q, k, v, mask: TileMask | None = None):
    _, H, S, D = q.shape
    if D != HEAD_DIM or not (q.stride(3) == k.stride(3) == v.stride(3) == 1):
        raise ValueError("fp8 attention: head_dim 128 with a contiguous last dim")
    if not (q.stride(1) == k.stride(1) == v.stride(1) and q.stride(2) == k.stride(2) == v.stride(2)):
        q, k, v = (t.contiguous() for t in (q, k, v))
    out = torch.empty((S, H * D), dtype=torch.bfloat16, device=q.device)
    fp8_tokens(q, k, v, S, H, q.stride(2), q.stride(1), out, mask=mask)
    return out.view(1, S, H, D).transpose(1, 2)


def fp8_sparse(mask: TileMask):
    """A backend function (q, k, v) -> o running the FP8 kernel under ``mask``."""

    def run(q, k, v):
        return fp8(q, k, v, mask)

    return run


BACKENDS = {"sdpa": sdpa_flash, "cudnn": sdpa_cudnn, "fp8": fp8}
BENCH: dict = {}
DEFAULT = "fp8"


def get(name: str):
    if name == "auto":
        name = DEFAULT
    if name not in BACKENDS:
        raise ValueError(f"attention backend {name!r}: one of {', '.join(['auto', *BACKENDS])}")
    return BACKENDS[name]
