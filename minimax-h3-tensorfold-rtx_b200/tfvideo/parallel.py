"""Ulysses head-parallel sequence parallelism over torch.distributed (NCCL over NVLink on B200s; gloo on CPU tests).

Each rank holds a contiguous shard of S / P tokens for everything but attention: norms, the four GEMMs, RoPE and the
gated residuals are token-local.  Around attention, one all-to-all per tensor turns q, k, v [S/P, H, Dh] into
[S, H/P, Dh] (every token, this rank's heads), and one more brings the output [S, H/P * Dh] back to
[S/P, H * Dh] -- received as P column blocks [P, S/P, H/P * Dh], which the out-projection's quantiser reads in place.
The reference runs on one GPU and has no collective; this is the B200 build's multi-GPU layer.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class SequenceParallel:
    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def shard(self, S: int) -> tuple[int, int]:
        """(first token, token count) of this rank's shard of an S-token sequence (S % world == 0)."""

        if S % self.world:
            raise ValueError(f"sequence length {S} does not split evenly over {self.world} ranks")
        n = S // self.world
        return self.rank * n, n

    def heads_from_tokens(self, t: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """t [S/P, H, Dh] (any row stride) -> out [S, H/P, Dh]: all tokens of this rank's heads."""

        P = self.world
        n, H, Dh = t.shape
        if H % P:
            raise ValueError(f"{H} heads do not split over {P} ranks")
        send = t.reshape(n, P, H // P, Dh).permute(1, 0, 2, 3).contiguous()
        dist.all_to_all_single(out.view(P, n, H // P, Dh), send, group=self.group)
        return out

    def qkv_heads_from_tokens(self, qkv: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """qkv [S/P, 3, H, Dh] (the qkv GEMM's rows) -> out [S, 3, H/P, Dh]: q, k and v of this rank's heads for every
        token, in one all-to-all.  The result has the qkv buffer's own row layout, so attention reads q / k / v from
        it with row stride 3 (H/P) Dh, as it reads the single-GPU qkv buffer."""

        P = self.world
        n, three, H, Dh = qkv.shape
        if H % P:
            raise ValueError(f"{H} heads do not split over {P} ranks")
        send = qkv.reshape(n, 3, P, H // P, Dh).permute(2, 0, 1, 3, 4).contiguous()
        dist.all_to_all_single(out.view(P, n, 3, H // P, Dh), send, group=self.group)
        return out

    def tokens_from_heads(self, o: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """o [S, H/P * Dh] -> out [P, S/P, H/P * Dh]: this rank's tokens, column block r from rank r's heads."""

        P = self.world
        dist.all_to_all_single(out, o.view(P, o.shape[0] // P, o.shape[1]), group=self.group)
        return out

    def max_(self, t: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t


def unshard_columns(recv: torch.Tensor) -> torch.Tensor:
    """[P, n, C] column blocks -> [n, P * C] rows (a copy; the GEMM path reads the blocks in place instead)."""

    P, n, C = recv.shape
    return recv.permute(1, 0, 2).reshape(n, P * C)
