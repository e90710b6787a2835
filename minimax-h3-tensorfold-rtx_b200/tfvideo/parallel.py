"""Ulysses head-parallel sequence parallelism over torch.distributed (NCCL over NVLink on B200s; gloo on CPU tests).

Each rank holds a contiguous shard of S / P tokens for everything but attention: norms, the four GEMMs, RoPE and the
gated residuals are token-local.  Around attention, one all-to-all per tensor turns q, k, v [S/P, H, Dh] into
[S, H/P, Dh] (every token, this rank's heads), and one more brings the output [S, H/P * Dh] back to
[S/P, H * Dh] -- received as P column blocks [P, S/P, H/P * Dh], which the out-projection's quantiser reads in place.
The reference runs on one GPU and has no collective; this is the B200 build's multi-GPU layer.

On GPUs the engine does both exchanges inside the kernels that produce the data: the qkv GEMM's epilogue and the
attention kernel's epilogue store each head's columns / each token's row straight into the owning rank's receive
buffer (a PeerBuffer: device memory every rank maps through CUDA IPC), and a barrier after the kernel stands in for
the all-to-all.  The all-to-all methods below remain for library attention backends and CPU (gloo) runs.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import native as N


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

    def barrier(self, device) -> None:
        """In stream order: returns (on the device) once every rank's work before it has finished, so the peer stores
        that work made are visible to what follows (a one-element all-reduce).  The element carries each rank's device
        status word (max over ranks, sticky): a rank whose kernel gave up a bounded wait -- leaving some receive rows
        unwritten -- makes ``failed()`` nonzero on every rank, with no host read at the barrier itself."""

        if getattr(self, "_flag", None) is None or self._flag.device != torch.device(device):
            self._flag = torch.zeros(1, dtype=torch.float32, device=device)
        if self._flag.is_cuda:
            N.status_publish(self._flag)
        dist.all_reduce(self._flag, op=dist.ReduceOp.MAX, group=self.group)

    def failed(self) -> int:
        """The largest device status any rank published at a barrier so far (0 = none failed); one host read."""

        flag = getattr(self, "_flag", None)
        return 0 if flag is None else int(flag.item())


class QkvExchange:
    """Addresses of the fused qkv exchange of one rank (pure arithmetic, no device work).

    The qkv GEMM's STORE_PEERS epilogue stores column (part, head, d) of its local row ``row`` to
    ``base[owner] + ((rank * M + row) * 3 + part) * Hr * 128 + (head % Hr) * 128 + d`` (bf16 elements; M the launch's
    rows, Hr = H / world).  This rank's own heads go straight into its receive buffer; every other rank's go into that
    rank's contiguous block of a local staging buffer, [world, n, 3 Hr Dh], later copied to that rank's receive
    buffer at row rank * n.  ``recv``: every rank's receive buffer as mapped here; ``send``: the staging buffer."""

    def __init__(self, rank: int, world: int, n: int, row_elems: int, elem_bytes: int, recv: list[int], send: int):
        self.rank, self.world, self.n = rank, world, n
        self.row = row_elems * elem_bytes   # bytes of one token's row in a receive buffer (3 Hr Dh elements)
        self.recv, self.send = recv, send

    def row_parts(self, tile: int = 128, parts: int = 2) -> list[tuple[int, int]]:
        """The qkv GEMM's row parts: up to ``parts`` contiguous ranges of near-equal length, split at multiples of
        ``tile`` rows (the last part takes the ragged end; one part when n is below two tiles).  Every part but the
        last goes to the other ranks by the copy engines while the GEMM computes the next part."""

        tiles = self.n // tile
        k = max(1, min(parts, tiles))
        cuts = [(tiles * j // k) * tile for j in range(k)] + [self.n]
        return [(a, b) for a, b in zip(cuts, cuts[1:]) if b > a]

    def bases(self, m0: int, M: int) -> list[int]:
        """The epilogue's base for each rank, for a launch over local rows [m0, m0 + M) (the kernel adds
        (rank * M + row) rows; the bases carry the rest of each destination's offset)."""

        rank, n = self.rank, self.n
        shift = (rank * n + m0 - rank * M) * self.row
        return [(self.recv[rank] if r == rank else self.send + (r - rank) * n * self.row) + shift
                for r in range(self.world)]

    def copies(self, r0: int, r1: int) -> list[tuple[int, int, int]]:
        """(src, dst, bytes): rows [r0, r1) of every other rank's staged block into that rank's receive buffer."""

        rank, n = self.rank, self.n
        return [(self.send + (r * n + r0) * self.row, self.recv[r] + (rank * n + r0) * self.row, (r1 - r0) * self.row)
                for r in range(self.world) if r != rank]


class PeerBuffer:
    """A device buffer this rank owns and every rank of the group stores into: a plain allocation shared through
    CUDA IPC (no multicast object), mapped by each rank once.  ``ptrs[r]`` is rank r's buffer as mapped here;
    ``tensor`` views this rank's own.  The mappings last until the process exits."""

    def __init__(self, sp: SequenceParallel, shape: tuple[int, ...], dtype: torch.dtype, device):
        nbytes = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
        local, handle = N.peer_alloc(nbytes)
        handles = [None] * sp.world
        dist.all_gather_object(handles, handle, group=sp.group)
        self.ptrs = [local if r == sp.rank else N.peer_open(handles[r]) for r in range(sp.world)]
        self.tensor = N.tensor_at(local, shape, dtype, device)


def unshard_columns(recv: torch.Tensor) -> torch.Tensor:
    """[P, n, C] column blocks -> [n, P * C] rows (a copy; the GEMM path reads the blocks in place instead)."""

    P, n, C = recv.shape
    return recv.permute(1, 0, 2).reshape(n, P * C)
