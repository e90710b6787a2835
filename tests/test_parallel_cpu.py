"""Ulysses sequence parallelism (tfvideo/parallel.py) on CPU ranks over gloo, world size 2 and 4.

The same SequenceParallel code the engine runs over NCCL: tokens sharded over ranks, one all-to-all per q / k / v to
head-parallel layout, attention per rank on its heads over the full sequence, one all-to-all back.  Checked against
the unsharded computation; plus the failure paths: a rank that never joins ends the others' collective with an
error, within the process group's timeout.
"""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout=30):
    sys.path.insert(0, str(ROOT / "minimax-h3-tensorfold-rtx_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout))


def _ulysses_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from tfvideo.parallel import SequenceParallel, unshard_columns

        sp = SequenceParallel()
        S, H, Dh = 48, 8, 16
        g = torch.Generator().manual_seed(0)
        qkv = torch.randn(S, 3, H, Dh, generator=g)
        t0, n = sp.shard(S)
        local = qkv[t0:t0 + n]
        outs = []
        for j in range(3):
            buf = torch.empty(S, H // world, Dh)
            sp.heads_from_tokens(local[:, j], buf)
            ref = qkv[:, j, rank * (H // world):(rank + 1) * (H // world)]
            assert torch.equal(buf, ref), f"rank {rank}: head gather mismatch for tensor {j}"
            outs.append(buf)
        # the engine's form: q, k and v in one all-to-all, received in the qkv buffer's row layout
        both = torch.empty(S, 3, H // world, Dh)
        sp.qkv_heads_from_tokens(local.contiguous(), both)
        for j in range(3):
            assert torch.equal(both[:, j], outs[j]), f"rank {rank}: fused q/k/v exchange differs for tensor {j}"
        # attention on this rank's heads over the full sequence, then back to token-sharded rows
        qh, kh, vh = (t.transpose(0, 1) for t in outs)
        o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh).transpose(0, 1).reshape(S, -1)
        recv = torch.empty(world, n, (H // world) * Dh)
        sp.tokens_from_heads(o.contiguous(), recv)
        got = unshard_columns(recv)
        full = torch.nn.functional.scaled_dot_product_attention(*(qkv[:, j].transpose(0, 1) for j in range(3)))
        want = full.transpose(0, 1).reshape(S, H * Dh)[t0:t0 + n]
        assert torch.allclose(got, want, atol=1e-5), f"rank {rank}: attention through Ulysses differs"
        m = torch.tensor([float(rank + 1)])
        sp.max_(m)
        assert m.item() == world
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_ulysses_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
    assert all(v == "ok" for v in res.values()), res


def _straggler_worker(rank, world, port, q):
    """Rank 1 joins the group but never enters the all-to-all: rank 0's collective must fail, not hang."""

    try:
        _init(rank, world, port, timeout=5)
        from tfvideo.parallel import SequenceParallel

        sp = SequenceParallel()
        if rank == 1:
            q.put((rank, "skipped"))
            import time
            time.sleep(15)
            return
        buf = torch.empty(8, 2, 4)
        try:
            sp.heads_from_tokens(torch.randn(4, 4, 4), buf)
            q.put((rank, "no error"))
        except Exception as e:  # noqa: BLE001
            q.put((rank, f"error: {type(e).__name__}"))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


def test_missing_rank_fails_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_straggler_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert res[1] == "skipped"
    assert res[0].startswith("error"), res



def _peer_buffer_worker(rank, world, port, q):
    """PeerBuffer's rendezvous on gloo ranks, the CUDA IPC calls replaced by fakes that tag pointers and handles
    with the owning rank: every rank must end up with its own allocation and every other rank's opened handle."""

    try:
        _init(rank, world, port)
        from tfvideo import native as N
        from tfvideo import parallel as P

        opened = []
        N.peer_alloc = lambda nbytes: (0x1000 * (rank + 1), bytes([rank]) * N.IPC_HANDLE_BYTES)
        N.peer_open = lambda h: opened.append(h[0]) or 0x9000 + h[0]
        N.tensor_at = lambda p, shape, dtype, device: torch.empty(shape, dtype=dtype)
        sp = P.SequenceParallel()
        pb = P.PeerBuffer(sp, (4, 3, 2, 8), torch.bfloat16, "cpu")
        want = [0x1000 * (rank + 1) if r == rank else 0x9000 + r for r in range(world)]
        assert pb.ptrs == want, (pb.ptrs, want)
        assert sorted(opened) == [r for r in range(world) if r != rank]
        assert tuple(pb.tensor.shape) == (4, 3, 2, 8) and pb.tensor.dtype == torch.bfloat16
        sp.barrier("cpu")   # the barrier is a collective every rank passes
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_peer_buffer_rendezvous(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_peer_buffer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert all(v == "ok" for v in res.values()), res


def test_shard_requires_even_split():
    from tfvideo.parallel import SequenceParallel

    sp = SequenceParallel.__new__(SequenceParallel)
    sp.world, sp.rank, sp.group = 8, 3, None
    assert sp.shard(37760) == (3 * 4720, 4720)
    with pytest.raises(ValueError):
        sp.shard(37790)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("tile,nparts", [(128, 2), (2, 2), (1, 4)])   # one launch at this n; two and four row parts
def test_peer_store_layout_matches_all_to_all(world, tile, nparts):
    """The fused qkv exchange's addresses (tfvideo.parallel.QkvExchange, as the engine uses them) with the qkv
    GEMM's STORE_PEERS epilogue restated element by element (csrc/gemm_nvfp4.cuh: column (part, head, d) of launch
    row `row` goes to base[owner] + ((rank * M + row) * 3 + part) * Hr * 128 + (head % Hr) * 128 + d), then the
    block copies, on a simulated byte-addressed memory: every rank's receive buffer must end up in the all-to-all's
    [S, 3, H/P, Dh] layout."""

    sys.path.insert(0, str(ROOT / "minimax-h3-tensorfold-rtx_b200"))
    from tfvideo.parallel import QkvExchange

    n, H, Dh, es = 5, 2 * world, 128, 4          # fp32 elements stand in for bf16 (only the addresses matter)
    Hr, S = H // world, n * world
    C = 3 * Hr * Dh
    region = S * C * es                          # bytes of one receive buffer; staging buffers are as large
    mem = np.full(2 * world * region // es, np.nan, dtype=np.float32)   # [recv of every rank | staging of every rank]
    recv = [r * region for r in range(world)]
    send = [world * region + r * region for r in range(world)]
    g = np.random.RandomState(11)
    local = [g.randn(n, 3, H, Dh).astype(np.float32) for _ in range(world)]
    for rank in range(world):
        xq = QkvExchange(rank, world, n, C, es, recv, send[rank])
        parts = xq.row_parts(tile, nparts)
        assert len(parts) == (1 if tile == 128 else nparts)
        assert parts[0][0] == 0 and parts[-1][1] == n and all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        for r0, r1 in parts:
            M, base = r1 - r0, xq.bases(r0, r1 - r0)
            for row in range(M):
                for part in range(3):
                    for head in range(H):
                        owner = head // Hr
                        off = ((rank * M + row) * 3 + part) * Hr * 128 + (head - owner * Hr) * 128
                        at = base[owner] // es + off
                        mem[at:at + Dh] = local[rank][r0 + row, part, head]
        for r0, r1 in parts:
            for src, dst, nbytes in xq.copies(r0, r1):
                mem[dst // es:(dst + nbytes) // es] = mem[src // es:(src + nbytes) // es]
    full = np.concatenate(local)   # [S, 3, H, Dh], tokens in rank order
    for q in range(world):
        got = mem[recv[q] // es:(recv[q] + region) // es]
        assert np.array_equal(got, full[:, :, q * Hr:(q + 1) * Hr, :].reshape(-1))
