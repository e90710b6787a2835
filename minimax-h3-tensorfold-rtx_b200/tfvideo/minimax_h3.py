"""MiniMax H3's DiT blocks on B200 (libh3b200): the ``EngineBlock`` drop-in for ComfyUI's ``DiTBlock``.

Mirrors tfvideo/minimax_h3.py of the reference: ``Config`` (:28-36), ``Block`` (:39-49), ``MiniMaxH3Engine``
(:139-333: ``begin_forward`` :220-230, ``end_run`` :232-235, ``row_index`` :252-263, ``modulation`` :265-269,
``block`` :275-312, ``_mlp_half`` :314-324), ``AttnFacade`` (:355-364) and ``EngineBlock`` (:367-381).

B200 design, against the reference's (RTX 16 GB) one:
  * all 50 blocks stay resident (8.9 GB of NVFP4 weights at BASELINE's shapes), so there is no weight streaming;
  * the MLP runs on the whole sequence (no 8192-row chunks): activations at 37.8k tokens fit in HBM;
  * every linear input is quantised by the kernel that produces it: norm_mod -> qkv / fc1, the fc1 GEMM epilogue
    (activation + NVFP4) -> fc2; gate_add is fused into the out / fc2 GEMM epilogues;
  * activation scales stay on the device (H3ScaleSlot): the first forward measures each input's absmax (dynamic),
    later forwards use the previous forward's absmax x margin (delayed) -- the reference's policy, with no host read;
  * with a process group, tokens are sharded over ranks and attention runs Ulysses head-parallel (tfvideo/parallel.py).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import attention as A
from . import kernels as K
from . import linear as L
from . import native as N
from .parallel import QkvExchange
from .profiling import maybe

LIN_NAMES = ("qkv", "out", "fc1", "fc2")
SOURCE = {"qkv": "attn.qkv_proj", "out": "attn.out_proj", "fc1": "mlp.fc1", "fc2": "mlp.fc2"}
SLOT = {name: i for i, name in enumerate(LIN_NAMES)}   # a block's input-scale slots: 4 * block + SLOT[name]


@dataclass(frozen=True)
class Config:
    layers: int = 50
    dim: int = 5376
    heads: int = 56
    head_dim: int = 128
    ffn: int = 14336
    eps: float = 1e-5
    qk_eps: float = 1e-5
    act: str = "swiglu"      # MiniMax H3: fc1 emits [gate | up]; BASELINE's H3-shaped configs use "gelu"
    t_dim: int = 8

    @property
    def inner(self) -> int:
        return self.heads * self.head_dim

    @property
    def fc1_out(self) -> int:
        return 2 * self.ffn if self.act == "swiglu" else self.ffn


H3 = Config()
BASELINE = Config(dim=5120, heads=40, ffn=20480, act="gelu")


@dataclass
class Block:
    lins: dict
    norm1: torch.Tensor            # fp32 [D]
    norm2: torch.Tensor
    q_norm: torch.Tensor           # fp32 [head_dim]
    k_norm: torch.Tensor
    ada_w: torch.Tensor            # fp32 [3 * 6 * D, t_dim]
    ada_b: torch.Tensor            # fp32 [3 * 6 * D]
    host: dict = field(default_factory=dict)
    resident: bool = True


def synthetic_weights(cfg: Config, seed: int = 1, device="cuda"):
    """Seeded random block weights of cfg's shapes (W ~ N(0, 0.02) bf16, norms 1 + N(0, 0.02), ada_w ~ N(0, 0.1 /
    sqrt(t_dim)), biases 0), generated on ``device`` one block at a time."""

    g = torch.Generator(device=device).manual_seed(seed)
    D, HD = cfg.dim, cfg.inner
    dims = {"qkv": (3 * HD, D), "out": (D, HD), "fc1": (cfg.fc1_out, D), "fc2": (D, cfg.ffn)}
    for _ in range(cfg.layers):
        w = {n: (torch.randn(s, generator=g, device=device) * 0.02).to(torch.bfloat16) for n, s in dims.items()}
        w["norm1"] = 1 + 0.02 * torch.randn(D, generator=g, device=device)
        w["norm2"] = 1 + 0.02 * torch.randn(D, generator=g, device=device)
        w["q_norm"] = 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device)
        w["k_norm"] = 1 + 0.02 * torch.randn(cfg.head_dim, generator=g, device=device)
        w["ada_w"] = torch.randn(18 * D, cfg.t_dim, generator=g, device=device) * (0.1 / math.sqrt(cfg.t_dim))
        w["ada_b"] = torch.zeros(18 * D, device=device)
        yield w


class _Buffers:
    """Per-sequence-length activations and scratch (allocated once per shape, reused by every block)."""

    def __init__(self, cfg: Config, n: int, S: int, world: int, M: int, device, peers=None):
        D, HD, F = cfg.dim, cfg.inner, cfg.ffn
        e = dict(device=device)
        self.key = (n, S, M)
        self.h4 = torch.empty((n, D // 2), dtype=torch.uint8, **e)
        self.h4sf = torch.zeros(N.sf_tiled_bytes(n, D), dtype=torch.uint8, **e)
        self.qkv = torch.empty((n, 3 * HD), dtype=torch.bfloat16, **e)
        Hl = cfg.heads // world
        self.attn_ws = torch.empty(N.attn_workspace_bytes(S, Hl) + 1024, dtype=torch.uint8, **e)
        self.o = torch.empty((S, Hl * cfg.head_dim), dtype=torch.bfloat16, **e)
        self.o4 = torch.empty((n, HD // 2), dtype=torch.uint8, **e)
        self.o4sf = torch.zeros(N.sf_tiled_bytes(n, HD), dtype=torch.uint8, **e)
        self.a4 = torch.empty((n, F // 2), dtype=torch.uint8, **e)
        self.a4sf = torch.zeros(N.sf_tiled_bytes(n, F), dtype=torch.uint8, **e)
        self.mod = torch.empty((M, 18 * D), dtype=torch.float32, **e)
        self.peers = None
        if world > 1:
            if peers is not None:   # receive buffers the other ranks' kernels store into (fused exchanges)
                self.peers = peers
                self.qkv_all, self.o_recv = peers[0].tensor, peers[1].tensor
            else:
                self.qkv_all = torch.empty((S, 3, Hl, cfg.head_dim), dtype=torch.bfloat16, **e)
                self.o_recv = torch.empty((world, n, Hl * cfg.head_dim), dtype=torch.bfloat16, **e)
        self._dyn = None

    def dynamic(self, cfg: Config, n: int, device):
        """bf16 copies of h and the activation: only the first (dynamic-scale) forward writes them."""

        if self._dyn is None:
            self._dyn = (torch.empty((n, cfg.dim), dtype=torch.bfloat16, device=device),
                         torch.empty((n, cfg.ffn), dtype=torch.bfloat16, device=device))
        return self._dyn


class MiniMaxH3Engine:
    """The DiT blocks with NVFP4 linears on B200; ``attn`` picks the attention backend (fp8 by default).
    ``attn_mask`` (an attention.TileMask for the sequence length) runs the FP8 attention block-sparse."""

    MLP_CHUNK = None                      # the whole sequence at once (HBM holds it)

    def __init__(self, blocks: list[Block], kind: str = "nvfp4", cfg: Config = Config(), device="cuda",
                 attn: str = "auto", slots: torch.Tensor | None = None, group=None):
        self.blocks, self.kind, self.cfg, self.device = blocks, kind, cfg, torch.device(device)
        self.attn = A.get(attn)
        self.attn_name = attn
        self.slots = slots if slots is not None else L.new_slots(4 * len(blocks), self.device)
        self.sp = None
        if group is not None or (torch.distributed.is_available() and torch.distributed.is_initialized()
                                 and torch.distributed.get_world_size() > 1):
            from .parallel import SequenceParallel
            self.sp = SequenceParallel(group)
        self.delayed_scales = os.environ.get("TFVIDEO_DELAYED_SCALES", "1") != "0"
        self.on_forward = None
        self.source: str | None = None
        self.lora_sig = ""
        self._forwards = 0
        self._delayed_now = False
        self._buf = None
        self._idx_key = self._idx = None
        self._rope_key = self._rope = None
        self.clipped = torch.zeros((), dtype=torch.int32, device=self.device)
        self.timer = None                  # a profiling.StageTimer to time each stage of each block
        self.attn_mask = None              # attention.TileMask: block-sparse FP8 attention when set
        self.qkv_parts = 4                 # Ulysses: row parts of the qkv GEMM (all but the last sent by copy engines)
        self.copy_streams = 7              # Ulysses: side streams for those copies (one per destination rank at 8)
        self.part_sender = "auto"          # Ulysses: "copy" (copy engines), "push" (a push kernel beside the GEMM),
                                           # "auto": push at 8 or more ranks, where it measured faster, else copy

    # ------------------------------------------------------------------ construction
    @classmethod
    def from_weights(cls, weights, cfg: Config, device="cuda", attn: str = "auto", group=None,
                     layers: int | None = None) -> "MiniMaxH3Engine":
        """Quantise per-block bf16 weight dicts (qkv, out, fc1, fc2, norm1, norm2, q_norm, k_norm, ada_w, ada_b) into
        resident NVFP4 blocks.  ``weights`` may be a generator (one block at a time)."""

        n = cfg.layers if layers is None else layers
        slots = L.new_slots(4 * n, device)
        blocks = []
        for i, w in enumerate(weights):
            if i >= n:
                break
            lins = {name: L.Nvfp4Linear(w[name], slots=slots, slot=4 * i + SLOT[name],
                                        interleave16=(name == "fc1" and cfg.act == "swiglu"))
                    for name in LIN_NAMES}
            f = lambda t: t.to(device=device, dtype=torch.float32).contiguous()   # noqa: E731
            blocks.append(Block(lins, f(w["norm1"]), f(w["norm2"]), f(w["q_norm"]), f(w["k_norm"]), f(w["ada_w"]),
                                f(w["ada_b"])))
        return cls(blocks, "nvfp4", cfg, device, attn, slots=slots, group=group)

    @classmethod
    def synthetic(cls, cfg: Config, seed: int = 1, device="cuda", attn: str = "auto", group=None):
        return cls.from_weights(synthetic_weights(cfg, seed, device), cfg, device, attn, group)

    # ------------------------------------------------------------------ per forward
    def begin_forward(self, S: int, transformer_options: dict | None = None):
        """Block 0 of each forward.  First forward after a reset: dynamic scales (each input's own absmax); after
        that (TFVIDEO_DELAYED_SCALES != 0): last forward's absmax x margin, updated on the device in one kernel."""

        if self.on_forward is not None:
            self.on_forward(self, S, transformer_options or {})
        self._rope_key = None
        delayed = self.delayed_scales and self._forwards > 0
        if delayed and self.sp is not None:
            amax = self.slots[:, 0].contiguous()
            self.sp.max_(amax)
            self.slots[:, 0].copy_(amax)
        N.scales_begin(self.slots, delayed, self.clipped)
        self._delayed_now = delayed
        self._forwards += 1

    def end_run(self):
        """A sampling run is over: the next run starts with exact per-call scales again."""

        self._forwards = 0
        N.scales_begin(self.slots, False)

    def replace_blocks(self, blocks: list[Block], lora_sig: str = "", slots: torch.Tensor | None = None) -> None:
        """Swap in re-converted blocks (a LoRA set merged, or the base weights restored); the next forward starts a
        new run with exact per-call scales."""

        if len(blocks) != len(self.blocks) and self.blocks:
            raise ValueError(f"replace_blocks: {len(blocks)} blocks for an engine of {len(self.blocks)}")
        self.blocks = blocks
        if slots is not None:
            self.slots = slots
        self.lora_sig = lora_sig
        self.end_run()

    def release_vram(self):
        self._buf = None
        torch.cuda.empty_cache()

    def row_index(self, mod_segments, S: int) -> torch.Tensor:
        """Device int32 [S] mapping every token to the row of the modulation table it uses.

        ``mod_segments`` lists (first token, end token, row) with ``row`` an int or a per-token tensor.  ComfyUI hands
        all 50 blocks of one forward the same list object, so the table is built and uploaded once per forward and
        looked up by the list's identity afterwards; the list is kept referenced so that its id cannot be reused by
        a different list while the cached table is alive."""

        if (id(mod_segments), S) == self._idx_key:
            return self._idx
        host = torch.empty(S, dtype=torch.int32)
        for first, end, row in mod_segments:
            host[first:end] = row.cpu().to(torch.int32) if torch.is_tensor(row) else int(row)
        self._idx = host.to(self.device, non_blocking=True)
        self._idx_key, self._idx_ref = (id(mod_segments), S), mod_segments
        return self._idx

    def rope_table(self, rope_freqs: torch.Tensor, S: int) -> torch.Tensor:
        """fp32 [S, rot/2, 2, 2] from ComfyUI's [1, S, 1, rot/2, 2, 2] rotation table (cached within a forward)."""

        key = (id(rope_freqs), rope_freqs.data_ptr(), rope_freqs._version)
        if key != self._rope_key:
            self._rope = rope_freqs.reshape(S, -1, 2, 2).to(device=self.device, dtype=torch.float32).contiguous()
            self._rope_key = key
        return self._rope

    def modulation(self, b: Block, t_emb: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """fp32 [M * 3, 6, D]: ada_b + t_emb @ ada_w^T viewed as ComfyUI's mod rows."""

        t = t_emb.to(device=self.device, dtype=torch.float32).contiguous()
        out = torch.empty((t.shape[0], b.ada_w.shape[0]), dtype=torch.float32, device=self.device) if out is None \
            else out
        N.modulation(t, b.ada_w, b.ada_b, out)
        return out.view(-1, 6, self.cfg.dim)

    def _buffers(self, n: int, S: int, M: int) -> _Buffers:
        world = 1 if self.sp is None else self.sp.world
        if self._buf is None or self._buf.key != (n, S, M):
            self._buf = None
            self._buf = _Buffers(self.cfg, n, S, world, M, self.device, self._peer_buffers(n, S))
        return self._buf

    def _peer_buffers(self, n: int, S: int):
        """The qkv and attention-output receive buffers of the fused Ulysses exchanges (NCCL groups on GPUs), made
        once per sequence length: every rank maps every rank's, so they are kept rather than freed."""

        if self.sp is None or self.device.type != "cuda" or dist.get_backend(self.sp.group) != "nccl":
            return None
        key = (n, S)
        cache = self.__dict__.setdefault("_peer_cache", {})
        if key not in cache:
            from .parallel import PeerBuffer
            Hl, Dh = self.cfg.heads // self.sp.world, self.cfg.head_dim
            cache[key] = (PeerBuffer(self.sp, (S, 3, Hl, Dh), torch.bfloat16, self.device),
                          PeerBuffer(self.sp, (self.sp.world, n, Hl * Dh), torch.bfloat16, self.device))
        return cache[key]

    def _slot(self, i: int, name: str) -> int:
        return N.slot_ptr(self.slots, 4 * i + SLOT[name])

    def _dynamic_scale(self, i: int, name: str) -> None:
        if self.sp is not None:
            self.sp.max_(self.slots[4 * i + SLOT[name], 0:1])
        N.scales_dynamic(self._slot(i, name))

    # ------------------------------------------------------------------ the block
    def block(self, i: int, x: torch.Tensor, t_emb, mod_segments, rope_freqs, attention=None,
              transformer_options=None) -> torch.Tensor:
        cfg, b = self.cfg, self.blocks[i]
        if x.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
            raise ValueError(f"EngineBlock expects a contiguous bf16 [S, D] x, got {tuple(x.shape)} {x.dtype}")
        n = x.shape[0]
        world = 1 if self.sp is None else self.sp.world
        S = n * world
        t0 = 0 if self.sp is None else self.sp.rank * n
        H, Dh, D = cfg.heads, cfg.head_dim, cfg.dim
        HD = H * Dh
        buf = self._buffers(n, S, t_emb.shape[0] if t_emb.dim() == 2 else 1)
        idx = self.row_index(mod_segments, S)[t0:t0 + n]
        mod = self.modulation(b, t_emb.reshape(-1, t_emb.shape[-1]), buf.mod)
        delayed = self._delayed_now
        lq, lo, l1, l2 = (b.lins[k] for k in LIN_NAMES)

        # ---- norm1 (+ NVFP4 of the qkv input)
        if attention is not None or not delayed:
            h = buf.dynamic(cfg, n, self.device)[0]
            N.norm_mod(x, b.norm1, mod, idx, 0, cfg.eps, out=h, slot=self._slot(i, "qkv"))
        if attention is not None:
            # An attention override handed in by ComfyUI (a sparse-attention patch, for instance) owns the whole
            # attention half: given the normed input it computes qkv, q/k norms, RoPE and attention through
            # EngineBlock.attn and returns the out-projection's output, which the gate adds to the residual here.
            a = attention(h, rope_freqs=rope_freqs, transformer_options=transformer_options or {})
            K.gate_add(x, a, mod, 0, idx)
            return self._mlp_half(i, b, x, mod, idx, buf, delayed)
        T = self.timer
        with maybe(T, "norm_mod+quant"):
            if delayed:
                N.norm_mod(x, b.norm1, mod, idx, 0, cfg.eps, codes=buf.h4, sf=buf.h4sf, slot=self._slot(i, "qkv"))
            else:
                self._dynamic_scale(i, "qkv")
                N.nvfp4_quant(h, buf.h4, buf.h4sf, g_ptr=self._slot(i, "qkv") + 4)
        # ---- qkv, q/k RMSNorm + RoPE, attention
        rope_all = self.rope_table(rope_freqs, S)
        rot = rope_all.shape[1] * 2
        ws = A.aligned_workspace(buf.attn_ws)
        if self.sp is not None and buf.peers is not None and self.attn is A.fp8:
            # Ulysses with the exchanges in the producing kernels: the qkv GEMM's epilogue writes each head's columns
            # in the receiving rank's row layout -- this rank's heads straight into its own receive buffer, the other
            # ranks' into one contiguous block each of a local staging buffer, which one push kernel then streams
            # into their receive buffers over NVLink (row-scattered stores from the epilogue itself would cross the
            # link as 16-byte requests).  The attention kernel stores each token's output rows straight into the
            # owner's buffer: those stores are few and spread over the kernel's run (staging and pushing them measured
            # no faster).  A barrier after each replaces the all-to-all.  RMSNorm + RoPE run on the received rows
            # (all S tokens, this rank's heads): the same per-(token, head) arithmetic as before the exchange.
            Hl, rank = H // world, self.sp.rank
            qp, op = buf.peers
            xq = QkvExchange(rank, world, n, 3 * Hl * Dh, buf.qkv.element_size(), qp.ptrs, buf.qkv.data_ptr())
            # row parts: each part's blocks but the last leave on the copy engines (no SMs) while the GEMM computes
            # the next part, one side stream per destination rank so that the copies to different ranks run on
            # different copy engines at once; the last part's go by the push kernel once the GEMM has freed the SMs
            parts = xq.row_parts(parts=self.qkv_parts)
            sides = self.__dict__.setdefault(
                "_side_streams", [torch.cuda.Stream(device=self.device) for _ in range(max(1, self.copy_streams))])
            cur = torch.cuda.current_stream(self.device)
            with maybe(T, "gemm_qkv"):
                for j, (r0, r1) in enumerate(parts):
                    epi = N.H3Epilogue(kind=N.H3_EPI_STORE_PEERS, ranks=world, rank=rank)
                    for r, pp in enumerate(xq.bases(r0, r1 - r0)):
                        epi.peer[r] = pp
                    lq.gemm(buf.h4[r0:r1], buf.h4sf[N.sf_tiled_bytes(r0, D) if r0 else 0:], r1 - r0, epi)
                    if j + 1 < len(parts):
                        sender = self.part_sender
                        if sender == "auto":
                            sender = "push" if world >= 8 else "copy"
                        if sender == "push":    # one push kernel beside the GEMM's next part
                            sides[0].wait_stream(cur)
                            N.peer_push(xq.copies(r0, r1), sides[0].cuda_stream)
                        else:
                            for c, copy in enumerate(xq.copies(r0, r1)):
                                side = sides[c % len(sides)]
                                side.wait_stream(cur)
                                N.peer_copy([copy], side.cuda_stream)
            with maybe(T, "exchange_push"):
                N.peer_push(xq.copies(*parts[-1]))
                for side in sides:
                    cur.wait_stream(side)
            with maybe(T, "exchange_barrier"):
                self.sp.barrier(self.device)
            qa = buf.qkv_all.view(S, 3 * Hl * Dh)
            q, k, v = qa[:, :Hl * Dh], qa[:, Hl * Dh:2 * Hl * Dh], qa[:, 2 * Hl * Dh:]
            with maybe(T, "qknorm_rope"):
                N.qknorm_rope(q, k, 3 * Hl * Dh, S, Hl, rot, b.q_norm, b.k_norm, rope_all, cfg.qk_eps)
            with maybe(T, "attention"):
                m = self.attn_mask
                if m is not None and m.S != S:
                    raise ValueError(f"attn_mask is for S={m.S}, the sequence has S={S}")
                N.attn_fp8_peers(q, k, v, 3 * Hl * Dh, Dh, S, Hl, op.ptrs, rank, Hl * Dh, ws,
                                 kv_ptr=None if m is None else m.kv_ptr, kv_idx=None if m is None else m.kv_idx)
            with maybe(T, "exchange_barrier"):
                self.sp.barrier(self.device)
            src = dict(x=buf.o_recv, R=n, K=HD, ldx=Hl * Dh, cblk=Hl * Dh, blk_stride=n * Hl * Dh)
        else:
            with maybe(T, "gemm_qkv"):
                lq.gemm(buf.h4, buf.h4sf, n, N.H3Epilogue(kind=N.H3_EPI_STORE, out=buf.qkv.data_ptr(), ldo=3 * HD))
            rope = rope_all[t0:t0 + n]
            q, k, v = buf.qkv[:, :HD], buf.qkv[:, HD:2 * HD], buf.qkv[:, 2 * HD:]
            with maybe(T, "qknorm_rope"):
                N.qknorm_rope(q, k, 3 * HD, n, H, rot, b.q_norm, b.k_norm, rope, cfg.qk_eps)
            if self.sp is None:
                with maybe(T, "attention"):
                    self._attend(q, k, v, S, H, 3 * HD, buf.o, ws)
                src = dict(x=buf.o, R=n, K=HD)
            else:
                Hl = H // world
                with maybe(T, "all_to_all"):
                    self.sp.qkv_heads_from_tokens(buf.qkv.view(n, 3, H, Dh), buf.qkv_all)
                qa = buf.qkv_all.view(S, 3 * Hl * Dh)
                with maybe(T, "attention"):
                    self._attend(qa[:, :Hl * Dh], qa[:, Hl * Dh:2 * Hl * Dh], qa[:, 2 * Hl * Dh:], S, Hl,
                                 3 * Hl * Dh, buf.o, ws)
                with maybe(T, "all_to_all"):
                    self.sp.tokens_from_heads(buf.o, buf.o_recv)
                src = dict(x=buf.o_recv, R=n, K=HD, ldx=Hl * Dh, cblk=Hl * Dh, blk_stride=n * Hl * Dh)
        # ---- out-projection input -> NVFP4, out GEMM with the gated residual fused
        sl = self._slot(i, "out")
        with maybe(T, "quant_attn_out"):
            if delayed:
                N.nvfp4_quant(codes=buf.o4, sf=buf.o4sf, g_ptr=sl + 4, amax_ptr=sl, **src)
            else:
                N.absmax_into(src["x"].reshape(-1, src["x"].shape[-1]), sl)
                self._dynamic_scale(i, "out")
                N.nvfp4_quant(codes=buf.o4, sf=buf.o4sf, g_ptr=sl + 4, **src)
        with maybe(T, "gemm_out+gate"):
            lo.gemm(buf.o4, buf.o4sf, n, N.H3Epilogue(kind=N.H3_EPI_GATE_RESID, x=x.data_ptr(), ldx=D,
                                                      mod=mod.data_ptr(), idx=idx.data_ptr(), gate_part=0))
        x = self._mlp_half(i, b, x, mod, idx, buf, delayed)
        if buf.peers is not None and i == len(self.blocks) - 1:
            # the last block of a Ulysses forward: every barrier of the forward carried the ranks' device status;
            # a rank whose exchange kernel gave up a wait fails the forward here on every rank (one host read)
            status = self.sp.failed()
            if status:
                raise RuntimeError(f"Ulysses forward failed: a rank's kernel gave up a bounded wait (device status "
                                   f"{status}); the receive buffers of this forward are incomplete")
        return x

    def _attend(self, q, k, v, S, H, ld, out, ws):
        m = self.attn_mask
        if self.attn is A.fp8 and m is not None:
            if m.S != S:
                raise ValueError(f"attn_mask is for S={m.S}, the sequence has S={S}")
            N.attn_fp8_sparse(q, k, v, ld, self.cfg.head_dim, S, H, m.kv_ptr, m.kv_idx, out, out.stride(0), ws)
        elif self.attn is A.fp8:
            N.attn_fp8(q, k, v, ld, self.cfg.head_dim, S, H, out, out.stride(0), ws)
        else:   # a library backend (sdpa / cudnn), for comparisons
            Dh = self.cfg.head_dim
            qh, kh, vh = (t.as_strided((1, H, S, Dh), (0, Dh, ld, 1)) for t in (q, k, v))
            o = self.attn(qh, kh, vh)
            out.view(S, H, Dh).copy_(o[0].transpose(0, 1))

    def _mlp_half(self, i, b, x, mod, idx, buf, delayed):
        cfg = self.cfg
        n = x.shape[0]
        l1, l2 = b.lins["fc1"], b.lins["fc2"]
        act_kind = N.ACT_SWIGLU if cfg.act == "swiglu" else N.ACT_GELU
        s1, s2 = self._slot(i, "fc1"), self._slot(i, "fc2")
        T = self.timer
        if delayed:
            with maybe(T, "norm_mod+quant"):
                N.norm_mod(x, b.norm2, mod, idx, 1, cfg.eps, codes=buf.h4, sf=buf.h4sf, slot=s1)
            with maybe(T, "gemm_fc1+act+quant"):
                l1.gemm(buf.h4, buf.h4sf, n, N.H3Epilogue(kind=N.H3_EPI_ACT_Q, act_kind=act_kind,
                                                          qcodes=buf.a4.data_ptr(), qsf=buf.a4sf.data_ptr(),
                                                          q_slot=s2))
        else:
            h, a = buf.dynamic(cfg, n, self.device)
            N.norm_mod(x, b.norm2, mod, idx, 1, cfg.eps, out=h, slot=s1)
            self._dynamic_scale(i, "fc1")
            N.nvfp4_quant(h, buf.h4, buf.h4sf, g_ptr=s1 + 4)
            l1.gemm(buf.h4, buf.h4sf, n, N.H3Epilogue(kind=N.H3_EPI_ACT_BF16, act_kind=act_kind, out=a.data_ptr(),
                                                      ldo=a.stride(0), q_slot=s2))
            self._dynamic_scale(i, "fc2")
            N.nvfp4_quant(a, buf.a4, buf.a4sf, g_ptr=s2 + 4)
        with maybe(T, "gemm_fc2+gate"):
            l2.gemm(buf.a4, buf.a4sf, n, N.H3Epilogue(kind=N.H3_EPI_GATE_RESID, x=x.data_ptr(), ldx=cfg.dim,
                                                      mod=mod.data_ptr(), idx=idx.data_ptr(), gate_part=1))
        return x

    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options=None):
        """All blocks in order (what ComfyUI's model does through 50 EngineBlock calls)."""

        for i in range(len(self.blocks)):
            if i == 0:
                self.begin_forward(x.shape[0] * (1 if self.sp is None else self.sp.world), transformer_options)
            x = self.block(i, x, t_emb, mod_segments, rope_freqs, None, transformer_options)
        return x

    # ------------------------------------------------------------------ info
    def linears(self):
        for i, b in enumerate(self.blocks):
            for name in LIN_NAMES:
                yield f"{i}.{name}", b.lins[name]

    def block_bytes(self) -> int:
        return sum(l.nbytes() for l in self.blocks[0].lins.values()) if self.blocks else 0

    def nbytes(self) -> int:
        return sum(l.nbytes() for _, l in self.linears())


class _Proj:
    """Calls block ``i``'s linear ``name`` as a plain projection (bf16 [M, K] -> [M, N]) on the NVFP4 GEMM, with
    the input's own dynamic scale: the form in which an attention override computes qkv and the out-projection."""

    def __init__(self, engine, i, name):
        self.engine, self.i, self.name = engine, i, name

    def __call__(self, x):
        return self.engine.blocks[self.i].lins[self.name](x.contiguous())


class _Norm:
    """One of block ``i``'s per-head RMSNorm weights (fp32 [head_dim]) behind a ``.weight`` attribute, read from the
    engine when asked, so it follows LoRA re-conversions and block swaps; ``eps`` is the norm's epsilon."""

    def __init__(self, engine, i, name, eps):
        self.engine, self.i, self.name, self.eps = engine, i, name, eps

    @property
    def weight(self):
        return getattr(self.engine.blocks[self.i], self.name)


class AttnFacade:
    """``block.attn`` for code written against ComfyUI's own MiniMax H3 block: the attributes an attention override
    reads (``heads``, ``head_dim``, ``qkv_proj``, ``out_proj``, ``q_norm``, ``k_norm``, ``to_gate_compress``), each
    resolving to the engine's weights for block ``i``.  The override gets the engine's projections and norms and can
    run any attention in between, the engine's block-sparse FP8 kernel included."""

    def __init__(self, engine, i):
        cfg = engine.cfg
        self.heads, self.head_dim = cfg.heads, cfg.head_dim
        self.qkv_proj, self.out_proj = _Proj(engine, i, "qkv"), _Proj(engine, i, "out")
        self.q_norm, self.k_norm = _Norm(engine, i, "q_norm", cfg.qk_eps), _Norm(engine, i, "k_norm", cfg.qk_eps)
        self.to_gate_compress = None       # MiniMax H3 has no gated attention compression


class EngineBlock(torch.nn.Module):
    """A stand-in for ComfyUI's MiniMax H3 ``DiTBlock`` in the model's block list: the same forward signature,
    computed by the engine's block ``i``.  It owns no parameters (the engine keeps every weight), updates ``x`` in
    place and returns it, and starts the engine's forward (scale policy, LoRA sync) when it is block 0."""

    def __init__(self, engine: MiniMaxH3Engine, i: int):
        super().__init__()
        self.engine, self.i = engine, i
        self.attn = AttnFacade(engine, i)

    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}, attention=None):
        with _outside_comfy_allocation_capture():
            if self.i == 0:
                sp = self.engine.sp
                self.engine.begin_forward(x.shape[0] * (1 if sp is None else sp.world), transformer_options)
            return self.engine.block(self.i, x, t_emb, mod_segments, rope_freqs, attention, transformer_options)


def _outside_comfy_allocation_capture():
    """ComfyUI (dynamic-VRAM mode) records each block's device allocations in order to replay them; the engine keeps
    its own buffers per sequence length, so its block runs with that recording paused when this ComfyUI offers the
    switch (``comfy.model_prefetch.pause_malloc_graph``), and as is otherwise."""

    try:
        from comfy.model_prefetch import pause_malloc_graph
    except ImportError:
        import contextlib
        return contextlib.nullcontext()
    return pause_malloc_graph()
