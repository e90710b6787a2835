"""Parity at BASELINE.json's own shapes (configs 0, 1 and 2), against the CPU oracle.

The other GPU tests prove each kernel at small shapes.  These run the kernels at the sizes the benchmark times and
check them the way the reference checks its own kernels at scale: on sampled rows (tools/check_fp4attn.py:62-79
samples query rows; its bar for bf16-class outputs is cosine >= 0.998, AGENTS.md:43).

  * config 1 -- NVFP4 W4A4 GEMM, M in {4096, 37760} x (K, N) in {(5120, 15360), (5120, 5120), (5120, 20480),
    (20480, 5120)}, bf16 out with fused bias: rel-L2 <= 1e-3 against bf16(fp64 dequantise-then-matmul) of the
    device's own operand codes, on 512 sampled rows that include the last 64; the sampled activation and weight rows'
    codes and scales bit-exact against the oracle quantiser; the fc1 GELU + NVFP4 epilogue at M = 4096 bit-exact on
    its own bf16 output.
  * config 2 -- FP8 attention, H = 40, S in {4096, 16384, 37760}: cosine >= 0.998 against fp32 SDPA over all keys on
    256 sampled query rows of every head; at S = 37760 also under the seeded 25% block-sparse mask of config 4.
  * config 0 -- one block, S = 4096, D = 5120, 40 x 128 heads, GELU 20480, through EngineBlock: cosine >= 0.998
    against the oracle's bf16 / SDPA block (all rows); the NVFP4 codes the block itself wrote for its fc1 and fc2
    inputs bit-exact against the oracle quantiser at that shape.
  * the real MiniMax H3 shape the drop-in serves -- one block, S = 1024, D = 5376, 56 x 128 heads, SwiGLU 14336,
    RoPE over 96 dims: cosine >= 0.998 against the oracle's bf16 / SDPA block.

Inputs are made on the device from seeded generators with BASELINE's distributions (activations N(0, 1) with 1% of
channels x 20, weights N(0, 0.02)); only the sampled rows and the operands the oracle needs come back to the host.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import block as OB
from oracle import nvfp4 as ON
from oracle import ops as OO

from helpers import device_ok, need_gpu, to_np, u8
from tfvideo.synthetic import dev_activations, dev_qkv, dev_weight

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-3          # rel-L2, the north star's GEMM bar
COS_BAR = 0.998          # attention and block outputs against the bf16 / fp32 reference
CFG1_SHAPES = [(5120, 15360), (5120, 5120), (5120, 20480), (20480, 5120)]   # (K, N): qkv, out, fc1 (up), fc2 (down)


@pytest.fixture(autouse=True)
def _gpu():
    need_gpu()


# ------------------------------------------------------------------------------------------------ inputs
def sample_rows(M: int, n: int, seed: int, tail: int = 64) -> np.ndarray:
    """n distinct row indices of [0, M): the last ``tail`` rows plus a seeded draw from the rest."""

    rs = np.random.RandomState(seed)
    last = np.arange(max(0, M - tail), M)
    rest = rs.choice(M - len(last), size=min(n - len(last), M - len(last)), replace=False)
    return np.unique(np.concatenate([rest, last]))


def tiled_rows(sf_tiled: torch.Tensor, rows: np.ndarray, groups: int) -> np.ndarray:
    """The [len(rows), groups] e4m3 scale bytes of the given rows, read out of a tiled scale buffer."""

    buf = u8(sf_tiled).reshape(-1)
    r, k = np.meshgrid(rows, np.arange(groups), indexing="ij")
    return buf[ON.sf_tiled_offset(r, k, groups)]


def dequant_matmul(a: np.ndarray, codes_b: np.ndarray, sf_b: np.ndarray, g_b: float, chunk: int = 4096):
    """a [R, K] (fp64) @ dequantise(B)^T in fp64, B dequantised ``chunk`` rows at a time (bounded host memory)."""

    outs = []
    at = torch.from_numpy(a)
    for n0 in range(0, codes_b.shape[0], chunk):
        b = ON.dequantize(codes_b[n0:n0 + chunk], sf_b[n0:n0 + chunk], g_b).astype(np.float64)
        outs.append((at @ torch.from_numpy(b).T).numpy())
    return np.concatenate(outs, 1)


# ------------------------------------------------------------------------------------------------ config 1
@pytest.mark.parametrize("K,N", CFG1_SHAPES)
def test_config1_gemm_store_bias(K, N):
    from tfvideo import linear as L
    from tfvideo import native as Nat

    w = dev_weight(N, K, seed=100 + N + K)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.1
    lin = L.Nvfp4Linear(w, bias=bias)
    codes_b, sf_b = u8(lin.codes), ON.sf_from_tiled(u8(lin.sf), N, K // 16)
    # the weight quantiser at this shape: sampled rows bit-exact against the oracle
    wr = sample_rows(N, 256, seed=1)
    rc, rsf = ON.quantize(to_np(w[torch.from_numpy(wr).cuda()]), np.float32(lin.g))
    assert np.array_equal(codes_b[wr], rc)
    assert np.array_equal(sf_b[wr], rsf)
    del w
    bias_np = bias.numpy().astype(np.float64)
    for M in (4096, 37760):
        x = dev_activations(M, K, seed=M + K)
        g = ON.global_scale(float(x.float().abs().amax()))
        lin.set_act(float(g))
        codes, sf = L.quantize(x, g=float(g), tiled=True)
        out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        lin.gemm(codes, sf, M, Nat.H3Epilogue(kind=Nat.H3_EPI_STORE, out=out.data_ptr(), ldo=N))
        torch.cuda.synchronize()
        rows = sample_rows(M, 512, seed=M)
        ri = torch.from_numpy(rows).cuda()
        a_codes, a_sf = u8(codes[ri]), tiled_rows(sf, rows, K // 16)
        qc, qsf = ON.quantize(to_np(x[ri]), g)
        assert np.array_equal(a_codes, qc), f"M={M}: activation codes differ from the oracle quantiser"
        assert np.array_equal(a_sf, qsf), f"M={M}: activation scales differ from the oracle quantiser"
        A = ON.dequantize(a_codes, a_sf, g).astype(np.float64)
        ref = ON.bf16_round((dequant_matmul(A, codes_b, sf_b, lin.g) + bias_np[None, :]).astype(np.float32))
        got = to_np(out[ri])
        err = OO.rel_l2(got, ref)
        assert err <= GEMM_TOL, f"M={M} K={K} N={N}: rel-L2 {err:.2e} > {GEMM_TOL}"
        del x, codes, sf, out
    device_ok()


def test_config1_fc1_gelu_nvfp4_epilogue():
    """fc1 at M = 4096 (5120 -> 20480) with the GELU-tanh + NVFP4 requantising epilogue the step runs: the bf16
    activation against GELU of the dequant-matmul reference, and the NVFP4 codes / scales the epilogue wrote bit-exact
    against the oracle quantiser applied to that same bf16 activation."""

    from tfvideo import linear as L
    from tfvideo import native as Nat

    M, K, N = 4096, 5120, 20480
    lin = L.Nvfp4Linear(dev_weight(N, K, seed=77))
    codes_b, sf_b = u8(lin.codes), ON.sf_from_tiled(u8(lin.sf), N, K // 16)
    x = dev_activations(M, K, seed=78)
    g = ON.global_scale(float(x.float().abs().amax()))
    lin.set_act(float(g))
    codes, sf = L.quantize(x, g=float(g), tiled=True)
    act = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    qs = L.new_slots(1, "cuda")
    g2 = np.float32(0.05)                       # a fixed scale for fc2's input, as a delayed-scale forward has
    qs[0, 1] = float(g2)
    qc = torch.empty((M, N // 2), dtype=torch.uint8, device="cuda")
    qsf = torch.zeros(Nat.sf_tiled_bytes(M, N), dtype=torch.uint8, device="cuda")
    lin.gemm(codes, sf, M, Nat.H3Epilogue(kind=Nat.H3_EPI_ACT_Q, act_kind=Nat.ACT_GELU, out=act.data_ptr(), ldo=N,
                                          qcodes=qc.data_ptr(), qsf=qsf.data_ptr(), q_slot=Nat.slot_ptr(qs, 0)))
    torch.cuda.synchronize()
    rows = sample_rows(M, 512, seed=3)
    ri = torch.from_numpy(rows).cuda()
    A = ON.dequantize(u8(codes[ri]), tiled_rows(sf, rows, K // 16), g).astype(np.float64)
    y = ON.bf16_round(dequant_matmul(A, codes_b, sf_b, lin.g).astype(np.float32))
    a = to_np(act[ri])
    assert OO.rel_l2(a, OO.gelu_tanh(y)) <= 5e-3
    rc, rsf = ON.quantize(a, g2)
    assert np.array_equal(u8(qc[ri]), rc)
    assert np.array_equal(tiled_rows(qsf, rows, N // 16), rsf)
    assert to_np(qs)[0, 0] == float(act.float().abs().amax())
    device_ok()


# ------------------------------------------------------------------------------------------------ config 2
def sampled_sdpa(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor, key_mask=None) -> torch.Tensor:
    """fp32 softmax(q k^T / sqrt(128)) v for a few query rows of one head over all keys (CPU)."""

    s = (q_rows.float() @ k.float().T) / math.sqrt(128.0)
    if key_mask is not None:
        s = s.masked_fill(~key_mask, float("-inf"))
    return torch.softmax(s, -1) @ v.float()


def _attention_case(S: int, H: int, mask=None):
    from tfvideo import attention as A

    qkv = dev_qkv(S, H, seed=S)
    HD = H * 128
    flat = qkv.view(S, 3 * HD)
    out = torch.empty((S, HD), dtype=torch.bfloat16, device="cuda")
    A.fp8_tokens(flat[:, :HD], flat[:, HD:2 * HD], flat[:, 2 * HD:], S, H, 3 * HD, 128, out, mask=mask)
    torch.cuda.synchronize()
    device_ok()
    rows = sample_rows(S, 256, seed=S + 1, tail=16)
    host = qkv.cpu()                                  # [S, 3, H, 128] bf16
    rt = torch.from_numpy(rows)
    got = out.view(S, H, 128)[torch.from_numpy(rows).cuda()].float().cpu()
    key_mask = None
    if mask is not None:
        keep = torch.zeros(len(rows), S, dtype=torch.bool)
        for i, r in enumerate(rows):
            for c in mask.lists[int(r) // 128]:
                keep[i, c * 128:(c + 1) * 128] = True
        key_mask = keep
    ref = torch.empty_like(got)
    for h in range(H):
        ref[:, h] = sampled_sdpa(host[rt, 0, h], host[:, 1, h], host[:, 2, h], key_mask)
    got_np, ref_np = got.numpy(), ref.numpy()
    assert np.isfinite(got_np).all()
    per_head = [OO.cosine(got_np[:, h], ref_np[:, h]) for h in range(H)]
    c = OO.cosine(got_np, ref_np)
    assert c >= COS_BAR, f"S={S} H={H}: cosine {c:.6f} (worst head {min(per_head):.6f})"
    assert min(per_head) >= COS_BAR - 0.002, f"S={S}: worst head cosine {min(per_head):.6f}"


@pytest.mark.parametrize("S", [4096, 16384, 37760])
def test_config2_attention_h40(S):
    _attention_case(S, 40)


def test_config4_block_sparse_attention_h40_s37760():
    from tfvideo import attention as A

    S = 37760
    _attention_case(S, 40, mask=A.TileMask.block_sparse(S, keep=0.25, text_tokens=512, seed=4))


# ------------------------------------------------------------------------------------------------ config 0
def test_config0_block_s4096():
    from tfvideo import minimax_h3 as M

    S = 4096
    cfg = M.Config(layers=1, dim=5120, heads=40, head_dim=128, ffn=20480, act="gelu", t_dim=8)
    w = next(M.synthetic_weights(cfg, seed=11, device="cuda"))
    eng = M.MiniMaxH3Engine.from_weights([w], cfg, device="cuda")
    x = dev_activations(S, cfg.dim, seed=12)
    x_np = to_np(x)
    t_emb = torch.randn(1, cfg.t_dim, generator=torch.Generator().manual_seed(13))
    segs = [(0, S, 0)]                               # config 0: one segment, per-token rows all from t_emb[0]
    rope = OB.rope_table(S, 128)
    rope_t = torch.from_numpy(rope).cuda().reshape(1, S, 1, 64, 2, 2)
    out = to_np(M.EngineBlock(eng, 0)(x, t_emb.cuda(), segs, rope_t))
    device_ok()
    assert np.isfinite(out).all()
    # the quantised fc1 / fc2 inputs this (first, dynamic-scale) forward wrote, against the oracle quantiser applied
    # to the block's own bf16 h2 / activation under the scales the block measured
    buf = eng._buf
    h2, act = (to_np(t) for t in buf.dynamic(cfg, S, "cuda"))
    slots = to_np(eng.slots)
    for name, a, codes, sf in (("fc1", h2, buf.h4, buf.h4sf), ("fc2", act, buf.a4, buf.a4sf)):
        s = slots[M.SLOT[name]]
        assert s[0] == np.abs(a).max(), f"{name}: amax slot"
        g = ON.global_scale(float(s[0]))
        assert np.float32(s[1]) == g, f"{name}: dynamic scale"
        rc, rsf = ON.quantize(a, g)
        assert np.array_equal(u8(codes), rc), f"{name}: NVFP4 codes differ from the oracle quantiser"
        assert np.array_equal(ON.sf_from_tiled(u8(sf), S, a.shape[1] // 16), rsf), f"{name}: scales differ"
    # the block against the oracle's bf16 / fp32-SDPA block (the north star's bar)
    shape = OB.BlockShape(dim=cfg.dim, heads=cfg.heads, head_dim=cfg.head_dim, ffn=cfg.ffn, act="gelu", rot_dim=128)
    p = OB.BlockParams(w={n: to_np(w[n]) for n in ("qkv", "out", "fc1", "fc2")}, norm1=to_np(w["norm1"]),
                       norm2=to_np(w["norm2"]), q_norm=to_np(w["q_norm"]), k_norm=to_np(w["k_norm"]),
                       ada_w=to_np(w["ada_w"]), ada_b=to_np(w["ada_b"]))
    del w
    ref = OB.block_forward(shape, p, x_np, t_emb.numpy(), segs, rope, linears="bf16", attn="sdpa")
    c = OO.cosine(out, ref)
    cu = OO.cosine(out - x_np, ref - x_np)
    assert c >= COS_BAR, f"block cosine {c:.6f}"
    assert cu >= 0.95, f"block update cosine {cu:.6f}"


# ------------------------------------------------------------------------------------------------ real H3 shape
def test_h3_shape_block_s1024():
    """One block at the real MiniMax H3 shape the drop-in serves (tfvideo/minimax_h3.py:28-36: D 5376, 56 x 128 heads,
    SwiGLU 14336, RoPE over 96 dims) against the oracle's bf16 / fp32-SDPA block, two modulation segments."""

    from tfvideo import minimax_h3 as M

    S = 1024
    cfg = M.Config(layers=1)
    assert (cfg.dim, cfg.heads, cfg.ffn, cfg.act) == (5376, 56, 14336, "swiglu")
    w = next(M.synthetic_weights(cfg, seed=21, device="cuda"))
    eng = M.MiniMaxH3Engine.from_weights([w], cfg, device="cuda")
    x = dev_activations(S, cfg.dim, seed=22)
    x_np = to_np(x)
    t_emb = torch.randn(2, cfg.t_dim, generator=torch.Generator().manual_seed(23))
    segs = [(0, 256, 0), (256, S, 1)]
    rope = OB.rope_table(S, 96)
    rope_t = torch.from_numpy(rope).cuda().reshape(1, S, 1, 48, 2, 2)
    out = to_np(M.EngineBlock(eng, 0)(x, t_emb.cuda(), segs, rope_t))
    device_ok()
    assert np.isfinite(out).all()
    shape = OB.BlockShape(dim=cfg.dim, heads=cfg.heads, head_dim=cfg.head_dim, ffn=cfg.ffn, act="swiglu", rot_dim=96)
    p = OB.BlockParams(w={n: to_np(w[n]) for n in ("qkv", "out", "fc1", "fc2")}, norm1=to_np(w["norm1"]),
                       norm2=to_np(w["norm2"]), q_norm=to_np(w["q_norm"]), k_norm=to_np(w["k_norm"]),
                       ada_w=to_np(w["ada_w"]), ada_b=to_np(w["ada_b"]))
    del w
    ref = OB.block_forward(shape, p, x_np, t_emb.numpy(), segs, rope, linears="bf16", attn="sdpa")
    c = OO.cosine(out, ref)
    cu = OO.cosine(out - x_np, ref - x_np)
    assert c >= COS_BAR, f"block cosine {c:.6f}"
    assert cu >= 0.95, f"block update cosine {cu:.6f}"
