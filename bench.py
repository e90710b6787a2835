#!/usr/bin/env python
"""Benchmark: one 50-block MiniMax H3-shaped DiT denoising step at 37,760 tokens (BASELINE configs 3 / 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N

A step = 50 EngineBlock forwards of the 37,760-token sequence (text 512 + keyframe 1,680 + audio 496 + video 35,072)
at BASELINE's H3 shape (hidden 5120, 40 x 128 heads, GELU-tanh FFN 20480) with random N(0, 0.02) weights quantised
to NVFP4 once at load, FP8 attention, per-token adaLN modulation.  At N > 1 the sequence is token-sharded and
attention runs Ulysses head-parallel (config 4; total work fixed, so scaling is "strong").

Timing: W warm-up steps (the first runs on dynamic scales, later ones on delayed scales -- the reference's steady
state), then K steps bracketed by a barrier + synchronize, timed with CUDA events on the launching stream, max over
ranks.  Every step reads 8.9 GB of weights plus GBs of activations, far beyond the 126 MB L2.  `e2e` repeats the step
through the public API with host buffers (pinned H2D of the step's inputs, D2H of its output, inside the timed region).

At N = 1 the same run also records, in the same JSON line:
  * `parity`: one block of the timed engine at the config-3 shape, checked on 512 sampled rows against the CPU oracle
    (bf16 linears, fp32 softmax over the device's own keys and values);
  * `configs`: the config-1 NVFP4 GEMM sweep, the config-2 FP8 attention sweep (each launch timed alone, L2 flushed
    before every timed launch) and one block at the real MiniMax H3 shape;
  * `cpu_baseline`: the reference's torch path restated on the host CPU (oracle/): the config-3 step extrapolated from
    a 512-row sample, and config 0 (one full 4,096-token block) timed outright.
`--impl reference` times that CPU restatement alone on the config-3 step (a bounded sample per step, extrapolated).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "minimax-h3-tensorfold-rtx_b200"
sys.path.insert(0, str(PKG))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "s/denoise step, 50-block H3 DiT @37.8k tok, 1/2/4/8 B200; NVFP4 GEMM TFLOPS"
# DRAM bytes (read + written) of one attention launch per (token, head): 181.7 MB measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum) for one launch at S = 8,192, H = 40.  Traffic grows with S x H, not
# S^2: the K/V of a head stay in L2 while its CTAs stream them, so the figure scales by tokens x heads.
ATTN_DRAM_BYTES_PER_TOKEN_HEAD = 181.7e6 / (8192 * 40)
SEQ = 37760
SEGS = (512, 1680, 496, 35072)          # text | keyframe | audio | video (33 latent frames x 24 x 44 patches)
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NOMINAL_TFLOPS = {"fp8": 4500.0, "nvfp4": 9000.0}   # B200 dense peaks (NVIDIA's sparse figures halved)
CFG1_SHAPES = {"qkv": (5120, 15360), "out": (5120, 5120), "fc1": (5120, 20480), "fc2": (20480, 5120)}   # (K, N)


def mod_segments(S: int):
    a = np.cumsum((0,) + SEGS[:-1]).tolist()
    segs = [(a[i], a[i] + SEGS[i], i) for i in range(3)] + [(a[3], S, 3)]
    return segs


def rope_3d(S: int, rot: int = 128, splits=(44, 42, 42), grid=(33, 24, 44), theta: float = 10000.0) -> torch.Tensor:
    """ComfyUI-style rotation table [1, S, 1, rot/2, 2, 2] fp32: text / keyframe / audio tokens at t = 0..; the video
    tokens on the (33, 24, 44) latent grid; pairs split over (t, h, w) in proportion to ``splits`` dims."""

    half = rot // 2
    parts = [s // 2 for s in splits]
    s = torch.arange(S, dtype=torch.float64)
    v0 = S - grid[0] * grid[1] * grid[2]
    vi = (s - v0).clamp_min(0)
    t = torch.where(s < v0, s, vi // (grid[1] * grid[2]))
    hh = torch.where(s < v0, torch.zeros_like(s), (vi // grid[2]) % grid[1])
    ww = torch.where(s < v0, torch.zeros_like(s), vi % grid[2])
    angs = []
    for pos, n in zip((t, hh, ww), parts):
        f = theta ** (-torch.arange(n, dtype=torch.float64) / n)
        angs.append(pos[:, None] * f[None, :])
    ang = torch.cat(angs, 1)[:, :half]
    c, sn = torch.cos(ang), torch.sin(ang)
    rope = torch.stack([torch.stack([c, -sn], -1), torch.stack([sn, c], -1)], -2)
    return rope.float().reshape(1, S, 1, half, 2, 2)


def activations(S: int, D: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(S, D, generator=g)
    ch = torch.randperm(D, generator=torch.Generator().manual_seed(2))[: D // 100]
    x[:, ch] *= 20
    return x.to(torch.bfloat16)


def peaks() -> tuple[dict, str]:
    if PEAKS.exists():
        return json.loads(PEAKS.read_text()), "measured"
    return FALLBACK, "fallback"


def cpu_info() -> dict:
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "cpu_model": model}


class Clocks:
    """nvidia-smi clock / throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self) -> dict:
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "samples": len(rows), "reasons": reasons}


# ------------------------------------------------------------------------------------------------ CPU leg
def cpu_block(rows: int, S: int, threads: int | None = None, seed: int = 0) -> dict:
    """The reference's torch path on the host CPU (oracle/torch_path.py) for one block of the H3-shaped config,
    timed: norm + modulation, NVFP4 fake-quant of every linear input, fp32 matmuls, q / k RMSNorm + RoPE, attention,
    gated residuals, GELU-tanh MLP, with all the host threads torch can use.

    rows == S is the exact block (config 0 at S = 4,096).  rows < S is a sample of an S-token block: the ``rows``
    token rows do all their per-row work (their share of every projection, the ones that make keys and values
    included) and attend over all S keys and values -- their own, written into the first ``rows`` positions, and
    S - rows others (unit-RMS rows drawn before the clock starts, standing for the rest of the sequence, whose
    projections are the other rows' per-row work)."""

    sys.path.insert(0, str(ROOT))
    from oracle import block as OB
    from oracle import torch_path as TP

    torch.set_num_threads(threads or os.cpu_count())
    D, H, Dh, F = 5120, 40, 128, 20480
    g = torch.Generator().manual_seed(seed)
    W = {n: torch.randn(s, generator=g) * 0.02 for n, s in
         {"qkv": (3 * H * Dh, D), "out": (D, H * Dh), "fc1": (F, D), "fc2": (D, F)}.items()}
    norms = {"norm1": 1 + 0.02 * torch.randn(D, generator=g), "norm2": 1 + 0.02 * torch.randn(D, generator=g),
             "q_norm": 1 + 0.02 * torch.randn(Dh, generator=g), "k_norm": 1 + 0.02 * torch.randn(Dh, generator=g)}
    x = activations(rows, D).float()
    mod = 0.1 * torch.randn(4, 6, D, generator=g)
    idx = torch.zeros(rows, dtype=torch.long)
    rope = torch.from_numpy(OB.rope_table(rows, 128))
    kv = None
    if S > rows:
        kv = tuple(torch.randn(H, S, Dh, generator=g) for _ in range(2))
        for t in kv:
            t /= t.pow(2).mean(-1, keepdim=True).sqrt()
    t0 = time.perf_counter()
    TP.block(x, W, norms, mod, idx, rope, H, kv_buffer=kv)
    dt = time.perf_counter() - t0
    return {"seconds": dt, "cores": torch.get_num_threads()}


def cpu_step_sample(rows: int, S: int = SEQ, layers: int = 50) -> dict:
    r = cpu_block(rows, S)
    return {"value": r["seconds"] * (S / rows) * layers, "sample_s": r["seconds"], "cores": r["cores"],
            "extrapolated": True,
            "sample": f"one block for {rows} of {S} token rows (their per-row work, attention over all {S} keys), "
                      f"timed, x {S / rows:.2f} rows x {layers} blocks"}


def reference_arm(a) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    rows = a.cpu_rows
    for _ in range(a.warmup):
        cpu_step_sample(rows)
    vals = [cpu_step_sample(rows) for _ in range(a.steps)]
    v = statistics.mean(r["value"] for r in vals)
    line = {"metric": METRIC, "value": v, "unit": "s/step", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": v * 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32 (NVFP4 fake-quant)", "data": "synthetic", "impl": "reference",
            "config": {"workload": "config 3 step on the host CPU (oracle restatement of the reference's torch path), "
                                   "extrapolated from a per-step sample", "global_batch": 1, "seq_len": SEQ,
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "s/step", "cores": vals[0]["cores"], "kind": "port",
                             "extrapolated": True, "sample": vals[0]["sample"],
                             "sample_seconds_per_step": statistics.mean(r["sample_s"] for r in vals), **cpu_info()},
            "e2e": {"value": v, "unit": "s/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ single ops
class Flush:
    """Writes 512 MB (> the 126 MB L2) before each timed launch, outside the timed events."""

    def __init__(self):
        self.buf = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")

    def __call__(self):
        self.buf.zero_()


def time_launches(run, reps: int, warmup: int = 2, flush: Flush | None = None) -> float:
    """Median CUDA-event milliseconds of ``run()`` over ``reps`` launches, each after an L2 flush."""

    flush = flush or Flush()
    for _ in range(warmup):
        run()
    ev = []
    for _ in range(reps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in ev)


def gemm_sweep(sustained: float, reps: int = 5) -> list[dict]:
    """Config 1: NVFP4 W4A4 GEMM, M in {4096, 37760} x the four (K, N) of a block, bf16 out with fused bias."""

    from tfvideo.synthetic import dev_activations, dev_weight
    from tfvideo import linear as L
    from tfvideo import native as N

    flush = Flush()
    res = []
    for name, (K, Nn) in CFG1_SHAPES.items():
        lin = L.Nvfp4Linear(dev_weight(Nn, K, seed=Nn + K), bias=torch.randn(Nn) * 0.1)
        for M in (4096, 37760):
            x = dev_activations(M, K, seed=M + K)
            lin.set_act(max(float(x.float().abs().amax()), 1e-6) / 2688.0)
            codes, sf = L.quantize(x, g_ptr=lin.slot_ptr() + 4)
            out = torch.empty(M, Nn, dtype=torch.bfloat16, device="cuda")
            epi = N.H3Epilogue(kind=N.H3_EPI_STORE, out=out.data_ptr(), ldo=Nn)
            ms = time_launches(lambda: lin.gemm(codes, sf, M, epi), reps, flush=flush)
            tf = 2.0 * M * Nn * K / ms / 1e9
            res.append({"gemm": name, "M": M, "K": K, "N": Nn, "ms": round(ms, 4), "tflops": round(tf, 1),
                        "frac": round(tf / (4 * sustained), 4), "frac_nominal": round(tf / NOMINAL_TFLOPS["nvfp4"], 4)})
            del x, codes, sf, out
    return res


def attn_sweep(sustained: float, reps: int = 3) -> list[dict]:
    """Config 2: FP8 attention (prepare + kernel), H = 40, S in {4096, 16384, 37760}."""

    from tfvideo.synthetic import dev_qkv
    from tfvideo import attention as A
    from tfvideo import native as N

    flush = Flush()
    res = []
    H = 40
    for S in (4096, 16384, 37760):
        qkv = dev_qkv(S, H, seed=S).view(S, 3 * H * 128)
        HD = H * 128
        out = torch.empty(S, HD, dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(N.attn_workspace_bytes(S, H) + 1024, dtype=torch.uint8, device="cuda")

        def run():
            A.fp8_tokens(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], S, H, 3 * HD, 128, out, ws)
        ms = time_launches(run, reps, flush=flush)
        tf = 4.0 * S * S * H * 128 / ms / 1e9
        res.append({"S": S, "H": H, "ms": round(ms, 3), "tflops": round(tf, 1), "frac": round(tf / (2 * sustained), 4),
                    "frac_nominal": round(tf / NOMINAL_TFLOPS["fp8"], 4)})
        del qkv, out, ws
    return res


def h3_real_block(S: int = SEQ, reps: int = 5) -> dict:
    """One block at the real MiniMax H3 shape (D 5376, 56 x 128 heads, SwiGLU 14336, rot 96) on the config-3
    sequence, delayed scales, timed per block."""

    from tfvideo import minimax_h3 as M

    cfg = M.Config(layers=1)
    eng = M.MiniMaxH3Engine.synthetic(cfg, seed=9, device="cuda")
    x0 = activations(S, cfg.dim, seed=5).cuda()
    t_emb = torch.randn(2, cfg.t_dim, generator=torch.Generator().manual_seed(3)).cuda()
    rope = rope_3d(S, rot=96, splits=(32, 32, 32)).cuda()
    segs = mod_segments(S)
    x = torch.empty_like(x0)

    def fwd():
        x.copy_(x0)
        eng.forward(x, t_emb, segs, rope)
    for _ in range(3):
        fwd()
    ev = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fwd()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    copy_ms = 387e6 * 2 / 6.5e12 * 1e3      # the x0 -> x restore inside each timed forward (about 0.1 ms)
    return {"shape": "D 5376, 56 x 128 heads, SwiGLU 14336, rot 96, S 37760", "ms_per_block": round(ms, 3),
            "s_per_50_blocks": round(ms * 50 / 1e3, 4), "note": f"includes a {copy_ms:.2f} ms input restore per block"}


def parity_probe(eng, cfg, x0, t_emb, segs, rope, rows: int = 512) -> dict:
    """Block 0 of the timed engine (delayed scales, as timed) on the config-3 input, checked on ``rows`` sampled token
    rows against the CPU oracle: bf16 linears from the block's own bf16 weights (regenerated from the engine's seed),
    fp32 attention of the sampled queries over all S keys and values as the device produced them (after its QK-norm
    + RoPE), fp32 elementwise.  Reports cosine of the block output and of the block's update (out - in)."""

    sys.path.insert(0, str(ROOT))
    from oracle import ops as OO
    from oracle.nvfp4 import bf16_round
    from tfvideo import minimax_h3 as M

    S, D = x0.shape
    H, Dh = cfg.heads, cfg.head_dim
    HD = H * Dh
    eng.begin_forward(S)
    x = x0.clone()
    eng.block(0, x, t_emb, segs, rope)
    torch.cuda.synchronize()
    rs = np.random.RandomState(17)
    ri = np.unique(np.concatenate([rs.choice(S - 64, rows - 64, replace=False), np.arange(S - 64, S)]))
    rt = torch.from_numpy(ri).cuda()
    qkv = eng._buf.qkv
    q_dev = qkv[rt, :HD].float().cpu().numpy()
    k_dev_rows = qkv[rt, HD:2 * HD].float().cpu().numpy()
    kv = qkv[:, HD:].cpu()                                  # [S, 2 HD] bf16: every key and value of the block
    x_in, x_out = x0[rt].float().cpu().numpy(), x[rt].float().cpu().numpy()
    w = next(M.synthetic_weights(cfg, seed=1, device="cuda"))
    wh = {n: w[n].float().cpu().numpy() for n in w}
    del w
    idx = OO.row_index(segs, S)[ri]
    mod = OO.modulation(t_emb.float().cpu().numpy(), wh["ada_w"], wh["ada_b"], D)
    rope_r = rope[0, rt, 0].float().cpu().numpy()
    t0 = time.perf_counter()
    h = OO.norm_mod(x_in, wh["norm1"], mod, 0, idx, cfg.eps)
    y = OO.linear_bf16(h, wh["qkv"])
    q = OO.qknorm_rope(y[:, :HD].reshape(-1, H, Dh), wh["q_norm"], rope_r, cfg.qk_eps).reshape(-1, HD)
    k = OO.qknorm_rope(y[:, HD:2 * HD].reshape(-1, H, Dh), wh["k_norm"], rope_r, cfg.qk_eps).reshape(-1, HD)
    o = np.empty((len(ri), HD), dtype=np.float32)
    qt = torch.from_numpy(q).view(-1, H, Dh)
    for hh in range(H):
        K = kv[:, hh * Dh:(hh + 1) * Dh].float()
        V = kv[:, HD + hh * Dh:HD + (hh + 1) * Dh].float()
        p = torch.softmax((qt[:, hh] @ K.T) / np.sqrt(Dh), -1)
        o[:, hh * Dh:(hh + 1) * Dh] = (p @ V).numpy()
    o = bf16_round(o)
    xm = OO.gate_add(x_in, OO.linear_bf16(o, wh["out"]), mod, 0, idx)
    a = OO.gelu_tanh(OO.linear_bf16(OO.norm_mod(xm, wh["norm2"], mod, 1, idx, cfg.eps), wh["fc1"]))
    ref = OO.gate_add(xm, OO.linear_bf16(a, wh["fc2"]), mod, 1, idx)
    c = OO.cosine(x_out, ref)
    return {"rows": int(len(ri)), "block_cosine": round(c, 6), "update_cosine": round(OO.cosine(x_out - x_in, ref - x_in), 6),
            "q_cosine": round(OO.cosine(q_dev, q), 6), "k_cosine": round(OO.cosine(k_dev_rows, k), 6),
            "bar": 0.998, "pass": bool(c >= 0.998), "cpu_seconds": round(time.perf_counter() - t0, 1),
            "reference": "oracle block, bf16 linears, fp32 softmax over the device's keys/values, sampled rows incl. "
                         "the last 64"}


# ------------------------------------------------------------------------------------------------ micro (one op)
def micro(a) -> None:
    """One op alone on synthetic inputs, timed with CUDA events (kernel-level numbers and ncu targets)."""

    from tfvideo.synthetic import dev_qkv
    from tfvideo import attention as A
    from tfvideo import linear as L
    from tfvideo import native as N

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.micro == "elem":
        return micro_elem(a)
    if a.micro == "attn":
        S, H = a.seq, a.heads
        qkv = dev_qkv(S, H, seed=S).view(S, 3 * H * 128)
        out = torch.empty(S, H * 128, dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(N.attn_workspace_bytes(S, H) + 1024, dtype=torch.uint8, device="cuda")
        HD = H * 128

        mask = A.TileMask.block_sparse(S) if a.sparse else None

        def run():
            A.fp8_tokens(qkv[:, :HD], qkv[:, HD:2 * HD], qkv[:, 2 * HD:], S, H, 3 * HD, 128, out, ws, mask=mask)
        flops = 4.0 * S * S * H * 128 * (mask.density if mask is not None else 1.0)
        what = f"attn S={S} H={H}" + (f" block-sparse {mask.density:.3f}" if mask is not None else "")
    else:
        M, Nn, K = (int(v) for v in a.mnk.split(","))
        w = (torch.randn(Nn, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        lin = L.Nvfp4Linear(w)
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        lin.set_act(float(x.float().abs().amax()) / 2688)
        codes, sf = L.quantize(x, g_ptr=lin.slot_ptr() + 4)
        out = torch.empty(M, Nn, dtype=torch.bfloat16, device="cuda")
        mod = torch.randn(4, 6, Nn, generator=g, device="cuda") * 0.1
        idx = torch.zeros(M, dtype=torch.int32, device="cuda")
        qs = L.new_slots(1, "cuda")
        qs[0, 1] = 1.0
        qc = torch.empty(M, Nn // 2, dtype=torch.uint8, device="cuda")
        qsf = torch.zeros(N.sf_tiled_bytes(M, Nn), dtype=torch.uint8, device="cuda")
        epi = {"store": N.H3Epilogue(kind=N.H3_EPI_STORE, out=out.data_ptr(), ldo=Nn),
               "gate": N.H3Epilogue(kind=N.H3_EPI_GATE_RESID, x=out.data_ptr(), ldx=Nn, mod=mod.data_ptr(),
                                    idx=idx.data_ptr(), gate_part=0),
               "act_q": N.H3Epilogue(kind=N.H3_EPI_ACT_Q, act_kind=N.ACT_GELU, qcodes=qc.data_ptr(),
                                     qsf=qsf.data_ptr(), q_slot=N.slot_ptr(qs, 0))}[a.epi]

        def run():
            lin.gemm(codes, sf, M, epi)
        flops = 2.0 * M * Nn * K
        what = f"gemm M={M} N={Nn} K={K} epi={a.epi}"
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(a.steps):
        run()
    en.record()
    torch.cuda.synchronize()
    ms = st.elapsed_time(en) / a.steps
    print(json.dumps({"micro": what, "ms": ms, "tflops": flops / ms / 1e9, "device_status": N.device_status()}),
          flush=True)


def micro_elem(a) -> None:
    """The HBM-bound kernels of a block alone at S tokens (BASELINE shapes), each launch timed with CUDA events after
    an L2 flush; rates are algorithmic bytes (read + written once) over the measured copy bandwidth."""

    from tfvideo import linear as L
    from tfvideo import native as N
    from tfvideo.synthetic import dev_activations

    S, D, H = a.seq, 5120, a.heads
    pk, src = peaks()
    hbm = pk["hbm_gbs"]
    g = torch.Generator(device="cuda").manual_seed(1)
    x = dev_activations(S, D, seed=3)
    w = 1 + 0.02 * torch.randn(D, generator=g, device="cuda")
    mod = 0.1 * torch.randn(4, 6, D, generator=g, device="cuda")
    idx = torch.randint(0, 4, (S,), generator=g, device="cuda", dtype=torch.int32)
    slots = L.new_slots(1, "cuda")
    slots[0, 1] = float(x.float().abs().amax()) / 2688.0
    codes = torch.empty(S, D // 2, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(N.sf_tiled_bytes(S, D), dtype=torch.uint8, device="cuda")
    yb = torch.empty_like(x)
    qkv = dev_activations(S, 3 * H * 128, seed=4)
    rope = rope_3d(S).cuda().reshape(S, -1, 2, 2).contiguous()
    qw, kw = (1 + 0.02 * torch.randn(128, generator=g, device="cuda") for _ in range(2))
    HD = H * 128
    sp = N.slot_ptr(slots, 0)
    cases = {
        "norm_mod+nvfp4 (delayed-scale forward)": (lambda: N.norm_mod(x, w, mod, idx, 0, 1e-5, codes=codes, sf=sf,
                                                                      slot=sp), S * D * (2 + 0.5625)),
        "norm_mod bf16 + amax (first forward)": (lambda: N.norm_mod(x, w, mod, idx, 0, 1e-5, out=yb, slot=sp),
                                                 S * D * 4),
        "nvfp4_quant [S, 5120]": (lambda: N.nvfp4_quant(x, codes, sf, g_ptr=sp + 4, amax_ptr=sp), S * D * 2.5625),
        "qknorm_rope (q, k in place)": (lambda: N.qknorm_rope(qkv[:, :HD], qkv[:, HD:2 * HD], 3 * HD, S, H, 128, qw,
                                                             kw, rope, 1e-5), S * 2 * HD * 4),
    }
    flush = Flush()
    for name, (run, nbytes) in cases.items():
        ms = time_launches(run, reps=a.steps, warmup=max(a.warmup, 1), flush=flush)
        gbs = nbytes / ms / 1e6
        print(json.dumps({"micro": name, "S": S, "us": round(ms * 1e3, 1), "gb_s": round(gbs, 1),
                          "frac": round(gbs / hbm, 4), "peak_note": f"{src} copy bandwidth {hbm} GB/s"}), flush=True)
    print(json.dumps({"device_status": N.device_status()}), flush=True)


# ------------------------------------------------------------------------------------------------ GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq", type=int, default=SEQ)
    ap.add_argument("--layers", type=int, default=50)
    ap.add_argument("--cpu-rows", type=int, default=512)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-full-block", action="store_true",
                    help="also time one whole S-token block on the host CPU (minutes), beside the per-row sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the parity probe and the config sweeps")
    ap.add_argument("--micro", choices=["attn", "gemm", "elem"],
                    help="time one op alone (BASELINE configs 1 / 2; elem: the HBM-bound kernels)")
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--part-sender", choices=["copy", "push", "auto"], default=None,
                    help="Ulysses: how the qkv parts but the last are sent while the GEMM runs (engine default)")
    ap.add_argument("--copy-streams", type=int, default=None,
                    help="Ulysses: side streams for the qkv exchange copies (engine default)")
    ap.add_argument("--qkv-parts", type=int, default=None,
                    help="Ulysses: row parts of the qkv GEMM whose exchange overlaps the next part (engine default)")
    ap.add_argument("--mnk", default="37760,15360,5120", help="--micro gemm: M,N,K")
    ap.add_argument("--epi", default="store", choices=["store", "gate", "act_q"])
    ap.add_argument("--sparse", action="store_true",
                    help="block-sparse attention (config 4's second run: 25%% of 128x128 tiles per query row, "
                         "diagonal and text tiles kept, seed 4)")
    a = ap.parse_args()
    if a.impl == "reference":
        return reference_arm(a)
    if a.micro:
        return micro(a)

    from tfvideo import minimax_h3 as M
    from tfvideo import native as N
    from tfvideo.profiling import StageTimer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
        group = torch.distributed.group.WORLD
    cfg = M.Config(layers=a.layers, dim=5120, heads=40, head_dim=128, ffn=20480, act="gelu", t_dim=8)
    S = a.seq
    n = S // world
    t0 = n * rank
    eng = M.MiniMaxH3Engine.synthetic(cfg, seed=1, device="cuda", group=group)
    if a.sparse:
        from tfvideo import attention as A
        eng.attn_mask = A.TileMask.block_sparse(S)
    if a.qkv_parts:
        eng.qkv_parts = a.qkv_parts
    if a.copy_streams:
        eng.copy_streams = a.copy_streams
    if a.part_sender:
        eng.part_sender = a.part_sender
    x0 = activations(S, cfg.dim)[t0:t0 + n].cuda()
    t_emb = torch.randn(2, cfg.t_dim, generator=torch.Generator().manual_seed(3)).cuda()
    segs = mod_segments(S)
    rope = rope_3d(S).cuda()
    x = torch.empty_like(x0)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    def step():
        x.copy_(x0)
        eng.forward(x, t_emb, segs, rope)

    for _ in range(max(a.warmup, 1)):
        step()
    torch.cuda.synchronize()
    assert N.device_status() == 0
    timer = StageTimer()
    eng.timer = timer
    barrier()
    torch.cuda.synchronize()
    launches0 = N.LAUNCHES
    with Clocks(local) as clocks:
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        for _ in range(a.steps):
            step()
        en.record()
        torch.cuda.synchronize()
        barrier()
    launches = N.LAUNCHES - launches0
    eng.timer = None
    ms = st.elapsed_time(en) / a.steps
    stages = timer.summary()
    stage_ranks = None
    if world > 1:   # every rank's own stage times: the exchange waits show which rank the others wait for
        mine = {k: round(v["ms"] / a.steps, 3) for k, v in stages.items()}
        every = [None] * world
        torch.distributed.all_gather_object(every, mine)
        stage_ranks = {k: [r.get(k) for r in every] for k in mine}
    status = N.device_status()
    finite = bool(torch.isfinite(x).all())
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())

    # ---- e2e through the public API: EngineBlock per block, host inputs and outputs
    e2e = None
    if not a.no_e2e:
        blocks = [M.EngineBlock(eng, i) for i in range(len(eng.blocks))]
        xh = x0.cpu().pin_memory()
        rh = rope.cpu().pin_memory()
        th = t_emb.cpu().pin_memory()
        out_h = torch.empty_like(xh).pin_memory()
        xd, rd, td = torch.empty_like(x0), torch.empty_like(rope), torch.empty_like(t_emb)

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            rd.copy_(rh, non_blocking=True)
            td.copy_(th, non_blocking=True)
            sg = [tuple(s) for s in segs]           # a fresh segment list: the row index is rebuilt and uploaded
            h = xd
            for blk in blocks:
                h = blk(h, td, sg, rd)
            out_h.copy_(h, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        te = torch.tensor([e0.elapsed_time(e1) / a.steps], device="cuda")
        if world > 1:
            torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        h2d = xh.numel() * 2 + rh.numel() * 4 + th.numel() * 4 + S * 4
        e2e = {"value": float(te.item()) / 1e3, "unit": "s/step", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(out_h.numel() * 2)}

    # ---- roofline of the dominant kernel (attention at this shape) and the GEMMs
    pk, src = peaks()
    sustained = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    per_block = {k: v["ms"] / v["calls"] for k, v in stages.items()}
    Hl = cfg.heads // world
    density = eng.attn_mask.density if eng.attn_mask is not None else 1.0
    attn_flops = 4.0 * S * S * Hl * cfg.head_dim * density   # kept tiles only under the block-sparse mask
    attn_ms = per_block.get("attention", float("nan"))
    gemm_flops = {"gemm_qkv": 2.0 * n * 3 * cfg.inner * cfg.dim, "gemm_out+gate": 2.0 * n * cfg.dim * cfg.inner,
                  "gemm_fc1+act+quant": 2.0 * n * cfg.ffn * cfg.dim, "gemm_fc2+gate": 2.0 * n * cfg.dim * cfg.ffn}
    gemm_ms = sum(per_block.get(k, 0.0) for k in gemm_flops)
    gemm_tflops = sum(gemm_flops.values()) / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    achieved = attn_flops / (attn_ms * 1e-3) / 1e12
    fp8_peak = 2 * sustained
    roofline = {"kernel": "attn_fp8 (tcgen05 FP8 flash attention incl. its prepare)", "bound": "tensor",
                "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s", "frac": achieved / fp8_peak,
                "frac_nominal": achieved / NOMINAL_TFLOPS["fp8"],
                "traffic": ATTN_DRAM_BYTES_PER_TOKEN_HEAD * S * Hl,
                "traffic_note": "dram read+write per launch: 181.7 MB measured by ncu for one launch at S=8192, H=40, "
                                "scaled by tokens x heads (K/V of a head stay in L2)",
                "peak_note": f"2 x {src} bf16 sustained ({sustained} TF/s): dense FP8 = 2 x bf16 on B200; "
                             f"frac_nominal against the 4.5 PF/s dense FP8 figure",
                "work_per_launch": f"4*S^2*H*Dh*density = {attn_flops:.4g} FLOP (S={S}, H={Hl}, "
                                   f"tile density {density:.4f})",
                "nvfp4_gemm": {"achieved": gemm_tflops, "peak": 4 * sustained, "unit": "TFLOP/s",
                               "frac": (gemm_tflops / (4 * sustained)) if gemm_tflops else None,
                               "frac_nominal": (gemm_tflops / NOMINAL_TFLOPS["nvfp4"]) if gemm_tflops else None,
                               "peak_note": f"4 x {src} bf16 sustained: dense NVFP4 = 4 x bf16 on B200; "
                                            f"frac_nominal against the 9 PF/s dense NVFP4 figure"}}

    eng_parts = eng.qkv_parts
    # ---- single GPU only: parity at the timed shape, the config-1 / config-2 sweeps and the real-H3 block
    parity = configs = None
    if world == 1 and not a.no_extra:
        parity = parity_probe(eng, cfg, x0, t_emb, segs, rope)
        del eng, x, x0
        torch.cuda.empty_cache()
        configs = {"config1_gemm": gemm_sweep(sustained), "config2_attention": attn_sweep(sustained),
                   "h3_real_block": h3_real_block(S)}
        assert N.device_status() == 0

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu:
        r = cpu_step_sample(a.cpu_rows)
        c0 = cpu_block(4096, 4096)
        cpu = {"value": r["value"], "unit": "s/step", "cores": r["cores"], "kind": "port", "extrapolated": True,
               "sample": r["sample"], "sample_seconds": r["sample_s"],
               "config0_block_seconds": c0["seconds"],
               "config0": "one full block, 4,096 tokens, D 5120, 40 x 128 heads, GELU 20480, NVFP4 fake-quant, timed "
                          "outright", **cpu_info()}
        if a.cpu_full_block:   # the sample's check: one whole 37,760-token block (minutes, ~30 GB of host memory)
            full = cpu_block(S, S)
            cpu["config3_full_block_seconds"] = full["seconds"]
            cpu["config3_full_block_x50"] = full["seconds"] * a.layers
    if rank == 0:
        line = {"metric": METRIC, "value": ms / 1e3, "unit": "s/step", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "nvfp4 linears / fp8-e4m3 attention, fp32 accumulate",
                "data": "synthetic (seeded N(0,1) activations with 1% x20 outlier channels; N(0,0.02) weights)",
                "config": {"workload": "config 3/4: 50-block H3-shaped DiT step, 37,760 tokens (512/1680/496/35072), "
                                       "D=5120, 40x128 heads, GELU-tanh FFN 20480, NVFP4 W4A4 + FP8 attention",
                           "global_batch": 1, "seq_len": S, "layers": cfg.layers,
                           "parallelism": ("single GPU" if world == 1 else
                                           f"ulysses sp{world} (token-sharded, qkv exchange in {eng_parts} row parts)"),
                           "attention_mask": (f"block-sparse 128x128 tiles, {density:.4f} kept (seed 4)"
                                              if a.sparse else "dense"),
                           "l2": "inputs larger than L2 (8.9 GB weights + activations per step); sweeps flush L2 "
                                 "before each timed launch"},
                "stages_ms_per_step": {k: round(v["ms"] / a.steps, 3) for k, v in stages.items()},
                "stages_ms_per_step_by_rank": stage_ranks,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clocks.summary(), "device_status": status, "finite": finite, "parity": parity,
                "configs": configs}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
