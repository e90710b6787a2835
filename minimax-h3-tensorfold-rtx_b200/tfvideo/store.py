"""Converting a MiniMax H3 checkpoint to a B200 engine, and converted engines on disk (the reference's
tfvideo/store.py:84-207, for the NVFP4 path).

``convert`` reads every block linear in the model's basis (source.Checkpoint undoes ComfyUI's int8 + ConvRot
storage), applies LoRA patches through ``merge`` when given, and quantises to NVFP4 on the GPU with libh3b200's
quantiser (weights: one global scale amax / (6 * 448), e4m3 scale per 16, tiled scale layout for the GEMM).  The
result goes to a cache keyed by the source file's path, size and mtime, the precision spec and the LoRA set's
signature; loading it back reads codes and scales and needs no requantisation.  All blocks stay resident in HBM
(~9-11 GB at H3 size).

Precision specs: ``"nvfp4"``.  The reference's other specs (``int8``, ``fp8``, ``bf16-check``, per-projection
overrides such as ``nvfp4:fc2=fp8,edge=2``) select linears that are not on this build's path and raise ValueError.
"""

from __future__ import annotations

import hashlib
import json
import os
import time
from pathlib import Path

import torch
from safetensors.torch import save_file

from . import linear as L
from .minimax_h3 import LIN_NAMES, SLOT, SOURCE, Block, Config, MiniMaxH3Engine
from .source import SMALL, Checkpoint, SafeTensors

FORMAT = 1


def cache_dir() -> Path:
    base = os.environ.get("TFVIDEO_CACHE") or os.path.join(
        os.environ.get("XDG_CACHE_HOME", os.path.join(str(Path.home()), ".cache")), "tfvideo")
    path = Path(base)
    path.mkdir(parents=True, exist_ok=True)
    return path


def key(source: str | Path, spec: str, merge_sig: str = "") -> str:
    st = os.stat(source)
    raw = f"{Path(source).resolve()}|{st.st_size}|{st.st_mtime_ns}|{spec}|{FORMAT}|b200|{merge_sig}"
    tag = spec.replace(":", "_").replace(",", "_").replace("=", "-") + ("-lora" if merge_sig else "")
    return f"{Path(source).stem}-{tag}-b200-{hashlib.sha1(raw.encode()).hexdigest()[:10]}"


def _check_spec(spec: str) -> None:
    if spec != "nvfp4":
        raise ValueError(f"precision {spec!r}: the B200 build converts to 'nvfp4' only")


def convert(source: str | Path, spec: str = "nvfp4", merge=None, device="cuda", log=print,
            attn: str = "auto") -> MiniMaxH3Engine:
    """``merge(name, w)``: the patched fp32 weight of block linear ``name`` (e.g. ``blocks.3.mlp.fc1``), or None."""

    _check_spec(spec)
    src = Checkpoint(source)
    cfg = src.config()
    slots = L.new_slots(4 * cfg.layers, device)
    blocks, merged, t0 = [], 0, time.perf_counter()
    for i in range(cfg.layers):
        lins = {}
        for name in LIN_NAMES:
            lin_name = f"blocks.{i}.{SOURCE[name]}"
            w = src.linear(lin_name, device)
            if merge is not None:
                patched = merge(lin_name, w)
                if patched is not None:
                    w, merged = patched, merged + 1
            lins[name] = L.Nvfp4Linear(w.to(torch.bfloat16), slots=slots, slot=4 * i + SLOT[name],
                                       interleave16=(name == "fc1" and cfg.act == "swiglu"))
            del w
        blocks.append(Block(lins, **src.small(i, device)))
        if i % 10 == 9:
            log(f"[tfvideo] converted {i + 1}/{cfg.layers} blocks ({time.perf_counter() - t0:.0f} s)")
    if merge is not None:
        log(f"[tfvideo] merged LoRA patches into {merged} block linears")
    return MiniMaxH3Engine(blocks, spec, cfg, device, attn, slots=slots)


def save(engine: MiniMaxH3Engine, path: str | Path) -> None:
    """Write a converted engine: per block its norms and adaLN tensors, per linear its codes, tiled scales and global
    scale (the metadata JSON holds the config and each linear's g / shape)."""

    path = Path(path)
    tensors, lin_meta = {}, {}
    for i, b in enumerate(engine.blocks):
        for small in SMALL:
            tensors[f"{i}.{small}"] = getattr(b, small)
        for name in LIN_NAMES:
            lin = b.lins[name]
            if not isinstance(lin, L.Nvfp4Linear):
                raise ValueError(f"save: block {i} {name} is {type(lin).__name__}, not Nvfp4Linear")
            tensors[f"{i}.{name}.codes"] = lin.codes
            tensors[f"{i}.{name}.sf"] = lin.sf
            lin_meta[f"{i}.{name}"] = {"n": lin.n, "k": lin.k, "g": lin.g, "interleaved": lin.interleaved}
    c = engine.cfg
    meta = {"format": FORMAT, "kind": "nvfp4", "linears": lin_meta,
            "config": {"layers": len(engine.blocks), "dim": c.dim, "heads": c.heads, "head_dim": c.head_dim,
                       "ffn": c.ffn, "eps": c.eps, "qk_eps": c.qk_eps, "act": c.act, "t_dim": c.t_dim}}
    tmp = path.with_suffix(".tmp")
    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()}, str(tmp),
              metadata={"tfvideo_b200": json.dumps(meta)})
    os.replace(tmp, path)


def load(path: str | Path, device="cuda", attn: str = "auto") -> MiniMaxH3Engine:
    f = SafeTensors(path)
    if "tfvideo_b200" not in f.metadata:
        raise ValueError(f"{path}: not a converted B200 engine")
    meta = json.loads(f.metadata["tfvideo_b200"])
    if meta.get("format") != FORMAT:
        raise ValueError(f"{path}: format {meta.get('format')} (this build reads {FORMAT})")
    cfg = Config(**meta["config"])
    slots = L.new_slots(4 * cfg.layers, device)
    blocks = []
    for i in range(cfg.layers):
        lins = {}
        for name in LIN_NAMES:
            m = meta["linears"][f"{i}.{name}"]
            lins[name] = L.Nvfp4Linear.from_quantized(f.get(f"{i}.{name}.codes"), f.get(f"{i}.{name}.sf"), m["g"],
                                                      m["n"], m["k"], m["interleaved"], slots=slots,
                                                      slot=4 * i + SLOT[name])
        blocks.append(Block(lins, **{s: f.get(f"{i}.{s}").to(device=device, dtype=torch.float32) for s in SMALL}))
    return MiniMaxH3Engine(blocks, "nvfp4", cfg, device, attn, slots=slots)


def load_or_convert(source: str | Path, spec: str = "nvfp4", device="cuda", log=print, merge=None,
                    merge_sig: str = "", attn: str = "auto") -> MiniMaxH3Engine:
    _check_spec(spec)
    path = cache_dir() / (key(source, spec, merge_sig) + ".safetensors")
    if path.is_file():
        t0 = time.perf_counter()
        engine = load(path, device, attn)
        log(f"[tfvideo] loaded converted {path.name} in {time.perf_counter() - t0:.1f} s")
    else:
        what = " with LoRA" if merge_sig else ""
        log(f"[tfvideo] converting {Path(source).name} to {spec}{what} (once; cached at {path})")
        engine = convert(source, spec, merge, device, log, attn)
        save(engine, path)
    engine.source, engine.lora_sig = str(source), merge_sig
    return engine
