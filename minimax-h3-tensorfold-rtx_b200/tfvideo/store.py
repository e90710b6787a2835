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
import re
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


def cache_name(source: str | Path, spec: str, lora_sig: str = "") -> str:
    """File name of a converted engine in the cache: ``<checkpoint stem>.<spec>[.lora].<id>.b200.safetensors``.

    ``id`` digests everything the conversion result depends on -- the checkpoint's resolved path, size and
    modification time, the precision spec, this file format's version and the LoRA set's signature -- so editing the
    checkpoint, changing the spec or the LoRAs, or a new format gives a new file instead of a stale one.  The
    ``b200`` suffix keeps these files apart from the reference's TensorFold caches."""

    st = os.stat(source)
    ident = json.dumps({"path": str(Path(source).resolve()), "size": st.st_size, "mtime_ns": st.st_mtime_ns,
                        "spec": spec, "format": FORMAT, "lora": lora_sig}, sort_keys=True)
    digest = hashlib.blake2b(ident.encode(), digest_size=6).hexdigest()
    parts = [Path(source).stem, re.sub(r"[^A-Za-z0-9]+", "-", spec).strip("-")]
    if lora_sig:
        parts.append("lora")
    return ".".join(parts + [digest, "b200"]) + ".safetensors"


def _check_spec(spec: str) -> None:
    if spec != "nvfp4":
        raise ValueError(f"precision {spec!r} is not converted by the B200 build (it converts to 'nvfp4')")


class _Progress:
    """Logs conversion progress at most every ``every`` seconds (converting 50 blocks takes tens of seconds)."""

    def __init__(self, log, total: int, every: float = 10.0):
        self.log, self.total, self.every = log, total, every
        self.t0 = self.last = time.perf_counter()

    def step(self, done: int) -> None:
        now = time.perf_counter()
        if done == self.total or now - self.last >= self.every:
            self.log(f"[tfvideo] NVFP4 conversion: block {done} of {self.total}, {now - self.t0:.0f} s")
            self.last = now


def _convert_block(src: Checkpoint, i: int, cfg: Config, slots, device, merge) -> tuple[Block, int]:
    """Block i with its four linears read in the model's basis, LoRA-merged where ``merge`` patches them, and
    quantised to NVFP4 on the GPU.  Returns the block and how many of its linears ``merge`` changed."""

    lins, patched = {}, 0
    for name in LIN_NAMES:
        full = f"blocks.{i}.{SOURCE[name]}"
        w = src.linear(full, device)
        if merge is not None:
            merged = merge(full, w)
            if merged is not None:
                w, patched = merged, patched + 1
        lins[name] = L.Nvfp4Linear(w.to(torch.bfloat16), slots=slots, slot=4 * i + SLOT[name],
                                   interleave16=(name == "fc1" and cfg.act == "swiglu"))
        del w
    return Block(lins, **src.small(i, device)), patched


def convert(source: str | Path, spec: str = "nvfp4", merge=None, device="cuda", log=print,
            attn: str = "auto") -> MiniMaxH3Engine:
    """A B200 engine from a ComfyUI-layout MiniMax H3 checkpoint.  ``merge(name, w)`` returns the LoRA-patched fp32
    weight of block linear ``name`` (e.g. ``blocks.3.mlp.fc1``), or None to keep ``w``."""

    _check_spec(spec)
    src = Checkpoint(source)
    cfg = src.config()
    slots = L.new_slots(4 * cfg.layers, device)
    progress = _Progress(log, cfg.layers)
    blocks, patched = [], 0
    for i in range(cfg.layers):
        block, n = _convert_block(src, i, cfg, slots, device, merge)
        blocks.append(block)
        patched += n
        progress.step(i + 1)
    if merge is not None:
        log(f"[tfvideo] LoRA set applied to {patched} of {4 * cfg.layers} block linears")
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
    """The engine for (checkpoint, spec, LoRA set): read from the cache when converted before, else converted now and
    written to the cache.  A cache file this build cannot read (another format version) is converted again."""

    _check_spec(spec)
    path = cache_dir() / cache_name(source, spec, merge_sig)
    engine = None
    if path.is_file():
        t0 = time.perf_counter()
        try:
            engine = load(path, device, attn)
            log(f"[tfvideo] {path.name}: cached NVFP4 engine read in {time.perf_counter() - t0:.1f} s")
        except ValueError as e:
            log(f"[tfvideo] {path.name}: not usable ({e}); converting again")
    if engine is None:
        log(f"[tfvideo] converting {Path(source).name} to NVFP4{' with its LoRA set' if merge_sig else ''}; "
            f"the result is cached as {path}")
        engine = convert(source, spec, merge, device, log, attn)
        save(engine, path)
    engine.source, engine.lora_sig = str(source), merge_sig
    return engine
