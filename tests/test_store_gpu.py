"""Checkpoint -> B200 engine conversion and the converted-engine cache (tfvideo/store.py).

A ComfyUI-layout checkpoint (int8 + ConvRot linears and a float one) converts to NVFP4 linears whose codes and
scales equal those quantised from the model-basis weights directly; the converted engine's block matches the oracle
block on the same weights; and an engine saved and loaded back computes the same output bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import ckpt_fixture as F
from helpers import bf16_array, device_ok, need_gpu, to_dev, to_np
from oracle import block as OB
from oracle import ops as OO

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    need_gpu()


@pytest.mark.parametrize("act,ffn", [("gelu", 1024), ("swiglu", 512)])
def test_convert_save_load(tmp_path, monkeypatch, act, ffn):
    from tfvideo import linear as L
    from tfvideo import store
    from tfvideo.source import Checkpoint

    src = tmp_path / "h3.safetensors"
    F.write(src, layers=2, act=act, ffn=ffn)
    eng = store.convert(src, log=lambda *_: None)
    cfg = eng.cfg
    assert (cfg.layers, cfg.dim, cfg.act) == (2, 512, act)
    ck = Checkpoint(src)
    # codes / scales: the conversion is the plain NVFP4 quantisation of the model-basis weight
    w = ck.linear("blocks.1.attn.qkv_proj", "cuda").to(torch.bfloat16)
    direct = L.Nvfp4Linear(w)
    assert torch.equal(eng.blocks[1].lins["qkv"].codes, direct.codes)
    assert torch.equal(eng.blocks[1].lins["qkv"].sf, direct.sf)

    # the converted engine's first block against the oracle block on the same (model-basis, bf16) weights
    S, rot = 256, 128
    shape = OB.BlockShape(dim=cfg.dim, heads=cfg.heads, head_dim=cfg.head_dim, ffn=cfg.ffn, act=act, rot_dim=rot)
    wq = {n: OO.bf16_round(ck.linear(f"blocks.0.{src_name}", "cpu").float().numpy()) for n, src_name in
          (("qkv", "attn.qkv_proj"), ("out", "attn.out_proj"), ("fc1", "mlp.fc1"), ("fc2", "mlp.fc2"))}
    sm = {k: v.numpy() for k, v in ck.small(0, "cpu").items()}
    p = OB.BlockParams(w=wq, **sm)
    x = bf16_array((S, cfg.dim), 3)
    t_emb = np.random.RandomState(4).randn(2, cfg.t_dim).astype(np.float32)
    segs = [(0, 64, 0), (64, S, 3)]
    rope = OB.rope_table(S, rot)
    rope_t = to_dev(rope, torch.float32).reshape(1, S, 1, rot // 2, 2, 2)
    from tfvideo import minimax_h3 as M

    out = to_np(M.EngineBlock(eng, 0)(to_dev(x), to_dev(t_emb, torch.float32), segs, rope_t))
    ref = OB.block_forward(shape, p, x, t_emb, segs, rope, linears="bf16", attn="sdpa")
    assert OO.cosine(out, ref) >= 0.998

    # save / load round trip, and the cache
    monkeypatch.setenv("TFVIDEO_CACHE", str(tmp_path / "cache"))
    path = tmp_path / "engine.safetensors"
    store.save(eng, path)
    back = store.load(path)
    xt = to_dev(x)
    eng.end_run()                                                    # both engines start a new run: dynamic scales
    a = eng.forward(xt.clone(), to_dev(t_emb, torch.float32), segs, rope_t)
    b = back.forward(xt.clone(), to_dev(t_emb, torch.float32), segs, rope_t)
    assert torch.equal(a, b)
    e1 = store.load_or_convert(src, log=lambda *_: None)            # converts and caches
    e2 = store.load_or_convert(src, log=lambda *_: None)            # loads the cache
    assert torch.equal(e1.blocks[1].lins["fc2"].codes, e2.blocks[1].lins["fc2"].codes)
    with pytest.raises(ValueError):
        store.convert(src, spec="int8")
    device_ok()


def test_lora_merge_reconverts_and_caches_per_set(tmp_path, monkeypatch):
    """store.load_or_convert with ``merge``: only the linears the merge function patches change, each equal to the
    NVFP4 quantisation of the patched model-basis weight; the LoRA set gets its own cache file and loads back from it;
    an engine swapped to the merged blocks computes what the merged engine computes."""

    from tfvideo import linear as L
    from tfvideo import minimax_h3 as M
    from tfvideo import store
    from tfvideo.source import Checkpoint

    src = tmp_path / "h3.safetensors"
    F.write(src, layers=2)
    cache = tmp_path / "cache"
    monkeypatch.setenv("TFVIDEO_CACHE", str(cache))
    quiet = lambda *_: None                                           # noqa: E731
    base = store.load_or_convert(src, log=quiet)
    delta = 0.01
    seen = []

    def merge(name, w):
        seen.append(name)
        return w + delta if name == "blocks.1.mlp.fc1" else None

    sig = "abc123@0.7500"
    lora = store.load_or_convert(src, log=quiet, merge=merge, merge_sig=sig)
    assert len(seen) == 8 and lora.lora_sig == sig
    w = Checkpoint(src).linear("blocks.1.mlp.fc1", "cuda")
    direct = L.Nvfp4Linear((w + delta).to(torch.bfloat16))
    assert torch.equal(lora.blocks[1].lins["fc1"].codes, direct.codes)
    assert torch.equal(lora.blocks[1].lins["fc1"].sf, direct.sf)
    assert not torch.equal(lora.blocks[1].lins["fc1"].codes, base.blocks[1].lins["fc1"].codes)
    for i, name in ((0, "fc1"), (1, "qkv"), (1, "fc2")):
        assert torch.equal(lora.blocks[i].lins[name].codes, base.blocks[i].lins[name].codes)
    files = sorted(p.name for p in cache.iterdir())
    assert len(files) == 2 and sum(".lora." in f for f in files) == 1
    seen.clear()
    again = store.load_or_convert(src, log=quiet, merge=merge, merge_sig=sig)   # from the cache: no merge calls
    assert seen == [] and torch.equal(again.blocks[1].lins["fc1"].codes, direct.codes)

    S, rot = 128, 128
    x = to_dev(bf16_array((S, base.cfg.dim), 9))
    te = to_dev(np.random.RandomState(4).randn(2, base.cfg.t_dim).astype(np.float32), torch.float32)
    segs = [(0, S, 1)]
    rope_t = to_dev(OB.rope_table(S, rot), torch.float32).reshape(1, S, 1, rot // 2, 2, 2)
    base.replace_blocks(lora.blocks, sig, slots=lora.slots)
    a = M.EngineBlock(base, 0)(x.clone(), te, segs, rope_t)
    lora.end_run()
    b = M.EngineBlock(lora, 0)(x.clone(), te, segs, rope_t)
    assert torch.equal(a, b)
    device_ok()
