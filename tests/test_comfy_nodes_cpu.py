"""The ComfyUI loader node (tfvideo/comfy_nodes.py) against a stub ComfyUI, on the CPU.

ComfyUI is not installed in this image; the stubs below provide the functions and classes the node calls, with the
signatures of ComfyUI's own.  Checked: the node's identity, inputs and defaults (reference comfy_nodes.py:242-273);
the precision / attention choices this build runs; the LoRA routing (block linears to the engine, the rest to
ComfyUI's patcher, reference comfy_nodes.py:125-166) and the engine-side re-merge at the next forward; and the MODEL
assembly on a real ComfyUI-layout checkpoint file: ComfyUI's model built with no blocks from the non-block tensors,
its block list replaced by EngineBlocks, the hook-patch guard and the end-of-run callback.
"""

from __future__ import annotations

import sys
import types

import pytest
import torch

import ckpt_fixture as F


@pytest.fixture()
def stub(monkeypatch):
    """Stub ComfyUI modules; ``rec`` records what the node did with them."""

    rec = {}
    fp = types.ModuleType("folder_paths")
    fp.get_filename_list = lambda kind: ["flux.safetensors", "minimax_h3_t2v.safetensors", "notes.txt"]
    fp.get_full_path_or_raise = lambda kind, name: f"/models/{kind}/{name}"
    comfy = types.ModuleType("comfy")
    mods = {m: types.ModuleType(f"comfy.{m}") for m in ("sd", "lora", "lora_convert", "model_detection",
                                                         "model_management", "model_patcher", "patcher_extension")}

    def stock_load_lora(model, clip, lora_sd, strength_model, strength_clip, lora_metadata=None):
        rec["stock"] = (model, clip, strength_model, strength_clip)
        return model, clip

    mods["sd"].load_lora_for_models = stock_load_lora
    mods["lora"].model_lora_keys_unet = lambda model, key_map: {
        "diffusion_model.token_refiner.w": "diffusion_model.token_refiner.w.weight"}
    mods["lora"].load_lora = lambda lora_sd, key_map: {key_map[k]: ("adapter", k) for k in lora_sd if k in key_map}

    def calculate_weight(patches, w, name):
        rec.setdefault("calculated", []).append((name, len(patches)))
        return w + 1.0

    mods["lora"].calculate_weight = calculate_weight
    mods["lora_convert"].convert_lora = lambda x: x

    md = mods["model_detection"]
    md.unet_prefix_from_state_dict = lambda sd: "model.diffusion_model."
    md.detect_unet_config = lambda sd, prefix: {"image_model": "minimax_h3", "num_layers": 2}

    class Model:
        def __init__(self, state):
            self.diffusion_model = torch.nn.Module()
            self.diffusion_model.blocks = torch.nn.ModuleList()
            rec["get_model_state"] = sorted(state)

        def load_model_weights(self, sd, prefix, assign=False):
            rec["loaded"] = (sorted(sd), prefix, assign)

    class ModelConfig:
        def __init__(self, cfg, state):
            rec["unet_config"] = cfg

        def set_inference_dtype(self, dtype, manual_cast, device=None):
            rec["dtype"] = dtype

        def get_model(self, state, prefix):
            return Model(state)

    md.model_config_from_unet_config = ModelConfig
    mods["model_management"].get_torch_device = lambda: torch.device("cpu")
    mods["model_management"].unet_offload_device = lambda: torch.device("cpu")

    class CoreModelPatcher:
        def __init__(self, model, load_device, offload_device):
            self.model, self.wrappers, self.callbacks = model, {}, {}

        def is_dynamic(self):
            return False

        def add_wrapper(self, kind, fn):
            self.wrappers[kind] = fn

        def add_callback_with_key(self, kind, key, fn):
            self.callbacks[(kind, key)] = fn

    mods["model_patcher"].CoreModelPatcher = CoreModelPatcher
    mods["patcher_extension"].WrappersMP = types.SimpleNamespace(DIFFUSION_MODEL="diffusion_model")
    mods["patcher_extension"].CallbacksMP = types.SimpleNamespace(ON_CLEANUP="on_cleanup")
    for name, m in mods.items():
        setattr(comfy, name, m)
        monkeypatch.setitem(sys.modules, f"comfy.{name}", m)
    monkeypatch.setitem(sys.modules, "comfy", comfy)
    monkeypatch.setitem(sys.modules, "folder_paths", fp)
    return rec


class FakeEngine:
    """What the node and EngineBlock read from an engine, without a GPU."""

    def __init__(self, layers=2):
        from tfvideo import minimax_h3 as M

        self.cfg = M.Config(layers=layers, dim=512, heads=4, head_dim=128, ffn=1024, act="gelu")
        self.blocks = [object()] * layers
        self.lora_sig, self.source, self.kind = "", "/models/h3.safetensors", "nvfp4"
        self.calls = []

    def release_vram(self):
        self.calls.append("release_vram")

    def end_run(self):
        self.calls.append("end_run")

    def replace_blocks(self, blocks, sig, slots=None):
        self.calls.append(("replace_blocks", sig))
        self.lora_sig = sig


def test_node_identity_and_inputs(stub):
    from tfvideo import comfy_nodes as C

    assert C.NODE_CLASS_MAPPINGS == {"TFMiniMaxH3Loader": C.TFMiniMaxH3Loader}
    assert C.NODE_DISPLAY_NAME_MAPPINGS == {"TFMiniMaxH3Loader": "TensorFold MiniMax H3 Loader"}
    req = C.TFMiniMaxH3Loader.INPUT_TYPES()["required"]
    assert req["unet_name"] == (["flux.safetensors", "minimax_h3_t2v.safetensors"],
                                {"default": "minimax_h3_t2v.safetensors"})
    assert req["precision"] == (["nvfp4", "int8", "nvfp4:edge=2", "fp8", "bf16-check"], {"default": "nvfp4"})
    assert req["attention"] == (["auto", "fp4", "fp8", "int8", "sdpa", "cudnn"], {"default": "auto"})
    assert (C.TFMiniMaxH3Loader.RETURN_TYPES, C.TFMiniMaxH3Loader.FUNCTION) == (("MODEL",), "load")
    assert C.TFMiniMaxH3Loader.CATEGORY == "TensorFold"


def test_choices_this_build_runs():
    from tfvideo import comfy_nodes as C

    for att in ("auto", "fp8", "sdpa", "cudnn"):
        assert C.check_choices("nvfp4", att) == "nvfp4"
    for prec in ("int8", "nvfp4:edge=2", "fp8", "bf16-check", "bogus"):
        with pytest.raises(ValueError):
            C.check_choices(prec, "auto")
    for att in ("fp4", "int8", "bogus"):
        with pytest.raises(ValueError):
            C.check_choices("nvfp4", att)


def test_lora_routing_and_engine_sync(stub, monkeypatch):
    from tfvideo import comfy_nodes as C
    from tfvideo import store

    B = C.LoraBridge
    aliases = B.block_aliases(2)
    assert len(set(aliases.values())) == 8 and len(aliases) == 16
    assert aliases["lora_unet_blocks_1_mlp_fc2"] == "diffusion_model.blocks.1.mlp.fc2.weight"
    assert B.linear_name("diffusion_model.blocks.1.mlp.fc2.weight") == "blocks.1.mlp.fc2"

    engine = FakeEngine()

    class Patcher:
        def __init__(self):
            self.model = types.SimpleNamespace(diffusion_model=types.SimpleNamespace(tfvideo_engine=engine))
            self.model_options = {"transformer_options": {}}
            self.patches = None

        def clone(self):
            c = Patcher()
            c.model = self.model
            c.model_options = {"transformer_options": dict(self.model_options["transformer_options"])}
            return c

        def add_patches(self, patches, strength):
            self.patches = (patches, strength)

    B.install()
    B.install()                                                    # idempotent
    import comfy.sd

    assert getattr(comfy.sd.load_lora_for_models, "tfvideo_bridge", False)
    lora_sd = {"diffusion_model.blocks.0.attn.qkv_proj": 1, "lora_unet_blocks_1_mlp_fc1": 2,
               "diffusion_model.token_refiner.w": 3}
    m1, _ = comfy.sd.load_lora_for_models(Patcher(), None, lora_sd, 0.75, 1.0)
    entries = m1.model_options["transformer_options"][B.OPTION]
    assert len(entries) == 1 and entries[0].strength == 0.75
    assert set(entries[0].adapters) == {"diffusion_model.blocks.0.attn.qkv_proj.weight",
                                        "diffusion_model.blocks.1.mlp.fc1.weight"}
    assert set(m1.patches[0]) == {"diffusion_model.token_refiner.w.weight"} and m1.patches[1] == 0.75
    m2, _ = comfy.sd.load_lora_for_models(m1, None, {"lora_unet_blocks_1_mlp_fc1": 4}, 0.5, 1.0)
    entries2 = m2.model_options["transformer_options"][B.OPTION]
    assert [e.strength for e in entries2] == [0.75, 0.5]           # appended in order; m1 keeps its own set
    assert len(m1.model_options["transformer_options"][B.OPTION]) == 1
    lists = B.patch_lists(entries2)
    assert set(lists) == {"blocks.0.attn.qkv_proj", "blocks.1.mlp.fc1"} and len(lists["blocks.1.mlp.fc1"]) == 2
    sig = B.signature(entries2)
    assert sig.endswith("@0.5000") and sig != B.signature(entries)

    # not an engine MODEL, or strength 0: ComfyUI's own path
    plain = types.SimpleNamespace(model=types.SimpleNamespace(diffusion_model=types.SimpleNamespace()))
    comfy.sd.load_lora_for_models(plain, None, lora_sd, 1.0, 1.0)
    assert stub["stock"][0] is plain

    # the engine side: at the next forward the engine re-converts with ComfyUI's calculate_weight applied
    seen = {}

    def fake_load_or_convert(source, spec, device="cuda", log=print, merge=None, merge_sig="", attn="auto"):
        seen.update(source=source, spec=spec, merge_sig=merge_sig)
        if merge is not None:
            w = torch.zeros(2, 2)
            seen["merged"] = {n: merge(n, w) for n in ("blocks.1.mlp.fc1", "blocks.0.mlp.fc2")}
        return types.SimpleNamespace(blocks=["new"] * 2, slots=None)

    monkeypatch.setattr(store, "load_or_convert", fake_load_or_convert)
    assert C.on_forward(engine, 64, m2.model_options["transformer_options"]) is None
    assert engine.lora_sig == sig and seen["spec"] == "nvfp4" and seen["merge_sig"] == sig
    assert torch.equal(seen["merged"]["blocks.1.mlp.fc1"], torch.ones(2, 2))
    assert seen["merged"]["blocks.0.mlp.fc2"] is None              # no patch for that linear
    assert stub["calculated"] == [("blocks.1.mlp.fc1", 2)]
    assert B.sync(engine, m2.model_options["transformer_options"]) is False     # same set: nothing to do
    assert B.sync(engine, {}) is True and engine.lora_sig == ""                 # LoRAs removed: base weights


def test_model_shell_swaps_in_engine_blocks(stub, tmp_path):
    from tfvideo import comfy_nodes as C
    from tfvideo import minimax_h3 as M

    path = tmp_path / "h3.safetensors"
    F.write(path, layers=2)
    engine = FakeEngine(layers=2)
    patcher = C.ModelShell(str(path)).patcher(engine)
    inner = patcher.model.diffusion_model
    assert [type(b) for b in inner.blocks] == [M.EngineBlock, M.EngineBlock]
    assert [b.i for b in inner.blocks] == [0, 1] and inner.tfvideo_engine is engine
    assert engine.comfy_model is patcher.model
    assert stub["unet_config"]["num_layers"] == 0 and stub["dtype"] == torch.bfloat16
    assert stub["get_model_state"] == ["video_patch_proj.weight"]            # non-block tensors, prefix removed
    assert stub["loaded"] == (["video_patch_proj.weight"], "", False)
    facade = inner.blocks[1].attn
    assert (facade.heads, facade.head_dim) == (4, 128)

    wrapper = patcher.wrappers["diffusion_model"]
    assert wrapper(lambda x, t, c, o, **kw: "ran", 1, 2, 3, {}) == "ran"
    patcher.model.current_patcher = types.SimpleNamespace(hook_patches={"k": 1})
    with pytest.raises(RuntimeError, match="hook"):
        wrapper(lambda *a, **kw: "ran", 1, 2, 3, {})
    patcher.callbacks[("on_cleanup", "tfvideo")](patcher)
    assert engine.calls == ["release_vram", "end_run"]


def test_model_shell_rejects_other_models(stub, tmp_path):
    import comfy.model_detection as md

    from tfvideo import comfy_nodes as C

    path = tmp_path / "other.safetensors"
    F.write(path, layers=1)
    md.detect_unet_config = lambda sd, prefix: {"image_model": "flux"}
    with pytest.raises(RuntimeError, match="not a MiniMax H3"):
        C.ModelShell(str(path)).patcher(FakeEngine(layers=1))
