"""The ComfyUI loader node (tfvideo/comfy_nodes.py) against a stub ComfyUI: node identity and inputs as in the
reference (comfy_nodes.py:242-273), the precision / attention choices this build runs, and the LoRA routing (block
linears to the engine, the rest to ComfyUI's patcher; comfy_nodes.py:131-168).  ComfyUI itself is not installed here;
the stub provides only the functions the node calls."""

from __future__ import annotations

import sys
import types

import pytest
import torch


@pytest.fixture()
def comfy_stub(monkeypatch):
    fp = types.ModuleType("folder_paths")
    fp.get_filename_list = lambda kind: ["flux.safetensors", "minimax_h3_t2v.safetensors", "notes.txt"]
    fp.get_full_path_or_raise = lambda kind, name: f"/models/{kind}/{name}"
    comfy = types.ModuleType("comfy")
    sd, lora, lora_convert = (types.ModuleType(f"comfy.{m}") for m in ("sd", "lora", "lora_convert"))
    calls = {}

    def original(model, clip, lora_sd, strength_model, strength_clip, lora_metadata=None):
        calls["original"] = (model, clip, strength_model, strength_clip)
        return model, clip

    sd.load_lora_for_models = original
    lora.model_lora_keys_unet = lambda model, key_map: {"diffusion_model.token_refiner.w": "diffusion_model.token_refiner.w.weight"}
    lora.load_lora = lambda lora_sd, key_map: {key_map[k]: ("adapter", k) for k in lora_sd if k in key_map}
    lora.calculate_weight = lambda patches, w, name: w + 1.0
    lora_convert.convert_lora = lambda x: x
    comfy.sd, comfy.lora, comfy.lora_convert = sd, lora, lora_convert
    for name, mod in {"folder_paths": fp, "comfy": comfy, "comfy.sd": sd, "comfy.lora": lora,
                      "comfy.lora_convert": lora_convert}.items():
        monkeypatch.setitem(sys.modules, name, mod)
    return calls


def test_node_identity_and_inputs(comfy_stub):
    from tfvideo import comfy_nodes as C

    assert C.NODE_CLASS_MAPPINGS == {"TFMiniMaxH3Loader": C.TFMiniMaxH3Loader}
    assert C.NODE_DISPLAY_NAME_MAPPINGS == {"TFMiniMaxH3Loader": "TensorFold MiniMax H3 Loader"}
    req = C.TFMiniMaxH3Loader.INPUT_TYPES()["required"]
    assert req["unet_name"] == (["flux.safetensors", "minimax_h3_t2v.safetensors"],
                                {"default": "minimax_h3_t2v.safetensors"})
    assert req["precision"] == (["nvfp4", "int8", "nvfp4:edge=2", "fp8", "bf16-check"], {"default": "nvfp4"})
    assert req["attention"] == (["auto", "fp4", "fp8", "int8", "sdpa", "cudnn"], {"default": "auto"})
    assert (C.TFMiniMaxH3Loader.RETURN_TYPES, C.TFMiniMaxH3Loader.FUNCTION) == (("MODEL",), "load")


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


def test_lora_routing_and_signatures(comfy_stub):
    from tfvideo import comfy_nodes as C

    km = C.block_key_map(2)
    assert len(set(km.values())) == 8 and len(km) == 16
    assert km["lora_unet_blocks_1_mlp_fc2"] == "diffusion_model.blocks.1.mlp.fc2.weight"

    class Model:
        def __init__(self):
            self.model = types.SimpleNamespace(diffusion_model=types.SimpleNamespace(
                tfvideo_engine=types.SimpleNamespace(blocks=[0, 1])))
            self.model_options = {"transformer_options": {}}
            self.patches = None

        def clone(self):
            m = Model()
            m.model = self.model
            return m

        def add_patches(self, patches, strength):
            self.patches = (patches, strength)

    C._install_lora_hook()
    import comfy.sd

    assert getattr(comfy.sd.load_lora_for_models, "_tfvideo", False)
    lora_sd = {"diffusion_model.blocks.0.attn.qkv_proj": 1, "lora_unet_blocks_1_mlp_fc1": 2,
               "diffusion_model.token_refiner.w": 3}
    new_model, _ = comfy.sd.load_lora_for_models(Model(), None, lora_sd, 0.75, 1.0)
    loras = new_model.model_options["transformer_options"][C.LORA_KEY]
    assert len(loras) == 1 and loras[0][2] == 0.75
    assert set(loras[0][1]) == {"diffusion_model.blocks.0.attn.qkv_proj.weight",
                                "diffusion_model.blocks.1.mlp.fc1.weight"}
    assert set(new_model.patches[0]) == {"diffusion_model.token_refiner.w.weight"}
    patches = C.lora_patches(loras)
    assert set(patches) == {"blocks.0.attn.qkv_proj", "blocks.1.mlp.fc1"}
    assert C.lora_signature(loras).endswith("x0.7500")
    plain = types.SimpleNamespace(model=types.SimpleNamespace(diffusion_model=types.SimpleNamespace()))
    comfy.sd.load_lora_for_models(plain, None, lora_sd, 1.0, 1.0)      # not an engine MODEL: ComfyUI's own path
    assert comfy_stub["original"][0] is plain
    _ = torch
