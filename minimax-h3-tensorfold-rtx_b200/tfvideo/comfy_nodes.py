"""ComfyUI's "TensorFold MiniMax H3 Loader" node on B200 (the reference's tfvideo/comfy_nodes.py:1-273).

The node loads a MiniMax H3 DiT checkpoint into a B200 engine (converted to NVFP4 once, cached) and returns ComfyUI's
own MiniMaxH3 MODEL built without blocks, whose ``blocks`` list is the engine's EngineBlocks: model sampling,
sequence packing, conditioning, RoPE tables, the output heads and the VAE latents stay ComfyUI's, so a workflow
swaps one loader node and keeps everything else.  The same node name, display name, inputs and defaults as the
reference, so saved workflows load unchanged.

B200 differences:
  * precision: "nvfp4" is this build's path.  The reference's "int8", "fp8", "nvfp4:edge=2" and "bf16-check" are
    kept in the list (saved workflows carry them) and raise ValueError when chosen.
  * attention: "auto" / "fp8" (libh3b200's FP8 kernel), "sdpa" / "cudnn" (PyTorch's); "fp4" and "int8" raise.
  * every block stays resident in HBM, so there is no per-sequence memory plan and no block streaming; at the end of
    a sampling run (ComfyUI's ON_CLEANUP) the activation buffers are released and the scales reset.
LoRAs go through ComfyUI's LoRA nodes as in the reference: for an engine MODEL, ``load_lora_for_models`` hands the
block-linear patches to the engine (merged into the source weights with ComfyUI's ``calculate_weight`` and
re-quantised, cached per LoRA set) and everything else to ComfyUI's patcher.

ComfyUI modules are imported inside the functions that need them; importing this module needs only torch.
"""

from __future__ import annotations

import hashlib
import logging

import torch

PRECISIONS = ["nvfp4", "int8", "nvfp4:edge=2", "fp8", "bf16-check"]
ATTENTION = ["auto", "fp4", "fp8", "int8", "sdpa", "cudnn"]
SUPPORTED_PRECISIONS = ("nvfp4",)
LORA_KEY = "tfvideo_loras"          # transformer_options: [(fingerprint, {block key: adapter}, strength), ...]
_ENGINE: dict = {}                  # the one resident engine: {"key": (path, spec), "engine": MiniMaxH3Engine}


def check_choices(precision: str, attention: str) -> str:
    """The engine spec for a node's (precision, attention), or ValueError naming what this build cannot run."""

    if precision not in PRECISIONS:
        raise ValueError(f"precision {precision!r}: one of {PRECISIONS}")
    if precision not in SUPPORTED_PRECISIONS:
        raise ValueError(f"precision {precision!r} has no B200 build; use 'nvfp4'")
    from . import attention as A

    A.get(attention)                # raises ValueError for "fp4" / "int8" / unknown names
    return precision


def _engine(path: str, spec: str):
    from . import store

    if _ENGINE.get("key") == (path, spec):
        return _ENGINE["engine"]
    _ENGINE.clear()
    torch.cuda.empty_cache()
    engine = store.load_or_convert(path, spec, device="cuda", log=logging.info)
    engine.on_forward = _on_forward
    _ENGINE.update(key=(path, spec), engine=engine)
    return engine


# ------------------------------------------------------------------------------------------------ LoRA
def fingerprint(part: dict) -> str:
    """A short signature of a LoRA's block-linear patches: their keys, shapes and first values."""

    h = hashlib.sha1()
    for k in sorted(part):
        h.update(k.encode())
        for t in getattr(part[k], "weights", ()):
            if torch.is_tensor(t):
                h.update(str(tuple(t.shape)).encode())
                h.update(t.flatten()[:64].float().cpu().numpy().tobytes())
    return h.hexdigest()[:16]


def lora_signature(loras) -> str:
    return "|".join(f"{fp}x{strength:.4f}" for fp, _, strength in loras)


def lora_patches(loras) -> dict[str, list]:
    """{block linear name (e.g. ``blocks.3.mlp.fc1``): ComfyUI patch list} from the transformer_options LoRA set."""

    patches: dict[str, list] = {}
    for _, part, strength in loras:
        for key, adapter in part.items():
            name = key[len("diffusion_model."):-len(".weight")]
            patches.setdefault(name, []).append((strength, adapter, 1.0, None, None))
    return patches


def _on_forward(engine, S, transformer_options):
    """Block 0 of each forward: bring the engine's weights in line with the MODEL's LoRA set."""

    _sync_loras(engine, transformer_options)


def _sync_loras(engine, transformer_options):
    loras = (transformer_options or {}).get(LORA_KEY, [])
    sig = lora_signature(loras)
    if sig == engine.lora_sig:
        return
    import comfy.lora

    from . import store

    patches = lora_patches(loras)

    def merge(name, w):
        p = patches.get(name)
        return comfy.lora.calculate_weight(p, w, name) if p else None

    logging.info(f"[tfvideo] LoRA set changed ({len(loras)} LoRA(s)): "
                 f"{'re-merging' if loras else 'restoring base weights'}")
    engine.release_vram()
    new = store.load_or_convert(engine.source, engine.kind, device="cuda", log=logging.info,
                                merge=merge if loras else None, merge_sig=sig)
    engine.replace_blocks(new.blocks, sig, slots=new.slots)


def block_key_map(layers: int) -> dict[str, str]:
    """ComfyUI LoRA key aliases of the block linears -> their model keys (``diffusion_model.blocks.i.<lin>.weight``)."""

    from .minimax_h3 import SOURCE

    key_map = {}
    for i in range(layers):
        for src in SOURCE.values():
            k = f"diffusion_model.blocks.{i}.{src}.weight"
            key_map[k[:-len(".weight")]] = k
            key_map["lora_unet_blocks_{}_{}".format(i, src.replace(".", "_"))] = k
    return key_map


def _install_lora_hook():
    import comfy.sd

    original = comfy.sd.load_lora_for_models
    if getattr(original, "_tfvideo", False):
        return

    def load_lora_for_models(model, clip, lora, strength_model, strength_clip, lora_metadata=None):
        engine = getattr(getattr(getattr(model, "model", None), "diffusion_model", None), "tfvideo_engine", None)
        if engine is None or strength_model == 0:
            return original(model, clip, lora, strength_model, strength_clip, lora_metadata)
        import comfy.lora
        import comfy.lora_convert

        key_map = comfy.lora.model_lora_keys_unet(model.model, {})
        blocks = block_key_map(len(engine.blocks))
        key_map.update(blocks)
        block_keys = set(blocks.values())
        loaded = comfy.lora.load_lora(comfy.lora_convert.convert_lora(lora), key_map)
        part = {k: v for k, v in loaded.items() if k in block_keys}
        rest = {k: v for k, v in loaded.items() if k not in block_keys}
        new_model = model.clone()
        new_model.add_patches(rest, strength_model)
        to = dict(new_model.model_options.get("transformer_options", {}))
        to[LORA_KEY] = list(to.get(LORA_KEY, [])) + [(fingerprint(part), part, float(strength_model))]
        new_model.model_options["transformer_options"] = to
        if lora_metadata:
            new_model.set_attachments("lora_metadata", lora_metadata)
        logging.info(f"[tfvideo] LoRA: {len(part)} block linears to the engine, {len(rest)} other weights to ComfyUI")
        new_clip = None
        if clip is not None:
            _, new_clip = original(None, clip, lora, 0.0, strength_clip, lora_metadata)
        return new_model, new_clip

    load_lora_for_models._tfvideo = True
    comfy.sd.load_lora_for_models = load_lora_for_models


# ------------------------------------------------------------------------------------------------ the MODEL
def build_model(path: str, engine):
    """ComfyUI's MiniMaxH3 MODEL from the checkpoint's non-block tensors, with the engine's blocks."""

    import comfy.model_detection
    import comfy.model_management as mm
    import comfy.model_patcher
    import comfy.patcher_extension

    from .minimax_h3 import EngineBlock
    from .source import SafeTensors

    f = SafeTensors(path)
    probe = {k: torch.empty(f.shape(k), device="meta") for k in f.keys()}
    prefix = comfy.model_detection.unet_prefix_from_state_dict(probe)
    if not any(k.startswith(prefix) for k in probe):
        prefix = ""
    unet_config = comfy.model_detection.detect_unet_config(probe, prefix)
    if unet_config is None or unet_config.get("image_model") != "minimax_h3":
        raise RuntimeError(f"TensorFold MiniMax H3: {path} is not a MiniMax H3 DiT")
    unet_config["num_layers"] = 0
    sd = {k[len(prefix):]: f.get(k) for k in f.keys()
          if k.startswith(prefix) and not k[len(prefix):].startswith("blocks.")}
    model_config = comfy.model_detection.model_config_from_unet_config(unet_config, sd)
    load_device = mm.get_torch_device()
    model_config.set_inference_dtype(torch.bfloat16, torch.bfloat16, device=load_device)
    model = model_config.get_model(sd, "")
    model.diffusion_model.blocks = torch.nn.ModuleList(EngineBlock(engine, i) for i in range(len(engine.blocks)))
    model.diffusion_model.tfvideo_engine = engine
    engine.comfy_model = model
    patcher = comfy.model_patcher.CoreModelPatcher(model, load_device=load_device,
                                                   offload_device=mm.unet_offload_device())
    model.load_model_weights(sd, "", assign=patcher.is_dynamic())
    patcher.add_wrapper(comfy.patcher_extension.WrappersMP.DIFFUSION_MODEL, _wrapper(model))
    patcher.add_callback_with_key(comfy.patcher_extension.CallbacksMP.ON_CLEANUP, "tfvideo", _cleanup(engine))
    return patcher


def _wrapper(model):
    """Around each diffusion-model call: refuse what the engine cannot honour (scheduled hook weight patches)."""

    def wrapper(executor, x, timestep, context, transformer_options={}, **kwargs):
        patcher = getattr(model, "current_patcher", None)
        if patcher is not None and getattr(patcher, "hook_patches", None):
            raise RuntimeError("TensorFold MiniMax H3: hook (scheduled) weight patches are not supported")
        return executor(x, timestep, context, transformer_options, **kwargs)
    return wrapper


def _cleanup(engine):
    """End of a sampling run (ComfyUI's ON_CLEANUP): release the activation buffers, reset the scales."""

    def cleanup(patcher):
        engine.release_vram()
        engine.end_run()
    return cleanup


def _model_files() -> list[str]:
    import folder_paths

    return [n for n in folder_paths.get_filename_list("diffusion_models") if n.endswith(".safetensors")]


class TFMiniMaxH3Loader:
    """Load a MiniMax H3 DiT into the B200 engine (converted to NVFP4 once, cached)."""

    @classmethod
    def INPUT_TYPES(cls):
        files = _model_files()
        default = next((f for f in files if "minimax_h3" in f), files[0] if files else "")
        return {"required": {"unet_name": (files, {"default": default}),
                             "precision": (PRECISIONS, {"default": "nvfp4"}),
                             "attention": (ATTENTION, {"default": "auto"})}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = "TensorFold"

    def load(self, unet_name: str, precision: str, attention: str = "auto"):
        import folder_paths

        from . import attention as A

        spec = check_choices(precision, attention)
        _install_lora_hook()
        path = folder_paths.get_full_path_or_raise("diffusion_models", unet_name)
        engine = _engine(path, spec)
        engine.attn, engine.attn_name = A.get(attention), attention
        logging.info(f"[tfvideo] MiniMax H3 engine ready: {spec}, attention {attention}, "
                     f"{engine.nbytes() / 2**30:.2f} GiB of block weights")
        return (build_model(path, engine),)


NODE_CLASS_MAPPINGS = {"TFMiniMaxH3Loader": TFMiniMaxH3Loader}
NODE_DISPLAY_NAME_MAPPINGS = {"TFMiniMaxH3Loader": "TensorFold MiniMax H3 Loader"}
