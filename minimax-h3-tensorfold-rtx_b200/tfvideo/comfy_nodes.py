"""The ComfyUI loader node on B200: "TensorFold MiniMax H3 Loader" (reference: tfvideo/comfy_nodes.py).

What stays ComfyUI's: model sampling, sequence packing, conditioning, RoPE tables, the output heads and the VAE
latents -- its own MiniMaxH3 model object, built here from the checkpoint's non-block tensors.  What the engine takes
over: the 50 DiT blocks, whose slots in that model hold ``EngineBlock`` modules.  A workflow therefore swaps the loader
node and nothing else.  The node keeps the reference's class name, display name, inputs, choice lists and defaults
(comfy_nodes.py:242-273), because saved workflows refer to them.

Pieces, each usable on its own:
  ``EngineCache``   one resident engine per process, keyed by (checkpoint path, precision); NVFP4 conversion happens
                    once and is cached on disk (tfvideo/store.py).
  ``LoraBridge``    wraps ``comfy.sd.load_lora_for_models``: for a MODEL whose blocks are engine blocks, the LoRA
                    patches that target block linears travel in the MODEL's transformer_options as a LoRA set, and
                    every other patch goes to ComfyUI's patcher; at the first block of a forward the engine compares
                    the set with its weights and, when it changed, re-converts with ComfyUI's ``calculate_weight``
                    applied (cached per set).
  ``ModelShell``    ComfyUI's MiniMaxH3 model without blocks, plus the engine's blocks, wrapped in a ModelPatcher with
                    two hooks: a diffusion-model wrapper that rejects scheduled (hook) weight patches, which merged
                    weights cannot follow, and an ON_CLEANUP callback that releases activations and resets the
                    activation scales when a sampling run ends.
B200 choices: precision "nvfp4" runs; the reference's other precisions stay in the list and are refused with
ValueError.  Attention "auto" / "fp8" run libh3b200's FP8 kernel, "sdpa" / "cudnn" PyTorch's; "fp4" and "int8" are
refused.  All blocks stay resident in HBM, so there is no memory plan and no block streaming.

ComfyUI's modules are imported where they are used: importing this module needs only torch.
"""

from __future__ import annotations

import hashlib
import logging
from dataclasses import dataclass, field

import torch

log = logging.getLogger("tfvideo")

# ---- node identity: fixed by the reference, saved workflows depend on it
PRECISIONS = ["nvfp4", "int8", "nvfp4:edge=2", "fp8", "bf16-check"]
ATTENTION = ["auto", "fp4", "fp8", "int8", "sdpa", "cudnn"]
RUNNABLE_PRECISIONS = ("nvfp4",)


def check_choices(precision: str, attention: str) -> str:
    """Validate a node's (precision, attention) for this build; returns the conversion spec."""

    if precision not in PRECISIONS:
        raise ValueError(f"unknown precision {precision!r} (choices: {', '.join(PRECISIONS)})")
    if precision not in RUNNABLE_PRECISIONS:
        raise ValueError(f"precision {precision!r} is not built for B200: choose 'nvfp4'")
    from . import attention as A

    A.get(attention)                               # ValueError for 'fp4', 'int8' and unknown backends
    return precision


# ------------------------------------------------------------------------------------------------ engine cache
class EngineCache:
    """The process's one resident engine.  Asking for another (path, spec) drops the current engine first, so two
    sets of block weights never share the GPU."""

    def __init__(self):
        self.ident: tuple[str, str] | None = None
        self.engine = None

    def acquire(self, path: str, spec: str, on_forward=None):
        if self.ident == (path, spec) and self.engine is not None:
            return self.engine
        self.ident, self.engine = None, None
        torch.cuda.empty_cache()
        from . import store

        engine = store.load_or_convert(path, spec, device="cuda", log=log.info)
        engine.on_forward = on_forward
        self.ident, self.engine = (path, spec), engine
        return engine


# ------------------------------------------------------------------------------------------------ LoRA
@dataclass
class LoraEntry:
    """One LoRA applied to an engine MODEL: its block-linear adapters (model key -> ComfyUI adapter) and strength."""

    adapters: dict
    strength: float
    digest: str = field(default="")

    def __post_init__(self):
        if not self.digest:
            self.digest = LoraBridge.digest(self.adapters)


class LoraBridge:
    """Routes LoRA weight patches between the engine (block linears) and ComfyUI's patcher (everything else)."""

    OPTION = "tfvideo_loras"          # transformer_options key holding the MODEL's list of LoraEntry

    # -- naming
    @staticmethod
    def block_aliases(layers: int) -> dict[str, str]:
        """Every name a LoRA file may use for a block linear -> its model key ``diffusion_model.blocks.i.<lin>.weight``
        (ComfyUI's dotted key without ``.weight``, and the kohya-style ``lora_unet_blocks_i_<lin>``)."""

        from .minimax_h3 import SOURCE

        out = {}
        for i in range(layers):
            for lin in SOURCE.values():
                model_key = f"diffusion_model.blocks.{i}.{lin}.weight"
                out[model_key.removesuffix(".weight")] = model_key
                out[f"lora_unet_blocks_{i}_{lin.replace('.', '_')}"] = model_key
        return out

    @staticmethod
    def linear_name(model_key: str) -> str:
        """``diffusion_model.blocks.3.mlp.fc1.weight`` -> ``blocks.3.mlp.fc1`` (the engine's name for the linear)."""

        return model_key.removeprefix("diffusion_model.").removesuffix(".weight")

    # -- identity of a LoRA set
    @staticmethod
    def digest(adapters: dict) -> str:
        """A short content digest of a LoRA's block adapters: keys, tensor shapes and leading values."""

        h = hashlib.blake2b(digest_size=8)
        for k in sorted(adapters):
            h.update(k.encode())
            for t in getattr(adapters[k], "weights", ()):
                if torch.is_tensor(t):
                    h.update(repr(tuple(t.shape)).encode())
                    h.update(t.detach().reshape(-1)[:64].float().cpu().numpy().tobytes())
        return h.hexdigest()

    @staticmethod
    def signature(entries) -> str:
        """The cache identity of an ordered LoRA set ("" for none)."""

        return ";".join(f"{e.digest}@{e.strength:.4f}" for e in entries)

    @staticmethod
    def patch_lists(entries) -> dict[str, list]:
        """Engine linear name -> the patch list ComfyUI's ``calculate_weight`` takes, in application order."""

        lists: dict[str, list] = {}
        for e in entries:
            for model_key, adapter in e.adapters.items():
                lists.setdefault(LoraBridge.linear_name(model_key), []).append((e.strength, adapter, 1.0, None, None))
        return lists

    # -- ComfyUI side
    @staticmethod
    def engine_of(model):
        """The engine behind a ComfyUI MODEL, or None for any other model."""

        inner = getattr(getattr(model, "model", None), "diffusion_model", None)
        return getattr(inner, "tfvideo_engine", None)

    @classmethod
    def install(cls) -> None:
        """Wrap ``comfy.sd.load_lora_for_models`` once per process."""

        import comfy.sd

        stock = comfy.sd.load_lora_for_models
        if getattr(stock, "tfvideo_bridge", False):
            return

        def load_lora_for_models(model, clip, lora, strength_model, strength_clip, lora_metadata=None):
            engine = cls.engine_of(model)
            if engine is None or strength_model == 0:
                return stock(model, clip, lora, strength_model, strength_clip, lora_metadata)
            new_model = cls.split_into(model, engine, lora, float(strength_model), lora_metadata)
            new_clip = None
            if clip is not None:                      # the text encoder's part: ComfyUI's own path, model strength 0
                new_clip = stock(None, clip, lora, 0.0, strength_clip, lora_metadata)[1]
            return new_model, new_clip

        load_lora_for_models.tfvideo_bridge = True
        comfy.sd.load_lora_for_models = load_lora_for_models

    @classmethod
    def split_into(cls, model, engine, lora: dict, strength: float, lora_metadata=None):
        """A clone of ``model`` carrying the LoRA: block-linear adapters appended to its LoRA set, the rest patched
        by ComfyUI."""

        import comfy.lora
        import comfy.lora_convert

        aliases = cls.block_aliases(len(engine.blocks))
        keys = comfy.lora.model_lora_keys_unet(model.model, {})
        keys.update(aliases)
        loaded = comfy.lora.load_lora(comfy.lora_convert.convert_lora(lora), keys)
        engine_keys = set(aliases.values())
        blocks = {k: a for k, a in loaded.items() if k in engine_keys}
        others = {k: a for k, a in loaded.items() if k not in engine_keys}
        clone = model.clone()
        clone.add_patches(others, strength)
        options = dict(clone.model_options.get("transformer_options", {}))
        options[cls.OPTION] = [*options.get(cls.OPTION, []), LoraEntry(blocks, strength)]
        clone.model_options["transformer_options"] = options
        if lora_metadata:
            clone.set_attachments("lora_metadata", lora_metadata)
        log.info("[tfvideo] LoRA at strength %.3f: %d block linear(s) merged by the engine, %d tensor(s) patched "
                 "by ComfyUI", strength, len(blocks), len(others))
        return clone

    # -- engine side (called at block 0 of every forward)
    @classmethod
    def sync(cls, engine, transformer_options) -> bool:
        """Bring the engine's weights to the MODEL's LoRA set; True when it re-converted."""

        entries = list((transformer_options or {}).get(cls.OPTION, []))
        sig = cls.signature(entries)
        if sig == engine.lora_sig:
            return False
        from . import store

        merge = None
        if entries:
            import comfy.lora

            lists = cls.patch_lists(entries)

            def merge(name, w):
                return comfy.lora.calculate_weight(lists[name], w, name) if name in lists else None
        log.info("[tfvideo] engine weights follow a new LoRA set (%d LoRA(s))%s", len(entries),
                 "" if entries else ": back to the base checkpoint")
        engine.release_vram()
        fresh = store.load_or_convert(engine.source, engine.kind, device="cuda", log=log.info, merge=merge,
                                      merge_sig=sig)
        engine.replace_blocks(fresh.blocks, sig, slots=fresh.slots)
        return True


def on_forward(engine, S, transformer_options) -> None:
    """The engine's per-forward hook (block 0): keep its weights in line with the MODEL's LoRA set."""

    LoraBridge.sync(engine, transformer_options)


# ------------------------------------------------------------------------------------------------ the MODEL
class ModelShell:
    """ComfyUI's MiniMaxH3 model for a checkpoint, built without its DiT blocks, then given the engine's."""

    def __init__(self, path: str):
        from .source import SafeTensors

        self.path = path
        self.file = SafeTensors(path)

    def detect(self) -> tuple[str, dict]:
        """(key prefix, ComfyUI unet config) from the checkpoint's key names and shapes alone."""

        import comfy.model_detection as md

        shapes = {k: torch.empty(self.file.shape(k), device="meta") for k in self.file.keys()}
        prefix = md.unet_prefix_from_state_dict(shapes)
        if not any(k.startswith(prefix) for k in shapes):
            prefix = ""                                # bare keys, as ComfyUI's own loader accepts
        config = md.detect_unet_config(shapes, prefix)
        if not config or config.get("image_model") != "minimax_h3":
            raise RuntimeError(f"{self.path}: not a MiniMax H3 DiT checkpoint (ComfyUI detected "
                               f"{(config or {}).get('image_model')!r})")
        return prefix, config

    def outside_blocks(self, prefix: str) -> dict:
        """The checkpoint's tensors outside the DiT blocks, keys without the prefix (the engine owns the blocks)."""

        return {k[len(prefix):]: self.file.get(k) for k in self.file.keys()
                if k.startswith(prefix) and not k[len(prefix):].startswith("blocks.")}

    def patcher(self, engine):
        import comfy.model_detection as md
        import comfy.model_management as mm
        import comfy.model_patcher as mp
        import comfy.patcher_extension as pe

        from .minimax_h3 import EngineBlock

        prefix, config = self.detect()
        config = dict(config, num_layers=0)          # ComfyUI builds no blocks of its own
        state = self.outside_blocks(prefix)
        model_config = md.model_config_from_unet_config(config, state)
        device = mm.get_torch_device()
        model_config.set_inference_dtype(torch.bfloat16, torch.bfloat16, device=device)
        model = model_config.get_model(state, "")
        inner = model.diffusion_model
        inner.blocks = torch.nn.ModuleList([EngineBlock(engine, i) for i in range(len(engine.blocks))])
        inner.tfvideo_engine = engine
        engine.comfy_model = model
        patcher = mp.CoreModelPatcher(model, load_device=device, offload_device=mm.unet_offload_device())
        model.load_model_weights(state, "", assign=patcher.is_dynamic())
        patcher.add_wrapper(pe.WrappersMP.DIFFUSION_MODEL, reject_hook_patches(model))
        patcher.add_callback_with_key(pe.CallbacksMP.ON_CLEANUP, "tfvideo", end_of_run(engine))
        return patcher


def reject_hook_patches(model):
    """Diffusion-model wrapper: scheduled (hook) weight patches change weights per step, which merged NVFP4 weights
    cannot follow -- refuse them instead of silently ignoring them."""

    def wrapper(executor, x, timestep, context, transformer_options={}, **kwargs):
        current = getattr(model, "current_patcher", None)
        if current is not None and getattr(current, "hook_patches", None):
            raise RuntimeError("MiniMax H3 on the B200 engine: scheduled (hook) weight patches are not available; "
                               "apply LoRAs with a regular LoRA loader")
        return executor(x, timestep, context, transformer_options, **kwargs)

    return wrapper


def end_of_run(engine):
    """ON_CLEANUP callback: the sampling run is over -- drop activation buffers, start the next run on exact scales."""

    def callback(patcher):
        engine.release_vram()
        engine.end_run()

    return callback


# ------------------------------------------------------------------------------------------------ the node
ENGINES = EngineCache()


def diffusion_model_files() -> list[str]:
    import folder_paths

    return [n for n in folder_paths.get_filename_list("diffusion_models") if n.endswith(".safetensors")]


class TFMiniMaxH3Loader:
    """Loads a MiniMax H3 DiT whose 50 blocks run on the B200 engine (NVFP4 weights, converted once and cached)."""

    @classmethod
    def INPUT_TYPES(cls):
        files = diffusion_model_files()
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
        LoraBridge.install()
        path = folder_paths.get_full_path_or_raise("diffusion_models", unet_name)
        engine = ENGINES.acquire(path, spec, on_forward)
        engine.attn, engine.attn_name = A.get(attention), attention
        log.info("[tfvideo] B200 engine for %s: %s linears, %s attention, %.2f GiB of block weights resident",
                 unet_name, spec, attention, engine.nbytes() / 2 ** 30)
        return (ModelShell(path).patcher(engine),)


NODE_CLASS_MAPPINGS = {"TFMiniMaxH3Loader": TFMiniMaxH3Loader}
NODE_DISPLAY_NAME_MAPPINGS = {"TFMiniMaxH3Loader": "TensorFold MiniMax H3 Loader"}
