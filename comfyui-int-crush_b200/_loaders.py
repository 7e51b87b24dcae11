"""ComfyUI loader nodes (API of the reference's ``_loaders.py``).

``SimpleINT4UNetLoader``, ``SimpleINT8UNetLoader``, ``IntCrushLoRALoader`` and
``IntCrushLoRAUnloader`` with the same inputs, categories and safetensors
metadata handling: ``int_crush.format_version`` (INT4 "2"/"3", INT8 "1"),
``int_crush.rot_size`` and ``int_crush.padded_layers`` (``_loaders.py:21-25,
46-67,72-226``).  The models they build run their linears on the B200 ops.
"""

from __future__ import annotations

import logging

import torch

from ._lora import attach_lora_as_buffers, clear_intcrush_lora
from ._ops import make_intcrush_ops

log = logging.getLogger(__name__)

VALID_ROT_SIZES: tuple[int, ...] = (0, 16, 64, 256, 1024, 4096)
_INT4_FORMAT_VERSIONS: tuple[str, ...] = ("2", "3")
_INT8_FORMAT_VERSIONS: tuple[str, ...] = ("1",)


def _get_diffusion_model_list() -> list[str]:
    try:
        import folder_paths
        return folder_paths.get_filename_list("diffusion_models")
    except Exception:
        return []


def _get_lora_list() -> list[str]:
    try:
        import folder_paths
        return folder_paths.get_filename_list("loras")
    except Exception:
        return []


def _detect_rot_size(metadata: dict | None, default_rot_size: int, format_versions: tuple[str, ...]) -> int:
    """rot_size from safetensors metadata when the format version matches."""
    if not metadata or metadata.get("int_crush.format_version") not in format_versions:
        return default_rot_size
    detected = metadata.get("int_crush.rot_size")
    if detected is not None:
        try:
            detected = int(detected)
            if detected in VALID_ROT_SIZES:
                log.info("[INT-Crush] Auto-detected rot_size=%d from metadata", detected)
                return detected
        except (ValueError, TypeError):
            pass
    log.warning("[INT-Crush] Metadata confirms INT-Crush format but rot_size is missing; using default "
                "rot_size=%d. This may produce incorrect results if the model was quantized with a "
                "different rot_size.", default_rot_size)
    return default_rot_size


def _parse_padded_layers(padded_str: str) -> dict[str, int]:
    """``"key=orig_in;key2=orig_in2"`` -> ``{key: orig_in}``."""
    out: dict[str, int] = {}
    for entry in padded_str.split(";"):
        if "=" in entry:
            k, v = entry.split("=", 1)
            out[k.strip()] = int(v.strip())
    return out


def _load_model(unet_name: str, fmt: str, rot_size: int, format_versions, use_w4a16_if_unrotated: bool):
    import comfy.utils
    import folder_paths
    from comfy.sd import load_diffusion_model
    path = folder_paths.get_full_path("diffusion_models", unet_name)
    if path is None:
        raise FileNotFoundError(f"Model not found: {unet_name}")
    try:
        _, metadata = comfy.utils.load_torch_file(path, return_metadata=True)
    except Exception:
        metadata = {}
    rot_size = _detect_rot_size(metadata, rot_size, format_versions)
    use_w4a16 = False
    if use_w4a16_if_unrotated and rot_size == 0:
        log.info("[INT-Crush] W4A8 requires rotation — falling back to W4A16")
        use_w4a16 = True
    ops_cls = make_intcrush_ops(fmt, rot_size, use_w4a16=use_w4a16) if fmt == "int4_crush" \
        else make_intcrush_ops(fmt, rot_size)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    model = load_diffusion_model(path, model_options={"custom_operations": ops_cls})
    return model, metadata or {}


class SimpleINT4UNetLoader:
    """ComfyUI node: loads an INT-Crush model with INT4 weights."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"unet_name": (_get_diffusion_model_list(),),
                             "rot_size": ([s for s in VALID_ROT_SIZES], {"default": 256})}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = "loaders/INT-Crush"

    def load(self, unet_name: str, rot_size: int) -> tuple[object]:
        model, _ = _load_model(unet_name, "int4_crush", rot_size, _INT4_FORMAT_VERSIONS, True)
        return (model,)


class SimpleINT8UNetLoader:
    """ComfyUI node: loads an INT-Crush model with INT8 weights."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"unet_name": (_get_diffusion_model_list(),),
                             "rot_size": ([s for s in VALID_ROT_SIZES], {"default": 256})}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = "loaders/INT-Crush"

    def load(self, unet_name: str, rot_size: int) -> tuple[object]:
        model, metadata = _load_model(unet_name, "int8_crush", rot_size, _INT8_FORMAT_VERSIONS, False)
        padded = metadata.get("int_crush.padded_layers", "")
        if padded:
            _apply_padded_layer_fixes(model, padded)
        return (model,)


def _apply_padded_layer_fixes(model, padded_str: str) -> None:
    """Trim INT8 weight columns of layers whose in_features were padded at
    conversion time and fix ``in_channels`` of ``img_in`` (``_loaders.py:164-226``)."""
    import comfy.utils
    m = model.model
    for layer_key, orig_in in _parse_padded_layers(padded_str).items():
        module_path = layer_key.rsplit(".weight", 1)[0]
        try:
            module = comfy.utils.get_attr(m, module_path)
        except AttributeError:
            continue
        weight = getattr(module, "weight", None)
        if weight is not None:
            if hasattr(weight, "_qdata"):
                qdata, params = weight._qdata, weight._params
                padded_in = qdata.shape[1] if qdata.dim() > 1 else qdata.shape[0]
                if padded_in > orig_in:
                    new_params = type(params)(
                        scale=params.scale, orig_dtype=params.orig_dtype,
                        orig_shape=(params.orig_shape[0], orig_in),
                        **{k: v for k, v in {"rot_need": getattr(params, "rot_need", None),
                                             "rot_size": getattr(params, "rot_size", None),
                                             "perm": getattr(params, "perm", None),
                                             "zp": getattr(params, "zp", None)}.items() if v is not None})
                    from comfy.quant_ops import QuantizedTensor
                    module.weight = torch.nn.Parameter(
                        QuantizedTensor(qdata[:, :orig_in].contiguous(), weight._layout_type, new_params),
                        requires_grad=False)
                    if hasattr(module, "_b200"):
                        module._b200 = None
                        module._graph_runner = None
                    log.info("[INT-Crush] INT8: Fixed %s in_features %d -> %d", layer_key, padded_in, orig_in)
            else:
                padded_in = weight.shape[1]
                if padded_in > orig_in:
                    module.weight = torch.nn.Parameter(weight[:, :orig_in].contiguous(), requires_grad=False)
                    log.info("[INT-Crush] INT8: Fixed %s in_features %d -> %d", layer_key, padded_in, orig_in)
        if module_path == "img_in" and hasattr(m, "in_channels"):
            ps = getattr(m, "patch_size", 1)
            m.in_channels = orig_in // (ps * ps) if ps else orig_in
            log.info("[INT-Crush] INT8: Fixed model.in_channels = %d", m.in_channels)


class IntCrushLoRALoader:
    """Attach a LoRA as a residual on the raw (unrotated) activation, keeping
    the quantised weights and the B200 GEMMs."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",),
                             "lora_name": (_get_lora_list(), {"tooltip": "The name of the LoRA."}),
                             "strength": ("FLOAT", {"default": 1.0, "min": -10.0, "max": 10.0, "step": 0.01})}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = "loaders/INT-Crush"

    def load(self, model: object, lora_name: str, strength: float) -> tuple[object]:
        import comfy.utils
        import folder_paths
        path = folder_paths.get_full_path_or_raise("loras", lora_name)
        lora_sd, _ = comfy.utils.load_torch_file(path, safe_load=True, return_metadata=True)
        if not lora_sd:
            raise ValueError(f"INT-Crush LoRA: empty file '{lora_name}'")
        attached, total = attach_lora_as_buffers(model, lora_sd, strength)
        if attached == 0:
            log.warning("[INT-Crush LoRA] No modules matched (%d patches parsed but none mapped to INT-Crush "
                        "layers)", total)
        else:
            log.info("[INT-Crush LoRA] Attached to %d layer(s)", attached)
        return (model,)


class IntCrushLoRAUnloader:
    """Remove INT-Crush LoRA residuals from a model."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",)}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "unload"
    CATEGORY = "loaders/INT-Crush"

    def unload(self, model: object) -> tuple[object]:
        n = clear_intcrush_lora(model)
        log.info("[INT-Crush LoRA] Cleared LoRA from %d layer(s)", n)
        return (model,)


NODE_CLASS_MAPPINGS = {
    "SimpleINT4UNetLoader": SimpleINT4UNetLoader,
    "SimpleINT8UNetLoader": SimpleINT8UNetLoader,
    "IntCrushLoRALoader": IntCrushLoRALoader,
    "IntCrushLoRAUnloader": IntCrushLoRAUnloader,
}

NODE_DISPLAY_NAME_MAPPINGS = {
    "SimpleINT4UNetLoader": "INT4 UNet Loader (INT-Crush)",
    "SimpleINT8UNetLoader": "INT8 UNet Loader (INT-Crush)",
    "IntCrushLoRALoader": "LoRA Loader (INT-Crush)",
    "IntCrushLoRAUnloader": "LoRA Unloader (INT-Crush)",
}

__all__ = ["SimpleINT4UNetLoader", "SimpleINT8UNetLoader", "IntCrushLoRALoader", "IntCrushLoRAUnloader",
           "NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS"]
