"""ComfyUI loader nodes with the reference's node interface.

Node names, inputs, return types, categories and the safetensors metadata
keys are the reference's (``_loaders.py:21-25,46-67,72-226``), so saved
workflows and INT-Crush checkpoints keep working:

* ``int_crush.format_version``: "2" or "3" marks an INT4 file, "1" an INT8
  file; only then is ``int_crush.rot_size`` trusted;
* ``int_crush.rot_size``: the rotation block the file was quantised with
  (one of :data:`VALID_ROT_SIZES`); it overrides the node's widget value;
* ``int_crush.padded_layers``: ``"key=in_features;..."`` for INT8 layers
  whose input width was padded at conversion time.

An INT4 file without rotation cannot use W4A8 (its activations would be
quantised unrotated), so it is loaded with the W4A16 path.  The models run
their linears on the B200 kernels through :func:`make_intcrush_ops`.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass, field

import torch

from ._lora import attach_lora_as_buffers, clear_intcrush_lora
from ._ops import make_intcrush_ops

log = logging.getLogger(__name__)

VALID_ROT_SIZES: tuple[int, ...] = (0, 16, 64, 256, 1024, 4096)
_CATEGORY = "loaders/INT-Crush"


def _model_files(kind: str) -> list[str]:
    """File names ComfyUI lists for ``kind`` ("diffusion_models", "loras");
    empty outside ComfyUI."""
    try:
        import folder_paths
    except ImportError:
        return []
    try:
        return folder_paths.get_filename_list(kind)
    except Exception:   # folder not configured
        return []


@dataclass
class CheckpointInfo:
    """What an INT-Crush safetensors header says about its file."""

    metadata: dict = field(default_factory=dict)

    def is_format(self, versions: tuple[str, ...]) -> bool:
        return self.metadata.get("int_crush.format_version") in versions

    def rot_size(self, requested: int, versions: tuple[str, ...]) -> int:
        """The file's own rotation block when it declares a valid one; the
        node's value otherwise (with a warning when the file is an INT-Crush
        file that omits it, since a mismatch corrupts every rotated layer)."""
        if not self.is_format(versions):
            return requested
        raw = self.metadata.get("int_crush.rot_size")
        try:
            value = int(raw) if raw is not None else None
        except (TypeError, ValueError):
            value = None
        if value in VALID_ROT_SIZES:
            if value != requested:
                log.info("[INT-Crush] rot_size %d taken from the checkpoint (node value %d)", value, requested)
            return value
        log.warning("[INT-Crush] checkpoint has no usable int_crush.rot_size (%r); using the node value %d, "
                    "which must match the rotation the model was quantised with", raw, requested)
        return requested

    def padded_layers(self) -> dict[str, int]:
        """``int_crush.padded_layers`` as {weight key: original in_features}."""
        table: dict[str, int] = {}
        for item in str(self.metadata.get("int_crush.padded_layers", "") or "").split(";"):
            key, sep, width = item.partition("=")
            if sep and key.strip():
                table[key.strip()] = int(width.strip())
        return table


def _read_checkpoint_info(path: str) -> CheckpointInfo:
    import comfy.utils
    try:
        _, metadata = comfy.utils.load_torch_file(path, return_metadata=True)
    except Exception:   # a file without a readable header: no metadata
        metadata = None
    return CheckpointInfo(dict(metadata or {}))


class _QuantisedModelLoader:
    """Shared body of the two model nodes; subclasses name the weight format."""

    QUANT_FORMAT = ""
    FORMAT_VERSIONS: tuple[str, ...] = ()

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = _CATEGORY

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"unet_name": (_model_files("diffusion_models"),),
                             "rot_size": (list(VALID_ROT_SIZES), {"default": 256})}}

    def _ops_for(self, rot_size: int):
        return make_intcrush_ops(self.QUANT_FORMAT, rot_size)

    def _after_load(self, model, info: CheckpointInfo) -> None:
        """Format-specific fix-ups once the model is built."""

    def load(self, unet_name: str, rot_size: int) -> tuple[object]:
        import folder_paths
        from comfy.sd import load_diffusion_model
        path = folder_paths.get_full_path("diffusion_models", unet_name)
        if path is None:
            raise FileNotFoundError(f"Model not found: {unet_name}")
        info = _read_checkpoint_info(path)
        ops = self._ops_for(info.rot_size(rot_size, self.FORMAT_VERSIONS))
        if torch.cuda.is_available():
            torch.cuda.empty_cache()   # the model is about to take most of the device
        model = load_diffusion_model(path, model_options={"custom_operations": ops})
        self._after_load(model, info)
        return (model,)


class SimpleINT4UNetLoader(_QuantisedModelLoader):
    """ComfyUI node: an INT-Crush model with packed INT4 weights."""

    QUANT_FORMAT = "int4_crush"
    FORMAT_VERSIONS = ("2", "3")

    def _ops_for(self, rot_size: int):
        if rot_size == 0:
            log.info("[INT-Crush] INT4 model without rotation: W4A16 (W4A8 needs rotated activations)")
            return make_intcrush_ops(self.QUANT_FORMAT, rot_size, use_w4a16=True)
        return make_intcrush_ops(self.QUANT_FORMAT, rot_size)


class SimpleINT8UNetLoader(_QuantisedModelLoader):
    """ComfyUI node: an INT-Crush model with INT8 weights."""

    QUANT_FORMAT = "int8_crush"
    FORMAT_VERSIONS = ("1",)

    def _after_load(self, model, info: CheckpointInfo) -> None:
        table = info.padded_layers()
        if table:
            _restore_padded_inputs(model, table)


def _trimmed_weight(weight, width: int):
    """The weight with its input columns cut back to ``width``, or None when
    it is not wider.  Quantised weights keep their layout type and scales;
    only the recorded original shape changes."""
    if hasattr(weight, "_qdata"):
        data, params = weight._qdata, weight._params
        have = data.shape[1] if data.dim() > 1 else data.shape[0]
        if have <= width:
            return None
        extra = {k: getattr(params, k) for k in ("rot_need", "rot_size", "perm", "zp")
                 if getattr(params, k, None) is not None}
        params2 = type(params)(scale=params.scale, orig_dtype=params.orig_dtype,
                               orig_shape=(params.orig_shape[0], width), **extra)
        from comfy.quant_ops import QuantizedTensor
        return QuantizedTensor(data[:, :width].contiguous(), weight._layout_type, params2), have
    if weight.shape[1] <= width:
        return None
    return weight[:, :width].contiguous(), weight.shape[1]


def _restore_padded_inputs(model, table: dict[str, int]) -> None:
    """Undo conversion-time input padding of INT8 layers
    (``int_crush.padded_layers``): drop the padded weight columns, forget the
    layer's prepared device weights, and for the patch embedding ``img_in``
    also restore the model's ``in_channels``."""
    import comfy.utils
    root = model.model
    for key, width in table.items():
        path = key[: -len(".weight")] if key.endswith(".weight") else key
        try:
            module = comfy.utils.get_attr(root, path)
        except AttributeError:
            log.info("[INT-Crush] padded layer %s not in this model; skipped", key)
            continue
        weight = getattr(module, "weight", None)
        trimmed = None if weight is None else _trimmed_weight(weight, width)
        if trimmed is not None:
            new_weight, old_width = trimmed
            module.weight = torch.nn.Parameter(new_weight, requires_grad=False)
            for cache in ("_b200", "_graph_runner"):
                if hasattr(module, cache):
                    setattr(module, cache, None)
            log.info("[INT-Crush] %s: input width %d -> %d", key, old_width, width)
        if path == "img_in" and hasattr(root, "in_channels"):
            patch = getattr(root, "patch_size", 1) or 1
            root.in_channels = width // (patch * patch)
            log.info("[INT-Crush] model in_channels restored to %d", root.in_channels)


class IntCrushLoRALoader:
    """ComfyUI node: attach a LoRA as a residual on the raw (unrotated)
    activations of the INT-Crush layers; the quantised weights stay as they
    are and keep running on the B200 GEMMs."""

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "load"
    CATEGORY = _CATEGORY

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",),
                             "lora_name": (_model_files("loras"), {"tooltip": "The name of the LoRA."}),
                             "strength": ("FLOAT", {"default": 1.0, "min": -10.0, "max": 10.0, "step": 0.01})}}

    def load(self, model: object, lora_name: str, strength: float) -> tuple[object]:
        import comfy.utils
        import folder_paths
        path = folder_paths.get_full_path_or_raise("loras", lora_name)
        weights, _ = comfy.utils.load_torch_file(path, safe_load=True, return_metadata=True)
        if not weights:
            raise ValueError(f"INT-Crush LoRA: empty file '{lora_name}'")
        attached, parsed = attach_lora_as_buffers(model, weights, strength)
        if attached:
            log.info("[INT-Crush LoRA] %s: %d layer(s) patched", lora_name, attached)
        else:
            log.warning("[INT-Crush LoRA] %s: %d patch(es) read, none matched an INT-Crush layer", lora_name, parsed)
        return (model,)


class IntCrushLoRAUnloader:
    """ComfyUI node: remove the LoRA residuals attached by IntCrushLoRALoader."""

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "unload"
    CATEGORY = _CATEGORY

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",)}}

    def unload(self, model: object) -> tuple[object]:
        log.info("[INT-Crush LoRA] removed from %d layer(s)", clear_intcrush_lora(model))
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
           "NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS", "VALID_ROT_SIZES", "CheckpointInfo"]
