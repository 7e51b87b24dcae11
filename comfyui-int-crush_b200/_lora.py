"""Adapter attach/detach for INT-Crush layers (API of the reference's ``_lora.py``).

``attach_lora_as_buffers`` parses a LoRA state dict with ComfyUI and stores
each adapter object on its INT-Crush ``Linear`` (``_lora.py:38-87``);
``clear_intcrush_lora`` removes them (``_lora.py:22-35``).  At forward time a
standard LoRA runs on the B200 low-rank kernels; other adapter types use
their own ``h()``/``g()`` math.
"""

from __future__ import annotations

import logging
from typing import Any

__all__ = ["clear_intcrush_lora", "attach_lora_as_buffers"]

_log = logging.getLogger(__name__)

_ADAPTER_ATTRS = {
    "_intcrush_adapter": None, "_intcrush_lora_strength": None, "_intcrush_adapter_ready": False,
    "_intcrush_adapter_device": None, "_intcrush_lokr_cache": None, "_intcrush_lokr_cache_adapter_id": None,
    "_intcrush_lokr_cache_strength": None,
}


def clear_intcrush_lora(model: Any) -> int:
    """Remove adapter residuals from every INT-Crush Linear; returns the count."""
    count = 0
    for module in model.model.modules():
        if hasattr(module, "_intcrush_adapter"):
            for k, v in _ADAPTER_ATTRS.items():
                setattr(module, k, v)
            count += 1
    return count


def attach_lora_as_buffers(model: Any, lora_sd: dict, strength: float) -> tuple[int, int]:
    """Attach the adapters of ``lora_sd`` to matching INT-Crush Linears.
    Returns ``(attached, total_patches)``."""
    import comfy.lora
    import comfy.lora_convert
    import comfy.weight_adapter

    lora_sd = comfy.lora_convert.convert_lora(lora_sd)
    key_map = comfy.lora.model_lora_keys_unet(model.model, {})
    patches = comfy.lora.load_lora(lora_sd, key_map)
    if not patches:
        return 0, 0
    clear_intcrush_lora(model)
    by_key = {f"{name}.weight": m for name, m in model.model.named_modules() if hasattr(m, "_intcrush_adapter")}
    attached = 0
    for weight_key, patch in patches.items():
        module = by_key.get(weight_key)
        if module is None or not isinstance(patch, comfy.weight_adapter.WeightAdapterBase):
            continue
        module._intcrush_adapter = patch
        module._intcrush_lora_strength = strength
        attached += 1
    if attached == 0:
        _log.warning("[INT-Crush LoRA] No modules matched (%d patches parsed but none mapped to INT-Crush layers)",
                     len(patches))
    return attached, len(patches)
