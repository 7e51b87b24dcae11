"""QuantizedTensor layout classes for the INT-Crush INT4/INT8 formats.

API of the reference's ``quant_layout.py`` (``IntCrushInt4Layout`` /
``IntCrushInt8Layout`` with their ``Params`` dataclasses, ``state_dict_tensors``,
``dequantize``, ``quantize``, ``supports_fast_matmul`` and
``register_intcrush_layouts``, ``quant_layout.py:44-234``).  Differences, by
design: ``dequantize`` of INT4 honours group scales ``[N, G]`` (the reference's
``scale.reshape(-1, 1)`` rejects them), and ``supports_fast_matmul`` reports
whether the B200 kernels are usable.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ._quant_utils import (INT4_MAX, INT4_MIN, INT4_SCALE_DIVISOR, INT4_TWOS_COMPLEMENT_BIAS, INT8_MAX,
                           INT8_MIN, INT8_SCALE_DIVISOR, unpack_int4)

__all__ = ["IntCrushInt4Layout", "IntCrushInt8Layout", "register_intcrush_layouts"]

try:  # the host's base class when ComfyUI's kitchen package is present
    from comfy_kitchen.tensor.base import BaseLayoutParams  # type: ignore
except ImportError:
    @dataclass(frozen=True)
    class BaseLayoutParams:
        scale: torch.Tensor
        orig_dtype: torch.dtype
        orig_shape: tuple

        def __post_init__(self):
            pass


def _scale_full(scale: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    """Expand per-row ``[N]``/``[N,1]`` or group ``[N,G]`` scales to ``[N,K]``."""
    s = scale.reshape(rows, -1).float()
    G = s.shape[1]
    if G == 1:
        return s
    gs = -(-K // G)
    return s.repeat_interleave(gs, dim=1)[:, :K]


def _b200_ready() -> bool:
    try:
        from . import _b200_runtime as rt
        return bool(rt.B200_AVAILABLE)
    except Exception:
        return False


class _ParamsMixin:
    def _tensor_fields(self) -> list[str]:
        fields = ["scale"]
        if self.perm is not None:
            fields.append("perm")
        if self.zp is not None:
            fields.append("zp")
        return fields

    def _validate_tensor_fields(self):
        if isinstance(self.scale, torch.Tensor):
            object.__setattr__(self, "scale", self.scale.to(dtype=torch.float32, non_blocking=True))


class IntCrushInt4Layout:
    """Packed INT4 (uint8, two values per byte, low nibble = even k) with fp16
    scales, per row or per group; optional zero point and PermuQuant perm."""

    @dataclass(frozen=True)
    class Params(_ParamsMixin, BaseLayoutParams):
        rot_need: bool = True
        rot_size: int = 256
        perm: torch.Tensor | None = None
        zp: torch.Tensor | None = None

    @classmethod
    def state_dict_tensors(cls, qdata, params):
        t = {"": qdata, "weight_scale": params.scale}
        if params.perm is not None:
            t["weight_perm"] = params.perm
        if params.zp is not None:
            t["weight_zp"] = params.zp
        return t

    @classmethod
    def dequantize(cls, qdata, params):
        N, K = params.orig_shape[0], params.orig_shape[1]
        q = unpack_int4(qdata, K).float()
        s = _scale_full(params.scale, N, K)
        if params.zp is not None:
            q = q - params.zp.reshape(-1, 1).float()
        return q * s

    @classmethod
    def supports_fast_matmul(cls):
        return _b200_ready()

    @classmethod
    def quantize(cls, tensor, scale=None, stochastic_rounding=0, inplace_ops=False):
        """Per-row INT4 quantisation of an already rotated/permuted weight
        (one B200 kernel for a CUDA weight with recalculated scales)."""
        if _device_requant(tensor, scale):
            from . import _b200_runtime as rt
            packed, scales = rt.quantize_weight(tensor, 4)
            return packed, cls.Params(scale=scales, orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape))
        amax = tensor.abs().amax(dim=1, keepdim=True)
        if scale is None or (isinstance(scale, str) and scale == "recalculate"):
            scales = (amax / INT4_SCALE_DIVISOR).clamp(min=1e-8).to(torch.float16)
        elif isinstance(scale, torch.Tensor):
            scales = scale.to(torch.float16)
        else:
            scales = torch.tensor([scale], dtype=torch.float16, device=tensor.device)
        q = (tensor / scales.to(tensor.dtype)).round().clamp(INT4_MIN, INT4_MAX).to(torch.int8)
        if q.shape[-1] % 2:
            q = torch.cat([q, torch.zeros(*q.shape[:-1], 1, dtype=torch.int8, device=q.device)], dim=-1)
        u = torch.where(q < 0, INT4_TWOS_COMPLEMENT_BIAS + q.to(torch.int16), q.to(torch.int16)).to(torch.uint8)
        packed = u[..., 0::2] | (u[..., 1::2] << 4)
        params = cls.Params(scale=scales.reshape(-1), orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape))
        return packed, params


def _device_requant(tensor, scale) -> bool:
    """The weight is a 2-D CUDA tensor whose scales are recalculated: the
    device kernel applies (same arithmetic as the torch form below)."""
    recalc = scale is None or (isinstance(scale, str) and scale == "recalculate")
    return recalc and isinstance(tensor, torch.Tensor) and tensor.is_cuda and tensor.dim() == 2


class IntCrushInt8Layout:
    """Plain int8 weights with per-row scales; optional zero point and perm."""

    @dataclass(frozen=True)
    class Params(_ParamsMixin, BaseLayoutParams):
        rot_need: bool = True
        rot_size: int = 256
        perm: torch.Tensor | None = None
        zp: torch.Tensor | None = None

    @classmethod
    def state_dict_tensors(cls, qdata, params):
        t = {"": qdata, "weight_scale": params.scale}
        if params.perm is not None:
            t["weight_perm"] = params.perm
        if params.zp is not None:
            t["weight_zp"] = params.zp
        return t

    @classmethod
    def dequantize(cls, qdata, params):
        q = qdata.float()
        if params.zp is not None:
            q = q - params.zp.reshape(-1, 1).float()
        return q * params.scale.reshape(-1, 1).float()

    @classmethod
    def supports_fast_matmul(cls):
        return _b200_ready()

    @classmethod
    def quantize(cls, tensor, scale=None, stochastic_rounding=0, inplace_ops=False):
        """Per-row INT8 quantisation (one B200 kernel for a CUDA weight with
        recalculated scales)."""
        if _device_requant(tensor, scale):
            from . import _b200_runtime as rt
            q, scales = rt.quantize_weight(tensor, 8)
            return q, cls.Params(scale=scales, orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape))
        amax = tensor.abs().amax(dim=1, keepdim=True)
        if scale is None or (isinstance(scale, str) and scale == "recalculate"):
            scales = (amax / INT8_SCALE_DIVISOR).clamp(min=1e-8).to(torch.float32)
        elif isinstance(scale, torch.Tensor):
            scales = scale.to(torch.float32)
        else:
            scales = torch.tensor([scale], dtype=torch.float32, device=tensor.device)
        q = (tensor / scales.to(tensor.dtype)).round().clamp(INT8_MIN, INT8_MAX).to(torch.int8)
        params = cls.Params(scale=scales.reshape(-1), orig_dtype=tensor.dtype, orig_shape=tuple(tensor.shape))
        return q, params


def register_intcrush_layouts():
    """Register the layouts and the ``int4_crush``/``int8_crush`` algorithms with
    ComfyUI's quantisation registry (no-op without ComfyUI), like
    ``quant_layout.py:205-234``."""
    import logging
    log = logging.getLogger(__name__)
    try:
        from comfy.quant_ops import QUANT_ALGOS, register_layout_class  # type: ignore
    except ImportError:
        log.warning("INT-Crush: comfy.quant_ops not available; layout registration skipped")
        return
    try:
        register_layout_class("IntCrushInt4Layout", IntCrushInt4Layout)
        register_layout_class("IntCrushInt8Layout", IntCrushInt8Layout)
    except Exception:
        log.warning("INT-Crush: layout class registration failed", exc_info=True)
    QUANT_ALGOS.setdefault("int4_crush", {
        "storage_t": torch.uint8,
        "parameters": {"weight_scale", "weight_zp", "weight_perm"},
        "comfy_tensor_layout": "IntCrushInt4Layout",
    })
    QUANT_ALGOS.setdefault("int8_crush", {
        "storage_t": torch.int8,
        "parameters": {"weight_scale", "weight_perm", "weight_zp"},
        "comfy_tensor_layout": "IntCrushInt8Layout",
    })
