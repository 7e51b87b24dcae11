"""Standalone quantised linear modules with the reference's ``convlinear.py``
interface (``ConvLinear4bit`` / ``ConvLinear8bit``: constructor arguments,
``weight`` / ``scale`` / ``bias`` buffers, ``from_float``, ``forward``;
``convlinear.py:22-42,73-109,154-199``).

Behaviour: ``from_float`` takes an ``nn.Linear``, rotates its weight rows
block-wise with the Hadamard transform (when ``rot_need``), optionally
permutes the input columns (PermuQuant, INT4 only), and quantises per output
row (INT4 packed two per byte, or INT8).  ``forward`` applies the same
rotation / permutation to the activations and multiplies with the
dequantised weight.

Here the INT4 module runs the B200 kernels end to end (one prep launch for
rotation + permutation, then the W4A16 GEMM with the bias fused; fp16 or
bf16 CUDA activations).  The INT8 module is a W8A16 layer: its activation
prep runs on the B200 prep kernel on CUDA, and the dequantised linear is
torch's, which is the reference's own arithmetic for this module.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _quant_utils as _qu

__all__ = ["ConvLinear4bit", "ConvLinear8bit"]


def _rotated_weight(linear: nn.Linear, rot_need: bool, rot_size: int, perm: torch.Tensor | None) -> torch.Tensor:
    """The float32 weight in the rotated (and permuted) input basis the
    module's activations are prepared into."""
    if rot_need and not _qu.is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    w = linear.weight.detach().float()
    if rot_need:
        w = _qu.rotate_activations(w, rot_size)
    return w if perm is None else w[:, perm]


class _QuantLinearBase(nn.Module):
    """Buffers and activation prep shared by the two module types."""

    def __init__(self, weight: torch.Tensor, scale: torch.Tensor, rot_need: bool, bias: torch.Tensor | None,
                 rot_size: int, in_features: int, perm: torch.Tensor | None = None) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = weight.shape[-2]
        self.rot_need = rot_need
        self.rot_size = rot_size
        self._perm = perm
        self.register_buffer("weight", weight)
        self.register_buffer("scale", scale)
        if bias is None:
            self.bias = None
        else:
            self.register_buffer("bias", bias)

    def _prepared(self, x2: torch.Tensor) -> torch.Tensor:
        """Rotation (and permutation): one prep launch on CUDA fp16 / bf16
        activations, the torch restatement elsewhere (CPU modules)."""
        rot = self.rot_size if self.rot_need else 0
        if not rot and self._perm is None:
            return x2
        if x2.is_cuda and x2.dtype in (torch.float16, torch.bfloat16):
            from . import _b200_runtime as rt
            perm = None if self._perm is None else self._perm.to(x2.device)
            _, _, xp, _ = rt.prep_quantize(x2, rot_size=rot, w_in=self.in_features, perm=perm, quantize=False,
                                           want_prep=True)
            return xp
        xp = _qu.rotate_activations(x2, rot) if rot else x2
        if xp.shape[-1] < self.in_features:
            xp = F.pad(xp, (0, self.in_features - xp.shape[-1]))
        return xp if self._perm is None else xp[..., self._perm.to(xp.device)]

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rot_size={self.rot_size}, rot_need={self.rot_need}")


class ConvLinear8bit(_QuantLinearBase):
    """W8A16 linear: optional rotation, int8 weights with per-row scales."""

    def __init__(self, weight, scale, rot_need=True, bias=None, rot_size=256):
        super().__init__(weight, scale, rot_need, bias, rot_size, in_features=weight.shape[-1])

    def forward(self, x):
        xp = self._prepared(x.reshape(-1, x.shape[-1]))
        w = self.weight.to(xp.dtype) * self.scale.to(xp.dtype)
        y = F.linear(xp, w, None if self.bias is None else self.bias.to(xp.dtype))
        return y.reshape(*x.shape[:-1], -1)

    @staticmethod
    def from_float(module: nn.Linear, rot_need: bool = True, rot_size: int = 256) -> "ConvLinear8bit":
        w = _rotated_weight(module, rot_need, rot_size, None)
        s = _qu.calculate_scales_int8(w, w.shape[1])
        q = _qu.quantize_weights_int8(w, s, w.shape[1])
        b = None if module.bias is None else module.bias.detach().clone()
        return ConvLinear8bit(weight=q, scale=s, rot_need=rot_need, bias=b, rot_size=rot_size)


class ConvLinear4bit(_QuantLinearBase):
    """W4A16 linear: optional rotation and permutation, packed INT4 weights
    with per-row scales; B200 kernels only (CUDA fp16 / bf16 activations)."""

    def __init__(self, weight, scale, rot_need=True, bias=None, rot_size=256, perm=None, in_features=None):
        super().__init__(weight, scale, rot_need, bias, rot_size,
                         in_features=in_features if in_features is not None else weight.shape[-1] * 2, perm=perm)

    def forward(self, x):
        if not (x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)):
            raise RuntimeError("ConvLinear4bit runs on the B200 kernels: float16 / bfloat16 CUDA activations "
                               f"required (got {x.dtype} on {x.device})")
        from . import _b200_runtime as rt
        xp = self._prepared(x.reshape(-1, x.shape[-1]))
        b = None if self.bias is None else self.bias.to(x.dtype)
        y = rt.gemm_w4a16(xp, self.weight, self.scale.reshape(-1, 1), bias=b, K=self.in_features)
        return y.reshape(*x.shape[:-1], -1)

    @staticmethod
    def from_float(module: nn.Linear, rot_need: bool = True, rot_size: int = 256,
                   perm: torch.Tensor | None = None) -> "ConvLinear4bit":
        w = _rotated_weight(module, rot_need, rot_size, perm)
        s = _qu.calculate_scales(w, w.shape[1])
        packed = _qu.pack_int4(_qu.quantize_weights(w, s, w.shape[1])).to(torch.uint8)
        b = None if module.bias is None else module.bias.detach().clone()
        return ConvLinear4bit(weight=packed, scale=s, rot_need=rot_need, bias=b, rot_size=rot_size, perm=perm,
                              in_features=w.shape[1])
