"""Standalone quantised linear modules (API of the reference's ``convlinear.py``).

``ConvLinear4bit`` / ``ConvLinear8bit`` with ``from_float`` (rotate, optional
PermuQuant permutation, per-row quantisation; ``convlinear.py:22-42,84-109,
170-199``) and ``forward`` (rotate -> permute -> dequantised linear;
``convlinear.py:73-82,154-168``).  ``ConvLinear4bit.forward`` runs the B200
prep kernel and the W4A16 GEMM (bias fused) and needs fp16 CUDA activations.  ``ConvLinear8bit`` is
a W8A16 module; its dequantised linear uses torch, as in the reference.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _quant_utils as _qu

__all__ = ["ConvLinear4bit", "ConvLinear8bit"]


def _prepare_rotated_weight(module: nn.Linear, rot_need: bool, rot_size: int,
                            perm: torch.Tensor | None = None) -> torch.Tensor:
    if rot_need and not _qu.is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be a power of 2, got {rot_size}")
    W = module.weight.float()
    if rot_need:
        W = _qu.rotate_activations(W, rot_size)
    if perm is not None:
        W = W[:, perm]
    return W


class ConvLinear8bit(nn.Module):
    """W8A16 linear: optional rotation, int8 weights with per-row scales."""

    def __init__(self, weight, scale, rot_need=True, bias=None, rot_size=256):
        super().__init__()
        self.in_features = weight.shape[-1]
        self.out_features = weight.shape[-2]
        self.rot_need = rot_need
        self.rot_size = rot_size
        self.register_buffer("weight", weight)
        self.register_buffer("scale", scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None

    def forward(self, x):
        x_rot = _qu.rotate_activations(x, self.rot_size) if self.rot_need else x
        w = self.weight.to(x_rot.dtype) * self.scale.to(x_rot.dtype)
        b = self.bias.to(x_rot.dtype) if self.bias is not None else None
        return F.linear(x_rot, w, b)

    @staticmethod
    def from_float(module: nn.Linear, rot_need: bool = True, rot_size: int = 256) -> "ConvLinear8bit":
        W = _prepare_rotated_weight(module, rot_need, rot_size)
        K = W.shape[1]
        scales = _qu.calculate_scales_int8(W, K)
        q = _qu.quantize_weights_int8(W, scales, K)
        bias = module.bias.data.clone() if module.bias is not None else None
        return ConvLinear8bit(weight=q, scale=scales, rot_need=rot_need, bias=bias, rot_size=rot_size)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rot_size={self.rot_size}, rot_need={self.rot_need}")


class ConvLinear4bit(nn.Module):
    """W4A16 linear: optional rotation and permutation, packed INT4 weights
    with per-row fp16 scales."""

    def __init__(self, weight, scale, rot_need=True, bias=None, rot_size=256, perm=None, in_features=None):
        super().__init__()
        self.in_features = in_features if in_features is not None else weight.shape[-1] * 2
        self.out_features = weight.shape[-2]
        self.rot_need = rot_need
        self.rot_size = rot_size
        self._perm = perm
        self.register_buffer("weight", weight)
        self.register_buffer("scale", scale)
        if bias is not None:
            self.register_buffer("bias", bias)
        else:
            self.bias = None

    def forward(self, x):
        if x.is_cuda and x.dtype == torch.float16:
            from . import _b200_runtime as rt
            x2 = x.reshape(-1, x.shape[-1])
            rot = self.rot_size if self.rot_need else 0
            if rot or self._perm is not None:
                _, _, x2, _ = rt.prep_quantize(x2, rot_size=rot, w_in=self.in_features,
                                               perm=None if self._perm is None else self._perm.to(x.device),
                                               quantize=False, want_prep=True)
            b = self.bias.to(torch.float16) if self.bias is not None else None
            out = rt.gemm_w4a16(x2, self.weight, self.scale.reshape(-1, 1), bias=b, K=self.in_features)
            return out.reshape(*x.shape[:-1], -1)
        raise RuntimeError("ConvLinear4bit runs on the B200 kernels: float16 CUDA activations required "
                           f"(got {x.dtype} on {x.device})")

    @staticmethod
    def from_float(module: nn.Linear, rot_need: bool = True, rot_size: int = 256,
                   perm: torch.Tensor | None = None) -> "ConvLinear4bit":
        W = _prepare_rotated_weight(module, rot_need, rot_size, perm)
        K = W.shape[1]
        scales = _qu.calculate_scales(W, K)
        packed = _qu.pack_int4(_qu.quantize_weights(W, scales, K)).to(torch.uint8)
        bias = module.bias.data.clone() if module.bias is not None else None
        return ConvLinear4bit(weight=packed, scale=scales, rot_need=rot_need, bias=bias, rot_size=rot_size,
                              perm=perm, in_features=K)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rot_size={self.rot_size}, rot_need={self.rot_need}")
