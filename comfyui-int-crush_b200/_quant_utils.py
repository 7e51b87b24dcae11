"""Quantisation primitives with the API of the reference's ``_quant_utils.py``.

Same names, signatures and results as ComfyUI-INT-Crush ``_quant_utils.py``
(constants ``:151-155,200-201``; Hadamard ``:64-114``; rotation ``:117-147``;
INT4/INT8 packing ``:158-197,204-221``; scales / weight quantisers
``:226-292``).  These are load/conversion-time helpers.  On a CUDA tensor,
``rotate_activations`` runs the B200 prep kernel (fp64 butterflies, one
rounding to the activation dtype) instead of a matmul against H^T; on CPU
tensors it uses torch, as conversion tools do.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

__all__ = [
    "make_hadamard_regular", "is_power_of_two", "rotate_activations", "pack_int4", "unpack_int4",
    "pack_int8", "unpack_int8", "validate_int4_range", "calculate_scales", "calculate_scales_int8",
    "quantize_weights", "quantize_weights_int8", "INT4_MIN", "INT4_MAX", "INT4_SCALE_DIVISOR",
    "INT4_TWOS_COMPLEMENT_BIAS", "INT8_MIN", "INT8_MAX", "INT8_SCALE_DIVISOR", "DEFAULT_GROUP_SIZE",
]

INT4_MIN = -8
INT4_MAX = 7
INT4_SCALE_DIVISOR = 7.0
INT4_TWOS_COMPLEMENT_BIAS = 16
INT8_MIN = -128
INT8_MAX = 127
INT8_SCALE_DIVISOR = 127.0
DEFAULT_GROUP_SIZE = 128


def is_power_of_two(n: int) -> bool:
    return n > 0 and (n & (n - 1)) == 0


_is_power_of_two = is_power_of_two


def _is_power_of_four(n: int) -> bool:
    return n >= 4 and is_power_of_two(n) and (n & 0x55555555) == n


_H_cache: dict[tuple, torch.Tensor] = {}

_H4 = ((1.0, 1.0, 1.0, -1.0), (1.0, 1.0, -1.0, 1.0), (1.0, -1.0, 1.0, 1.0), (-1.0, 1.0, 1.0, 1.0))


def make_hadamard_regular(n: int, dtype: torch.dtype = torch.float16, device: str = "cpu") -> torch.Tensor:
    """Regular Hadamard ``kron(H4/2, ..., H4/2)`` of size ``n`` (a power of 4)."""
    if not _is_power_of_four(n):
        raise ValueError(f"Regular Hadamard requires power of 4, got {n}. Use rot_size=16/64/256/1024/4096.")
    key = (n, str(dtype), str(device))
    H = _H_cache.get(key)
    if H is None:
        base = torch.tensor(_H4, dtype=torch.float64) / 2.0
        H = base
        while H.shape[0] < n:
            H = torch.kron(H, base)
        H = H.to(dtype=dtype, device=device)
        _H_cache[key] = H
    return H


def _make_hadamard_sylvester(n: int, dtype: torch.dtype = torch.float16, device: str = "cpu") -> torch.Tensor:
    """Sylvester Hadamard of size ``n`` (a power of 2), entries ``+-1/sqrt(n)``
    materialised like the reference: the +-1 matrix in ``dtype`` times the
    Python float ``1/sqrt(n)``."""
    if not is_power_of_two(n):
        raise ValueError(f"n must be a power of 2, got {n}")
    key = (n, str(dtype), str(device), "sylvester")
    H = _H_cache.get(key)
    if H is None:
        W2 = torch.tensor([[1.0, 1.0], [1.0, -1.0]], dtype=dtype, device=device)
        H = torch.ones((1, 1), dtype=dtype, device=device)
        while H.shape[0] < n:
            H = torch.kron(W2, H)
        H = H * (1.0 / math.sqrt(n))
        _H_cache[key] = H
    return H


def rotate_activations(x: torch.Tensor, rot_size: int, H: torch.Tensor | None = None) -> torch.Tensor:
    """Group-wise Hadamard rotation of the last dimension (padded to a multiple
    of ``rot_size``); regular Hadamard for powers of 4, Sylvester otherwise."""
    if not is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be power of 2, got {rot_size}")
    if x.is_cuda and H is None and x.dtype in (torch.float16, torch.bfloat16) and rot_size <= 4096:
        from . import _b200_runtime as rt
        lead = x.shape[:-1]
        _, _, xp, _ = rt.prep_quantize(x, rot_size=rot_size, quantize=False, want_prep=True)
        return xp.reshape(*lead, xp.shape[-1])
    K = x.shape[-1]
    if K % rot_size:
        x = F.pad(x, (0, rot_size - K % rot_size))
    Kp = x.shape[-1]
    lead = x.shape[:-1]
    if H is None:
        H = (make_hadamard_regular if _is_power_of_four(rot_size) else _make_hadamard_sylvester)(
            rot_size, dtype=x.dtype, device=str(x.device))
    H = H.to(dtype=x.dtype, device=x.device)
    y = torch.matmul(x.reshape(-1, Kp // rot_size, rot_size), H.T)
    return y.reshape(*lead, Kp)


def validate_int4_range(tensor: torch.Tensor) -> None:
    if tensor.numel() == 0:
        return
    lo, hi = int(tensor.min()), int(tensor.max())
    if lo < INT4_MIN or hi > INT4_MAX:
        raise ValueError(f"Values must be in [{INT4_MIN}, {INT4_MAX}], got [{lo}, {hi}]")


def pack_int4(values: torch.Tensor) -> torch.Tensor:
    """Two signed nibbles per byte, low nibble = even index (odd lengths are
    zero padded)."""
    validate_int4_range(values)
    v = values.to(torch.int8)
    if v.shape[-1] % 2:
        v = torch.cat([v, torch.zeros(*v.shape[:-1], 1, dtype=torch.int8, device=v.device)], dim=-1)
    u = (v.to(torch.int16) & 0xF).to(torch.uint8)
    return u[..., 0::2] | (u[..., 1::2] << 4)


def unpack_int4(packed: torch.Tensor, K: int) -> torch.Tensor:
    lo = (packed & 0x0F).to(torch.int16)
    hi = ((packed >> 4) & 0x0F).to(torch.int16)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    out = torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)
    return out[..., :K].to(torch.int8)


def pack_int8(values: torch.Tensor) -> torch.Tensor:
    if values.numel() and (int(values.min()) < INT8_MIN or int(values.max()) > INT8_MAX):
        raise ValueError(f"Values must be in [{INT8_MIN}, {INT8_MAX}], "
                         f"got [{int(values.min())}, {int(values.max())}]")
    return values.to(torch.int8)


def unpack_int8(packed: torch.Tensor, K: int) -> torch.Tensor:
    return packed[..., :K]


def _pad_to_group_multiple(W: torch.Tensor, group_size: int) -> tuple[torch.Tensor, int]:
    rem = W.shape[1] % group_size
    if rem:
        W = F.pad(W, (0, group_size - rem))
    return W, W.shape[1]


def _calculate_scales(W: torch.Tensor, scale_divisor: float, group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    if W.dim() != 2:
        raise ValueError(f"Expected 2D tensor, got {W.dim()}D")
    Wp, width = _pad_to_group_multiple(W, group_size)
    amax = Wp.reshape(W.shape[0], width // group_size, group_size).abs().amax(dim=2)
    return (amax / scale_divisor).clamp(min=1e-8).to(torch.float16)


def _quantize_weights(W: torch.Tensor, scales: torch.Tensor, clamp_min: int, clamp_max: int,
                      group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    Wp, width = _pad_to_group_multiple(W, group_size)
    g = Wp.reshape(W.shape[0], width // group_size, group_size) / scales.unsqueeze(2).to(Wp.dtype)
    return g.round().clamp(clamp_min, clamp_max).reshape(W.shape[0], width).to(torch.int8)


def calculate_scales(W: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    return _calculate_scales(W, INT4_SCALE_DIVISOR, group_size)


def calculate_scales_int8(W: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    return _calculate_scales(W, INT8_SCALE_DIVISOR, group_size)


def quantize_weights(W: torch.Tensor, scales: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    return _quantize_weights(W, scales, INT4_MIN, INT4_MAX, group_size)


def quantize_weights_int8(W: torch.Tensor, scales: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE) -> torch.Tensor:
    return _quantize_weights(W, scales, INT8_MIN, INT8_MAX, group_size)
