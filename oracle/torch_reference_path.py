"""Torch CPU restatement of the reference's PyTorch forward path.

TEST / BASELINE INFRASTRUCTURE ONLY: ``bench.py`` times this as the CPU
baseline (``cpu_baseline`` key and ``--impl reference``) and tests may use it
as a second checker.  The product never imports it.

It follows the reference's own CPU code path step by step, in the
activation dtype as the reference does:

* ``Linear._prep_activation`` (``_ops.py:337-365``): ``x / smoothrot``, then
  ``rotate_activations`` (``_quant_utils.py:117-147``: pad, reshape to
  ``[-1, G, rot]``, ``@ H.T`` in the activation dtype), pad to ``w_in``,
  ``x[..., perm]``;
* INT4 PyTorch path ``_forward_int4_pytorch`` (``_ops.py:483-491``): full
  dequantisation ``unpacked.float() * scale`` (``quant_layout.py:81-87``; here
  with the group-128 scale semantics of ``_quant_utils.py:255-270``, since the
  reference's own reshape(-1, 1) rejects ``[N, G>1]`` scales), cast to the
  activation dtype, ``F.linear`` without bias;
* INT8 PyTorch path (``_ops.py:537-545``): ``q.to(dt) * scale.to(dt)`` and
  ``F.linear`` with bias.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _hadamard(n: int, dtype: torch.dtype) -> torch.Tensor:
    if n >= 4 and (n & (n - 1)) == 0 and (n & 0x55555555) == n:
        H4 = torch.tensor([[1.0, 1.0, 1.0, -1.0], [1.0, 1.0, -1.0, 1.0], [1.0, -1.0, 1.0, 1.0],
                           [-1.0, 1.0, 1.0, 1.0]], dtype=dtype) / 2.0
        H = H4
        while H.shape[0] < n:
            H = torch.kron(H, H4)
        return H
    H = torch.tensor([[1.0]], dtype=dtype)
    while H.shape[0] < n:
        H = torch.kron(torch.tensor([[1.0, 1.0], [1.0, -1.0]], dtype=dtype), H)
    return H * (1.0 / math.sqrt(n))


def prep(x, smoothrot=None, rot_size=0, w_in=None, perm=None, H=None, smooth=None):
    x2 = x.reshape(-1, x.shape[-1])
    if smoothrot is not None:
        x2 = x2 / smoothrot.to(x2.dtype)
    if rot_size:
        K = x2.shape[-1]
        if K % rot_size:
            x2 = F.pad(x2, (0, rot_size - K % rot_size))
        Kp = x2.shape[-1]
        H = _hadamard(rot_size, x2.dtype) if H is None else H
        x2 = torch.matmul(x2.reshape(-1, Kp // rot_size, rot_size), H.T).reshape(-1, Kp)
    if w_in is not None and x2.shape[-1] < w_in:
        x2 = F.pad(x2, (0, w_in - x2.shape[-1]))
    if perm is not None:
        x2 = x2[..., perm]
    if smooth is not None and smoothrot is None:   # INT8 SmoothQuant divide (_ops.py:529-533)
        x2 = x2 / smooth.to(x2.dtype)
    return x2


def unpack_int4(packed: torch.Tensor, K: int) -> torch.Tensor:
    low = (packed & 0x0F).to(torch.int8)
    high = ((packed >> 4) & 0x0F).to(torch.int8)
    low = torch.where(low >= 8, low - 16, low)
    high = torch.where(high >= 8, high - 16, high)
    out = torch.empty(*packed.shape[:-1], packed.shape[-1] * 2, dtype=torch.int8)
    out[..., 0::2] = low
    out[..., 1::2] = high
    return out[..., :K]


def dequant_int4(packed, scale, K, group_size):
    q = unpack_int4(packed, K).float()
    s = scale.float()
    if s.dim() == 1 or s.shape[1] == 1:
        return q * s.reshape(-1, 1)
    return (q.reshape(q.shape[0], -1, group_size) * s.unsqueeze(2)).reshape(q.shape[0], -1)[:, :K]


def forward_int4_pytorch(x, packed, scale, K, group_size, **prep_kw):
    w = dequant_int4(packed, scale, K, group_size).to(x.dtype)
    return F.linear(prep(x, **prep_kw), w)


def forward_int8_pytorch(x, q, scale, bias=None, **prep_kw):
    w = q.to(x.dtype) * scale.reshape(-1, 1).to(x.dtype)
    return F.linear(prep(x, **prep_kw), w, bias)
