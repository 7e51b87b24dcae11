"""CPU oracle for the INT-Crush quantized-linear forward path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this file:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use it, and only as the checker (or as the timed CPU restatement).

Every function restates, in numpy, one piece of the reference's arithmetic
(ComfyUI-INT-Crush; paths below are relative to that project):

* ``hadamard_regular``      -- ``_quant_utils.py:67-93`` (kron of H4/2)
* ``hadamard_sylvester``    -- ``_quant_utils.py:96-114`` (kron of [[1,1],[1,-1]], * 1/sqrt(n))
* ``rotate``                -- ``_quant_utils.py:117-147`` (pad to rot multiple, x_g @ H^T)
* ``prep_activation``       -- ``_ops.py:337-365`` + the INT8-only smooth divide ``_ops.py:529-533``
* ``quantize_rows``         -- ``kernels/triton_quantize.py:43-54`` (CPU form, round half-even)
* ``pack_int4/unpack_int4`` -- ``_quant_utils.py:170-197``
* ``gemm_a8``               -- ``kernels/triton_int8_gemm.py:96-117`` (int32 acc * s_a * s_w + bias),
                               with group scales following ``_quant_utils.py:255-270``
* ``dequant_int4_f16``      -- ``quant_layout.py:81-87`` / ``kernels/triton_int4_unpack.py:48-56``
* ``lora_residual``         -- ``_ops.py:236-244``

Exactness choices (the reference's own arithmetic is order-dependent in a few
places; the oracle pins the mathematically exact value):

* The block-Hadamard rotation runs in the activation dtype (fp16) in the
  reference (``_quant_utils.py:145``); its matmul accumulates in fp32 in an
  unspecified order.  The oracle computes the exact sum in float64 (sums of
  at most 4096 fp16 values times +-1 are exact in 53 bits) and rounds once to
  fp16.  The reference agrees with this except for values within a few fp32
  ulps of an fp16 rounding midpoint; tests/golden pins the agreement on the
  reference's own outputs.
* Quantisation: ``s = max(amax, 1e-8) / 127`` in fp32, ``q = clamp(rint(x / s))``
  with IEEE division and round-half-to-even, exactly the CPU path
  ``kernels/triton_quantize.py:52-53``.
* Integer GEMM accumulators are exact (float64 matmul of int8 values is
  exact below 2^53).
"""

from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------
# Hadamard matrices
# ---------------------------------------------------------------------------

_H4 = np.array(
    [[1, 1, 1, -1],
     [1, 1, -1, 1],
     [1, -1, 1, 1],
     [-1, 1, 1, 1]], dtype=np.float64)


def is_power_of_two(n: int) -> bool:
    return n > 0 and (n & (n - 1)) == 0


def is_power_of_four(n: int) -> bool:
    # _quant_utils.py:49-61
    return n >= 4 and is_power_of_two(n) and (n & 0x55555555) == n


def hadamard_regular(n: int) -> np.ndarray:
    """H = kron(H4/2, H4/2, ...) as float64 (entries +-2^-k, exact in fp16)."""
    if not is_power_of_four(n):
        raise ValueError(f"regular Hadamard needs a power of 4, got {n}")
    H = _H4 / 2.0
    while H.shape[0] < n:
        H = np.kron(H, _H4 / 2.0)
    return H


def sylvester_entry(n: int) -> float:
    """The magnitude of a Sylvester entry as the reference stores it: the fp16
    tensor of +-1 is multiplied by the Python float 1/sqrt(n) (computed in
    fp32 opmath, rounded to fp16), ``_quant_utils.py:112``."""
    return float(np.float16(np.float32(1.0 / math.sqrt(n))))


def hadamard_sylvester(n: int) -> np.ndarray:
    if not is_power_of_two(n):
        raise ValueError(f"n must be a power of 2, got {n}")
    H = np.ones((1, 1))
    W2 = np.array([[1.0, 1.0], [1.0, -1.0]])
    while H.shape[0] < n:
        H = np.kron(W2, H)
    return H * sylvester_entry(n)


def hadamard(n: int) -> np.ndarray:
    return hadamard_regular(n) if is_power_of_four(n) else hadamard_sylvester(n)


# ---------------------------------------------------------------------------
# Activation prep
# ---------------------------------------------------------------------------

def f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64).astype(np.float16)


def bf16(a) -> np.ndarray:
    """Round to bfloat16 (nearest, ties to even) directly from float64, returned
    as float32 values (numpy has no bfloat16 dtype).  bf16 keeps 8 significant
    bits; frexp's mantissa in [0.5, 1) times 2^8 is rounded half-even by rint.
    Subnormal and overflowing values are outside what the tests feed it."""
    x = np.asarray(a, dtype=np.float64)
    m, e = np.frexp(x)
    return np.ldexp(np.rint(np.ldexp(m, 8)), e - 8).astype(np.float32)


def round_act(a, act: str = "f16") -> np.ndarray:
    """Round float64 values to the activation dtype: fp16 (as float16) or
    bf16 (as float32 holding bf16 values)."""
    return f16(a) if act == "f16" else bf16(a)


def div_f16(x16: np.ndarray, d, act: str = "f16") -> np.ndarray:
    """Activation tensor divided by a vector cast to the activation dtype, as
    ``x / f.to(x.dtype)``: the quotient is correctly rounded to that dtype
    (fp64 then fp16/bf16 is a safe double rounding for division)."""
    d_act = round_act(np.asarray(d, dtype=np.float32), act)
    return round_act(np.asarray(x16, np.float64) / np.asarray(d_act, np.float64), act)


def rotate(x16: np.ndarray, rot_size: int, act: str = "f16") -> np.ndarray:
    """``rotate_activations`` (``_quant_utils.py:117-147``) with an exact sum."""
    if not is_power_of_two(rot_size):
        raise ValueError(f"rot_size must be power of 2, got {rot_size}")
    M, K = x16.shape
    Kp = -(-K // rot_size) * rot_size
    xp = np.zeros((M, Kp), dtype=np.float64)
    xp[:, :K] = np.asarray(x16, np.float64)
    H = hadamard(rot_size)
    y = xp.reshape(M, Kp // rot_size, rot_size) @ H.T
    return round_act(y.reshape(M, Kp), act)


def prep_activation(x16, *, smoothrot=None, rot_need=False, rot_size=0, w_in=None,
                    perm=None, smooth=None, int8_path=True, act: str = "f16") -> np.ndarray:
    """``Linear._prep_activation`` (``_ops.py:337-365``) plus the INT8 smooth
    divide that only applies when there are no SmoothRot factors
    (``_ops.py:529-533``).  ``act`` = "f16" (input and result float16) or
    "bf16" (input and result float32 arrays holding bf16 values)."""
    adt = np.float16 if act == "f16" else np.float32
    x = np.asarray(x16, dtype=adt).reshape(-1, np.shape(x16)[-1])
    if smoothrot is not None:
        x = div_f16(x, smoothrot, act)
    if rot_need:
        x = rotate(x, rot_size, act)
    if w_in is not None and x.shape[1] < w_in:
        x = np.concatenate([x, np.zeros((x.shape[0], w_in - x.shape[1]), adt)], 1)
    if perm is not None:
        x = x[:, np.asarray(perm, dtype=np.int64)]
    if int8_path and smoothrot is None and smooth is not None:
        x = div_f16(x, smooth, act)
    return x


def layer_norm_rows(x, gamma, beta=None, eps=1e-5, out_dtype=np.float16) -> np.ndarray:
    """CPU form of ``fused_layernorm_quantize``'s normalisation
    (``kernels/triton_quantize.py:316-321``): ``F.layer_norm`` in fp32 (here in
    fp64, then rounded to fp32), cast to the activation dtype."""
    xf = np.asarray(x, np.float64)
    mean = xf.mean(axis=1, keepdims=True)
    var = ((xf - mean) ** 2).mean(axis=1, keepdims=True)
    y = (xf - mean) / np.sqrt(var + eps) * np.asarray(gamma, np.float64)
    if beta is not None:
        y = y + np.asarray(beta, np.float64)
    return y.astype(np.float32).astype(out_dtype)


def rms_norm_rows(x, gamma, eps=1e-6, out_dtype=np.float16) -> np.ndarray:
    """CPU form of ``fused_rmsnorm_quantize`` (``kernels/triton_quantize.py:430-435``)."""
    xf = np.asarray(x, np.float64)
    rms = np.sqrt((xf * xf).mean(axis=1, keepdims=True) + eps)
    return (xf / rms * np.asarray(gamma, np.float64)).astype(np.float32).astype(out_dtype)


def quantize_rows(x16: np.ndarray):
    """Per-token symmetric INT8 (``kernels/triton_quantize.py:43-54``)."""
    xf = np.asarray(x16).astype(np.float32)
    amax = np.abs(xf).max(axis=1) if xf.shape[1] else np.zeros(xf.shape[0], np.float32)
    s = np.maximum(amax, np.float32(1e-8)).astype(np.float32) / np.float32(127.0)
    q = np.rint(xf / s[:, None]).clip(-128, 127).astype(np.int8)
    return q, s.astype(np.float32)


# ---------------------------------------------------------------------------
# INT4 packing
# ---------------------------------------------------------------------------

def pack_int4(q: np.ndarray) -> np.ndarray:
    """Low nibble = even k, two's complement (``_quant_utils.py:170-182``)."""
    q = np.asarray(q, dtype=np.int8)
    if q.min(initial=0) < -8 or q.max(initial=0) > 7:
        raise ValueError("values must be in [-8, 7]")
    if q.shape[-1] % 2:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (1,), np.int8)], -1)
    u = (q.astype(np.int16) & 0xF).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(p: np.ndarray, K: int) -> np.ndarray:
    """``_quant_utils.py:185-197``."""
    p = np.asarray(p, dtype=np.uint8)
    lo = (p & 0xF).astype(np.int8)
    hi = (p >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo).astype(np.int8)
    hi = np.where(hi >= 8, hi - 16, hi).astype(np.int8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out[..., :K]


# ---------------------------------------------------------------------------
# GEMMs
# ---------------------------------------------------------------------------

def int_accumulators(xq: np.ndarray, wq: np.ndarray, group_size: int | None = None) -> np.ndarray:
    """Exact int32 accumulators ``[G, M, N]`` of ``xq @ wq^T`` per K-group."""
    M, K = xq.shape
    gs = K if group_size is None else group_size
    G = -(-K // gs)
    out = np.empty((G, M, wq.shape[0]), np.int64)
    for g in range(G):
        a = xq[:, g * gs:(g + 1) * gs].astype(np.float64)
        b = wq[:, g * gs:(g + 1) * gs].astype(np.float64)
        out[g] = (a @ b.T).astype(np.int64)
    return out


def gemm_a8(xq, s_a, wq, s_w, bias=None, group_size=None) -> np.ndarray:
    """``out = s_a[m] * sum_g s_w[n,g] * P_g[m,n] + bias[n]`` in float64.

    ``s_w`` is ``[N]`` (per channel, the W8A8 / per-row W4A8 form of
    ``kernels/triton_int8_gemm.py:105-117``) or ``[N, G]`` (the group form
    defined by ``_quant_utils.py:255-270``).
    """
    s_w = np.asarray(s_w, np.float64)
    if s_w.ndim == 1 or (s_w.ndim == 2 and s_w.shape[1] == 1):
        P = int_accumulators(xq, wq)[0].astype(np.float64)
        acc = P * s_w.reshape(1, -1)
    else:
        G = s_w.shape[1]
        gs = group_size if group_size is not None else -(-xq.shape[1] // G)
        P = int_accumulators(xq, wq, gs).astype(np.float64)
        acc = np.einsum("gmn,ng->mn", P, s_w)
    out = acc * np.asarray(s_a, np.float64)[:, None]
    if bias is not None:
        out = out + np.asarray(bias, np.float64)[None, :]
    return out


def dequant_int4_f16(packed, scale, K: int, group_size: int | None = None) -> np.ndarray:
    """fp16 weights ``fp16(q * s[n, k // gs])`` (``quant_layout.py:81-87`` for one
    group; ``_quant_utils.py:255-270`` for several)."""
    q = unpack_int4(packed, K).astype(np.float64)
    s = np.asarray(scale, np.float64)
    if s.ndim == 1:
        s = s[:, None]
    G = s.shape[1]
    gs = group_size if group_size is not None else -(-K // G)
    s_full = np.repeat(s, gs, axis=1)[:, :K]
    return (q * s_full).astype(np.float32).astype(np.float16)


def linear_f16(x16, w16, bias=None) -> np.ndarray:
    """``F.linear`` in fp16 with fp32-or-better accumulation, as float64."""
    out = np.asarray(x16, np.float64) @ np.asarray(w16, np.float64).T
    if bias is not None:
        out = out + np.asarray(bias, np.float64)[None, :]
    return out


def lora_mid(x_raw16, down16) -> np.ndarray:
    """``mid = F.linear(x_raw, down)`` rounded to fp16 (``_ops.py:242``)."""
    return linear_f16(x_raw16, down16).astype(np.float16)


def lora_residual(x_raw16, down16, up16, scale: float) -> np.ndarray:
    """``scale * mid @ up^T`` (``_ops.py:243``), float64."""
    mid = lora_mid(x_raw16, down16).astype(np.float64)
    return scale * (mid @ np.asarray(up16, np.float64).T)


def max_rel(y, y_ref) -> float:
    """``max|y - y_ref| / max|y_ref|`` -- the tolerance metric of the parity tests."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    den = max(np.abs(y_ref).max(initial=0.0), 1e-30)
    return float(np.abs(y - y_ref).max(initial=0.0) / den)
