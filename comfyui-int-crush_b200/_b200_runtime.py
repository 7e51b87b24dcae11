"""B200 kernel runtime: the drop-in replacement of ``_triton_runtime``.

Exports the same module attributes as the reference's
``_triton_runtime.py:16-41,114-130`` -- the availability flags
``TRITON_AVAILABLE, TRITON_INT4_UNPACK, TRITON_INT8_GEMM,
TRITON_INT4_INT8_UNPACK, TRITON_DYNQUANT, TRITON_W4A8_GEMM, TRITON_FUSED_QGD``,
the toggles ``USE_FUSED_W8A8`` and ``USE_CUDA_GRAPHS`` (env
``INTCRUSH_NO_CUDA_GRAPHS=1`` disables graphs, ``_triton_runtime.py:60-61``) and
the six kernel callables with their signatures -- but every callable runs the
hand-written sm_100a kernels of ``libintcrush_b200.so``.  A flag is True when
the library loaded and a CUDA device is present.  There is no CPU fallback:
an op given CPU tensors, or called while the library is missing, raises.

New fused ops beyond the reference's set: ``prep_quantize`` (SmoothRot +
Hadamard + pad + PermuQuant + smooth + per-token INT8 in one pass),
``gemm_a8`` (W8A8 / W4A8 with per-channel or group scales, bias and the
zero-point term fused), ``gemm_w4a16`` (weight-streaming W4A16 with the
low-rank residual fused), ``lowrank_down`` / ``lowrank_add``.
"""

from __future__ import annotations

import ctypes
import logging
import os

import torch

from . import _lib as L

log = logging.getLogger(__name__)

# ── availability flags (names of the reference runtime) ─────────────────────
try:
    L.lib()
    B200_LIBRARY_LOADED = True
    _load_error: str | None = None
except OSError as exc:  # pragma: no cover - depends on the build
    B200_LIBRARY_LOADED = False
    _load_error = str(exc)

B200_AVAILABLE = B200_LIBRARY_LOADED and torch.cuda.is_available()

TRITON_AVAILABLE = B200_AVAILABLE
TRITON_INT4_UNPACK = B200_AVAILABLE
TRITON_INT8_GEMM = B200_AVAILABLE
TRITON_INT4_INT8_UNPACK = B200_AVAILABLE
TRITON_DYNQUANT = B200_AVAILABLE
TRITON_W4A8_GEMM = B200_AVAILABLE
TRITON_FUSED_QGD = B200_AVAILABLE

USE_FUSED_W8A8: bool = False
USE_CUDA_GRAPHS: bool = True
if os.environ.get("INTCRUSH_NO_CUDA_GRAPHS", "0") == "1":
    USE_CUDA_GRAPHS = False

_DT = {torch.float16: L.IC_DTYPE_F16, torch.bfloat16: L.IC_DTYPE_BF16, torch.float32: L.IC_DTYPE_F32}


def _p(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need_cuda(what: str, *ts: torch.Tensor | None) -> None:
    if not B200_LIBRARY_LOADED:
        raise RuntimeError(f"{what}: libintcrush_b200.so is not loaded ({_load_error})")
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{what}: intcrush_b200 ops run on CUDA tensors only (got {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on different devices ({dev}, {t.device})")


def _f32c(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    return t.to(torch.float32).contiguous()


def _round16(n: int) -> int:
    return (n + 15) // 16 * 16


# ── activation prep ──────────────────────────────────────────────────────────

def prep_quantize(
    x: torch.Tensor,
    *,
    smoothrot: torch.Tensor | None = None,
    rot_size: int = 0,
    w_in: int | None = None,
    perm: torch.Tensor | None = None,
    smooth: torch.Tensor | None = None,
    quantize: bool = True,
    want_prep: bool = False,
    want_rowsum: bool = False,
    s_a_out: torch.Tensor | None = None,
    x_int8_out: torch.Tensor | None = None,
    x_prep_out: torch.Tensor | None = None,
    norm: tuple | None = None,
):
    """One-pass activation prep (``_ops.py:337-365`` + ``_ops.py:529-533``) and
    per-token INT8 quantisation (``kernels/triton_quantize.py:151-198``).

    ``norm`` = ``("layer", gamma, beta_or_None, eps)`` or ``("rms", gamma,
    None, eps)`` normalises each row first (fp32 statistics, one rounding to
    x's dtype), in the same pass (``ic_prep_quant_norm``).

    Returns ``(x_int8, s_a, x_prep, rowsum)``; entries not requested are None.
    ``x_int8`` is ``[M, w_in]`` (a view of a buffer whose row stride is w_in
    rounded up to 16 bytes; the padding columns hold zeros).
    """
    _need_cuda("prep_quantize", x, smoothrot, perm, smooth)
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if x2.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"prep_quantize: x must be float16/bfloat16, got {x2.dtype}")
    M, K = x2.shape
    Kr = K if not rot_size else -(-K // rot_size) * rot_size
    w_in = Kr if w_in is None else max(int(w_in), Kr)
    # the kernel indexes these vectors without bounds checks: check lengths here
    if smoothrot is not None and smoothrot.numel() != K:
        raise ValueError(f"prep_quantize: smoothrot has {smoothrot.numel()} entries, expected K={K}")
    if perm is not None and perm.numel() != w_in:
        raise ValueError(f"prep_quantize: perm has {perm.numel()} entries, expected w_in={w_in}")
    if smooth is not None and smooth.numel() != w_in:
        raise ValueError(f"prep_quantize: smooth has {smooth.numel()} entries, expected w_in={w_in}")
    if perm is not None and perm.dtype != torch.int32:
        perm = perm.to(torch.int32)
    perm = None if perm is None else perm.contiguous()
    x_int8 = s_a = x_prep = rowsum = None
    xq_full = None
    if quantize:
        ldq = _round16(w_in)
        if x_int8_out is not None:
            xq_full = x_int8_out
            if xq_full.shape[0] != M or xq_full.stride(0) < w_in or xq_full.dtype != torch.int8:
                raise ValueError("prep_quantize: x_int8_out must be int8 [M, >= w_in]")
        else:
            xq_full = torch.empty((M, ldq), dtype=torch.int8, device=x.device)
        s_a = s_a_out if s_a_out is not None else torch.empty(M, dtype=torch.float32, device=x.device)
        x_int8 = xq_full[:, :w_in]
    if want_prep:
        x_prep = x_prep_out if x_prep_out is not None else torch.empty((M, w_in), dtype=x2.dtype, device=x.device)
    if want_rowsum:
        rowsum = torch.empty(M, dtype=torch.float32, device=x.device)
    sr = _f32c(smoothrot)
    sm = _f32c(smooth)
    if norm is not None:
        kind, gamma, beta, eps = norm
        code = {"layer": 1, "rms": 2}[kind]
        if sm is not None:
            raise ValueError("prep_quantize: a norm with SmoothQuant factors is not supported")
        g = _f32c(gamma.reshape(-1))
        b = None if beta is None else _f32c(beta.reshape(-1))
        if g.numel() != K or (b is not None and b.numel() != K):
            raise ValueError("prep_quantize: gamma / beta must have K entries")
        _need_cuda("prep_quantize", g, b)
        st = L.lib().ic_prep_quant_norm(
            _p(x2), _DT[x2.dtype], M, K, x2.stride(0), code, _p(g), _p(b), float(eps), _p(sr), int(rot_size), w_in,
            _p(perm), _p(xq_full), xq_full.stride(0) if xq_full is not None else 0, _p(s_a), _p(x_prep),
            _p(rowsum), _stream(x2))
        L.check(st, "ic_prep_quant_norm")
        return x_int8, s_a, x_prep, rowsum
    st = L.lib().ic_prep_quant(
        _p(x2), _DT[x2.dtype], M, K, x2.stride(0), _p(sr), int(rot_size), w_in, _p(perm), _p(sm),
        _p(xq_full), xq_full.stride(0) if xq_full is not None else 0, _p(s_a), _p(x_prep), _p(rowsum),
        _stream(x2))
    L.check(st, "ic_prep_quant")
    return x_int8, s_a, x_prep, rowsum


def dynamic_quantize_activation(
    x: torch.Tensor,
    s_a_out: torch.Tensor | None = None,
    x_int8_out: torch.Tensor | None = None,
):
    """``kernels/triton_quantize.py:151-198``: per-token symmetric INT8.

    Rounding is half-to-even with IEEE division (the reference's CPU form,
    ``kernels/triton_quantize.py:43-54``).  Leading dimensions are restored
    like ``_reshape_if_needed``.
    """
    orig = x.shape
    x2 = x.reshape(-1, orig[-1])
    if s_a_out is not None and s_a_out.shape != (x2.shape[0],):
        s_a_out = None
    if x_int8_out is not None and x_int8_out.shape != x2.shape:
        x_int8_out = None
    x_int8, s_a, _, _ = prep_quantize(x2, s_a_out=s_a_out, x_int8_out=x_int8_out)
    if len(orig) > 2:
        x_int8 = x_int8.reshape(orig)
        s_a = s_a.reshape(orig[:-1])
    return x_int8, s_a


def _norm_quantize(x, norm, s_a_out, x_int8_out):
    orig = x.shape
    x2 = x.reshape(-1, orig[-1])
    if s_a_out is not None and s_a_out.shape != (x2.shape[0],):
        s_a_out = None
    if x_int8_out is not None and x_int8_out.shape != x2.shape:
        x_int8_out = None
    x_int8, s_a, _, _ = prep_quantize(x2, norm=norm, s_a_out=s_a_out, x_int8_out=x_int8_out)
    if len(orig) > 2:
        x_int8 = x_int8.reshape(orig)
        s_a = s_a.reshape(orig[:-1])
    return x_int8, s_a


def fused_layernorm_quantize(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor | None = None,
                             eps: float = 1e-5, s_a_out: torch.Tensor | None = None,
                             x_int8_out: torch.Tensor | None = None):
    """``kernels/triton_quantize.py:274-338``: LayerNorm + per-row INT8 in one
    pass.  Follows the reference's CPU form: normalised values are cast to
    x's dtype (fp16/bf16), then quantised half-to-even."""
    return _norm_quantize(x, ("layer", gamma, beta, eps), s_a_out, x_int8_out)


def fused_rmsnorm_quantize(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-6,
                           s_a_out: torch.Tensor | None = None, x_int8_out: torch.Tensor | None = None):
    """``kernels/triton_quantize.py:395-451``: RMSNorm + per-row INT8 in one pass
    (CPU form: ``x / sqrt(mean(x^2) + eps) * gamma`` cast to x's dtype)."""
    return _norm_quantize(x, ("rms", gamma, None, eps), s_a_out, x_int8_out)


# ── GEMMs ────────────────────────────────────────────────────────────────────

def gemm_a8(
    x_int8: torch.Tensor,
    w: torch.Tensor,
    s_w: torch.Tensor,
    s_a: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
    group_size: int | None = None,
    rowsum: torch.Tensor | None = None,
    zp_corr: torch.Tensor | None = None,
    repacked: bool = False,
    splits: int | None = None,
    activation: int = 0,
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """``out = s_a[m] * sum_g s_w[n,g] * (xq @ w^T)_g + bias - rowsum (x) zp_corr``.

    ``activation`` (0 none, 1 SiLU, 2 GELU erf, 3 GELU tanh) and then
    ``residual`` ([M, N], any float dtype, unit column stride) are applied in
    fp32 in the epilogue before the output cast.

    ``w`` is int8 ``[N, K]`` or packed INT4 uint8 ``[N, K/2]``; ``s_w`` is
    ``[N]``/``[N,1]`` (per channel) or ``[N, G]`` (groups of ``group_size``,
    default ``ceil(K / G)`` rounded to a multiple of 128).

    ``splits`` cuts K into that many parts run as separate work units (split-K,
    fp32 partials in a workspace allocated here, then a reduce kernel); None
    picks it from the tile count so that small-M calls fill the GPU
    (``INTCRUSH_SPLITK=0`` turns that off).
    """
    _need_cuda("gemm_a8", x_int8, w, s_w, s_a, bias, out, rowsum, zp_corr)
    if x_int8.dtype != torch.int8:
        raise AssertionError(f"x_int8 must be int8, got {x_int8.dtype}")
    M, K = x_int8.shape
    if x_int8.stride(1) != 1:
        x_int8 = x_int8.contiguous()
    if w.dtype == torch.int8:
        kind = L.IC_W_INT8
        N = w.shape[0]
        if w.shape[1] != K:
            raise AssertionError(f"K mismatch: {K} vs {w.shape[1]}")
    elif w.dtype == torch.uint8:
        kind = L.IC_W_INT4R if repacked else L.IC_W_INT4
        N = w.shape[0]
        if w.shape[1] != (K + 1) // 2:
            raise AssertionError(f"packed K mismatch: {K} vs {w.shape[1]} bytes")
    else:
        raise AssertionError(f"w must be int8 or uint8 (packed int4), got {w.dtype}")
    if w.stride(1) != 1:
        w = w.contiguous()
    sw = s_w.to(torch.float32)
    if sw.dim() == 1:
        sw = sw.reshape(N, -1)
    sw = sw.reshape(N, -1).contiguous()
    G = sw.shape[1]
    if G > 1 and group_size is None:
        group_size = -(-K // G)
    gs = int(group_size) if G > 1 else K
    sa = s_a.to(torch.float32).contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=x_int8.device)
    elif out.shape != (M, N) or out.stride(1) != 1:
        raise AssertionError(f"out shape mismatch: {tuple(out.shape)} vs ({M}, {N})")
    b = None if bias is None else bias.contiguous()
    rs = _f32c(rowsum)
    zc = _f32c(zp_corr)
    if splits is None:
        splits = _auto_splits(M, N, K, G, gs, x_int8.device, kind != L.IC_W_INT8)
    if activation or residual is not None:
        r = residual
        if r is not None:
            if r.shape != (M, N):
                raise AssertionError(f"residual shape mismatch: {tuple(r.shape)} vs ({M}, {N})")
            _need_cuda("gemm_a8", r)
            if r.stride(1) != 1:
                r = r.contiguous()
        ws = torch.empty(splits * M * N if splits > 1 else 0, dtype=torch.float32, device=x_int8.device)
        st = L.lib().ic_gemm_a8_ex(
            _p(x_int8), M, K, x_int8.stride(0), _p(w), kind, N, w.stride(0), _p(sw), G, gs, _p(sa),
            _p(b), _DT[b.dtype] if b is not None else 0, _p(rs), _p(zc), int(activation),
            _p(r), _DT[r.dtype] if r is not None else 0, r.stride(0) if r is not None else 0,
            _p(out), _DT[out.dtype], out.stride(0), int(splits), _p(ws) if splits > 1 else None, ws.numel(),
            _stream(x_int8))
        L.check(st, "ic_gemm_a8_ex")
        return out
    if splits > 1:
        ws = torch.empty(splits * M * N, dtype=torch.float32, device=x_int8.device)
        st = L.lib().ic_gemm_a8_splitk(
            _p(x_int8), M, K, x_int8.stride(0), _p(w), kind, N, w.stride(0), _p(sw), G, gs, _p(sa),
            _p(b), _DT[b.dtype] if b is not None else 0, _p(rs), _p(zc), _p(out), _DT[out.dtype], out.stride(0),
            int(splits), _p(ws), ws.numel(), _stream(x_int8))
        L.check(st, "ic_gemm_a8_splitk")
        return out
    st = L.lib().ic_gemm_a8(
        _p(x_int8), M, K, x_int8.stride(0), _p(w), kind, N, w.stride(0), _p(sw), G, gs, _p(sa),
        _p(b), _DT[b.dtype] if b is not None else 0, _p(rs), _p(zc), _p(out), _DT[out.dtype], out.stride(0),
        _stream(x_int8))
    L.check(st, "ic_gemm_a8")
    return out


_SMS: dict = {}


def _num_sms(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def _auto_splits(M: int, N: int, K: int, G: int, gs: int, device: torch.device, int4: bool) -> int:
    """Split-K factor for ``gemm_a8``: 1 unless the output tiles cover less
    than half of the SMs; then the largest divisor of the K-block count (and
    of G for group scales) that keeps at least 4 K blocks per part and the
    work units within one wave."""
    if os.environ.get("INTCRUSH_SPLITK", "1") == "0":
        return 1
    grouped = G > 1
    # token-tile width as the library picks it (pick_bn in gemm_tc.cu)
    sms = _num_sms(device)
    bn = 32 if M <= 32 else 64 if M <= 64 else 128 if M <= 128 else (192 if grouped else 256)
    while bn > 64 and -(-M // bn) * -(-N // 128) * 2 < sms:
        bn = 128 if bn > 128 else 64
    tiles = -(-M // bn) * -(-N // 128)
    if tiles * 2 > sms:
        return 1
    nkb = -(-K // 128)
    best = 1
    for d in range(2, 17):
        if nkb % d or nkb // d < 4:
            continue
        if grouped and (K % gs or G % d):
            continue
        if tiles * d <= sms:
            best = d
    return best


def fused_int8_gemm_dequant(
    x_int8: torch.Tensor,
    w_int8: torch.Tensor,
    s_w: torch.Tensor,
    s_a: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    activation: int = 0,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``kernels/triton_int8_gemm.py:135-205`` on tcgen05 (kind::i8), with
    the reference's epilogue: ``activation`` 0 none, 1 SiLU, 2 GELU (erf),
    plus 3 GELU with the tanh approximation; then ``+ residual``."""
    if activation not in (0, 1, 2, 3):
        raise ValueError(f"activation must be 0, 1, 2 or 3, got {activation}")
    return gemm_a8(x_int8, w_int8, s_w, s_a, bias=bias, out_dtype=out_dtype, out=out, activation=activation,
                   residual=residual)


def int8_gemm_int8out(
    x_int8: torch.Tensor,
    w_int8: torch.Tensor,
    s_w: torch.Tensor,
    s_a: torch.Tensor,
    c_out: torch.Tensor | None = None,
    s_c_out: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    activation: int = 0,
    group_size: int | None = None,
    repacked: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``kernels/triton_int8_gemm.py:472-536``: a GEMM whose output is
    re-quantised to int8 for the next GEMM of a chain (``s_c`` feeds it as
    ``s_a``).

    The scale is row-global: ``s_c[m] = max(max_n |y[m, n]|, 1e-8) / 127``
    over the whole output row, ``c = rint(y / s_c)`` (ties to even), so that
    ``(c, s_c)`` equals ``dynamic_quantize_activation`` of the fp32 output,
    which the reference's docstring promises.  (The reference kernel takes
    the max over one BLOCK_N tile and lets the tiles of a row race on
    ``s_c``.)  Weights may be int8 or packed INT4 (``group_size`` /
    ``repacked`` as in :func:`gemm_a8`).
    """
    _need_cuda("int8_gemm_int8out", x_int8, w_int8, s_w, s_a, c_out, s_c_out, bias)
    if x_int8.dtype != torch.int8:
        raise AssertionError(f"x_int8 must be int8, got {x_int8.dtype}")
    M, K = x_int8.shape
    if x_int8.stride(1) != 1:
        x_int8 = x_int8.contiguous()
    if w_int8.dtype == torch.int8:
        kind, N = L.IC_W_INT8, w_int8.shape[0]
        if w_int8.shape[1] != K:
            raise AssertionError(f"K mismatch: {K} vs {w_int8.shape[1]}")
    elif w_int8.dtype == torch.uint8:
        kind, N = (L.IC_W_INT4R if repacked else L.IC_W_INT4), w_int8.shape[0]
        if w_int8.shape[1] != (K + 1) // 2:
            raise AssertionError(f"packed K mismatch: {K} vs {w_int8.shape[1]} bytes")
    else:
        raise AssertionError(f"w must be int8 or uint8 (packed int4), got {w_int8.dtype}")
    w = w_int8 if w_int8.stride(1) == 1 else w_int8.contiguous()
    sw = s_w.to(torch.float32).reshape(N, -1).contiguous()
    G = sw.shape[1]
    if G > 1 and group_size is None:
        group_size = -(-K // G)
    gs = int(group_size) if G > 1 else K
    sa = s_a.to(torch.float32).contiguous()
    if c_out is not None:
        if c_out.shape != (M, N) or c_out.dtype != torch.int8 or c_out.stride(1) != 1:
            raise AssertionError(f"c_out must be int8 [{M}, {N}] with unit column stride")
        c = c_out
    else:
        c = torch.empty((M, N), dtype=torch.int8, device=x_int8.device)
    if s_c_out is not None:
        if s_c_out.shape != (M,) or s_c_out.dtype != torch.float32 or not s_c_out.is_contiguous():
            raise AssertionError(f"s_c_out must be contiguous float32 [{M}]")
        s_c = s_c_out
    else:
        s_c = torch.empty(M, dtype=torch.float32, device=x_int8.device)
    b = None if bias is None else bias.contiguous()
    ws = torch.empty(M * N + M, dtype=torch.float32, device=x_int8.device)
    st = L.lib().ic_gemm_a8_int8out(
        _p(x_int8), M, K, x_int8.stride(0), _p(w), kind, N, w.stride(0), _p(sw), G, gs, _p(sa),
        _p(b), _DT[b.dtype] if b is not None else 0, int(activation), _p(c), c.stride(0), _p(s_c),
        _p(ws), ws.numel(), _stream(x_int8))
    L.check(st, "ic_gemm_a8_int8out")
    return c, s_c


def fused_w4a8_gemm_dequant(
    x_int8: torch.Tensor,
    w_int8: torch.Tensor,
    s_w: torch.Tensor,
    s_a: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``kernels/triton_w4a8_gemm.py:111-169``.  Accepts the unpacked int8
    weights of the reference or, without materialising them, packed INT4."""
    return gemm_a8(x_int8, w_int8, s_w, s_a, bias=bias, out_dtype=out_dtype, out=out)


def fused_quant_int8_gemm_dequant(
    x_fp16: torch.Tensor,
    w_int8: torch.Tensor,
    s_w: torch.Tensor,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``kernels/triton_int8_gemm.py:331-389``: quantise + GEMM + dequant."""
    if x_fp16.dtype not in (torch.float16, torch.bfloat16):
        raise AssertionError(f"x must be fp16/bf16, got {x_fp16.dtype}")
    x_int8, s_a, _, _ = prep_quantize(x_fp16)
    if out is not None and out.shape != (x_int8.shape[0], w_int8.shape[0]):
        out = None
    return gemm_a8(x_int8, w_int8, s_w, s_a, bias=bias, out_dtype=out_dtype, out=out)


def gemm_w4a16(
    x: torch.Tensor,
    packed: torch.Tensor,
    scale: torch.Tensor,
    group_size: int | None = None,
    bias: torch.Tensor | None = None,
    lr_mid: torch.Tensor | None = None,
    lr_up: torch.Tensor | None = None,
    lr_scale: float = 1.0,
    out: torch.Tensor | None = None,
    K: int | None = None,
    w_layout: int = 0,
    splits: int | None = None,
) -> torch.Tensor:
    """W4A16: ``T(x @ W^T (+ bias))`` then ``+= lr_scale * lr_mid @ lr_up^T``,
    T = x's dtype.  fp16: ``W = fp16(q * fp16(s))`` (the Triton unpack's
    product); bf16: ``W = bf16(q * s)`` from the fp32 product (the PyTorch
    path's dequantisation cast to the activation dtype).

    ``splits`` (M > 128 only): K parts run as separate work units with fp32
    partials in a workspace allocated here; None picks the count that fills
    the SMs (token tiles of 128), 1 runs unsplit.

    Replaces ``unpack_int4_to_float16`` + ``F.linear`` (``_ops.py:473-474``)
    and the PyTorch INT4 path (``_ops.py:483-491``).
    """
    _need_cuda("gemm_w4a16", x, packed, scale, bias, lr_mid, lr_up, out)
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"gemm_w4a16: activations must be float16 or bfloat16, got {x.dtype}")
    x2 = x if x.stride(-1) == 1 else x.contiguous()
    M, Kx = x2.shape
    K = Kx if K is None else K
    N = packed.shape[0]
    if packed.dtype != torch.uint8 or packed.shape[1] != (K + 1) // 2:
        raise AssertionError("packed must be uint8 [N, ceil(K/2)]")
    sc = scale.reshape(N, -1)
    if sc.dtype not in (torch.float16, torch.float32):
        sc = sc.to(torch.float32)
    sc = sc.contiguous()
    G = sc.shape[1]
    gs = int(group_size) if (G > 1 and group_size is not None) else (-(-K // G) if G > 1 else K)
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    elif out.dtype != x.dtype:
        raise TypeError("gemm_w4a16: out must have x's dtype")
    b = None if bias is None else bias.contiguous()
    mid = None if lr_mid is None else lr_mid.to(x.dtype).contiguous()
    up = None if lr_up is None else lr_up.to(x.dtype).contiguous()
    R = 0 if mid is None else mid.shape[1]
    if splits is None:
        splits = _w4a16_splits(M, N, K, x.device)
    ws = torch.empty(splits * M * N if (splits > 1 and M > 128) else 0, dtype=torch.float32, device=x.device)
    st = L.lib().ic_gemm_w4a16_splitk(
        _p(x2), _DT[x.dtype], M, K, x2.stride(0), _p(packed), N, packed.stride(0), int(w_layout),
        _p(sc), _DT[sc.dtype],
        G, gs, _p(b), _DT[b.dtype] if b is not None else 0, _p(mid), _p(up), R, float(lr_scale),
        _p(out), out.stride(0), int(splits), _p(ws) if ws.numel() else None, ws.numel(), _stream(x2))
    L.check(st, "ic_gemm_w4a16_splitk")
    return out


def _w4a16_splits(M: int, N: int, K: int, device) -> int:
    """The split count ``ic_gemm_w4a16_splitk`` plans for splits = 0 (token
    tiles of 128, one work unit per SM, at most 8 parts dividing the 64-wide
    K blocks); 1 for the M <= 128 weight-stream kernel."""
    if M <= 128:
        return 1
    tiles = -(-M // 128) * -(-N // 128)
    s = max(1, min(8, _num_sms(device) // max(tiles, 1)))
    nkb = -(-K // 64)
    while s > 1 and nkb % s:
        s -= 1
    return s


def lowrank_down(x: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """``mid = T(x @ down^T)`` (``F.linear(x_raw, down)``, ``_ops.py:242``),
    T = x's dtype (fp16 or bf16; other dtypes compute in fp16)."""
    _need_cuda("lowrank_down", x, down)
    dt = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.float16
    x2 = x.reshape(-1, x.shape[-1]).to(dt)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    d = down.to(dt).contiguous()
    M, K = x2.shape
    R = d.shape[0]
    mid = torch.empty((M, R), dtype=dt, device=x.device)
    L.check(L.lib().ic_lowrank_down_ex(_p(x2), _DT[dt], M, K, x2.stride(0), _p(d), R, _p(mid), _stream(x2)),
            "ic_lowrank_down_ex")
    return mid


def lowrank_add(out: torch.Tensor, mid: torch.Tensor, up: torch.Tensor, scale: float) -> torch.Tensor:
    """In place ``out = T(out + scale * mid @ up^T)`` (``out.addmm_``,
    ``_ops.py:243``); out fp16 or bf16, rank up to 256."""
    _need_cuda("lowrank_add", out, mid, up)
    if out.dtype not in (torch.float16, torch.bfloat16) or out.stride(1) != 1:
        raise TypeError("lowrank_add: out must be a row-major float16 / bfloat16 matrix")
    m = mid.to(out.dtype).contiguous()
    u = up.to(out.dtype).contiguous()
    M, N = out.shape
    L.check(L.lib().ic_lowrank_add_ex(_p(out), _DT[out.dtype], M, N, out.stride(0), _p(m), _p(u), m.shape[1],
                                      float(scale), _stream(out)), "ic_lowrank_add_ex")
    return out


def quantize_weight(w: torch.Tensor, bits: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row requantisation of a float weight on the device (the layout
    classes' ``quantize``, ``quant_layout.py:100-129,179-200``): returns
    (packed uint8 ``[N, ceil(K/2)]``, fp16 scales ``[N]``) for ``bits`` 4 and
    (int8 ``[N, K]``, fp32 scales ``[N]``) for 8."""
    _need_cuda("quantize_weight", w)
    if w.dim() != 2:
        raise AssertionError(f"weight must be 2-D, got {tuple(w.shape)}")
    wf = w.to(torch.float32)
    if wf.stride(1) != 1:
        wf = wf.contiguous()
    N, K = wf.shape
    if bits == 4:
        q = torch.empty((N, (K + 1) // 2), dtype=torch.uint8, device=w.device)
        s = torch.empty(N, dtype=torch.float16, device=w.device)
    elif bits == 8:
        q = torch.empty((N, K), dtype=torch.int8, device=w.device)
        s = torch.empty(N, dtype=torch.float32, device=w.device)
    else:
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    st = L.lib().ic_quantize_weight(_p(wf), N, K, wf.stride(0), int(bits), _p(q), q.stride(0), _p(s), _stream(wf))
    L.check(st, "ic_quantize_weight")
    return q, s


def lokr_add(out: torch.Tensor, x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, scale: float) -> torch.Tensor:
    """``out[t] (viewed [out_l, out_k]) += scale * (w1 @ x[t].view(in_m, in_n)) @ w2^T``
    in place (``_apply_lokr``, ``_ops.py:88-138``): ``w1`` [out_l, in_m],
    ``w2`` [out_k, in_n] (the reference's ``w2_t`` transposed), ``out``
    contiguous [M, out_l * out_k], ``x`` [M, in_m * in_n], all fp16 or bf16.
    The first product is rounded to the activation dtype, as the
    reference's matmul does."""
    _need_cuda("lokr_add", out, x, w1, w2)
    if out.dtype not in (torch.float16, torch.bfloat16) or {x.dtype, w1.dtype, w2.dtype} != {out.dtype}:
        raise TypeError("lokr_add: out, x, w1 and w2 must share one dtype, float16 or bfloat16")
    if not out.is_contiguous():
        raise AssertionError("lokr_add: out must be contiguous")
    if x.stride(1) != 1:
        x = x.contiguous()
    w1c, w2c = w1.contiguous(), w2.contiguous()
    M, N = out.shape
    out_l, in_m = w1c.shape
    out_k, in_n = w2c.shape
    temp = torch.empty(M * out_l * in_n, dtype=out.dtype, device=out.device)
    st = L.lib().ic_lokr_add(_p(out), _DT[out.dtype], M, N, _p(x), x.stride(0), x.shape[1], _p(w1c), out_l, in_m,
                             _p(w2c), out_k, in_n, float(scale), _p(temp), temp.numel(), _stream(out))
    L.check(st, "ic_lokr_add")
    return out


def repack_int4(packed: torch.Tensor, K: int, layout: int) -> torch.Tensor:
    """Load-time nibble permutation of packed INT4 weights (``ic_repack_int4``):
    layout 0 feeds ``gemm_a8(..., repacked=True)``, layout 1 feeds
    ``gemm_w4a16(..., w_layout=1)``.  Same shape and size as the input."""
    _need_cuda("repack_int4", packed)
    p = packed.contiguous()
    out = torch.empty_like(p)
    L.check(L.lib().ic_repack_int4(_p(p), p.shape[0], K, p.stride(0), _p(out), out.stride(0), int(layout),
                                   _stream(p)), "ic_repack_int4")
    return out


def unpack_int4_to_int8(packed: torch.Tensor, K: int) -> torch.Tensor:
    """``kernels/triton_int4_to_int8_unpack.py:55-81``."""
    _need_cuda("unpack_int4_to_int8", packed)
    p = packed.contiguous()
    N = p.shape[0]
    out = torch.empty((N, K), dtype=torch.int8, device=p.device)
    L.check(L.lib().ic_unpack_int4_to_int8(_p(p), N, K, p.stride(0), _p(out), _stream(p)),
            "ic_unpack_int4_to_int8")
    return out


def unpack_int4_to_float16(packed: torch.Tensor, scale: torch.Tensor, K: int,
                           group_size: int | None = None) -> torch.Tensor:
    """``kernels/triton_int4_unpack.py:62-88`` (scale ``[N]``), extended to
    group scales ``[N, G]``."""
    _need_cuda("unpack_int4_to_float16", packed, scale)
    p = packed.contiguous()
    N = p.shape[0]
    sc = scale.reshape(N, -1)
    if sc.dtype not in (torch.float16, torch.float32):
        sc = sc.to(torch.float32)
    sc = sc.contiguous()
    G = sc.shape[1]
    gs = int(group_size) if group_size else -(-K // G)
    out = torch.empty((N, K), dtype=torch.float16, device=p.device)
    L.check(L.lib().ic_unpack_int4_to_f16(_p(p), N, K, p.stride(0), _p(sc), _DT[sc.dtype], G, gs,
                                          _p(out), _stream(p)), "ic_unpack_int4_to_f16")
    return out


def device_error(clear: bool = True) -> int:
    """Device error word of the library (1 = a bounded wait timed out)."""
    return L.read_device_error(clear)


__all__ = [
    "TRITON_AVAILABLE", "TRITON_INT4_UNPACK", "TRITON_INT8_GEMM", "TRITON_INT4_INT8_UNPACK",
    "TRITON_DYNQUANT", "TRITON_W4A8_GEMM", "TRITON_FUSED_QGD", "USE_FUSED_W8A8", "USE_CUDA_GRAPHS",
    "B200_AVAILABLE", "B200_LIBRARY_LOADED",
    "dynamic_quantize_activation", "fused_int8_gemm_dequant", "int8_gemm_int8out", "quantize_weight", "lokr_add",
    "fused_quant_int8_gemm_dequant",
    "fused_w4a8_gemm_dequant", "unpack_int4_to_int8", "unpack_int4_to_float16",
    "prep_quantize", "gemm_a8", "gemm_w4a16", "repack_int4", "lowrank_down", "lowrank_add", "device_error",
    "fused_layernorm_quantize", "fused_rmsnorm_quantize",
]
