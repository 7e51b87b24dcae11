"""INT-Crush ops factory: ``make_intcrush_ops`` -> ``IntCrushOps.Linear``.

Same API and behaviour as the reference's ``_ops.py`` (factory
``_ops.py:146-162``, state-dict loading ``:583-761``, weight/bias setters
``:763-815``, forward dispatch ``:817-862``): the module keeps ComfyUI's
``QuantizedTensor`` weight, its ``_intcrush_*`` attributes and the same path
selection (W4A8 / W4A16 / PyTorch-semantics INT4, INT8 with optional CUDA
graphs).  Every numeric step of the forward runs on the B200 kernels of
``_b200_runtime``:

* activation prep + quantisation: one ``prep_quantize`` launch;
* INT8 / W4A8: ``gemm_a8`` with bias and the zero-point term fused;
* W4A16 and the PyTorch INT4 path (identical dequant-then-linear semantics,
  no bias as in the reference): ``gemm_w4a16``;
* standard-LoRA residual on the raw input and the SVD residual on the
  prepped input: ``lowrank_down`` + ``lowrank_add`` (fused into ``gemm_w4a16``
  on that path).

Weights are prepared once per layer and device (int32 perm, fp32 scales, the
nibble-repacked INT4 layout the GEMMs expand fastest) and cached on the
module; ``set_weight`` drops the cache.  There is no CPU fallback: a forward
on CPU tensors raises.  LoKr and the other non-LoRA adapters keep the
reference's own adapter math (``adapter.h``/``adapter.g`` and the LoKr
Kronecker accumulation), which is outside the quantised hot path.
"""

from __future__ import annotations

import logging
from typing import Any, Callable

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _b200_runtime as _rt
from .quant_layout import IntCrushInt4Layout, IntCrushInt8Layout
from ._cuda_graph import CudaGraphRunner

_log = logging.getLogger(__name__)

# Layer-name substrings that disable rotation (_ops.py:30-32).
_NO_ROTATION_NAME_SUBSTRINGS: tuple[str, ...] = (
    "embed", "norm", "modulation", "output", "lm_head", "proj_out",
)

# State-dict key suffixes (_ops.py:36-45).
_SD_KEY_WEIGHT = "weight"
_SD_KEY_SCALE = "weight_scale"
_SD_KEY_ZP = "weight_zp"
_SD_KEY_PERM = "weight_perm"
_SD_KEY_SMOOTH = "weight_smooth"
_SD_KEY_SMOOTHROT = "weight_smoothrot_factors"
_SD_KEY_L1 = "weight_L1"
_SD_KEY_L2 = "weight_L2"
_SD_KEY_QUANT = "comfy_quant"
_SD_KEY_BIAS = "bias"
_VALID_SCALE_DTYPES = (torch.float16, torch.float32)

_QuantizedTensor = None
_cast_bias_weight = None
_uncast_bias_weight = None


def _get_qt():
    global _QuantizedTensor
    if _QuantizedTensor is None:
        from comfy.quant_ops import QuantizedTensor
        _QuantizedTensor = QuantizedTensor
    return _QuantizedTensor


def _get_cast():
    global _cast_bias_weight, _uncast_bias_weight
    if _cast_bias_weight is None:
        from comfy.ops import cast_bias_weight, uncast_bias_weight
        _cast_bias_weight = cast_bias_weight
        _uncast_bias_weight = uncast_bias_weight
    return _cast_bias_weight, _uncast_bias_weight


def _move_adapter_weights(adapter: Any, device: torch.device, dtype: torch.dtype) -> None:
    adapter.weights = type(adapter.weights)(
        w.to(device=device, dtype=dtype) if isinstance(w, torch.Tensor) else w for w in adapter.weights)


def _apply_lokr(cache: dict[str, Any], x_raw: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """LoKr residual with pre-combined factors (reference ``_ops.py:88-138``):
    ``out[n] += scale * w1 @ X[n] @ w2_t`` per token, in chunks."""
    w1, w2_t, scale = cache["w1"], cache["w2_t"], cache["scale"]
    T = x_raw.shape[0]
    out_l, in_m = w1.shape
    in_n, out_k = w2_t.shape
    if (out.is_cuda and out.dtype in (torch.float16, torch.bfloat16) and out.is_contiguous()
            and x_raw.dtype == out.dtype and in_n <= 256 and out_l * in_m <= 12288):
        # two B200 kernels: T(w1 @ X_t) per token, then the in-place rank-in_n update
        if "w2" not in cache:
            cache["w2"] = w2_t.t().contiguous()
        return _rt.lokr_add(out, x_raw.reshape(T, -1), w1, cache["w2"], scale)
    chunk = max(1, min(T, (64 << 20) // max(out_l * (in_n + out_k) * x_raw.element_size(), 1)))
    if not out.is_contiguous():
        out = out.contiguous()
    out3 = out.view(T, out_l, out_k)
    for s in range(0, T, chunk):
        e = min(s + chunk, T)
        tmp = w1 @ x_raw[s:e].reshape(e - s, in_m, in_n)
        out3[s:e].reshape(-1, out_k).addmm_(tmp.reshape(-1, in_n), w2_t, beta=1.0, alpha=scale)
    return out


class _B200Weights:
    """Per-layer device-side weight preparation, built once and reused."""

    __slots__ = ("key", "perm32", "s_w", "group_size", "rep_a8", "rep_a16", "scale16", "zp_corr",
                 "smoothrot", "smooth", "K", "N")

    def __init__(self, key, **kw):
        self.key = key
        for k in self.__slots__[1:]:
            setattr(self, k, kw.get(k))


_ops_cache: dict[tuple, type] = {}


def make_intcrush_ops(quant_format: str, rot_size: int, use_pytorch: bool = False,
                      use_w4a16: bool = False) -> type:
    """Build the ``manual_cast`` ops class (reference ``_ops.py:146-883``).

    Args:
        quant_format: "int4_crush" or "int8_crush"
        rot_size: Hadamard rotation group size (0 disables rotation)
        use_pytorch: INT4 layers use the dequant-then-linear semantics of the
            reference's PyTorch path (run by the B200 W4A16 kernel)
        use_w4a16: INT4 layers use W4A16 instead of W4A8
    """
    cache_key = (quant_format, rot_size, use_pytorch, use_w4a16)
    if cache_key in _ops_cache:
        return _ops_cache[cache_key]
    from comfy.ops import manual_cast

    class IntCrushOps(manual_cast):

        class Linear(manual_cast.Linear):
            """INT-Crush Linear: QuantizedTensor storage, B200 kernels in forward()."""

            def __init__(self, *args: Any, **kwargs: Any) -> None:
                super().__init__(*args, **kwargs)
                self._intcrush_is_quantized = False
                self._intcrush_rot_need = True
                self._intcrush_rot_size = rot_size
                self._intcrush_perm = None
                self._intcrush_smooth = None
                self._intcrush_smoothrot_factors = None
                self._intcrush_L1 = None
                self._intcrush_L2 = None
                self._intcrush_use_pytorch = use_pytorch
                self._intcrush_use_w4a16 = use_w4a16
                self._intcrush_w_in = None
                self.quant_format = None
                self.layout_type = None
                self._intcrush_adapter = None
                self._intcrush_lora_strength = None
                self._intcrush_adapter_ready = False
                self._intcrush_adapter_device = None
                self._intcrush_lokr_cache = None
                self._intcrush_lokr_cache_adapter_id = None
                self._intcrush_lokr_cache_strength = None
                self._graph_runner = None
                self._b200 = None

            # ── device-side weight preparation ──────────────────────────────
            def _b200_weights(self, weight: Any, device: torch.device) -> _B200Weights:
                qdata, params = weight._qdata, weight._params
                key = (id(qdata), qdata.data_ptr(), str(device), qdata.dtype)
                bw = self._b200
                if bw is not None and bw.key == key:
                    return bw
                N = qdata.shape[0]
                is_int4 = isinstance(params, IntCrushInt4Layout.Params)
                K = self._intcrush_w_in if is_int4 else qdata.shape[1]
                s = params.scale.to(device=device, dtype=torch.float32).reshape(N, -1).contiguous()
                G = s.shape[1]
                gs = -(-K // G) if G > 1 else K
                perm = self._intcrush_perm
                zp = params.zp
                zp_corr = None
                if zp is not None:
                    zp_corr = (s.reshape(-1)[:N] * zp.to(device).reshape(-1).float()[:N]).contiguous()
                bw = _B200Weights(
                    key,
                    perm32=perm.to(device=device, dtype=torch.int32).contiguous() if perm is not None else None,
                    s_w=s, group_size=gs, K=K, N=N, zp_corr=zp_corr,
                    scale16=s.to(torch.float16).contiguous() if is_int4 else None,
                    smoothrot=(self._intcrush_smoothrot_factors.to(device).float().contiguous()
                               if self._intcrush_smoothrot_factors is not None else None),
                    smooth=(self._intcrush_smooth.to(device).float().contiguous()
                            if self._intcrush_smooth is not None else None))
                self._b200 = bw
                return bw

            def _repacked(self, bw: _B200Weights, qdata: torch.Tensor, layout: int):
                """Nibble-repacked INT4 copy for the GEMMs (on by default; it
                costs a second copy of the INT4 weights, INTCRUSH_REPACK=0 turns
                it off)."""
                if not _REPACK:
                    return None
                attr = "rep_a8" if layout == 0 else "rep_a16"
                rep = getattr(bw, attr)
                if rep is None:
                    rep = _rt.repack_int4(qdata, bw.K, layout)
                    setattr(bw, attr, rep)
                return rep

            # ── adapters ────────────────────────────────────────────────────
            def _lora_factors(self, x_raw: torch.Tensor):
                """(down, up, scale) of an attached standard LoRA, else None."""
                adapter = self._intcrush_adapter
                if adapter is None or getattr(adapter, "name", None) != "lora":
                    return None
                self._ready_adapter(x_raw)
                up, down, alpha = adapter.weights[0], adapter.weights[1], adapter.weights[2]
                rank = down.shape[0]
                scale = (float(alpha) / rank) if alpha else 1.0
                return down, up, scale * float(self._intcrush_lora_strength)

            def _ready_adapter(self, x_raw: torch.Tensor) -> None:
                if not self._intcrush_adapter_ready or self._intcrush_adapter_device != x_raw.device:
                    _move_adapter_weights(self._intcrush_adapter, x_raw.device, x_raw.dtype)
                    self._intcrush_adapter_ready = True
                    self._intcrush_adapter_device = x_raw.device

            def _apply_adapter(self, x_raw: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
                """Adapter residual on the unrotated input (``_ops.py:195-271``).
                Standard LoRA runs on the B200 low-rank kernels; other adapter
                types use their own math."""
                adapter = self._intcrush_adapter
                if adapter is None:
                    return out
                lora = self._lora_factors(x_raw)
                if lora is not None:
                    down, up, scale = lora
                    return _lowrank_residual(out, x_raw, down, up, scale)
                self._ready_adapter(x_raw)
                strength = self._intcrush_lora_strength
                if adapter.name == "lokr":
                    if (id(adapter) != self._intcrush_lokr_cache_adapter_id
                            or strength != self._intcrush_lokr_cache_strength):
                        self._intcrush_lokr_cache = self._setup_lokr_cache(adapter, x_raw.device, x_raw.dtype,
                                                                           strength)
                        self._intcrush_lokr_cache_adapter_id = id(adapter)
                        self._intcrush_lokr_cache_strength = strength
                    return _apply_lokr(self._intcrush_lokr_cache, x_raw, out)
                adapter.multiplier = strength
                out.add_(adapter.h(x_raw, out).to(out.dtype))
                return adapter.g(out)

            def _setup_lokr_cache(self, adapter: Any, device, dtype, strength: float) -> dict:
                v = adapter.weights
                w1, w2, alpha = v[0], v[1], v[2]
                w1_a, w1_b, w2_a, w2_b = v[3], v[4], v[5], v[6]
                t2 = v[7] if len(v) > 7 else None
                cast = lambda t: t.to(device=device, dtype=dtype)
                cache: dict[str, Any] = {"w1": cast(w1) if w1 is not None else cast(w1_a) @ cast(w1_b)}
                if w2 is not None:
                    w2d = cast(w2)
                elif t2 is not None:
                    w2d = torch.einsum("i j k l, j r, i p -> p r k l", cast(t2), cast(w2_b), cast(w2_a))
                else:
                    w2d = cast(w2_a) @ cast(w2_b)
                cache["w2_t"] = w2d.t().contiguous()
                rank = w1_b.shape[0] if w1_a is not None else (w2_b.shape[0] if w2_a is not None else None)
                cache["scale"] = (float(alpha) / rank) * strength if (rank is not None and alpha is not None) \
                    else strength
                return cache

            # ── prep / residuals / finish ───────────────────────────────────
            def _prep_activation(self, x: torch.Tensor, pad_to_w_in: bool = True,
                                 apply_perm: bool = True) -> torch.Tensor:
                """SmoothRot -> Hadamard -> pad -> permute (``_ops.py:337-365``), one kernel."""
                x2 = x.reshape(-1, x.shape[-1])
                bw = self._b200 if self._b200 is not None else None
                sr = self._intcrush_smoothrot_factors
                rot = self._intcrush_rot_size if self._intcrush_rot_need else 0
                perm = self._intcrush_perm if apply_perm else None
                w_in = self._intcrush_w_in if pad_to_w_in else None
                if sr is None and rot == 0 and perm is None and (w_in is None or w_in <= x2.shape[-1]):
                    return x2
                _, _, xp, _ = _rt.prep_quantize(
                    x2, smoothrot=(bw.smoothrot if bw is not None and bw.smoothrot is not None else sr),
                    rot_size=rot, w_in=w_in,
                    perm=(bw.perm32 if (bw is not None and perm is not None) else perm),
                    quantize=False, want_prep=True)
                return xp

            def _apply_residuals(self, x: torch.Tensor, out: torch.Tensor,
                                 x_prep: torch.Tensor | None = None) -> torch.Tensor:
                """SVD low-rank residual (on ``x_prep`` when given, as the reference
                does) and the adapter residual (``_ops.py:367-387``)."""
                L1, L2 = self._intcrush_L1, self._intcrush_L2
                if L1 is not None and L2 is not None:
                    if L1.device != x.device or L1.dtype != x.dtype:
                        L1 = L1.to(device=x.device, dtype=x.dtype)
                        self._intcrush_L1 = L1
                    if L2.device != x.device or L2.dtype != x.dtype:
                        L2 = L2.to(device=x.device, dtype=x.dtype)
                        self._intcrush_L2 = L2
                    svd_x = x_prep if x_prep is not None else x.reshape(-1, x.shape[-1])
                    out = _lowrank_residual(out, svd_x, L2, L1, 1.0)
                return self._apply_adapter(x.reshape(-1, x.shape[-1]), out)

            def _finish_forward(self, out: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
                return out.to(x.dtype).reshape(*x.shape[:-1], -1)

            def _needs_cast(self) -> bool:
                return bool(self.comfy_cast_weights or self.weight_function or self.bias_function
                            or getattr(self, "weight_lowvram_function", None) is not None
                            or getattr(self, "bias_lowvram_function", None) is not None)

            def _setup_casting(self, x: torch.Tensor):
                QT = _get_qt()
                if self._needs_cast():
                    weight_dtype = self.weight._params.orig_dtype if isinstance(self.weight, QT) else x.dtype
                    cbw, ucbw = _get_cast()
                    weight, bias, offload_stream = cbw(self, input=None, dtype=weight_dtype, device=x.device,
                                                       bias_dtype=x.dtype, offloadable=True)
                    return weight, bias, (lambda: ucbw(self, weight, bias, offload_stream)), QT
                return self.weight, self.bias, None, QT

            # ── forward paths ───────────────────────────────────────────────
            def _forward_predequant(self, weight: torch.Tensor, bias: torch.Tensor | None,
                                    x: torch.Tensor) -> torch.Tensor:
                """Weight already dequantised by a host wrapper: rotate only,
                then a plain linear with that float weight (``_ops.py:435-441``)."""
                x_2d = self._prep_activation(x, pad_to_w_in=False, apply_perm=False)
                out = F.linear(x_2d, weight, bias)
                out = self._apply_residuals(x, out, x_prep=x_2d)
                return self._finish_forward(out, x)

            def _quant_prep(self, x: torch.Tensor, bw: _B200Weights, *, int8_smooth: bool,
                            quantize: bool, want_prep: bool, want_rowsum: bool):
                x2 = x.reshape(-1, x.shape[-1])
                rot = self._intcrush_rot_size if self._intcrush_rot_need else 0
                smooth = bw.smooth if (int8_smooth and bw.smoothrot is None) else None
                return _rt.prep_quantize(
                    x2, smoothrot=bw.smoothrot, rot_size=rot, w_in=self._intcrush_w_in, perm=bw.perm32,
                    smooth=smooth, quantize=quantize, want_prep=want_prep, want_rowsum=want_rowsum)

            def _forward_int4_w4a8(self, qdata: torch.Tensor, weight: Any, bias: torch.Tensor | None,
                                   x: torch.Tensor) -> torch.Tensor:
                """INT4 W4A8 (``_ops.py:443-464``): prep+quant kernel, then the
                group-scale INT4 GEMM with the unpack fused and bias fused."""
                bw = self._b200_weights(weight, x.device)
                needs_zp = bw.zp_corr is not None
                svd = self._intcrush_L1 is not None and self._intcrush_L2 is not None
                xq, s_a, x_prep, rowsum = self._quant_prep(x, bw, int8_smooth=False, quantize=True,
                                                           want_prep=svd, want_rowsum=needs_zp)
                rep = self._repacked(bw, qdata, 0)
                out = _rt.gemm_a8(xq, rep if rep is not None else qdata, bw.s_w, s_a, bias=bias,
                                  out_dtype=x.dtype, group_size=bw.group_size, repacked=rep is not None,
                                  rowsum=_round_to(rowsum, x.dtype) if needs_zp else None,
                                  zp_corr=_round_to(bw.zp_corr, x.dtype) if needs_zp else None)
                out = self._apply_residuals(x, out, x_prep=x_prep)
                return self._finish_forward(out, x)

            def _forward_int4_w4a16(self, qdata: torch.Tensor, weight: Any, bias: torch.Tensor | None,
                                    x: torch.Tensor) -> torch.Tensor:
                """INT4 W4A16 (``_ops.py:466-481``) and the PyTorch INT4 path
                (``:483-491``): ``x_prep @ W^T`` with the weights dequantised in
                the activation dtype (fp16: fp16(q * s); bf16: bf16(q * s)),
                no bias (as in the reference)."""
                bw = self._b200_weights(weight, x.device)
                needs_zp = bw.zp_corr is not None
                svd = self._intcrush_L1 is not None and self._intcrush_L2 is not None
                _, _, x_prep, rowsum = self._quant_prep(x, bw, int8_smooth=False, quantize=False,
                                                        want_prep=True, want_rowsum=needs_zp)
                lora = None if (needs_zp or svd) else self._lora_factors(x.reshape(-1, x.shape[-1]))
                mid = up = None
                scale = 1.0
                if lora is not None:
                    down, up, scale = lora
                    mid = _rt.lowrank_down(x.reshape(-1, x.shape[-1]), down)
                rep = self._repacked(bw, qdata, 1)
                out = _rt.gemm_w4a16(x_prep, rep if rep is not None else qdata, bw.scale16,
                                     group_size=bw.group_size, lr_mid=mid, lr_up=up, lr_scale=scale,
                                     K=bw.K, w_layout=1 if rep is not None else 0)
                if needs_zp:
                    # out -= T(rowsum) * T(s*zp), one rounding (out.addmm_ of _ops.py:476-478)
                    _rt.lowrank_add(out, _round_to(rowsum, x.dtype).to(x.dtype).reshape(-1, 1),
                                    bw.zp_corr.to(x.dtype).reshape(-1, 1), -1.0)
                if lora is not None:
                    if svd:
                        out = self._apply_residuals_svd_only(x, out, x_prep)
                    return self._finish_forward(out, x)
                out = self._apply_residuals(x, out, x_prep=x_prep)
                return self._finish_forward(out, x)

            def _apply_residuals_svd_only(self, x, out, x_prep):
                L1, L2 = self._intcrush_L1, self._intcrush_L2
                return _lowrank_residual(out, x_prep, L2.to(x.device, x.dtype), L1.to(x.device, x.dtype), 1.0)

            def _forward_int4_pytorch(self, qdata: torch.Tensor, weight: Any, x: torch.Tensor) -> torch.Tensor:
                return self._forward_int4_w4a16(qdata, weight, None, x)

            def _forward_int8(self, qdata: torch.Tensor, weight: Any, bias: torch.Tensor | None,
                              x: torch.Tensor) -> torch.Tensor:
                """INT8 W8A8 (``_ops.py:493-579``): CUDA-graph replay when possible,
                else prep+quant kernel and the INT8 GEMM with bias fused."""
                zp = weight._params.zp
                compute_dtype = x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
                bw = self._b200_weights(weight, x.device)
                can_graph = (_rt.B200_AVAILABLE and zp is None and not self._needs_cast()
                             and _rt.USE_CUDA_GRAPHS and x.is_cuda)
                if can_graph:
                    if self._graph_runner is None:
                        self._graph_runner = CudaGraphRunner(self, safe_no_clone=True)
                    out = self._graph_runner.run(x, bias, compute_dtype)
                    out = self._apply_residuals(x, out)
                    return self._finish_forward(out, x)
                needs_zp = zp is not None
                xq, s_a, _, rowsum = self._quant_prep(x.to(compute_dtype) if x.dtype != compute_dtype else x,
                                                      bw, int8_smooth=True, quantize=True, want_prep=False,
                                                      want_rowsum=needs_zp)
                out = _rt.gemm_a8(xq, qdata, bw.s_w, s_a, bias=bias, out_dtype=compute_dtype,
                                  rowsum=_round_to(rowsum, compute_dtype) if needs_zp else None,
                                  zp_corr=_round_to(bw.zp_corr, compute_dtype) if needs_zp else None)
                out = self._apply_residuals(x, out)
                return self._finish_forward(out, x)

            # ── state-dict loading (``_ops.py:583-761``) ────────────────────
            @staticmethod
            def _detect_weight_format(weight, scale) -> str | None:
                if weight is None or scale is None or scale.dtype not in _VALID_SCALE_DTYPES:
                    return None
                if weight.dtype == torch.uint8:
                    return "int4_crush"
                if weight.dtype == torch.int8:
                    return "int8_crush"
                return None

            def _pop_intcrush_tensors(self, state_dict: dict, prefix: str) -> dict[str, Any]:
                r = {
                    "weight": state_dict.pop(prefix + _SD_KEY_WEIGHT),
                    "scale": state_dict.pop(prefix + _SD_KEY_SCALE),
                    "zp": state_dict.pop(prefix + _SD_KEY_ZP, None),
                    "perm": state_dict.pop(prefix + _SD_KEY_PERM, None),
                    "smooth": state_dict.pop(prefix + _SD_KEY_SMOOTH, None),
                    "smoothrot_factors": state_dict.pop(prefix + _SD_KEY_SMOOTHROT, None),
                    "L1": state_dict.pop(prefix + _SD_KEY_L1, None),
                    "L2": state_dict.pop(prefix + _SD_KEY_L2, None),
                    "bias": state_dict.pop(prefix + _SD_KEY_BIAS, None),
                }
                state_dict.pop(prefix + _SD_KEY_QUANT, None)
                return r

            def _store_intcrush_attrs(self, tensors: dict[str, Any], params: Any, device) -> None:
                self._intcrush_perm = params.perm
                self._intcrush_w_in = self.in_features
                self._intcrush_smooth = (tensors["smooth"].float().to(device=device)
                                         if tensors["smooth"] is not None else None)
                self._intcrush_smoothrot_factors = (tensors["smoothrot_factors"].float().to(device=device)
                                                    if tensors["smoothrot_factors"] is not None else None)
                self._intcrush_L1 = (tensors["L1"].to(device=device, dtype=torch.float16)
                                     if tensors["L1"] is not None else None)
                self._intcrush_L2 = (tensors["L2"].to(device=device, dtype=torch.float16)
                                     if tensors["L2"] is not None else None)

            @staticmethod
            def _clear_known_missing_keys(missing_keys: list[str], prefix: str) -> None:
                for suffix in (_SD_KEY_WEIGHT, _SD_KEY_SCALE, _SD_KEY_ZP, _SD_KEY_PERM, _SD_KEY_SMOOTH,
                               _SD_KEY_SMOOTHROT, _SD_KEY_L1, _SD_KEY_L2, _SD_KEY_BIAS, _SD_KEY_QUANT):
                    if prefix + suffix in missing_keys:
                        missing_keys.remove(prefix + suffix)

            def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs) -> None:
                from comfy.quant_ops import QUANT_ALGOS, QuantizedTensor, get_layout_class
                fmt = self._detect_weight_format(state_dict.get(prefix + _SD_KEY_WEIGHT),
                                                 state_dict.get(prefix + _SD_KEY_SCALE))
                if fmt is None:
                    super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                                  unexpected_keys, error_msgs)
                    return
                qconfig = QUANT_ALGOS[fmt]
                layout_type = qconfig["comfy_tensor_layout"]
                layout_cls = get_layout_class(layout_type)
                tensors = self._pop_intcrush_tensors(state_dict, prefix)
                w = getattr(self, "weight", None)
                device = w.device if w is not None else torch.device("cpu")
                name_lower = prefix.lower()
                rot_need = rot_size > 0 and not any(p in name_lower for p in _NO_ROTATION_NAME_SUBSTRINGS)
                self._intcrush_rot_need = rot_need
                self._intcrush_rot_size = rot_size
                self._intcrush_is_quantized = True
                perm, zp = tensors["perm"], tensors["zp"]
                scale = tensors["scale"].float()
                if fmt == "int8_crush":
                    scale = scale.reshape(-1)
                params = layout_cls.Params(
                    scale=scale.to(device=device), orig_dtype=torch.float16,
                    orig_shape=(self.out_features, self.in_features), rot_need=rot_need, rot_size=rot_size,
                    perm=perm.to(device=device) if perm is not None else None,
                    zp=zp.to(device=device) if zp is not None else None)
                self._store_intcrush_attrs(tensors, params, device)
                self.weight = nn.Parameter(
                    QuantizedTensor(tensors["weight"].to(device=device, dtype=qconfig["storage_t"]),
                                    layout_type, params), requires_grad=False)
                self.quant_format = fmt
                self.layout_type = layout_type
                b = tensors["bias"]
                self.bias = nn.Parameter(b.to(device=device), requires_grad=False) if b is not None else None
                if perm is not None:
                    self.register_parameter("weight_perm", nn.Parameter(perm.to(device=device), requires_grad=False))
                if zp is not None:
                    self.register_parameter("weight_zp", nn.Parameter(zp.to(device=device), requires_grad=False))
                self._b200 = None
                self._graph_runner = None
                self._clear_known_missing_keys(missing_keys, prefix)

            def convert_weight(self, weight: torch.Tensor, inplace: bool = False) -> torch.Tensor:
                from comfy.quant_ops import QuantizedTensor
                if self._intcrush_is_quantized and isinstance(weight, QuantizedTensor):
                    return weight
                return super().convert_weight(weight, inplace)

            def set_weight(self, out_weight: torch.Tensor, inplace_update: bool = False, seed: int = 0,
                           return_weight: bool = False, **kwargs: Any):
                """Requantise float weights, keeping rotation and permutation
                (``_ops.py:770-807``); drops the device weight cache and graphs."""
                self._graph_runner = None
                self._b200 = None
                if not self._intcrush_is_quantized:
                    new_weight = out_weight.to(self.weight.dtype)
                    if return_weight:
                        return new_weight
                    self.weight = nn.Parameter(new_weight, requires_grad=False)
                    return None
                import dataclasses
                from comfy.quant_ops import QuantizedTensor, get_layout_class
                if isinstance(out_weight, QuantizedTensor):
                    if return_weight:
                        return out_weight
                    self.weight = nn.Parameter(out_weight, requires_grad=False)
                    return None
                layout_cls = get_layout_class(self.layout_type)
                packed, params = layout_cls.quantize(out_weight.float(), scale="recalculate",
                                                     stochastic_rounding=seed)
                params = dataclasses.replace(params, rot_need=self._intcrush_rot_need,
                                             rot_size=self._intcrush_rot_size, perm=self._intcrush_perm)
                qt = QuantizedTensor(packed, self.layout_type, params)
                if return_weight:
                    return qt
                self.weight = nn.Parameter(qt, requires_grad=False)
                return None

            def set_bias(self, out_bias, inplace_update: bool = False, seed: int = 0,
                         return_weight: bool = False, **kwargs: Any):
                if out_bias is None:
                    return None
                if return_weight:
                    return out_bias
                self.bias = nn.Parameter(out_bias, requires_grad=False)
                self._graph_runner = None
                return None

            @torch.no_grad()
            def forward(self, x: torch.Tensor) -> torch.Tensor:
                if not self._intcrush_is_quantized:
                    return super().forward(x)
                weight, bias, uncast, QT = self._setup_casting(x)
                try:
                    if not isinstance(weight, QT):
                        return self._forward_predequant(weight, bias, x)
                    qdata = weight._qdata
                    if isinstance(weight._params, IntCrushInt4Layout.Params):
                        if (not self._intcrush_use_pytorch and not self._intcrush_use_w4a16
                                and self._intcrush_rot_need and _rt.B200_AVAILABLE):
                            return self._forward_int4_w4a8(qdata, weight, bias, x)
                        if not self._intcrush_use_pytorch:
                            return self._forward_int4_w4a16(qdata, weight, bias, x)
                        return self._forward_int4_pytorch(qdata, weight, x)
                    if isinstance(weight._params, IntCrushInt8Layout.Params):
                        return self._forward_int8(qdata, weight, bias, x)
                    return super().forward(x)
                finally:
                    if uncast is not None:
                        uncast()

        class GroupNorm(manual_cast.GroupNorm):
            pass

        class LayerNorm(manual_cast.LayerNorm):
            pass

        class Conv2d(manual_cast.Conv2d):
            pass

        class Conv3d(manual_cast.Conv3d):
            pass

        class ConvTranspose2d(manual_cast.ConvTranspose2d):
            pass

        class Embedding(manual_cast.Embedding):
            pass

    _ops_cache[cache_key] = IntCrushOps
    return IntCrushOps


# ── module helpers ───────────────────────────────────────────────────────────

import os as _os

# Keep a nibble-repacked copy of INT4 weights for the GEMMs (faster INT4
# expansion, costs one extra copy of the INT4 weights).  On by default;
# INTCRUSH_REPACK=0 keeps only the reference packing.
_REPACK = _os.environ.get("INTCRUSH_REPACK", "1") == "1"


def _round_to(t: torch.Tensor | None, dtype: torch.dtype) -> torch.Tensor | None:
    """Round fp32 values through ``dtype`` (the reference keeps these terms in
    the activation dtype) and return fp32."""
    if t is None:
        return None
    return t.to(dtype).to(torch.float32)


def _lowrank_residual(out: torch.Tensor, x2: torch.Tensor, down: torch.Tensor, up: torch.Tensor,
                      scale: float) -> torch.Tensor:
    """``out += scale * T(x2 @ down^T) @ up^T`` (``F.linear`` then ``addmm_``
    of ``_ops.py:242-243`` / ``:383-384``) on the low-rank kernels for fp16 /
    bf16 outputs up to rank 256; other output dtypes or larger ranks run the
    reference's own two torch calls on the GPU."""
    if out.dtype in (torch.float16, torch.bfloat16) and down.shape[0] <= 256 and out.stride(-1) == 1:
        mid = _rt.lowrank_down(x2.to(out.dtype), down)
        return _rt.lowrank_add(out, mid, up, scale)
    mid = F.linear(x2.to(down.dtype), down)
    return out.addmm_(mid.to(out.dtype), up.t().to(out.dtype), beta=1, alpha=scale)


__all__ = ["make_intcrush_ops"]
