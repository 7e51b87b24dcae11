"""CUDA-graph runner for the INT8 path (API of the reference's ``_cuda_graph.py``).

One ``CudaGraphRunner`` per INT8 ``IntCrushOps.Linear`` (no zero point, no
weight casting) caches one graph per ``(M, N, K, dtype, has_bias)`` with an
LRU of 4 entries, like ``_cuda_graph.py:80-175``.  The captured body is the
whole B200 forward of the layer: the fused prep/quant kernel and the INT8
GEMM, writing into static buffers (``static_x_int8``, ``static_s_a``,
``static_out``).  A replay is one ``copy_`` into ``static_x`` and one graph
launch; with ``safe_no_clone`` the static output is returned directly and must
be consumed before the next replay.  Both kernels are capture-safe: they take
torch's current stream, synchronise nothing and allocate nothing.
"""

from __future__ import annotations

import logging
from collections import OrderedDict

import torch

from . import _b200_runtime as _rt

log = logging.getLogger(__name__)

__all__ = ["CudaGraphRunner"]


class _GraphEntry:
    """A captured graph and every buffer it reads or writes (all must stay
    referenced for the graph's lifetime)."""

    __slots__ = ("graph", "static_x", "static_x_int8", "static_s_a", "static_out", "bias_snapshot", "_no_clone")

    def __init__(self, graph, static_x, static_x_int8, static_s_a, static_out, bias_snapshot, no_clone=False):
        self.graph = graph
        self.static_x = static_x
        self.static_x_int8 = static_x_int8
        self.static_s_a = static_s_a
        self.static_out = static_out
        self.bias_snapshot = bias_snapshot
        self._no_clone = no_clone

    def replay(self, x_2d: torch.Tensor) -> torch.Tensor:
        self.static_x.copy_(x_2d)
        self.graph.replay()
        return self.static_out if self._no_clone else self.static_out.clone()


class CudaGraphRunner:
    """Per-layer cache of captured INT8 forwards.

    Args:
        layer: the ``IntCrushOps.Linear`` whose attributes are read once.
        safe_no_clone: return the static output without a copy.
        max_cached_shapes: LRU capacity (default 4).
    """

    _MAX_CACHED_SHAPES: int = 4

    def __init__(self, layer, safe_no_clone: bool = True, max_cached_shapes: int | None = None) -> None:
        self._layer = layer
        self._w_int8: torch.Tensor = layer.weight._qdata
        self._s_w: torch.Tensor = layer.weight._params.scale
        self._smoothrot_factors = layer._intcrush_smoothrot_factors
        self._rot_need: bool = layer._intcrush_rot_need
        self._rot_size: int = layer._intcrush_rot_size
        self._w_in: int = layer._intcrush_w_in
        self._perm = layer._intcrush_perm
        self._smooth = layer._intcrush_smooth
        self._zp = layer.weight._params.zp
        self._safe_no_clone = safe_no_clone
        self._max_cached = max_cached_shapes if max_cached_shapes is not None else self._MAX_CACHED_SHAPES
        self._graphs: OrderedDict[tuple, _GraphEntry] = OrderedDict()
        self._dev = None   # device-side copies (int32 perm, fp32 vectors)

    # ── public API ───────────────────────────────────────────────────────────
    def run(self, x: torch.Tensor, bias: torch.Tensor | None, compute_dtype: torch.dtype) -> torch.Tensor:
        x_2d = x.reshape(-1, x.shape[-1])
        M, K = x_2d.shape
        N = self._w_int8.shape[0]
        if self._zp is not None or not x_2d.is_cuda:
            return self._run_eager(x_2d, bias, compute_dtype)
        key = (M, N, K, x.dtype, bias is not None)
        entry = self._graphs.get(key)
        if entry is not None:
            if entry.bias_snapshot is bias:
                self._graphs.move_to_end(key)
                return entry.replay(x_2d)
            del self._graphs[key]
        out = self._run_eager(x_2d, bias, compute_dtype)
        self._capture(key, x_2d, bias, compute_dtype)
        while len(self._graphs) > self._max_cached:
            self._graphs.popitem(last=False)
            log.debug("[INT-Crush] Evicted oldest CUDA graph entry (cache full)")
        return out

    def invalidate(self) -> None:
        self._graphs.clear()

    # ── internals ────────────────────────────────────────────────────────────
    def _device_tensors(self, device):
        if self._dev is None or self._dev[0] != device:
            f32 = lambda t: None if t is None else t.to(device=device, dtype=torch.float32).contiguous()
            self._dev = (device,
                         None if self._perm is None else self._perm.to(device=device, dtype=torch.int32).contiguous(),
                         f32(self._smoothrot_factors), f32(self._smooth), f32(self._s_w.reshape(-1)))
        return self._dev[1:]

    def _prep_and_quantize(self, x_2d, bias, compute_dtype, *, s_a_out=None, x_int8_out=None, out=None):
        perm32, sr, sm, s_w = self._device_tensors(x_2d.device)
        if x_2d.dtype != compute_dtype:
            x_2d = x_2d.to(compute_dtype)
        x_int8, s_a, _, _ = _rt.prep_quantize(
            x_2d, smoothrot=sr, rot_size=self._rot_size if self._rot_need else 0, w_in=self._w_in,
            perm=perm32, smooth=sm if sr is None else None, s_a_out=s_a_out, x_int8_out=x_int8_out)
        return _rt.gemm_a8(x_int8, self._w_int8, s_w, s_a, bias=bias, out_dtype=compute_dtype, out=out)

    def _run_eager(self, x_2d, bias, compute_dtype):
        return self._prep_and_quantize(x_2d, bias, compute_dtype)

    def _capture(self, key, x_2d, bias, compute_dtype) -> None:
        M, K = x_2d.shape
        N = self._w_int8.shape[0]
        dev = x_2d.device
        static_x = torch.empty(M, K, dtype=x_2d.dtype, device=dev)
        static_x_int8 = torch.empty(M, (self._w_in + 15) // 16 * 16, dtype=torch.int8, device=dev)
        static_s_a = torch.empty(M, dtype=torch.float32, device=dev)
        static_out = torch.empty(M, N, dtype=compute_dtype, device=dev)
        static_x.copy_(x_2d)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._prep_and_quantize(static_x, bias, compute_dtype, s_a_out=static_s_a,
                                    x_int8_out=static_x_int8, out=static_out)
        self._graphs[key] = _GraphEntry(graph, static_x, static_x_int8, static_s_a, static_out, bias,
                                        no_clone=self._safe_no_clone)
        log.debug("[INT-Crush] Captured CUDA graph: M=%d N=%d K=%d dtype=%s has_bias=%s",
                  M, N, K, compute_dtype, bias is not None)
