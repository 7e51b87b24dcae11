"""``torch.library`` registrations of the B200 kernels (namespace ``intcrush_b200``).

The C ABI (``libintcrush_b200.so``, reached through ctypes in ``_lib``) is the
boundary; these custom ops wrap the same entry points so that the fused
prep / GEMM calls are single graph nodes for ``torch.compile`` and
``torch.export`` (with fake kernels for shape propagation), instead of
graph breaks at every ctypes call:

* ``intcrush_b200::prep_quantize(x, smoothrot?, perm?, smooth?, rot_size,
  w_in) -> (x_int8, s_a)`` -- ``_b200_runtime.prep_quantize``;
* ``intcrush_b200::gemm_a8(x_int8, w, s_w, s_a, bias?, out_dtype,
  group_size, repacked) -> out`` -- ``_b200_runtime.gemm_a8``;
* ``intcrush_b200::gemm_w4a16(x, packed, scale, group_size, w_layout) ->
  out`` -- ``_b200_runtime.gemm_w4a16``.

The ops mirror the reference runtime's callables (``_triton_runtime.py:
16-41,114-130``): CUDA tensors in, freshly allocated outputs, launch on the
current stream.  ``register()`` is idempotent; importing this module
registers the ops.
"""

from __future__ import annotations

import torch

from . import _b200_runtime as _rt

_NS = "intcrush_b200"
_DTYPES = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}
_CODES = {v: k for k, v in _DTYPES.items()}
_done = False


def register() -> None:
    global _done
    if _done:
        return

    @torch.library.custom_op(f"{_NS}::prep_quantize", mutates_args=())
    def prep_quantize(x: torch.Tensor, smoothrot: torch.Tensor | None, perm: torch.Tensor | None,
                      smooth: torch.Tensor | None, rot_size: int, w_in: int) -> tuple[torch.Tensor, torch.Tensor]:
        xq, s_a, _, _ = _rt.prep_quantize(x, smoothrot=smoothrot, rot_size=rot_size, w_in=w_in, perm=perm,
                                          smooth=smooth)
        return xq.contiguous(), s_a

    @prep_quantize.register_fake
    def _(x, smoothrot, perm, smooth, rot_size, w_in):
        M = x.numel() // x.shape[-1]
        return (x.new_empty((M, w_in), dtype=torch.int8), x.new_empty((M,), dtype=torch.float32))

    @torch.library.custom_op(f"{_NS}::gemm_a8", mutates_args=())
    def gemm_a8(x_int8: torch.Tensor, w: torch.Tensor, s_w: torch.Tensor, s_a: torch.Tensor,
                bias: torch.Tensor | None, out_dtype: int, group_size: int, repacked: bool) -> torch.Tensor:
        return _rt.gemm_a8(x_int8, w, s_w, s_a, bias=bias, out_dtype=_DTYPES[out_dtype],
                           group_size=group_size or None, repacked=repacked)

    @gemm_a8.register_fake
    def _(x_int8, w, s_w, s_a, bias, out_dtype, group_size, repacked):
        return x_int8.new_empty((x_int8.shape[0], w.shape[0]), dtype=_DTYPES[out_dtype])

    @torch.library.custom_op(f"{_NS}::gemm_w4a16", mutates_args=())
    def gemm_w4a16(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, group_size: int,
                   w_layout: int) -> torch.Tensor:
        return _rt.gemm_w4a16(x, packed, scale, group_size=group_size or None, w_layout=w_layout)

    @gemm_w4a16.register_fake
    def _(x, packed, scale, group_size, w_layout):
        return x.new_empty((x.shape[0], packed.shape[0]), dtype=x.dtype)

    _done = True


def dtype_code(dtype: torch.dtype) -> int:
    """The ``out_dtype`` integer of ``gemm_a8`` for a torch dtype."""
    return _CODES[dtype]


register()

__all__ = ["register", "dtype_code"]
