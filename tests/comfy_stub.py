"""Minimal stand-in for the parts of ComfyUI that the INT-Crush layers touch.

ComfyUI is the host application and is not installed here.  The layers need:
``comfy.ops.manual_cast`` (Linear/GroupNorm/LayerNorm/Conv*/Embedding with
``comfy_cast_weights``, ``weight_function``, ``bias_function``),
``cast_bias_weight``/``uncast_bias_weight`` and ``comfy.quant_ops``
(``QuantizedTensor``, ``QUANT_ALGOS``, ``register_layout_class``,
``get_layout_class``).  ``install()`` puts such modules into ``sys.modules``.
Used by the tests (and by ``tests/golden/make_golden.py`` to run the
reference's own layer on CPU).
"""

from __future__ import annotations

import sys
import types

import torch
import torch.nn as nn


class QuantizedTensor(torch.Tensor):
    """Tensor subclass carrying ``_qdata``, ``_layout_type`` and ``_params``."""

    @staticmethod
    def __new__(cls, qdata, layout_type, params):
        t = torch.Tensor._make_subclass(cls, torch.empty(0, device=qdata.device), False)
        t._qdata = qdata
        t._layout_type = layout_type
        t._params = params
        return t

    def __init__(self, qdata, layout_type, params):
        pass

    def detach(self):
        return self

    @property
    def device(self):
        return self._qdata.device

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        return super().__torch_function__(func, types, args, kwargs)


def install() -> None:
    if "comfy" in sys.modules and getattr(sys.modules["comfy"], "_intcrush_stub", False):
        return
    comfy = types.ModuleType("comfy")
    comfy._intcrush_stub = True
    ops = types.ModuleType("comfy.ops")
    qops = types.ModuleType("comfy.quant_ops")

    class _CastMixin:
        comfy_cast_weights = False

        def _init_cast(self):
            self.weight_function = []
            self.bias_function = []

    class manual_cast:
        class Linear(nn.Linear, _CastMixin):
            def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
                super().__init__(in_features, out_features, bias=bias)
                self._init_cast()

        class GroupNorm(nn.GroupNorm, _CastMixin):
            pass

        class LayerNorm(nn.LayerNorm, _CastMixin):
            pass

        class Conv2d(nn.Conv2d, _CastMixin):
            pass

        class Conv3d(nn.Conv3d, _CastMixin):
            pass

        class ConvTranspose2d(nn.ConvTranspose2d, _CastMixin):
            pass

        class Embedding(nn.Embedding, _CastMixin):
            pass

    def cast_bias_weight(module, input=None, dtype=None, device=None, bias_dtype=None, offloadable=False):
        return module.weight, module.bias, None

    def uncast_bias_weight(module, weight, bias, offload_stream):
        return None

    ops.manual_cast = manual_cast
    ops.cast_bias_weight = cast_bias_weight
    ops.uncast_bias_weight = uncast_bias_weight

    layouts: dict = {}
    qops.QUANT_ALGOS = {}
    qops.QuantizedTensor = QuantizedTensor
    qops.register_layout_class = lambda name, cls: layouts.__setitem__(name, cls)
    qops.get_layout_class = lambda name: layouts[name]

    comfy.ops = ops
    comfy.quant_ops = qops
    sys.modules["comfy"] = comfy
    sys.modules["comfy.ops"] = ops
    sys.modules["comfy.quant_ops"] = qops


def make_parent(linear_cls, in_features, out_features, name="blocks.0.attn.qkv", bias=True):
    """A parent module holding one Linear at ``name`` (so the state-dict
    prefix is non-empty, as in a real model)."""
    root = nn.Module()
    cur = root
    parts = name.split(".")
    for p in parts[:-1]:
        nxt = nn.Module()
        cur.add_module(p, nxt)
        cur = nxt
    cur.add_module(parts[-1], linear_cls(in_features, out_features, bias=bias))
    return root, cur._modules[parts[-1]]
