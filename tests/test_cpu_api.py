"""Host-side API of the package on CPU: quantisation utilities (the
reference's tests/test_quant_utils.py and test_convlinear.py cases), layouts,
loader metadata handling, LoRA attach/clear, layer state-dict loading and the
no-CPU-fallback rule."""

import math
import types

import numpy as np
import pytest
import torch

import comfy_stub
from _pkg import load

comfy_stub.install()
qu = load("_quant_utils")
ql = load("quant_layout")
ql.register_intcrush_layouts()
rt = load("_b200_runtime")
ops = load("_ops")
loaders = load("_loaders")
lora = load("_lora")
conv = load("convlinear")
tr = load("_triton_runtime")


# ── _quant_utils (reference tests/test_quant_utils.py) ──────────────────────
def test_power_checks():
    assert qu.is_power_of_two(1) and qu.is_power_of_two(64) and not qu.is_power_of_two(12)
    assert qu._is_power_of_four(4) and qu._is_power_of_four(4096) and not qu._is_power_of_four(8)
    assert not qu._is_power_of_four(-4)


@pytest.mark.parametrize("n", [4, 16, 64, 256, 1024])
def test_hadamard_regular(n):
    H = qu.make_hadamard_regular(n, dtype=torch.float32)
    assert H.shape == (n, n)
    assert torch.allclose(H @ H.T, torch.eye(n), atol=1e-5)
    assert torch.allclose(H.abs(), torch.full_like(H, 1 / math.sqrt(n)), atol=1e-6)
    with pytest.raises(ValueError):
        qu.make_hadamard_regular(12)


def test_hadamard_sylvester_orthonormal():
    H = qu._make_hadamard_sylvester(32, dtype=torch.float32)
    assert torch.allclose(H @ H.T, torch.eye(32), atol=1e-5)


@pytest.mark.parametrize("vals,K", [([-8, -1, 0, 1, 7, -3, 5, 0], 8), ([-8, 0, 7], 3)])
def test_pack_roundtrip(vals, K):
    v = torch.tensor(vals, dtype=torch.int8)
    assert torch.equal(qu.unpack_int4(qu.pack_int4(v), K), v)


def test_pack_shapes_and_extremes():
    v = torch.randint(-8, 8, (4, 33), dtype=torch.int8)
    assert qu.pack_int4(v).shape == (4, 17)
    for c in (-8, 7):
        v = torch.full((2, 16), c, dtype=torch.int8)
        assert torch.equal(qu.unpack_int4(qu.pack_int4(v), 16), v)
    with pytest.raises(ValueError):
        qu.validate_int4_range(torch.tensor([8]))
    with pytest.raises(ValueError):
        qu.validate_int4_range(torch.tensor([-9]))
    assert qu.INT4_SCALE_DIVISOR == 7.0 and (qu.INT4_MIN, qu.INT4_MAX) == (-8, 7)


def test_rotate_activations_cpu_pads_and_preserves_norm():
    x = torch.randn(3, 100)
    y = qu.rotate_activations(x, 64)
    assert y.shape == (3, 128)
    assert torch.allclose(y.norm(dim=1), x.norm(dim=1), rtol=1e-5)


def test_group_scales_and_quantize():
    W = torch.randn(8, 300)
    s = qu.calculate_scales(W, 128)
    assert s.shape == (8, 3) and s.dtype == torch.float16
    q = qu.quantize_weights(W, s, 128)
    assert q.shape == (8, 384) and q.min() >= -8 and q.max() <= 7


def test_convlinear_from_float_shapes():
    lin = torch.nn.Linear(32, 32)
    m = conv.ConvLinear4bit.from_float(lin, rot_need=True, rot_size=16)
    assert m.weight.shape == (32, 16) and m.scale.shape == (32, 1)
    m8 = conv.ConvLinear8bit.from_float(lin, rot_need=True, rot_size=16)
    assert m8.weight.dtype == torch.int8 and m8.scale.shape == (32, 1)
    with pytest.raises(RuntimeError):
        m(torch.randn(2, 32).half())   # no CPU fallback


# ── layouts ─────────────────────────────────────────────────────────────────
def test_int4_layout_dequantize_per_row_and_group():
    q = torch.randint(-8, 8, (4, 256), dtype=torch.int8)
    packed = qu.pack_int4(q)
    s_row = torch.rand(4) + 0.1
    p = ql.IntCrushInt4Layout.Params(scale=s_row, orig_dtype=torch.float16, orig_shape=(4, 256))
    assert torch.allclose(ql.IntCrushInt4Layout.dequantize(packed, p), q.float() * s_row[:, None])
    s_grp = torch.rand(4, 2) + 0.1
    p = ql.IntCrushInt4Layout.Params(scale=s_grp, orig_dtype=torch.float16, orig_shape=(4, 256))
    ref = q.float() * s_grp.repeat_interleave(128, dim=1)
    assert torch.allclose(ql.IntCrushInt4Layout.dequantize(packed, p), ref)


def test_layout_quantize_roundtrip_and_registry():
    W = torch.randn(8, 64)
    packed, params = ql.IntCrushInt4Layout.quantize(W)
    back = ql.IntCrushInt4Layout.dequantize(packed, params)
    assert (back - W).abs().max() <= params.scale.float().max() * 0.51 + 1e-6
    import comfy.quant_ops as cq
    assert "int4_crush" in cq.QUANT_ALGOS and cq.get_layout_class("IntCrushInt8Layout") is ql.IntCrushInt8Layout
    assert not ql.IntCrushInt4Layout.supports_fast_matmul() or torch.cuda.is_available()


# ── runtime flags / boundary ────────────────────────────────────────────────
def test_runtime_exports_reference_names():
    for name in ["TRITON_AVAILABLE", "TRITON_INT4_UNPACK", "TRITON_INT8_GEMM", "TRITON_INT4_INT8_UNPACK",
                 "TRITON_DYNQUANT", "TRITON_W4A8_GEMM", "TRITON_FUSED_QGD", "USE_FUSED_W8A8", "USE_CUDA_GRAPHS",
                 "dynamic_quantize_activation", "fused_int8_gemm_dequant", "fused_quant_int8_gemm_dequant",
                 "fused_w4a8_gemm_dequant", "unpack_int4_to_int8", "unpack_int4_to_float16"]:
        assert hasattr(tr, name)
    assert rt.B200_LIBRARY_LOADED
    assert rt.TRITON_AVAILABLE == torch.cuda.is_available()


def test_ops_refuse_cpu_tensors():
    with pytest.raises(RuntimeError):
        rt.dynamic_quantize_activation(torch.randn(4, 64).half())
    with pytest.raises(RuntimeError):
        rt.gemm_a8(torch.zeros(4, 64, dtype=torch.int8), torch.zeros(8, 64, dtype=torch.int8),
                   torch.ones(8), torch.ones(4))


# ── loaders ─────────────────────────────────────────────────────────────────
def test_checkpoint_rot_size_from_metadata():
    info = loaders.CheckpointInfo
    assert info({}).rot_size(256, ("1",)) == 256
    assert info({"int_crush.format_version": "1", "int_crush.rot_size": "1024"}).rot_size(256, ("1",)) == 1024
    assert info({"int_crush.format_version": "2", "int_crush.rot_size": "1024"}).rot_size(256, ("1",)) == 256
    assert info({"int_crush.format_version": "1", "int_crush.rot_size": "48"}).rot_size(256, ("1",)) == 256
    assert info({"int_crush.format_version": "3"}).rot_size(64, ("2", "3")) == 64


def test_padded_layers_and_node_api():
    meta = {"int_crush.padded_layers": "img_in.weight=64; a.b.weight=3072"}
    assert loaders.CheckpointInfo(meta).padded_layers() == {"img_in.weight": 64, "a.b.weight": 3072}
    assert loaders.CheckpointInfo({}).padded_layers() == {}
    for cls in ("SimpleINT4UNetLoader", "SimpleINT8UNetLoader", "IntCrushLoRALoader", "IntCrushLoRAUnloader"):
        c = loaders.NODE_CLASS_MAPPINGS[cls]
        assert c.CATEGORY == "loaders/INT-Crush" and "required" in c.INPUT_TYPES()
        assert c.RETURN_TYPES == ("MODEL",) and callable(getattr(c, c.FUNCTION))
    assert loaders.SimpleINT4UNetLoader.INPUT_TYPES()["required"]["rot_size"][0] == [0, 16, 64, 256, 1024, 4096]
    assert loaders.SimpleINT4UNetLoader.INPUT_TYPES()["required"]["rot_size"][1] == {"default": 256}


def test_int4_loader_without_rotation_uses_w4a16():
    ops_cls = loaders.SimpleINT4UNetLoader()._ops_for(0)
    lin = ops_cls.Linear(64, 32)
    assert lin._intcrush_use_w4a16 is True
    assert loaders.SimpleINT4UNetLoader()._ops_for(256).Linear(64, 32)._intcrush_use_w4a16 is False


# ── layer loading (no forward on CPU) ───────────────────────────────────────
def _int4_layer(rot=256, name="blocks.0.attn.qkv", zp=False):
    Ops = ops.make_intcrush_ops("int4_crush", rot)
    parent, lin = comfy_stub.make_parent(Ops.Linear, 512, 64, name=name)
    sd = {"weight": qu.pack_int4(torch.randint(-8, 8, (64, 512), dtype=torch.int8)),
          "weight_scale": torch.rand(64, 4).half(), "weight_perm": torch.randperm(512),
          "weight_smoothrot_factors": torch.rand(512).half() + 0.5, "bias": torch.randn(64).half(),
          "comfy_quant": torch.tensor([0], dtype=torch.uint8)}
    if zp:
        sd["weight_zp"] = torch.zeros(64)
    missing = parent.load_state_dict({f"{name}.{k}": v for k, v in sd.items()}, strict=False)
    return lin, missing


def test_state_dict_loading_int4():
    lin, missing = _int4_layer()
    assert lin._intcrush_is_quantized and lin.quant_format == "int4_crush"
    assert lin._intcrush_rot_need and lin._intcrush_w_in == 512
    assert lin.weight._params.scale.dtype == torch.float32 and lin.weight._params.scale.shape == (64, 4)
    assert lin._intcrush_smoothrot_factors.dtype == torch.float32
    assert not [k for k in missing.missing_keys if "qkv" in k]


@pytest.mark.parametrize("name,expect", [("blocks.0.norm_out.linear", False), ("final_layer.proj_out", False),
                                         ("blocks.3.ff.net.0", True)])
def test_rotation_disabled_by_name(name, expect):
    lin, _ = _int4_layer(name=name)
    assert lin._intcrush_rot_need is expect


def test_forward_on_cpu_raises_no_fallback():
    lin, _ = _int4_layer()
    with pytest.raises((RuntimeError, NotImplementedError)):
        lin(torch.randn(2, 512).half())


def test_set_weight_requantises_and_drops_caches():
    lin, _ = _int4_layer()
    lin._b200 = object()
    lin._graph_runner = object()
    lin.set_weight(torch.randn(64, 512))
    assert lin._b200 is None and lin._graph_runner is None
    assert lin.weight._params.perm is lin._intcrush_perm


# ── LoRA attach / clear ─────────────────────────────────────────────────────
def test_lora_attach_and_clear(monkeypatch):
    lin, _ = _int4_layer()
    model = types.SimpleNamespace(model=torch.nn.ModuleDict({"blk": lin}))

    class Adapter:
        name = "lora"

    import sys
    wa = types.ModuleType("comfy.weight_adapter")
    wa.WeightAdapterBase = Adapter
    lc = types.ModuleType("comfy.lora_convert")
    lc.convert_lora = lambda sd: sd
    lm = types.ModuleType("comfy.lora")
    lm.model_lora_keys_unet = lambda m, d: {}
    lm.load_lora = lambda sd, km: {"blk.weight": Adapter(), "other.weight": Adapter()}
    import comfy
    for n, m in [("comfy.weight_adapter", wa), ("comfy.lora_convert", lc), ("comfy.lora", lm)]:
        monkeypatch.setitem(sys.modules, n, m)
        monkeypatch.setattr(comfy, n.split(".")[1], m, raising=False)
    attached, total = lora.attach_lora_as_buffers(model, {"x": 1}, 0.5)
    assert (attached, total) == (1, 2)
    assert lin._intcrush_lora_strength == 0.5 and isinstance(lin._intcrush_adapter, Adapter)
    assert lora.clear_intcrush_lora(model) == 1 and lin._intcrush_adapter is None


def test_torch_custom_ops_registered_with_fake_kernels():
    """The kernels are ``torch.library`` custom ops (``intcrush_b200::*``) with
    fake implementations: shapes and dtypes propagate on meta tensors
    without a GPU (what torch.compile / export trace through)."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    load("_torch_ops")
    ops = torch.ops.intcrush_b200
    with FakeTensorMode():
        x = torch.empty(37, 3000, dtype=torch.float16)
        xq, s_a = ops.prep_quantize(x, None, None, None, 256, 3072)
        assert xq.shape == (37, 3072) and xq.dtype == torch.int8 and s_a.shape == (37,)
        w = torch.empty(640, 1536, dtype=torch.uint8)
        s_w = torch.empty(640, 24)
        y = ops.gemm_a8(xq, w, s_w, s_a, None, 1, 128, False)
        assert y.shape == (37, 640) and y.dtype == torch.bfloat16
        z = ops.gemm_w4a16(torch.empty(5, 3072, dtype=torch.bfloat16), w, torch.empty(640, 24, dtype=torch.float16),
                           128, 0)
        assert z.shape == (5, 640) and z.dtype == torch.bfloat16
