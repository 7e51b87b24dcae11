"""GPU parity of the drop-in layer (``IntCrushOps.Linear``) against the
reference's own outputs (tests/golden) and the oracle.

Bars: A8 paths (INT8 W8A8, INT4 W4A8) max-rel <= 3e-2 against the reference's
dequant-then-linear output; W4A16 / PyTorch-semantics INT4 paths max-rel
<= 1e-3; graph replay bit-identical to the eager B200 forward.
max-rel = max|y - y_ref| / max|y_ref|.
"""

import os
import types

import numpy as np
import pytest
import torch

import comfy_stub
import intcrush_oracle as O
from _pkg import load

pytestmark = pytest.mark.gpu

comfy_stub.install()
ql = load("quant_layout")
ql.register_intcrush_layouts()
rt = load("_b200_runtime")
ops = load("_ops")

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz"))


def h(name):
    return torch.from_numpy(G[name].view(np.float16).copy())


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda")


def make_layer(fmt, rot, sd, K, N, name="blocks.0.attn.qkv", **kw):
    Ops = ops.make_intcrush_ops(fmt, rot, **kw)
    parent, lin = comfy_stub.make_parent(Ops.Linear, K, N, name=name)
    parent.cuda()
    parent.load_state_dict({f"{name}.{k}": v for k, v in sd.items()}, strict=False)
    return lin


def int8_layer():
    return make_layer("int8_crush", 64, {
        "weight": torch.from_numpy(G["int8_q"]), "weight_scale": h("int8_s"),
        "weight_perm": torch.from_numpy(G["int8_perm"]), "weight_smooth": h("int8_smooth"),
        "bias": h("int8_bias")}, 512, 128)


@pytest.mark.parametrize("graphs", [False, True])
def test_int8_layer_vs_reference(graphs, monkeypatch):
    _dev()
    monkeypatch.setattr(rt, "USE_CUDA_GRAPHS", graphs)
    lin = int8_layer()
    x = h("int8_x").cuda()
    y = lin(x)
    y2 = lin(x)   # graph replay on the second call
    assert y.dtype == torch.float16 and y.shape == (8, 128)
    assert O.max_rel(y.float().cpu().numpy(), G["int8_y"].view(np.float16)) <= 3e-2
    assert torch.equal(y, y2)
    if graphs:
        assert lin._graph_runner is not None and len(lin._graph_runner._graphs) == 1


def test_int8_graph_replay_matches_eager(monkeypatch):
    _dev()
    x = torch.randn(33, 512, dtype=torch.float16, device="cuda")
    monkeypatch.setattr(rt, "USE_CUDA_GRAPHS", False)
    y_eager = int8_layer()(x).clone()
    monkeypatch.setattr(rt, "USE_CUDA_GRAPHS", True)
    lin = int8_layer()
    lin(x)
    x2 = torch.randn(33, 512, dtype=torch.float16, device="cuda")
    y_graph = lin(x2).clone()
    monkeypatch.setattr(rt, "USE_CUDA_GRAPHS", False)
    assert torch.equal(lin(x2), y_graph)
    assert torch.equal(int8_layer()(x), y_eager)


def int4_sd(rowwise=True, G_=4):
    packed = torch.from_numpy(G["int4_packed"])
    s = h("int4_s") if rowwise else (torch.rand(128, G_) * 1.9e-2 + 1e-3).half()
    return {"weight": packed, "weight_scale": s, "weight_perm": torch.from_numpy(G["int4_perm"]),
            "weight_smoothrot_factors": h("int4_sr")}


def test_int4_pytorch_path_vs_reference():
    _dev()
    lin = make_layer("int4_crush", 256, int4_sd(), 512, 128, name="blocks.0.mlp.fc1", use_pytorch=True)
    y = lin(h("int4_x").cuda())
    assert O.max_rel(y.float().cpu().numpy(), G["int4_y"].view(np.float16)) <= 1e-3


def test_int4_w4a16_rot0_vs_reference():
    _dev()
    lin = make_layer("int4_crush", 0, {"weight": torch.from_numpy(G["int4_packed"]), "weight_scale": h("int4_s")},
                     512, 128, name="blocks.0.mlp.fc2", use_w4a16=True)
    y = lin(h("int4r0_x").cuda())
    assert O.max_rel(y.float().cpu().numpy(), G["int4r0_y"].view(np.float16)) <= 1e-3


def test_int4_w4a8_per_row_vs_reference():
    """W4A8 (INT8 activations) against the reference's dequant-linear output."""
    _dev()
    lin = make_layer("int4_crush", 256, int4_sd(), 512, 128, name="blocks.0.mlp.fc1")
    y = lin(h("int4_x").cuda())
    assert O.max_rel(y.float().cpu().numpy(), G["int4_y"].view(np.float16)) <= 3e-2


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_int4_w4a8_group_scales_vs_oracle(dtype):
    _dev()
    sd = int4_sd(rowwise=False)
    sd["bias"] = (torch.randn(128) * 0.02).half()
    lin = make_layer("int4_crush", 256, sd, 512, 128, name="blocks.0.mlp.fc1")
    x = h("int4_x").to(dtype)
    y = lin(x.cuda())
    assert y.dtype == dtype
    # bf16 activations: the oracle runs on the bf16 values (float32 arrays)
    act = "f16" if dtype == torch.float16 else "bf16"
    x_in = x.float().numpy().astype(np.float16 if act == "f16" else np.float32)
    xp = O.prep_activation(x_in, smoothrot=sd["weight_smoothrot_factors"].float().numpy(), rot_need=True,
                           rot_size=256, w_in=512, perm=G["int4_perm"], int8_path=False, act=act)
    q, s = O.quantize_rows(xp)
    ref = O.gemm_a8(q, s, O.unpack_int4(G["int4_packed"], 512), sd["weight_scale"].float().numpy(),
                    bias=sd["bias"].numpy(), group_size=128)
    assert O.max_rel(y.float().cpu().numpy(), ref) <= 3e-2
    assert O.max_rel(y.float().cpu().numpy(), ref) <= 5e-3


class _Lora:
    name = "lora"

    def __init__(self, up, down, alpha):
        self.weights = (up, down, alpha)


def test_standard_lora_residual_on_raw_input():
    _dev()
    for path in ("w4a8", "w4a16"):
        kw = {"use_w4a16": True} if path == "w4a16" else {}
        lin = make_layer("int4_crush", 256, int4_sd(), 512, 128, name="blocks.0.mlp.fc1", **kw)
        x = h("int4_x").cuda()
        base = lin(x).float().cpu().numpy()
        g = torch.Generator().manual_seed(3)
        up = (torch.randn(128, 16, generator=g) * 0.05).half()
        down = (torch.randn(16, 512, generator=g) * 0.05).half()
        lin._intcrush_adapter = _Lora(up, down, 8.0)
        lin._intcrush_lora_strength = 0.75
        y = lin(x).float().cpu().numpy()
        res = O.lora_residual(h("int4_x").numpy(), down.numpy(), up.numpy(), 8.0 / 16 * 0.75)
        assert O.max_rel(y - base, res) <= 2e-2, path


def test_int8_zero_point_eager():
    _dev()
    sd = {"weight": torch.from_numpy(G["int8_q"]), "weight_scale": h("int8_s"),
          "weight_zp": torch.randint(-3, 4, (128,)).float(), "bias": h("int8_bias")}
    lin = make_layer("int8_crush", 64, sd, 512, 128)
    x = h("int8_x")
    y = lin(x.cuda()).float().cpu().numpy()
    xp = O.prep_activation(x.numpy(), rot_need=True, rot_size=64, w_in=512)
    q, s = O.quantize_rows(xp)
    sw = sd["weight_scale"].float().numpy().reshape(-1)
    ref = O.gemm_a8(q, s, G["int8_q"], sw, bias=sd["bias"].numpy())
    ref -= xp.astype(np.float64).sum(1, keepdims=True) * (sw * sd["weight_zp"].numpy())[None, :]
    assert O.max_rel(y, ref) <= 3e-2


def test_svd_residual_w4a8():
    _dev()
    sd = int4_sd()
    g = torch.Generator().manual_seed(5)
    sd["weight_L1"] = (torch.randn(128, 8, generator=g) * 0.05).half()
    sd["weight_L2"] = (torch.randn(8, 512, generator=g) * 0.05).half()
    lin = make_layer("int4_crush", 256, sd, 512, 128, name="blocks.0.mlp.fc1")
    x = h("int4_x")
    y = lin(x.cuda()).float().cpu().numpy()
    lin2 = make_layer("int4_crush", 256, int4_sd(), 512, 128, name="blocks.0.mlp.fc1")
    base = lin2(x.cuda()).float().cpu().numpy()
    xp = O.prep_activation(x.numpy(), smoothrot=h("int4_sr").float().numpy(), rot_need=True, rot_size=256,
                           w_in=512, perm=G["int4_perm"], int8_path=False)
    res = O.lora_residual(xp, sd["weight_L2"].numpy(), sd["weight_L1"].numpy(), 1.0)
    assert O.max_rel(y - base, res) <= 2e-2


def test_rotate_activations_cuda_matches_reference_golden():
    _dev()
    qu = load("_quant_utils")
    for rot, K in [(16, 80), (64, 256), (256, 1000), (1024, 3072), (32, 96), (128, 512)]:
        x = h(f"rot{rot}_K{K}_x").cuda()
        y = qu.rotate_activations(x, rot).cpu().numpy().view(np.uint16)
        ref = G[f"rot{rot}_K{K}_y"]
        assert (y != ref).mean() <= 1e-3


@pytest.mark.gpu
def test_flux_block_fused_norm_matches_torch_norm():
    """The benchmark's DiT block with LayerNorm + adaLN modulation fused into
    the prep kernel agrees with the same block doing them as torch ops (the
    two differ only in where fp16 rounding happens)."""
    import os
    import sys
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    rt = bench._pkg()
    dev = torch.device("cuda")
    kw = dict(hidden=512, heads=4, mlp=1024)
    fused = bench.FluxDoubleBlock(rt, dev, seed=3, fused_norm=True, **kw)
    plain = bench.FluxDoubleBlock(rt, dev, seed=3, fused_norm=False, **kw)
    g = torch.Generator().manual_seed(5)
    img = torch.randn(1, 96, 512, generator=g).half().to(dev)
    txt = torch.randn(1, 32, 512, generator=g).half().to(dev)
    vec = torch.randn(1, 512, generator=g).half().to(dev)
    with torch.no_grad():
        a_img, a_txt = fused(img, txt, vec)
        b_img, b_txt = plain(img, txt, vec)
    for a, b in ((a_img, b_img), (a_txt, b_txt)):
        assert torch.isfinite(a).all()
        err = (a.float() - b.float()).abs().max() / b.float().abs().max()
        assert err <= 2e-2, float(err)


@pytest.mark.parametrize("path", ["pytorch", "w4a16"])
def test_int4_bf16_activation_paths_with_rank128_lora(path):
    """bf16 models on the dequant-then-linear INT4 paths, with a rank-128
    standard LoRA: the reference's PyTorch path (_ops.py:483-491) casts the
    dequantised weight to the activation dtype, and its LoRA takes any dtype
    and rank (_ops.py:236-244).  Checked against that math in float64 on the
    same bf16 values.  Bar: max-rel 4e-3 (bf16 output rounding is 2^-9)."""
    _dev()
    kw = {"use_pytorch": True} if path == "pytorch" else {"use_w4a16": True}
    lin = make_layer("int4_crush", 256, int4_sd(), 512, 128, name="blocks.0.mlp.fc1", **kw)
    x = h("int4_x").to(torch.bfloat16)
    g = torch.Generator().manual_seed(7)
    up = (torch.randn(128, 128, generator=g) * 0.05).to(torch.bfloat16)
    down = (torch.randn(128, 512, generator=g) * 0.05).to(torch.bfloat16)
    lin._intcrush_adapter = _Lora(up, down, 64.0)
    lin._intcrush_lora_strength = 0.5
    y = lin(x.cuda())
    assert y.dtype == torch.bfloat16
    xp = O.prep_activation(x.float().numpy(), smoothrot=h("int4_sr").float().numpy(), rot_need=True, rot_size=256,
                           w_in=512, perm=G["int4_perm"], int8_path=False, act="bf16")
    q = O.unpack_int4(G["int4_packed"], 512).astype(np.float64)
    s = h("int4_s").float().numpy().astype(np.float64).reshape(-1, 1)
    wb = O.bf16(q * s)
    ref = xp.astype(np.float64) @ wb.T.astype(np.float64)
    ref += O.lora_residual(x.float().numpy(), down.float().numpy(), up.float().numpy(), 64.0 / 128 * 0.5)
    assert O.max_rel(y.float().cpu().numpy(), ref) <= 4e-3


def test_torch_custom_ops_match_runtime_calls():
    """``torch.ops.intcrush_b200.*`` run the same kernels as the ctypes
    runtime calls: identical bits."""
    _dev()
    load("_torch_ops")
    tops = load("_torch_ops")
    ops = torch.ops.intcrush_b200
    g = torch.Generator().manual_seed(2)
    x = torch.randn(300, 3072, generator=g).half().cuda()
    sr = (torch.rand(3072, generator=g) * 3.5 + 0.5).cuda()
    perm = torch.randperm(3072, generator=g).int().cuda()
    xq, s_a = ops.prep_quantize(x, sr, perm, None, 256, 3072)
    xq2, s_a2, _, _ = rt.prep_quantize(x, smoothrot=sr, rot_size=256, w_in=3072, perm=perm)
    assert torch.equal(xq, xq2) and torch.equal(s_a, s_a2)
    q = torch.randint(-8, 8, (640, 3072), generator=g, dtype=torch.int8)
    qu = (q.to(torch.int16) & 0xF).to(torch.uint8)
    packed = (qu[:, 0::2] | (qu[:, 1::2] << 4)).contiguous().cuda()
    s_w = (torch.rand(640, 24, generator=g) * 1e-2 + 1e-3).cuda()
    y = ops.gemm_a8(xq, packed, s_w, s_a, None, tops.dtype_code(torch.float16), 128, False)
    assert torch.equal(y, rt.gemm_a8(xq2, packed, s_w, s_a2, out_dtype=torch.float16, group_size=128))
    z = ops.gemm_w4a16(x[:16], packed, s_w.half(), 128, 0)
    assert torch.equal(z, rt.gemm_w4a16(x[:16], packed, s_w.half(), group_size=128))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_convlinear_modules_on_cuda(dtype):
    """ConvLinear4bit (B200 prep + W4A16 kernels) and ConvLinear8bit (B200
    prep, torch dequantised linear) against their math in float64: rotate,
    permute, dequantise per row, linear, bias."""
    _dev()
    conv = load("convlinear")
    qu = load("_quant_utils")
    g = torch.Generator().manual_seed(4)
    lin = torch.nn.Linear(512, 192)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(192, 512, generator=g) * 0.05)
        lin.bias.copy_(torch.randn(192, generator=g) * 0.02)
    perm = torch.randperm(512, generator=g)
    x = torch.randn(40, 512, generator=g).to(dtype)
    m4 = conv.ConvLinear4bit.from_float(lin, rot_need=True, rot_size=64, perm=perm).cuda()
    m8 = conv.ConvLinear8bit.from_float(lin, rot_need=True, rot_size=64).cuda()
    y4 = m4(x.cuda())
    y8 = m8(x.cuda())
    assert y4.dtype == dtype and y8.dtype == dtype
    H = torch.from_numpy(O.hadamard(64))
    xr = (x.double().reshape(40, 8, 64) @ H.T).reshape(40, 512).to(dtype).double()
    w4 = qu.unpack_int4(m4.weight.cpu(), 512).double() * m4.scale.cpu().double().reshape(-1, 1)
    w4 = w4.to(dtype).double()
    ref4 = xr[:, perm] @ w4.T + lin.bias.detach().double()
    w8 = (m8.weight.cpu().to(dtype) * m8.scale.cpu().to(dtype)).double()
    ref8 = xr @ w8.T + lin.bias.detach().double()
    tol = 1e-3 if dtype == torch.float16 else 4e-3
    assert float((y4.cpu().double() - ref4).abs().max() / ref4.abs().max()) <= tol
    assert float((y8.cpu().double() - ref8).abs().max() / ref8.abs().max()) <= tol


class _LoKr:
    name = "lokr"

    def __init__(self, w1, w2_a, w2_b, alpha):
        # (w1, w2, alpha, w1_a, w1_b, w2_a, w2_b): w2 from its low-rank factors
        self.weights = (w1, None, alpha, None, None, w2_a, w2_b)


def test_lokr_residual_through_the_layer():
    """A LoKr adapter on an INT8 layer adds the Kronecker residual
    scale * (w1 (x) w2) x_raw (fp64 oracle) to the layer's plain output."""
    _dev()
    lin = int8_layer()
    x = h("int8_x").cuda()
    base = lin(x).float()
    g = torch.Generator().manual_seed(5)
    w1 = (torch.randn(4, 4, generator=g) * 0.5).half()              # out_l = in_m = 4
    w2_a = (torch.randn(32, 8, generator=g) * 0.1).half()           # out_k = 32 (128 / 4), rank 8
    w2_b = (torch.randn(8, 128, generator=g) * 0.1).half()          # in_n = 128 (512 / 4)
    lin._intcrush_adapter = _LoKr(w1, w2_a, w2_b, 4.0)
    lin._intcrush_lora_strength = 0.5
    y = lin(x).float()
    w2 = w2_a.double() @ w2_b.double()
    dW = torch.kron(w1.double(), w2) * (4.0 / 8 * 0.5)
    res = h("int8_x").double() @ dW.T
    # the residual is added to the layer's fp16 output and the sum rounded:
    # compare y with base + res at one fp16 ulp of y plus 5e-3 of the
    # residual's scale (its fp16 factors and intermediates); the difference
    # y - base alone would be dominated by the fp16 rounding of two outputs
    # ~100 times larger than the residual
    err = (y.double().cpu() - (base.double().cpu() + res)).abs()
    tol = y.double().cpu().abs() * 2.0 ** -10 + 5e-3 * res.abs().max()
    assert torch.all(err <= tol), (err - tol).max().item()


def test_set_weight_requantises_on_device():
    """set_weight with a float weight on CUDA requantises through the device
    kernel: same int8 data and scales as the layout's torch form on CPU."""
    _dev()
    lin = int8_layer()
    g = torch.Generator().manual_seed(9)
    w = torch.randn(128, 512, generator=g) * 0.02
    lin.set_weight(w.cuda())
    q_ref, p_ref = ql.IntCrushInt8Layout.quantize(w, scale="recalculate")
    assert torch.equal(lin.weight._qdata.cpu(), q_ref)
    assert torch.equal(lin.weight._params.scale.cpu(), p_ref.scale)
    y = lin(h("int8_x").cuda())
    assert torch.isfinite(y).all()
