"""Pin the CPU oracle on the reference's own outputs (tests/golden, produced by
tests/golden/make_golden.py from the reference's CPU code)."""

import os

import numpy as np
import pytest

import intcrush_oracle as O

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_golden.npz"))


def h(name):
    return G[name].view(np.float16)


@pytest.mark.parametrize("rot,K", [(16, 80), (64, 256), (256, 1000), (1024, 3072), (32, 96), (128, 512)])
def test_oracle_rotation_matches_reference(rot, K):
    """The oracle rotates exactly and rounds once; the reference accumulates the
    fp16 matmul in fp32.  They must agree except at fp16 rounding ties."""
    x, y = h(f"rot{rot}_K{K}_x"), h(f"rot{rot}_K{K}_y")
    mine = O.rotate(x, rot)
    assert mine.shape == y.shape
    diff = mine.view(np.uint16) != y.view(np.uint16)
    assert diff.mean() <= 1e-3, f"{diff.sum()} of {diff.size} differ"
    # any difference is a single fp16 ulp
    d = np.abs(mine.astype(np.float64) - y.astype(np.float64))
    ulp = np.spacing(np.abs(y).astype(np.float16)).astype(np.float64)
    assert np.all(d <= ulp + 1e-12)


@pytest.mark.parametrize("M,K", [(1, 64), (4, 256), (16, 1024)])
def test_oracle_quantisation_bit_exact(M, K):
    x = h(f"dq_M{M}_K{K}_x")
    q, s = O.quantize_rows(x)
    assert np.array_equal(q, G[f"dq_M{M}_K{K}_q"])
    assert np.array_equal(s, G[f"dq_M{M}_K{K}_s"])


def test_oracle_pack_known_answer():
    assert np.array_equal(O.pack_int4(G["pack_vals"]), G["pack_bytes"])
    assert np.array_equal(O.unpack_int4(G["pack_bytes"], 8), G["pack_vals"])


def test_oracle_int8_layer_dequant_path():
    """Reference INT8 PyTorch path: prep (rot 64, perm, smooth) then
    F.linear(x, fp16(q) * fp16(s), bias)."""
    x = h("int8_x")
    xp = O.prep_activation(x, rot_need=True, rot_size=64, w_in=512, perm=G["int8_perm"],
                           smooth=h("int8_smooth").astype(np.float32), int8_path=True)
    w16 = (G["int8_q"].astype(np.float16) * h("int8_s")).astype(np.float16)
    y = O.linear_f16(xp, w16, h("int8_bias"))
    assert O.max_rel(y, h("int8_y")) <= 1e-3


def test_oracle_int4_layer_pytorch_path():
    x = h("int4_x")
    xp = O.prep_activation(x, smoothrot=h("int4_sr").astype(np.float32), rot_need=True, rot_size=256,
                           w_in=512, perm=G["int4_perm"], int8_path=False)
    w16 = O.dequant_int4_f16(G["int4_packed"], h("int4_s").astype(np.float32), 512)
    assert O.max_rel(O.linear_f16(xp, w16), h("int4_y")) <= 1e-3
    xr = h("int4r0_x")
    assert O.max_rel(O.linear_f16(xr, w16), h("int4r0_y")) <= 1e-3


def test_torch_reference_path_matches_reference_golden():
    """The torch restatement timed as the CPU baseline reproduces the
    reference's own layer outputs (max-rel <= 1e-3, the fp16 output bar)."""
    import torch
    import torch_reference_path as TR

    def t(name):
        return torch.from_numpy(h(name).copy())

    y4 = TR.forward_int4_pytorch(t("int4_x"), torch.from_numpy(G["int4_packed"]), t("int4_s"), 512, 512,
                                 smoothrot=t("int4_sr"), rot_size=256, w_in=512,
                                 perm=torch.from_numpy(G["int4_perm"]))
    assert O.max_rel(y4.numpy(), h("int4_y")) <= 1e-3
    y40 = TR.forward_int4_pytorch(t("int4r0_x"), torch.from_numpy(G["int4_packed"]), t("int4_s"), 512, 512)
    assert O.max_rel(y40.numpy(), h("int4r0_y")) <= 1e-3
    y8 = TR.forward_int8_pytorch(t("int8_x"), torch.from_numpy(G["int8_q"]), t("int8_s"), t("int8_bias"),
                                 rot_size=64, w_in=512, perm=torch.from_numpy(G["int8_perm"]),
                                 smooth=t("int8_smooth"))
    assert O.max_rel(y8.numpy(), h("int8_y")) <= 1e-3
    # the group-128 dequantisation the baseline uses reduces to the per-row one for equal group scales
    s_g = t("int4_s").float().repeat(1, 4)
    yg = TR.forward_int4_pytorch(t("int4r0_x"), torch.from_numpy(G["int4_packed"]), s_g, 512, 128)
    assert O.max_rel(yg.numpy(), h("int4r0_y")) <= 1e-3
