"""Generate golden fixtures by running the reference ComfyUI-INT-Crush on CPU.

Run once in a checkout where the reference is available (it is not shipped
with this repository, and the GPU test machines do not have it):

    python tests/golden/make_golden.py /path/to/ComfyUI-INT-Crush

Writes ``tests/golden/reference_golden.npz``.  Everything is computed by the
reference's own functions and its own ``IntCrushOps.Linear`` forward
(PyTorch CPU paths; the Triton paths need a GPU):

* ``rotate_activations`` (``_quant_utils.py:117-147``) for regular and
  Sylvester sizes, with K not a multiple of the rotation size;
* ``dynamic_quantize_activation`` CPU form (``kernels/triton_quantize.py:43-54``);
* ``pack_int4`` on the reference's own known-answer values;
* full layer forwards: INT8 (``_ops.py:537-545``, rot 64, perm, SmoothQuant,
  bias) and INT4 PyTorch path (``_ops.py:483-491``, per-row scales,
  SmoothRot + rot 256 + perm; and rot 0 / W4A16 semantics).
"""

from __future__ import annotations

import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))   # tests/ (comfy_stub)

REF_PKG = "ComfyUI-INT-Crush"


def load_reference(path: str):
    pkg = types.ModuleType(REF_PKG)
    pkg.__path__ = [path]
    pkg.__package__ = REF_PKG
    sys.modules[REF_PKG] = pkg
    return lambda name: importlib.import_module(f"{REF_PKG}.{name}")


def x_with_outliers(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    ch = torch.randperm(K, generator=g)[: max(1, round(0.01 * K))]
    x[:, ch] *= 20
    return x.half()


def build_layer(ops_cls, name, sd, in_f, out_f):
    import comfy_stub
    parent, lin = comfy_stub.make_parent(ops_cls.Linear, in_f, out_f, name=name)
    prefix = name + "."
    full = {prefix + k: v for k, v in sd.items()}
    parent.load_state_dict(full, strict=False)
    return lin


def main(ref_path: str) -> None:
    import comfy_stub
    comfy_stub.install()
    load = load_reference(ref_path)
    qu = load("_quant_utils")
    tq = load("kernels.triton_quantize")
    ql = load("quant_layout")
    ql.register_intcrush_layouts()
    tr = load("_triton_runtime")
    tr.TRITON_AVAILABLE = False          # reference CPU paths
    tr.USE_CUDA_GRAPHS = False
    ops = load("_ops")

    out: dict[str, np.ndarray] = {}
    # rotation
    for rot, K in [(16, 80), (64, 256), (256, 1000), (1024, 3072), (32, 96), (128, 512)]:
        x = x_with_outliers(4, K, seed=rot + K)
        y = qu.rotate_activations(x, rot)
        out[f"rot{rot}_K{K}_x"] = x.numpy().view(np.uint16)
        out[f"rot{rot}_K{K}_y"] = y.numpy().view(np.uint16)
    # dynamic quantisation (CPU form of the reference)
    for M, K in [(1, 64), (4, 256), (16, 1024)]:
        torch.manual_seed(M)
        x = x_with_outliers(M, K, seed=M * 3 + K)
        q, s = tq.dynamic_quantize_activation(x)
        out[f"dq_M{M}_K{K}_x"] = x.numpy().view(np.uint16)
        out[f"dq_M{M}_K{K}_q"] = q.numpy()
        out[f"dq_M{M}_K{K}_s"] = s.numpy()
    # pack KAT
    vals = torch.tensor([-8, -1, 0, 1, 7, -3, 5, 0], dtype=torch.int8)
    out["pack_vals"] = vals.numpy()
    out["pack_bytes"] = qu.pack_int4(vals).numpy()

    g = torch.Generator().manual_seed(7)
    # INT8 layer: rot 64, perm, SmoothQuant (no SmoothRot), bias
    N, K, M = 128, 512, 8
    q8 = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s8 = (torch.rand(N, 1, generator=g) * 9e-3 + 1e-3).half()
    perm = torch.randperm(K, generator=g)
    smooth = (torch.rand(K, generator=g) * 1.5 + 0.5).half()
    bias = (torch.randn(N, generator=g) * 0.02).half()
    x = x_with_outliers(M, K, seed=11)
    ops8 = ops.make_intcrush_ops("int8_crush", 64)
    lin = build_layer(ops8, "blocks.0.attn.qkv",
                      {"weight": q8, "weight_scale": s8, "weight_perm": perm, "weight_smooth": smooth,
                       "bias": bias}, K, N)
    y = lin(x)
    out.update(int8_x=x.numpy().view(np.uint16), int8_q=q8.numpy(), int8_s=s8.numpy().view(np.uint16),
               int8_perm=perm.numpy(), int8_smooth=smooth.numpy().view(np.uint16),
               int8_bias=bias.numpy().view(np.uint16), int8_y=y.numpy().view(np.uint16))

    # INT4 layer, PyTorch path: SmoothRot + rot 256 + perm, per-row scales
    N, K, M = 128, 512, 8
    q4 = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int8)
    packed = qu.pack_int4(q4)
    s4 = (torch.rand(N, 1, generator=g) * 1.9e-2 + 1e-3).half()
    perm4 = torch.randperm(K, generator=g)
    sr = (torch.rand(K, generator=g) * 3.5 + 0.5).half()
    x = x_with_outliers(M, K, seed=12)
    ops4 = ops.make_intcrush_ops("int4_crush", 256, use_pytorch=True)
    lin = build_layer(ops4, "blocks.0.mlp.fc1",
                      {"weight": packed, "weight_scale": s4, "weight_perm": perm4,
                       "weight_smoothrot_factors": sr}, K, N)
    y = lin(x)
    out.update(int4_x=x.numpy().view(np.uint16), int4_packed=packed.numpy(), int4_s=s4.numpy().view(np.uint16),
               int4_perm=perm4.numpy(), int4_sr=sr.numpy().view(np.uint16), int4_y=y.numpy().view(np.uint16))

    # INT4 layer with rot 0 (the W4A16 configuration; same dequant-linear math)
    ops40 = ops.make_intcrush_ops("int4_crush", 0, use_pytorch=True)
    x = x_with_outliers(M, K, seed=13)
    lin = build_layer(ops40, "blocks.0.mlp.fc2", {"weight": packed, "weight_scale": s4}, K, N)
    y = lin(x)
    out.update(int4r0_x=x.numpy().view(np.uint16), int4r0_y=y.numpy().view(np.uint16))

    np.savez_compressed(os.path.join(HERE, "reference_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_golden.npz"), len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("INTCRUSH_REFERENCE", ""))
