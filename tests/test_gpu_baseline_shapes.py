"""GPU parity of the GEMMs and the layer at the benchmark's own shapes.

The GEMM the benchmark times (W4A8, M=4096, N=12288,
K=3072, group 128) runs 22 x 96 = 2112 work units over one persistent CTA per
SM, so every CTA walks many tiles, the tile raster has two groups of 16
token tiles, and the ring and accumulator-buffer phases carry across tiles.
These tests check that path, at that shape, three ways:

* the whole output against torch's own int8 GEMM (``torch._int_mm``, cuBLAS)
  on the same GPU: exact for unit scales (the integer accumulators), and per
  K-group rescaled in float64 for real scales;
* rows and columns that touch every tile against the CPU oracle (float64,
  exact integer sums), the parity contract proper;
* the drop-in layer (``IntCrushOps.Linear``) against the oracle's
  prep -> quantise -> GEMM on the same seeded inputs.

Bars: integer accumulators bit-exact; max-rel ``max|y - y_ref| / max|y_ref|``
<= 3e-2 (A8 contract) and, since both accumulate in fp32 or better, <= 5e-3.
"""

import numpy as np
import pytest
import torch

import comfy_stub
import intcrush_oracle as O
from _pkg import load

pytestmark = pytest.mark.gpu

rt = load("_b200_runtime")


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda")


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _sample(n, step, rng):
    """One random index in each block of ``step`` plus both ends: every tile of
    every tile width (>= step) is sampled at least once."""
    idx = {0, n - 1}
    for b in range(0, n, step):
        idx.add(int(b + rng.integers(0, min(step, n - b))))
    return np.array(sorted(idx))


def _oracle_rows_cols(xq, wq, s_a, s_w, bias, group_size, rows, cols):
    """Oracle output on the selected rows (all columns) and columns (all rows)."""
    r = O.gemm_a8(xq[rows], s_a[rows], wq, s_w, bias=bias, group_size=group_size)
    c = O.gemm_a8(xq, s_a, wq[cols], s_w[cols], bias=None if bias is None else bias[cols],
                  group_size=group_size)
    return r, c


def _torch_exact(xq_d, wq_d, s_a, s_w, bias, group_size):
    """float64 ``s_a * sum_g s_w[:, g] * P_g + bias`` from cuBLAS int8 GEMMs."""
    M, K = xq_d.shape
    G = s_w.shape[1] if s_w.dim() == 2 else 1
    gs = group_size if G > 1 else K
    acc = torch.zeros(M, wq_d.shape[0], dtype=torch.float64, device=xq_d.device)
    for g in range(G):
        P = torch._int_mm(xq_d[:, g * gs:(g + 1) * gs].contiguous(), wq_d[:, g * gs:(g + 1) * gs].t().contiguous())
        acc += P.double() * s_w.reshape(-1, G)[:, g].double()[None, :]
    acc *= s_a.double()[:, None]
    if bias is not None:
        acc += bias.double()[None, :]
    return acc


def _max_rel_t(y, ref):
    return float((y.double() - ref).abs().max() / ref.abs().max())


CONFIG2 = dict(M=4096, N=12288, K=3072, G=24)


@pytest.mark.parametrize("layout", ["reference", "repacked"])
def test_w4a8_config2_full_shape(layout):
    """configs[1]'s GEMM: 4096 x 12288 x 3072, INT4 group 128, bias, fp16 out."""
    dev = _dev()
    M, N, K, G = CONFIG2["M"], CONFIG2["N"], CONFIG2["K"], CONFIG2["G"]
    rng = np.random.default_rng(2)
    xq = rng.integers(-128, 128, (M, K), dtype=np.int64).astype(np.int8)
    wq = rng.integers(-8, 8, (N, K), dtype=np.int64).astype(np.int8)
    packed = _t(O.pack_int4(wq), dev)
    w = rt.repack_int4(packed, K, 0) if layout == "repacked" else packed
    rep = layout == "repacked"
    xq_d, wq_d = _t(xq, dev), _t(wq, dev)

    # 1. integer accumulators, whole output, exact (|acc| < 2^24 for INT4)
    ones = rt.gemm_a8(xq_d, w, torch.ones(N, G, device=dev), torch.ones(M, device=dev), out_dtype=torch.float32,
                      group_size=128, repacked=rep)
    ref_int = torch._int_mm(xq_d, wq_d.t().contiguous())
    assert torch.equal(ones.to(torch.int64), ref_int.to(torch.int64)), "integer accumulators differ"

    # 2. real scales and bias: whole output against the float64 group rescale
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    out = rt.gemm_a8(xq_d, w, _t(s_w, dev), _t(s_a, dev), bias=_t(bias, dev), out_dtype=torch.float16,
                     group_size=128, repacked=rep)
    ref = _torch_exact(xq_d, wq_d, _t(s_a, dev), _t(s_w, dev), _t(bias, dev), 128)
    err = _max_rel_t(out, ref)
    assert err <= 3e-2 and err <= 5e-3, err

    # 3. CPU oracle on rows / columns that touch every tile
    rows, cols = _sample(M, 64, rng), _sample(N, 128, rng)
    r, c = _oracle_rows_cols(xq, wq, s_a, s_w, bias, 128, rows, cols)
    o = out.float().cpu().numpy()
    assert O.max_rel(o[rows], r) <= 5e-3
    assert O.max_rel(o[:, cols], c) <= 5e-3


@pytest.mark.parametrize("M,N,K", [(4096, 12288, 3072), (256, 3072, 3072)])
def test_w8a8_baseline_shapes(M, N, K):
    """W8A8 per channel at the config-2 GEMM shape and at configs[0]
    (256 x 3072 x 3072, the split-K route)."""
    dev = _dev()
    rng = np.random.default_rng(M + N)
    # |x| <= 16 keeps the unit-scale accumulators below 2^24 (exact in fp32)
    xs = rng.integers(-16, 17, (M, K), dtype=np.int64).astype(np.int8)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    xs_d, wq_d = _t(xs, dev), _t(wq, dev)
    ones = rt.gemm_a8(xs_d, wq_d, torch.ones(N, device=dev), torch.ones(M, device=dev), out_dtype=torch.float32)
    assert torch.equal(ones.to(torch.int64), torch._int_mm(xs_d, wq_d.t().contiguous()).to(torch.int64))

    xq = rng.integers(-128, 128, (M, K), dtype=np.int64).astype(np.int8)
    xq_d = _t(xq, dev)
    s_w = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    out = rt.gemm_a8(xq_d, wq_d, _t(s_w, dev), _t(s_a, dev), bias=_t(bias, dev), out_dtype=torch.float16)
    ref = _torch_exact(xq_d, wq_d, _t(s_a, dev), _t(s_w, dev), _t(bias, dev), K)
    assert _max_rel_t(out, ref) <= 5e-3
    rows, cols = _sample(M, 64, rng), _sample(N, 128, rng)
    r, c = _oracle_rows_cols(xq, wq, s_a, s_w, bias, None, rows, cols)
    o = out.float().cpu().numpy()
    assert O.max_rel(o[rows], r) <= 5e-3
    assert O.max_rel(o[:, cols], c) <= 5e-3


def _x_outliers(M, K, rng):
    x = rng.standard_normal((M, K)).astype(np.float32)
    ch = rng.permutation(K)[: round(0.01 * K)]
    x[:, ch] *= 20
    return x.astype(np.float16)


def test_config1_prep_and_gemm():
    """configs[0] end to end on the kernels: rot 256 prep + quantise, then
    the W8A8 GEMM with fp16 per-channel scales and bias."""
    dev = _dev()
    M, K, N = 256, 3072, 3072
    rng = np.random.default_rng(0)
    x = _x_outliers(M, K, rng)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    s_w = rng.uniform(1e-3, 1e-2, N).astype(np.float16)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    xq, s_a, _, _ = rt.prep_quantize(_t(x, dev), rot_size=256)
    out = rt.gemm_a8(xq, _t(wq, dev), _t(s_w.astype(np.float32), dev), s_a, bias=_t(bias, dev),
                     out_dtype=torch.float16)
    ref_x = O.prep_activation(x, rot_need=True, rot_size=256, w_in=K)
    q_ref, s_ref = O.quantize_rows(ref_x)
    assert np.array_equal(xq.cpu().numpy(), q_ref)
    assert np.array_equal(s_a.cpu().numpy(), s_ref)
    ref = O.gemm_a8(q_ref, s_ref, wq, s_w.astype(np.float32), bias=bias)
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 5e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_config2_layer_forward(dtype):
    """configs[1] through the drop-in layer (``IntCrushOps.Linear.forward``):
    INT4 W4A8, group 128, SmoothRot, rot 256, PermuQuant, bias, 4096 tokens;
    against the oracle's prep -> quantise -> group GEMM on the same inputs."""
    dev = _dev()
    comfy_stub.install()
    ql = load("quant_layout")
    ql.register_intcrush_layouts()
    ops = load("_ops")
    M, N, K, G = CONFIG2["M"], CONFIG2["N"], CONFIG2["K"], CONFIG2["G"]
    rng = np.random.default_rng(1)
    x = _x_outliers(M, K, rng)
    sr = rng.uniform(0.5, 4.0, K).astype(np.float16)
    perm = rng.permutation(K).astype(np.int64)
    wq = rng.integers(-8, 8, (N, K), dtype=np.int64).astype(np.int8)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float16)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    name = "blocks.0.mlp.fc1"
    Ops = ops.make_intcrush_ops("int4_crush", 256)
    parent, lin = comfy_stub.make_parent(Ops.Linear, K, N, name=name)
    parent.cuda()
    sd = {"weight": torch.from_numpy(O.pack_int4(wq)), "weight_scale": torch.from_numpy(s_w),
          "weight_perm": torch.from_numpy(perm), "weight_smoothrot_factors": torch.from_numpy(sr),
          "bias": torch.from_numpy(bias)}
    parent.load_state_dict({f"{name}.{k}": v for k, v in sd.items()}, strict=False)
    xt = torch.from_numpy(x).to(dtype)
    y = lin(xt.to(dev))
    assert y.dtype == dtype and y.shape == (M, N)
    act = "f16" if dtype == torch.float16 else "bf16"
    x_in = x if act == "f16" else xt.float().numpy()
    xp = O.prep_activation(x_in, smoothrot=sr.astype(np.float32), rot_need=True, rot_size=256, w_in=K, perm=perm,
                           int8_path=False, act=act)
    q, s = O.quantize_rows(xp)
    rows, cols = _sample(M, 64, rng), _sample(N, 128, rng)
    r, c = _oracle_rows_cols(q, wq, s, s_w.astype(np.float32), bias, 128, rows, cols)
    yo = y.float().cpu().numpy()
    assert O.max_rel(yo[rows], r) <= 3e-2 and O.max_rel(yo[rows], r) <= 5e-3
    assert O.max_rel(yo[:, cols], c) <= 5e-3


@pytest.mark.parametrize("kind", ["w4a8_g128", "w4a8_g128_repacked", "w4a8_per_channel", "w8a8"])
def test_pair_tiles_match_single_cta_tiles(kind):
    """Large GEMMs run on CTA pairs (one 256-row tile per two SMs, tcgen05
    cta_group::2); INTCRUSH_PAIR=0 keeps one CTA per 128-row tile.  The
    integer sums and the fp32 epilogue are the same operations in the same
    order, so the outputs are bit-identical (fresh processes: the switch is
    read once)."""
    import os, subprocess, sys, tempfile
    _dev()
    code = (
        "import sys; sys.path[:0] = %r\n"
        "import conftest, numpy as np, torch, intcrush_oracle as O\n"
        "from _pkg import load\n"
        "rt = load('_b200_runtime')\n"
        "kind = %r\n"
        "M, N, K = 2500, 6400, 3072\n"   # ragged: 2500 = 13 x 192 + 4, 6400 = 25 x 256
        "rng = np.random.default_rng(11)\n"
        "xq = torch.from_numpy(rng.integers(-128, 128, (M, K)).astype(np.int8)).cuda()\n"
        "int4 = kind != 'w8a8'\n"
        "wq = rng.integers(-8, 8, (N, K)) if int4 else rng.integers(-127, 128, (N, K))\n"
        "w = torch.from_numpy(O.pack_int4(wq.astype(np.int8)) if int4 else wq.astype(np.int8)).cuda()\n"
        "G = 24 if kind.startswith('w4a8_g') else 1\n"
        "rep = kind.endswith('repacked')\n"
        "if rep: w = rt.repack_int4(w, K, 0)\n"
        "s_w = torch.from_numpy(rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)).cuda()\n"
        "s_a = torch.from_numpy(rng.uniform(1e-3, 5e-2, M).astype(np.float32)).cuda()\n"
        "b = torch.from_numpy((rng.standard_normal(N) * 0.02).astype(np.float16)).cuda()\n"
        "y = rt.gemm_a8(xq, w, s_w, s_a, bias=b, out_dtype=torch.float16, group_size=128, repacked=rep)\n"
        "torch.cuda.synchronize(); assert rt.device_error() == 0\n"
        "np.save(sys.argv[1], y.cpu().numpy())\n"
    ) % ([os.path.dirname(__file__)], kind)
    outs = []
    for pair in ("1", "0"):
        f = tempfile.mktemp(suffix=".npy")
        env = dict(os.environ, INTCRUSH_PAIR=pair)
        r = subprocess.run([sys.executable, "-c", code, f], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
        os.remove(f)
    assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16))
