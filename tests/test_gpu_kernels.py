"""GPU parity of every C-ABI kernel against the CPU oracle (``oracle/``).

Bars (stated per test): bit-exact for the INT8 activations, scales, prepped
fp16 rows, unpacked weights and integer accumulators; max-rel
``max|y - y_ref| / max|y_ref|`` <= 1e-3 for W4A16 / dequant paths and
<= 3e-2 for the A8 paths (the tolerances of the parity contract).
"""

import numpy as np
import pytest
import torch

import intcrush_oracle as O
from _pkg import load

pytestmark = pytest.mark.gpu

rt = load("_b200_runtime")


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA required")
    return torch.device("cuda")


def _x(M, K, seed, outliers=True, dtype=np.float16):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    if outliers and K >= 10:
        ch = rng.permutation(K)[: max(1, round(0.01 * K))]
        x[:, ch] *= 20
    return x.astype(dtype)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


# ───────────────────────────── a1: prep + quant ─────────────────────────────

PREP_CASES = [
    # M, K, rot, w_in, perm, smoothrot, smooth
    (1, 64, 0, 64, False, False, False),
    (7, 256, 16, 256, False, False, False),
    (16, 1024, 64, 1024, True, False, False),
    (129, 3072, 256, 3072, True, True, False),
    (33, 3000, 256, 3072, True, False, True),      # K pad to a rot multiple
    (5, 3072, 1024, 3072, False, True, False),
    (4, 3072, 4096, 4096, True, False, False),     # K=3072 padded to 4096
    (9, 5120, 1024, 5120, False, False, True),
    (3, 13824, 1024, 14336, True, False, False),  # 13824 pads to 14336
    (6, 96, 32, 96, False, False, False),          # Sylvester size
    (6, 512, 128, 512, True, True, False),         # Sylvester size
    (2, 100, 0, 112, True, False, True),           # no rotation, pad to w_in
    (2500, 3072, 256, 3072, True, True, False),    # more rows than resident warps
    (5, 1000, 16, 1010, True, False, True),        # ragged K and w_in (scalar gather)
    (3, 9000, 64, 9024, True, True, False),        # long row in the per-warp buffer
    (600, 12288, 256, 12288, True, True, False),   # many wide rows (row kernel route)
]


@pytest.mark.parametrize("M,K,rot,w_in,use_perm,use_sr,use_sm", PREP_CASES)
def test_prep_quant_bit_exact(M, K, rot, w_in, use_perm, use_sr, use_sm):
    dev = _dev()
    x = _x(M, K, seed=M * 7 + K)
    rng = np.random.default_rng(1)
    perm = rng.permutation(w_in).astype(np.int64) if use_perm else None
    sr = rng.uniform(0.5, 4.0, K).astype(np.float32) if use_sr else None
    sm = rng.uniform(0.5, 2.0, w_in).astype(np.float32) if use_sm else None
    ref = O.prep_activation(x, smoothrot=sr, rot_need=rot > 0, rot_size=rot, w_in=w_in, perm=perm,
                            smooth=sm, int8_path=True)
    q_ref, s_ref = O.quantize_rows(ref)
    xq, s_a, xp, rs = rt.prep_quantize(
        _t(x, dev), smoothrot=None if sr is None else _t(sr, dev), rot_size=rot, w_in=w_in,
        perm=None if perm is None else _t(perm, dev), smooth=None if sm is None else _t(sm, dev),
        want_prep=True, want_rowsum=True)
    torch.cuda.synchronize()
    assert np.array_equal(xp.cpu().numpy().view(np.uint16), ref.view(np.uint16)), "prepped fp16 row differs"
    assert np.array_equal(s_a.cpu().numpy(), s_ref), "scales differ"
    assert np.array_equal(xq.cpu().numpy(), q_ref), "int8 activations differ"
    np.testing.assert_allclose(rs.cpu().numpy(), ref.astype(np.float64).sum(1), rtol=1e-3, atol=1e-2)
    # quantised output alone: the 4-row tile kernel's route where it applies
    xq2, s_a2, _, _ = rt.prep_quantize(
        _t(x, dev), smoothrot=None if sr is None else _t(sr, dev), rot_size=rot, w_in=w_in,
        perm=None if perm is None else _t(perm, dev), smooth=None if sm is None else _t(sm, dev))
    assert np.array_equal(s_a2.cpu().numpy(), s_ref), "scales differ (quantised output only)"
    assert np.array_equal(xq2.cpu().numpy(), q_ref), "int8 activations differ (quantised output only)"


def test_prep_both_kernels_bit_identical():
    """Few rows take prep_row_kernel, many rows prep_quant_kernel; with
    INTCRUSH_PREP_V1=1 every request takes prep_quant_kernel.  Both give the
    same bits (fresh processes, the switch is read once)."""
    import subprocess, sys, os
    _dev()
    code = (
        "import sys; sys.path[:0] = %r\n"
        "import conftest, numpy as np, torch, intcrush_oracle as O\n"
        "from _pkg import load\n"
        "rt = load('_b200_runtime')\n"
        "rng = np.random.default_rng(3)\n"
        "x = torch.from_numpy((rng.standard_normal((100, 3000)) * 3).astype(np.float16)).cuda()\n"
        "sr = torch.from_numpy(rng.uniform(0.5, 4, 3000).astype(np.float32)).cuda()\n"
        "perm = torch.from_numpy(rng.permutation(3072).astype(np.int32)).cuda()\n"
        "q, s, xp, rs = rt.prep_quantize(x, smoothrot=sr, rot_size=256, w_in=3072, perm=perm, want_prep=True)\n"
        "np.save(sys.argv[1], np.concatenate([q.cpu().numpy().view(np.uint8).ravel(), s.cpu().numpy().view(np.uint8),"
        " xp.cpu().numpy().view(np.uint8).ravel()]))\n"
    ) % ([os.path.dirname(__file__)],)
    import tempfile
    outs = []
    for v1 in ("0", "1"):
        f = tempfile.mktemp(suffix=".npy")
        env = dict(os.environ, INTCRUSH_PREP_V1=v1)
        r = subprocess.run([sys.executable, "-c", code, f], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
        os.remove(f)
    assert np.array_equal(outs[0], outs[1])


def _int8_close(q, q_ref):
    """int8 within +-1 everywhere and identical in >= 99.5% of entries: the
    normalisation's fp32 statistics are summed in a different order than the
    reference's, which moves a value across an fp16 or int8 rounding boundary
    now and then (the reference's own CUDA test allows +-1)."""
    d = np.abs(q.astype(np.int16) - q_ref.astype(np.int16))
    assert d.max() <= 1, d.max()
    assert (d == 0).mean() >= 0.995, (d == 0).mean()


@pytest.mark.parametrize("kind", ["layer", "rms"])
@pytest.mark.parametrize("M,K", [(1, 64), (4, 256), (16, 1024), (64, 4096), (700, 3072)])
def test_fused_norm_quantize_matches_cpu_form(kind, M, K):
    """fused_layernorm_quantize / fused_rmsnorm_quantize (the reference's API,
    kernels/triton_quantize.py:274-451) against their CPU form."""
    dev = _dev()
    rng = np.random.default_rng(M + K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    gamma = rng.standard_normal(K).astype(np.float32)
    beta = rng.standard_normal(K).astype(np.float32)
    if kind == "layer":
        q, s = rt.fused_layernorm_quantize(_t(x, dev), _t(gamma, dev), _t(beta, dev))
        ref = O.layer_norm_rows(x, gamma, beta)
    else:
        q, s = rt.fused_rmsnorm_quantize(_t(x, dev), _t(gamma, dev))
        ref = O.rms_norm_rows(x, gamma)
    q_ref, s_ref = O.quantize_rows(ref)
    _int8_close(q.cpu().numpy(), q_ref)
    np.testing.assert_allclose(s.cpu().numpy(), s_ref, rtol=2e-3)


def test_fused_norm_prep_with_rotation_and_perm():
    """LayerNorm with per-sample affine (adaLN modulation) fused ahead of the
    layer's SmoothRot + rot 256 + PermuQuant prep."""
    dev = _dev()
    M, K = 300, 3072
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((M, K)) * 2).astype(np.float16)
    gamma = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(K)).astype(np.float32)
    sr = rng.uniform(0.5, 4.0, K).astype(np.float32)
    perm = rng.permutation(K).astype(np.int32)
    q, s, xp, _ = rt.prep_quantize(_t(x, dev), smoothrot=_t(sr, dev), rot_size=256, w_in=K, perm=_t(perm, dev),
                                   norm=("layer", _t(gamma, dev), _t(beta, dev), 1e-6), want_prep=True)
    xn = O.layer_norm_rows(x, gamma, beta, eps=1e-6)
    ref = O.prep_activation(xn, smoothrot=sr, rot_need=True, rot_size=256, w_in=K, perm=perm)
    q_ref, s_ref = O.quantize_rows(ref)
    _int8_close(q.cpu().numpy(), q_ref)
    np.testing.assert_allclose(s.cpu().numpy(), s_ref, rtol=2e-3)
    d = np.abs(xp.float().cpu().numpy() - ref.astype(np.float32))
    assert d.max() <= 2e-2 * np.abs(ref.astype(np.float32)).max()


def test_fused_norm_zero_row_is_finite():
    dev = _dev()
    x = torch.zeros(2, 64, dtype=torch.float16, device=dev)
    q, s = rt.fused_layernorm_quantize(x, torch.ones(64, device=dev), torch.zeros(64, device=dev))
    assert torch.isfinite(s).all() and (q == 0).all()


def test_prep_bf16_runs_and_matches_fp16_semantics():
    dev = _dev()
    x = torch.randn(8, 256, device=dev, dtype=torch.bfloat16)
    xq, s_a, xp, _ = rt.prep_quantize(x, rot_size=64, want_prep=True)
    H = torch.from_numpy(O.hadamard(64)).to(dev)
    ref = (x.double().reshape(8, 4, 64) @ H.T).reshape(8, 256).to(torch.bfloat16)
    assert torch.equal(xp, ref)


def test_dynamic_quantize_matches_reference_cpu_formula():
    """Mirror of the reference's ``test_cpu_fallback`` cases, on the GPU."""
    dev = _dev()
    for M, K in [(1, 64), (4, 256), (16, 1024), (256, 4096)]:
        torch.manual_seed(0)
        x = torch.randn(M, K).half()
        q, s = rt.dynamic_quantize_activation(x.to(dev))
        ref_s = x.float().abs().amax(dim=1).clamp(min=1e-8) / 127.0
        ref_q = (x.float() / ref_s.unsqueeze(1)).round().clamp(-128, 127).to(torch.int8)
        assert torch.equal(q.cpu(), ref_q)
        assert torch.equal(s.cpu(), ref_s)


def test_dynamic_quantize_3d_and_zero_rows():
    dev = _dev()
    x = torch.zeros(2, 3, 128, dtype=torch.float16, device=dev)
    x[1, 2, 5] = 3.0
    q, s = rt.dynamic_quantize_activation(x)
    assert q.shape == (2, 3, 128) and s.shape == (2, 3)
    assert int(q.abs().sum()) == 127
    assert torch.all(s[0] == torch.tensor(1e-8, dtype=torch.float32) / 127.0)


# ───────────────────────────── a2/a3: A8 GEMMs ──────────────────────────────

def _int_inputs(M, N, K, seed, int4):
    rng = np.random.default_rng(seed)
    xq = rng.integers(-128, 128, (M, K), dtype=np.int64).astype(np.int8)
    if int4:
        wq = rng.integers(-8, 8, (N, K), dtype=np.int64).astype(np.int8)
    else:
        wq = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    return xq, wq


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("G", [1, 4])
@pytest.mark.parametrize("M,N,K", [(1, 128, 512), (37, 200, 512), (130, 384, 1024), (300, 256, 512)])
def test_gemm_a8_integer_accumulators_exact(int4, G, M, N, K):
    """With unit scales the output is the int32 accumulator (sum over groups):
    exact in fp32 below 2^24."""
    dev = _dev()
    if G > 1 and not int4 and K // G != 128:
        G = K // 128
    xq, wq = _int_inputs(M, N, K, seed=M + N + K, int4=int4)
    w = O.pack_int4(wq) if int4 else wq
    s_w = np.ones((N, G), np.float32)
    s_a = np.ones(M, np.float32)
    out = rt.gemm_a8(_t(xq, dev), _t(w, dev), _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32,
                     group_size=K // G)
    ref = O.int_accumulators(xq, wq)[0]
    assert np.array_equal(out.cpu().numpy().astype(np.int64), ref)


@pytest.mark.parametrize("int4,G", [(False, 1), (True, 1), (True, 24), (False, 24)])
@pytest.mark.parametrize("M", [1, 16, 64, 129, 256, 520])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_gemm_a8_dequant_parity(int4, G, M, out_dtype):
    dev = _dev()
    N, K = 384, 3072
    xq, wq = _int_inputs(M, N, K, seed=M, int4=int4)
    rng = np.random.default_rng(M + 1)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    w = O.pack_int4(wq) if int4 else wq
    out = rt.gemm_a8(_t(xq, dev), _t(w, dev), _t(s_w, dev), _t(s_a, dev), bias=_t(bias, dev),
                     out_dtype=out_dtype, group_size=K // G)
    ref = O.gemm_a8(xq, s_a, wq, s_w if G > 1 else s_w[:, 0], bias=bias, group_size=K // G)
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 3e-2
    # fp32 accumulation makes it far tighter than the contract
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 5e-3


def test_gemm_a8_zero_point_term():
    dev = _dev()
    M, N, K = 40, 256, 512
    xq, wq = _int_inputs(M, N, K, seed=3, int4=False)
    rng = np.random.default_rng(4)
    s_w = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    rowsum = rng.standard_normal(M).astype(np.float32)
    zpc = rng.standard_normal(N).astype(np.float32) * 0.01
    out = rt.gemm_a8(_t(xq, dev), _t(wq, dev), _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32,
                     rowsum=_t(rowsum, dev), zp_corr=_t(zpc, dev))
    ref = O.gemm_a8(xq, s_a, wq, s_w) - rowsum[:, None].astype(np.float64) * zpc[None, :]
    assert O.max_rel(out.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("int4,G", [(False, 1), (True, 1), (True, 24), (False, 24)])
@pytest.mark.parametrize("splits", [2, 3, 4, 6])
@pytest.mark.parametrize("M", [1, 40, 256])
def test_gemm_a8_splitk_matches_oracle(int4, G, splits, M):
    """Split-K (fp32 partials in a workspace + reduce) against the oracle, with
    bias and the zero-point term; unit scales give the exact integer sums."""
    dev = _dev()
    N, K = 320, 3072
    xq, wq = _int_inputs(M, N, K, seed=M + splits, int4=int4)
    w = _t(O.pack_int4(wq) if int4 else wq, dev)
    ones = rt.gemm_a8(_t(xq, dev), w, torch.ones(N, G, device=dev), torch.ones(M, device=dev),
                      out_dtype=torch.float32, group_size=K // G, splits=splits)
    assert np.array_equal(ones.cpu().numpy().astype(np.int64), O.int_accumulators(xq, wq)[0])
    rng = np.random.default_rng(splits)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.02).astype(np.float16)
    rowsum = rng.standard_normal(M).astype(np.float32)
    zpc = (rng.standard_normal(N) * 0.01).astype(np.float32)
    out = rt.gemm_a8(_t(xq, dev), w, _t(s_w, dev), _t(s_a, dev), bias=_t(bias, dev), out_dtype=torch.float32,
                     group_size=K // G, rowsum=_t(rowsum, dev), zp_corr=_t(zpc, dev), splits=splits)
    ref = O.gemm_a8(xq, s_a, wq, s_w if G > 1 else s_w[:, 0], bias=bias, group_size=K // G)
    ref = ref - rowsum[:, None].astype(np.float64) * zpc[None, :]
    assert O.max_rel(out.cpu().numpy(), ref) <= 1e-5
    one = rt.gemm_a8(_t(xq, dev), w, _t(s_w, dev), _t(s_a, dev), bias=_t(bias, dev), out_dtype=torch.float32,
                     group_size=K // G, rowsum=_t(rowsum, dev), zp_corr=_t(zpc, dev), splits=1)
    assert O.max_rel(out.cpu().numpy(), one.cpu().numpy().astype(np.float64)) <= 1e-6


def test_gemm_a8_splitk_rejects_bad_splits():
    dev = _dev()
    M, N, K = 8, 128, 640       # 5 K blocks
    xq, wq = _int_inputs(M, N, K, seed=1, int4=False)
    with pytest.raises(Exception):
        rt.gemm_a8(_t(xq, dev), _t(wq, dev), torch.ones(N, device=dev), torch.ones(M, device=dev),
                   out_dtype=torch.float32, splits=2)


@pytest.mark.parametrize("G", [1, 24])
@pytest.mark.parametrize("M", [1, 64, 300])
def test_gemm_a8_repacked_int4_bit_identical(G, M):
    """The load-time repacked layout gives the same output bits as the reference packing."""
    dev = _dev()
    N, K = 256, 3072
    xq, wq = _int_inputs(M, N, K, seed=M + G, int4=True)
    rng = np.random.default_rng(7)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    packed = _t(O.pack_int4(wq), dev)
    rep = rt.repack_int4(packed, K, 0)
    a = rt.gemm_a8(_t(xq, dev), packed, _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32, group_size=K // G)
    b = rt.gemm_a8(_t(xq, dev), rep, _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32, group_size=K // G,
                   repacked=True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M", [1, 16, 33, 256])
def test_w4a16_repacked_bit_identical(M):
    dev = _dev()
    N, K = 512, 3072
    rng = np.random.default_rng(M)
    x = _t(rng.standard_normal((M, K)).astype(np.float16), dev)
    packed = _t(O.pack_int4(rng.integers(-8, 8, (N, K)).astype(np.int8)), dev)
    scale = _t(rng.uniform(1e-3, 2e-2, (N, 24)).astype(np.float16), dev)
    a = rt.gemm_w4a16(x, packed, scale, group_size=128)
    b = rt.gemm_w4a16(x, rt.repack_int4(packed, K, 1), scale, group_size=128, w_layout=1)
    assert torch.equal(a, b)


@pytest.mark.parametrize("bn", [32, 64, 128, 160, 192, 256])
def test_gemm_a8_grouped_every_tile_width(bn, monkeypatch):
    """Each token-tile width of the group-scale kernel, in a fresh process."""
    import subprocess, sys, os
    dev = _dev()
    code = (
        "import sys; sys.path[:0] = %r\n"
        "import conftest, numpy as np, torch, intcrush_oracle as O\n"
        "from _pkg import load\n"
        "rt = load('_b200_runtime')\n"
        "rng = np.random.default_rng(5); M, N, K = 300, 256, 1024\n"
        "xq = rng.integers(-128, 128, (M, K)).astype(np.int8); wq = rng.integers(-8, 8, (N, K)).astype(np.int8)\n"
        "s_w = rng.uniform(1e-3, 2e-2, (N, 8)).astype(np.float32); s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)\n"
        "t = lambda a: torch.from_numpy(a).cuda()\n"
        "out = rt.gemm_a8(t(xq), rt.repack_int4(t(O.pack_int4(wq)), K, 0), t(s_w), t(s_a), out_dtype=torch.float32, group_size=128, repacked=True)\n"
        "err = O.max_rel(out.cpu().numpy(), O.gemm_a8(xq, s_a, wq, s_w, group_size=128))\n"
        "assert err <= 1e-5, err\n"
    ) % ([os.path.dirname(__file__)],)
    env = dict(os.environ, INTCRUSH_FORCE_BN=str(bn))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,ld_pad", [(1, 200, 0), (100, 384, 8), (300, 1000, 0), (777, 200, 3),
                                        (2500, 4000, 0)])
def test_gemm_a8_grouped_tma_store_matches_plain_store(out_dtype, M, N, ld_pad):
    """Group-scaled tiles with a 16-bit output write through shared memory
    and TMA bulk-tensor stores (clipped at the M / N edges; an output row
    stride that is not a multiple of 16 bytes falls back to plain stores).
    Both must give the bits of the fp32 epilogue value rounded once."""
    dev = _dev()
    K, G = 1024, 8
    xq, wq = _int_inputs(M, N, K, seed=M + N, int4=True)
    rng = np.random.default_rng(N)
    s_w = _t(rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32), dev)
    s_a = _t(rng.uniform(1e-3, 5e-2, M).astype(np.float32), dev)
    bias = _t((rng.standard_normal(N) * 0.02).astype(np.float16), dev)
    x, w = _t(xq, dev), _t(O.pack_int4(wq), dev)
    y32 = rt.gemm_a8(x, w, s_w, s_a, bias=bias, out_dtype=torch.float32, group_size=128)
    big = torch.full((M, N + ld_pad), 7.0, dtype=out_dtype, device=dev)
    out = big[:, :N]
    rt.gemm_a8(x, w, s_w, s_a, bias=bias, out_dtype=out_dtype, group_size=128, out=out)
    assert torch.equal(out, y32.to(out_dtype))
    if ld_pad:
        assert torch.all(big[:, N:] == 7.0)   # nothing written past the slice
    ref = O.gemm_a8(xq, s_a.cpu().numpy(), wq, s_w.cpu().numpy(), bias=bias.cpu().numpy(), group_size=128)
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 5e-3


def test_gemm_a8_unpacked_int4_matches_packed():
    dev = _dev()
    M, N, K = 64, 256, 1024
    xq, wq = _int_inputs(M, N, K, seed=9, int4=True)
    s_w = np.full((N, 8), 0.01, np.float32)
    s_a = np.full(M, 0.02, np.float32)
    a = rt.gemm_a8(_t(xq, dev), _t(wq, dev), _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32)
    b = rt.gemm_a8(_t(xq, dev), _t(O.pack_int4(wq), dev), _t(s_w, dev), _t(s_a, dev), out_dtype=torch.float32)
    assert torch.equal(a, b)


# ───────────────────────────── a4: W4A16 ────────────────────────────────────

@pytest.mark.parametrize("M", [1, 5, 16, 32, 33, 64, 256])
@pytest.mark.parametrize("G", [1, 24])
def test_w4a16_parity(M, G):
    dev = _dev()
    N, K = 3072, 3072
    rng = np.random.default_rng(M * 3 + G)
    x = (rng.standard_normal((M, K))).astype(np.float16)
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    packed = O.pack_int4(q)
    scale = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float16)
    out = rt.gemm_w4a16(_t(x, dev), _t(packed, dev), _t(scale, dev), group_size=K // G)
    w16 = O.dequant_int4_f16(packed, scale, K, K // G)
    ref = O.linear_f16(x, w16)
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,splits", [(129, 3072, None), (256, 3072, None), (256, 3072, 3), (300, 200, 4),
                                        (512, 1024, 2), (4096, 384, None)])
def test_w4a16_splitk_matches_unsplit_and_oracle(dtype, M, N, splits):
    """The tcgen05 W4A16 path with K cut into parts (fp32 partials + reduce)
    against the unsplit kernel and the dequant-linear oracle (1e-3 for fp16;
    bf16 at two bf16 ulps)."""
    dev = _dev()
    K = 3072
    rng = np.random.default_rng(M + N)
    x = rng.standard_normal((M, K)).astype(np.float16)
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    packed = O.pack_int4(q)
    scale = rng.uniform(1e-3, 2e-2, (N, 24)).astype(np.float16)
    xt = _t(x, dev).to(dtype)
    bias = _t((rng.standard_normal(N) * 0.02).astype(np.float16), dev).to(dtype)
    got = rt.gemm_w4a16(xt, _t(packed, dev), _t(scale, dev), group_size=128, bias=bias, splits=splits)
    one = rt.gemm_w4a16(xt, _t(packed, dev), _t(scale, dev), group_size=128, bias=bias, splits=1)
    tol = 1e-3 if dtype == torch.float16 else 2 * 2.0 ** -8
    assert O.max_rel(got.float().cpu().numpy(), one.float().cpu().numpy()) <= tol
    if dtype == torch.float16:
        w16 = O.dequant_int4_f16(packed, scale, K, 128)
        ref_o = O.linear_f16(x, w16) + bias.float().cpu().numpy()
        assert O.max_rel(got.float().cpu().numpy(), ref_o) <= 1e-3


def test_w4a16_splitk_rejects_bad_splits():
    dev = _dev()
    x = torch.zeros(256, 3072, dtype=torch.float16, device=dev)
    packed = torch.zeros(512, 1536, dtype=torch.uint8, device=dev)
    scale = torch.ones(512, 24, dtype=torch.float16, device=dev)
    with pytest.raises(Exception):
        rt.gemm_w4a16(x, packed, scale, group_size=128, splits=5)   # 48 K blocks: not a multiple of 5
    with pytest.raises(Exception):
        rt.gemm_w4a16(x, packed, scale, group_size=128, splits=9)


@pytest.mark.parametrize("M", [1, 16, 256])
def test_w4a16_with_lora_parity(M):
    dev = _dev()
    N, K, R = 3072, 3072, 32
    rng = np.random.default_rng(M)
    x = rng.standard_normal((M, K)).astype(np.float16)
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    packed = O.pack_int4(q)
    scale = rng.uniform(1e-3, 2e-2, (N, 24)).astype(np.float16)
    A = (rng.standard_normal((R, K)) * 0.01).astype(np.float16)
    B = (rng.standard_normal((N, R)) * 0.01).astype(np.float16)
    mid = rt.lowrank_down(_t(x, dev), _t(A, dev))
    assert np.array_equal(mid.cpu().numpy(), O.lora_mid(x, A)) or \
        np.abs(mid.float().cpu().numpy() - O.lora_mid(x, A).astype(np.float32)).max() <= 2e-3
    out = rt.gemm_w4a16(_t(x, dev), _t(packed, dev), _t(scale, dev), group_size=128,
                        lr_mid=mid, lr_up=_t(B, dev), lr_scale=1.0)
    ref = O.linear_f16(x, O.dequant_int4_f16(packed, scale, K, 128)) + O.lora_residual(x, A, B, 1.0)
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 1e-3


def test_unpack_kernels_bit_exact():
    dev = _dev()
    rng = np.random.default_rng(0)
    q = rng.integers(-8, 8, (16, 256)).astype(np.int8)
    packed = O.pack_int4(q)
    got = rt.unpack_int4_to_int8(_t(packed, dev), 256)
    assert np.array_equal(got.cpu().numpy(), q)
    scale = rng.uniform(1e-3, 2e-2, (16, 2)).astype(np.float16)
    w16 = rt.unpack_int4_to_float16(_t(packed, dev), _t(scale, dev), 256, group_size=128)
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), O.dequant_int4_f16(packed, scale, 256, 128).view(np.uint16))


def test_no_device_timeouts_recorded():
    _dev()
    assert rt.device_error(clear=True) == 0


@pytest.mark.parametrize("M,K,rot,w_in,perm,sr,sm,dt", [
    (4096, 3072, 256, 3072, True, True, False, "f16"),
    (37, 3000, 256, 3072, True, False, True, "f16"),
    (100, 1000, 16, 1010, True, False, True, "bf16"),
    (9, 4096, 64, 4096, False, True, False, "bf16"),
    (513, 2048, 128, 2048, True, True, False, "f16"),
    (70, 96, 32, 100, True, False, False, "f16"),
    (1, 64, 0, 80, True, False, True, "f16"),
    (2050, 1536, 0, 1536, False, False, False, "bf16"),
])
def test_prep_tile_kernel_matches_previous_kernels(M, K, rot, w_in, perm, sr, sm, dt):
    """The 4-row tile kernel (default route for quantised output of rows of
    <= 4096 columns, rotation 0 or 16..256) against the earlier per-row
    kernels (INTCRUSH_PREP_TILE=0): same int8 values and scales, bit for bit
    (fresh processes, the switch is read once)."""
    import subprocess, sys, os, tempfile
    _dev()
    code = (
        "import sys; sys.path[:0] = %r\n"
        "import conftest, numpy as np, torch\n"
        "from _pkg import load\n"
        "rt = load('_b200_runtime')\n"
        "M, K, rot, w_in, perm, sr, sm, dt = %r\n"
        "rng = np.random.default_rng(M + K)\n"
        "x = torch.from_numpy((rng.standard_normal((M, K)) * 3).astype(np.float32))\n"
        "x = x.to(torch.float16 if dt == 'f16' else torch.bfloat16).cuda()\n"
        "P = torch.from_numpy(rng.permutation(w_in).astype(np.int32)).cuda() if perm else None\n"
        "S = torch.from_numpy(rng.uniform(0.5, 4, K).astype(np.float32)).cuda() if sr else None\n"
        "Q = torch.from_numpy(rng.uniform(0.5, 2, w_in).astype(np.float32)).cuda() if sm else None\n"
        "q, s, _, _ = rt.prep_quantize(x, smoothrot=S, rot_size=rot, w_in=w_in, perm=P, smooth=Q)\n"
        "np.save(sys.argv[1], np.concatenate([q.cpu().numpy().view(np.uint8).ravel(), s.cpu().numpy().view(np.uint8)]))\n"
    ) % ([os.path.dirname(__file__)], (M, K, rot, w_in, perm, sr, sm, dt))
    outs = []
    for tile in ("1", "0"):
        f = tempfile.mktemp(suffix=".npy")
        env = dict(os.environ, INTCRUSH_PREP_TILE=tile)
        r = subprocess.run([sys.executable, "-c", code, f], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(np.load(f))
        os.remove(f)
    assert np.array_equal(outs[0], outs[1])


# ───────────────────────── bf16 W4A16 and low-rank ──────────────────────────

def _bf16_t(a, dev):
    """float32 numpy holding bf16 values -> bf16 CUDA tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).to(dev)


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("G", [1, 24])
@pytest.mark.parametrize("M", [1, 16, 100, 129, 256])
def test_w4a16_bf16_parity(M, G, layout):
    """bf16 activations: W = bf16(q * s) from the fp32 product (the reference's
    PyTorch path, quant_layout.py:81-87 then .to(x.dtype)), bf16 GEMM with
    fp32 accumulation, bf16 output.  Bar: max-rel 4e-3, the size of one bf16
    rounding of the output (2^-9 relative) with margin; the W4A16 contract's
    1e-3 is below bf16's own output resolution."""
    dev = _dev()
    N, K = 1024, 3072
    rng = np.random.default_rng(M * 5 + G)
    x = O.bf16(rng.standard_normal((M, K)))
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    packed = _t(O.pack_int4(q), dev)
    scale = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float16)
    w = packed if layout == 0 else rt.repack_int4(packed, K, 1)
    out = rt.gemm_w4a16(_bf16_t(x, dev), w, _t(scale, dev), group_size=K // G, w_layout=layout)
    assert out.dtype == torch.bfloat16
    wb = O.bf16(q.astype(np.float64) * np.repeat(scale.astype(np.float64), K // G, axis=1))
    ref = x.astype(np.float64) @ wb.astype(np.float64).T
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 4e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("R", [16, 64, 128, 256])
def test_lowrank_kernels_any_rank_and_dtype(dtype, R):
    """mid = T(x @ down^T), out = T(out + s * mid @ up^T) for ranks up to 256
    in fp16 and bf16 (the reference's F.linear + addmm_, _ops.py:242-243)."""
    dev = _dev()
    M, K, N = 40, 1536, 700
    g = torch.Generator().manual_seed(R)
    x = torch.randn(M, K, generator=g).to(dtype)
    down = (torch.randn(R, K, generator=g) * 0.02).to(dtype)
    up = (torch.randn(N, R, generator=g) * 0.02).to(dtype)
    base = torch.randn(M, N, generator=g).to(dtype)
    mid = rt.lowrank_down(x.to(dev), down.to(dev))
    ref_mid = (x.double() @ down.double().T)
    assert mid.dtype == dtype
    tol = 2e-3 if dtype == torch.float16 else 8e-3
    assert float((mid.cpu().double() - ref_mid).abs().max() / ref_mid.abs().max()) <= tol
    out = base.to(dev).clone()
    rt.lowrank_add(out, mid, up.to(dev), 0.7)
    ref = base.double() + 0.7 * (mid.cpu().double() @ up.double().T)
    assert float((out.cpu().double() - ref).abs().max() / ref.abs().max()) <= tol


def test_w4a16_bf16_with_rank128_lora():
    dev = _dev()
    M, N, K, R = 16, 1024, 3072, 128
    rng = np.random.default_rng(3)
    x = O.bf16(rng.standard_normal((M, K)))
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    scale = rng.uniform(1e-3, 2e-2, (N, 24)).astype(np.float16)
    A = O.bf16(rng.standard_normal((R, K)) * 0.01)
    B = O.bf16(rng.standard_normal((N, R)) * 0.01)
    mid = rt.lowrank_down(_bf16_t(x, dev), _bf16_t(A, dev))
    out = rt.gemm_w4a16(_bf16_t(x, dev), _t(O.pack_int4(q), dev), _t(scale, dev), group_size=128,
                        lr_mid=mid, lr_up=_bf16_t(B, dev), lr_scale=1.0)
    wb = O.bf16(q.astype(np.float64) * np.repeat(scale.astype(np.float64), 128, axis=1))
    ref = x.astype(np.float64) @ wb.T.astype(np.float64) + (x.astype(np.float64) @ A.T.astype(np.float64)) @ B.T
    # the reference's double rounding (bf16 GEMM output, then bf16 of the sum)
    # plus the bf16 rank-128 intermediate: within 2 bf16 ulps (2^-7) of max|y|
    assert O.max_rel(out.float().cpu().numpy(), ref) <= 2 ** -7


def test_bounded_wait_runs_out_and_reports_timeout():
    """A device-side wait that nothing completes gives up after its limit
    (1 ms here), records IC_DEV_ERR_TIMEOUT for the host and returns; the
    context stays usable for the next launch."""
    _dev()
    L = load("_lib")
    assert rt.device_error(clear=True) == 0
    st = __import__("ctypes").c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.lib().ic_selftest_wait_timeout(1_000_000, st) == L.IC_OK
    torch.cuda.synchronize()
    assert rt.device_error(clear=True) == L.IC_DEV_ERR_TIMEOUT
    assert rt.device_error(clear=True) == 0            # cleared
    x = torch.randn(8, 256, device="cuda").half()      # the context still works
    q, s = rt.dynamic_quantize_activation(x)
    assert q.shape == (8, 256) and torch.isfinite(s).all()


# ─────────────── f2: epilogue activation / residual, INT8-out ───────────────

def _torch_act(y, act):
    if act == 1:
        return torch.nn.functional.silu(y)
    if act == 2:
        return torch.nn.functional.gelu(y)
    if act == 3:
        return torch.nn.functional.gelu(y, approximate="tanh")
    return y


@pytest.mark.parametrize("act", [0, 1, 2, 3])
@pytest.mark.parametrize("int4,G", [(False, 1), (True, 24)])
@pytest.mark.parametrize("M,splits", [(16, 1), (40, 3), (256, 1), (300, 1), (4096, 1)])
def test_gemm_epilogue_activation_and_residual(act, int4, G, M, splits):
    """act(GEMM + bias) + residual in the epilogue equals the same GEMM's
    fp32 output passed through torch's fp32 SiLU / GELU and the residual add
    (max-abs <= 2e-6 * max|y| + 1e-6: libm-level differences of
    expf / erff / tanhf only); the fp16 output is the rounding of that."""
    dev = _dev()
    N, K = (3072 if M >= 4096 else 384), 3072   # the full-size case runs the CTA-pair tiles
    xq, wq = _int_inputs(M, N, K, seed=M + act, int4=int4)
    rng = np.random.default_rng(M + 7)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = _t((rng.standard_normal(N) * 0.02).astype(np.float16), dev)
    res = _t(rng.standard_normal((M, N)).astype(np.float16), dev)
    w = _t(O.pack_int4(wq) if int4 else wq, dev)
    args = (_t(xq, dev), w, _t(s_w, dev), _t(s_a, dev))
    base = rt.gemm_a8(*args, bias=bias, out_dtype=torch.float32, group_size=K // G, splits=splits)
    ref = _torch_act(base, act) + res.float()
    got = rt.gemm_a8(*args, bias=bias, out_dtype=torch.float32, group_size=K // G, splits=splits,
                     activation=act, residual=res)
    tol = 2e-6 * ref.abs().max().item() + 1e-6
    assert (got - ref).abs().max().item() <= tol
    got16 = rt.fused_int8_gemm_dequant(*args, bias=bias, out_dtype=torch.float16, activation=act, residual=res) \
        if not int4 else rt.gemm_a8(*args, bias=bias, out_dtype=torch.float16, group_size=K // G,
                                    splits=splits, activation=act, residual=res)
    assert (got16.float() - ref).abs().max().item() <= ref.abs().max().item() * 2 ** -10 + tol
    if M >= 4096:
        return   # the full-size GEMM itself is pinned to the oracle in the baseline-shape tests
    # and against the oracle end to end
    full = O.gemm_a8(xq, s_a, wq, s_w if G > 1 else s_w[:, 0], bias=bias.cpu().numpy(), group_size=K // G)
    ref_o = _torch_act(torch.from_numpy(full).float(), act) + res.float().cpu()
    assert O.max_rel(got.cpu().numpy(), ref_o.numpy()) <= 3e-2


@pytest.mark.parametrize("act", [0, 3])
@pytest.mark.parametrize("int4,G", [(False, 1), (True, 24)])
@pytest.mark.parametrize("M", [1, 64, 300, 4096])
def test_int8_gemm_int8out_row_global_scale(act, int4, G, M):
    """(c, s_c) is exactly dynamic quantisation of the GEMM's own fp32
    epilogue values: s_c = max(max|y|, 1e-8) / 127 (bit-exact), c =
    rint(y / s_c) ties to even (bit-exact); then it chains into the next
    GEMM as its activation scale."""
    dev = _dev()
    N, K = (3072 if M >= 4096 else 640), 3072
    xq, wq = _int_inputs(M, N, K, seed=3 * M + act, int4=int4)
    rng = np.random.default_rng(M)
    s_w = rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)
    s_a = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    bias = _t((rng.standard_normal(N) * 0.02).astype(np.float16), dev)
    w = _t(O.pack_int4(wq) if int4 else wq, dev)
    args = (_t(xq, dev), w, _t(s_w, dev), _t(s_a, dev))
    y = rt.gemm_a8(*args, bias=bias, out_dtype=torch.float32, group_size=K // G, splits=1, activation=act)
    c, s_c = rt.int8_gemm_int8out(*args, bias=bias, activation=act, group_size=K // G)
    # a tensor divisor: torch turns division by a Python scalar into a
    # multiplication by its reciprocal, which is not the IEEE quotient
    amax = y.abs().amax(1).clamp(min=1e-8)
    s_ref = amax / torch.full_like(amax, 127.0)
    assert torch.equal(s_c, s_ref)
    c_ref = torch.round(y / s_ref[:, None]).clamp(-128, 127).to(torch.int8)
    assert torch.equal(c, c_ref)
    # chain: the int8 output feeds an INT8 GEMM with s_c as its activation scale
    w2 = torch.randint(-127, 128, (128, N), dtype=torch.int8, device=dev)
    s_w2 = torch.full((128,), 1e-2, device=dev)
    y2 = rt.fused_int8_gemm_dequant(c, w2, s_w2, s_c, out_dtype=torch.float32)
    ref2 = (c.float() * s_c[:, None]) @ (w2.float() * s_w2[:, None]).T
    assert (y2 - ref2).abs().max().item() <= 1e-4 * ref2.abs().max().item() + 1e-6


# ─────────────── f4: device requantisation (set_weight) and LoKr ───────────────

@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("N,K", [(1, 1), (7, 33), (128, 3072), (300, 1001)])
def test_quantize_weight_matches_layout_quantize_bit_exact(bits, N, K):
    """The device kernel equals the layout classes' torch quantize on the
    same fp32 weight (CPU), including a zero row and an odd K."""
    dev = _dev()
    ql = load("quant_layout")
    g = torch.Generator().manual_seed(N * 7 + K)
    w = torch.randn(N, K, generator=g) * torch.rand(N, 1, generator=g) * 0.05
    if N > 2:
        w[1] = 0.0
        w[2, : min(K, 5)] = torch.tensor([1e-3, -7e-3, 0.5e-3, 3.5e-3, -3.5e-3])[: min(K, 5)]
    layout = ql.IntCrushInt4Layout if bits == 4 else ql.IntCrushInt8Layout
    q_ref, p_ref = layout.quantize(w, scale="recalculate")
    q, s = rt.quantize_weight(w.to(dev), bits)
    assert torch.equal(s.cpu(), p_ref.scale.reshape(-1).to(s.dtype))
    nz = p_ref.scale.reshape(-1).float() > 0   # rows whose fp16 scale underflows store 0 here
    assert torch.equal(q.cpu()[nz], q_ref[nz])
    # and the layout class routes a CUDA weight to the kernel
    q2, p2 = layout.quantize(w.to(dev), scale="recalculate")
    assert torch.equal(q2, q) and torch.equal(p2.scale, s)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,out_l,in_m,out_k,in_n", [(1, 4, 4, 32, 64), (37, 16, 16, 192, 192),
                                                     (256, 8, 12, 384, 256), (4096, 16, 16, 192, 192)])
def test_lokr_add_matches_reference_two_matmul_form(dtype, M, out_l, in_m, out_k, in_n):
    """out += scale * (w1 @ X) @ w2_t, the reference's two products, on the
    GPU in torch (cuBLAS, same dtype) vs the kernels: within 2 ulps of the
    dtype relative to max|out|."""
    dev = _dev()
    g = torch.Generator().manual_seed(M + in_n)
    K, N = in_m * in_n, out_l * out_k
    x = torch.randn(M, K, generator=g).to(dtype).to(dev)
    w1 = (torch.randn(out_l, in_m, generator=g) * 0.3).to(dtype).to(dev)
    w2 = (torch.randn(out_k, in_n, generator=g) * 0.05).to(dtype).to(dev)
    base = torch.randn(M, N, generator=g).to(dtype).to(dev)
    ref = base.clone()
    tmp = w1 @ x.reshape(M, in_m, in_n)
    ref.view(M, out_l, out_k).reshape(-1, out_k).addmm_(tmp.reshape(-1, in_n), w2.t(), beta=1.0, alpha=0.7)
    got = rt.lokr_add(base.clone(), x, w1, w2, 0.7)
    ulp = 2 ** -10 if dtype == torch.float16 else 2 ** -7
    assert (got.float() - ref.float()).abs().max().item() <= 2 * ulp * ref.float().abs().max().item()
    assert rt.device_error() == 0
