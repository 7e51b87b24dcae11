"""Multi-rank layouts on CPU: world_size 2 over gloo.

The GEMM itself is CUDA-only, so these tests give ``FeatureShardedLinear``
CPU stand-ins for the prep and GEMM callables (the numpy oracle) and check
the sharding logic: which weight rows each rank keeps, the padding of the
last rank, the all-gather and the column order of the assembled output, and
that the assembled output equals the single-process forward exactly.  The
last test runs the benchmark's DiT block sequence-parallel (one sample split
by image tokens, K/V all-gathered) with CPU stand-ins for the linears and
compares it with the single-process block.
"""

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import intcrush_oracle as O
from _pkg import load

sh = load("_sharded")


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_prep(x, *, smoothrot=None, rot_size=0, w_in=None, perm=None, smooth=None):
    xp = O.prep_activation(x.numpy(), smoothrot=None if smoothrot is None else smoothrot.numpy(),
                           rot_need=rot_size > 0, rot_size=rot_size, w_in=w_in,
                           perm=None if perm is None else perm.numpy(),
                           smooth=None if smooth is None else smooth.numpy())
    q, s = O.quantize_rows(xp)
    return torch.from_numpy(q), torch.from_numpy(s), None, None


def _oracle_gemm(xq, w, s_w, s_a, *, bias=None, out_dtype=torch.float32, group_size=None):
    wq = O.unpack_int4(w.numpy(), xq.shape[1]) if w.dtype == torch.uint8 else w.numpy()
    sw = s_w.numpy()
    y = O.gemm_a8(xq.numpy(), s_a.numpy(), wq, sw if sw.shape[1] > 1 else sw[:, 0],
                  bias=None if bias is None else bias.float().numpy(), group_size=group_size)
    return torch.from_numpy(y.astype(np.float32)).to(out_dtype)


def _case(N, seed=3):
    rng = np.random.default_rng(seed)
    M, K, G = 6, 256, 2
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16))
    q = rng.integers(-8, 8, (N, K)).astype(np.int8)
    w = torch.from_numpy(O.pack_int4(q))
    s_w = torch.from_numpy(rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32))
    bias = torch.from_numpy((rng.standard_normal(N) * 0.02).astype(np.float16))
    sr = torch.from_numpy(rng.uniform(0.5, 4, K).astype(np.float16))
    perm = torch.from_numpy(rng.permutation(K).astype(np.int32))
    return x, w, s_w, bias, sr, perm


def _worker(rank, world, port, N, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, w, s_w, bias, sr, perm = _case(N)
        lin = sh.FeatureShardedLinear(w, s_w, bias, group_size=128, smoothrot=sr, rot_size=64, w_in=256,
                                      perm=perm, prep=_oracle_prep, gemm=_oracle_gemm)
        y = lin(x.to(torch.float32))
        # the chunked form (async all-gather per token chunk) gives the same bits
        x_long = torch.cat([x] * 50).to(torch.float32)          # 300 tokens: 3 chunks of 128 / 44
        y_ov = lin.forward_overlapped(x_long, chunks=3)
        assert torch.equal(y_ov, lin(x_long)), "overlapped form differs"
        out_q.put((rank, lin.weight.shape[0], y.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("N", [256, 200])
def test_feature_sharded_matches_single_process(N):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, w, s_w, bias, sr, perm = _case(N)
    xq, s_a, _, _ = _oracle_prep(x, smoothrot=sr, rot_size=64, w_in=256, perm=perm)
    ref = _oracle_gemm(xq, w, s_w, s_a, bias=bias, out_dtype=torch.float32, group_size=128).numpy()
    for rank, rows, y in res:
        assert rows == -(-N // world)            # padded per-rank width
        assert y.shape == (6, N)
        np.testing.assert_array_equal(y, ref)    # same computation per element


def test_feature_rows_cover_once():
    for N in (1, 7, 128, 12288, 12289):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                a, b, nr = sh.feature_rows(N, r, world)
                assert 0 <= b - a <= nr
                seen.extend(range(a, b))
            assert seen == list(range(N))


def test_shard_tokens_cover_once():
    x = torch.arange(11 * 3).reshape(11, 3)
    parts = [sh.shard_tokens(x, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts), x)


class _TorchLinear:
    """CPU stand-in for the quantised layer of the benchmark's DiT block."""

    def __init__(self, n_out, n_in, g):
        self.w = torch.randn(n_out, n_in, generator=g) / n_in ** 0.5
        self.b = torch.randn(n_out, generator=g) * 0.02

    def __call__(self, x, norm=None):
        if norm is not None:
            _, gamma, beta, eps = norm
            x = torch.nn.functional.layer_norm(x, (x.shape[-1],), eps=eps) * gamma + beta
        return x @ self.w.T + self.b


def _block(sp_group):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    return bench.FluxDoubleBlock(None, torch.device("cpu"), seed=4, hidden=256, heads=2, mlp=512,
                                 sp_group=sp_group, linear=_TorchLinear, dtype=torch.float32)


def _block_inputs():
    g = torch.Generator().manual_seed(8)
    return (torch.randn(1, 64, 256, generator=g), torch.randn(1, 16, 256, generator=g),
            torch.randn(1, 256, generator=g))


def _sp_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        img, txt, vec = _block_inputs()
        per, pt = img.shape[1] // world, txt.shape[1] // world
        blk = _block(dist.group.WORLD)
        with torch.no_grad():
            o_img, o_txt = blk(img[:, rank * per:(rank + 1) * per].contiguous(),
                               txt[:, rank * pt:(rank + 1) * pt].contiguous(), vec)
        out_q.put((rank, o_img.numpy(), o_txt.numpy()))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_block_matches_single_process():
    """One sample split by image and text tokens over 2 gloo ranks (K/V
    all-gather of both streams) gives the rows of the single-process block."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    img, txt, vec = _block_inputs()
    with torch.no_grad():
        r_img, r_txt = _block(None)(img, txt, vec)
    got = np.concatenate([r[1] for r in res], axis=1)
    np.testing.assert_allclose(got, r_img.numpy(), rtol=1e-4, atol=1e-4)
    got_t = np.concatenate([r[2] for r in res], axis=1)
    np.testing.assert_allclose(got_t, r_txt.numpy(), rtol=1e-4, atol=1e-4)
