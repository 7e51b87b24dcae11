"""Multi-GPU layouts of the quantised linear (one process per GPU).

The reference runs one layer on one device.  Across the GPUs of one box the
layer is split in one of two ways, over ``torch.distributed`` (NCCL on GPUs):

* token sharding (:func:`shard_tokens`): every rank holds the whole layer and
  runs its own contiguous slice of tokens.  There is no data exchange; this is
  the layout for batches and long sequences (weak scaling).
* output-feature sharding (:class:`FeatureShardedLinear`): rank ``r`` holds
  weight rows ``[r * Nr, (r + 1) * Nr)`` of the ``[N, K]`` weight (with their
  scales and bias entries).  Every rank preps and quantises the same
  activations, runs the GEMM over its own rows, and one all-gather assembles
  the ``[M, N]`` output.  This is the layout for a single large layer whose
  weights should not be replicated (strong scaling).

Each output element is computed by exactly one rank with the same kernel and
inputs as on one GPU, so both layouts give results bit-identical to the
single-GPU forward.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

__all__ = ["shard_tokens", "feature_rows", "FeatureShardedLinear"]


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows ``[rank * ceil(M / world), ...)`` of ``x`` viewed as ``[M, K]``."""
    x2 = x.reshape(-1, x.shape[-1])
    per = -(-x2.shape[0] // world)
    return x2[rank * per:(rank + 1) * per]


def feature_rows(N: int, rank: int, world: int) -> tuple[int, int, int]:
    """``(start, stop, Nr)``: this rank's weight rows and the padded per-rank
    width ``Nr = ceil(N / world)`` (every rank contributes Nr output columns to
    the all-gather; the last rank's missing rows are zero and trimmed)."""
    nr = -(-N // world)
    start = min(N, rank * nr)
    return start, min(N, start + nr), nr


def _pad_rows(t: torch.Tensor | None, rows: int) -> torch.Tensor | None:
    if t is None or t.shape[0] == rows:
        return t
    pad = torch.zeros((rows - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    return torch.cat([t, pad], dim=0)


class FeatureShardedLinear:
    """Output-feature-sharded W8A8 / W4A8 linear.

    Args:
        weight: the full weight, int8 ``[N, K]`` or packed INT4 uint8
            ``[N, ceil(K/2)]`` (reference packing); only this rank's rows are kept.
        weight_scale: ``[N]``, ``[N, 1]`` or ``[N, G]`` scales.
        bias: optional ``[N]``.
        group_size: K-group size when ``weight_scale`` has G > 1 columns.
        smoothrot, rot_size, w_in, perm, smooth: the activation prep of the
            layer (``_ops.py:337-365``), applied identically on every rank.
        group: process group (default: the world).
        repack: store INT4 weights in the expansion-friendly nibble layout.
        prep, gemm: the prep/quantise and GEMM callables; default to the B200
            runtime (``prep_quantize``, ``gemm_a8``).  Tests substitute a CPU
            restatement to check the sharding logic without a GPU.
    """

    def __init__(self, weight: torch.Tensor, weight_scale: torch.Tensor, bias: torch.Tensor | None = None, *,
                 group_size: int | None = None, smoothrot: torch.Tensor | None = None, rot_size: int = 0,
                 w_in: int | None = None, perm: torch.Tensor | None = None, smooth: torch.Tensor | None = None,
                 group=None, repack: bool = True, device: torch.device | None = None,
                 prep: Callable | None = None, gemm: Callable | None = None) -> None:
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1   # no process group: one rank
        self.rank = dist.get_rank(group) if dist_on else 0
        self.N = weight.shape[0]
        self.int4 = weight.dtype == torch.uint8
        self.K_w = weight.shape[1] * 2 if self.int4 else weight.shape[1]
        start, stop, self.Nr = feature_rows(self.N, self.rank, self.world)
        dev = device if device is not None else weight.device
        sw = weight_scale.reshape(self.N, -1)
        self.weight = _pad_rows(weight[start:stop], self.Nr).to(dev).contiguous()
        self.scale = _pad_rows(sw[start:stop].float(), self.Nr).to(dev).contiguous()
        self.bias = None if bias is None else _pad_rows(bias[start:stop], self.Nr).to(dev).contiguous()
        self.group_size = group_size
        self.smoothrot = None if smoothrot is None else smoothrot.to(dev)
        self.rot_size = rot_size
        self.w_in = w_in
        self.perm = None if perm is None else perm.to(dev, torch.int32)
        self.smooth = None if smooth is None else smooth.to(dev)
        if prep is None or gemm is None:
            from . import _b200_runtime as rt
            prep = prep or rt.prep_quantize
            gemm = gemm or rt.gemm_a8
            self.repacked = bool(repack and self.int4)
            if self.repacked:
                self.weight = rt.repack_int4(self.weight, self.K_w, 0)
        else:
            self.repacked = False
        self._prep = prep
        self._gemm = gemm

    def local_forward(self, x: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """This rank's ``[M, Nr]`` output columns (no communication)."""
        xq, s_a, _, _ = self._prep(x, smoothrot=self.smoothrot, rot_size=self.rot_size, w_in=self.w_in,
                                   perm=self.perm, smooth=self.smooth)
        kw = {"repacked": True} if self.repacked else {}
        return self._gemm(xq, self.weight, self.scale, s_a, bias=self.bias, out_dtype=out_dtype,
                          group_size=self.group_size, **kw)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        local = self.local_forward(x2, x.dtype)
        if self.world == 1:
            return local[:, :self.N].reshape(*lead, self.N)
        parts = [torch.empty_like(local) for _ in range(self.world)]
        dist.all_gather(parts, local.contiguous(), group=self.group)
        out = torch.cat(parts, dim=1)[:, :self.N]
        return out.reshape(*lead, self.N)

    def forward_overlapped(self, x: torch.Tensor, chunks: int = 4) -> torch.Tensor:
        """Same result as ``__call__`` with the all-gather hidden behind the
        GEMM: the tokens are prepped once, then the GEMM runs chunk by chunk
        (``chunks`` contiguous token ranges) and each chunk's all-gather is
        issued asynchronously as soon as its GEMM is queued, so the exchange
        of chunk i overlaps the GEMM of chunk i + 1 (NCCL runs on its own
        stream, ordered after the chunk's GEMM).  The chunks are assembled
        into ``[M, N]`` once every exchange has completed."""
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if self.world == 1:
            return self(x)
        M = x2.shape[0]
        xq, s_a, _, _ = self._prep(x2, smoothrot=self.smoothrot, rot_size=self.rot_size, w_in=self.w_in,
                                   perm=self.perm, smooth=self.smooth)
        kw = {"repacked": True} if self.repacked else {}
        step = -(-M // max(1, chunks))
        step = -(-step // 128) * 128 if step > 128 else step   # whole token tiles per chunk
        pending = []
        for m0 in range(0, M, step):
            m1 = min(M, m0 + step)
            local = self._gemm(xq[m0:m1], self.weight, self.scale, s_a[m0:m1], bias=self.bias,
                               out_dtype=x.dtype, group_size=self.group_size, **kw).contiguous()
            parts = [torch.empty_like(local) for _ in range(self.world)]
            work = dist.all_gather(parts, local, group=self.group, async_op=True)
            pending.append((m0, m1, parts, work, local))
        out = torch.empty((M, self.N), dtype=x.dtype, device=x2.device)
        for m0, m1, parts, work, _ in pending:
            work.wait()
            out[m0:m1] = torch.cat(parts, dim=1)[:, :self.N]
        return out.reshape(*lead, self.N)
