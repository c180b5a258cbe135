"""Column split of one NVFP4 linear over the ranks of a process group.

The reference runs a linear on one device (`nvfp4_linear_forward`,
nvfp4/nvfp4_gemm_gpu.mojo:185-224).  Split by output features, rank g holds
output rows [n0_g, n1_g) of the weight -- its packed codes, blockscales and
per-row weight_scale_2 -- and computes that slice of y = x W^T on its own
GPU: no collective, since every output row needs all of x and none of the
other rows.  The bounds fall on 16-row tiles (the GEMV's and GEMM's row
unit), as evenly as the tile count allows.  `gather=True` all-gathers the
slices (equal-size padded blocks over the process group, then the padding
dropped) for a caller that needs the whole y on every rank.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from .config import NvFp4Linear
from .nvfp4_gemm_gpu import nvfp4_linear

TILE_ROWS = 16


def shard_bounds(out_features: int, world: int, rank: int) -> Tuple[int, int]:
    """Output rows [n0, n1) of `rank`: 16-row tiles split as evenly as
    possible, the last tile possibly partial."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    tiles = (out_features + TILE_ROWS - 1) // TILE_ROWS
    t0, t1 = tiles * rank // world, tiles * (rank + 1) // world
    return min(t0 * TILE_ROWS, out_features), min(t1 * TILE_ROWS, out_features)


def _shard_linear(linear: NvFp4Linear, n0: int, n1: int) -> NvFp4Linear:
    rows = linear.weight_scale_2_rows
    return NvFp4Linear(linear.in_features, n1 - n0, input_scale=linear.input_scale,
                       weight_scale_2=linear.weight_scale_2,
                       weight_scale_2_rows=None if rows is None else rows[n0:n1].contiguous())


class ColumnSplitLinear:
    """This rank's slice of a linear split by output features.

    `packed_weights` [out, in/2] and `blockscales` [out, in/16] may be the
    whole weight (this rank's rows are taken) or, with `sharded=True`,
    already this rank's rows [n1 - n0, ...].  `compute` replaces the
    per-rank linear (tests run the CPU oracle through it); by default it is
    the CUDA linear of this package."""

    def __init__(self, linear: NvFp4Linear, packed_weights: torch.Tensor,
                 blockscales: torch.Tensor, group=None, sharded: bool = False,
                 compute: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.out_features = linear.out_features
        self.n0, self.n1 = shard_bounds(linear.out_features, self.world, self.rank)
        self.local = _shard_linear(linear, self.n0, self.n1)
        rows = self.n1 - self.n0
        if sharded:
            if packed_weights.shape[0] != rows or blockscales.shape[0] != rows:
                raise ValueError(f"rank {self.rank} expects {rows} weight rows")
            self.w, self.sf = packed_weights, blockscales
        else:
            self.w = packed_weights[self.n0:self.n1]
            self.sf = blockscales[self.n0:self.n1]
        self.compute = compute or nvfp4_linear
        # Largest slice: the all-gather's block size.
        self.max_rows = max(shard_bounds(linear.out_features, self.world, r)[1] -
                            shard_bounds(linear.out_features, self.world, r)[0]
                            for r in range(self.world))

    def forward(self, activations: torch.Tensor, out_dtype=torch.bfloat16, flags: int = 0,
                gather: bool = False) -> torch.Tensor:
        """y slice [M, n1 - n0] of this rank, or with `gather` the whole y
        [M, out_features] (identical on every rank)."""
        y = self.compute(self.local, self.w, self.sf, activations, out_dtype=out_dtype,
                         flags=flags)
        if not gather or self.world == 1:
            return y
        M = activations.shape[0]
        block = torch.zeros((M, self.max_rows), dtype=y.dtype, device=y.device)
        block[:, :y.shape[1]] = y
        flat = torch.empty((self.world * M, self.max_rows), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(flat, block.contiguous(), group=self.group)
        blocks = flat.view(self.world, M, self.max_rows)
        parts = []
        for r in range(self.world):
            a, b = shard_bounds(self.out_features, self.world, r)
            parts.append(blocks[r, :, :b - a])
        return torch.cat(parts, dim=1)

    __call__ = forward
