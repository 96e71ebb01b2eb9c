"""Tensor-parallel fused MLP over NCCL: the single-image latency mode of the DiT step (this build's addition).

One image cannot be split by seed, so for the step latency the MLP -- two thirds of a block's linear FLOPs -- is
split over G ranks while attention, qkv and out stay replicated:

* gate/up is column-split with the pairs kept local: rank r holds gate rows [rF/G, (r+1)F/G) and the same up rows,
  so its SwiGLU epilogue sees matching gate/up columns;
* down is split along K (its input columns) to match;
* each rank's fused pair yields a partial down output (bf16 [M, dim]); an NCCL all-reduce (sum) over NVLink adds the
  G partials; the gated residual follows.

Because down's input scale is static and F/G is a multiple of 16, the NVFP4 codes and scales of a rank's SwiGLU
output are exactly the corresponding columns of the unsharded ones; the result differs from one GPU only by the
bf16 rounding of the partials and the order of the sum.
"""

from __future__ import annotations

import torch

from . import linear as L


def shard_gate_up(gu: L.Fp4Linear, rank: int, world: int) -> L.Fp4Linear:
    """[gate; up] (2F rows) -> [gate rows of rank r; up rows of rank r] (2F/G rows)."""
    F = gu.n // 2
    if F % world or (F // world) % 128:
        raise ValueError(f"gate/up width F={F} must split into multiples of 128 over {world} ranks")
    f, lo = F // world, rank * (F // world)
    codes, scales = gu.codes, gu.scales()
    c = torch.cat([codes[lo:lo + f], codes[F + lo:F + lo + f]])
    s = torch.cat([scales[lo:lo + f], scales[F + lo:F + lo + f]])
    return L.Fp4Linear.from_checkpoint(c, s, gu.scale, gu.act)


def shard_down(down: L.Fp4Linear, rank: int, world: int) -> L.Fp4Linear:
    """down [dim, F] -> its input columns [rF/G, (r+1)F/G) (K split)."""
    F = down.k
    if F % world or (F // world) % 128:
        raise ValueError(f"down input width F={F} must split into multiples of 128 over {world} ranks")
    f, lo = F // world, rank * (F // world)
    c = down.codes[:, lo // 2:(lo + f) // 2].contiguous()
    s = down.scales()[:, lo // 16:(lo + f) // 16].contiguous()
    return L.Fp4Linear.from_checkpoint(c, s, down.scale, down.act)


class TPMLP:
    """This rank's shard of a static-scale NVFP4 gate/up + down pair; ``__call__`` runs the fused pair on the shard,
    all-reduces the partial output over ``group`` and returns it (or adds it into a residual stream)."""

    def __init__(self, gate_up: L.Nvfp4Linear, down: L.Nvfp4Linear, group=None):
        import torch.distributed as dist

        if gate_up.dynamic or down.dynamic:
            raise ValueError("tensor-parallel MLP needs static input scales (calibrate first)")
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.gate_up = L.Nvfp4Linear.from_fp4(shard_gate_up(gate_up.lin, self.rank, self.world))
        self.down = L.Nvfp4Linear.from_fp4(shard_down(down.lin, self.rank, self.world))

    def __call__(self, x, residual=None) -> torch.Tensor:
        import torch.distributed as dist

        y = L.swiglu_mlp(self.gate_up, self.down, x)
        dist.all_reduce(y, group=self.group)
        if residual is None:
            return y
        res, gate = residual
        return res.addcmul_(y.view_as(res), gate)
