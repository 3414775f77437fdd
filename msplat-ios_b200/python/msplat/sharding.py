"""Tile-row sharding of the training step across GPUs (one process per GPU).

Every rank holds the full parameter set and projects all Gaussians; rank r
bins, sorts and rasterises the tile rows [row0, row1) (plus a one-tile-row
halo that the 11x11 SSIM window needs), evaluates the loss and the backward on
its own rows, and leaves per-Gaussian raster-space gradients [N, 16]. Those are
summed across ranks with an NCCL reduce-scatter so that rank r receives the
Gaussian slice [g_begin, g_end); it runs the projection VJP and Adam on that
slice, and the six parameter groups are all-gathered in place. Adam moments
stay sharded (each rank only touches its slice).
"""
from __future__ import annotations

import dataclasses


@dataclasses.dataclass
class ShardPlan:
    n: int
    tiles_y: int
    world: int
    rank: int

    def __post_init__(self):
        rows = -(-self.tiles_y // self.world)
        self.row0 = min(self.rank * rows, self.tiles_y)
        self.row1 = min((self.rank + 1) * rows, self.tiles_y)
        self.chunk = -(-self.n // self.world)
        self.chunk = -(-self.chunk // 256) * 256
        self.padded = self.chunk * self.world
        self.g_begin = min(self.rank * self.chunk, self.n)
        self.g_end = min((self.rank + 1) * self.chunk, self.n)


def pad_gaussians(g, padded: int):
    """Re-home each parameter group in a [padded, ...] buffer (rows >= n stay
    zero) so that all-gathers can run in place; g keeps contiguous [n] views."""
    import torch
    n = g.n
    g.full = []
    for name in ("means", "scales", "quats", "f_dc", "f_rest", "opacities"):
        t = getattr(g, name)
        full = torch.zeros((padded,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        full[:n].copy_(t)
        setattr(g, name, full[:n])
        g.full.append(full)
    return g


def sharded_step(B, dist, g, cam, degree, bg, gt, l1, ld, lssim, adam, stats, plan, rg, rg_shard, parts):
    B.shard_forward_backward(g, cam, degree, bg, gt, l1, ld, lssim, plan.row0, plan.row1, rg, parts)
    dist.reduce_scatter_tensor(rg_shard, rg, op=dist.ReduceOp.SUM)
    adam.step += 1
    B.shard_project_backward_adam(g, cam, degree, rg_shard.data_ptr() - plan.g_begin * 64, plan.g_begin,
                                  plan.g_end, adam, stats=stats, count_step=False)
    for full in g.full:
        if full.numel() == 0:
            continue
        dist.all_gather_into_tensor(full, full[plan.rank * plan.chunk:(plan.rank + 1) * plan.chunk])
    dist.all_reduce(parts)
