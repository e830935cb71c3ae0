"""Host-side logic of the two multi-GPU modes (one process per GPU, torch.distributed).

* Image-per-GPU data parallelism (config 3): ``images_for_rank`` deals a batch of image ids round-robin;
  no collective touches the data path.
* Tile-row sharded fitting (config 4): rank r renders native rows ``row_bands(H, R)[r]`` with
  ``render_alpha_octave(..., row_band=...)``; the L2 loss is normalised by the GLOBAL pixel count
  (``band_mse``) so the per-rank gradients are partial sums over disjoint pixel sets.  ``ShardedAdam`` sums
  and splits them with one reduce-scatter, each rank runs Adam on its 1/R of the flattened splat
  parameters, and one all-gather hands every rank the full updated parameters (the bytes of the
  all-reduce it replaces, ``allreduce_grads``, with 1/R of the optimizer work and state per rank).
"""

from __future__ import annotations

import torch


def row_bands(H: int, world: int):
    """[(y0, y1)] partition of the H native rows into `world` contiguous bands (sizes differ by <= 1)."""
    if world < 1 or world > H:
        raise ValueError(f"cannot split {H} rows over {world} ranks")
    cuts = [H * i // world for i in range(world + 1)]
    return [(cuts[i], cuts[i + 1]) for i in range(world)]


def images_for_rank(n_images: int, rank: int, world: int):
    """Image indices this rank processes (round-robin deal)."""
    return list(range(rank, n_images, world))


def band_mse(out: torch.Tensor, target: torch.Tensor, band, H: int, W: int) -> torch.Tensor:
    """This band's share of mean((out - target)^2) over the whole [B,C,H,W] image."""
    y0, y1 = band
    B, C = out.shape[0], out.shape[1]
    return (out[:, :, y0:y1] - target[:, :, y0:y1]).square().sum() / float(B * C * H * W)


def flatten_into(flat: torch.Tensor, tensors) -> torch.Tensor:
    off = 0
    for t in tensors:
        n = t.numel()
        flat[off:off + n].copy_(t.reshape(-1))
        off += n
    return flat


def views_of(flat: torch.Tensor, like):
    out, off = [], 0
    for t in like:
        n = t.numel()
        out.append(flat[off:off + n].view_as(t))
        off += n
    return out


def allreduce_grads(grads, flat: torch.Tensor, group=None):
    """Sum the per-rank partial gradients in place (one all-reduce over a flat buffer) and return views of
    the summed gradients shaped like `grads`."""
    import torch.distributed as dist

    flatten_into(flat, grads)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(flat, group=group)
    return views_of(flat, grads)


class ShardedAdam:
    """Adam (lr, torch's defaults otherwise) over the leaves' flattened parameters, sharded over the ranks
    of `group`: ``step(grads)`` reduce-scatters the per-rank partial gradients (each rank receives the SUM
    over ranks of its 1/R slice), updates its slice with torch's fused Adam, all-gathers the slices and
    copies the full parameters back into the leaves.  Adam is elementwise, so the result equals one Adam
    over the summed gradients; every rank ends the step with the same parameters.  The flat buffers are
    padded to a multiple of the world size (padding: zero gradient, zero parameter).  CUDA-graph
    capturable on CUDA devices (fused, capturable Adam; NCCL collectives)."""

    def __init__(self, leaves, lr: float, group=None):
        import torch.distributed as dist

        self.leaves = list(leaves)
        self.group = group
        dev = self.leaves[0].device
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0
        n = sum(t.numel() for t in self.leaves)
        self.shard = (n + self.world - 1) // self.world
        self.flat_g = torch.zeros(self.shard * self.world, device=dev)
        self.flat_p = torch.zeros(self.shard * self.world, device=dev)
        with torch.no_grad():
            flatten_into(self.flat_p, [t.detach() for t in self.leaves])
        lo = self.rank * self.shard
        self.param = torch.nn.Parameter(self.flat_p[lo:lo + self.shard].clone())
        self.gshard = torch.zeros(self.shard, device=dev) if self.world > 1 else None
        cuda = dev.type == "cuda"
        self.opt = torch.optim.Adam([self.param], lr=lr, fused=True, capturable=cuda)

    @torch.no_grad()
    def step(self, grads):
        import torch.distributed as dist

        flatten_into(self.flat_g, grads)
        if self.world > 1:
            dist.reduce_scatter_tensor(self.gshard, self.flat_g, group=self.group)
            self.param.grad = self.gshard
        else:
            self.param.grad = self.flat_g
        self.opt.step()
        if self.world > 1:
            dist.all_gather_into_tensor(self.flat_p, self.param.data, group=self.group)
        else:
            self.flat_p.copy_(self.param.data)
        for t, v in zip(self.leaves, views_of(self.flat_p, self.leaves)):
            t.data.copy_(v)
