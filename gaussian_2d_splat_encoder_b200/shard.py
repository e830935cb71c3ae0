"""Host-side logic of the two multi-GPU modes (one process per GPU, torch.distributed).

* Image-per-GPU data parallelism (config 3): ``images_for_rank`` deals a batch of image ids round-robin;
  no collective touches the data path.
* Tile-row sharded fitting (config 4): rank r renders native rows ``row_bands(H, R)[r]`` with
  ``render_alpha_octave(..., row_band=...)``; the L2 loss is normalised by the GLOBAL pixel count
  (``band_mse``) so the per-rank gradients are partial sums over disjoint pixel sets, and one all-reduce
  (``allreduce_grads``) of the flattened splat gradients makes every rank's Adam step identical.
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
