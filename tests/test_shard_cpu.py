"""Multi-process host logic on CPU (gloo, world size 2): row bands partition the image, per-band partial
gradients (the oracle's gradients of the band's share of the loss) all-reduce to the full gradient, and
the replicated Adam steps stay identical across ranks; the sharded Adam (reduce-scatter, Adam on 1/R of
the parameters, all-gather) gives the same parameters; image dealing covers every image once."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, sharded=False):
    import torch.distributed as dist

    from gaussian_2d_splat_encoder_b200 import shard
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(7)
    B, N, H, W = 1, 400, 48, 40
    ins = dict(mu=torch.rand(B, N, 2, generator=g), log_scale=torch.rand(B, N, 2, generator=g) * 2 - 5.5,
               color=torch.rand(B, N, 3, generator=g), opacity=torch.rand(B, N, generator=g) * 0.9,
               bg=torch.rand(B, 3, generator=g), theta=torch.rand(B, N, generator=g) * 3.0)
    target = torch.rand(B, 3, H, W, generator=g)
    keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
    band = shard.row_bands(H, world)[rank]
    leaves = [ins[k].clone() for k in keys]
    opt = (shard.ShardedAdam(leaves, lr=1e-2) if sharded
           else torch.optim.Adam([t.requires_grad_(True) for t in leaves], lr=1e-2))
    flat = torch.zeros(sum(t.numel() for t in leaves))
    for _ in range(2):
        npi = [t.detach().numpy() for t in leaves]
        out = O.render_alpha_octave(*npi[:5], H, W, theta=npi[5], odds=True)
        gout = np.zeros_like(out)
        y0, y1 = band
        gout[:, :, y0:y1] = 2.0 * (out - target.numpy())[:, :, y0:y1] / out.size    # d band_mse / d out
        _, og = O.render_alpha_octave(*npi[:5], H, W, theta=npi[5], odds=True, grad_out=gout)
        if sharded:
            opt.step([torch.from_numpy(og[k]) for k in keys])
            continue
        grads = shard.allreduce_grads([torch.from_numpy(og[k]) for k in keys], flat)
        for t, gr in zip(leaves, grads):
            t.grad = gr.clone()
        opt.step()
    q.put((rank, [t.detach().numpy().copy() for t in leaves]))
    dist.destroy_process_group()


def test_row_bands_and_images():
    from gaussian_2d_splat_encoder_b200 import shard

    for H in (7, 768, 2048):
        for R in (1, 2, 3, 8):
            if R > H:
                continue
            b = shard.row_bands(H, R)
            assert b[0][0] == 0 and b[-1][1] == H and all(b[i][1] == b[i + 1][0] for i in range(R - 1))
            assert max(y1 - y0 for y0, y1 in b) - min(y1 - y0 for y0, y1 in b) <= 1
    seen = sorted(i for r in range(3) for i in shard.images_for_rank(64, r, 3))
    assert seen == list(range(64))


def test_sharded_fit_matches_single_process():
    from gaussian_2d_splat_encoder_b200 import shard  # noqa: F401
    from oracle import oracle as O

    O.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # both ranks hold identical parameters after the replicated Adam steps ...
    for a, b in zip(res[0], res[1]):
        assert np.array_equal(a, b)
    # ... equal to a single-process run over the whole image
    q1 = ctx.Queue()
    p = ctx.Process(target=_worker, args=(0, 1, _free_port(), q1))
    p.start()
    _, single = q1.get(timeout=300)
    p.join(timeout=60)
    for a, b in zip(res[0], single):
        assert np.allclose(a, b, atol=1e-6, rtol=1e-5)


def test_sharded_adam_matches_replicated():
    """ShardedAdam over 2 gloo ranks: both ranks end with identical parameters, equal to the replicated
    all-reduce + Adam run of the same steps."""
    from oracle import oracle as O

    O.build()
    ctx = mp.get_context("spawn")
    runs = {}
    for sharded in (False, True):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, q, sharded)) for r in range(2)]
        for p in procs:
            p.start()
        runs[sharded] = dict(q.get(timeout=300) for _ in procs)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    for a, b in zip(runs[True][0], runs[True][1]):
        assert np.array_equal(a, b)
    for a, b in zip(runs[True][0], runs[False][0]):
        assert np.allclose(a, b, atol=1e-6, rtol=1e-6)
