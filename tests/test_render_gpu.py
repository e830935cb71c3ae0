"""GPU parity of the CUDA renderer (through the C ABI) against the reference fixtures and the oracle.

Tolerances are those the target states: rendered pixels within 1e-4 absolute, splat gradients within
1e-3 relative (the reference self-tests' metric max|d| / max|ref|), binning bit-exact."""

import ctypes as C

import numpy as np
import pytest
import torch

from golden_util import GOLDEN, REORDER_TOL, fnv_tile_hash, grad_rel, load_render, render_cases

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3


def _api():
    from gaussian_2d_splat_encoder_b200 import render_triton as rt

    return rt


def _run_api(fn, ins, H, W, gC, kw, dev="cuda"):
    leaves = {k: torch.tensor(v, device=dev, requires_grad=True) for k, v in ins.items()}
    out = fn(leaves["mu"], leaves["log_scale"], leaves["color"], leaves["opacity"], leaves["bg"], H, W,
             theta=leaves.get("theta"), **kw)
    (out * torch.tensor(gC, device=dev)).sum().backward()
    torch.cuda.synchronize()
    return out.detach().cpu().numpy(), {k: v.grad.cpu().numpy() for k, v in leaves.items()}


@pytest.mark.parametrize("name", render_cases())
def test_render_matches_reference(lib, name):
    c = load_render(name)
    fn = getattr(_api(), c["fn"])
    out, g = _run_api(fn, c["ins"], c["H"], c["W"], c["gC"], c["kw"])
    assert out.shape == c["out"].shape
    fd = float(np.abs(out - c["out"]).max())
    assert fd < FWD_TOL, fd
    rel = grad_rel(g, c["grads"])
    assert max(rel.values()) < GRAD_TOL, rel


def _bins(lib, mode, mu, ls, H, W, TILE=8, cutoff=3.0, max_octaves=6, base_texels=8.0):
    """Run a forward through the C ABI and read back the CSR it built."""
    from gaussian_2d_splat_encoder_b200 import _lib
    from gaussian_2d_splat_encoder_b200.render_triton import _desc

    B, N = mu.shape[0], mu.shape[1]
    dev = torch.device("cuda")
    mu_t = torch.tensor(mu, device=dev).contiguous()
    ls_t = torch.tensor(ls, device=dev).contiguous()
    col = torch.rand(B, N, 3, device=dev)
    op = torch.rand(B, N, device=dev)
    bg = torch.rand(B, 3, device=dev)
    d = _desc(mode=mode, B=B, N=N, C=3, H=H, W=W, TILE=TILE, odds=True, has_theta=False, cutoff=cutoff,
              base_texels=base_texels, max_octaves=max_octaves, max_pairs=-1)
    cap = lib.gs_render_pair_bound(C.byref(d))
    if cap > (1 << 26):
        from gaussian_2d_splat_encoder_b200.render_triton import _size_pairs

        cap = _size_pairs(d, mu_t, ls_t, dev, H, W, N, TILE, cutoff)
    d.pair_capacity = cap
    nb = lib.gs_render_workspace_size(C.byref(d), 0)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    out = torch.empty(B, 3, H, W, device=dev)
    p = _lib.ptr
    assert lib.gs_render_fwd(C.byref(d), p(mu_t), p(ls_t), p(col), p(op), p(bg), None, p(out), p(ws), nb,
                             _lib.stream_of(dev)) == 0
    torch.cuda.synchronize()
    tot = C.c_int64(0)
    tpi = C.c_int32(0)
    geom = (C.c_int32 * 40)()
    assert lib.gs_render_debug_bins(C.byref(d), p(ws), C.byref(tot), C.byref(tpi), geom, None, None, None) == 0
    ranges = np.zeros((B * tpi.value, 2), np.int32)
    ids = np.zeros(max(tot.value, 1), np.int32)
    octv = np.zeros(B * N, np.int32)
    assert lib.gs_render_debug_bins(C.byref(d), p(ws), None, None, None, ranges.ctypes.data_as(C.c_void_p),
                                    ids.ctypes.data_as(C.c_void_p), octv.ctypes.data_as(C.c_void_p)) == 0
    g = np.array(geom[:40]).reshape(8, 5)
    scale = torch.empty_like(ls_t)
    assert lib.gs_activate_scale(p(ls_t), p(scale), ls_t.numel(), _lib.stream_of(dev)) == 0
    torch.cuda.synchronize()
    return dict(total=tot.value, tpi=tpi.value, geom=g, ranges=ranges, ids=ids[:tot.value], oct=octv,
                scale=scale.cpu().numpy())


def _group_csr(bins, b, g, N):
    """(starts, ids local to the image) of group g of image b from the CUDA CSR."""
    H, W, ntx, nty, toff = bins["geom"][g]
    nt = ntx * nty
    r = bins["ranges"][b * bins["tpi"] + toff: b * bins["tpi"] + toff + nt]
    lens = np.where(r[:, 1] > r[:, 0], r[:, 1] - r[:, 0], 0)
    starts = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    # each tile's ids ascending (the renderer keeps them in the order its atomic cursor handed out slots)
    ids = np.concatenate([np.sort(bins["ids"][a:e]) for a, e in r if e > a] or [np.zeros(0, np.int32)]) - b * N
    return starts, ids.astype(np.int32)


def test_binning_bit_exact_small(lib, oracle):
    """Cull-mode CSR == the oracle's _build_tiles on the same (device-activated) scales, TILE 8/16/4,
    ragged sizes and off-image splats: each tile's set of splats (in the order its atomic cursor gave)."""
    from gaussian_2d_splat_encoder_b200 import _lib

    rng = np.random.default_rng(3)
    for (N, H, W, TILE, cutoff, spread) in ((1024, 64, 64, 8, 3.0, 1.0), (1024, 64, 64, 16, 5.0, 1.0),
                                            (700, 50, 37, 8, 3.0, 1.4), (300, 33, 71, 4, 3.0, 1.4)):
        mu = (rng.random((2, N, 2), dtype=np.float32) * spread - (spread - 1) / 2).astype(np.float32)
        ls = (rng.standard_normal((2, N, 2)) * 1.5 - 4.0).astype(np.float32)
        bins = _bins(lib, _lib.MODE_CULL, mu, ls, H, W, TILE, cutoff)
        for b in range(2):
            st_o, gid_o = oracle.build_tiles(mu[b], bins["scale"][b], H, W, TILE, cutoff)
            st_c, gid_c = _group_csr(bins, b, 0, N)
            assert np.array_equal(st_c, st_o)
            assert np.array_equal(gid_c, gid_o)


def test_binning_cfg1_full_size_vs_reference(lib, oracle):
    """Octave routing + per-octave tile lists of config 1 (768^2, 92,160 splats) against the digests of
    the reference's own _build_tiles (tests/golden/tiles_cfg1.npz) and the oracle."""
    from gaussian_2d_splat_encoder_b200 import _lib, synth

    d = np.load(GOLDEN / "tiles_cfg1.npz")
    s = synth.synth_splats_cfg1()
    mu, ls = s["mu"].numpy(), s["log_scale"].numpy()
    bins = _bins(lib, _lib.MODE_OCTAVE, mu, ls, 768, 768)
    assert np.array_equal(bins["oct"], d["oct"].astype(np.int32))
    ref_scale = (torch.nn.functional.softplus(s["log_scale"]) + 1e-4).numpy()
    assert np.abs(bins["scale"] - ref_scale).max() <= 1.2e-7 * np.abs(ref_scale).max()
    N = mu.shape[1]
    for o in range(7):
        starts, gid = _group_csr(bins, 0, o, N)
        if f"o{o}_starts" not in d.files:
            assert starts[-1] == 0
            continue
        assert np.array_equal(starts, d[f"o{o}_starts"])
        idx = np.nonzero(bins["oct"] == o)[0]
        assert np.array_equal(fnv_tile_hash(np.searchsorted(idx, gid), starts), d[f"o{o}_hash"])
    # the cull path bins the whole set at native resolution
    bins = _bins(lib, _lib.MODE_CULL, mu, ls, 768, 768)
    starts, gid = _group_csr(bins, 0, 0, N)
    assert np.array_equal(starts, d["cull_starts"])
    assert np.array_equal(fnv_tile_hash(gid, starts), d["cull_hash"])


def test_full_size_cfg1_vs_oracle(lib, oracle):
    """Config 1 at full size: render_alpha_octave(odds) forward + backward of an L2 loss, CUDA vs
    oracle."""
    from gaussian_2d_splat_encoder_b200 import synth

    s = synth.synth_splats_cfg1()
    ins = {k: s[k].numpy() for k in ("mu", "log_scale", "color", "opacity", "bg", "theta")}
    target = s["target"].numpy()
    rt = _api()
    leaves = {k: torch.tensor(v, device="cuda", requires_grad=True) for k, v in ins.items()}
    out = rt.render_alpha_octave(leaves["mu"], leaves["log_scale"], leaves["color"], leaves["opacity"],
                                 leaves["bg"], 768, 768, theta=leaves["theta"], odds=True)
    loss = (out - torch.tensor(target, device="cuda")).square().sum()
    loss.backward()
    gC = 2.0 * (out.detach().cpu().numpy() - target)
    o_out, o_g = oracle.render_alpha_octave(ins["mu"], ins["log_scale"], ins["color"], ins["opacity"], ins["bg"],
                                            768, 768, theta=ins["theta"], odds=True, grad_out=gC)
    assert np.abs(out.detach().cpu().numpy() - o_out).max() < FWD_TOL
    rel = grad_rel({k: v.grad.cpu().numpy() for k, v in leaves.items()}, o_g)
    assert max(rel.values()) < GRAD_TOL, rel


def test_pair_budget_exceeded(lib):
    rt = _api()
    g = torch.Generator().manual_seed(0)
    mu = torch.rand(1, 500, 2, generator=g).cuda()
    ls = torch.full((1, 500, 2), -3.0).cuda()
    col = torch.rand(1, 500, 3, generator=g).cuda()
    op = torch.rand(1, 500, generator=g).cuda()
    bg = torch.rand(1, 3, generator=g).cuda()
    with pytest.raises(rt.PairBudgetExceeded):
        rt.render_alpha_octave(mu, ls, col, op, bg, 256, 256, max_pairs=100)
    out = rt.render_alpha_octave(mu, ls, col, op, bg, 256, 256, max_pairs=10**7)
    assert torch.isfinite(out).all()


def test_repeat_and_batch_consistency(lib):
    """Two renders of the same splats, and a batch of three against three single renders, agree to the
    rounding of the per-tile sums (REORDER_TOL)."""
    from gaussian_2d_splat_encoder_b200 import synth

    rt = _api()
    s = synth.synth_splats_cfg1(N=20000, H=384, W=384, seed=5)
    args = [s[k].cuda() for k in ("mu", "log_scale", "color", "opacity", "bg")]
    a = rt.render_alpha_octave(*args, 384, 384, theta=s["theta"].cuda(), odds=True)
    b = rt.render_alpha_octave(*args, 384, 384, theta=s["theta"].cuda(), odds=True)
    assert torch.allclose(a, b, atol=REORDER_TOL, rtol=0)
    # batch of 3 (the same image, a shifted copy, a recoloured copy) == three single renders
    s2 = synth.synth_splats_cfg1(N=20000, H=384, W=384, seed=6)
    s3 = synth.synth_splats_cfg1(N=20000, H=384, W=384, seed=7)
    batch = {k: torch.cat([x[k] for x in (s, s2, s3)]).cuda() for k in ("mu", "log_scale", "color", "opacity",
                                                                       "bg", "theta")}
    ob = rt.render_alpha_octave(batch["mu"], batch["log_scale"], batch["color"], batch["opacity"], batch["bg"],
                                384, 384, theta=batch["theta"], odds=True)
    for i, x in enumerate((s, s2, s3)):
        oi = rt.render_alpha_octave(*[x[k].cuda() for k in ("mu", "log_scale", "color", "opacity", "bg")],
                                    384, 384, theta=x["theta"].cuda(), odds=True)
        assert torch.allclose(ob[i:i + 1], oi, atol=REORDER_TOL, rtol=0)


def test_empty_and_single(lib):
    rt = _api()
    z = torch.zeros(1, 0, 2, device="cuda")
    bg = torch.tensor([[0.1, 0.2, 0.3]], device="cuda")
    out = rt.render_alpha_octave(z, z, torch.zeros(1, 0, 3, device="cuda"), torch.zeros(1, 0, device="cuda"), bg,
                                 40, 24, odds=True)
    assert torch.allclose(out, bg[:, :, None, None].expand(1, 3, 40, 24))


def test_row_band_partition_sums_to_full(lib):
    """Tile-row sharding: rendering a partition of the native rows reproduces the full image row by row,
    and the band gradients (each from the loss restricted to its rows) sum to the full gradient."""
    from gaussian_2d_splat_encoder_b200 import synth

    rt = _api()
    s = synth.synth_splats_cfg1(N=30000, H=320, W=256, seed=11)
    keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
    d = {k: v.cuda() for k, v in s.items()}
    tgt = torch.rand(1, 3, 320, 256, generator=torch.Generator().manual_seed(3)).cuda()
    L = [d[k].clone().requires_grad_(True) for k in keys]
    full = rt.render_alpha_octave(*L[:5], 320, 256, theta=L[5], odds=True)
    loss = (full - tgt).square().sum()
    ref = torch.autograd.grad(loss, L)
    acc = [torch.zeros_like(g) for g in ref]
    for y0, y1 in ((0, 88), (88, 200), (200, 320)):
        Lb = [d[k].clone().requires_grad_(True) for k in keys]
        out = rt.render_alpha_octave(*Lb[:5], 320, 256, theta=Lb[5], odds=True, row_band=(y0, y1))
        assert torch.allclose(out[:, :, y0:y1], full[:, :, y0:y1].detach(), atol=REORDER_TOL, rtol=0)
        lb = (out[:, :, y0:y1] - tgt[:, :, y0:y1]).square().sum()
        for a, g in zip(acc, torch.autograd.grad(lb, Lb)):
            a += g
    for a, r in zip(acc, ref):
        rel = (a - r).abs().max().item() / max(r.abs().max().item(), 1e-30)
        assert rel < 1e-4, rel
