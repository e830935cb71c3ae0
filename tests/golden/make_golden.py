"""Generate the golden fixtures under tests/golden/ by running the REFERENCE implementation.

Run once in a container that has the reference checkout, next to this repository (``../reference``)
or wherever ``GSPLAT_REFERENCE`` points:

    python tests/golden/make_golden.py [case ...]

The reference's Triton kernels run on CPU through ``TRITON_INTERPRET=1``.  The interpreter cannot
evaluate the *method* form ``x.cos()`` / ``x.sin()`` used by the reference kernels, so before importing
the reference this script rebinds ``triton.language.core.tensor.cos/sin`` to ``tl.cos/tl.sin`` (a
harness-level shim; the reference files are untouched).  Every fixture stores the inputs it was made
from, so the tests never need the reference at run time.

Cases mirror the reference's own self-tests (render_triton.py:983-1533: same seeds, shapes and cutoffs)
plus edge cases (ragged image sizes, off-image splats, a single splat, theta=None), the binning of
config 1 at full size (768^2, 92,160 splats) and the pixel-list render (render.py:68-87).
"""

from __future__ import annotations

import math
import os
import sys
import time
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton.language as tl  # noqa: E402
import triton.language.core as tlc  # noqa: E402

tlc.tensor.cos = lambda self: tl.cos(self)
tlc.tensor.sin = lambda self: tl.sin(self)

REF = Path(os.environ.get("GSPLAT_REFERENCE", Path(__file__).resolve().parents[3] / "reference"))
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parents[1]))

from gaussian_splat_encoder import render as ref_render  # noqa: E402
from gaussian_splat_encoder import render_triton as rt  # noqa: E402

from gaussian_2d_splat_encoder_b200 import synth  # noqa: E402

NAMES = ("mu", "log_scale", "color", "opacity", "bg", "theta")


def tile_hash(gid_sorted: np.ndarray, starts: np.ndarray) -> np.ndarray:
    """Order-independent per-tile digest: per tile, the ids sorted ascending, hashed with a 64-bit
    polynomial (wrapping).  Used where the full id lists would be too large for a fixture."""
    nt = starts.shape[0] - 1
    out = np.zeros(nt, dtype=np.uint64)
    g = gid_sorted.astype(np.uint64)
    with np.errstate(over="ignore"):
        for t in range(nt):
            s, e = int(starts[t]), int(starts[t + 1])
            if e > s:
                v = np.sort(g[s:e])
                w = np.uint64(1469598103934665603)
                for x in v:
                    w = (w ^ x) * np.uint64(1099511628211)
                out[t] = w
    return out


def canonical_tiles(gid: torch.Tensor, starts: torch.Tensor):
    """Sort ids within each tile (the reference's argsort is unstable; only the per-tile SET is
    defined)."""
    g = gid.numpy().astype(np.int32).copy()
    s = starts.numpy().astype(np.int32)
    for t in range(s.shape[0] - 1):
        a, b = s[t], s[t + 1]
        if b > a:
            g[a:b] = np.sort(g[a:b])
    return g, s


def leaves(seed, B, N, C, ls_off, op_mul=1.0, theta=True):
    torch.manual_seed(seed)
    mu = torch.rand(B, N, 2)
    ls = torch.rand(B, N, 2) - ls_off
    col = torch.rand(B, N, C)
    op = torch.rand(B, N) * op_mul
    bg = torch.rand(B, C)
    th = torch.rand(B, N) * 3.14 if theta else None
    return [mu, ls, col, op, bg, th]


def upstream_grad(shape, gseed):
    """The upstream gradient dL/dout of a render fixture: standard normal from a CPU generator."""
    return torch.randn(shape, generator=torch.Generator().manual_seed(gseed))


def run_render(fn, L, H, W, gseed=1234, **kw):
    """Forward + backward of sum(out * gC) through a reference entry point; returns arrays.  gC is not
    stored: it is regenerated from ``gseed`` with ``upstream_grad``."""
    Lr = [t.detach().clone().requires_grad_(True) if t is not None else None for t in L]
    out = fn(*Lr[:5], H, W, theta=Lr[5], **kw)
    gC = upstream_grad(out.shape, gseed)
    (out * gC).sum().backward()
    rec = {f"in_{n}": t.detach().numpy() for n, t in zip(NAMES, L) if t is not None}
    rec.update({"H": H, "W": W, "gseed": gseed, "out": out.detach().numpy()})
    for n, t in zip(NAMES, Lr):
        if t is not None:
            rec[f"grad_{n}"] = t.grad.numpy()
    return rec


def case_render():
    cases = {}
    B, C = 2, 3
    # mirrors _selftest_odds_fields_equiv (render_triton.py:1500-1533)
    L = leaves(29, B, 1024, C, 2.5, 0.9)
    cases["octave_odds_m0"] = (rt.render_alpha_octave, L, 64, 64,
                               dict(cutoff=3.0, max_octaves=0, odds=True))
    # mirrors _selftest_odds (render_triton.py:1460-1497)
    L = leaves(23, B, 256, C, 1.5, 0.9)
    cases["octave_odds_c6"] = (rt.render_alpha_octave, L, 32, 32,
                               dict(cutoff=6.0, max_octaves=0, odds=True))
    # mirrors _selftest_octave_split (render_triton.py:1370-1402): log-uniform scales over ~6 octaves
    torch.manual_seed(17)
    N = 800
    mu = torch.rand(1, N, 2)
    sig = torch.exp(torch.rand(1, N) * (math.log(0.31) - math.log(0.006)) + math.log(0.006))
    ls = torch.log(torch.exp(sig).clamp_min(1 + 1e-6) - 1.0).unsqueeze(-1).expand(1, N, 2).contiguous()
    col = torch.rand(1, N, C)
    op = torch.rand(1, N) * 0.4
    th = torch.rand(1, N) * 3.14159
    bgv = torch.rand(1, C)
    L = [mu, ls, col, op, bgv, th]
    cases["octave_split_odds"] = (rt.render_alpha_octave, L, 256, 256, dict(odds=True))
    cases["octave_split_alpha"] = (rt.render_alpha_octave, L, 256, 256, dict(odds=False))
    # mirrors _selftest_fields_equiv (render_triton.py:1214-1253)
    L = leaves(7, B, 1024, C, 2.5)
    cases["cull_alpha"] = (rt.render_alpha_full_triton, L, 64, 64, dict(cull=True, cutoff=3.0))
    cases["cull_odds"] = (rt.render_alpha_full_triton, L, 64, 64, dict(cull=True, cutoff=3.0, odds=True))
    cases["multires_none"] = (rt.render_alpha_multires, L, 64, 64, dict(n_coarse=None, cutoff=3.0))
    # mirrors _selftest_cull_backward (render_triton.py:983-1017): TILE 16 is exercised too
    L = leaves(3, B, 1024, C, 2.0)
    cases["cull_tile16_c5"] = (rt.render_alpha_full_triton, L, 64, 64, dict(cull=True, cutoff=5.0, TILE=16))
    # mirrors _selftest_backward (render_triton.py:1076-1120): exact path with and without theta
    L = leaves(1, B, 256, C, 1.5)
    cases["exact_theta"] = (rt.render_alpha_full_triton, L, 32, 32, dict(cull=False))
    cases["exact_notheta"] = (rt.render_alpha_full_triton, L[:5] + [None], 32, 32, dict(cull=False))
    cases["torch_full_notheta"] = (ref_render.render_alpha_full, L[:5] + [None], 32, 32,
                                   dict(chunk_pixels=300))
    # mirrors _selftest_multires_split (render_triton.py:1256-1298)
    torch.manual_seed(11)
    Nc, Nf = 64, 512
    N = Nc + Nf
    mu = torch.rand(1, N, 2)
    ls = torch.empty(1, N, 2)
    ls[:, :Nc] = math.log(math.exp(0.12) - 1.0)
    ls[:, Nc:] = math.log(math.exp(0.015) - 1.0)
    col = torch.rand(1, N, C)
    op = torch.rand(1, N) * 0.5
    bgv = torch.rand(1, C)
    th = torch.rand(1, N) * 3.14159
    L = [mu, ls, col, op, bgv, th]
    cases["multires_split"] = (rt.render_alpha_multires, L, 128, 128, dict(n_coarse=Nc, coarse_factor=8))
    cases["multires_split_odds"] = (rt.render_alpha_multires, L, 128, 128,
                                    dict(n_coarse=Nc, coarse_factor=8, odds=True))
    # edge cases: ragged non-square size, splats off the image, huge and tiny splats, theta=None
    torch.manual_seed(5)
    N = 300
    mu = torch.rand(2, N, 2) * 1.4 - 0.2
    ls = torch.randn(2, N, 2) * 1.5 - 4.0
    col = torch.rand(2, N, C)
    op = torch.rand(2, N)
    op[:, :10] = 1.0                                        # clamp branch (a = 1 - 1e-4)
    bgv = torch.rand(2, C)
    th = torch.rand(2, N) * 3.14
    L = [mu, ls, col, op, bgv, th]
    cases["octave_ragged_odds"] = (rt.render_alpha_octave, L, 50, 37, dict(odds=True))
    cases["octave_ragged_alpha_noth"] = (rt.render_alpha_octave, L[:5] + [None], 37, 50, dict(odds=False))
    cases["cull_ragged_odds"] = (rt.render_alpha_full_triton, L, 50, 37, dict(cull=True, odds=True))
    # a single splat, and the encoder's internal 384^2 coarse render shape (coarse-scale splats)
    L = [torch.tensor([[[0.5, 0.4]]]), torch.tensor([[[-3.0, -2.5]]]), torch.tensor([[[0.2, 0.7, 0.9]]]),
         torch.tensor([[0.8]]), torch.tensor([[0.1, 0.2, 0.3]]), torch.tensor([[0.6]])]
    cases["octave_single"] = (rt.render_alpha_octave, L, 40, 40, dict(odds=True))
    torch.manual_seed(9)
    N = 2 * 16 * 16
    mu = torch.rand(1, N, 2)
    ls = torch.full((1, N, 2), math.log(math.exp(0.04) - 1.0)) + torch.rand(1, N, 2) * 0.5
    col = torch.rand(1, N, C)
    op = torch.sigmoid(torch.randn(1, N) * 2.0)
    bgv = torch.rand(1, C)
    th = (torch.rand(1, N) - 0.5) * 3.14
    L = [mu, ls, col, op, bgv, th]
    cases["octave_coarse384"] = (rt.render_alpha_octave, L, 384, 384, dict(odds=True))
    # colour-channel counts other than 3 (the reference takes any C; the encoder uses 3) and TILE 16 on
    # the octave path
    L = leaves(31, 2, 400, 1, 2.0, 0.9)
    cases["octave_c1_odds"] = (rt.render_alpha_octave, L, 64, 48, dict(odds=True))
    L = leaves(37, 1, 300, 2, 2.2)
    cases["cull_c2_alpha_noth"] = (rt.render_alpha_full_triton, L[:5] + [None], 40, 56, dict(cull=True))
    L = leaves(41, 2, 500, C, 2.0, 0.9)
    cases["octave_tile16_odds"] = (rt.render_alpha_octave, L, 96, 80, dict(odds=True, TILE=16))
    L = leaves(43, 1, 400, 5, 2.0, 0.9)
    cases["octave_c5_odds"] = (rt.render_alpha_octave, L, 48, 64, dict(odds=True))
    return cases


def make_render(names):
    allc = case_render()
    for name, (fn, L, H, W, kw) in allc.items():
        if names and name not in names:
            continue
        t0 = time.time()
        rec = run_render(fn, L, H, W, **kw)
        kwn = {f"kw_{k}": (v if v is not None else -1) for k, v in kw.items()}
        np.savez_compressed(HERE / f"render_{name}.npz", fn=fn.__name__, **kwn, **rec)
        print(f"render_{name}: {time.time() - t0:.1f}s", flush=True)


def make_tiles(names):
    """Binning fixtures: the reference's _build_tiles CSR, canonicalised."""
    if names and "tiles" not in names:
        return
    t0 = time.time()
    # small: full id lists, TILE 8 and 16, cutoffs 3 and 5
    torch.manual_seed(2)
    mu = torch.rand(1, 1024, 2)
    sc = rt.activate_scale(torch.rand(1, 1024, 2) - 2.5)
    rec = {"in_mu": mu.numpy(), "in_scale": sc.numpy()}
    for TILE, cutoff, H, W in ((8, 3.0, 64, 64), (16, 5.0, 64, 64), (8, 3.0, 50, 37)):
        gid, st, ntx, nt = rt._build_tiles(mu, sc, H, W, TILE, cutoff)
        g, s = canonical_tiles(gid[0], st[0])
        key = f"T{TILE}_c{int(cutoff)}_{H}x{W}"
        rec[f"{key}_gid"] = g
        rec[f"{key}_starts"] = s
    # edge: off-image / huge / tiny splats -> clamped tile rectangles
    torch.manual_seed(5)
    mu2 = torch.rand(1, 300, 2) * 1.4 - 0.2
    sc2 = rt.activate_scale(torch.randn(1, 300, 2) * 1.5 - 4.0)
    rec["in_mu_edge"] = mu2.numpy()
    rec["in_scale_edge"] = sc2.numpy()
    gid, st, ntx, nt = rt._build_tiles(mu2, sc2, 50, 37, 8, 3.0)
    g, s = canonical_tiles(gid[0], st[0])
    rec["edge_gid"] = g
    rec["edge_starts"] = s
    np.savez_compressed(HERE / "tiles_small.npz", **rec)
    # config 1 at full size: octave routing + per-octave CSR digests
    d = synth.synth_splats_cfg1()
    sc = rt.activate_scale(d["log_scale"])
    H = W = 768
    scale_px = sc.amax(-1) * float(min(H, W))
    octv = rt._octave_of(scale_px, 8.0, 6)[0]
    rec = {"oct": octv.numpy().astype(np.int8)}
    for o in range(7):
        idx = (octv == o).nonzero(as_tuple=True)[0]
        if idx.numel() == 0:
            continue
        Ho, Wo = max(8, H >> o), max(8, W >> o)
        gid, st, ntx, nt = rt._build_tiles(d["mu"][:, idx], sc[:, idx], Ho, Wo, 8, 3.0)
        # ids are LOCAL to the octave subset (the reference gathers the subset with nonzero())
        g, s = canonical_tiles(gid[0], st[0])
        rec[f"o{o}_starts"] = s
        rec[f"o{o}_hash"] = tile_hash(g, s)
    # the single-resolution cull binning of the whole set at 768^2
    gid, st, ntx, nt = rt._build_tiles(d["mu"], sc, H, W, 8, 3.0)
    g, s = canonical_tiles(gid[0], st[0])
    rec["cull_starts"] = s
    rec["cull_hash"] = tile_hash(g, s)
    np.savez_compressed(HERE / "tiles_cfg1.npz", **rec)
    print(f"tiles: {time.time() - t0:.1f}s", flush=True)


def _param_digest(model):
    """Per-parameter (sum, sum of squares, first value) so a re-implementation can prove its
    random init matches without the fixture holding 833k floats."""
    return {f"p_{k}": np.array([v.double().sum().item(), v.double().square().sum().item(),
                                v.flatten()[0].item()]) for k, v in model.state_dict().items()}


def make_encoder(names):
    """Encoder fixtures: the golden checkpoint on a 64^2 card, and config 0 (random init, seed 0) on
    the 128^2 card followed by the octave odds render and the backward of an L2 loss."""
    import inspect

    from gaussian_splat_encoder.efficient_encoder import EfficientGaussianEncoder

    ck = torch.load(REF / "weights" / "encoder_golden_d256.pt", map_location="cpu", weights_only=True)
    cfg = dict(ck["cfg"]["encoder"])
    accepted = set(inspect.signature(EfficientGaussianEncoder.__init__).parameters) - {"self"}
    cfg = {k: v for k, v in cfg.items() if k in accepted}
    keys = ("mu", "log_scale", "color", "opacity", "theta", "bg", "backbone_features")
    if not names or "encoder_golden" in names:
        t0 = time.time()
        enc = EfficientGaussianEncoder(**cfg)
        enc.load_state_dict(ck["model"], strict=True)
        enc.eval()
        x = synth.synth_card(64, 64, 12, 6, seed=21)
        with torch.no_grad():
            out = enc(x)
        rec = {"image": x.numpy(), "n_coarse": out["n_coarse"]}
        rec.update({k: out[k].numpy() for k in keys})
        np.savez_compressed(HERE / "encoder_golden64.npz", **rec)
        print(f"encoder_golden64: {time.time() - t0:.1f}s", flush=True)
    if not names or "encoder_cfg0" in names:
        t0 = time.time()
        torch.manual_seed(0)
        enc = EfficientGaussianEncoder(**cfg)
        enc.eval()
        x = synth.card_for_config(0)
        with torch.no_grad():
            out = enc(x)
        rec = {"image": x.numpy(), "n_coarse": out["n_coarse"]}
        rec.update({k: out[k].numpy() for k in keys})
        rec.update(_param_digest(enc))
        L = [out["mu"], out["log_scale"], out["color"], out["opacity"], out["bg"], out["theta"]]
        Lr = [t.detach().clone().requires_grad_(True) for t in L]
        img = rt.render_alpha_octave(*Lr[:5], 128, 128, theta=Lr[5], odds=True)
        loss = (img - x).square().mean()
        loss.backward()
        rec["render"] = img.detach().numpy()
        rec["loss"] = loss.item()
        for n, t in zip(NAMES, Lr):
            rec[f"grad_{n}"] = t.grad.numpy()
        np.savez_compressed(HERE / "encoder_cfg0.npz", **rec)
        print(f"encoder_cfg0: {time.time() - t0:.1f}s", flush=True)


def make_points(names):
    """render_alpha_subsampled (render.py:68-87) at seeded pixel lists (duplicates included, as
    torch.randint draws them), with and without theta, one batch holding opacity-1 splats (the
    alpha clamp)."""
    if names and "points" not in names:
        return
    specs = {"points_theta": (31, 2, 300, 40, 56, 500, True), "points_notheta": (37, 1, 200, 33, 29, 700, False)}
    for name, (seed, B, N, H, W, P, theta) in specs.items():
        t0 = time.time()
        L = leaves(seed, B, N, 3, 2.0, 0.9, theta=theta)
        L[3][:, :5] = 1.0
        idx = torch.randint(0, H * W, (B, P), generator=torch.Generator().manual_seed(seed + 1))
        Lr = [t.detach().clone().requires_grad_(True) if t is not None else None for t in L]
        out, pidx = ref_render.render_alpha_subsampled(*Lr[:5], H, W, theta=Lr[5], pixel_indices=idx)
        gseed = 4321
        gC = upstream_grad(out.shape, gseed)
        (out * gC).sum().backward()
        rec = {f"in_{n}": t.detach().numpy() for n, t in zip(NAMES, L) if t is not None}
        rec.update({"H": H, "W": W, "gseed": gseed, "px_idx": pidx.numpy(), "out": out.detach().numpy()})
        for n, t in zip(NAMES, Lr):
            if t is not None:
                rec[f"grad_{n}"] = t.grad.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(f"{name}: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    names = set(sys.argv[1:])
    make_tiles(names)
    make_render(names)
    make_encoder(names)
    make_points(names)
