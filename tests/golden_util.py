"""Fixture loading and the comparison metrics of the reference's self-tests
(render_triton.py:1000-1015: forward max|diff|; per-leaf rel = max|diff| / max|ref|)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
# A tile's splats enter its list in the order its atomic cursor hands out slots, so two renders of the same
# inputs agree only to the float rounding of the per-tile sums (the fields are order-independent sums, and
# the reference's own per-tile order comes from an unstable argsort): the absolute tolerance of
# render-against-render checks.
REORDER_TOL = 1e-5
LEAVES = ("mu", "log_scale", "color", "opacity", "bg", "theta")


def render_cases():
    return sorted(p.stem[len("render_"):] for p in GOLDEN.glob("render_*.npz"))


def load_render(name):
    d = np.load(GOLDEN / f"render_{name}.npz", allow_pickle=False)
    kw = {k[3:]: d[k].item() for k in d.files if k.startswith("kw_")}
    if kw.get("n_coarse", 0) == -1:
        kw["n_coarse"] = None
    fn = str(d["fn"])
    if fn == "render_alpha_full":
        kw.pop("chunk_pixels", None)
        fn = "render_alpha_full_triton"
    ins = {n: d[f"in_{n}"] for n in LEAVES if f"in_{n}" in d.files}
    gC = torch.randn(d["out"].shape, generator=torch.Generator().manual_seed(int(d["gseed"]))).numpy()
    ref_grads = {n: d[f"grad_{n}"] for n in LEAVES if f"grad_{n}" in d.files}
    return dict(fn=fn, kw=kw, H=int(d["H"]), W=int(d["W"]), ins=ins, gC=gC, out=d["out"], grads=ref_grads)


def grad_rel(ours: dict, ref: dict):
    """Per-leaf relative error max|d| / max|ref|.  The denominator is floored at 1e-4 x the largest
    leaf gradient: on isotropic splats the reference's theta gradient is pure rounding noise (~1e-7)."""
    scale = max(float(np.abs(v).max()) for v in ref.values() if v.size)
    out = {}
    for n, r in ref.items():
        o = ours[n]
        den = max(float(np.abs(r).max()), 1e-4 * scale, 1e-30)
        out[n] = float(np.abs(np.asarray(o) - r).max()) / den if r.size else 0.0
    return out


def fnv_tile_hash(gid_sorted: np.ndarray, starts: np.ndarray) -> np.ndarray:
    """Vectorised form of tests/golden/make_golden.py:tile_hash (per tile, ids ascending, FNV-style)."""
    starts = starts.astype(np.int64)
    nt = starts.shape[0] - 1
    lens = np.diff(starts)
    g = gid_sorted.astype(np.uint64)
    # sort within each tile
    tile_of = np.repeat(np.arange(nt), lens)
    order = np.lexsort((g, tile_of))
    g = g[order]
    out = np.full(nt, np.uint64(1469598103934665603))
    with np.errstate(over="ignore"):
        for k in range(int(lens.max()) if nt else 0):
            m = lens > k
            idx = starts[:-1][m] + k
            out[m] = (out[m] ^ g[idx]) * np.uint64(1099511628211)
    out[lens == 0] = 0
    return out
