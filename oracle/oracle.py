"""TEST INFRASTRUCTURE ONLY: numpy front end of the C oracle (oracle/gsplat_oracle.c).

The oracle is the CPU restatement of the reference renderer (bigwolfeman/gaussian-2d-splat-encoder,
gaussian_splat_encoder/render_triton.py and render.py) that the parity tests, ``smoke()`` and the CPU
baseline of ``bench.py`` use as the checker.  The product package never imports this module.

Every function takes and returns numpy float32 arrays in the reference's layouts (mu [B,N,2] as (y,x),
log_scale [B,N,2] pre-softplus, color [B,N,C], opacity [B,N], bg [B,C], theta [B,N] or None, images
[B,C,H,W]).  Passing ``grad_out`` ([B,C,H,W]) also runs the backward of sum(out * grad_out) and returns
the gradients of the six leaves, matching what the reference's autograd returns.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libgsplat_oracle.so"

_lib = None


class OracleBudgetExceeded(RuntimeError):
    """The oracle's counterpart of the reference's PairBudgetExceeded (render_triton.py:51-54)."""


def build() -> Path:
    """Compile the oracle with its Makefile (gcc); returns the library path."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = C.CDLL(str(LIB))
        f = C.c_float
        i = C.c_int
        p = C.c_void_p
        L = C.c_long
        _lib.orc_render_octave.argtypes = [i, i, i, p, p, p, p, p, p, i, i, f, i, f, i, L, i, p, p, p, p, p, p, p, p]
        _lib.orc_render_octave_l2.argtypes = [i, i, i, p, p, p, p, p, p, i, i, f, i, f, i, L, i, p, f, p, p, p,
                                              p, p, p, p, p, p]
        _lib.orc_render_multires.argtypes = [i, i, i, p, p, p, p, p, p, i, i, i, i, f, i, L, i, p, p, p, p, p, p, p, p]
        _lib.orc_render_cull.argtypes = [i, i, i, p, p, p, p, p, p, i, i, i, f, i, p, p, p, p, p, p, p, p]
        _lib.orc_render_exact.argtypes = [i, i, i, p, p, p, p, p, p, i, i, p, p, p, p, p, p, p, p]
        _lib.orc_bin_octave.argtypes = [i, p, p, i, i, f, i, f, i, p, p, p, p, p]
        _lib.orc_bin_octave.restype = L
        _lib.orc_count_pairs.restype = L
        _lib.orc_activate_scale.argtypes = [p, p, L]
        _lib.orc_octave_of.argtypes = [f, f, f, f, i]
        _lib.orc_octave_of.restype = i
        _lib.orc_set_threads.argtypes = [i]
        _lib.orc_num_threads.restype = i
    return _lib


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def _f32(a):
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def activate_scale(log_scale):
    ls = _f32(log_scale)
    out = np.empty_like(ls)
    lib().orc_activate_scale(_ptr(ls), _ptr(out), ls.size)
    return out


def _run(kind, mu, log_scale, color, opacity, bg, H, W, theta, grad_out, extra):
    mu, ls, col, op, bg, th = map(_f32, (mu, log_scale, color, opacity, bg, theta))
    B, N, Cc = col.shape
    out = np.empty((B, Cc, H, W), np.float32)
    g = _f32(grad_out)
    grads = None
    if g is not None:
        grads = dict(mu=np.empty_like(mu), log_scale=np.empty_like(ls), color=np.empty_like(col),
                     opacity=np.empty_like(op), bg=np.empty_like(bg),
                     theta=np.empty_like(th) if th is not None else None)
    gp = [_ptr(grads[k]) if grads is not None and grads[k] is not None else None
          for k in ("mu", "log_scale", "color", "opacity", "bg", "theta")]
    head = [B, N, Cc, _ptr(mu), _ptr(ls), _ptr(col), _ptr(op), _ptr(bg), _ptr(th), H, W]
    fn = getattr(lib(), f"orc_render_{kind}")
    st = fn(*head, *extra, _ptr(out), _ptr(g), *gp)
    if st == 1:
        raise OracleBudgetExceeded(f"oracle: a (tile, splat) pair count exceeds max_pairs @ {H}x{W}")
    return (out, grads) if g is not None else out


def render_alpha_octave(mu, log_scale, color, opacity, bg, H, W, theta=None, cutoff=3.0, TILE=8,
                        base_texels=8.0, max_octaves=6, max_pairs=48_000_000, odds=False, grad_out=None):
    """render_triton.py:935-980."""
    mp = -1 if max_pairs is None else int(max_pairs)
    return _run("octave", mu, log_scale, color, opacity, bg, H, W, theta, grad_out,
                [float(cutoff), int(TILE), float(base_texels), int(max_octaves), mp, int(bool(odds))])


def render_alpha_octave_l2(mu, log_scale, color, opacity, bg, H, W, target, theta=None, scale=None, cutoff=3.0,
                           TILE=8, base_texels=8.0, max_octaves=6, max_pairs=48_000_000, odds=False):
    """One fitting step's render: render_alpha_octave forward (render_triton.py:935-980), the loss
    scale * sum (out - target)^2 (scale defaults to 1/out.size: mse_loss) and the backward of that loss,
    with the forward run once.  Returns (out, loss, grad_out, grads)."""
    mu, ls, col, op, bg, th, tg = map(_f32, (mu, log_scale, color, opacity, bg, theta, target))
    B, N, Cc = col.shape
    out = np.empty((B, Cc, H, W), np.float32)
    if tg.shape != out.shape:
        raise ValueError(f"target shape {tg.shape} != {out.shape}")
    g = np.empty_like(out)
    sc = np.float32(1.0 / out.size if scale is None else scale)
    grads = dict(mu=np.empty_like(mu), log_scale=np.empty_like(ls), color=np.empty_like(col),
                 opacity=np.empty_like(op), bg=np.empty_like(bg), theta=np.empty_like(th) if th is not None else None)
    loss = C.c_double(0.0)
    mp = -1 if max_pairs is None else int(max_pairs)
    st = lib().orc_render_octave_l2(B, N, Cc, _ptr(mu), _ptr(ls), _ptr(col), _ptr(op), _ptr(bg), _ptr(th), H, W,
                                    float(cutoff), int(TILE), float(base_texels), int(max_octaves), mp,
                                    int(bool(odds)), _ptr(tg), float(sc), _ptr(out), _ptr(g), C.byref(loss),
                                    *[_ptr(grads[k]) for k in ("mu", "log_scale", "color", "opacity", "bg", "theta")])
    if st == 1:
        raise OracleBudgetExceeded(f"oracle: a (tile, splat) pair count exceeds max_pairs @ {H}x{W}")
    return out, float(loss.value), g, grads


def render_alpha_multires(mu, log_scale, color, opacity, bg, H, W, theta=None, n_coarse=None,
                          coarse_factor=8, cutoff=3.0, TILE=8, max_pairs=48_000_000, odds=False, grad_out=None):
    """render_triton.py:879-922."""
    nc = -1 if n_coarse is None else int(n_coarse)
    mp = -1 if max_pairs is None else int(max_pairs)
    return _run("multires", mu, log_scale, color, opacity, bg, H, W, theta, grad_out,
                [nc, int(coarse_factor), float(cutoff), int(TILE), mp, int(bool(odds))])


def render_alpha_full_triton(mu, log_scale, color, opacity, bg, H, W, theta=None, cull=False, TILE=8,
                             cutoff=3.0, odds=False, grad_out=None):
    """render_triton.py:326-347 (cull=True: tile-binned; cull=False: exact, alpha mode only)."""
    if cull:
        return _run("cull", mu, log_scale, color, opacity, bg, H, W, theta, grad_out,
                    [int(TILE), float(cutoff), int(bool(odds))])
    if odds:
        raise NotImplementedError("odds compositing is only wired through the cull/octave path")
    return _run("exact", mu, log_scale, color, opacity, bg, H, W, theta, grad_out, [])


def octave_of(scale_yx, H, W, base_texels=8.0, max_octaves=6):
    sc = _f32(scale_yx).reshape(-1, 2)
    rep = float(min(H, W))
    return np.array([lib().orc_octave_of(float(a), float(b), rep, float(base_texels), int(max_octaves))
                     for a, b in sc], dtype=np.int32)


def bin_octave(mu, scale, H, W, cutoff=3.0, TILE=8, base_texels=8.0, max_octaves=6):
    """One image's octave routing and per-octave tile CSR (ids are global splat ids, ascending inside a
    tile).  Returns (oct [N], [(starts_o, gid_o) for each octave o])."""
    mu = _f32(mu).reshape(-1, 2)
    sc = _f32(scale).reshape(-1, 2)
    N = mu.shape[0]
    oct_ = np.empty(N, np.int32)
    soff = np.zeros(max_octaves + 2, np.int64)
    goff = np.zeros(max_octaves + 2, np.int64)
    L = lib()
    args = [N, _ptr(mu), _ptr(sc), H, W, float(cutoff), int(TILE), float(base_texels), int(max_octaves),
            _ptr(oct_), _ptr(soff), _ptr(goff)]
    tot = L.orc_bin_octave(*args, None, None)
    starts = np.empty(int(soff[-1]), np.int32)
    gid = np.empty(max(int(tot), 1), np.int32)
    L.orc_bin_octave(*args, _ptr(starts), _ptr(gid))
    per = []
    for o in range(max_octaves + 1):
        per.append((starts[soff[o]:soff[o + 1]], gid[goff[o]:goff[o + 1]]))
    return oct_, per


def build_tiles(mu, scale, H, W, TILE=8, cutoff=3.0):
    """_build_tiles (render_triton.py:351-409) for one group: (starts [nt+1], gid [pairs])."""
    oct_, per = bin_octave(mu, scale, H, W, cutoff, TILE, base_texels=1e30, max_octaves=0)
    return per[0]


if os.environ.get("GSPLAT_ORACLE_THREADS"):
    set_threads(int(os.environ["GSPLAT_ORACLE_THREADS"]))
