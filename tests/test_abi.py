"""The C-ABI library loads and exports every entry point include/gsplat_b200.h declares; the host-only
queries (bounds, workspace sizes) answer without touching a GPU."""

import ctypes as C
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared(header="gsplat_b200.h"):
    txt = (ROOT / "include" / header).read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return set(re.findall(r"\b(gs_[a-z0-9_]+)\s*\(", txt))


def test_header_symbols_exported(lib):
    from gaussian_2d_splat_encoder_b200 import _lib

    names = declared()
    assert names, "no declarations parsed"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (gs_\w+)", out))
    missing = names - exported
    assert not missing, f"declared but not exported: {missing}"
    for n in names:
        assert hasattr(lib, n)
    assert names <= set(_lib.SIGNATURES), "python binding misses a declared entry point"


def test_build_arch(lib):
    assert lib.gs_build_arch() == 100


def _desc(**kw):
    from gaussian_2d_splat_encoder_b200.render_triton import _desc as mk

    return mk(**kw)


def test_pair_bound_and_workspace_host_only(lib):
    from gaussian_2d_splat_encoder_b200 import _lib

    d = _desc(mode=_lib.MODE_OCTAVE, B=1, N=92160, C=3, H=768, W=768, TILE=8, odds=True, has_theta=True,
              cutoff=3.0, base_texels=8.0, max_octaves=6, max_pairs=48_000_000)
    bound = lib.gs_render_pair_bound(C.byref(d))
    # octaves 0..5: sigma <= 8 texels -> bbox <= 8 x 8 tiles; octave 6 at 12x12 px -> 2 x 2 tiles
    assert bound == 64 * 92160
    ws_f = lib.gs_render_workspace_size(C.byref(d), 0)
    ws_b = lib.gs_render_workspace_size(C.byref(d), 1)
    assert 0 < ws_f < ws_b < (1 << 31)
    d.pair_capacity = (1 << 31) - 1  # the largest capacity 32-bit pair positions address
    assert lib.gs_render_workspace_size(C.byref(d), 0) > 0
    d.pair_capacity = 1 << 31
    assert lib.gs_render_workspace_size(C.byref(d), 0) == 0
    d.pair_capacity = 0
    d.tile = 5
    assert lib.gs_render_workspace_size(C.byref(d), 0) == 0
    assert lib.gs_render_pair_bound(C.byref(d)) == -1


def test_bad_arguments_rejected_without_gpu(lib):
    from gaussian_2d_splat_encoder_b200 import _lib

    d = _desc(mode=_lib.MODE_EXACT, B=1, N=4, C=3, H=8, W=8, TILE=8, odds=True, has_theta=False, cutoff=3.0)
    assert lib.gs_render_fwd(C.byref(d), *([None] * 8), 0, None) == _lib.GS_ERR_BAD_ARGUMENT
    assert lib.gs_activate_scale(None, None, 4, None) == _lib.GS_ERR_BAD_ARGUMENT


def test_no_cpu_fallback():
    """CPU tensors are refused loudly; the product has no CPU or Triton path."""
    import pytest
    import torch

    from gaussian_2d_splat_encoder_b200 import render_triton as rt

    t = torch.zeros(1, 4, 2)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        rt.render_alpha_octave(t, t, torch.zeros(1, 4, 3), torch.zeros(1, 4), torch.zeros(1, 3), 16, 16)


def test_points_workspace_host_only(lib):
    """gs_render_points_workspace_size: positive for the pixel-list render's exact mode, with backward
    larger than forward; 0 for the octave/odds modes it does not serve and for an empty pixel list."""
    from gaussian_2d_splat_encoder_b200 import _lib

    d = _desc(mode=_lib.MODE_EXACT, B=2, N=4096, C=3, H=256, W=256, TILE=8, odds=False, has_theta=True,
              cutoff=3.0)
    f = lib.gs_render_points_workspace_size(C.byref(d), 10000, 0)
    b = lib.gs_render_points_workspace_size(C.byref(d), 10000, 1)
    # splat records + per-slice partial sums of 5 fields for every (image, pixel)
    assert 2 * 10000 * 5 * 4 * 2 < f < b < (1 << 28)
    assert lib.gs_render_points_workspace_size(C.byref(d), 0, 0) == 0
    d.odds = 1
    assert lib.gs_render_points_workspace_size(C.byref(d), 10000, 0) == 0
    d.odds, d.mode = 0, _lib.MODE_OCTAVE
    assert lib.gs_render_points_workspace_size(C.byref(d), 10000, 0) == 0


def test_encode_render_workspace_host_only(lib):
    """The fused encode+render workspace is the encoder's plus a render's; unsupported image sizes give 0."""
    import torch
    from enc_util import GOLDEN_CFG
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    torch.manual_seed(0)
    m = EfficientGaussianEncoder(**GOLDEN_CFG)
    d = m._desc(1, 256, 256)
    enc = lib.gs_encoder_workspace_size(C.byref(d))
    both = lib.gs_encode_render_workspace_size(C.byref(d))
    assert 0 < enc < both < (1 << 32)
    d.H = 250
    assert lib.gs_encoder_workspace_size(C.byref(d)) == 0
    assert lib.gs_encode_render_workspace_size(C.byref(d)) == 0


def test_plain_c_consumer(lib, tmp_path):
    """A C99 program that includes only include/gsplat_b200.h and links libgsplat_b200.so gets the same
    host-side answers as the Python binding (the boundary needs no torch and no C++)."""
    import shutil

    from gaussian_2d_splat_encoder_b200 import _lib

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        import pytest

        pytest.skip("no C compiler")
    exe = tmp_path / "consumer"
    libdir = str(_lib.LIB_PATH.parent)
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_abi_consumer.c"), "-o", str(exe), "-L", libdir,
                    f"-l:{_lib.LIB_PATH.name}", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    got = dict(kv.split("=") for kv in out.split())
    assert got["arch"] == "100" and int(got["bound"]) == 64 * 92160
    assert 0 < int(got["ws_fwd"]) < int(got["ws_bwd"])
    assert int(got["bad_args"]) == _lib.GS_ERR_BAD_ARGUMENT and got["ws_bad_tile"] == "0"


def test_host_queries_fuzz(lib):
    """Random descriptors (valid and invalid): the host-only queries never fault, a valid descriptor gets a
    forward workspace no larger than the forward+backward one, and an invalid one gets 0 / -1."""
    import numpy as np

    from gaussian_2d_splat_encoder_b200 import _lib

    rng = np.random.default_rng(0)
    for _ in range(400):
        mode = int(rng.integers(-1, 5))
        kw = dict(mode=mode, B=int(rng.integers(0, 5)), N=int(rng.integers(-2, 5000)), C=int(rng.integers(0, 5)),
                  H=int(rng.integers(0, 700)), W=int(rng.integers(0, 700)), TILE=int(rng.choice([3, 4, 8, 16, 32])),
                  odds=bool(rng.integers(0, 2)), has_theta=bool(rng.integers(0, 2)),
                  cutoff=float(rng.choice([0.0, 3.0, 5.0])))
        d = _desc(**kw)
        d.max_octaves = int(rng.integers(-1, 9))
        valid = (0 <= mode <= 3 and kw["B"] >= 1 and kw["N"] >= 0 and 1 <= kw["C"] <= 3 and kw["H"] >= 1
                 and kw["W"] >= 1 and kw["TILE"] in (4, 8, 16) and kw["cutoff"] > 0
                 and not (mode == _lib.MODE_EXACT and kw["odds"])
                 and not (mode == _lib.MODE_OCTAVE and not 0 <= d.max_octaves <= 7))
        f = lib.gs_render_workspace_size(C.byref(d), 0)
        b = lib.gs_render_workspace_size(C.byref(d), 1)
        bound = lib.gs_render_pair_bound(C.byref(d))
        if valid:
            assert 0 < f <= b, kw
            assert bound >= 0, kw
        else:
            assert f == 0 and b == 0, kw
