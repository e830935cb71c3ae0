"""The render entry point keeps the reference's pair budget through the C ABI (render_triton.py:378-385:
_build_tiles raises PairBudgetExceeded instead of allocating) and never returns a truncated render:
an over-budget descriptor returns GS_ERR_PAIR_BUDGET, a pair capacity below the real pair count returns
GS_ERR_WORKSPACE, and an exact budget / capacity renders exactly what the default call renders."""

import ctypes as C

import pytest
import torch

from golden_util import REORDER_TOL

pytestmark = pytest.mark.gpu

KEYS = ("mu", "log_scale", "color", "opacity", "bg", "theta")
H = W = 768
N = 92160


@pytest.fixture(scope="module")
def cfg1():
    from gaussian_2d_splat_encoder_b200 import synth

    s = synth.synth_splats_cfg1(N=N, H=H, W=W, seed=1)
    return [s[k].cuda().contiguous() for k in KEYS]


def _desc(max_pairs=48_000_000, capacity=0):
    from gaussian_2d_splat_encoder_b200 import _lib
    from gaussian_2d_splat_encoder_b200.render_triton import _desc as mk

    return mk(mode=_lib.MODE_OCTAVE, B=1, N=N, C=3, H=H, W=W, TILE=8, odds=True, has_theta=True, cutoff=3.0,
              base_texels=8.0, max_octaves=6, max_pairs=max_pairs, capacity=capacity)


def _fwd(lib, d, ins):
    from gaussian_2d_splat_encoder_b200 import _lib

    nb = lib.gs_render_workspace_size(C.byref(d), 0)
    assert nb > 0
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.full((1, 3, H, W), float("nan"), device="cuda")
    st = lib.gs_render_fwd(C.byref(d), *[_lib.ptr(t) for t in ins], _lib.ptr(out), _lib.ptr(ws), nb,
                           _lib.stream_of(torch.device("cuda")))
    torch.cuda.synchronize()
    return st, out


def _counts(lib, ins):
    from gaussian_2d_splat_encoder_b200 import _lib

    d = _desc(capacity=1)
    ws = torch.empty(lib.gs_render_workspace_size(C.byref(d), 0), dtype=torch.uint8, device="cuda")
    counts = (C.c_int64 * 7)()
    ng = C.c_int32(0)
    assert lib.gs_render_count(C.byref(d), _lib.ptr(ins[0]), _lib.ptr(ins[1]), _lib.ptr(ws), ws.numel(), counts,
                               C.byref(ng), _lib.stream_of(torch.device("cuda"))) == 0
    return list(counts)[:ng.value]


def test_over_budget_refused(lib, cfg1):
    from gaussian_2d_splat_encoder_b200 import _lib

    counts = _counts(lib, cfg1)
    worst = max(counts)
    st, _ = _fwd(lib, _desc(max_pairs=worst - 1), cfg1)
    assert st == _lib.GS_ERR_PAIR_BUDGET
    assert b"budget" in lib.gs_last_error()
    st, out = _fwd(lib, _desc(max_pairs=worst), cfg1)      # the budget exactly met renders
    assert st == 0
    st, ref = _fwd(lib, _desc(), cfg1)
    assert st == 0 and torch.allclose(out, ref, atol=REORDER_TOL, rtol=0)


def test_undersized_pair_capacity_refused(lib, cfg1):
    from gaussian_2d_splat_encoder_b200 import _lib

    total = sum(_counts(lib, cfg1))
    for cap in (1000, total - 1):
        st, _ = _fwd(lib, _desc(capacity=cap), cfg1)
        assert st == _lib.GS_ERR_WORKSPACE, cap
    st, out = _fwd(lib, _desc(capacity=total), cfg1)      # exactly enough capacity
    assert st == 0
    st, ref = _fwd(lib, _desc(), cfg1)
    assert st == 0 and torch.allclose(out, ref, atol=REORDER_TOL, rtol=0)


def test_python_budget_raises(lib, cfg1):
    from gaussian_2d_splat_encoder_b200.render_triton import PairBudgetExceeded, render_alpha_octave

    mu, ls, col, op, bg, th = cfg1
    with pytest.raises(PairBudgetExceeded):
        render_alpha_octave(mu, ls, col, op, bg, H, W, theta=th, odds=True, max_pairs=1000)
