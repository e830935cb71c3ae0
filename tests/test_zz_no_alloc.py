"""gs_render_fwd_noalloc: the forward render for callers that cannot allocate device memory (for example
a host whose device memory is owned by an allocator it cannot call, or a latency-critical path that must
not pay for cudaMalloc).  It uses a fixed scratch array inside the library instead of a caller workspace.

Checked through the C ABI against gs_render_fwd with a caller workspace, on two calls in a row (the
shared array keeps the previous call's contents, so the second call must not depend on them), and the
refusal of a render too large for the array.  Kept in a file that pytest collects last."""

import ctypes as C

import pytest
import torch

from golden_util import REORDER_TOL

pytestmark = pytest.mark.gpu

KEYS = ("mu", "log_scale", "color", "opacity", "bg", "theta")


def _inputs(N, H, W, seed):
    from gaussian_2d_splat_encoder_b200 import synth

    s = synth.synth_splats_cfg1(N=N, H=H, W=W, seed=seed)
    return [s[k].cuda().contiguous() for k in KEYS]


def _desc(N, H, W, capacity=0):
    from gaussian_2d_splat_encoder_b200 import _lib
    from gaussian_2d_splat_encoder_b200.render_triton import _desc as mk

    return mk(mode=_lib.MODE_OCTAVE, B=1, N=N, C=3, H=H, W=W, TILE=8, odds=True, has_theta=True, cutoff=3.0,
              base_texels=8.0, max_octaves=6, max_pairs=48_000_000, capacity=capacity)


def _with_workspace(lib, d, ins, H, W):
    from gaussian_2d_splat_encoder_b200 import _lib

    nb = lib.gs_render_workspace_size(C.byref(d), 0)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out = torch.empty(1, 3, H, W, device="cuda")
    p = _lib.ptr
    assert lib.gs_render_fwd(C.byref(d), *[p(t) for t in ins], p(out), p(ws), nb,
                             _lib.stream_of(torch.device("cuda"))) == 0
    return out


def _no_alloc(lib, d, ins, H, W):
    from gaussian_2d_splat_encoder_b200 import _lib

    out = torch.empty(1, 3, H, W, device="cuda")
    p = _lib.ptr
    st = lib.gs_render_fwd_noalloc(C.byref(d), *[p(t) for t in ins], p(out), _lib.stream_of(torch.device("cuda")))
    return st, out


def test_no_alloc_forward_matches_workspace_forward(lib):
    H = W = 256
    N = 6000
    d = _desc(N, H, W)
    assert lib.gs_render_workspace_size(C.byref(d), 0) <= (32 << 20)
    for seed in (21, 22):                      # two calls in a row, different inputs
        ins = _inputs(N, H, W, seed)
        ref = _with_workspace(lib, d, ins, H, W)
        st, got = _no_alloc(lib, d, ins, H, W)
        torch.cuda.synchronize()
        assert st == 0
        assert torch.allclose(got, ref, atol=REORDER_TOL, rtol=0), (got - ref).abs().max().item()


def test_no_alloc_smaller_render_after_larger(lib):
    """A smaller render (other size, fewer splats) right after a 256^2 one: the previous call's tile ranges
    and fields left in the shared array must not leak into it."""
    big = _desc(6000, 256, 256)
    ins = _inputs(6000, 256, 256, 23)
    st, _ = _no_alloc(lib, big, ins, 256, 256)
    assert st == 0
    H, W, N = 96, 160, 700
    d = _desc(N, H, W)
    ins = _inputs(N, H, W, 24)
    ref = _with_workspace(lib, d, ins, H, W)
    st, got = _no_alloc(lib, d, ins, H, W)
    torch.cuda.synchronize()
    assert st == 0
    assert torch.allclose(got, ref, atol=REORDER_TOL, rtol=0), (got - ref).abs().max().item()


def test_no_alloc_explicit_pair_capacity(lib):
    """An explicit pair capacity below the real pair count is refused (GS_ERR_WORKSPACE), never rendered
    with pairs dropped; a capacity that holds every pair renders like the default."""
    from gaussian_2d_splat_encoder_b200 import _lib

    H = W = 256
    N = 6000
    ins = _inputs(N, H, W, 25)
    ref = _with_workspace(lib, _desc(N, H, W), ins, H, W)
    st, _ = _no_alloc(lib, _desc(N, H, W, capacity=500), ins, H, W)
    torch.cuda.synchronize()
    assert st == _lib.GS_ERR_WORKSPACE
    st, got = _no_alloc(lib, _desc(N, H, W, capacity=64 * N), ins, H, W)
    torch.cuda.synchronize()
    assert st == 0
    assert torch.allclose(got, ref, atol=REORDER_TOL, rtol=0), (got - ref).abs().max().item()


def test_no_alloc_refuses_oversized_render(lib):
    from gaussian_2d_splat_encoder_b200 import _lib

    H = W = 768
    N = 92160
    d = _desc(N, H, W)
    assert lib.gs_render_workspace_size(C.byref(d), 0) > (32 << 20)
    ins = _inputs(N, H, W, 1)
    st, _ = _no_alloc(lib, d, ins, H, W)
    assert st == _lib.GS_ERR_WORKSPACE
