"""ctypes binding of libgsplat_b200.so (the C ABI declared in include/gsplat_b200.h).

The library is built in-tree by ``gaussian_2d_splat_encoder_b200.build`` (nvcc, sm_100a).  There is no
fallback: if the library is missing or no CUDA device is present, every entry point raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("GSPLAT_B200_LIB", PKG / "libgsplat_b200.so"))

GS_OK = 0
GS_ERR_PAIR_BUDGET = 1
GS_ERR_BAD_ARGUMENT = 2
GS_ERR_TIMEOUT = 3
GS_ERR_CUDA = 4
GS_ERR_WORKSPACE = 5

MODE_OCTAVE, MODE_CULL, MODE_MULTIRES, MODE_EXACT = 0, 1, 2, 3


class GsRenderDesc(C.Structure):
    """Mirror of gs_render_desc."""

    _fields_ = [("mode", C.c_int32), ("B", C.c_int32), ("N", C.c_int32), ("C", C.c_int32),
                ("H", C.c_int32), ("W", C.c_int32), ("tile", C.c_int32), ("odds", C.c_int32),
                ("has_theta", C.c_int32), ("max_octaves", C.c_int32), ("n_coarse", C.c_int32),
                ("coarse_factor", C.c_int32), ("cutoff", C.c_float), ("base_texels", C.c_float),
                ("max_pairs", C.c_int64), ("pair_capacity", C.c_int64), ("row_begin", C.c_int32),
                ("row_end", C.c_int32)]


# every exported symbol of include/gsplat_b200.h, with its ctypes signature
_P = C.c_void_p
_DESC = C.POINTER(GsRenderDesc)
SIGNATURES = {
    "gs_render_pair_bound": (C.c_int64, [_DESC]),
    "gs_render_workspace_size": (C.c_size_t, [_DESC, C.c_int]),
    "gs_render_count": (C.c_int, [_DESC, _P, _P, _P, C.c_size_t, _P, _P, _P]),
    "gs_render_fwd": (C.c_int, [_DESC, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "gs_render_fwd_noalloc": (C.c_int, [_DESC, _P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_render_bwd": (C.c_int, [_DESC, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "gs_render_points_workspace_size": (C.c_size_t, [_DESC, C.c_int32, C.c_int]),
    "gs_render_points_fwd": (C.c_int, [_DESC, C.c_int32, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "gs_render_points_bwd": (C.c_int, [_DESC, C.c_int32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       C.c_size_t, _P]),
    "gs_render_debug_bins": (C.c_int, [_DESC, _P, _P, _P, _P, _P, _P, _P]),
    "gs_activate_scale": (C.c_int, [_P, _P, C.c_int64, _P]),
    "gs_l2_loss_grad": (C.c_int, [_P, _P, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_float, _P, _P,
                                  _P]),
    "gs_conv2d": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P]),
    "gs_encoder_workspace_size": (C.c_size_t, [_P]),
    "gs_encoder_fwd": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "gs_encoder_error_flag": (C.c_int, [_P, _P, _P]),
    "gs_encode_render_debug_pairs": (C.c_int, [_P, _P, _P]),
    "gs_encode_render_workspace_size": (C.c_size_t, [_P]),
    "gs_encode_render_fwd": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "gs_last_error": (C.c_char_p, []),
    "gs_kernel_launches": (C.c_uint64, []),
    "gs_profile_enable": (None, [C.c_int]),
    "gs_profile_collect": (C.c_int, [_P, _P]),
    "gs_profile_collect2": (C.c_int, [_P, _P, C.c_int]),
    "gs_build_arch": (C.c_int, []),
}

_lib = None


def load(path: Path | None = None):
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p.name} is not built ({p}); run gaussian_2d_splat_encoder_b200.build.build() "
                           "(nvcc, sm_100a). There is no CPU or Triton fallback.")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_of(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(status: int, what: str = "") -> None:
    if status == GS_OK:
        return
    msg = load().gs_last_error().decode(errors="replace")
    if status == GS_ERR_PAIR_BUDGET:
        from .render_triton import PairBudgetExceeded
        raise PairBudgetExceeded(f"{what}: pair budget exceeded {msg}")
    if status == GS_ERR_BAD_ARGUMENT:
        raise ValueError(f"{what}: invalid argument")
    if status == GS_ERR_WORKSPACE:
        raise RuntimeError(f"{what}: workspace too small")
    if status == GS_ERR_TIMEOUT:
        raise RuntimeError(f"{what}: device wait timed out")
    raise RuntimeError(f"{what}: CUDA error: {msg}")


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("gaussian_2d_splat_encoder_b200 kernels run on CUDA tensors only "
                               f"(got a tensor on {t.device}); there is no CPU fallback")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("all tensors must be on the same CUDA device")
    return dev
