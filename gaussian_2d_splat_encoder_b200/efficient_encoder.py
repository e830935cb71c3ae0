"""EfficientGaussianEncoder on B200: the reference's module interface over the libgsplat_b200 encoder.

Drop-in for bigwolfeman/gaussian-2d-splat-encoder ``gaussian_splat_encoder/efficient_encoder.py``.  The
module keeps the reference's constructor signature, attribute names and sub-module structure, so
``load_state_dict`` accepts the released checkpoint unchanged and ``torch.manual_seed(s)`` followed by
construction yields the same random initialisation.  ``forward`` runs the whole 'adaptive' pipeline
(backbone, heads, the internal coarse render, fine decoder) in ``gs_encoder_fwd``: tcgen05 implicit-GEMM
convolutions in bf16 with fp32 accumulation, fused bias/GELU/GroupNorm statistics, and fused head
activations.  The forward is inference-only (the encoder is frozen in the reference's release): its
outputs carry no autograd history.

Supported configuration on the CUDA path: variant='adaptive', d_feature=256, stride=8, fine_stride=4,
norm_type='group', use_grad_input=True, 1-2 splats per cell, H and W multiples of 8 with
(H/4)(W/4) a multiple of 64 -- the released checkpoint's architecture.  Other configurations can be
constructed (state-dict compatible) but their forward raises NotImplementedError.
"""

from __future__ import annotations

import ctypes as C
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .render import render_alpha_full  # noqa: F401  (the reference module imports it too)
from .render_triton import render_alpha_full_triton, render_alpha_octave  # noqa: F401


def _norm(channels, norm_type):
    if norm_type == "group":
        return nn.GroupNorm(8, channels)
    if norm_type == "instance":
        return nn.InstanceNorm2d(channels, affine=True)
    if norm_type == "none":
        return nn.Identity()
    raise ValueError(f"Unknown norm_type: {norm_type}")


class _Backbone(nn.Module):
    """Three (four for stride 16) strided Conv -> GELU -> Norm stages exposing s2/s4/s8 skips
    (efficient_encoder.py:41-72).  Parameters only: the forward runs in the CUDA encoder."""

    def __init__(self, in_ch, d, norm_type, stride):
        super().__init__()
        if stride not in (8, 16):
            raise ValueError(f"stride must be 8 or 16, got {stride}")
        self.stride = stride
        self.stage_s2 = nn.Sequential(nn.Conv2d(in_ch, d // 4, 7, stride=2, padding=3), nn.GELU(),
                                      _norm(d // 4, norm_type))
        self.stage_s4 = nn.Sequential(nn.Conv2d(d // 4, d // 2, 3, stride=2, padding=1), nn.GELU(),
                                      _norm(d // 2, norm_type))
        self.stage_s8 = nn.Sequential(nn.Conv2d(d // 2, d, 3, stride=2, padding=1), nn.GELU(), _norm(d, norm_type))
        if stride == 16:
            self.stage_s16 = nn.Sequential(nn.Conv2d(d, d, 3, stride=2, padding=1), nn.GELU(), _norm(d, norm_type))


def _skip_channels(d):
    return {2: d // 4, 4: d // 2, 8: d, 16: d}


class _UpBlock(nn.Module):
    """bilinear upsample to the skip's size, concat the skip, 3x3 Conv -> GELU -> Norm
    (efficient_encoder.py:80-91)."""

    def __init__(self, in_ch, skip_ch, out_ch, norm_type):
        super().__init__()
        self.fuse = nn.Sequential(nn.Conv2d(in_ch + skip_ch, out_ch, 3, stride=1, padding=1), nn.GELU(),
                                  _norm(out_ch, norm_type))


class _FineDecoder(nn.Module):
    """U-Net decoder from the base stride down to fine_stride (efficient_encoder.py:94-120)."""

    def __init__(self, d, base_stride, fine_stride, norm_type):
        super().__init__()
        if fine_stride not in (2, 4, 8) or fine_stride > base_stride:
            raise ValueError(f"fine_stride must be in (2,4,8) and <= stride, got {fine_stride}")
        skip_ch = _skip_channels(d)
        self.blocks = nn.ModuleList()
        self.target_strides = []
        s, in_ch = base_stride, d
        while s > fine_stride:
            tgt = s // 2
            out_ch = max(d // 2, 32)
            self.blocks.append(_UpBlock(in_ch, skip_ch[tgt], out_ch, norm_type))
            self.target_strides.append(tgt)
            in_ch, s = out_ch, tgt
        self.out_ch = in_ch


class _SplatHead(nn.Module):
    """1x1 heads of M splats per cell: mu (grid + tanh offset), log_scale, colour (sigmoid), opacity
    (sigmoid, optional floor), theta (tanh * pi/2) (efficient_encoder.py:144-197)."""

    def __init__(self, in_ch, M, color_dim=3, scale_bias=-3.0, opacity_bias=2.0, offset_cells=1.0,
                 use_rotation=True, min_opacity=0.0):
        super().__init__()
        self.M, self.color_dim, self.use_rotation = M, color_dim, use_rotation
        self.offset_cells = offset_cells
        self.min_opacity = min_opacity
        self.mu_head = nn.Conv2d(in_ch, 2 * M, 1)
        self.scale_head = nn.Conv2d(in_ch, 2 * M, 1)
        self.color_head = nn.Conv2d(in_ch, color_dim * M, 1)
        self.opacity_head = nn.Conv2d(in_ch, M, 1)
        if use_rotation:
            self.theta_head = nn.Conv2d(in_ch, M, 1)
        nn.init.zeros_(self.mu_head.weight)
        nn.init.zeros_(self.mu_head.bias)
        nn.init.constant_(self.scale_head.bias, scale_bias)
        nn.init.constant_(self.opacity_head.bias, opacity_bias)

    def packed(self):
        """[9M (8M without rotation), Cin] weight rows (mu, scale, colour, opacity, theta) and biases."""
        mods = [self.mu_head, self.scale_head, self.color_head, self.opacity_head]
        if self.use_rotation:
            mods.append(self.theta_head)
        w = torch.cat([m.weight.detach().flatten(1) for m in mods], 0).float().contiguous()
        b = torch.cat([m.bias.detach() for m in mods], 0).float().contiguous()
        return w, b


def sobel_gradmag(img: torch.Tensor) -> torch.Tensor:
    """[B,3,H,W] -> [B,1,H,W] gradient magnitude sqrt(gx^2 + gy^2 + 1e-6) of the channel-mean image with
    the Sobel kernels / 4 (efficient_encoder.py:123-130).  API helper (torch ops); the encoder computes
    it inside its CUDA input-preparation kernel."""
    gray = img.mean(1, keepdim=True)
    kx = torch.tensor([[-1, 0, 1], [-2, 0, 2], [-1, 0, 1]], dtype=img.dtype, device=img.device) / 4.0
    ky = kx.t().contiguous()
    gx = F.conv2d(gray, kx.view(1, 1, 3, 3), padding=1)
    gy = F.conv2d(gray, ky.view(1, 1, 3, 3), padding=1)
    return torch.sqrt(gx * gx + gy * gy + 1e-6)


def edge_pixel_indices(images: torch.Tensor, n_px: int, lam: float) -> torch.Tensor:
    """n_px pixel indices per image drawn with probability proportional to (1-lam)*|grad I| + lam/HW
    (efficient_encoder.py:133-141)."""
    B, _, H, W = images.shape
    g = sobel_gradmag(images).float().reshape(B, -1)
    g = g / g.sum(1, keepdim=True).clamp_min(1e-8)
    pmf = (1 - lam) * g + lam / (H * W)
    return torch.multinomial(pmf, min(n_px, H * W), replacement=True)


class _GsEncoderDesc(C.Structure):
    _fields_ = [("B", C.c_int32), ("H", C.c_int32), ("W", C.c_int32), ("d", C.c_int32), ("M", C.c_int32),
                ("Mf", C.c_int32), ("residual_grid", C.c_int32), ("odds", C.c_int32), ("use_rotation", C.c_int32),
                ("coarse_ls_floor", C.c_float), ("coarse_offset", C.c_float), ("fine_offset", C.c_float),
                ("coarse_min_opacity", C.c_float)]


_WEIGHT_FIELDS = ("w1", "w2", "w3", "w4", "b1", "b2", "b3", "b4", "gn1_w", "gn1_b", "gn2_w", "gn2_b", "gn3_w",
                  "gn3_b", "gn4_w", "gn4_b", "bg_w", "bg_b", "hc_w", "hc_b", "hf_w", "hf_b")


class _GsEncoderWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _WEIGHT_FIELDS]


def pack_first_layer(w: torch.Tensor) -> torch.Tensor:
    """[Co,4,7,7] stride-2 pad-3 weights -> [Co, 256] weights of the equivalent 4x4 stride-1 convolution on
    the space-to-depth input Z[p,q,(dy*2+dx)*4+c] = X[2p+dy, 2q+dx, c] (taps (i,j), K index
    (i*4+j)*16 + (dy*2+dx)*4 + c, with W''[i,j,dy,dx,c] = W[c, 2i+dy-1, 2j+dx-1] and 0 outside)."""
    Co, Ci, kh, kw = w.shape
    assert (Ci, kh, kw) == (4, 7, 7)
    out = w.new_zeros(Co, 4, 4, 2, 2, 4)
    for i in range(4):
        for dy in range(2):
            a = 2 * i + dy - 1
            if not 0 <= a < 7:
                continue
            for j in range(4):
                for dx in range(2):
                    b = 2 * j + dx - 1
                    if 0 <= b < 7:
                        out[:, i, j, dy, dx, :] = w[:, :, a, b]
    return out.reshape(Co, 256)


def space_to_depth_input(x4: torch.Tensor) -> torch.Tensor:
    """[B,4,H,W] -> NHWC [B,H/2,W/2,16] with channel (dy*2+dx)*4 + c (the first layer's GEMM input)."""
    B, Ci, H, W = x4.shape
    z = x4.reshape(B, Ci, H // 2, 2, W // 2, 2).permute(0, 2, 4, 3, 5, 1)  # b, p, q, dy, dx, c
    return z.reshape(B, H // 2, W // 2, 16).contiguous()


def pack_conv(w: torch.Tensor) -> torch.Tensor:
    """[Co,Ci,kh,kw] -> [Co, kh*kw*Ci] (tap-major, channel-minor: the implicit-GEMM K order)."""
    return w.permute(0, 2, 3, 1).reshape(w.shape[0], -1)


def make_desc(fields: dict, B: int, H: int, W: int) -> _GsEncoderDesc:
    d = _GsEncoderDesc()
    d.B, d.H, d.W = B, H, W
    for k, v in fields.items():
        setattr(d, k, v)
    return d


def _weight_struct(t: dict) -> _GsEncoderWeights:
    return _GsEncoderWeights(**{k: t[k].data_ptr() for k in _WEIGHT_FIELDS})


def pack_weights(enc, device) -> dict:
    """The encoder's parameters in the layouts gs_encoder_fwd reads: bf16 implicit-GEMM weights
    ([Co, taps*Ci], tap-major; the first layer as its 4x4 space-to-depth equivalent), fp32 biases,
    GroupNorm affines, the background linear layer and the two heads' packed 1x1 weights."""
    bb = enc.backbone
    blk = enc.fine_decoder.blocks[0].fuse

    def f32(t):
        return t.detach().to(device, torch.float32).contiguous()

    def b16(t):
        return t.detach().to(device, torch.float32).to(torch.bfloat16).contiguous()

    hc_w, hc_b = enc.coarse_head.packed()
    hf_w, hf_b = enc.fine_head.packed()
    return dict(
        w1=b16(pack_first_layer(bb.stage_s2[0].weight.float())), w2=b16(pack_conv(bb.stage_s4[0].weight)),
        w3=b16(pack_conv(bb.stage_s8[0].weight)), w4=b16(pack_conv(blk[0].weight)),
        b1=f32(bb.stage_s2[0].bias), b2=f32(bb.stage_s4[0].bias), b3=f32(bb.stage_s8[0].bias), b4=f32(blk[0].bias),
        gn1_w=f32(bb.stage_s2[2].weight), gn1_b=f32(bb.stage_s2[2].bias),
        gn2_w=f32(bb.stage_s4[2].weight), gn2_b=f32(bb.stage_s4[2].bias),
        gn3_w=f32(bb.stage_s8[2].weight), gn3_b=f32(bb.stage_s8[2].bias),
        gn4_w=f32(blk[2].weight), gn4_b=f32(blk[2].bias),
        bg_w=f32(enc.bg_head.weight), bg_b=f32(enc.bg_head.bias),
        hc_w=f32(hc_w), hc_b=f32(hc_b), hf_w=f32(hf_w), hf_b=f32(hf_b))


def cuda_forward(enc, image, return_latents, render, workspace=None):
    """gs_encoder_fwd / gs_encode_render_fwd for any object that provides the packed weights
    (`_weights(device)` -> (tensors, _GsEncoderWeights)), `_desc(B, H, W)` and the attributes M, Mf,
    d_feature, use_rotation and latent_ch: the nn.Module and the pre-packed checkpoint share it.
    `workspace` (optional): a caller-owned uint8 CUDA tensor of at least the size the library asks for,
    used instead of a fresh allocation (it then holds the call's binning for the debug accessors)."""
    dev = _lib.require_cuda(image)
    if image.dim() != 4 or image.shape[1] != 3:
        raise ValueError("image must be [B,3,H,W]")
    B, _, H, W = image.shape
    if H % 8 or W % 8 or ((H // 4) * (W // 4)) % 64:
        raise NotImplementedError(f"image size {H}x{W}: the CUDA encoder needs H, W multiples of 8 and "
                                  "(H/4)(W/4) a multiple of 64")
    x = image.detach().contiguous().float()
    with torch.cuda.device(dev):
        L = _lib.load()
        tens, wst = enc._weights(dev)
        d = enc._desc(B, H, W)
        size_fn = L.gs_encode_render_workspace_size if render else L.gs_encoder_workspace_size
        nbytes = int(size_fn(C.byref(d)))
        if nbytes == 0 and render and int(L.gs_encoder_workspace_size(C.byref(d))) > 0:
            # the fused call sizes its final render from the host pair bound; where that bound passes the
            # reference's per-image budget, the encoder runs alone and render_alpha_octave (which counts
            # the pairs exactly before it refuses, render_triton.py:378-385) renders its splats
            o, _ = cuda_forward(enc, image, return_latents, render=False)
            rec = render_alpha_octave(o["mu"], o["log_scale"], o["color"], o["opacity"], o["bg"], H, W,
                                      theta=o["theta"], odds=bool(enc.odds))
            return o, rec
        if nbytes == 0:
            raise ValueError("unsupported encoder configuration")
        Nc = (H // 8) * (W // 8) * enc.M
        N = Nc + (H // 4) * (W // 4) * enc.Mf
        o = dict(mu=torch.empty(B, N, 2, device=dev), log_scale=torch.empty(B, N, 2, device=dev),
                 color=torch.empty(B, N, 3, device=dev), opacity=torch.empty(B, N, device=dev),
                 theta=torch.empty(B, N, device=dev) if enc.use_rotation else None,
                 bg=torch.empty(B, 3, device=dev))
        feat = torch.empty(B, H // 8, W // 8, enc.d_feature, device=dev)
        lat = torch.empty(B, H // 4, W // 4, enc.latent_ch, device=dev) if return_latents else None
        if workspace is not None:
            if workspace.dtype != torch.uint8 or workspace.device != dev or workspace.numel() < nbytes:
                raise ValueError(f"workspace must be a uint8 tensor on {dev} of at least {nbytes} bytes")
            ws = workspace
        else:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        p = _lib.ptr
        args = [C.byref(d), C.byref(wst), p(x), p(o["mu"]), p(o["log_scale"]), p(o["color"]), p(o["opacity"]),
                p(o["theta"]), p(o["bg"]), p(feat), p(lat)]
        rec = None
        if render:
            rec = torch.empty(B, 3, H, W, device=dev)
            _lib.check(L.gs_encode_render_fwd(*args, p(rec), p(ws), nbytes, _lib.stream_of(dev)),
                       "gs_encode_render_fwd")
        else:
            _lib.check(L.gs_encoder_fwd(*args, p(ws), nbytes, _lib.stream_of(dev)), "gs_encoder_fwd")
    o["n_gaussians"] = N
    o["n_coarse"] = Nc
    o["backbone_features"] = feat.permute(0, 3, 1, 2)
    if return_latents:
        o["splat_features"] = lat.permute(0, 3, 1, 2)
    return o, rec


class EfficientGaussianEncoder(nn.Module):
    def __init__(self, d_feature=128, stride=8, variant="free", norm_type="group",
                 use_rotation=True, use_grad_input=True,
                 gaussians_per_cell=2, fine_per_cell=2, free_offset_cells=4.0, coarse_scale_bias=-1.5,
                 coarse_min_scale=0.04, fine_scale_bias=-4.0, free_scale_bias=-3.0, opacity_bias=2.0,
                 residual_grid=64, fine_stride=None, coarse_min_opacity=0.0, coarse_offset_cells=2.0,
                 fine_offset_cells=2.0, odds=False):
        super().__init__()
        assert variant in ("free", "adaptive")
        assert stride in (8, 16), "efficient encoder supports stride 8 or 16 (16 = scarce)"
        self.variant = variant
        self.stride = stride
        self.fine_stride = fine_stride if fine_stride is not None else stride
        self.odds = odds
        self.use_grad_input = use_grad_input
        self.residual_grid = residual_grid
        self.norm_type = norm_type
        self.d_feature = d_feature
        self.use_rotation = use_rotation
        self.coarse_ls_floor = math.log(math.exp(coarse_min_scale) - 1.0) if coarse_min_scale > 0 else None
        self.M = gaussians_per_cell
        self.Mf = fine_per_cell
        in_ch = 3 + (1 if use_grad_input else 0)
        self.backbone = _Backbone(in_ch, d_feature, norm_type, stride)
        self.bg_head = nn.Linear(d_feature, 3)
        g_ch = 1 if use_grad_input else 0
        head_in = d_feature + g_ch
        if variant == "free":
            self.head = _SplatHead(head_in, self.M, scale_bias=free_scale_bias, opacity_bias=opacity_bias,
                                   offset_cells=free_offset_cells, use_rotation=use_rotation)
        else:
            self.coarse_head = _SplatHead(head_in, self.M, scale_bias=coarse_scale_bias,
                                          opacity_bias=opacity_bias, offset_cells=coarse_offset_cells,
                                          use_rotation=use_rotation, min_opacity=coarse_min_opacity)
            self.fine_decoder = _FineDecoder(d_feature, stride, self.fine_stride, norm_type)
            self.fine_head = _SplatHead(self.fine_decoder.out_ch + g_ch + 4, self.Mf,
                                        scale_bias=fine_scale_bias, opacity_bias=opacity_bias,
                                        offset_cells=fine_offset_cells, use_rotation=use_rotation)
        self._packed = None
        self._packed_key = None

    # ---------------------------------------------------------------- CUDA path
    def _cuda_supported(self):
        return (self.variant == "adaptive" and self.d_feature == 256 and self.stride == 8 and self.fine_stride == 4
                and self.norm_type == "group" and self.use_grad_input and 1 <= self.M <= 2 and 1 <= self.Mf <= 2
                and len(self.fine_decoder.blocks) == 1)

    def _weights(self, device):
        """Pack the parameters once (bf16 implicit-GEMM layouts, fp32 vectors) and cache them until a
        parameter changes."""
        key = (device, tuple((p.data_ptr(), p._version) for p in self.parameters()))
        if self._packed is not None and self._packed_key == key:
            return self._packed
        t = pack_weights(self, device)
        self._packed = (t, _weight_struct(t))
        self._packed_key = key
        return self._packed

    @property
    def latent_ch(self):
        return self.fine_decoder.out_ch

    def desc_fields(self):
        """The architecture fields of gs_encoder_desc (everything but the batch and image size)."""
        return dict(d=int(self.d_feature), M=int(self.M), Mf=int(self.Mf), residual_grid=int(self.residual_grid),
                    odds=int(bool(self.odds)), use_rotation=int(self.use_rotation),
                    coarse_ls_floor=self.coarse_ls_floor if self.coarse_ls_floor is not None else -float("inf"),
                    coarse_offset=float(self.coarse_head.offset_cells), fine_offset=float(self.fine_head.offset_cells),
                    coarse_min_opacity=float(self.coarse_head.min_opacity))

    def _desc(self, B, H, W):
        return make_desc(self.desc_fields(), B, H, W)

    def _bg(self, feat):
        return torch.sigmoid(self.bg_head(feat.mean(dim=(2, 3))))

    def gather_splat_latents(self, output):
        """Per-splat latent [B, N, C] aligned with output['mu'] (cell-major, then slot); coarse splats get
        zeros (efficient_encoder.py:270-296).  Needs forward(..., return_latents=True)."""
        if "splat_features" not in output:
            raise KeyError("no 'splat_features' -- call forward(image, return_latents=True)")
        feat = output["splat_features"]
        B, Cc, fH, fW = feat.shape
        per_cell = self.Mf if self.variant == "adaptive" else self.M
        latents = feat.permute(0, 2, 3, 1).reshape(B, fH * fW, 1, Cc)
        latents = latents.expand(B, fH * fW, per_cell, Cc).reshape(B, fH * fW * per_cell, Cc)
        n_coarse = int(output.get("n_coarse", 0))
        if n_coarse:
            latents = torch.cat([latents.new_zeros(B, n_coarse, Cc), latents], dim=1)
        if latents.shape[1] != output["mu"].shape[1]:
            raise RuntimeError(f"latent/splat axis mismatch: {latents.shape[1]} vs {output['mu'].shape[1]}")
        return latents

    def forward(self, image, return_latents: bool = False):
        """image [B,3,H,W] in [0,1] (CUDA) -> dict(mu, log_scale, color, opacity, theta, bg, n_gaussians,
        n_coarse, backbone_features) in the reference's layouts (efficient_encoder.py:306-378)."""
        return self._run(image, return_latents, render=False)[0]

    def forward_and_render(self, image, return_latents: bool = False):
        """The encode-and-render pipeline (examples/encode_and_render.py:31-38) in one library call
        (gs_encode_render_fwd): returns (the forward's dict, render_alpha_octave(its splats, H, W,
        odds=self.odds) with that function's defaults).  At H = W = 2 * residual_grid the render reuses the
        octave fields of the coarse splats computed by the encoder's internal render."""
        return self._run(image, return_latents, render=True)

    def _run(self, image, return_latents, render):
        if not self._cuda_supported():
            raise NotImplementedError("the CUDA encoder implements the released 'adaptive' architecture "
                                      "(d_feature=256, stride 8, fine_stride 4, GroupNorm, gradient input)")
        return cuda_forward(self, image, return_latents, render)
