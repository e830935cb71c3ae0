"""Checkpoint loading for the encoder (reference: examples/encode_and_render.py:19-28).

The released checkpoint is a torch pickle ``{step, model, cfg}``; ``cfg['encoder']`` holds the constructor
keywords (plus ``image_size``, which the module does not take).  ``load_encoder`` reads it with
``weights_only=True`` (no arbitrary unpickling), rejects unknown architecture fields like the reference,
and loads the state dict strictly.

Pre-packed format (serving): ``save_packed`` writes the weights in the layouts the CUDA forward reads
(bf16 implicit-GEMM convolution weights, fp32 vectors and head matrices) plus the architecture fields of
``gs_encoder_desc``; ``load_packed`` returns a ``PackedEncoder`` that runs the same forward /
forward_and_render without building the nn.Module or repacking (about half the bytes of the fp32
checkpoint, and no per-process packing work).
"""

from __future__ import annotations

import inspect

import torch

from . import efficient_encoder as _ee
from .efficient_encoder import EfficientGaussianEncoder

PACKED_FORMAT = "gsplat_b200.packed_encoder"
PACKED_VERSION = 1


def load_encoder(checkpoint_path, device="cuda"):
    ck = torch.load(checkpoint_path, map_location="cpu", weights_only=True)
    config = dict(ck["cfg"]["encoder"])
    accepted = set(inspect.signature(EfficientGaussianEncoder.__init__).parameters) - {"self"}
    unknown = set(config) - accepted - {"image_size"}
    if unknown:
        raise ValueError(f"Unknown checkpoint architecture fields: {sorted(unknown)}")
    enc = EfficientGaussianEncoder(**{k: v for k, v in config.items() if k in accepted})
    enc.load_state_dict(ck["model"], strict=True)
    return enc.to(device).eval()


def save_packed(encoder: EfficientGaussianEncoder, path) -> None:
    """Write `encoder`'s weights in the CUDA forward's packed layouts (CPU tensors) with its descriptor
    fields; only the architecture the CUDA forward implements is accepted."""
    if not encoder._cuda_supported():
        raise NotImplementedError("only the released 'adaptive' architecture has a packed layout")
    weights = _ee.pack_weights(encoder, torch.device("cpu"))
    torch.save({"format": PACKED_FORMAT, "version": PACKED_VERSION, "desc": encoder.desc_fields(),
                "latent_ch": int(encoder.latent_ch), "weights": weights}, path)


def load_packed(path, device="cuda") -> "PackedEncoder":
    blob = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(blob, dict) or blob.get("format") != PACKED_FORMAT:
        raise ValueError(f"{path}: not a packed encoder file")
    if blob.get("version") != PACKED_VERSION:
        raise ValueError(f"{path}: packed encoder version {blob.get('version')} (this build reads {PACKED_VERSION})")
    missing = set(_ee._WEIGHT_FIELDS) - set(blob["weights"])
    if missing:
        raise ValueError(f"{path}: missing packed weights {sorted(missing)}")
    return PackedEncoder(blob["desc"], blob["latent_ch"], blob["weights"], device)


class PackedEncoder:
    """EfficientGaussianEncoder's inference entry points over pre-packed weights: forward(image,
    return_latents=False) and forward_and_render(image) return what the module's do (same kernels,
    same packed weights, so the same bytes); gather_splat_latents as the module's."""

    variant = "adaptive"

    def __init__(self, desc: dict, latent_ch: int, weights: dict, device="cuda"):
        self.fields = dict(desc)
        self.d_feature, self.M, self.Mf = int(desc["d"]), int(desc["M"]), int(desc["Mf"])
        self.use_rotation, self.odds = bool(desc["use_rotation"]), bool(desc["odds"])
        self.residual_grid = int(desc["residual_grid"])
        self.latent_ch = int(latent_ch)
        self.device = torch.device(device)
        self._host = weights
        self._dev = {}

    def _weights(self, device):
        key = str(device)
        if key not in self._dev:
            t = {k: v.to(device).contiguous() for k, v in self._host.items()}
            self._dev[key] = (t, _ee._weight_struct(t))
        return self._dev[key]

    def _desc(self, B, H, W):
        return _ee.make_desc(self.fields, B, H, W)

    def forward(self, image, return_latents: bool = False):
        return _ee.cuda_forward(self, image, return_latents, render=False)[0]

    __call__ = forward

    def forward_and_render(self, image, return_latents: bool = False):
        return _ee.cuda_forward(self, image, return_latents, render=True)

    gather_splat_latents = EfficientGaussianEncoder.gather_splat_latents
