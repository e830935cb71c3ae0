"""Checkpoint loading for the encoder (reference: examples/encode_and_render.py:19-28).

The released checkpoint is a torch pickle ``{step, model, cfg}``; ``cfg['encoder']`` holds the constructor
keywords (plus ``image_size``, which the module does not take).  This loader reads it with
``weights_only=True`` (no arbitrary unpickling), rejects unknown architecture fields like the reference,
and loads the state dict strictly.
"""

from __future__ import annotations

import inspect

import torch

from .efficient_encoder import EfficientGaussianEncoder


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
