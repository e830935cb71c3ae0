"""The CUDA-graph pipelines replay exactly the eager path."""

import numpy as np
import pytest
import torch

from enc_util import GOLDEN_CFG
from golden_util import REORDER_TOL

pytestmark = pytest.mark.gpu


def test_encode_render_graph_matches_eager(lib):
    from gaussian_2d_splat_encoder_b200 import pipeline, synth
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder
    from gaussian_2d_splat_encoder_b200.render_triton import render_alpha_octave

    torch.manual_seed(0)
    enc = EfficientGaussianEncoder(**GOLDEN_CFG).cuda().eval()
    imgs = [synth.synth_card(256, 256, 60, 20, s).cuda() for s in (3, 4)]
    pipe = pipeline.EncodeRender(enc, 1, 256, 256)
    for x in imgs:
        with torch.inference_mode():
            o = enc(x)
            ref = render_alpha_octave(o["mu"], o["log_scale"], o["color"], o["opacity"], o["bg"], 256, 256,
                                      theta=o["theta"], odds=True)
        got = pipe(x).clone()
        torch.cuda.synchronize()
        assert torch.allclose(got, ref, atol=1e-5, rtol=0), (got - ref).abs().max()
        assert torch.allclose(pipe.out["mu"], o["mu"], atol=1e-5, rtol=0)
    assert pipe.launches_per_replay > 20


@pytest.mark.parametrize("size,rg", [(256, 128), (256, 96), (768, 384)])
def test_forward_and_render_matches_separate_calls(lib, size, rg):
    """gs_encode_render_fwd (which, at H = W = 2 * residual_grid, takes the coarse splats' octave fields
    from the encoder's internal render) against the encoder forward followed by render_alpha_octave."""
    from gaussian_2d_splat_encoder_b200 import synth
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder
    from gaussian_2d_splat_encoder_b200.render_triton import render_alpha_octave

    torch.manual_seed(1)
    enc = EfficientGaussianEncoder(**{**GOLDEN_CFG, "residual_grid": rg}).cuda().eval()
    x = synth.synth_card(size, size, 80, 30, 7).cuda()
    with torch.inference_mode():
        o = enc(x)
        ref = render_alpha_octave(o["mu"], o["log_scale"], o["color"], o["opacity"], o["bg"], size, size,
                                  theta=o["theta"], odds=True)
        o2, rec = enc.forward_and_render(x)
    torch.cuda.synchronize()
    # the encoder outputs agree to the last bits the GroupNorm statistics' double-precision atomics leave
    for k in ("mu", "log_scale", "color", "opacity", "theta", "bg"):
        assert float((o[k] - o2[k]).abs().max()) < 1e-6, k
    assert float((rec - ref).abs().max()) < 2e-5


def test_encode_render_stream_matches_single(lib):
    """The streaming pipeline (copies overlapped with the kernels of neighbouring images) returns, for
    every image of a stream, exactly what the single-image pipeline returns."""
    from gaussian_2d_splat_encoder_b200 import pipeline, synth
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    torch.manual_seed(0)
    enc = EfficientGaussianEncoder(**GOLDEN_CFG).cuda().eval()
    imgs = [synth.synth_card(256, 256, 60, 20, s).contiguous().pin_memory() for s in range(5)]
    single = pipeline.EncodeRender(enc, 1, 256, 256)
    refs = []
    for x in imgs:
        refs.append(single(x).cpu())
    st = pipeline.EncodeRenderStream(enc, 256, 256).capture()
    outs = [torch.empty(1, 3, 256, 256).pin_memory() for _ in imgs]
    st.start_after()
    for x, o in zip(imgs, outs):
        st.submit(x, o)
    st.synchronize()
    for o, r in zip(outs, refs):
        assert float((o - r).abs().max()) < REORDER_TOL
    # device-resident images, several in flight on their own streams, results left in the slots
    dev_imgs = [x.cuda() for x in imgs[:len(st.slots)]]
    st.start_after()
    recs = [st.submit(x) for x in dev_imgs]
    st.synchronize()
    for rec, r in zip(recs, refs):
        assert float((rec.cpu() - r).abs().max()) < REORDER_TOL
    # batches of two images per graph replay (the bench's throughput form), host and device batches
    sb = pipeline.EncodeRenderStream(enc, 256, 256, depth=2, batch=2).capture()
    pairs = [torch.cat(imgs[i:i + 2]).pin_memory() for i in (0, 2)]
    bouts = [torch.empty(2, 3, 256, 256).pin_memory() for _ in pairs]
    sb.start_after()
    for x, o in zip(pairs, bouts):
        sb.submit(x, o)
    sb.synchronize()
    for j, o in enumerate(bouts):
        for t in range(2):
            assert float((o[t] - refs[2 * j + t][0]).abs().max()) < REORDER_TOL
    sb.start_after()
    rec = sb.submit(pairs[1].cuda())
    sb.synchronize()
    for t in range(2):
        assert float((rec[t].cpu() - refs[2 + t][0]).abs().max()) < REORDER_TOL


def test_render_fit_step_graph_matches_eager(lib):
    from gaussian_2d_splat_encoder_b200 import pipeline, synth
    from gaussian_2d_splat_encoder_b200.render_triton import render_alpha_octave

    s = synth.synth_splats_cfg1(N=20000, H=384, W=384, seed=9)
    keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
    d = {k: v.cuda() for k, v in s.items()}
    step = pipeline.RenderFitStep(20000, 384, 384, "cuda")
    step.load(*[d[k] for k in keys], d["target"])
    loss, grads = step.replay()
    L = [d[k].clone().requires_grad_(True) for k in keys]
    out = render_alpha_octave(*L[:5], 384, 384, theta=L[5], odds=True)
    ref_loss = torch.nn.functional.mse_loss(out, d["target"])
    ref = torch.autograd.grad(ref_loss, L)
    torch.cuda.synchronize()
    assert abs(loss.item() - ref_loss.item()) <= 1e-6 * abs(ref_loss.item())
    for g, r in zip(grads, ref):
        rel = (g - r).abs().max().item() / max(r.abs().max().item(), 1e-30)
        assert rel < 1e-4, rel
