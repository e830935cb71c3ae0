"""The pre-packed encoder format (host side): round trip, descriptor equality with the module's,
format/version checks, and the architecture gate."""

import ctypes as C

import pytest
import torch

from enc_util import GOLDEN_CFG


def _module():
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    torch.manual_seed(0)
    return EfficientGaussianEncoder(**GOLDEN_CFG)


def test_packed_round_trip(tmp_path, lib):
    from gaussian_2d_splat_encoder_b200 import checkpoint as ck
    from gaussian_2d_splat_encoder_b200 import efficient_encoder as ee

    m = _module()
    f = tmp_path / "enc.packed"
    ck.save_packed(m, f)
    pe = ck.load_packed(f, device="cpu")
    ref = ee.pack_weights(m, torch.device("cpu"))
    t, st = pe._weights(torch.device("cpu"))
    assert set(t) == set(ee._WEIGHT_FIELDS)
    for k, v in ref.items():
        assert t[k].dtype == v.dtype and torch.equal(t[k], v), k
    assert t["w4"].dtype == torch.bfloat16 and t["hf_w"].dtype == torch.float32
    assert st.w1 == t["w1"].data_ptr()
    for B, H, W in ((1, 256, 256), (2, 768, 512)):
        a, b = m._desc(B, H, W), pe._desc(B, H, W)
        for name, _ in a._fields_:
            assert getattr(a, name) == getattr(b, name), name
        assert lib.gs_encoder_workspace_size(C.byref(a)) == lib.gs_encoder_workspace_size(C.byref(b)) > 0
    assert (pe.M, pe.Mf, pe.latent_ch, pe.d_feature) == (m.M, m.Mf, m.latent_ch, m.d_feature)
    # bf16 GEMM weights: the packed file is well under the fp32 parameter bytes
    fp32_bytes = sum(p.numel() * 4 for p in m.parameters())
    assert f.stat().st_size < 0.6 * fp32_bytes


def test_packed_rejects_bad_files(tmp_path):
    from gaussian_2d_splat_encoder_b200 import checkpoint as ck

    m = _module()
    f = tmp_path / "enc.packed"
    ck.save_packed(m, f)
    blob = torch.load(f, weights_only=True)
    blob["version"] = 99
    torch.save(blob, tmp_path / "v99")
    with pytest.raises(ValueError, match="version"):
        ck.load_packed(tmp_path / "v99", device="cpu")
    torch.save({"step": 1, "model": {}}, tmp_path / "other")
    with pytest.raises(ValueError, match="not a packed"):
        ck.load_packed(tmp_path / "other", device="cpu")
    del blob["weights"]["w2"]
    blob["version"] = ck.PACKED_VERSION
    torch.save(blob, tmp_path / "partial")
    with pytest.raises(ValueError, match="missing"):
        ck.load_packed(tmp_path / "partial", device="cpu")


def test_packed_refuses_unsupported_architecture(tmp_path):
    from gaussian_2d_splat_encoder_b200 import checkpoint as ck
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    torch.manual_seed(0)
    m = EfficientGaussianEncoder(d_feature=64, variant="free")
    with pytest.raises(NotImplementedError):
        ck.save_packed(m, tmp_path / "x")


def test_packed_forward_needs_cuda(tmp_path):
    from gaussian_2d_splat_encoder_b200 import checkpoint as ck

    ck.save_packed(_module(), tmp_path / "enc.packed")
    pe = ck.load_packed(tmp_path / "enc.packed", device="cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        pe(torch.zeros(1, 3, 64, 64))


def test_pipeline_takes_a_packed_encoder(tmp_path):
    """pipeline.EncodeRender finds a PackedEncoder's device (it has no parameters)."""
    from gaussian_2d_splat_encoder_b200 import checkpoint as ck
    from gaussian_2d_splat_encoder_b200 import pipeline

    ck.save_packed(_module(), tmp_path / "enc.packed")
    pe = ck.load_packed(tmp_path / "enc.packed", device="cpu")
    er = pipeline.EncodeRender(pe, 1, 64, 64)
    assert er.dev == torch.device("cpu") and er.x.shape == (1, 3, 64, 64)
