"""The CPU oracle (oracle/gsplat_oracle.c) pinned against the reference's own outputs.

Every fixture under tests/golden/ was produced by the reference implementation itself
(tests/golden/make_golden.py runs its Triton kernels through the interpreter); the oracle must
reproduce them to fp32 round-off before any CUDA result is compared with it."""

import numpy as np
import pytest

from golden_util import GOLDEN, fnv_tile_hash, grad_rel, load_render, render_cases


@pytest.mark.parametrize("name", render_cases())
def test_oracle_matches_reference(oracle, name):
    c = load_render(name)
    fn = getattr(oracle, c["fn"])
    i = c["ins"]
    out, g = fn(i["mu"], i["log_scale"], i["color"], i["opacity"], i["bg"], c["H"], c["W"],
                theta=i.get("theta"), grad_out=c["gC"], **c["kw"])
    assert np.abs(out - c["out"]).max() < 2e-5
    rel = grad_rel(g, c["grads"])
    assert max(rel.values()) < 1e-4, rel


def test_oracle_tiles_small(oracle):
    d = np.load(GOLDEN / "tiles_small.npz")
    mu, sc = d["in_mu"][0], d["in_scale"][0]
    for TILE, cutoff, H, W in ((8, 3.0, 64, 64), (16, 5.0, 64, 64), (8, 3.0, 50, 37)):
        key = f"T{TILE}_c{int(cutoff)}_{H}x{W}"
        starts, gid = oracle.build_tiles(mu, sc, H, W, TILE, cutoff)
        assert np.array_equal(starts, d[f"{key}_starts"]), key
        assert np.array_equal(gid, d[f"{key}_gid"]), key
    starts, gid = oracle.build_tiles(d["in_mu_edge"][0], d["in_scale_edge"][0], 50, 37, 8, 3.0)
    assert np.array_equal(starts, d["edge_starts"])
    assert np.array_equal(gid, d["edge_gid"])


def test_oracle_tiles_cfg1_full_size(oracle):
    """Octave routing and per-octave tile lists of config 1 at 768^2 (92,160 splats)."""
    import torch

    from gaussian_2d_splat_encoder_b200 import synth

    d = np.load(GOLDEN / "tiles_cfg1.npz")
    s = synth.synth_splats_cfg1()
    sc = (torch.nn.functional.softplus(s["log_scale"]) + 1e-4)[0].numpy()
    mu = s["mu"][0].numpy()
    oct_, per = oracle.bin_octave(mu, sc, 768, 768)
    assert np.array_equal(oct_, d["oct"].astype(np.int32))
    for o, (starts, gid) in enumerate(per):
        if f"o{o}_starts" not in d.files:
            assert starts[-1] == 0
            continue
        assert np.array_equal(starts, d[f"o{o}_starts"])
        # the reference's ids are local to the octave subset (nonzero order == ascending global id)
        idx = np.nonzero(oct_ == o)[0]
        local = np.searchsorted(idx, gid)
        assert np.array_equal(fnv_tile_hash(local, starts), d[f"o{o}_hash"])
    starts, gid = oracle.build_tiles(mu, sc, 768, 768, 8, 3.0)
    assert np.array_equal(starts, d["cull_starts"])
    assert np.array_equal(fnv_tile_hash(gid, starts), d["cull_hash"])


def test_oracle_upsample_adjoint_is_transpose(oracle):
    """<up(x), y> == <x, up^T(y)> for the bilinear pair used by the octave combine."""
    import ctypes as C

    L = oracle.lib()
    L.orc_upsample_add.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
    L.orc_upsample_adjoint_add.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
    rng = np.random.default_rng(0)
    for (hi, wi, ho, wo) in ((8, 8, 50, 37), (12, 12, 768, 768), (24, 20, 96, 80)):
        x = rng.standard_normal((hi * wi, 1)).astype(np.float32)
        y = rng.standard_normal((ho * wo, 1)).astype(np.float32)
        ux = np.zeros((ho * wo, 1), np.float32)
        L.orc_upsample_add(x.ctypes.data, hi, wi, 1, ux.ctypes.data, ho, wo)
        aty = np.zeros((hi * wi, 1), np.float32)
        L.orc_upsample_adjoint_add(y.ctypes.data, ho, wo, 1, aty.ctypes.data, hi, wi)
        a, b = float((ux * y).sum(dtype=np.float64)), float((x * aty).sum(dtype=np.float64))
        assert abs(a - b) <= 1e-4 * max(1.0, abs(a))


def test_oracle_l2_step_matches_two_calls(oracle):
    """render_alpha_octave_l2 (forward once, mse gradient, backward) gives the same image and loss gradient,
    bit for bit, and the same splat gradients (up to the order of the oracle's threaded accumulation) as a
    forward followed by a backward call with that gradient."""
    from gaussian_2d_splat_encoder_b200 import synth

    s = {k: v.numpy() for k, v in synth.synth_splats_cfg1(600, 64, 96, seed=3).items()}
    tgt = np.random.default_rng(5).random((1, 3, 64, 96), dtype=np.float32)
    out, loss, g, grads = oracle.render_alpha_octave_l2(s["mu"], s["log_scale"], s["color"], s["opacity"],
                                                         s["bg"], 64, 96, tgt, theta=s["theta"], odds=True)
    ref = oracle.render_alpha_octave(s["mu"], s["log_scale"], s["color"], s["opacity"], s["bg"], 64, 96,
                                     theta=s["theta"], odds=True)
    assert np.array_equal(out, ref)
    g_ref = (2.0 / ref.size) * (ref - tgt)
    assert np.array_equal(g, g_ref)
    assert abs(loss - float(np.mean((ref.astype(np.float64) - tgt) ** 2))) < 1e-9
    _, grads_ref = oracle.render_alpha_octave(s["mu"], s["log_scale"], s["color"], s["opacity"], s["bg"], 64, 96,
                                              theta=s["theta"], odds=True, grad_out=g_ref)
    for k in grads_ref:
        np.testing.assert_allclose(grads[k], grads_ref[k], rtol=1e-5, atol=1e-9, err_msg=k)
