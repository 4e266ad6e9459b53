"""Global-scale search (gss.py) against the reference's own search.

The golden holds the reference's sampled tiles and its (scale, mse) for a
128x256 regularized weight at K=2, computed with its CPU encoder. CPU: the
sampling is bit-exact and the search with the C oracle as the encoder lands
on the same scale and MSE. GPU: the search with the B200 encoder lands on
the same scale (rel 1e-6) and MSE (rel 1e-5: the per-scale mean is reduced
on the device in another order).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exl3_intel_arc_quantizer_b200 import gss


@pytest.fixture(scope="module")
def gg(golden_dir):
    path = golden_dir / "gss_golden.npz"
    if not path.exists():
        pytest.skip("gss golden not generated")
    return np.load(path)


class OracleEncoder:
    K = 2

    def __init__(self):
        from oracle.trellis_oracle import COracle

        self.o = COracle(2, 2)

    def __call__(self, tiles):
        r = self.o.encode_batch(tiles.numpy())
        return (torch.from_numpy(r["recon"].astype(np.float32)),
                torch.from_numpy(r["indices"].view(np.int16)))


def test_sampling_matches_reference(gg):
    w = torch.from_numpy(gg["weight_r"])
    assert torch.equal(gss.sample_scale_tiles(w, 3), torch.from_numpy(gg["samples"]))


def test_refinement_rule():
    f = [0.5, 0.575, 0.65, 0.725, 0.8]
    assert gss.select_refined_scale(f, [5, 4, 3, 4, 5]) == pytest.approx(0.65)
    assert gss.select_refined_scale(f, [5, 4, 3, 3.5, 5]) > 0.65
    assert gss.select_refined_scale(f, [1, 4, 3, 4, 5]) == 0.5          # edge: no parabola
    assert gss.select_refined_scale([0.0, 0.005, 0.01, 0.015, 0.02], [9, 1, 9, 9, 9]) >= 0.01
    with pytest.raises(ValueError):
        gss.g_scale_search_batch([torch.zeros(4, 255)], OracleEncoder())


def test_search_with_oracle_encoder_matches_reference(gg):
    w = torch.from_numpy(gg["weight_r"])
    scale, mse = gss.g_scale_gss(w, OracleEncoder(), 3)
    ref_scale, ref_mse = (float(v) for v in gg["result"])
    assert scale == pytest.approx(ref_scale, rel=1e-9)
    assert mse == pytest.approx(ref_mse, rel=1e-6)


@pytest.mark.gpu
def test_search_with_b200_encoder_matches_reference(gg):
    from exl3_intel_arc_quantizer_b200.ldlq import make_xpu_tile_encoder

    w = torch.from_numpy(gg["weight_r"]).cuda()
    scale, mse = gss.g_scale_gss(w, make_xpu_tile_encoder(K=2), 3)
    ref_scale, ref_mse = (float(v) for v in gg["result"])
    assert scale == pytest.approx(ref_scale, rel=1e-6)
    assert mse == pytest.approx(ref_mse, rel=1e-5)
