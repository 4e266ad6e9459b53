"""The unmodified reference package on the B200 path, through the drop-in.

The reference's own ``exl3_quant.ldlq.ldlq`` and
``exl3_quant.layer_quant.quantize_linear_module`` (byte-compiled from its
sources into ``oracle/_ref``), with ``dropin.install()`` and the tile
encoder from the reference's own ``make_xpu_tile_encoder`` factory, must
reproduce the reference's golden LDLQ and module outputs bit for bit: the
factory now builds the B200 encoder. Its Hessian collector, routed to the
tcgen05 kernel, must agree with its own fp32 GEMM within the Hessian
tolerance (max relative error 1e-4).
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import build_ref  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not build_ref.available(),
                                 reason="compiled reference package (oracle/_ref) not built")]
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def reference():
    build_ref.enable()
    from exl3_intel_arc_quantizer_b200 import dropin

    pkg = dropin.install()
    try:
        yield pkg
    finally:
        dropin.uninstall()
        build_ref.disable()


@pytest.mark.parametrize("name", ["k2_32x128", "k4_64x128"])
def test_reference_ldlq_with_its_factory_encoder_is_bit_exact(reference, ldlq_golden, name):
    from exl3_quant.ldlq import ldlq, make_xpu_tile_encoder

    K, k, n, buf, seed = (int(v) for v in ldlq_golden[f"{name}/params"])
    enc = make_xpu_tile_encoder(K=K, device_index=0)
    res = ldlq(torch.from_numpy(ldlq_golden[f"{name}/weight"]),
               torch.from_numpy(ldlq_golden[f"{name}/L"]), enc, buf_size_k=buf)
    assert torch.equal(res.weight_q, torch.from_numpy(ldlq_golden[f"{name}/weight_q"]))
    assert torch.equal(res.encoded, torch.from_numpy(ldlq_golden[f"{name}/encoded"]))


def test_reference_module_driver_with_its_factory_encoder_is_bit_exact(reference,
                                                                       module_golden_arrays):
    from exl3_quant.layer_quant import quantize_linear_module
    from exl3_quant.ldlq import make_xpu_tile_encoder

    gm = module_golden_arrays
    res = quantize_linear_module("mod", torch.from_numpy(gm["W"]), torch.from_numpy(gm["H"]),
                                 K=2, tile_encoder=make_xpu_tile_encoder(K=2),
                                 skip_g_scale=True, buf_size_k=64)
    assert torch.equal(res.encoded, torch.from_numpy(gm["encoded"]))
    assert torch.equal(res.w_hat.float(), torch.from_numpy(gm["w_hat"]).float())


def test_reference_hessian_collector_runs_the_tcgen05_kernel(reference):
    from exl3_quant import calibration as ref_cal

    torch.manual_seed(3)
    layer = torch.nn.Sequential(torch.nn.Linear(256, 64, bias=False)).to(DEV).half()
    col = ref_cal.HessianCollector(layer, device=DEV, groups={"0": ["0"]})
    xs = [torch.randn(4, 100, 256, device=DEV).half() for _ in range(3)]
    xs[0][..., 5] *= 30.0
    with torch.no_grad():
        for x in xs:
            layer(x)
    col.close()
    want = torch.zeros(256, 256, device=DEV)
    for x in xs:
        xf = x.reshape(-1, 256).float()
        want += xf.T @ xf
    got = col.hessians["0"]
    assert col.token_counts["0"] == 1200
    assert float((got - want).abs().max() / want.abs().max()) <= 1e-4
    assert torch.equal(got, got.T)
