"""The drop-in shim against the reference package itself (host logic only).

``oracle/_ref`` holds the reference's ``exl3_quant`` package byte-compiled
from its own sources (``oracle/build_ref.py``). With
``dropin.install()``, the reference's unmodified factories and modules bind
this package's encoder; no GPU work runs here.
"""

from __future__ import annotations

import pytest

from oracle import build_ref

pytestmark = pytest.mark.skipif(not build_ref.available(),
                                reason="compiled reference package (oracle/_ref) not built")


@pytest.fixture()
def reference():
    build_ref.enable()
    from exl3_intel_arc_quantizer_b200 import dropin

    pkg = dropin.install()
    try:
        yield pkg
    finally:
        dropin.uninstall()
        build_ref.disable()


def test_reference_factories_bind_the_b200_encoder(reference):
    from exl3_intel_arc_quantizer_b200 import dropin, xpu_quantizer
    from exl3_quant import ldlq as ref_ldlq
    from exl3_quant import layer_quant as ref_layer_quant

    assert dropin.installed()
    assert reference.__name__ == "exl3_quant"
    assert ref_layer_quant.XPUTrellisEncoder is xpu_quantizer.XPUTrellisEncoder
    assert ref_layer_quant.ScratchArena is xpu_quantizer.ScratchArena
    enc = ref_ldlq.make_xpu_tile_encoder(K=3, device_index=0)
    assert enc.K == 3 and enc.cb == xpu_quantizer.CB_MUL1


def test_reference_hessian_hook_is_routed_and_restored(reference):
    from exl3_intel_arc_quantizer_b200 import dropin
    from exl3_quant import calibration as ref_cal

    acc = ref_cal.HessianCollector._accumulate
    assert getattr(acc, "_exl3_b200", False)
    dropin.install()                                   # idempotent
    assert ref_cal.HessianCollector._accumulate is acc
    dropin.uninstall()
    assert not getattr(ref_cal.HessianCollector._accumulate, "_exl3_b200", False)
    assert not dropin.installed()
    dropin.install()


def test_reference_cpu_collector_keeps_its_own_arithmetic(reference):
    """CPU activations are not the B200 path's: the routed hook hands them to
    the reference's own fp32 GEMM."""
    import torch
    from exl3_quant import calibration as ref_cal

    layer = torch.nn.Sequential(torch.nn.Linear(64, 32, bias=False))
    col = ref_cal.HessianCollector(layer, device=torch.device("cpu"),
                                   groups={"0": ["0"]})
    x = torch.randn(5, 7, 64)
    with torch.no_grad():
        layer(x)
    col.close()
    xf = x.reshape(-1, 64)
    assert torch.equal(col.hessians["0"], torch.zeros(64, 64) + xf.T @ xf)
    assert col.token_counts["0"] == 35
