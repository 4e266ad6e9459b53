"""GPU tests of the layer-level drivers.

* ``quantize_modules`` (batched global-scale search, one block-LDL per shared
  Hessian, interleaved LDLQ) gives bit-identical results to
  ``quantize_linear_module`` run module by module, with and without the
  global-scale search;
* ``converter.convert_layer`` (calibrate, quantize, reload, re-forward)
  equals the reference's sequential steps (``calibrate_layer`` then
  ``quantize_decoder_layer`` on an identical layer) module for module.
"""

from __future__ import annotations

import copy

import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200.calibration import (  # noqa: E402
    TransformerDecoderLayer,
    calibrate_layer,
)
from exl3_intel_arc_quantizer_b200.converter import convert_layer  # noqa: E402
from exl3_intel_arc_quantizer_b200.layer_quant import (  # noqa: E402
    quantize_decoder_layer,
    quantize_linear_module,
    quantize_modules,
)
from exl3_intel_arc_quantizer_b200.ldlq import make_xpu_tile_encoder  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _hess(k, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(2048, k, generator=g)
    x[:, :3] *= 10.0
    h = (x.T @ x / 2048).to(DEV)
    h.diagonal().add_(0.01 * h.diagonal().mean())
    return h


@pytest.mark.parametrize("skip_gss", [True, False])
def test_quantize_modules_equals_per_module(skip_gss):
    g = torch.Generator(device="cpu").manual_seed(2)
    H1, H2, H3 = _hess(256, 1), _hess(512, 2), _hess(256, 3)
    mods = {"q": (torch.randn(256, 256, generator=g) * 0.02, H1),
            "k": (torch.randn(128, 256, generator=g) * 0.02, H1.clone()),
            "gate": (torch.randn(512, 256, generator=g) * 0.02, H3),
            "down": (torch.randn(256, 512, generator=g) * 0.02, H2)}
    mods = {m: (w.to(DEV), h) for m, (w, h) in mods.items()}
    enc = make_xpu_tile_encoder(K=2)
    batched = quantize_modules(mods, K=2, tile_encoder=enc, skip_g_scale=skip_gss)
    for m, (w, h) in mods.items():
        one = quantize_linear_module(m, w, h, K=2, tile_encoder=enc, skip_g_scale=skip_gss)
        b = batched[m]
        assert torch.equal(b.encoded, one.encoded), m
        assert torch.equal(b.w_hat, one.w_hat), m
        assert b.metrics.g_scale == one.metrics.g_scale, m
        assert b.metrics.proxy_loss == one.metrics.proxy_loss, m


def test_convert_layer_equals_sequential_reference_steps():
    torch.manual_seed(0)
    layer = TransformerDecoderLayer(256, 512, 4, 2)
    for p in layer.parameters():
        if p.dim() == 2:
            torch.nn.init.normal_(p, std=0.02)
    layer2 = copy.deepcopy(layer)
    g = torch.Generator(device="cpu").manual_seed(4)
    hs = [torch.randn(2, 64, 256, generator=g).half().to(DEV) for _ in range(2)]
    res, nxt, tm = convert_layer(layer, hs, K=2, device=DEV)
    assert set(res) == {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                        "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"}
    assert tm.local_tokens == 256 and tm.tiles == sum(
        r.encoded.shape[0] * r.encoded.shape[1] for r in res.values())
    assert len(nxt) == 2 and nxt[0].shape == (2, 64, 256) and bool(torch.isfinite(nxt[0]).all())
    assert torch.equal(layer.self_attn.q_proj.weight.data,
                       res["self_attn.q_proj"].w_hat.T.to(torch.float16))

    hessians, _ = calibrate_layer(layer2, hs, DEV)
    rep = quantize_decoder_layer(layer2, hessians, K=2, device=DEV)
    for m, r in rep.module_results.items():
        assert torch.equal(r.encoded, res[m].encoded), m
        assert torch.equal(r.w_hat, res[m].w_hat), m
