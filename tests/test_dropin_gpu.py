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


def _write_mini_llama(d, layers=2, hidden=128, inter=256, heads=2, kv=2, vocab=512, seed=0):
    """A small dense Llama checkpoint (config.json + one safetensors file,
    fp16 weights N(0, 0.02^2)) in the layout the reference's converter reads."""
    import json

    from safetensors.torch import save_file

    d.mkdir(parents=True, exist_ok=True)
    hd = hidden // heads
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": hidden,
           "intermediate_size": inter, "num_hidden_layers": layers, "num_attention_heads": heads,
           "num_key_value_heads": kv, "head_dim": hd, "vocab_size": vocab, "rms_norm_eps": 1e-6,
           "torch_dtype": "float16", "tie_word_embeddings": False}
    (d / "config.json").write_text(json.dumps(cfg))
    g = torch.Generator().manual_seed(seed)

    def rnd(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).half()

    t = {"model.embed_tokens.weight": rnd(vocab, hidden),
         "model.norm.weight": torch.ones(hidden).half(), "lm_head.weight": rnd(vocab, hidden)}
    for i in range(layers):
        p = f"model.layers.{i}."
        for name, shape in (("self_attn.q_proj", (heads * hd, hidden)),
                            ("self_attn.k_proj", (kv * hd, hidden)),
                            ("self_attn.v_proj", (kv * hd, hidden)),
                            ("self_attn.o_proj", (hidden, heads * hd)),
                            ("mlp.gate_proj", (inter, hidden)), ("mlp.up_proj", (inter, hidden)),
                            ("mlp.down_proj", (hidden, inter))):
            t[p + name + ".weight"] = rnd(*shape)
        t[p + "input_layernorm.weight"] = torch.ones(hidden).half()
        t[p + "post_attention_layernorm.weight"] = torch.ones(hidden).half()
    save_file(t, str(d / "model.safetensors"))


def _c_oracle_factory(K=2):
    """The reference encoder's role served by the C restatement (bit-exact
    with the reference encoder): the comparison arm."""
    from oracle.module_oracle import c_encoder

    enc = c_encoder(K)

    def encode(tiles):
        w, i = enc(tiles.detach().cpu().float().contiguous())
        return w.to(tiles.device), i.to(tiles.device)

    encode.K = K
    encode.cb = 2
    return encode


def test_reference_convert_model_runs_on_the_b200_encoder(tmp_path):
    """The reference's own convert_model loop (calibrate -> quantize every
    projection -> reload -> re-forward, two layers, files and manifest) with
    the drop-in: on host tensors every quantized tensor it writes equals, bit
    for bit, the same loop with the C restatement of the reference encoder;
    on the GPU (device "cuda": torch ops, Hessians and encoder on the B200)
    it completes with the same quality."""
    from safetensors.torch import load_file

    from exl3_intel_arc_quantizer_b200 import dropin

    model = tmp_path / "model"
    _write_mini_llama(model)
    build_ref.enable()
    try:
        import exl3_quant.converter as conv
        import exl3_quant.layer_quant as ref_lq
        import exl3_quant.ldlq as ref_ldlq

        def run(out, device):
            cfg = conv.ConversionConfig(model_dir=str(model), output_dir=str(tmp_path / out), K=2,
                                        device=device, num_calibration_rows=2, batch_size=1,
                                        seq_len=64, skip_g_scale=True)
            return conv.convert_model(cfg)

        saved = (ref_lq.make_reference_tile_encoder, ref_ldlq.make_reference_tile_encoder)
        ref_lq.make_reference_tile_encoder = ref_ldlq.make_reference_tile_encoder = _c_oracle_factory
        try:
            rep_c = run("out_c", "cpu")
        finally:
            ref_lq.make_reference_tile_encoder, ref_ldlq.make_reference_tile_encoder = saved
        dropin.install(reference_encoder=True)
        try:
            assert ref_lq.make_reference_tile_encoder is not saved[0]
            rep_b = run("out_b200", "cpu")
            rep_g = run("out_gpu", "cuda")
        finally:
            dropin.uninstall()
        assert ref_lq.make_reference_tile_encoder is saved[0]
    finally:
        build_ref.disable()
    files = sorted(p.name for p in (tmp_path / "out_c" / "qtensors").glob("*.safetensors"))
    assert files == ["model.layers.0.safetensors", "model.layers.1.safetensors",
                     "untouched.safetensors"]
    for name in files:
        a = load_file(str(tmp_path / "out_c" / "qtensors" / name))
        b = load_file(str(tmp_path / "out_b200" / "qtensors" / name))
        assert a.keys() == b.keys()
        for key in a:
            assert torch.equal(a[key], b[key]), (name, key)
    assert len(rep_g.layers) == 2
    for lc, lg in zip(rep_c.layers, rep_g.layers):
        assert lc.quantized_tensors == lg.quantized_tensors
        assert abs(lg.mean_mse - lc.mean_mse) <= 0.05 * lc.mean_mse
