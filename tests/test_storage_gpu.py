"""GPU parity of the storage side (container pack/unpack, weight decode,
layer tensors, export and reload).

Tolerances: container words and states bit-exact; decoded weight within
1e-5 x max|w| of the reference's float32 GEMM rotation (the kernel's
rotation is a butterfly transform), and bit-identical to this package's own
``weight_from_quantized`` on the same w_hat (both use the same transform).
"""

from __future__ import annotations

import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200 import serialization as ser  # noqa: E402
from exl3_intel_arc_quantizer_b200.hadamard import weight_from_quantized  # noqa: E402
from exl3_intel_arc_quantizer_b200.trellis_format import CB_MUL1  # noqa: E402
from oracle import storage_oracle as so  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rand_cases(sg):
    return sorted({k.split("/")[0] for k in sg.files if k.startswith("rand_")})


def test_pack_unpack_decode_match_reference(storage_golden, module_golden_arrays):
    sg = storage_golden
    enc = torch.from_numpy(module_golden_arrays["encoded"]).to(DEV)
    tr = ser.pack_module_trellis(enc, K=2)
    assert tr.is_cuda and torch.equal(tr.cpu(), torch.from_numpy(sg["module/trellis"]))
    assert torch.equal(ser.unpack_module_trellis(tr, K=2).cpu(), enc.cpu())
    dec = ser.decode_weight_from_storage(tr, torch.from_numpy(module_golden_arrays["su"]).half(),
                                         torch.from_numpy(module_golden_arrays["sv"]).half(), K=2)
    ref = torch.from_numpy(sg["module/decoded"])
    assert (dec.cpu() - ref).abs().max() <= 1e-5 * ref.abs().max()
    for name in _rand_cases(sg):
        K, cb = (int(v) for v in sg[f"{name}/params"])
        tr = torch.from_numpy(sg[f"{name}/trellis"]).to(DEV)
        st = ser.unpack_module_trellis(tr, K)
        assert torch.equal(st.cpu(), torch.from_numpy(sg[f"{name}/unpacked"])), name
        su = torch.from_numpy(sg[f"{name}/suh"]).to(DEV)
        sv = torch.from_numpy(sg[f"{name}/svh"]).to(DEV)
        dec, w_hat = ser.decode_weight_from_storage(tr, su, sv, K=K, cb=cb, return_w_hat=True)
        ref = torch.from_numpy(sg[f"{name}/decoded"])
        assert (dec.cpu() - ref).abs().max() <= 1e-5 * ref.abs().max(), name
        assert torch.equal(w_hat.cpu(), torch.from_numpy(so.w_hat_from_trellis(
            sg[f"{name}/trellis"], K, cb))), name
        assert torch.equal(dec, weight_from_quantized(w_hat, su.float(), sv.float())), name


def test_layer_tensors_match_reference_schema(storage_golden, module_golden_arrays, tmp_path):
    sg = storage_golden

    class Res:
        K, cb = 2, CB_MUL1
        encoded = torch.from_numpy(module_golden_arrays["encoded"]).to(DEV)
        su = torch.from_numpy(module_golden_arrays["su"]).to(DEV)
        sv = torch.from_numpy(module_golden_arrays["sv"]).to(DEV)
        w_hat = torch.from_numpy(module_golden_arrays["w_hat"])

    tensors, storage = ser.build_layer_tensors({"self_attn.o_proj": Res()}, layer_idx=3)
    keys = sorted(tensors)
    assert keys == list(sg["module/layer_keys"])
    assert [json.dumps(list(tensors[k].shape)) for k in keys] == list(sg["module/layer_shapes"])
    assert [str(tensors[k].dtype) for k in keys] == list(sg["module/layer_dtypes"])
    assert json.dumps(storage, sort_keys=True) == str(sg["module/storage_json"])
    st_file, qc_file = ser.export_layer_safetensors({"self_attn.o_proj": Res()}, tmp_path,
                                                    layer_idx=3)
    assert json.loads(qc_file.read_text())["bits"] == 2
    # module golden w_hat is (k, n) in the quantized orientation (128 x 256)
    out = ser.load_and_verify_layer_safetensors(st_file, {"self_attn.o_proj": Res()}, atol=5e-3)
    assert list(out) == ["model.layers.3.self_attn.o_proj"]


def test_full_size_roundtrip_through_encoder():
    """4096 x 4096 module: encoder states -> container -> decode equals the
    module's own reconstruction bit for bit (fp32 scales) and within fp16
    scale rounding with the stored fp16 scales."""
    from exl3_intel_arc_quantizer_b200.ldlq import make_xpu_tile_encoder
    from exl3_intel_arc_quantizer_b200.layer_quant import quantize_linear_module

    g = torch.Generator(device="cpu").manual_seed(5)
    k = n = 1024
    W = (torch.randn(n, k, generator=g) * 0.02).to(DEV)
    X = torch.randn(2048, k, generator=g).to(DEV)
    H = X.T @ X / 2048
    H.diagonal().add_(0.01 * H.diagonal().mean())
    for K in (2, 4):
        res = quantize_linear_module("m", W, H, K=K, tile_encoder=make_xpu_tile_encoder(K=K))
        tr = ser.pack_module_trellis(res.encoded, K)
        assert torch.equal(ser.unpack_module_trellis(tr, K), res.encoded.to(DEV))
        dec = ser.decode_weight_from_storage(tr, res.su, res.sv, K=K)
        assert torch.equal(dec, res.w_hat)
        dec16 = ser.decode_weight_from_storage(tr, res.su.half(), res.sv.half(), K=K)
        assert float((dec16 - res.w_hat).abs().max()) <= 2e-3 * float(res.w_hat.abs().max())


@pytest.mark.parametrize("K", range(1, 9))
def test_decode_multi_block_every_k(K):
    """A 384 x 256 weight (3 x 2 blocks of 128 x 128) from a random container
    at every K and codebook: the decode kernel's w_hat equals the oracle's
    state -> codebook -> tile placement bit for bit, and the weight equals
    the package's own rotation of that w_hat bit for bit (fp32 scales) - so
    the per-block container offsets, the window table and both rotations
    are checked away from block (0, 0) for the shuffle (K = 1, 2, 4) and the
    staged (other K) window builds alike."""
    rng = np.random.default_rng(70 + K)
    tk, tn = 24, 16
    tr_np = rng.integers(-32768, 32768, size=(tk, tn, 16 * K)).astype(np.int16)
    su = torch.from_numpy(rng.uniform(0.5, 1.5, tk * 16).astype(np.float32)).to(DEV)
    sv = torch.from_numpy(rng.uniform(0.5, 1.5, tn * 16).astype(np.float32)).to(DEV)
    tr = torch.from_numpy(tr_np).to(DEV)
    for cb in (0, 1, 2):
        dec, w_hat = ser.decode_weight_from_storage(tr, su, sv, K=K, cb=cb, return_w_hat=True)
        assert torch.equal(w_hat.cpu(), torch.from_numpy(so.w_hat_from_trellis(tr_np, K, cb)))
        assert torch.equal(dec, weight_from_quantized(w_hat, su, sv)), (K, cb)
        ref = so.weight_from_quantized(w_hat.cpu().numpy(), su.cpu().numpy(), sv.cpu().numpy())
        assert float(np.abs(dec.cpu().numpy() - ref).max()) <= 1e-5 * float(np.abs(ref).max())


def test_validation():
    tr = torch.zeros(8, 8, 32, dtype=torch.int16, device=DEV)
    ones = torch.ones(128, dtype=torch.float16, device=DEV)
    with pytest.raises(ValueError):
        ser.pack_module_trellis(torch.zeros(2, 2, 255, dtype=torch.int16, device=DEV), 2)
    with pytest.raises(ValueError):
        ser.unpack_module_trellis(tr, 3)
    with pytest.raises(ValueError):
        ser.decode_weight_from_storage(tr, ones[:64], ones, K=2)
    with pytest.raises(ValueError):
        ser.decode_weight_from_storage(torch.zeros(2, 8, 32, dtype=torch.int16, device=DEV),
                                       ones[:32], ones, K=2)
    with pytest.raises(ValueError):
        ser.decode_weight_from_storage(tr, ones, ones, K=2, cb=7)
    assert ser.pack_module_trellis(torch.zeros(0, 4, 256, dtype=torch.int16, device=DEV),
                                   2).shape == (0, 4, 32)
