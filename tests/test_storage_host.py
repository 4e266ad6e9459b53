"""Storage-side oracle pinned against the reference's serialization outputs
(CPU only): container unpack bit for bit, weight decode within float32
GEMM rounding."""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import storage_oracle as so
from oracle.trellis_oracle import pack_trellis, swap16_storage


@pytest.fixture(scope="module")
def sg(golden_dir):
    path = golden_dir / "storage_golden.npz"
    if not path.exists():
        pytest.skip("storage golden not generated")
    return np.load(path)


def _rand_cases(sg):
    return sorted({k.split("/")[0] for k in sg.files if k.startswith("rand_")})


def test_unpack_oracle_matches_reference(sg):
    for name in _rand_cases(sg) + ["module"]:
        if name == "module":
            K = 2
        else:
            K = int(sg[f"{name}/params"][0])
        got = so.unpack_module_trellis(sg[f"{name}/trellis"], K)
        assert np.array_equal(got, sg[f"{name}/unpacked"]), name


def test_decode_oracle_matches_reference(sg):
    for name in _rand_cases(sg):
        K, cb = (int(v) for v in sg[f"{name}/params"])
        got = so.decode_weight_from_storage(sg[f"{name}/trellis"], sg[f"{name}/suh"],
                                            sg[f"{name}/svh"], K, cb)
        ref = sg[f"{name}/decoded"]
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max(), name


def test_module_pack_roundtrip(sg, module_golden_arrays):
    enc = module_golden_arrays["encoded"]
    words = np.stack([swap16_storage(pack_trellis(t.view(np.uint16), 2))
                      for t in enc.reshape(-1, 256)]).reshape(8, 16, 32)
    assert np.array_equal(words.view(np.int16), sg["module/trellis"])
    assert np.array_equal(sg["module/unpacked"], enc)   # encoder states are a consistent path
    storage = json.loads(str(sg["module/storage_json"]))
    assert list(storage) == ["model.layers.3.self_attn.o_proj"]
    assert list(sg["module/layer_keys"]) == sorted(
        f"model.layers.3.self_attn.o_proj.{s}" for s in ("mul1", "suh", "svh", "trellis"))
