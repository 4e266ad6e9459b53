"""Product format module (host side) against the reference's golden vectors,
plus the round-trip properties of the reference's format tests."""

from __future__ import annotations

import hashlib

import numpy as np

from exl3_intel_arc_quantizer_b200 import trellis_format as tf


def test_codebooks_match_reference(manifest):
    for cb in (0, 1, 2):
        lut = tf.codebook_lut(cb).view(np.uint16)
        assert hashlib.sha256(lut.tobytes()).hexdigest() == manifest["format"][f"lut{cb}_sha256"]


def test_perm_and_pack_match_reference(fmt_golden):
    np.testing.assert_array_equal(tf.tensor_core_perm(), fmt_golden["perm"])
    for K in range(1, 9):
        st = fmt_golden[f"pack_k{K}/states"]
        np.testing.assert_array_equal(tf.pack_trellis(st, K), fmt_golden[f"pack_k{K}/packed"])
        stored = tf.swap16_storage(tf.pack_trellis(st, K))
        np.testing.assert_array_equal(stored, fmt_golden[f"pack_k{K}/stored"])
        np.testing.assert_array_equal(tf.decode_states(stored, K), fmt_golden[f"pack_k{K}/decoded"])


def test_encoded_tiles_round_trip(manifest, enc_golden):
    """Reference-encoded containers decode back to their states and values."""
    for case in manifest["encoder"]:
        if case["L"] != 256 or not case["pre_permute"]:
            continue
        name, K, cb = case["name"], case["K"], case["cb"]
        for t in range(case["n"]):
            packed = enc_golden[f"{name}/packed"][t]
            np.testing.assert_array_equal(tf.decode_states(packed, K),
                                          enc_golden[f"{name}/indices"][t])
            np.testing.assert_array_equal(tf.decode_tile_values(packed, K, cb).view(np.uint16),
                                          enc_golden[f"{name}/recon"][t])


def test_swap16_pairing_and_validation():
    assert tf.swap16_storage(np.array([0x1111, 0x2222, 0x3333, 0x4444], np.uint16)).tolist() == [
        0x2222, 0x1111, 0x4444, 0x3333]
    import pytest

    with pytest.raises(ValueError):
        tf.pack_trellis(np.zeros(255, np.uint16), 2)
    with pytest.raises(ValueError):
        tf.pack_trellis(np.zeros(256, np.uint16), 9)
    with pytest.raises(ValueError):
        tf.codebook_lut(7)
