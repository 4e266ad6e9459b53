"""Pin the CPU oracle against golden vectors produced by the reference itself.

The golden files come from tests/golden/make_golden.py, which runs the
reference's ReferenceTrellisEncoder / trellis_format / forward pass. Both
oracle restatements (C and NumPy) must reproduce them bit for bit before any
GPU result is compared with the oracle.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle.trellis_oracle import (
    COracle,
    NumpyOracle,
    codebook_lut,
    decode_states,
    pack_trellis,
    swap16_storage,
    tensor_core_perm,
    tensor_core_perm_inv,
)


def _case_input(enc_golden, case):
    tiles = enc_golden[f"{case['name']}/tiles"]
    return tiles[:, tensor_core_perm()] if case["pre_permute"] else tiles


def test_c_oracle_matches_every_golden_encode(manifest, enc_golden):
    """All 364 reference-encoded tiles: indices, recon, packed, end state, path cost."""
    for case in manifest["encoder"]:
        name = case["name"]
        r = COracle(case["K"], case["cb"], case["L"]).encode_batch(_case_input(enc_golden, case))
        np.testing.assert_array_equal(r["indices"], enc_golden[f"{name}/indices"], err_msg=name)
        np.testing.assert_array_equal(r["recon"].view(np.uint16), enc_golden[f"{name}/recon_perm"],
                                      err_msg=name)
        np.testing.assert_array_equal(r["end_state"], enc_golden[f"{name}/end_state"], err_msg=name)
        np.testing.assert_array_equal(r["path_cost"].view(np.uint16),
                                      enc_golden[f"{name}/path_cost"], err_msg=name)
        if case["L"] == 256:
            np.testing.assert_array_equal(r["packed"], enc_golden[f"{name}/packed"], err_msg=name)


@pytest.mark.parametrize("name", ["parity_k2_cb1", "nonfinite_k4", "l160_k2", "cfg2_k7_mul1",
                                  "saturate_k3"])
def test_numpy_oracle_matches_golden(manifest, enc_golden, name):
    case = next(c for c in manifest["encoder"] if c["name"] == name)
    x = _case_input(enc_golden, case)[:2]
    o = NumpyOracle(case["K"], case["cb"], case["L"])
    for i in range(len(x)):
        r = o.encode(x[i])
        np.testing.assert_array_equal(r["indices"], enc_golden[f"{name}/indices"][i])
        assert r["end_state"] == enc_golden[f"{name}/end_state"][i]
        assert np.float16(r["path_cost"]).view(np.uint16) == enc_golden[f"{name}/path_cost"][i]


def test_forward_pass_audits(manifest, fwd_golden):
    """test_forward_semantics.py cases: predecessor table hash + final costs."""
    for case in manifest["forward"]:
        name = case["name"]
        w16 = fwd_golden[f"{name}/w16"].view(np.float16)
        edges, costs = COracle(case["K"], 2).forward(w16, case["roll"], case["pre_state"])
        assert hashlib.sha256(edges.tobytes()).hexdigest() == case["edges_sha256"], name
        np.testing.assert_array_equal(costs.view(np.uint16), fwd_golden[f"{name}/costs"])
        if name == "inf_k2":
            assert not np.isnan(costs.astype(np.float64)).any()


def test_format_primitives(manifest, fmt_golden):
    for cb in (0, 1, 2):
        lut = codebook_lut(cb).view(np.uint16)
        assert hashlib.sha256(lut.tobytes()).hexdigest() == manifest["format"][f"lut{cb}_sha256"]
        assert np.array_equal(COracle(2, cb).codebook().view(np.uint16), lut)
    np.testing.assert_array_equal(tensor_core_perm(), fmt_golden["perm"])
    np.testing.assert_array_equal(tensor_core_perm()[tensor_core_perm_inv()], np.arange(256))
    for K in range(1, 9):
        st = fmt_golden[f"pack_k{K}/states"]
        np.testing.assert_array_equal(pack_trellis(st, K), fmt_golden[f"pack_k{K}/packed"])
        stored = swap16_storage(pack_trellis(st, K))
        np.testing.assert_array_equal(stored, fmt_golden[f"pack_k{K}/stored"])
        np.testing.assert_array_equal(decode_states(stored, K), fmt_golden[f"pack_k{K}/decoded"])


def test_planted_mistake_is_detected(enc_golden):
    """The checker must notice a one-state difference (mutation planted in the
    oracle's output on the CPU)."""
    r = COracle(2, 2).encode_batch(enc_golden["cfg1_k2_mul1/tiles"][:1])
    idx = r["indices"].copy()
    idx[0, 37] ^= 1
    assert not np.array_equal(idx, enc_golden["cfg1_k2_mul1/indices"][:1])
