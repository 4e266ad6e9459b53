"""Cluster-split ACS passes (2, 4 or 8 CTAs per tile pair exchanging the
cost vector through distributed shared memory) against the C oracle and
against the one-CTA-per-pair kernel: bit-exact states, container and path
cost for K = 2..6, every codebook, NaN pairs, L=160, odd tile counts, more
pairs than resident clusters; no bounded inter-CTA wait ever gives up.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200 import trellis_format as tf  # noqa: E402
from exl3_intel_arc_quantizer_b200._ext import (  # noqa: E402
    encoder_cluster_capacity,
    encoder_fault_count,
    set_encoder_cluster,
    set_encoder_cluster_pairs,
)
from exl3_intel_arc_quantizer_b200.xpu_quantizer import XPUTrellisEncoder  # noqa: E402
from oracle.trellis_oracle import COracle  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
SIZES = (1, 2, 4, 8)


def _tiles(n, seed, L=256):
    rng = np.random.default_rng(seed)
    base = rng.standard_normal((n, L), dtype=np.float32)
    scale = np.exp(0.5 * rng.standard_normal((n, 1))).astype(np.float32)
    return base * scale


def _encode(K, cb, tiles, cluster, L=256, pairs=0):
    set_encoder_cluster(cluster)
    set_encoder_cluster_pairs(pairs)
    try:
        enc = XPUTrellisEncoder(K=K, cb=cb, tile_len=L)
        w, i, packed, cost = enc.encode_device(torch.from_numpy(tiles).to(DEV),
                                               want_packed=L == 256)
        out = (i.cpu().numpy().view(np.uint16), None if packed is None else packed.cpu().numpy(),
               np.float16(cost.cpu().numpy()).view(np.uint16), w.cpu().numpy())
        enc.arena.release()
        return out
    finally:
        set_encoder_cluster(0)
        set_encoder_cluster_pairs(0)


def _same_cost(got, want, msg):
    """fp16 path-cost bits equal; a NaN tile's cost is NaN on both sides (the
    GPU's canonical NaN payload differs from NumPy's)."""
    g_nan = (got & 0x7C00) == 0x7C00
    g_nan &= (got & 0x03FF) != 0
    w_nan = (want & 0x7C00) == 0x7C00
    w_nan &= (want & 0x03FF) != 0
    np.testing.assert_array_equal(g_nan, w_nan, err_msg=msg)
    np.testing.assert_array_equal(got[~g_nan], want[~w_nan], err_msg=msg)


@pytest.fixture(autouse=True)
def _no_faults():
    before = encoder_fault_count()
    yield
    assert encoder_fault_count() == before


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6])
def test_cluster_sizes_match_c_oracle(K):
    n = 9  # odd: the last pair repeats its A tile
    tiles = _tiles(n, 7100 + K)
    ref = COracle(K, tf.CB_MUL1).encode_batch(tiles)
    for c in SIZES:
        idx, packed, cost, _ = _encode(K, tf.CB_MUL1, tiles, c)
        np.testing.assert_array_equal(idx, ref["indices"], err_msg=f"cluster {c}")
        np.testing.assert_array_equal(packed.view(np.uint16), ref["packed"], err_msg=f"cluster {c}")
        _same_cost(cost, ref["path_cost"].view(np.uint16), f"cluster {c}")


@pytest.mark.parametrize("cb", [tf.CB_3INST, tf.CB_MCG, tf.CB_MUL1])
def test_cluster_codebooks_and_nan_pairs(cb):
    K = 3
    tiles = _tiles(6, 7200 + cb)
    tiles[1, 17] = np.nan          # pair 0 runs compare-and-select
    tiles[4, :] = 0.0              # all-zero tile: ties everywhere
    ref = COracle(K, cb).encode_batch(tiles)
    for c in SIZES:
        idx, packed, cost, _ = _encode(K, cb, tiles, c)
        np.testing.assert_array_equal(idx, ref["indices"], err_msg=f"cluster {c}")
        np.testing.assert_array_equal(packed.view(np.uint16), ref["packed"], err_msg=f"cluster {c}")
        _same_cost(cost, ref["path_cost"].view(np.uint16), f"cluster {c}")


def test_cluster_l160():
    tiles = _tiles(4, 7300, L=160)
    ref = COracle(2, tf.CB_MUL1, L=160).encode_batch(tiles)
    for c in SIZES:
        idx, _, cost, _ = _encode(2, tf.CB_MUL1, tiles, c, L=160)
        np.testing.assert_array_equal(idx, ref["indices"], err_msg=f"cluster {c}")
        _same_cost(cost, ref["path_cost"].view(np.uint16), f"cluster {c}")


@pytest.mark.parametrize("K", [2, 4])
def test_more_pairs_than_resident_clusters(K):
    """400 tiles = 200 pairs: forced clusters loop over pairs (persistent)."""
    tiles = _tiles(400, 7400 + K)
    base = _encode(K, tf.CB_MUL1, tiles, 1)
    for c in (2, 4, 8):
        got = _encode(K, tf.CB_MUL1, tiles, c)
        for a, b, what in zip(got, base, ("indices", "packed", "cost", "recon")):
            np.testing.assert_array_equal(a, b, err_msg=f"cluster {c} {what}")


def test_automatic_policy_matches_off():
    """Typical LDLQ step sizes of a column-sharded module (4..64 tiles)."""
    for n in (4, 32, 64):
        tiles = _tiles(n, 7500 + n)
        off = _encode(2, tf.CB_MUL1, tiles, 1)
        auto = _encode(2, tf.CB_MUL1, tiles, 0)
        for a, b in zip(auto, off):
            np.testing.assert_array_equal(a, b)


def test_cluster_capacity_and_policy_validation():
    for K in (2, 3, 4, 5, 6):
        assert encoder_cluster_capacity(K, 8) >= 1
        assert encoder_cluster_capacity(K, 2) >= encoder_cluster_capacity(K, 8)
    for K in (1, 7, 8):
        assert encoder_cluster_capacity(K, 4) == 0
    with pytest.raises(RuntimeError):
        set_encoder_cluster(3)
    with pytest.raises(RuntimeError):
        encoder_cluster_capacity(2, 16)


@pytest.mark.parametrize("K", [2, 4])
def test_last_partial_wave_split_matches_off(K):
    """More pairs than SMs with a small remainder: the whole waves run one
    pair per CTA and the last 11 pairs (one of them a lone tile) over
    clusters; identical to running everything one pair per CTA."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = 2 * (sms + 10) + 1
    tiles = _tiles(n, 7600 + K)
    off = _encode(K, tf.CB_MUL1, tiles, 1)
    auto = _encode(K, tf.CB_MUL1, tiles, 0)
    for a, b, what in zip(auto, off, ("indices", "packed", "cost", "recon")):
        np.testing.assert_array_equal(a, b, err_msg=what)
    ref = COracle(K, tf.CB_MUL1).encode_batch(tiles[-24:])   # the tail pairs, checked whole
    np.testing.assert_array_equal(auto[0][-24:], ref["indices"])


@pytest.mark.parametrize("K", [2, 3, 4, 5, 6])
@pytest.mark.parametrize("pairs", [2])
def test_several_pairs_per_cluster_match_c_oracle(K, pairs):
    """Clusters of 8 CTAs serving 2 tile pairs per exchange round; 11
    tiles: the last group repeats its first pair (and the last pair is a
    lone tile), so groups with missing pairs and odd tile counts are covered."""
    n = 11
    tiles = _tiles(n, 7700 + 10 * K + pairs)
    tiles[3, 40] = np.nan            # a NaN pair inside a group: compare-and-select
    ref = COracle(K, tf.CB_MUL1).encode_batch(tiles)
    idx, packed, cost, recon = _encode(K, tf.CB_MUL1, tiles, 8, pairs=pairs)
    np.testing.assert_array_equal(idx, ref["indices"])
    np.testing.assert_array_equal(packed.view(np.uint16), ref["packed"])
    _same_cost(cost, ref["path_cost"].view(np.uint16), f"{pairs} pairs per cluster")


@pytest.mark.parametrize("K", [2, 4])
def test_several_pairs_per_cluster_more_groups_than_clusters(K):
    """200 pairs in groups of 2 over the resident clusters of 8 CTAs (the
    clusters loop over groups): identical to one pair per CTA."""
    tiles = _tiles(400, 7800 + K)
    base = _encode(K, tf.CB_MUL1, tiles, 1)
    for pairs in (2,):
        got = _encode(K, tf.CB_MUL1, tiles, 8, pairs=pairs)
        for a, b, what in zip(got, base, ("indices", "packed", "cost", "recon")):
            np.testing.assert_array_equal(a, b, err_msg=f"{pairs} pairs {what}")


def test_automatic_policy_with_several_pairs_matches_off():
    """Call sizes whose pairs exceed the resident clusters of 8 CTAs (the
    automatic choice then groups pairs): identical to no split."""
    for K in (2, 4):
        for n in (32, 40, 64, 96):
            tiles = _tiles(n, 7900 + n + K)
            off = _encode(K, tf.CB_MUL1, tiles, 1)
            auto = _encode(K, tf.CB_MUL1, tiles, 0)
            for a, b in zip(auto, off):
                np.testing.assert_array_equal(a, b)
    with pytest.raises(RuntimeError):
        set_encoder_cluster_pairs(4)
