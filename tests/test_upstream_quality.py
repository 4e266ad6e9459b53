"""Upstream's encode checks (the reference's tests/test_upstream_encode_oracle.py:56-161,
from exllamav3 tests/test_quant_fn.py): per-K reconstruction MSE ceilings on
seeded N(0, scale^2) tiles, the tail-biting invariant, and the state layout
the container relies on. CPU: the reference's own outputs (golden) and the
host format code; GPU: the B200 encoder over K = 1..8 x 3 codebooks."""

from __future__ import annotations

import numpy as np
import pytest

from exl3_intel_arc_quantizer_b200 import trellis_format as tf

# Upstream's per-K MSE ceilings (test_upstream_encode_oracle.py:56-65).
MAX_MSE_PER_K = {1: 0.3, 2: 0.1, 3: 0.1, 4: 0.1, 5: 0.1, 6: 0.07, 7: 0.05, 8: 0.04}
# (codebook, input scale) pairs (upstream test_quant_fn.py:64).
CODEBOOK_CASES = ((tf.CB_3INST, 1.24371088), (tf.CB_MCG, 1.24371088), (tf.CB_MUL1, 1.0))


def upstream_tiles(batch: int, scale: float, seed: int = 0) -> np.ndarray:
    import torch

    torch.manual_seed(seed)
    return (torch.randn((batch, 256)) * scale).numpy().astype(np.float32)


def tail_biting(idx: np.ndarray, K: int) -> None:
    first = (idx[:, 0].astype(np.int64) & 0xFFFF) >> K
    last = idx[:, -1].astype(np.int64) & ((1 << (16 - K)) - 1)
    np.testing.assert_array_equal(first, last)


@pytest.mark.parametrize("cb,scale", CODEBOOK_CASES)
@pytest.mark.parametrize("K", [2, 3, 4])
def test_reference_outputs_meet_upstream_ceilings(enc_golden, K, cb, scale):
    """The golden (the reference encoder on upstream's tiles) passes
    upstream's checks, so the bit-exact device results do too."""
    name = f"upstream_k{K}_cb{cb}"
    tiles = enc_golden[f"{name}/tiles"]
    np.testing.assert_array_equal(tiles, upstream_tiles(1, scale))
    idx = enc_golden[f"{name}/indices"]
    recon = tf.codebook_lut(cb)[idx].astype(np.float32)
    assert float(np.mean(((tiles - recon) / scale) ** 2)) < MAX_MSE_PER_K[K]
    tail_biting(idx, K)


def test_symbol_occupies_the_low_k_bits():
    """Upstream's ideal-encoding construction (test_quant_fn.py:98-112): an
    element's K-bit symbol is the low K bits of its state, the preceding
    symbols shifted up."""
    K = 4
    rng = np.random.default_rng(0)
    symbols = rng.integers(0, 1 << K, size=256, dtype=np.int64)
    states = symbols.copy()
    for shift in range(1, int(np.ceil(16 / K))):
        states |= (np.roll(symbols, shift) << (K * shift)) & 0xFFFF
    np.testing.assert_array_equal(states & ((1 << K) - 1), symbols)
    np.testing.assert_array_equal((states >> K) & ((1 << K) - 1), np.roll(symbols, 1))
    # a valid tail-biting stream: the container round-trips it exactly
    back = tf.decode_states(tf.swap16_storage(tf.pack_trellis(states.astype(np.uint16), K)), K)
    np.testing.assert_array_equal(back, states)


@pytest.mark.parametrize("K", range(1, 9))
def test_packed_container_carries_the_low_bits(K):
    rng = np.random.default_rng(K)
    states = rng.integers(0, 65536, size=256, dtype=np.uint16)
    packed = tf.pack_trellis(states, K)
    assert packed.size == 256 * K // 16
    back = tf.decode_states(tf.swap16_storage(packed), K)
    np.testing.assert_array_equal(back & ((1 << K) - 1), states.astype(np.int64) & ((1 << K) - 1))


@pytest.mark.gpu
@pytest.mark.parametrize("K", range(1, 9))
def test_device_encoder_meets_upstream_ceilings(K):
    """64 of upstream's seeded tiles per codebook through the B200 encoder:
    MSE below upstream's ceiling for K, every tile tail-biting, and the
    container decodes to the states."""
    import torch

    from exl3_intel_arc_quantizer_b200.xpu_quantizer import XPUTrellisEncoder

    for cb, scale in CODEBOOK_CASES:
        tiles = upstream_tiles(64, scale)
        enc = XPUTrellisEncoder(K=K, cb=cb)
        w, i, packed, _ = enc.encode_device(torch.from_numpy(tiles).cuda())
        torch.cuda.synchronize()
        recon = w.cpu().numpy()
        idx = i.cpu().numpy().view(np.uint16)
        mse = float(np.mean(((tiles - recon) / scale) ** 2))
        assert mse < MAX_MSE_PER_K[K], (K, cb, mse)
        tail_biting(idx, K)
        np.testing.assert_array_equal(recon.astype(np.float16).view(np.uint16),
                                      tf.codebook_lut(cb)[idx].view(np.uint16))
        pk = packed.cpu().numpy().view(np.uint16)
        for t in range(0, 64, 9):
            np.testing.assert_array_equal(tf.decode_states(pk[t], K), idx[t])
        enc.arena.release()
