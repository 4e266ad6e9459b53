"""The cluster encoder's bounded waits report a timeout to the caller.

The test hook makes every CTA of the cluster-split ACS stop sending cost
words at the same step (so no message is in flight) and shortens the wait
limit to 5 ms: the next waits run out, the CTAs finish without waiting, and
the fault count on the device grows. The encoder API and the module driver
must raise EncoderFault instead of returning the invalid states; afterwards
the hook is cleared and the same device encodes bit-exactly again (the
context stays usable).
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200._ext import (  # noqa: E402
    EncoderFault,
    encoder_fault_count,
    set_cluster_wait_test_hook,
    set_encoder_cluster,
)
from exl3_intel_arc_quantizer_b200.layer_quant import quantize_linear_module  # noqa: E402
from exl3_intel_arc_quantizer_b200.xpu_quantizer import XPUTrellisEncoder  # noqa: E402
from oracle.trellis_oracle import COracle  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _tiles(n, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, 256), dtype=np.float32)
            * np.exp(0.5 * rng.standard_normal((n, 1))).astype(np.float32))


def test_timed_out_cluster_wait_raises_and_the_device_recovers():
    tiles = _tiles(16, 5)
    enc = XPUTrellisEncoder(K=2)
    g = torch.Generator().manual_seed(2)
    W = (torch.randn(128, 256, generator=g) * 0.02).to(DEV)
    X = torch.randn(512, 128, generator=g)
    H = (X.T @ X / 512 + 0.01 * torch.eye(128)).to(DEV)
    before = encoder_fault_count()
    set_encoder_cluster(8)
    set_cluster_wait_test_hook(5_000_000, 3)
    try:
        with pytest.raises(EncoderFault):
            enc.encode_batch_detailed(tiles, pre_permute=False)
        with pytest.raises(EncoderFault):
            quantize_linear_module("m", W, H, K=2, tile_encoder=None, buf_size_k=64)
    finally:
        set_cluster_wait_test_hook(0, -1)
        set_encoder_cluster(0)
    assert encoder_fault_count() > before
    with pytest.raises(RuntimeError):
        set_cluster_wait_test_hook(10, 3)        # below the smallest accepted limit
    with pytest.raises(RuntimeError):
        set_cluster_wait_test_hook(0, 255)       # beyond the last step that sends
    # hook cleared: the same device and encoder are exact again, with no new faults
    mid = encoder_fault_count()
    set_encoder_cluster(8)
    try:
        res = enc.encode_batch_detailed(tiles, pre_permute=False)
    finally:
        set_encoder_cluster(0)
    ref = COracle(2).encode_batch(tiles)
    assert np.array_equal(res.output_indices, ref["indices"])
    assert encoder_fault_count() == mid
    enc.arena.release()
