"""The module-driver oracle (oracle/module_oracle.py: regularize, Hadamard,
block-LDL, LDLQ with the C encoder, reconstruction, metrics on the CPU)
pinned against the reference's own quantize_linear_module output
(tests/golden/module_golden.npz, made by tests/golden/make_golden.py)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import module_oracle as mo


def test_module_oracle_matches_reference_golden(module_golden_arrays):
    g = module_golden_arrays
    W = torch.from_numpy(g["W"])
    H = torch.from_numpy(g["H"])
    r = mo.quantize_module(W, H, K=2, buf=64)
    np.testing.assert_allclose(r.reg_weight.numpy(), g["reg_weight"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r.su.numpy(), g["su"], rtol=1e-6)
    np.testing.assert_allclose(r.sv.numpy(), g["sv"], rtol=1e-6)
    np.testing.assert_allclose(r.L.numpy(), g["L"], rtol=1e-4, atol=1e-5)
    same = (r.encoded.numpy() == g["encoded"]).all(axis=-1).mean()
    assert same == 1.0, f"identical tiles {same:.3f}"
    rel = np.linalg.norm(r.w_hat.numpy() - g["w_hat"]) / np.linalg.norm(g["w_hat"])
    assert rel <= 1e-5
    np.testing.assert_allclose(np.array(r.metrics), g["metrics"], rtol=1e-4)


def test_block_ldl_and_hadamard_properties():
    gen = torch.Generator().manual_seed(5)
    A = torch.randn(256, 64, generator=gen)
    H = A @ A.T / 64 + 0.1 * torch.eye(256)
    L, chol, retries = mo.block_ldl(H)
    assert retries == 0
    assert torch.allclose(chol @ chol.T, H, atol=1e-4)
    for s in range(0, 256, 16):
        assert torch.equal(L[s:s + 16, s:s + 16], torch.eye(16))
    x = torch.randn(256, 384, generator=gen)
    y = mo.had_r_(mo.had_l_(x.clone()))
    assert abs(float(torch.linalg.norm(y) / torch.linalg.norm(x)) - 1.0) < 1e-5  # orthonormal
