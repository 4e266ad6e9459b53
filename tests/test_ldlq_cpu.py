"""LDLQ loop and block-LDL host logic on CPU tensors.

The loop is device-agnostic torch orchestration around a tile-encoder
callback; these tests pin it the way the reference's tests/test_ldlq_loop.py
and tests/test_ldlq.py do (fake encoders, a naive dense restatement, identity
L, added correction, span invariance, layout, validation), and bit for bit
against the reference's own LDLQ golden vectors with the CPU oracle as the
encoder.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from exl3_intel_arc_quantizer_b200.ldlq import LDLQResult, block_ldl, ldlq
from exl3_intel_arc_quantizer_b200.trellis_format import tensor_core_perm, tensor_core_perm_inv
from oracle.trellis_oracle import COracle


class GridEncoder:
    def __init__(self, step=0.25):
        self.step = step

    def __call__(self, tiles):
        idx = torch.arange(tiles.numel(), dtype=torch.int64).reshape(tiles.shape) % 65536
        return torch.round(tiles / self.step) * self.step, idx


class LinearEncoder:
    def __call__(self, tiles):
        idx = torch.arange(tiles.numel(), dtype=torch.int64).reshape(tiles.shape) % 65536
        return tiles * 1.1 + 0.05, idx


class RecordingEncoder:
    def __init__(self):
        self.inputs = []

    def __call__(self, tiles):
        self.inputs.append(tiles.clone())
        return torch.zeros_like(tiles), torch.zeros(tiles.shape, dtype=torch.int16)


class OracleEncoder:
    """The CPU oracle as the LDLQ callback (checker only)."""

    def __init__(self, K):
        self.o = COracle(K, 2)
        self.K = K

    def __call__(self, tiles):
        r = self.o.encode_batch(tiles.numpy())
        return (torch.from_numpy(r["recon"].astype(np.float32)),
                torch.from_numpy(r["indices"].view(np.int16)))


def rows_to_tiles(rows):
    tn = rows.shape[1] // 16
    return torch.stack([rows[:, t * 16:(t + 1) * 16].reshape(-1) for t in range(tn)])


def tiles_to_rows(tiles, n):
    out = torch.empty(16, n, dtype=tiles.dtype)
    for t in range(n // 16):
        out[:, t * 16:(t + 1) * 16] = tiles[t].reshape(16, 16)
    return out


def naive_ldlq(weight, L, encode, buf):
    """Dense index-explicit restatement (global indices, explicit tile loops)."""
    k, n = weight.shape
    perm = torch.as_tensor(tensor_core_perm())
    inv = torch.as_tensor(tensor_core_perm_inv())
    prod = torch.zeros((k, n))
    wq = torch.zeros((k, n))
    enc = torch.zeros((k // 16, n // 16, 256), dtype=torch.int16)
    for i in range(k - buf, -1, -buf):
        bw = weight[i:i + buf].clone()
        bq = torch.zeros_like(bw)
        for bi in range(buf - 16, -1, -16):
            bj = bi + 16
            err = bw[bj:] - bq[bj:]
            comp = prod[i + bi:i + bj].clone()
            if err.shape[0] > 0:
                comp = comp + L[i + bj:i + buf, i + bi:i + bj].T @ err
                prod[i + bi:i + bj] = comp
            qw, qi = encode(rows_to_tiles(bw[bi:bj] + comp)[:, perm])
            bq[bi:bj] = tiles_to_rows(qw[:, inv], n)
            enc[(i + bi) // 16] = qi.to(torch.int16)
        prod = prod + L[i:i + buf].T @ (bw - bq)
        wq[i:i + buf] = bq
    return wq, enc


def correlated_L(k, rank=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(k, rank, generator=g)
    H = a @ a.T + 0.05 * torch.eye(k)
    return H, block_ldl(H).transformed


def test_identity_L_is_independent_tile_quantization():
    torch.manual_seed(1)
    w = torch.randn(64, 128)
    L = block_ldl(torch.eye(64)).transformed
    assert torch.equal(L, torch.eye(64))
    enc = GridEncoder()
    res = ldlq(w, L, enc, buf_size_k=64)
    perm, inv = torch.as_tensor(tensor_core_perm()), torch.as_tensor(tensor_core_perm_inv())
    for b in range(4):
        qw, _ = enc(rows_to_tiles(w[16 * b:16 * b + 16])[:, perm])
        assert torch.equal(res.weight_q[16 * b:16 * b + 16], tiles_to_rows(qw[:, inv], 128))


def test_correction_is_added_through_strictly_lower_L():
    torch.manual_seed(3)
    w = torch.randn(32, 128)
    _, L = correlated_L(32, seed=4)
    rec = RecordingEncoder()
    ldlq(w, L, rec, buf_size_k=32)
    inv = torch.as_tensor(tensor_core_perm_inv())
    assert torch.equal(tiles_to_rows(rec.inputs[0][:, inv], 128), w[16:32])
    expected = w[0:16] + L[16:32, 0:16].T @ w[16:32]
    assert torch.allclose(tiles_to_rows(rec.inputs[1][:, inv], 128), expected, atol=1e-6)


@pytest.mark.parametrize("buf", [16, 32, 64])
def test_matches_naive_restatement(buf):
    torch.manual_seed(7)
    w = torch.randn(64, 128)
    _, L = correlated_L(64, seed=8)
    res = ldlq(w, L, LinearEncoder(), buf_size_k=buf)
    wq, enc = naive_ldlq(w, L, LinearEncoder(), buf)
    assert torch.allclose(res.weight_q, wq, atol=1e-5)
    assert torch.equal(res.encoded, enc)


def test_feedback_lowers_weighted_error_and_span_invariance():
    torch.manual_seed(9)
    w = torch.randn(64, 128) * 0.5
    H, L = correlated_L(64, rank=6, seed=10)
    fb = ldlq(w, L, GridEncoder(0.25), buf_size_k=32)
    nofb = ldlq(w, torch.diag(torch.diag(L)), GridEncoder(0.25), buf_size_k=32)

    def obj(r):
        e = w - r.weight_q
        return float(((H @ e) * e).sum() / ((H @ w) * w).sum())

    assert obj(fb) < obj(nofb)
    torch.manual_seed(11)
    w2 = torch.randn(128, 128)
    _, L2 = correlated_L(128, seed=12)
    a = ldlq(w2, L2, GridEncoder(0.3), buf_size_k=16)
    b = ldlq(w2, L2, GridEncoder(0.3), buf_size_k=128)
    assert torch.allclose(a.weight_q, b.weight_q, atol=1e-5)
    assert torch.equal(a.encoded, b.encoded)


def test_layout_validation_and_immutability():
    class TileId:
        def __call__(self, tiles):
            return tiles, torch.arange(tiles.shape[0]).reshape(-1, 1).expand(-1, 256)

    res = ldlq(torch.randn(32, 256), torch.eye(32), TileId(), buf_size_k=32)
    assert isinstance(res, LDLQResult) and res.encoded.shape == (2, 16, 256)
    assert res.encoded.dtype == torch.int16
    assert all(bool((res.encoded[r, t] == t).all()) for r in range(2) for t in range(16))
    w, L = torch.randn(32, 128), torch.eye(32)
    w0, L0 = w.clone(), L.clone()
    ldlq(w, L, GridEncoder(0.5), buf_size_k=32)
    assert torch.equal(w, w0) and torch.equal(L, L0)
    for bad in (lambda: ldlq(torch.randn(32), L, GridEncoder()),
                lambda: ldlq(w.double(), L, GridEncoder()),
                lambda: ldlq(torch.randn(30, 128), torch.eye(30), GridEncoder()),
                lambda: ldlq(w, torch.eye(48), GridEncoder()),
                lambda: ldlq(w, L, GridEncoder(), buf_size_k=24),
                lambda: ldlq(w, L, GridEncoder(), buf_size_k=48),
                lambda: ldlq(w, L, lambda t: (t[:-1], torch.zeros(t.shape)), 32)):
        with pytest.raises(ValueError):
            bad()


def test_block_ldl_contract():
    g = torch.Generator().manual_seed(7)
    A = torch.randn(64, 64, generator=g)
    H = (A @ A.T / 64 + torch.eye(64)).float()
    r = block_ldl(H, block_size=16)
    assert r.retries == 0 and not r.damping_applied
    assert torch.allclose(r.cholesky @ r.cholesky.T, H, atol=1e-4)
    for b in range(4):
        s = slice(16 * b, 16 * b + 16)
        assert torch.allclose(r.transformed[s, s], torch.eye(16), atol=1e-6)
        exp = r.cholesky[:, s] @ r.block_inverses[b]
        exp[s, :] = torch.eye(16)
        assert torch.allclose(r.transformed[:, s], exp, atol=1e-5)
    Q, _ = torch.linalg.qr(torch.randn(32, 32, generator=torch.Generator().manual_seed(3)))
    ev = torch.full((32,), 100.0)
    ev[-1] = -0.5
    Hn = (Q @ torch.diag(ev) @ Q.T).float()
    rn = block_ldl(Hn, block_size=16)
    assert 1 <= rn.retries <= 10 and rn.damping_applied
    with pytest.raises(torch.linalg.LinAlgError):
        block_ldl(-torch.eye(16), block_size=16, max_retries=2)
    for bad in (lambda: block_ldl(torch.randn(63, 63)), lambda: block_ldl(torch.randn(64, 63)),
                lambda: block_ldl(H.double()), lambda: block_ldl(H, block_size=0),
                lambda: block_ldl(H, block_size=128), lambda: block_ldl(H, max_retries=-1)):
        with pytest.raises(ValueError):
            bad()


@pytest.mark.parametrize("name", ["k2_32x128", "k4_64x128"])
def test_ldlq_reproduces_reference_golden_with_oracle_encoder(ldlq_golden, name):
    """Same loop op sequence on CPU tensors + the oracle encoder -> the
    reference's weight_q and encoded, bit for bit."""
    K, k, n, buf, seed = (int(v) for v in ldlq_golden[f"{name}/params"])
    w = torch.from_numpy(ldlq_golden[f"{name}/weight"])
    L = torch.from_numpy(ldlq_golden[f"{name}/L"])
    res = ldlq(w, L, OracleEncoder(K), buf_size_k=buf)
    assert torch.equal(res.weight_q, torch.from_numpy(ldlq_golden[f"{name}/weight_q"]))
    assert torch.equal(res.encoded, torch.from_numpy(ldlq_golden[f"{name}/encoded"]))


@pytest.mark.parametrize("name", ["k2_32x128", "k4_64x128"])
def test_fixed_order_ldlq_oracle_reproduces_reference_golden(ldlq_golden, name):
    """The fixed-summation-order restatement (the order of the device loop)
    gives the reference's own LDLQ output bit for bit on both golden cases."""
    from oracle.ldlq_oracle import ldlq_fixed_order
    from oracle.module_oracle import c_encoder

    K, k, n, buf, seed = (int(v) for v in ldlq_golden[f"{name}/params"])
    wq, enc = ldlq_fixed_order(torch.from_numpy(ldlq_golden[f"{name}/weight"]),
                               torch.from_numpy(ldlq_golden[f"{name}/L"]), c_encoder(K), buf)
    assert torch.equal(wq, torch.from_numpy(ldlq_golden[f"{name}/weight_q"]))
    assert torch.equal(enc, torch.from_numpy(ldlq_golden[f"{name}/encoded"]))


def test_fixed_order_ldlq_oracle_matches_the_loop_with_exact_products():
    """With a grid encoder (no trellis), the fixed-order loop and the torch
    loop differ only by the summation order of their products: the results
    agree to fp32 rounding, and the fixed order is the same on every call."""
    from oracle.ldlq_oracle import ldlq_fixed_order

    g = torch.Generator().manual_seed(5)
    w = torch.randn(256, 256, generator=g)
    _, L = correlated_L(256, seed=3)
    enc = GridEncoder(0.5)
    a = ldlq(w, L, enc, buf_size_k=64)
    b_q, b_e = ldlq_fixed_order(w, L, enc, buf=64)
    c_q, _ = ldlq_fixed_order(w, L, enc, buf=64)
    assert torch.equal(b_q, c_q)
    assert float((a.weight_q - b_q).abs().max()) <= 0.5 + 1e-6      # at most one grid step
    assert float((a.weight_q - b_q).norm() / a.weight_q.norm()) < 0.05
