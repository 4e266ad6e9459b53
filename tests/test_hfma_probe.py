"""fp16 FMA rounding of the encoder's metric: the reference's O-6 probes
(tests/test_xpu_extension.py:64-80 over exl3_quant/xpu_probe.py:153-270),
plus the exhaustive grid the adversarial table was drawn from
(xpu_probe.py:212-218), run through both instructions the encoder issues:
the ACS kernels' packed fma.rn.f16x2 (mode 0) and the tracebacks' scalar
fma.rn.f16 (mode 1)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from exl3_intel_arc_quantizer_b200 import _ext
from exl3_intel_arc_quantizer_b200 import xpu_probe as xp

EINVAL = -22


def discriminating_grid():
    """Every (dh, cost) with dh mantissa pattern 0x3C00..0x3CFF and a tiny
    cost 0x0001..0x0FFF (2^-24 .. 2^-11) on which the float32 double
    rounding differs from the exact single rounding, as uint16 bits."""
    dh = np.arange(0x3C00, 0x3D00, dtype=np.uint16)
    cost = np.arange(0x0001, 0x1000, dtype=np.uint16)
    D, C = np.meshgrid(dh, cost, indexing="ij")
    D, C = D.ravel(), C.ravel()
    ex = xp.exact_hfma(D.view(np.float16), C.view(np.float16)).view(np.uint16)
    em = xp.fp32_emulated_hfma(D.view(np.float16), C.view(np.float16)).view(np.uint16)
    sel = ex != em
    return D[sel], C[sel]


def test_adversarial_table_discriminates():
    dh = np.asarray(xp.ADVERSARIAL_DH_BITS, np.uint16).view(np.float16)
    cost = np.asarray(xp.ADVERSARIAL_COST_BITS, np.uint16).view(np.float16)
    ex = xp.exact_hfma(dh, cost).view(np.uint16)
    em = xp.fp32_emulated_hfma(dh, cost).view(np.uint16)
    assert np.all(ex != em)


def test_grid_contains_the_reference_table():
    D, C = discriminating_grid()
    assert 11 <= D.size < 100000
    pairs = set(zip(D.tolist(), C.tolist()))
    for d, c in zip(xp.ADVERSARIAL_DH_BITS, xp.ADVERSARIAL_COST_BITS):
        assert (d, c) in pairs


def test_oracle_rounds_the_metric_once():
    """The C oracle's metric (trellis_oracle.c: d2h of the exact double sum)
    is the exact single rounding on every discriminating pair and on a
    random block."""
    from oracle.trellis_oracle import f64_to_f16_bits

    D, C = discriminating_grid()
    rng = np.random.default_rng(2026)
    dr = rng.normal(0.0, 1.0, 2048).astype(np.float16).view(np.uint16)
    cr = (rng.random(2048) * 8.0).astype(np.float16).view(np.uint16)
    D, C = np.concatenate([D, dr]), np.concatenate([C, cr])
    d64 = D.view(np.float16).astype(np.float64)
    got = np.array([f64_to_f16_bits(float(a * a + c))
                    for a, c in zip(d64, C.view(np.float16).astype(np.float64))], np.uint16)
    assert np.array_equal(got, xp.exact_hfma(D.view(np.float16), C.view(np.float16)).view(np.uint16))


def test_abi_argument_checks_without_a_gpu():
    lib = _ext.lib()
    f = lib.exl3_probe_hfma
    f.restype = ctypes.c_int
    P = ctypes.c_void_p
    f.argtypes = [P, P, P, ctypes.c_int64, ctypes.c_int, P]
    dummy = P(16)
    assert f(dummy, dummy, dummy, 4, 2, None) == EINVAL
    assert b"mode must be 0" in lib.exl3_last_error()
    assert f(dummy, dummy, dummy, -1, 0, None) == EINVAL
    assert f(None, dummy, dummy, 4, 1, None) == EINVAL
    assert f(None, None, None, 0, 0, None) == 0  # n == 0: nothing to do


def test_binding_rejects_host_tensors():
    import torch

    x = torch.zeros(4, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        _ext.ext().probe_hfma(x, x, x, 0)


@pytest.mark.gpu
def test_random_block_matches_exact_single_rounding():
    r = xp.run_hfma_probe()
    assert r["fma_vs_exact_mismatches"] == 0, r
    assert r["expr_vs_exact_mismatches"] == 0, r
    assert r["fma_vs_expr_mismatches"] == 0, r


@pytest.mark.gpu
def test_adversarial_table_is_single_rounded_by_both_instructions():
    r = xp.run_hfma_adversarial_probe()
    assert "error" not in r, r
    assert r["fp32_emul_vs_exact_mismatches"] == r["n"] == 11
    assert r["fma_matches_exact"] == r["n"] and r["fma_matches_fp32_emul"] == 0, r
    assert r["expr_matches_exact"] == r["n"] and r["expr_matches_fp32_emul"] == 0, r
    assert r["conclusion"] == "device fma == exact single rounding"


@pytest.mark.gpu
def test_whole_discriminating_grid_is_single_rounded():
    D, C = discriminating_grid()
    r = xp.run_hfma_adversarial_probe(dh_bits=D, cost_bits=C)
    assert r["fma_matches_exact"] == r["n"] == D.size, {k: r[k] for k in r if k != "cases"}
    assert r["expr_matches_exact"] == r["n"]
    assert r["conclusion"] == "device fma == exact single rounding"


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, 4097])
def test_odd_lengths_and_special_values(n):
    """Odd n leaves the packed path's last lane alone; inf, NaN, -0 and
    overflow operands round as IEEE fma does (numpy's float64 reference)."""
    import torch

    rng = np.random.default_rng(n)
    dh = rng.normal(0.0, 4.0, n).astype(np.float16)
    cost = (rng.random(n) * 16.0).astype(np.float16)
    special = np.array([np.inf, -np.inf, np.nan, -0.0, 300.0, 0.0], np.float16)
    dh[: min(n, special.size)] = special[: min(n, special.size)]
    ex = xp.exact_hfma(dh, cost)
    e = _ext.ext()
    dh_t = torch.from_numpy(dh).cuda()
    c_t = torch.from_numpy(cost).cuda()
    for mode in (0, 1):
        out = torch.full_like(dh_t, 7.0)
        e.probe_hfma(dh_t, c_t, out, mode)
        got = out.cpu().numpy()
        nan = np.isnan(ex)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint16), ex[~nan].view(np.uint16))


@pytest.mark.gpu
def test_binding_errors():
    import torch

    e = _ext.ext()
    h = torch.zeros(4, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="mode must be 0"):
        e.probe_hfma(h, h, h, 2)
    with pytest.raises(RuntimeError, match="equal numel"):
        e.probe_hfma(h, h, torch.zeros(3, dtype=torch.float16, device="cuda"), 0)
    with pytest.raises(RuntimeError, match="wrong dtype"):
        e.probe_hfma(h.float(), h, h, 0)
