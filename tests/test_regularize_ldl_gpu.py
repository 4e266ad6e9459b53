"""The device regularization (exl3_regularize) and block-LDL fold
(exl3_block_ldl_fold) against the reference's own functions.

The checker is the reference's ``regularize`` and ``block_ldl``
(exl3_quant/regularize.py:83-211, ldlq.py:75-132), byte-compiled from its
sources into ``oracle/_ref``, run on the CPU. Every branch of the
reference's scale logic is covered: the skew heuristic on both sides of its
0.15 cutoff, forced output scales on and off, the fallback mode, no Hessian,
a zero column (its scale floored to 0.1, its sv zeroed) and an all-zero
weight (the ``zeros`` flag). Tolerances: flags exact; skew relative 1e-6;
scales relative 1e-6; the rotated weight relative Frobenius 1e-6 (the
device's sums and its Walsh-Hadamard rotation round differently from the
reference's torch reductions and GEMM); L and the block inverses max
absolute 1e-5 of the largest entry, with the identity diagonal blocks and the
zeros above them exact.
"""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200.ldlq import block_ldl  # noqa: E402
from exl3_intel_arc_quantizer_b200.regularize import regularize  # noqa: E402
from oracle import build_ref  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not build_ref.available(),
                                 reason="compiled reference package (oracle/_ref) not built")]
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ref():
    build_ref.enable()
    try:
        import exl3_quant.ldlq as ref_ldlq
        import exl3_quant.regularize as ref_reg

        yield ref_reg, ref_ldlq
    finally:
        build_ref.disable()


def _rel(a, b):
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    den = float(torch.linalg.norm(b))
    return float(torch.linalg.norm(a - b)) / (den if den > 0 else 1.0)


def _case(name, k=256, n=384, seed=0):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(k, n, generator=g) * 0.02
    W[:, torch.randperm(n, generator=g)[:4]] *= 8.0
    hd = torch.rand(k, generator=g) + 0.5
    args, q_fallback, H = {}, False, hd
    if name == "skewed":                  # a few dominant channels: skew >= 0.15
        hd[:6] = 1e4
    elif name == "force_on":
        hd[:6] = 1e4
        args["apply_out_scales"] = True
    elif name == "force_off":
        args["apply_out_scales"] = False
    elif name == "fallback":
        q_fallback = True
    elif name == "fallback_forced":
        q_fallback, args["apply_out_scales"] = True, True
    elif name == "no_hessian":
        H = None
    elif name == "zero_column":
        W[:, 7] = 0.0
    elif name == "all_zero":
        W.zero_()
        args["apply_out_scales"] = False
    su = torch.where(torch.rand(k, 1, generator=g) < 0.5, -1.0, 1.0)
    sv = torch.where(torch.rand(1, n, generator=g) < 0.5, -1.0, 1.0)
    return W, su, sv, H, args, q_fallback


CASES = ["auto", "skewed", "force_on", "force_off", "fallback", "fallback_forced", "no_hessian",
         "zero_column", "all_zero"]


@pytest.mark.parametrize("name", CASES)
def test_regularize_matches_reference_function(ref, name):
    ref_reg, _ = ref
    W, su, sv, H, args, qf = _case(name)
    a_ref, a_dev = dict(args), dict(args)
    want = ref_reg.regularize(W.clone(), su.clone(), sv.clone(), quant_args=a_ref, H_diag=H,
                              skip_g_scale=True, q_fallback=qf)
    got = regularize(W.to(DEV), su.to(DEV), sv.to(DEV), quant_args=a_dev,
                     H_diag=None if H is None else H.to(DEV), skip_g_scale=True, q_fallback=qf)
    assert got.apply_out_scales == want.apply_out_scales, name
    assert got.zeros == want.zeros and a_dev.get("zeros") == a_ref.get("zeros"), name
    if want.skew_factor is None:
        assert got.skew_factor is None
    else:
        assert abs(got.skew_factor - want.skew_factor) <= 1e-6 * abs(want.skew_factor), name
    assert got.su.shape == want.su.shape and got.sv.shape == want.sv.shape
    for key in ("su", "sv", "out_channel_scales", "in_channel_scales"):
        g, w = getattr(got, key), getattr(want, key)
        assert g.shape == w.shape, key
        assert _rel(g, w) <= 1e-6, (name, key, _rel(g, w))
    assert torch.equal((got.sv.cpu() == 0), (want.sv == 0)), name     # zeroed columns
    assert _rel(got.weight, want.weight) <= 1e-6, (name, _rel(got.weight, want.weight))


def test_regularize_skew_selects_the_kth_largest_exactly(ref):
    """Ties and duplicates at the cutoff: the radix select counts copies."""
    ref_reg, _ = ref
    k, n = 1024, 256
    W = torch.randn(k, n) * 0.02
    hd = torch.full((k,), 4.0)
    hd[:30] = 9.0                            # cutoff k/50 = 20 lands inside the ties
    hd[30:60] = 1.0
    want = ref_reg.regularize(W.clone(), torch.ones(k, 1), torch.ones(1, n), H_diag=hd)
    got = regularize(W.to(DEV), torch.ones(k, 1, device=DEV), torch.ones(1, n, device=DEV),
                     H_diag=hd.to(DEV))
    assert abs(got.skew_factor - want.skew_factor) <= 1e-6 * want.skew_factor


@pytest.mark.parametrize("n", [256, 1024])
def test_block_ldl_fold_matches_reference_function(ref, n):
    _, ref_ldlq = ref
    g = torch.Generator().manual_seed(n)
    a = torch.randn(n, n // 2, generator=g)
    H = a @ a.T / n + 0.05 * torch.eye(n)
    want = ref_ldlq.block_ldl(H.clone(), block_size=16)
    got = block_ldl(H.to(DEV), block_size=16)
    assert got.retries == want.retries
    scale = float(want.transformed.abs().max())
    assert float((got.transformed.cpu() - want.transformed).abs().max()) <= 1e-5 * scale
    assert float((got.block_inverses.cpu() - want.block_inverses).abs().max()) <= \
        1e-5 * float(want.block_inverses.abs().max())
    L = got.transformed.cpu()
    m = n // 16
    blocks = L.reshape(m, 16, m, 16)
    for b in range(m):
        assert torch.equal(blocks[b, :, b, :], torch.eye(16))
    assert float(torch.triu(L, diagonal=1).abs().max()) == 0.0    # zeros above the diagonal


@pytest.mark.parametrize("n", [80, 208, 4096])
def test_block_ldl_fold_equals_the_torch_fold_on_the_same_factor(n):
    """On one device factor, the kernel's fold agrees with the reference op
    sequence (batched inverse + batched product) run on the device; 80 and
    208 leave ragged 64 x 64 tiles at the edges."""
    from exl3_intel_arc_quantizer_b200._ext import ext

    w = max(n // 2, 64)
    g = torch.Generator(device=DEV).manual_seed(3 + n)
    a = torch.randn(n, w, generator=g, device=DEV)
    chol = torch.linalg.cholesky(a @ a.T / w + 0.01 * torch.eye(n, device=DEV)).contiguous()
    L = torch.empty_like(chol)
    inv = torch.empty((n // 16, 16, 16), device=DEV)
    ext().block_ldl_fold(chol, L, inv)
    m = n // 16
    d = torch.diagonal(chol.reshape(m, 16, m, 16), dim1=0, dim2=2).permute(2, 0, 1)
    want_inv = torch.linalg.inv(d)
    want = torch.einsum("rbi,bij->rbj", chol.reshape(n, m, 16), want_inv).reshape(n, n)
    tb = want.reshape(m, 16, m, 16)
    idx = torch.arange(m, device=DEV)
    tb[idx, :, idx, :] = torch.eye(16, device=DEV)
    assert float((inv - want_inv).abs().max()) <= 1e-5 * float(want_inv.abs().max())
    assert float((L - want).abs().max()) <= 1e-5 * float(want.abs().max())
