"""fp16 FMA rounding probes of the encoder's metric on the device.

Mirrors ``exl3_quant/xpu_probe.py:153-270`` (``run_hfma_probe``,
``run_hfma_adversarial_probe``; open item O-6 of the reference): the ACS
metric ``fma(v - w, v - w, cost)`` must round once to binary16, as the
reference encoder computes it (``reference_encoder.py:130-204``). The probe
op is ``probe_hfma`` of the PyTorch binding (C-ABI ``exl3_probe_hfma``):
mode 0 is the packed ``fma.rn.f16x2`` the ACS kernels issue, mode 1 the
scalar ``fma.rn.f16`` the tracebacks issue (the reference's mode 1 is its
compiler's plain ``a * a + c`` expression; here both modes must be the
single rounding, since the traceback re-evaluates the ACS's costs).

The host columns are the definitions being probed: the exact value
``dh * dh + cost`` in float64 (exact for these inputs: a binary16 square
has 22 significant bits and the sum spans < 53) rounded once to binary16,
and the float32 evaluation rounded twice (the old reference behaviour).
"""

from __future__ import annotations

import numpy as np

from . import _ext

# Discriminating pairs of the reference's adversarial probe
# (xpu_probe.py:221-224): fp32 double rounding != exact single rounding.
ADVERSARIAL_DH_BITS = (0x3C16, 0x3C27, 0x3C32, 0x3C5D, 0x3C71, 0x3C9B,
                       0x3CC9, 0x3CCE, 0x3CD3, 0x3CE1, 0x3CEA)
ADVERSARIAL_COST_BITS = (0x01C1, 0x00EF, 0x03C1, 0x0371, 0x01F1, 0x026F,
                         0x02EF, 0x03BF, 0x016F, 0x03EF, 0x01BF)


def exact_hfma(dh: np.ndarray, cost: np.ndarray) -> np.ndarray:
    """dh * dh + cost rounded once to binary16 (overflow gives inf)."""
    with np.errstate(over="ignore", invalid="ignore"):
        return (dh.astype(np.float64) * dh.astype(np.float64)
                + cost.astype(np.float64)).astype(np.float16)


def fp32_emulated_hfma(dh: np.ndarray, cost: np.ndarray) -> np.ndarray:
    """dh * dh + cost in float32, then rounded to binary16 (two roundings)."""
    with np.errstate(over="ignore", invalid="ignore"):
        v = dh.astype(np.float32) ** 2
        return (v + cost.astype(np.float32)).astype(np.float16)


def _device_hfma(ext, dh: np.ndarray, cost: np.ndarray, device=None):
    import torch

    dev = _ext.require_cuda(device)
    dh_t = torch.from_numpy(np.ascontiguousarray(dh)).to(dev)
    cost_t = torch.from_numpy(np.ascontiguousarray(cost)).to(dev)
    out = []
    for mode in (0, 1):
        o = torch.empty_like(dh_t)
        ext.probe_hfma(dh_t, cost_t, o, mode)
        out.append(o.cpu().numpy())
    return out


def run_hfma_probe(ext=None, n: int = 1 << 16, seed: int = 2026, device=None) -> dict:
    """Random block (xpu_probe.py:153-208): dh ~ N(0, 1), cost ~ U[0, 8) in
    binary16; counts where each device mode differs from the exact single
    rounding."""
    ext = ext if ext is not None else _ext.ext()
    rng = np.random.default_rng(seed=seed)
    dh = rng.normal(0.0, 1.0, size=n).astype(np.float16)
    cost = (rng.random(n) * 8.0).astype(np.float16)
    dev_fma, dev_scalar = _device_hfma(ext, dh, cost, device)
    exact = exact_hfma(dh, cost)
    emul32 = fp32_emulated_hfma(dh, cost)

    def first_mismatch(dev, ref):
        idx = np.flatnonzero(dev.view(np.uint16) != ref.view(np.uint16))
        if not idx.size:
            return None
        i = int(idx[0])
        return {"index": i, "dh": float(dh[i]), "cost": float(cost[i]),
                "device": float(dev[i]), "exact": float(exact[i])}

    def mism(a, b):
        return int(np.count_nonzero(a.view(np.uint16) != b.view(np.uint16)))

    return {
        "n": n,
        "seed": seed,
        "fma_vs_exact_mismatches": mism(dev_fma, exact),
        "expr_vs_exact_mismatches": mism(dev_scalar, exact),
        "fma_vs_expr_mismatches": mism(dev_fma, dev_scalar),
        "host_fp32_emul_vs_exact_mismatches": mism(emul32, exact),
        "first_fma_mismatch": first_mismatch(dev_fma, exact),
        "first_expr_mismatch": first_mismatch(dev_scalar, exact),
        "first_emul_mismatch": first_mismatch(emul32, exact),
    }


def run_hfma_adversarial_probe(ext=None, dh_bits=ADVERSARIAL_DH_BITS,
                               cost_bits=ADVERSARIAL_COST_BITS, device=None) -> dict:
    """Adversarial block (xpu_probe.py:211-270): pairs on which the float32
    double rounding differs from the exact single rounding, so only they
    tell the two semantics apart."""
    ext = ext if ext is not None else _ext.ext()
    dh = np.asarray(dh_bits, dtype=np.uint16).view(np.float16)
    cost = np.asarray(cost_bits, dtype=np.uint16).view(np.float16)
    exact = exact_hfma(dh, cost)
    emul32 = fp32_emulated_hfma(dh, cost)
    emul_differs = int(np.count_nonzero(emul32.view(np.uint16) != exact.view(np.uint16)))
    if emul_differs == 0:
        return {"error": "adversarial set no longer discriminates"}
    dev_fma, dev_scalar = _device_hfma(ext, dh, cost, device)

    def hits(a, b):
        return int(np.count_nonzero(a.view(np.uint16) == b.view(np.uint16)))

    fma_exact, fma_emul = hits(dev_fma, exact), hits(dev_fma, emul32)
    cases = [{"dh_bits": int(dh_bits[i]), "cost_bits": int(cost_bits[i]),
              "dh": float(dh[i]), "cost": float(cost[i]), "exact": float(exact[i]),
              "fp32_emul": float(emul32[i]), "device_fma": float(dev_fma[i]),
              "device_expr": float(dev_scalar[i])} for i in range(dh.size)]
    return {
        "n": int(dh.size),
        "fp32_emul_vs_exact_mismatches": emul_differs,
        "fma_matches_exact": fma_exact,
        "fma_matches_fp32_emul": fma_emul,
        "expr_matches_exact": hits(dev_scalar, exact),
        "expr_matches_fp32_emul": hits(dev_scalar, emul32),
        "conclusion": (
            "device fma == exact single rounding"
            if fma_exact == emul_differs and fma_emul == 0
            else "device fma == fp32 double rounding"
            if fma_emul == emul_differs and fma_exact == 0
            else "mixed/other semantics"),
        "cases": cases,
    }
