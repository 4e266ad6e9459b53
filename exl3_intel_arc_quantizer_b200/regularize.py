"""EXL3 weight regularization (same API as ``exl3_quant/regularize.py``).

Order (normative, upstream ``quantize.py:1130-1236``): output-channel RMS
scales into ``sv`` (optional, skew heuristic on the Hessian diagonal),
``W /= sv``, right Hadamard, input-channel RMS scales into
``su = su * rms / (-1.24371088) + 1e-10``, ``W /= su``, left Hadamard, optional
global scale. Decoding reverses it (``hadamard.weight_from_quantized``).
The reductions and scalings are torch ops on the device; the rotations are
the libexl3k Walsh-Hadamard kernels.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch

from .hadamard import HAD_DIM, blockwise_preapply_had_l_, blockwise_preapply_had_r_

CODEBOOK_SCALE = 1.24371088
OUT_SCALE_SKEW_CUTOFF = 0.15
SKEW_FRACTION = 50
ZERO_FLOOR = 0.1
EPS = 1e-10


def block_rms(x: torch.Tensor, dim: int, keepdim: bool = False, blocksize: int = 32) -> torch.Tensor:
    """``sqrt(mean(x^2, dim))`` with the sum of squares accumulated in
    32-slices along ``dim`` (the upstream accumulation order)."""
    n = x.size(dim)
    acc = None
    for block in torch.split(x, blocksize, dim=dim):
        s = block.square().sum(dim=dim, keepdim=keepdim)
        acc = s if acc is None else acc.add_(s)
    return (acc / n).sqrt()


@dataclass
class RegularizeResult:
    apply_out_scales: bool
    weight: torch.Tensor
    g_scale: float
    su: torch.Tensor
    sv: torch.Tensor
    out_channel_scales: torch.Tensor
    in_channel_scales: torch.Tensor
    zeros: bool
    skew_factor: Optional[float]


def regularize(weight: torch.Tensor, su: torch.Tensor, sv: torch.Tensor,
               quant_args: Optional[dict] = None, H_diag: Optional[torch.Tensor] = None,
               skip_g_scale: bool = True, q_fallback: bool = False,
               g_scale_fn: Optional[Callable[[torch.Tensor], float]] = None,
               had_dim: int = HAD_DIM) -> RegularizeResult:
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2-D, got shape {tuple(weight.shape)}")
    if weight.dtype != torch.float32:
        raise ValueError(f"weight must be float32, got {weight.dtype}")
    k, n = weight.shape
    if su.numel() != k or sv.numel() != n:
        raise ValueError(f"su must have {k} elements and sv {n}, got {su.numel()} / {sv.numel()}")
    if k % had_dim != 0 or n % had_dim != 0:
        raise ValueError(f"both dimensions must be divisible by {had_dim}, got {(k, n)}")

    args = {} if quant_args is None else quant_args
    force = args.get("apply_out_scales")
    skew: Optional[float] = None
    if not q_fallback and H_diag is not None:
        d, _ = torch.sort(H_diag.sqrt(), descending=True)
        cutoff = d.shape[0] // SKEW_FRACTION
        skew = float(d[:cutoff].sum() / d.sum())
        apply_out = (skew < OUT_SCALE_SKEW_CUTOFF) if force is None else bool(force)
    else:
        apply_out = True if force is None else bool(force)
    if q_fallback:
        apply_out = bool(force)

    work = weight.clone().contiguous()
    out_scales = block_rms(work, dim=0, keepdim=True)
    mean = out_scales.mean().item()
    if mean > 1e-30:
        out_scales /= mean
        zeros = False
    else:
        zeros = True
        if force is not None:
            apply_out = True
    zero_out = out_scales.abs() < 1e-30

    su = su.to(device=work.device, dtype=torch.float32).clone().reshape(k, 1)
    sv = sv.to(device=work.device, dtype=torch.float32).clone().reshape(1, n)
    if apply_out:
        out_scales[zero_out] = ZERO_FLOOR
        sv = (sv * out_scales + EPS).float()
    work /= sv
    sv[zero_out] = 0.0
    blockwise_preapply_had_r_(work, had_dim)

    in_scales = block_rms(work, dim=1, keepdim=True)
    in_scales[in_scales.abs() < 1e-30] = ZERO_FLOOR
    su = (su * in_scales / (-CODEBOOK_SCALE) + EPS).float()
    work /= su
    blockwise_preapply_had_l_(work, had_dim)

    if skip_g_scale:
        g_scale = 1.0
    else:
        if g_scale_fn is None:
            raise ValueError("skip_g_scale=False requires g_scale_fn (the global-scale search "
                             "test-quantizes sample tiles and needs the encoder)")
        g_scale = float(g_scale_fn(work))
        if not g_scale > 0.0:
            raise ValueError(f"g_scale_fn returned a non-positive scale: {g_scale}")
    work *= g_scale
    su /= g_scale
    if "zeros" in args or quant_args is not None:
        args["zeros"] = zeros
    return RegularizeResult(bool(apply_out), work, g_scale, su, sv, out_scales, in_scales, zeros,
                            skew)
