"""EXL3 weight regularization (same API as ``exl3_quant/regularize.py``).

Order (normative, upstream ``quantize.py:1130-1236``): output-channel RMS
scales into ``sv`` (optional, skew heuristic on the Hessian diagonal),
``W /= sv``, right Hadamard, input-channel RMS scales into
``su = su * rms / (-1.24371088) + 1e-10``, ``W /= su``, left Hadamard, optional
global scale. Decoding reverses it (``hadamard.weight_from_quantized``).
Everything but the optional global scale runs in the libexl3k kernels
(``exl3_regularize``: skew heuristic, block RMS of columns and rows, the
scale decisions, both scalings fused with the 128-block Walsh-Hadamard
rotations), with one read of four result words at the end; CUDA tensors only.
``block_rms`` keeps the reference's public helper (regularize.py:49-80).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch

from ._ext import ext, require_cuda
from .hadamard import HAD_DIM

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

    if had_dim != HAD_DIM:
        raise ValueError(f"had_dim must be {HAD_DIM} (the EXL3 rotation), got {had_dim}")
    dev = require_cuda(weight.device)

    args = {} if quant_args is None else quant_args
    force = args.get("apply_out_scales")
    f32 = dict(device=dev, dtype=torch.float32)
    W = weight.contiguous()
    work = torch.empty_like(W)
    su_out = torch.empty(k, **f32)
    sv_out = torch.empty(n, **f32)
    out_scales = torch.empty(n, **f32)
    in_scales = torch.empty(k, **f32)
    hd = None
    if not q_fallback and H_diag is not None:
        hd = H_diag.to(**f32)
        if hd.dim() != 1 or hd.shape[0] != k:
            raise ValueError(f"H_diag must have {k} elements, got shape {tuple(hd.shape)}")
    apply_out, zeros, skew, _mean = ext().regularize_(
        W, su.to(**f32).reshape(k).contiguous(), sv.to(**f32).reshape(n).contiguous(), hd,
        -1 if force is None else int(bool(force)), bool(q_fallback), work, su_out, sv_out,
        out_scales, in_scales)
    apply_out, zeros = bool(apply_out), bool(zeros)
    skew = None if hd is None else float(skew)
    su = su_out.reshape(k, 1)
    sv = sv_out.reshape(1, n)

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
    return RegularizeResult(apply_out, work, g_scale, su, sv, out_scales.reshape(1, n),
                            in_scales.reshape(k, 1), zeros, skew)
