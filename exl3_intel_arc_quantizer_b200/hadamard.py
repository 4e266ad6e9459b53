"""Blockwise Sylvester Hadamard transforms on B200.

Same API and semantics as the reference ``exl3_quant/hadamard.py``: the
orthonormal Sylvester ``H_128 / sqrt(128)`` applied on 128-row blocks (left,
``H @ x``) or 128-column blocks (right, ``x @ H``); H is symmetric and its own
inverse. The in-place transforms run the fast Walsh-Hadamard kernels of
libexl3k (``exl3_had128_left`` / ``_right``) on CUDA tensors; the matrix
builders are plain torch.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

HAD_DIM = 128
_HAD_CACHE: dict = {}


def sylvester_hadamard(n: int) -> torch.Tensor:
    """Unnormalised Sylvester matrix of order n (entries +-1, float64)."""
    if n < 1 or (n & (n - 1)) != 0:
        raise ValueError(f"Sylvester construction requires a power-of-two size, got {n}")
    idx = torch.arange(n)
    bits = torch.bitwise_and(idx[:, None], idx[None, :])
    parity = torch.zeros_like(bits)
    b = bits.clone()
    while bool(b.any()):
        parity ^= b & 1
        b >>= 1
    return (1 - 2 * parity).to(torch.float64)


def hadamard(n: int = HAD_DIM, dtype: torch.dtype = torch.float32,
             scale: Optional[float] = None, device: Optional[torch.device] = None) -> torch.Tensor:
    if scale is None:
        scale = 1.0 / math.sqrt(n)
    key = (n, dtype, float(scale), str(device) if device is not None else "cpu")
    m = _HAD_CACHE.get(key)
    if m is None:
        m = (sylvester_hadamard(n) * scale).to(dtype=dtype, device=device)
        _HAD_CACHE[key] = m
    return m


def _check_inplace(x: torch.Tensor, had_dim: int) -> None:
    if had_dim != HAD_DIM:
        raise ValueError(f"only 128-blocks are supported, got had_dim={had_dim}")
    if x.dtype != torch.float32:
        raise ValueError(f"in-place Hadamard requires float32, got {x.dtype}")
    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")


def blockwise_preapply_had_l_(x: torch.Tensor, had_dim: int = HAD_DIM) -> torch.Tensor:
    """In place ``H @ x`` on 128-row blocks (hadamard.py:94-105)."""
    from ._ext import ext, require_cuda

    _check_inplace(x, had_dim)
    if x.shape[0] % had_dim != 0:
        raise ValueError(f"rows ({x.shape[0]}) must be divisible by had_dim ({had_dim})")
    require_cuda(x.device)
    if not x.is_contiguous():
        raise ValueError("in-place Hadamard requires a contiguous tensor")
    ext().had128_left_(x)
    return x


def blockwise_preapply_had_r_(x: torch.Tensor, had_dim: int = HAD_DIM) -> torch.Tensor:
    """In place ``x @ H`` on 128-column blocks (hadamard.py:108-119)."""
    from ._ext import ext, require_cuda

    _check_inplace(x, had_dim)
    if x.shape[1] % had_dim != 0:
        raise ValueError(f"columns ({x.shape[1]}) must be divisible by had_dim ({had_dim})")
    require_cuda(x.device)
    if not x.is_contiguous():
        raise ValueError("in-place Hadamard requires a contiguous tensor")
    ext().had128_right_(x)
    return x


def preapply_had_l(x: torch.Tensor, had_dim: int = HAD_DIM) -> torch.Tensor:
    if x.shape[0] % had_dim != 0:
        raise ValueError(f"rows ({x.shape[0]}) must be divisible by had_dim ({had_dim})")
    work = x.to(torch.float32).contiguous().clone()
    return blockwise_preapply_had_l_(work, had_dim).to(x.dtype)


def preapply_had_r(x: torch.Tensor, had_dim: int = HAD_DIM) -> torch.Tensor:
    if x.shape[1] % had_dim != 0:
        raise ValueError(f"columns ({x.shape[1]}) must be divisible by had_dim ({had_dim})")
    work = x.to(torch.float32).contiguous().clone()
    return blockwise_preapply_had_r_(work, had_dim).to(x.dtype)


def weight_from_quantized(w_hat: torch.Tensor, su: torch.Tensor, sv: torch.Tensor) -> torch.Tensor:
    """Original-basis weight from the transformed reconstruction:
    ``H_l -> x su -> H_r -> x sv`` (hadamard.py:122-140)."""
    k, n = w_hat.shape
    if su.numel() != k or sv.numel() != n:
        raise ValueError(f"su must have {k} elements and sv {n}, got {su.numel()} / {sv.numel()}")
    work = w_hat.to(torch.float32).contiguous().clone()
    blockwise_preapply_had_l_(work)
    work.mul_(su.to(torch.float32).reshape(k, 1))
    blockwise_preapply_had_r_(work)
    work.mul_(sv.to(torch.float32).reshape(1, n))
    return work
