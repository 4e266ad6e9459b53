"""CPU oracle for the module driver — TEST AND BASELINE INFRASTRUCTURE ONLY.

Only ``tests/`` (as the checker) and ``bench.py``'s CPU-baseline leg (as the
timed CPU path) use this module; nothing in the package imports it. It
restates, with torch float32 ops on the CPU (the reference's own arithmetic,
so its roundings match), the reference's per-module pipeline:

* ``block_rms`` / ``regularize`` (``exl3_quant/regularize.py:49-211``):
  skew heuristic on the Hessian diagonal, output-channel RMS into ``sv``,
  ``W /= sv``, right Hadamard, input-channel RMS into
  ``su = su * rms / (-1.24371088) + 1e-10``, ``W /= su``, left Hadamard
  (no global-scale search: ``skip_g_scale=True``);
* the in-place blockwise Hadamards (``exl3_quant/hadamard.py:94-119``) and
  ``weight_from_quantized`` (``hadamard.py:122-140``, batched products);
* ``block_ldl`` (``exl3_quant/ldlq.py:75-132``): Cholesky with up to 10
  damped retries (diag += 2 * 0.025 * mean), 16x16 block inverses folded into
  their block columns, identity diagonal blocks;
* ``ldlq`` (``ldlq.py:163-309``): spans bottom-up, 16-row blocks bottom-up,
  compensation added, tensor-core permutation before encoding, trailing
  span update;
* ``quantize_linear_module`` (``exl3_quant/layer_quant.py:130-269``) with the
  metrics of ``layer_quant.py:95-127, 236-241``.

The tile encoder is the C restatement (``trellis_oracle.COracle``), threaded
over the tiles of each LDLQ step.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import numpy as np
import torch

from .storage_oracle import sylvester128
from .trellis_oracle import COracle, tensor_core_perm, tensor_core_perm_inv

HAD_DIM = 128
CODEBOOK_SCALE = 1.24371088


def hessian(X: torch.Tensor, damping: float = 0.01, floor: float = 1e-7) -> torch.Tensor:
    """X^T X of fp32 tokens, divided by the token count, diagonal damped by
    max(1e-8, damping * mean diag) and floored (``calibration.py:337-407``)."""
    H = X.float().T @ X.float()
    H = H / max(1, X.shape[0])
    d = H.diagonal()
    d.add_(max(1e-8, damping * d.mean().item()))
    d.copy_(torch.where(d.abs() < floor, torch.full_like(d, floor), d))
    return H


def _had() -> torch.Tensor:
    return torch.from_numpy(sylvester128())


def had_l_(x: torch.Tensor) -> torch.Tensor:
    h = _had()
    for r in range(0, x.shape[0], HAD_DIM):
        x[r:r + HAD_DIM, :] = h @ x[r:r + HAD_DIM, :]
    return x


def had_r_(x: torch.Tensor) -> torch.Tensor:
    h = _had()
    for c in range(0, x.shape[1], HAD_DIM):
        x[:, c:c + HAD_DIM] = x[:, c:c + HAD_DIM] @ h
    return x


def weight_from_quantized(w_hat: torch.Tensor, su: torch.Tensor, sv: torch.Tensor) -> torch.Tensor:
    k, n = w_hat.shape
    h = _had()
    work = (h @ w_hat.float().contiguous().view(-1, HAD_DIM, n)).view(k, n)
    work = work * su.float().reshape(k, 1)
    work = (work.contiguous().view(k, -1, HAD_DIM) @ h).view(k, n)
    return work * sv.float().reshape(1, n)


def block_rms(x: torch.Tensor, dim: int, keepdim: bool = False, blocksize: int = 32) -> torch.Tensor:
    acc = None
    for part in torch.split(x, blocksize, dim=dim):
        s = part.square().sum(dim=dim, keepdim=keepdim)
        acc = s if acc is None else acc + s
    return (acc / x.size(dim)).sqrt()


@dataclass
class Regularized:
    weight: torch.Tensor
    su: torch.Tensor
    sv: torch.Tensor
    apply_out_scales: bool


def regularize(W: torch.Tensor, H_diag: torch.Tensor) -> Regularized:
    k, n = W.shape
    d, _ = torch.sort(H_diag.sqrt(), descending=True)
    skew = float(d[:d.shape[0] // 50].sum() / d.sum())
    apply_out = skew < 0.15
    work = W.clone()
    out = block_rms(work, 0, keepdim=True)
    mean = out.mean().item()
    if mean > 1e-30:
        out /= mean
    zero_out = out.abs() < 1e-30
    su = torch.ones((k, 1), dtype=torch.float32)
    sv = torch.ones((1, n), dtype=torch.float32)
    if apply_out:
        out[zero_out] = 0.1
        sv = (sv * out + 1e-10).float()
    work /= sv
    sv[zero_out] = 0.0
    had_r_(work)
    inn = block_rms(work, 1, keepdim=True)
    inn[inn.abs() < 1e-30] = 0.1
    su = (su * inn / (-CODEBOOK_SCALE) + 1e-10).float()
    work /= su
    had_l_(work)
    return Regularized(work, su, sv, apply_out)


def blocked_cholesky(A: torch.Tensor, nb: int = 128) -> torch.Tensor:
    """Right-looking blocked Cholesky in fp32 with torch CPU ops: each
    diagonal block by ``torch.linalg.cholesky``, the panel under it by a
    triangular solve, the trailing matrix by one GEMM update. A valid fp32
    factorization whose rounding differs from a single LAPACK call; raises
    ``torch.linalg.LinAlgError`` like it on a non-positive pivot."""
    n = A.shape[0]
    work = A.clone()
    for j in range(0, n, nb):
        e = min(j + nb, n)
        ljj = torch.linalg.cholesky(work[j:e, j:e])
        work[j:e, j:e] = ljj
        if e < n:
            panel = torch.linalg.solve_triangular(ljj, work[e:, j:e].T.contiguous(),
                                                  upper=False).T
            work[e:, j:e] = panel
            work[e:, e:] -= panel @ panel.T
    return torch.tril(work)


def block_ldl(H: torch.Tensor, block: int = 16, sigma: float = 0.025,
              retries: int = 10, cholesky: Optional[Callable] = None
              ) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """(transformed L, Cholesky factor, retries used). ``cholesky`` defaults
    to ``torch.linalg.cholesky`` (the reference's call)."""
    work = H.clone()
    for attempt in range(retries + 1):
        try:
            chol = (cholesky or torch.linalg.cholesky)(work)
            break
        except torch.linalg.LinAlgError:
            if attempt == retries:
                raise
            work.diagonal().add_(2.0 * sigma * work.diagonal().mean())
    n = H.shape[0]
    L = chol.clone()
    for s in range(0, n, block):
        L[:, s:s + block] = chol[:, s:s + block] @ torch.linalg.inv(chol[s:s + block, s:s + block])
    eye = torch.eye(block, dtype=H.dtype)
    for s in range(0, n, block):
        L[s:s + block, s:s + block] = eye
    return L, chol, attempt


def c_encoder(K: int, cb: int = 2, threads: Optional[int] = None) -> Callable:
    """LDLQ tile-encoder callback over the C oracle: (N, 256) float32 tiles in
    tensor-core order -> (reconstruction float32, states int16)."""
    ora = COracle(K, cb)

    def encode(tiles: torch.Tensor):
        r = ora.encode_batch(tiles.numpy(), threads=threads)
        return (torch.from_numpy(r["recon"].astype(np.float32)),
                torch.from_numpy(r["indices"].view(np.int16).copy()))

    return encode


def ldlq(weight: torch.Tensor, L: torch.Tensor, encode: Callable,
         buf: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """(weight_q (k, n), encoded (k/16, n/16, 256) int16)."""
    k, n = weight.shape
    tn = n // 16
    perm = torch.as_tensor(tensor_core_perm(), dtype=torch.long)
    inv = torch.as_tensor(tensor_core_perm_inv(), dtype=torch.long)
    prod = torch.zeros((k, n), dtype=torch.float32)
    wq = torch.zeros((k, n), dtype=torch.float32)
    enc = torch.zeros((k // 16, tn, 256), dtype=torch.int16)
    for j in range(k, 0, -buf):
        i = j - buf
        for bj in range(buf, 0, -16):
            bi = bj - 16
            err = weight[i + bj:j] - wq[i + bj:j]
            comp = prod[i + bi:i + bj]
            if err.shape[0] > 0:
                comp.addmm_(L[i + bj:j, i + bi:i + bj].T, err, alpha=1.0, beta=1.0)
            rows = weight[i + bi:i + bj] + comp
            tiles = rows.reshape(16, tn, 16).permute(1, 0, 2).reshape(tn, 256)[:, perm]
            qw, qi = encode(tiles.contiguous())
            wq[i + bi:i + bj] = qw[:, inv].reshape(tn, 16, 16).permute(1, 0, 2).reshape(16, n)
            enc[(i + bi) // 16] = qi
        prod.addmm_(L[i:j].T, weight[i:j] - wq[i:j], alpha=1.0, beta=1.0)
    return wq, enc


@dataclass
class ModuleOracleResult:
    w_hat: torch.Tensor
    encoded: torch.Tensor
    su: torch.Tensor
    sv: torch.Tensor
    reg_weight: torch.Tensor
    L: torch.Tensor
    metrics: Tuple[float, float, float, float, float]  # mse, rel, tile dist, proxy, normalized
    factorization_residual: float
    seconds: float


def quantize_module(weight: torch.Tensor, H: torch.Tensor, K: int, cb: int = 2, buf: int = 128,
                    encode: Optional[Callable] = None,
                    ldlq_impl: Optional[Callable] = None,
                    cholesky: Optional[Callable] = None) -> ModuleOracleResult:
    """The module pipeline on the CPU. ``encode`` defaults to the C encoder;
    ``ldlq_impl(weight, L, encode, buf) -> (weight_q, encoded)`` defaults to
    :func:`ldlq` (torch CPU products, the reference's arithmetic on this host);
    ``ldlq_oracle.ldlq_fixed_order`` swaps in the device loop's fixed order;
    ``cholesky`` (e.g. :func:`blocked_cholesky`) replaces the LAPACK call."""
    t0 = time.perf_counter()
    kd = H.shape[0]
    W = (weight.T if weight.shape[1] == kd else weight).clone().float()
    H = H.float()
    reg = regularize(W, H.diagonal())
    Hr = had_r_(had_l_(H.clone()))
    L, chol, _ = block_ldl(Hr, cholesky=cholesky)
    fr = float(torch.linalg.norm(Hr - chol @ chol.T).item() / max(1e-12, torch.linalg.norm(Hr).item()))
    wq, enc = (ldlq_impl or ldlq)(reg.weight, L, encode if encode is not None else c_encoder(K, cb),
                                  buf)
    w_hat = weight_from_quantized(wq, reg.su, reg.sv)
    diff = W - w_hat
    mse = float(diff.pow(2).mean().item())
    rel = float(torch.linalg.norm(diff).item() / max(1e-12, torch.linalg.norm(W).item()))
    tile = float((reg.weight - wq).pow(2).mean().item())
    proxy = float(((H @ diff) * diff).sum().item())
    nproxy = proxy / max(1e-12, float(((H @ W) * W).sum().item()))
    return ModuleOracleResult(w_hat, enc, reg.su, reg.sv, reg.weight, L,
                              (mse, rel, tile, proxy, nproxy), fr, time.perf_counter() - t0)
