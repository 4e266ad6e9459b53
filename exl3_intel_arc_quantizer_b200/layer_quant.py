"""Per-module and per-layer quantization driver (API of ``exl3_quant/layer_quant.py``).

``quantize_linear_module`` runs, on the weight's CUDA device:
regularize -> left/right Hadamard on H -> block_ldl -> LDLQ with the B200
encoder -> original-basis reconstruction -> metrics, with the reference's
names, orientation rules, K guard and result types. Nothing leaves the device
until the scalar metrics are read.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .hadamard import HAD_DIM, blockwise_preapply_had_l_, blockwise_preapply_had_r_, weight_from_quantized
from .ldlq import (
    DEFAULT_BLOCK_SIZE,
    DEFAULT_BUF_SIZE_K,
    BlockLDLResult,
    TileEncoder,
    block_ldl,
    ldlq,
    make_xpu_tile_encoder,
)
from .regularize import RegularizeResult, regularize
from .trellis_format import CB_MUL1
from .xpu_quantizer import ScratchArena


@dataclass
class ModuleMetrics:
    mse: float
    relative_frobenius_error: float
    tile_distortion: float
    proxy_loss: float
    normalized_proxy_loss: float
    factorization_residual: float
    retries: int
    g_scale: float
    elapsed_seconds: float


@dataclass
class QuantizedModuleResult:
    name: str
    K: int
    cb: int
    original_shape: Tuple[int, int]
    weight_orig: torch.Tensor
    w_hat: torch.Tensor
    encoded: torch.Tensor
    su: torch.Tensor
    sv: torch.Tensor
    metrics: ModuleMetrics
    regularize_result: RegularizeResult
    ldl_result: BlockLDLResult


@dataclass
class LayerQuantizationReport:
    K: int
    codebook: str
    total_elapsed_seconds: float
    module_results: Dict[str, QuantizedModuleResult]
    total_proxy_loss: float
    mean_mse: float
    peak_device_memory_bytes: int
    scratch_arena_reused: bool
    device_index: int


def compute_factorization_residual(H: torch.Tensor, chol: torch.Tensor) -> float:
    """||H - L L^T||_F / ||H||_F."""
    diff = H - chol @ chol.T
    return float(torch.linalg.norm(diff).item() / max(1e-12, torch.linalg.norm(H).item()))


def compute_proxy_loss(W: torch.Tensor, W_hat: torch.Tensor, H: torch.Tensor) -> Tuple[float, float]:
    """tr(E^T H E) with E = W - W_hat, and its ratio to tr(W^T H W)."""
    E = (W - W_hat).to(dtype=torch.float32, device=H.device)
    Hf = H.to(torch.float32)
    proxy = float(((Hf @ E) * E).sum().item())
    Wf = W.to(dtype=torch.float32, device=H.device)
    energy = max(1e-12, float(((Hf @ Wf) * Wf).sum().item()))
    return proxy, proxy / energy


def quantize_linear_module(name: str, weight: torch.Tensor, H: torch.Tensor, K: int = 2,
                           cb: int = CB_MUL1, tile_encoder: Optional[TileEncoder] = None,
                           skip_g_scale: bool = True, buf_size_k: int = DEFAULT_BUF_SIZE_K,
                           block_size: int = DEFAULT_BLOCK_SIZE) -> QuantizedModuleResult:
    t0 = time.time()
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2D, got shape {tuple(weight.shape)}")
    kdim = H.shape[0]
    if weight.shape[1] == kdim:
        W = weight.T.clone().to(torch.float32).contiguous()
    elif weight.shape[0] == kdim:
        W = weight.clone().to(torch.float32).contiguous()
    else:
        raise ValueError(f"Weight shape {tuple(weight.shape)} does not match Hessian dim {kdim}")
    k, n = W.shape
    device = W.device
    su = torch.ones((k, 1), dtype=torch.float32, device=device)
    sv = torch.ones((1, n), dtype=torch.float32, device=device)

    if tile_encoder is None:
        if device.type != "cuda":
            raise RuntimeError("quantize_linear_module needs CUDA tensors (no CPU encoder path)")
        tile_encoder = make_xpu_tile_encoder(K=K, device_index=device.index or 0)
    enc_k = getattr(tile_encoder, "K", None)
    if enc_k is not None and enc_k != K:
        raise ValueError(
            f"Tile encoder K={enc_k} does not match the requested K={K}. The trellis container "
            f"would be packed at {K} bpw while the encoder emitted {enc_k} bpw states. Build the "
            f"encoder with K={K}.")
    g_scale_fn = None
    if not skip_g_scale:
        from .gss import g_scale_fn_from_encoder

        g_scale_fn = g_scale_fn_from_encoder(tile_encoder)

    Hd = H.to(device=device, dtype=torch.float32)
    reg = regularize(W, su, sv, H_diag=Hd.diagonal(), skip_g_scale=skip_g_scale,
                     g_scale_fn=g_scale_fn, had_dim=HAD_DIM)
    H_work = Hd.clone().contiguous()
    blockwise_preapply_had_l_(H_work, HAD_DIM)
    blockwise_preapply_had_r_(H_work, HAD_DIM)
    ldl = block_ldl(H_work, block_size=block_size)
    fact_res = compute_factorization_residual(H_work, ldl.cholesky)
    res = ldlq(reg.weight, ldl.transformed, tile_encoder, buf_size_k=buf_size_k)
    w_hat = weight_from_quantized(res.weight_q, reg.su, reg.sv)

    diff = W - w_hat
    mse = float(diff.pow(2).mean().item())
    rel = float(torch.linalg.norm(diff).item() / max(1e-12, torch.linalg.norm(W).item()))
    tile_dist = float((reg.weight - res.weight_q).pow(2).mean().item())
    proxy, nproxy = compute_proxy_loss(W, w_hat, Hd)
    metrics = ModuleMetrics(mse, rel, tile_dist, proxy, nproxy, fact_res, ldl.retries,
                            reg.g_scale, time.time() - t0)
    return QuantizedModuleResult(name, K, cb, (k, n), W, w_hat, res.encoded, reg.su, reg.sv,
                                 metrics, reg, ldl)


def quantize_decoder_layer(layer: nn.Module, hessians: Dict[str, torch.Tensor], K: int = 2,
                           cb: int = CB_MUL1, device: Optional[torch.device] = None,
                           skip_g_scale: bool = True, buf_size_k: int = DEFAULT_BUF_SIZE_K,
                           block_size: int = DEFAULT_BLOCK_SIZE, memory_policy=None,
                           module_names: Optional[List[str]] = None) -> LayerQuantizationReport:
    """Quantize every bias-free linear projection of a layer, sharing one
    encoder and one scratch arena across modules."""
    t0 = time.time()
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if device.type != "cuda":
        raise RuntimeError("quantize_decoder_layer needs a CUDA device (no CPU encoder path)")
    di = device.index or 0
    arena = ScratchArena(device_index=di, policy=memory_policy)
    enc = make_xpu_tile_encoder(K=K, device_index=di, arena=arena)
    available = {nm: m for nm, m in layer.named_modules()
                 if isinstance(m, nn.Linear) and m.bias is None}
    selected = list(available) if module_names is None else list(module_names)
    missing = [nm for nm in selected if nm not in available]
    if missing:
        raise KeyError(f"requested modules are not bias-free nn.Linear submodules: {missing}")
    torch.cuda.reset_peak_memory_stats(di)
    results: Dict[str, QuantizedModuleResult] = {}
    try:
        for nm in selected:
            if nm not in hessians:
                raise KeyError(f"Hessian missing for module {nm}")
            W = available[nm].weight.data.to(device)
            results[nm] = quantize_linear_module(nm, W, hessians[nm].to(device), K=K, cb=cb,
                                                 tile_encoder=enc, skip_g_scale=skip_g_scale,
                                                 buf_size_k=buf_size_k, block_size=block_size)
    finally:
        arena.release()
    return LayerQuantizationReport(
        K=K, codebook="mul1" if cb == CB_MUL1 else str(cb), total_elapsed_seconds=time.time() - t0,
        module_results=results, total_proxy_loss=sum(r.metrics.proxy_loss for r in results.values()),
        mean_mse=float(np.mean([r.metrics.mse for r in results.values()])) if results else 0.0,
        peak_device_memory_bytes=int(torch.cuda.max_memory_allocated(di)),
        scratch_arena_reused=True, device_index=di)
