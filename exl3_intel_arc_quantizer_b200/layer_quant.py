"""Per-module and per-layer quantization driver (API of ``exl3_quant/layer_quant.py``).

``quantize_linear_module`` runs, on the weight's CUDA device:
regularize -> left/right Hadamard on H -> block_ldl -> LDLQ with the B200
encoder -> original-basis reconstruction -> metrics, with the reference's
names, orientation rules, K guard and result types. Nothing leaves the device
until the scalar metrics are read.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from .hadamard import HAD_DIM, blockwise_preapply_had_l_, blockwise_preapply_had_r_, weight_from_quantized
from ._ext import encoder_fault_check, raise_on_faults
from .ldlq import (
    DEFAULT_BLOCK_SIZE,
    DEFAULT_BUF_SIZE_K,
    BlockLDLResult,
    TileEncoder,
    block_ldl,
    ldlq,
    ldlq_batched,
    ldlq_native,
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


def _orient(weight: torch.Tensor, kdim: int) -> torch.Tensor:
    """(k, n) fp32 copy: the quantized orientation has the Hessian's
    dimension first (layer_quant.py:130-160)."""
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2D, got shape {tuple(weight.shape)}")
    if weight.shape[1] == kdim:
        return weight.T.clone().to(torch.float32).contiguous()
    if weight.shape[0] == kdim:
        return weight.clone().to(torch.float32).contiguous()
    raise ValueError(f"Weight shape {tuple(weight.shape)} does not match Hessian dim {kdim}")


def _check_encoder_k(tile_encoder, K: int) -> None:
    enc_k = getattr(tile_encoder, "K", None)
    if enc_k is not None and enc_k != K:
        raise ValueError(
            f"Tile encoder K={enc_k} does not match the requested K={K}. The trellis container "
            f"would be packed at {K} bpw while the encoder emitted {enc_k} bpw states. Build the "
            f"encoder with K={K}.")


def _default_encoder(device: torch.device, K: int):
    if device.type != "cuda":
        raise RuntimeError("quantize_linear_module needs CUDA tensors (no CPU encoder path)")
    return make_xpu_tile_encoder(K=K, device_index=device.index or 0)


def _ldl_of(Hd: torch.Tensor, block_size: int, residual: bool = True):
    """Block-LDL of the rotated Hessian; with ``residual`` also its
    factorization residual, else the rotated matrix to compute it later."""
    H_work = Hd.clone().contiguous()
    blockwise_preapply_had_l_(H_work, HAD_DIM)
    blockwise_preapply_had_r_(H_work, HAD_DIM)
    ldl = block_ldl(H_work, block_size=block_size)
    if residual:
        return ldl, compute_factorization_residual(H_work, ldl.cholesky)
    return ldl, H_work


def _module_metrics(W: torch.Tensor, Hd: torch.Tensor, reg: RegularizeResult,
                    weight_q: torch.Tensor, w_hat: torch.Tensor) -> Tuple[float, ...]:
    """mse, relative Frobenius error, tile distortion, proxy loss and its
    normalised form (layer_quant.py:104-127, 236-241)."""
    diff = W - w_hat
    mse = float(diff.pow(2).mean().item())
    rel = float(torch.linalg.norm(diff).item() / max(1e-12, torch.linalg.norm(W).item()))
    tile_dist = float((reg.weight - weight_q).pow(2).mean().item())
    proxy, nproxy = compute_proxy_loss(W, w_hat, Hd)
    return mse, rel, tile_dist, proxy, nproxy


def _finish(name: str, K: int, cb: int, W: torch.Tensor, Hd: torch.Tensor,
            reg: RegularizeResult, ldl: BlockLDLResult, fact_res: float, weight_q: torch.Tensor,
            encoded: torch.Tensor, t0: float, w_hat: Optional[torch.Tensor] = None,
            metric_values: Optional[Tuple[float, ...]] = None) -> QuantizedModuleResult:
    k, n = W.shape
    if w_hat is None:
        w_hat = weight_from_quantized(weight_q, reg.su, reg.sv)
    if metric_values is None:
        metric_values = _module_metrics(W, Hd, reg, weight_q, w_hat)
    mse, rel, tile_dist, proxy, nproxy = metric_values
    metrics = ModuleMetrics(mse, rel, tile_dist, proxy, nproxy, fact_res, ldl.retries,
                            reg.g_scale, time.time() - t0)
    return QuantizedModuleResult(name, K, cb, (k, n), W, w_hat, encoded, reg.su, reg.sv,
                                 metrics, reg, ldl)


def quantize_linear_module(name: str, weight: torch.Tensor, H: torch.Tensor, K: int = 2,
                           cb: int = CB_MUL1, tile_encoder: Optional[TileEncoder] = None,
                           skip_g_scale: bool = True, buf_size_k: int = DEFAULT_BUF_SIZE_K,
                           block_size: int = DEFAULT_BLOCK_SIZE) -> QuantizedModuleResult:
    t0 = time.time()
    W = _orient(weight, H.shape[0])
    k, n = W.shape
    device = W.device
    su = torch.ones((k, 1), dtype=torch.float32, device=device)
    sv = torch.ones((1, n), dtype=torch.float32, device=device)
    if tile_encoder is None:
        tile_encoder = _default_encoder(device, K)
    _check_encoder_k(tile_encoder, K)
    g_scale_fn = None
    if not skip_g_scale:
        from .gss import g_scale_fn_from_encoder

        g_scale_fn = g_scale_fn_from_encoder(tile_encoder)

    # raises EncoderFault if an encoder call of this module timed out
    with encoder_fault_check(device):
        Hd = H.to(device=device, dtype=torch.float32)
        reg = regularize(W, su, sv, H_diag=Hd.diagonal(), skip_g_scale=skip_g_scale,
                         g_scale_fn=g_scale_fn, had_dim=HAD_DIM)
        ldl, fact_res = _ldl_of(Hd, block_size)
        res = _run_ldlq([(reg.weight, ldl.transformed)], tile_encoder, K, buf_size_k)[0]
        return _finish(name, K, cb, W, Hd, reg, ldl, fact_res, res.weight_q, res.encoded, t0)


def _run_ldlq(jobs, tile_encoder, K: int, buf_size_k: int):
    """The device loop for the B200 encoder on CUDA tensors, the callback loop
    (the reference's op sequence) for any other encoder."""
    if (getattr(tile_encoder, "native_ldlq", False) and jobs
            and all(w.is_cuda for w, _ in jobs)):
        return ldlq_native(jobs, K, getattr(tile_encoder, "cb", CB_MUL1), buf_size_k)
    return ldlq_batched(jobs, tile_encoder, buf_size_k)


def quantize_modules(modules: Dict[str, Tuple[torch.Tensor, torch.Tensor]], K: int = 2,
                     cb: int = CB_MUL1, tile_encoder: Optional[TileEncoder] = None,
                     skip_g_scale: bool = True, buf_size_k: int = DEFAULT_BUF_SIZE_K,
                     block_size: int = DEFAULT_BLOCK_SIZE,
                     group=None) -> Dict[str, QuantizedModuleResult]:
    """Quantize several ``name -> (weight, H)`` modules together, each with
    exactly the arithmetic of :func:`quantize_linear_module`:

    * the global-scale searches of all modules run as one batched search
      (every candidate tile of every module in shared encoder launches);
    * one block-LDL per distinct Hessian (q/k/v share one, gate/up share one);
    * one LDLQ over all modules: each step encodes the current 16-row block
      of every active module in a single launch (``ldlq.ldlq_native``; the
      longest module runs throughout, the others start where
      ``ldlq.ldlq_schedule`` places them; ``ldlq.ldlq_batched`` for other
      encoders);
    * the diagnostics that need no quantized weight (factorization
      residuals, the proxy-loss normalizers) run on a side stream while the
      LDLQ loop runs.

    With a process ``group`` (``torch.distributed``), every module's
    128-aligned column slices are dealt over the ranks, each rank runs the
    LDLQ on its slices, and one all-gather per module rebuilds the full
    result on every rank (column slices never interact in LDLQ). The metrics
    are then sums over every rank's column slices (fp64 partial sums, one
    all-reduce), so every rank ends with the same metrics.
    """
    t0 = time.time()
    if not modules:
        return {}
    names = list(modules)
    device = modules[names[0]][0].device
    if tile_encoder is None:
        tile_encoder = _default_encoder(device, K)
    _check_encoder_k(tile_encoder, K)
    # encoder CTAs that time out during this call are counted on the device;
    # the count is checked once the results are final (on every rank)
    faults = encoder_fault_check(device).__enter__()

    Ws, Hds, regs = {}, {}, {}
    for nm in names:
        weight, H = modules[nm]
        W = _orient(weight, H.shape[0])
        k, n = W.shape
        Ws[nm] = W
        Hds[nm] = H.to(device=W.device, dtype=torch.float32)
        su = torch.ones((k, 1), dtype=torch.float32, device=W.device)
        sv = torch.ones((1, n), dtype=torch.float32, device=W.device)
        regs[nm] = regularize(W, su, sv, H_diag=Hds[nm].diagonal(), skip_g_scale=True,
                              had_dim=HAD_DIM)
    if not skip_g_scale:
        from .gss import g_scale_search_batch, sample_scale_tiles

        found = g_scale_search_batch([sample_scale_tiles(regs[nm].weight) for nm in names],
                                     tile_encoder)
        for nm, (g, _mse) in zip(names, found):
            g = float(g)
            if not g > 0.0:
                raise ValueError(f"global-scale search returned a non-positive scale: {g}")
            regs[nm].weight.mul_(g)
            regs[nm].su.div_(g)
            regs[nm].g_scale = g

    # one block-LDL per distinct Hessian
    ldls: List[list] = []               # [H, ldl, rotated H]
    ldl_of: Dict[str, int] = {}
    for nm in names:
        Hd = Hds[nm]
        hit = next((i for i, (h, _, _) in enumerate(ldls)
                    if h.shape == Hd.shape and (h.data_ptr() == Hd.data_ptr() or torch.equal(h, Hd))),
                   None)
        if hit is None:
            ldl, H_rot = _ldl_of(Hd, block_size, residual=False)
            ldls.append([Hd, ldl, H_rot])
            hit = len(ldls) - 1
        ldl_of[nm] = hit

    if group is None:
        ws, rank = 1, 0
    else:
        import torch.distributed as dist

        from .distributed import gather_column_slices, shard_range

        ws, rank = dist.get_world_size(group), dist.get_rank(group)

    # The diagnostics that need no quantized weight (each Hessian's
    # factorization residual, each module's energy tr(W^T H W)) are fp32
    # GEMMs; they run on a side stream while the LDLQ loop, whose launches
    # leave most SMs idle, runs on the current one. With a group each rank
    # computes column slices of every product and the sums are all-reduced.
    main = torch.cuda.current_stream(device)
    side = torch.cuda.Stream(device=device)
    side.wait_stream(main)
    res_parts, energy_parts = [], {}
    with torch.cuda.stream(side):
        for _h, ldl, H_rot in ldls:
            for t in (H_rot, ldl.cholesky):
                t.record_stream(side)
            res_parts.append(_residual_parts(H_rot, ldl.cholesky, ws, rank))
        for nm in names:
            for t in (Ws[nm], Hds[nm]):
                t.record_stream(side)
            energy_parts[nm] = _energy_part(Hds[nm], Ws[nm], ws, rank)

    if group is None:
        jobs = [(regs[nm].weight, ldls[ldl_of[nm]][1].transformed) for nm in names]
        outs = _run_ldlq(jobs, tile_encoder, K, buf_size_k)
        wq = {nm: o.weight_q for nm, o in zip(names, outs)}
        enc = {nm: o.encoded for nm, o in zip(names, outs)}
    else:
        local = [nm for nm in names
                 if (lambda r: r[1] > r[0])(shard_range(Ws[nm].shape[1], ws, rank, 128))]
        jobs = []
        for nm in local:
            c0, c1 = shard_range(Ws[nm].shape[1], ws, rank, 128)
            jobs.append((regs[nm].weight[:, c0:c1].contiguous(), ldls[ldl_of[nm]][1].transformed))
        outs = dict(zip(local, _run_ldlq(jobs, tile_encoder, K, buf_size_k))) if jobs else {}
        wq, enc = {}, {}
        for nm in names:
            k, n = Ws[nm].shape
            o = outs.get(nm)
            wq[nm], enc[nm] = gather_column_slices(
                o.weight_q if o is not None else None, o.encoded if o is not None else None,
                k, n, group)
    main.wait_stream(side)

    w_hats = {nm: weight_from_quantized(wq[nm], regs[nm].su, regs[nm].sv) for nm in names}
    if group is None:
        raise_on_faults(faults.delta())
        # the arithmetic of compute_factorization_residual / _module_metrics
        fres = [float(a.item() / max(1e-12, b.item())) for a, b in res_parts]
        out = {}
        for nm in names:
            W, w_hat = Ws[nm], w_hats[nm]
            diff = W - w_hat
            mse = float(diff.pow(2).mean().item())
            rel = float(torch.linalg.norm(diff).item() / max(1e-12, torch.linalg.norm(W).item()))
            tile_dist = float((regs[nm].weight - wq[nm]).pow(2).mean().item())
            proxy = float(((Hds[nm] @ diff) * diff).sum().item())
            energy = max(1e-12, float(energy_parts[nm].item()))
            out[nm] = _finish(nm, K, cb, W, Hds[nm], regs[nm], ldls[ldl_of[nm]][1],
                              fres[ldl_of[nm]], wq[nm], enc[nm], t0, w_hat=w_hat,
                              metric_values=(mse, rel, tile_dist, proxy, proxy / energy))
        return out

    # sharded: partial sums over this rank's column slice of every module,
    # fp64, one all-reduce; every rank ends with every module's metrics
    parts = torch.zeros((len(names) * 5 + len(ldls) * 2 + 1,), dtype=torch.float64, device=device)
    parts[-1] = float(faults.delta())      # every rank raises if any rank's encoder faulted
    for idx, nm in enumerate(names):
        k, n = Ws[nm].shape
        c0, c1 = shard_range(n, ws, rank, 128)
        p = parts[5 * idx:5 * idx + 5]
        p[4] = energy_parts[nm]
        if c1 > c0:
            W = Ws[nm][:, c0:c1]
            d = W - w_hats[nm][:, c0:c1]
            p[0] = d.double().pow(2).sum()
            p[1] = W.double().pow(2).sum()
            p[2] = (regs[nm].weight[:, c0:c1] - wq[nm][:, c0:c1]).double().pow(2).sum()
            p[3] = ((Hds[nm] @ d) * d).double().sum()
    base = len(names) * 5
    for li, (a, b) in enumerate(res_parts):
        parts[base + 2 * li] = a
        parts[base + 2 * li + 1] = b
    dist.all_reduce(parts, group=group)
    v = parts.tolist()
    raise_on_faults(int(v[-1]))
    fres = [math.sqrt(v[base + 2 * li]) / max(1e-12, math.sqrt(v[base + 2 * li + 1]))
            for li in range(len(ldls))]
    out = {}
    for idx, nm in enumerate(names):
        k, n = Ws[nm].shape
        sd, sw, st, proxy, energy = v[5 * idx:5 * idx + 5]
        metric = (sd / (k * n), math.sqrt(sd) / max(1e-12, math.sqrt(sw)), st / (k * n), proxy,
                  proxy / max(1e-12, energy))
        out[nm] = _finish(nm, K, cb, Ws[nm], Hds[nm], regs[nm], ldls[ldl_of[nm]][1],
                          fres[ldl_of[nm]], wq[nm], enc[nm], t0, w_hat=w_hats[nm],
                          metric_values=metric)
    return out


def _residual_parts(H_rot: torch.Tensor, chol: torch.Tensor, ws: int, rank: int):
    """Numerator and denominator of ||H - L L^T||_F / ||H||_F. One rank: the
    two fp32 norms of compute_factorization_residual; several: the fp64
    sums of squares over this rank's 16-aligned column slice."""
    if ws == 1:
        return torch.linalg.norm(H_rot - chol @ chol.T), torch.linalg.norm(H_rot)
    from .distributed import shard_range

    k = H_rot.shape[0]
    c0, c1 = shard_range(k, ws, rank, 16)
    if c1 <= c0:
        z = torch.zeros((), dtype=torch.float64, device=H_rot.device)
        return z, z.clone()
    d = H_rot[:, c0:c1] - chol @ chol[c0:c1].T
    return d.double().pow(2).sum(), H_rot[:, c0:c1].double().pow(2).sum()


def _energy_part(H: torch.Tensor, W: torch.Tensor, ws: int, rank: int) -> torch.Tensor:
    """tr(W^T H W) (compute_proxy_loss's normalizer): whole on one rank,
    the fp64 sum over this rank's LDLQ column slice on several."""
    if ws == 1:
        return ((H @ W) * W).sum()
    from .distributed import shard_range

    c0, c1 = shard_range(W.shape[1], ws, rank, 128)
    if c1 <= c0:
        return torch.zeros((), dtype=torch.float64, device=W.device)
    Wc = W[:, c0:c1]
    return ((H @ Wc) * Wc).double().sum()


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
