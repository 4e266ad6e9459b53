"""Multi-GPU sharding of the conversion hot path.

One process per GPU with ``torch.distributed`` (NCCL between B200s; gloo
drives the same host logic in the CPU tests). The reference converts on one
Arc GPU; these are the independent units of its path (converter layer loop,
``exl3_quant/converter.py:1452-1612``) and how they shard:

1. **tiles** of an encoder sweep: contiguous, evenly split ranges
   (:func:`shard_range`); no collective;
2. **calibration tokens**: each rank accumulates ``X^T X`` of its own batches;
   :func:`all_reduce_hessians` sums the raw fp32 Hessians and the int64
   token counts once per group, then every rank finalizes identically
   (``calibration.py:337-407`` on the union of the shards);
3. **columns of a module** inside LDLQ: the feedback ``L^T (W - W_q)`` mixes
   rows only, so 128-aligned column slices are independent given the full
   ``L``: :func:`ldlq_column_sharded` runs the loop on this rank's slice and
   all-gathers ``weight_q`` and the trellis states;
4. **modules of a layer**: :func:`assign_modules` balances modules over ranks
   by tile count; :func:`quantize_layer_sharded` quantizes the local ones and
   broadcasts each result from its owner.

Every rank takes the same collective steps in the same order. Nothing here
uses TMA multicast or peer memory: the collectives are NCCL's.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from .ldlq import LDLQResult, TileEncoder, ldlq, ldlq_native


def world() -> Tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def shard_range(n_units: int, world_size: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """Contiguous ``[start, end)`` of ``n_units`` for ``rank``: blocks of
    ``align`` units dealt as evenly as possible (the first ranks take one
    block more). ``n_units`` must be a multiple of ``align``."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside world of size {world_size}")
    if align < 1 or n_units < 0 or n_units % align:
        raise ValueError(f"{n_units} units do not split into blocks of {align}")
    blocks = n_units // align
    base, extra = divmod(blocks, world_size)
    start = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return start * align, (start + count) * align


def all_reduce_hessians(hessians: Dict[str, torch.Tensor], token_counts: Dict[str, int],
                        group=None) -> Dict[str, int]:
    """Sum raw (un-normalised) Hessians and token counts over the group, in
    place, in sorted key order. Returns the global token counts. Every rank
    must hold the same keys."""
    keys = sorted(hessians)
    ws = dist.get_world_size(group)
    if ws == 1:
        return {k: int(token_counts[k]) for k in keys}
    names = [None] * ws
    dist.all_gather_object(names, keys, group=group)
    if any(n != keys for n in names):
        raise RuntimeError(f"Hessian groups differ across ranks: {names}")
    dev = hessians[keys[0]].device if keys else torch.device("cpu")
    counts = torch.tensor([int(token_counts[k]) for k in keys], dtype=torch.int64, device=dev)
    dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
    for k in keys:
        dist.all_reduce(hessians[k], op=dist.ReduceOp.SUM, group=group)
    return {k: int(c) for k, c in zip(keys, counts.tolist())}


def finalize_collector_distributed(collector, damping_lambda: float = 0.01,
                                   zero_floor: float = 1e-7, group=None):
    """``HessianCollector.finalize`` over the union of every rank's tokens:
    all-reduce the raw sums and counts, then the usual finalize."""
    collector.token_counts = all_reduce_hessians(collector.hessians, collector.token_counts, group)
    return collector.finalize(damping_lambda=damping_lambda, zero_floor=zero_floor)


def _wire(t: torch.Tensor) -> torch.Tensor:
    """Collectives move int16 trellis states as their bytes (neither NCCL nor
    gloo has a 16-bit integer type); a view, so in-place receives land in
    ``t``."""
    return t.view(torch.uint8) if t.dtype == torch.int16 else t


def _all_gather_cat(t: torch.Tensor, dim: int, sizes: Sequence[int], group=None) -> torch.Tensor:
    """Concatenate per-rank tensors of different extents along ``dim``."""
    ws = len(sizes)
    moved = t.movedim(dim, 0).contiguous()
    pad = max(sizes)
    buf = torch.zeros((pad,) + tuple(moved.shape[1:]), dtype=moved.dtype, device=moved.device)
    buf[:moved.shape[0]] = moved
    parts = [torch.empty_like(buf) for _ in range(ws)]
    dist.all_gather([_wire(p) for p in parts], _wire(buf), group=group)
    out = torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)
    return out.movedim(0, dim).contiguous()


def ldlq_column_sharded(weight: torch.Tensor, L: torch.Tensor, encode_tiles: TileEncoder,
                        buf_size_k: int = 128, group=None, align: int = 128) -> LDLQResult:
    """LDLQ of ``weight`` (k, n) with this rank's ``align``-column slice,
    then an all-gather of the slices: the same ``LDLQResult`` as the
    single-device loop (column slices never interact). With the B200
    encoder on CUDA tensors the slice runs the native loop, whose fixed
    per-output summation order does not depend on the slice's width, so the
    result equals the one-device native loop bit for bit."""
    ws, rank = dist.get_world_size(group), dist.get_rank(group)
    k, n = weight.shape
    if n % align:
        raise ValueError(f"columns ({n}) must be a multiple of {align} to shard")
    c0, c1 = shard_range(n, ws, rank, align)
    wq = enc = None
    if c1 > c0:
        part = weight[:, c0:c1].contiguous()
        if getattr(encode_tiles, "native_ldlq", False) and part.is_cuda:
            local = ldlq_native([(part, L)], encode_tiles.K, getattr(encode_tiles, "cb", 2),
                                buf_size_k)[0]
        else:
            local = ldlq(part, L, encode_tiles, buf_size_k=buf_size_k)
        wq, enc = local.weight_q, local.encoded
    else:  # more ranks than column blocks: this rank contributes nothing
        wq = torch.empty((k, 0), dtype=weight.dtype, device=weight.device)
        enc = torch.empty((k // 16, 0, 256), dtype=torch.int16, device=weight.device)
    weight_q, encoded = gather_column_slices(wq, enc, k, n, group, align)
    return LDLQResult(weight_q=weight_q, encoded=encoded, tiles_k=k // 16, tiles_n=n // 16,
                      buf_size_k=buf_size_k)


def gather_column_slices(weight_q: Optional[torch.Tensor], encoded: Optional[torch.Tensor],
                         k: int, n: int, group=None, align: int = 128
                         ) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather one module's LDLQ outputs from its column slices
    (``shard_range(n, world, rank, align)`` per rank; ``None`` for a rank
    with no slice) into the full ``weight_q`` (k, n) and ``encoded``
    (k/16, n/16, 256) on every rank."""
    ws, rank = dist.get_world_size(group), dist.get_rank(group)
    sizes = [e - s for s, e in (shard_range(n, ws, r, align) for r in range(ws))]
    dev = weight_q.device if weight_q is not None else torch.device(
        "cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
    if weight_q is None:
        weight_q = torch.empty((k, 0), dtype=torch.float32, device=dev)
        encoded = torch.empty((k // 16, 0, 256), dtype=torch.int16, device=dev)
    return (_all_gather_cat(weight_q, 1, sizes, group),
            _all_gather_cat(encoded, 1, [s // 16 for s in sizes], group))


def assign_modules(shapes: Dict[str, Tuple[int, int]], world_size: int) -> Dict[str, int]:
    """Owner rank of each module: largest first onto the least loaded rank
    (cost = tiles = k*n/256), ties to the lowest rank; deterministic."""
    load = [0] * world_size
    owner: Dict[str, int] = {}
    for name in sorted(shapes, key=lambda m: (-shapes[m][0] * shapes[m][1], m)):
        r = min(range(world_size), key=lambda i: (load[i], i))
        owner[name] = r
        load[r] += shapes[name][0] * shapes[name][1] // 256
    return owner


@dataclass
class ShardedModuleResult:
    """What every rank holds for a module after :func:`quantize_layer_sharded`."""
    name: str
    owner: int
    K: int
    cb: int
    w_hat: torch.Tensor
    encoded: torch.Tensor
    su: torch.Tensor
    sv: torch.Tensor
    result: Optional[object] = None   # the full module result, on the owner only


def quantize_layer_sharded(weights: Dict[str, torch.Tensor], hessians: Dict[str, torch.Tensor],
                           K: int = 2, group=None, quantize_fn=None,
                           **module_kwargs) -> Dict[str, ShardedModuleResult]:
    """Quantize the modules of one layer over the ranks of ``group``: each
    rank runs ``quantize_fn`` (default ``layer_quant.quantize_linear_module``)
    on the modules it owns, then every module's ``w_hat``, trellis states and
    scales are broadcast from its owner, in sorted module order."""
    if quantize_fn is None:
        from .layer_quant import quantize_linear_module as quantize_fn
    ws, rank = dist.get_world_size(group), dist.get_rank(group)
    names = sorted(weights)
    shapes = {}
    for nm in names:
        w = weights[nm]
        kdim = hessians[nm].shape[0]
        shapes[nm] = (kdim, w.numel() // kdim)
    owner = assign_modules(shapes, ws)
    local: Dict[str, object] = {}
    for nm in names:
        if owner[nm] == rank:
            local[nm] = quantize_fn(nm, weights[nm], hessians[nm], K=K, **module_kwargs)
    out: Dict[str, ShardedModuleResult] = {}
    for nm in names:
        k, n = shapes[nm]
        src = owner[nm]
        dev = weights[nm].device
        if src == rank:
            r = local[nm]
            w_hat, enc = r.w_hat.contiguous(), r.encoded.to(torch.int16).contiguous()
            su, sv = r.su.reshape(k, 1).contiguous(), r.sv.reshape(1, n).contiguous()
            cb = int(r.cb)
        else:
            w_hat = torch.empty((k, n), dtype=torch.float32, device=dev)
            enc = torch.empty((k // 16, n // 16, 256), dtype=torch.int16, device=dev)
            su = torch.empty((k, 1), dtype=torch.float32, device=dev)
            sv = torch.empty((1, n), dtype=torch.float32, device=dev)
            cb = 0
        gsrc = dist.get_global_rank(group, src) if group is not None else src
        for t in (w_hat, enc, su, sv):
            dist.broadcast(_wire(t), src=gsrc, group=group)
        cbt = torch.tensor([cb], dtype=torch.int64, device=dev)
        dist.broadcast(cbt, src=gsrc, group=group)
        out[nm] = ShardedModuleResult(nm, src, K, int(cbt.item()), w_hat, enc, su, sv,
                                      local.get(nm))
    return out
