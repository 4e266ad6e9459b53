"""Trellis tile encoder on B200 and its scratch arena.

Drop-in for the reference module ``exl3_quant/xpu_quantizer.py``
(alpha2beta/EXL3_Intel_Arc_quantizer): same class and function names,
arguments, validation errors and result types —
``build_quantize_extension`` (:65-98), ``verify_tile_encoding_quality``
(:108-169), ``ScratchArena`` (:188-506), ``BatchEncodingBreakdown`` (:509-526),
``XPUTrellisEncoder`` (:529-994) — over the sm_100a kernels of libexl3k.

Differences that follow from the hardware, not from the algorithm:
  * the scratch is one byte workspace of K-bit backpointers (the cost vectors
    live in shared memory), sized by ``exl3_quantize_tiles_ws_bytes``;
  * every traceback placement runs on the device: ``gpu_resident`` is the
    fused path, ``gpu_resident_split`` runs the reference-layout forward /
    backward ops, and the Arc unified-memory experiments ``d2h_cpu`` /
    ``usm_host`` are accepted and served by the fused device path;
  * ``sg_size``, ``force_global_costs`` and ``wave_cap_override`` select Intel
    sub-group / SLM variants; they are validated and otherwise ignored.
There is no CPU fallback: without a CUDA device every encode raises.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import numpy as np

from . import _build
from ._ext import encoder_fault_check, ext, require_cuda
from .memory_policy import MemoryPolicy, MemoryPressureError, capture_snapshot
from .trellis_format import (
    CB_3INST,
    CB_MCG,
    CB_MUL1,
    codebook_lut,
    tensor_core_perm,
    tensor_core_perm_inv,
)

TRACEBACK_MODES = ("gpu_resident", "gpu_resident_split", "d2h_cpu", "usm_host")
DEFAULT_CAP_B = 8192

_BUILD_SECONDS = {"cold_build_seconds": 0.0, "warm_load_seconds": 0.0}


@dataclass
class EncodingResult:
    """Result of trellis encoding of one tile (reference_encoder.py:47-59)."""

    output_indices: np.ndarray      # (L,) uint16 states, encoder order
    reconstructed: np.ndarray       # (L,) fp16, original tile order when pre-permuted
    reconstructed_perm: np.ndarray  # (L,) fp16, encoder order
    packed: np.ndarray              # (16*K,) uint16 container words (SWAP16), L=256 only
    end_state: int
    distortion: float
    mse: float
    path_cost: float
    K: int
    cb: int


def build_quantize_extension(verbose: bool = False, force_rebuild: bool = False):
    """Build (if stale) and load the native layer; returns the op module."""
    t0 = time.perf_counter()
    if force_rebuild:
        _build.build_all(force=True, verbose=verbose)
        _BUILD_SECONDS["cold_build_seconds"] = time.perf_counter() - t0
    module = ext()
    if not force_rebuild:
        _BUILD_SECONDS["warm_load_seconds"] = time.perf_counter() - t0
    return module


def get_build_timings() -> dict:
    return dict(_BUILD_SECONDS)


def verify_tile_encoding_quality(result: EncodingResult, reference: EncodingResult,
                                 cost_atol: float = 0.0, distortion_rtol: float = 1e-4) -> dict:
    """Check an encoding against a reference one, accepting equal-cost ties:
    ring continuity, exact reconstruction, end state, path cost and distortion
    (xpu_quantizer.py:108-169)."""
    L = len(result.output_indices)
    K = result.K
    mask = (65536 >> K) - 1
    idx = np.asarray(result.output_indices, dtype=np.int64)
    nxt = np.roll(idx, -1)
    breaks = np.nonzero((idx & mask) != (nxt >> K))[0]
    ring_valid = breaks.size == 0
    lut = codebook_lut(result.cb)
    rec_exact = bool(np.array_equal(np.asarray(result.reconstructed_perm).view(np.uint16),
                                    lut[idx].view(np.uint16)))
    end_state_valid = int(idx[L - 1] & mask) == int(result.end_state)
    cost_diff = abs(float(result.path_cost) - float(reference.path_cost))
    ref_dist = max(1e-12, float(reference.distortion))
    dist_rel = abs(float(result.distortion) - float(reference.distortion)) / ref_dist
    passed = ring_valid and rec_exact and end_state_valid and cost_diff <= cost_atol and (
        dist_rel <= distortion_rtol or cost_diff == 0.0)
    return {
        "passed": bool(passed),
        "indices_identical": bool(np.array_equal(idx, np.asarray(reference.output_indices))),
        "ring_valid": bool(ring_valid),
        "broken_step": int(breaks[0]) if breaks.size else -1,
        "rec_exact": rec_exact,
        "end_state_valid": bool(end_state_valid),
        "cost_diff": cost_diff,
        "distortion_rel_diff": dist_rel,
    }


@dataclass
class ScratchArenaLogEntry:
    action: str                 # allocate | reuse | evict | retry-shrink | release
    k: int
    tile_len: int
    requested_b: int
    admitted_b: int
    scratch_bytes: int
    distinct_staging_bytes: int
    outstanding_xpu_bytes: int
    usable_budget_bytes: int
    snapshot: dict


class ScratchArena:
    """One resident encoder workspace per arena, reused across calls.

    Same contract as the reference arena (xpu_quantizer.py:188-506): at most
    one buffer is resident; a request for another (device, K, L) or for more
    tiles than resident synchronizes the stream and evicts it first; when the
    requested batch does not fit the memory policy, or the allocator (or
    ``allocator_hook``) fails, the batch halves down to 1 before a
    :class:`MemoryPressureError` is raised. The buffer is a uint8 tensor of
    compact backpointers; ``acquire`` returns ``(workspace, tile_bytes,
    admitted_b)`` where the workspace holds at least ``admitted_b`` tiles.
    """

    def __init__(self, policy: Optional[MemoryPolicy] = None, device_index: int = 0,
                 default_cap_b: int = DEFAULT_CAP_B):
        self.policy = policy or MemoryPolicy()
        self.device_index = device_index
        self.default_cap_b = default_cap_b
        self._key: Optional[Tuple[int, int, int, int]] = None
        self._ws = None
        self.history: List[ScratchArenaLogEntry] = []
        self.high_water_scratch_bytes = 0
        self.evictions = 0
        self.reuses = 0
        self.allocations = 0
        self.retries = 0

    @property
    def current_key(self):
        return self._key

    @property
    def resident_bytes(self) -> int:
        return 0 if self._ws is None else int(self._ws.numel())

    @staticmethod
    def workspace_bytes(k: int, tile_len: int = 256, b: int = 1) -> int:
        return int(ext().quantize_tiles_ws_bytes(int(b), int(k), int(tile_len)))

    @classmethod
    def tile_bytes(cls, k: int, tile_len: int = 256) -> int:
        return cls.workspace_bytes(k, tile_len, 2) // 2

    def _log(self, action, k, tile_len, req, adm, scratch, staging, snap=None):
        import torch

        snap = snap or capture_snapshot(self.device_index)
        out = int(torch.cuda.memory_allocated(self.device_index)) if torch.cuda.is_available() else 0
        self.history.append(ScratchArenaLogEntry(
            action, k, tile_len, req, adm, scratch, staging, out,
            self.policy.usable_bytes(snap), snap.as_dict()))

    def resident(self, k: int, tile_len: int, b: int):
        """The resident workspace if it already serves (K, L, b tiles), else
        None; no bookkeeping (hot loops such as LDLQ call this per block)."""
        key = self._key
        if (key is not None and key[0] == self.device_index and key[1] == k
                and key[2] == tile_len and key[3] >= b):
            return self._ws
        return None

    def adaptive_batch_capacity(self, k: int, tile_len: int = 256,
                                requested_b: Optional[int] = None,
                                distinct_staging_bytes: int = 0) -> int:
        target = requested_b if requested_b is not None else self.default_cap_b
        if target < 1:
            raise ValueError(f"requested_b must be >= 1, got {target}")
        snap = capture_snapshot(self.device_index)
        per = self.tile_bytes(k, tile_len)
        usable = self.policy.usable_bytes(snap) + self.resident_bytes
        max_b = usable // per
        if self.policy.max_single_alloc_bytes is not None:
            max_b = min(max_b, self.policy.max_single_alloc_bytes // per)
        if max_b < 1:
            self.policy.check(per, snap, context=f"adaptive_batch_capacity K={k} B=1")
        return int(max(1, min(target, max_b)))

    def release(self) -> None:
        import torch

        if self._ws is None:
            return
        torch.cuda.synchronize(self.device_index)
        k, t, b = self._key[1], self._key[2], self._key[3]
        self._ws = None
        self._key = None
        torch.cuda.empty_cache()
        self._log("release", k, t, b, 0, 0, 0)

    def acquire(self, k: int, tile_len: int = 256, requested_b: Optional[int] = None,
                distinct_staging_bytes: int = 0,
                allocator_hook: Optional[Callable[[int], None]] = None):
        import torch

        target = requested_b if requested_b is not None else self.default_cap_b
        if target < 1:
            raise ValueError(f"requested_b must be >= 1, got {target}")
        per = self.tile_bytes(k, tile_len)
        key = self._key
        if (key is not None and key[0] == self.device_index and key[1] == k
                and key[2] == tile_len and key[3] >= target):
            # reuse is ordered on the stream the encoder launches on: no sync
            self.reuses += 1
            self._log("reuse", k, tile_len, target, target, self.resident_bytes,
                      distinct_staging_bytes)
            return self._ws, per, target
        if self._ws is not None:
            self.evictions += 1
            self.release()
        cand = target
        last_err: Optional[Exception] = None
        while cand >= 1:
            need = self.workspace_bytes(k, tile_len, cand)
            snap = capture_snapshot(self.device_index)
            ws = None
            try:
                self.policy.check(need, snap, context=f"K={k} B={cand} workspace")
                if allocator_hook is not None:
                    allocator_hook(cand)
                ws = torch.empty(need, dtype=torch.uint8, device=f"cuda:{self.device_index}")
                self._ws, self._key = ws, (self.device_index, k, tile_len, cand)
                self.allocations += 1
                self.high_water_scratch_bytes = max(self.high_water_scratch_bytes, need)
                self._log("allocate", k, tile_len, target, cand, need, distinct_staging_bytes)
                return ws, per, cand
            except Exception as exc:  # allocator failure or policy rejection
                del ws
                torch.cuda.empty_cache()
                last_err = exc
                if cand == 1:
                    break
                nxt = max(1, cand // 2)
                self.retries += 1
                self._log("retry-shrink", k, tile_len, cand, nxt, need, distinct_staging_bytes,
                          snap)
                cand = nxt
        if isinstance(last_err, MemoryPressureError):
            raise MemoryPressureError(str(last_err), last_err.need_bytes, last_err.usable_bytes,
                                      last_err.snapshot, last_err.context) from None
        snap = capture_snapshot(self.device_index)
        raise MemoryPressureError(
            f"workspace allocation failed even at B=1 for K={k}: {last_err}", per,
            self.policy.usable_bytes(snap), snap, f"K={k} B=1") from None


@dataclass
class BatchEncodingBreakdown:
    results: List[EncodingResult]
    reconstructed_tiles: np.ndarray     # (N, L) fp16, original order if pre_permute
    reconstructed_perm: np.ndarray      # (N, L) fp16, encoder order
    output_indices: np.ndarray          # (N, L) uint16
    admitted_b: int
    num_chunks: int
    total_seconds: float
    search_seconds: float
    traceback_seconds: float
    transfer_seconds: float
    postprocess_seconds: float
    traceback_mode: str
    sg_size: int
    force_global_costs: bool


class XPUTrellisEncoder:
    """B200 Viterbi trellis encoder matching the reference CPU encoder bit for bit."""

    def __init__(self, K: int = 2, cb: int = CB_MUL1, tile_len: int = 256,
                 arena: Optional[ScratchArena] = None, device_index: int = 0,
                 sg_size: int = 32, force_global_costs: bool = False,
                 wave_cap_override: int = 0):
        if not 1 <= K <= 8:
            raise ValueError(f"K must be between 1 and 8, got {K}")
        if cb not in (CB_3INST, CB_MCG, CB_MUL1):
            raise ValueError(f"Unknown codebook {cb}")
        if tile_len not in (256, 160):
            raise ValueError(f"tile_len must be 256 or 160, got {tile_len}")
        if tile_len == 160 and cb != CB_MUL1:
            raise ValueError("tile_len=160 is only supported with CB_MUL1")
        if sg_size not in (16, 32):
            raise ValueError(f"sg_size must be 16 or 32, got {sg_size}")
        self.K, self.cb, self.L = K, cb, tile_len
        self.edges = 65536 >> K
        self.device_index = device_index
        self.sg_size = sg_size
        self.force_global_costs = force_global_costs
        self.wave_cap_override = wave_cap_override
        self.arena = arena or ScratchArena(device_index=device_index)
        self.lut = codebook_lut(cb)
        self.perm = tensor_core_perm() if tile_len == 256 else None
        self.inv_perm = tensor_core_perm_inv() if tile_len == 256 else None
        self._perm_dev = None

    @property
    def mcg_flag(self) -> bool:
        return self.cb == CB_MCG

    @property
    def mul1_flag(self) -> bool:
        return self.cb == CB_MUL1

    # -- device-resident API -------------------------------------------------
    def encode_device(self, tiles, pre_permute: bool = False, requested_b: Optional[int] = None,
                      want_packed: bool = True):
        """Encode a CUDA tensor of tiles without leaving the device.

        Returns ``(recon f32 (N, L) encoder order, indices int16 (N, L),
        packed int16 (N, 16K) or None, path_cost f32 (N,))``.
        """
        import torch

        dev = require_cuda(f"cuda:{self.device_index}")
        x = tiles.reshape(-1, self.L).to(device=dev, dtype=torch.float32)
        if pre_permute:
            if self.L != 256:
                raise ValueError("pre_permute=True is only defined for L=256")
            if self._perm_dev is None:
                self._perm_dev = torch.as_tensor(self.perm, device=dev)
            x = x.index_select(1, self._perm_dev)
        x = x.contiguous()
        n = x.shape[0]
        if n <= 0:
            raise ValueError(f"num_tiles must be positive, got {n}")
        cap = min(n, requested_b if requested_b is not None else self.arena.default_cap_b)
        ws = self.arena.resident(self.K, self.L, cap)
        if ws is None:
            ws, _, _ = self.arena.acquire(self.K, self.L, cap)
        out_w = torch.empty_like(x)
        out_i = torch.empty((n, self.L), dtype=torch.int16, device=dev)
        packed = (torch.empty((n, 16 * self.K), dtype=torch.int16, device=dev)
                  if (want_packed and self.L == 256) else None)
        cost = torch.empty(n, dtype=torch.float32, device=dev)
        ext().encode_tiles(x, out_w, out_i, packed, cost, ws, self.K, self.cb)
        return out_w, out_i, packed, cost

    # -- reference API ---------------------------------------------------------
    def encode_tile(self, tile: np.ndarray, pre_permute: bool = True,
                    traceback_mode: str = "gpu_resident") -> EncodingResult:
        raw = np.asarray(tile, dtype=np.float32).reshape(-1)
        if raw.size != self.L:
            raise ValueError(f"Tile must have {self.L} elements, got {raw.size}")
        return self.encode_batch_detailed(raw.reshape(1, self.L), pre_permute=pre_permute,
                                          requested_b=1, traceback_mode=traceback_mode).results[0]

    def encode_batch(self, tiles: np.ndarray, pre_permute: bool = True,
                     requested_b: Optional[int] = None,
                     traceback_mode: str = "gpu_resident") -> List[EncodingResult]:
        return self.encode_batch_detailed(tiles, pre_permute=pre_permute,
                                          requested_b=requested_b,
                                          traceback_mode=traceback_mode).results

    def encode_batch_detailed(self, tiles: np.ndarray, pre_permute: bool = True,
                              requested_b: Optional[int] = None,
                              traceback_mode: str = "gpu_resident",
                              allocator_hook: Optional[Callable[[int], None]] = None
                              ) -> BatchEncodingBreakdown:
        import torch

        arr = np.asarray(tiles, dtype=np.float32)
        if arr.ndim == 2:
            num_tiles, width = arr.shape
        elif arr.ndim == 3 and arr.shape[1:] == (16, 16) and self.L == 256:
            num_tiles, width = arr.shape[0], 256
            arr = arr.reshape(num_tiles, 256)
        else:
            raise ValueError(f"Unsupported tiles shape {arr.shape} for L={self.L}")
        if num_tiles <= 0:
            raise ValueError(f"num_tiles must be positive, got {num_tiles}")
        if width != self.L:
            raise ValueError(f"Expected tile length {self.L}, got {width}")
        if pre_permute and self.L != 256:
            raise ValueError("pre_permute=True is only defined for L=256")
        if traceback_mode not in TRACEBACK_MODES:
            raise ValueError(f"Unknown traceback_mode {traceback_mode!r}")
        ext()
        dev = require_cuda(f"cuda:{self.device_index}")
        with encoder_fault_check(dev):   # EncoderFault if a cluster wait timed out
            return self._encode_batch_detailed(arr, num_tiles, pre_permute, requested_b,
                                               traceback_mode, allocator_hook, dev)

    def _encode_batch_detailed(self, arr, num_tiles, pre_permute, requested_b, traceback_mode,
                               allocator_hook, dev) -> BatchEncodingBreakdown:
        import torch

        t_total0 = time.perf_counter()
        perm_np = arr[:, self.perm] if pre_permute else arr
        w16 = np.ascontiguousarray(perm_np, dtype=np.float16)
        t0 = time.perf_counter()
        x = torch.from_numpy(np.ascontiguousarray(w16, dtype=np.float32)).to(dev)
        torch.cuda.synchronize(dev)
        t_transfer = time.perf_counter() - t0

        desired = min(num_tiles, requested_b if requested_b is not None else self.arena.default_cap_b)
        t_search = t_trace = 0.0
        if traceback_mode == "gpu_resident_split":
            out_w, out_i, cost, admitted, chunks, t_search, t_trace = self._encode_split(
                x, desired, allocator_hook)
            packed = None
            if self.L == 256:
                packed = torch.empty((num_tiles, 16 * self.K), dtype=torch.int16, device=dev)
                ext().pack_trellis(out_i, packed, self.K)
        else:
            ws, per, admitted = self.arena.acquire(self.K, self.L, desired,
                                                   allocator_hook=allocator_hook)
            out_w = torch.empty_like(x)
            out_i = torch.empty((num_tiles, self.L), dtype=torch.int16, device=dev)
            packed = (torch.empty((num_tiles, 16 * self.K), dtype=torch.int16, device=dev)
                      if self.L == 256 else None)
            cost = torch.empty(num_tiles, dtype=torch.float32, device=dev)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            ext().encode_tiles(x, out_w, out_i, packed, cost, ws, self.K, self.cb)
            ev1.record()
            ev1.synchronize()
            t_search = ev0.elapsed_time(ev1) / 1e3
            per_chunk = max(1, int(ws.numel()) // per)
            if self.K >= 2:
                per_chunk = max(2, per_chunk & ~1)
            chunks = -(-num_tiles // min(per_chunk, num_tiles))

        t0 = time.perf_counter()
        rec_perm = out_w.cpu().numpy().astype(np.float16)
        idx = out_i.cpu().numpy().view(np.uint16)
        packed_np = packed.cpu().numpy().view(np.uint16) if packed is not None else None
        cost_np = cost.cpu().numpy()
        t_transfer += time.perf_counter() - t0
        total = time.perf_counter() - t_total0

        t_post0 = time.perf_counter()
        rec_all = rec_perm[:, self.inv_perm] if pre_permute else rec_perm
        orig = arr if pre_permute else w16.astype(np.float32)
        dist = ((orig - rec_all.astype(np.float32)) ** 2).sum(axis=1, dtype=np.float32)
        mask = self.edges - 1
        empty = np.zeros(0, dtype=np.uint16)
        results = [
            EncodingResult(
                output_indices=idx[t], reconstructed=rec_all[t], reconstructed_perm=rec_perm[t],
                packed=packed_np[t] if packed_np is not None else empty,
                end_state=int(idx[t, self.L - 1]) & mask, distortion=float(dist[t]),
                mse=float(dist[t]) / self.L, path_cost=float(cost_np[t]), K=self.K, cb=self.cb)
            for t in range(num_tiles)
        ]
        post = time.perf_counter() - t_post0
        return BatchEncodingBreakdown(
            results=results, reconstructed_tiles=rec_all, reconstructed_perm=rec_perm,
            output_indices=idx, admitted_b=admitted, num_chunks=chunks,
            total_seconds=total + post, search_seconds=t_search, traceback_seconds=t_trace,
            transfer_seconds=t_transfer, postprocess_seconds=post, traceback_mode=traceback_mode,
            sg_size=self.sg_size, force_global_costs=self.force_global_costs)

    def _encode_split(self, x, desired: int, allocator_hook):
        """Reference-layout split passes (forward / backward ops), chunked."""
        import torch

        n = x.shape[0]
        dev = x.device
        cand = max(1, desired)
        while True:
            try:
                if allocator_hook is not None:
                    allocator_hook(cand)
                costs = torch.empty((cand, 2, self.edges), dtype=torch.float16, device=dev)
                edges = torch.empty((cand, self.L, self.edges), dtype=torch.int16, device=dev)
                break
            except Exception:
                if cand == 1:
                    raise
                cand //= 2
        e = ext()
        out_w = torch.empty_like(x)
        out_i = torch.empty((n, self.L), dtype=torch.int16, device=dev)
        cost = torch.empty(n, dtype=torch.float32, device=dev)
        t_search = t_trace = 0.0
        chunks = 0
        for s in range(0, n, cand):
            m = min(cand, n - s)
            chunks += 1
            pre = torch.full((m,), -1, dtype=torch.int32, device=dev)
            ends = torch.empty((m,), dtype=torch.int32, device=dev)
            c_in = x[s:s + m]
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            evs[0].record()
            e.quantize_tiles_forward_pass(c_in, costs, edges, pre, self.K, self.mcg_flag,
                                          self.mul1_flag, self.L // 2, 0)
            evs[1].record()
            e.quantize_tiles_backward_pass(costs, edges, out_w[s:s + m], out_i[s:s + m], ends, m,
                                           self.K, self.mcg_flag, self.mul1_flag, self.L // 2, 0,
                                           False)
            evs[2].record()
            e.quantize_tiles_forward_pass(c_in, costs, edges, ends, self.K, self.mcg_flag,
                                          self.mul1_flag, 0, 1)
            evs[3].record()
            e.quantize_tiles_backward_pass(costs, edges, out_w[s:s + m], out_i[s:s + m], ends, m,
                                           self.K, self.mcg_flag, self.mul1_flag, 0, 1, True)
            evs[4].record()
            evs[4].synchronize()
            t_search += (evs[0].elapsed_time(evs[1]) + evs[2].elapsed_time(evs[3])) / 1e3
            t_trace += (evs[1].elapsed_time(evs[2]) + evs[3].elapsed_time(evs[4])) / 1e3
            idx_end = ends.long()
            cost[s:s + m] = costs[torch.arange(m, device=dev), 1, idx_end].float()
        return out_w, out_i, cost, cand, chunks, t_search, t_trace


# B200 name for the same encoder.
CUDATrellisEncoder = XPUTrellisEncoder
