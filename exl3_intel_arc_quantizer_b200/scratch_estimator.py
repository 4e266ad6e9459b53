"""Encoder scratch sizing.

``ScratchEstimator`` keeps the reference API (``exl3_quant/scratch_estimator.py``:
``estimate_scratch``, ``calculate_max_batch_size``) and its formula for the
reference's scratch layout — ``temp_costs (B, 2, S)`` fp16 plus
``temp_edges (B, T, S)`` int16, ``S = 65536 >> K`` — which the reference-layout
split passes still use.

The B200 encoder itself needs far less: the cost vectors live in shared
memory; K = 1 stores the chosen branch per edge and step, K >= 2 stores a
cost-vector checkpoint every step or two (:func:`b200_workspace_bytes`),
e.g. 4 MiB per tile at K=2 against the reference layout's 8 MiB per pass.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

BYTES_PER_KIB = 1024
BYTES_PER_MIB = 1024 ** 2
BYTES_PER_GIB = 1024 ** 3
BYTES_PER_KB = 1000
BYTES_PER_MB = 1000 ** 2
BYTES_PER_GB = 1000 ** 3


@dataclass(frozen=True)
class ScratchAllocation:
    k: int
    states: int
    t: int
    b: int
    bytes_per_cost: int
    bytes_per_edge: int
    costs_bytes: int
    edges_bytes: int
    total_bytes: int

    @property
    def costs_mib(self) -> float:
        return self.costs_bytes / BYTES_PER_MIB

    @property
    def costs_mb(self) -> float:
        return self.costs_bytes / BYTES_PER_MB

    @property
    def edges_gib(self) -> float:
        return self.edges_bytes / BYTES_PER_GIB

    @property
    def edges_gb(self) -> float:
        return self.edges_bytes / BYTES_PER_GB

    @property
    def total_gib(self) -> float:
        return self.total_bytes / BYTES_PER_GIB

    @property
    def total_gb(self) -> float:
        return self.total_bytes / BYTES_PER_GB


class ScratchEstimator:
    """Reference scratch layout: S = 65536 >> K; costs B*2*S*2 B, edges B*T*S*2 B."""

    @staticmethod
    def get_state_count(k: int) -> int:
        if k < 1 or k > 16:
            raise ValueError(f"Trellis parameter K must be between 1 and 16, got {k}")
        return 65536 >> k

    @classmethod
    def estimate_scratch(cls, k: int, t: int = 256, b: int = 256,
                         bytes_per_cost: int = 2, bytes_per_edge: int = 2) -> ScratchAllocation:
        if b <= 0:
            raise ValueError(f"Batch size B must be positive, got {b}")
        if t <= 0:
            raise ValueError(f"Sequence length T must be positive, got {t}")
        s = cls.get_state_count(k)
        costs = b * 2 * s * bytes_per_cost
        edges = b * t * s * bytes_per_edge
        return ScratchAllocation(k, s, t, b, bytes_per_cost, bytes_per_edge, costs, edges,
                                 costs + edges)

    @classmethod
    def calculate_max_batch_size(cls, k: int, available_vram_bytes: int,
                                 vram_reserve_bytes: int = 2 * BYTES_PER_GIB,
                                 max_single_alloc_bytes: Optional[int] = 4 * BYTES_PER_GIB,
                                 t: int = 256, bytes_per_cost: int = 2,
                                 bytes_per_edge: int = 2) -> Tuple[int, ScratchAllocation]:
        usable = available_vram_bytes - vram_reserve_bytes
        if usable <= 0:
            raise ValueError(
                f"Available VRAM ({available_vram_bytes / BYTES_PER_GIB:.2f} GiB) must exceed "
                f"reserve ({vram_reserve_bytes / BYTES_PER_GIB:.2f} GiB)")
        s = cls.get_state_count(k)
        per_b = 2 * s * bytes_per_cost + t * s * bytes_per_edge
        max_b = usable // per_b
        if max_single_alloc_bytes is not None:
            max_b = min(max_b, max_single_alloc_bytes // (t * s * bytes_per_edge))
        if max_b < 1:
            raise ValueError(
                f"Insufficient memory: minimum batch size B=1 requires {per_b / BYTES_PER_MIB:.2f} "
                "MiB, which exceeds allowable memory budget.")
        return int(max_b), cls.estimate_scratch(k=k, t=t, b=int(max_b),
                                                bytes_per_cost=bytes_per_cost,
                                                bytes_per_edge=bytes_per_edge)


def b200_checkpoint_stride(k: int) -> int:
    """Steps between cost checkpoints: the tile-pair encoder (K >= 2) every
    2nd step at K=2 and every step above (``ck_stride``); the single-tile K=1
    encoder every 4th step."""
    if not 1 <= k <= 8:
        raise ValueError(f"K must be in 1..8, got {k}")
    return 4 if k == 1 else (2 if k == 2 else 1)


def b200_checkpoint_slots(k: int, t: int = 256) -> Tuple[int, int]:
    """Checkpointed steps of pass 1 and pass 2 (``ck_slots_pass1/2`` and
    ``single_slots_pass1/2`` in csrc/acs_pair.cu)."""
    r = b200_checkpoint_stride(k)
    return (t - t // 2 - 1) // r + 1, (t - 1) // r


def _checkpoint_word_bytes(k: int) -> int:
    # a pair checkpoint holds {cost_A, cost_B} per edge; K=1's one fp16 per edge
    return 2 if k == 1 else 4


def b200_checkpoint_bytes(k: int, t: int = 256) -> int:
    """Checkpoint workspace of one encoding unit (a tile pair for K >= 2,
    ``pair_ck_bytes``; one tile for K = 1, ``single_ck_bytes``): the larger
    pass's slots x (65536 >> K) edges x word bytes, 256-byte aligned."""
    s1, s2 = b200_checkpoint_slots(k, t)
    b = max(s1, s2) * (65536 >> k) * _checkpoint_word_bytes(k)
    return -(-b // 256) * 256


def b200_hbm_bytes_written_per_tile(k: int, t: int = 256) -> int:
    """Trellis bytes one tile writes to HBM over both passes: every
    checkpoint of its unit (half of a pair's for K >= 2)."""
    s1, s2 = b200_checkpoint_slots(k, t)
    per_unit = (s1 + s2) * (65536 >> k) * _checkpoint_word_bytes(k)
    return per_unit if k == 1 else per_unit // 2


def b200_workspace_bytes(k: int, t: int = 256, b: int = 1) -> int:
    """Device workspace of the B200 encoder for ``b`` tiles (matches
    ``exl3_quantize_tiles_ws_bytes``; K >= 2 rounds ``b`` up to whole pairs)."""
    if k == 1:
        return b * (b200_checkpoint_bytes(k, t) + 8)
    b = b + (b & 1)
    return b * (b200_checkpoint_bytes(k, t) // 2 + 8)
