"""Reserve-based admission for the encoder workspace on a CUDA device.

API of the reference ``exl3_quant/memory_policy.py`` (``MemorySnapshot``,
``capture_snapshot``, ``MemoryPressureError``, ``MemoryPolicy``), restated for
a discrete GPU with its own HBM: the budget is the device's free memory plus
what the PyTorch caching allocator holds unused, minus a reserve. The Arc
unified-memory counters of the reference (system RAM shared with the GPU) do
not apply and are reported for information only.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Optional

BYTES_PER_MIB = 1024 ** 2
BYTES_PER_GIB = 1024 ** 3

DEFAULT_RESERVE_BYTES = 2 * BYTES_PER_GIB
DEFAULT_SAFETY_SLACK_BYTES = 256 * BYTES_PER_MIB
ENV_RESERVE_BYTES = "EXL3_MEMORY_RESERVE_BYTES"
ENV_RESERVE_GIB = "EXL3_MEMORY_RESERVE_GIB"


def default_reserve_bytes() -> int:
    if os.environ.get(ENV_RESERVE_BYTES):
        return int(os.environ[ENV_RESERVE_BYTES])
    if os.environ.get(ENV_RESERVE_GIB):
        return int(float(os.environ[ENV_RESERVE_GIB]) * BYTES_PER_GIB)
    return DEFAULT_RESERVE_BYTES


def format_bytes(value: Optional[int]) -> str:
    if value is None:
        return "n/a"
    sign = "-" if value < 0 else ""
    value = abs(value)
    if value >= BYTES_PER_GIB:
        return f"{sign}{value / BYTES_PER_GIB:.2f} GiB"
    if value >= BYTES_PER_MIB:
        return f"{sign}{value / BYTES_PER_MIB:.1f} MiB"
    return f"{sign}{value} B"


def _meminfo() -> dict:
    out = {"MemTotal": 0, "MemAvailable": 0}
    try:
        with open("/proc/meminfo", "r", encoding="ascii") as fh:
            for line in fh:
                key, _, rest = line.partition(":")
                if key in out:
                    out[key] = int(rest.split()[0]) * 1024
    except OSError:
        pass
    return out


@dataclass(frozen=True)
class MemorySnapshot:
    """Point-in-time device (and host) memory counters."""

    gpu_available: bool
    system_total_bytes: int
    system_available_bytes: int
    device_free_bytes: int
    device_total_bytes: int
    device_allocated_bytes: int
    device_reserved_bytes: int

    @property
    def binding_available_bytes(self) -> int:
        """Device bytes a new allocation can obtain: driver-free memory plus
        what the caching allocator holds but does not use."""
        if not self.gpu_available:
            return 0
        return self.device_free_bytes + max(0, self.device_reserved_bytes - self.device_allocated_bytes)

    def as_dict(self) -> dict:
        d = dict(self.__dict__)
        d["binding_available_bytes"] = self.binding_available_bytes
        return d


def capture_snapshot(device_index: int = 0) -> MemorySnapshot:
    sysmem = _meminfo()
    free = total = alloc = resv = 0
    ok = False
    try:
        import torch

        if torch.cuda.is_available():
            free, total = (int(v) for v in torch.cuda.mem_get_info(device_index))
            alloc = int(torch.cuda.memory_allocated(device_index))
            resv = int(torch.cuda.memory_reserved(device_index))
            ok = True
    except Exception:  # pragma: no cover - broken driver
        ok = False
    return MemorySnapshot(ok, sysmem["MemTotal"], sysmem["MemAvailable"], free, total, alloc, resv)


class MemoryPressureError(RuntimeError):
    """An allocation would breach the configured device reserve."""

    def __init__(self, message: str, need_bytes: int, usable_bytes: int,
                 snapshot: MemorySnapshot, context: str = ""):
        super().__init__(message)
        self.need_bytes = need_bytes
        self.usable_bytes = usable_bytes
        self.snapshot = snapshot
        self.context = context

    def as_dict(self) -> dict:
        return {"error": "MemoryPressureError", "context": self.context,
                "need_bytes": self.need_bytes, "usable_bytes": self.usable_bytes,
                "message": str(self), "snapshot": self.snapshot.as_dict()}


@dataclass(frozen=True)
class MemoryPolicy:
    """Keep ``reserve_bytes`` of device memory free; optionally cap any single
    allocation at ``max_single_alloc_bytes``."""

    reserve_bytes: int = field(default_factory=default_reserve_bytes)
    safety_slack_bytes: int = DEFAULT_SAFETY_SLACK_BYTES
    max_single_alloc_bytes: Optional[int] = None

    def usable_bytes(self, snapshot: MemorySnapshot, outstanding_bytes: int = 0) -> int:
        if outstanding_bytes < 0:
            raise ValueError(f"outstanding_bytes must be non-negative, got {outstanding_bytes}")
        return max(0, snapshot.binding_available_bytes - self.reserve_bytes)

    def check(self, need_bytes: int, snapshot: MemorySnapshot,
              outstanding_bytes: int = 0, context: str = "") -> int:
        if need_bytes < 0:
            raise ValueError(f"need_bytes must be non-negative, got {need_bytes}")
        usable = self.usable_bytes(snapshot, outstanding_bytes)
        ctx = f" [{context}]" if context else ""
        if self.max_single_alloc_bytes is not None and need_bytes > self.max_single_alloc_bytes:
            raise MemoryPressureError(
                f"single-allocation ceiling exceeded{ctx}: need {format_bytes(need_bytes)} > "
                f"ceiling {format_bytes(self.max_single_alloc_bytes)}",
                need_bytes, usable, snapshot, context)
        if need_bytes > usable:
            raise MemoryPressureError(
                f"memory-pressure abort{ctx}: need {format_bytes(need_bytes)} but only "
                f"{format_bytes(usable)} usable (reserve {format_bytes(self.reserve_bytes)})",
                need_bytes, usable, snapshot, context)
        return usable

    def check_after_commit(self, snapshot: MemorySnapshot,
                           pre_snapshot: Optional[MemorySnapshot] = None,
                           expected_bytes: int = 0, context: str = "post-commit") -> None:
        if pre_snapshot is not None and expected_bytes > 0:
            growth = snapshot.device_allocated_bytes - pre_snapshot.device_allocated_bytes
            if growth < expected_bytes:
                raise MemoryPressureError(
                    f"allocator commitment failure [{context}]: expected {format_bytes(expected_bytes)}"
                    f" growth, observed {format_bytes(growth)}",
                    expected_bytes, self.usable_bytes(snapshot), snapshot, context)

    def describe(self, snapshot: MemorySnapshot) -> dict:
        return {"reserve_bytes": self.reserve_bytes,
                "safety_slack_bytes": self.safety_slack_bytes,
                "max_single_alloc_bytes": self.max_single_alloc_bytes,
                "usable_bytes": self.usable_bytes(snapshot),
                "snapshot": snapshot.as_dict()}
