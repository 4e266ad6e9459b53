"""Loader for the native layer.

The product path has no CPU fallback: every operation that needs the CUDA
kernels calls :func:`ext` (or :func:`lib`), which raises if the shipped
binaries are missing or stale and cannot be rebuilt, or if no CUDA device is
present.
"""

from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
import threading

from . import _build

_LOCK = threading.Lock()
_EXT = None
_LIB = None


class NativeUnavailable(RuntimeError):
    """The sm_100a kernels cannot be used in this process."""


def lib() -> ctypes.CDLL:
    """``libexl3k.so`` through ctypes (C ABI of ``include/exl3k.h``)."""
    global _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.library_path()
            if not _build._stamp_ok(path, _build.library_digest()):
                _build.build_library()
            _LIB = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
            _declare(_LIB)
        return _LIB


def _declare(handle: ctypes.CDLL) -> None:
    c = ctypes
    handle.exl3_last_error.restype = c.c_char_p
    handle.exl3_version.restype = c.c_char_p
    handle.exl3_quantize_tiles_ws_bytes.restype = c.c_size_t
    handle.exl3_quantize_tiles_ws_bytes.argtypes = [c.c_int64, c.c_int, c.c_int]
    handle.exl3_encoder_set_cluster.argtypes = [c.c_int]
    handle.exl3_encoder_set_cluster_pairs.argtypes = [c.c_int]
    handle.exl3_hessian_set_tile.argtypes = [c.c_int]
    handle.exl3_encoder_fault_count.argtypes = [c.POINTER(c.c_uint)]
    handle.exl3_encoder_test_cluster_wait.argtypes = [c.c_longlong, c.c_int]
    handle.exl3_encoder_cluster_capacity.argtypes = [c.c_int, c.c_int, c.POINTER(c.c_int)]


def _check(rc: int) -> None:
    if rc != 0:
        msg = lib().exl3_last_error()
        raise RuntimeError(msg.decode() if msg else f"libexl3k status {rc}")


def set_encoder_cluster(cluster_ctas: int) -> None:
    """Cluster split of the encoder's ACS passes (``exl3_encoder_set_cluster``):
    0 automatic, 1 never, 2 / 4 / 8 always that many CTAs per tile pair.
    Process-wide; outputs are bit-identical for every setting."""
    _check(lib().exl3_encoder_set_cluster(int(cluster_ctas)))


def set_encoder_cluster_pairs(pairs_per_cluster: int) -> None:
    """Tile pairs per cluster of the cluster-split ACS
    (``exl3_encoder_set_cluster_pairs``): 0 automatic, 1 / 2 forced (2 exists
    for clusters of 8 CTAs). Process-wide; outputs are bit-identical for every
    setting."""
    _check(lib().exl3_encoder_set_cluster_pairs(int(pairs_per_cluster)))


def set_hessian_tile(mode: int) -> None:
    """Tile shape of the Hessian accumulation (``exl3_hessian_set_tile``):
    0 chosen by width (default), 1 = 128 x 256 tiles, 2 = 256 x 256 tiles.
    Process-wide; the sums are bit-identical for every setting."""
    _check(lib().exl3_hessian_set_tile(int(mode)))


def encoder_cluster_capacity(K: int, cluster_ctas: int) -> int:
    """Clusters of ``cluster_ctas`` CTAs of the K-bit encoder that the current
    device holds at once (``exl3_encoder_cluster_capacity``; 0 = not
    available for this K)."""
    v = ctypes.c_int(0)
    _check(lib().exl3_encoder_cluster_capacity(int(K), int(cluster_ctas), ctypes.byref(v)))
    return int(v.value)


def encoder_fault_count() -> int:
    """Encoder CTAs that gave up a bounded inter-CTA wait on the current
    device since the library loaded (``exl3_encoder_fault_count``; 0 when
    every call was valid). Synchronizes the device."""
    v = ctypes.c_uint(0)
    _check(lib().exl3_encoder_fault_count(ctypes.byref(v)))
    return int(v.value)


class EncoderFault(RuntimeError):
    """An encoder CTA gave up a bounded inter-CTA wait while the call ran, so
    the call's trellis states and reconstructions are not valid."""


def set_cluster_wait_test_hook(wait_limit_ns: int, stop_sends_at_step: int) -> None:
    """Test hook of the cluster encoder's error path
    (``exl3_encoder_test_cluster_wait``): from ``stop_sends_at_step`` on,
    every CTA stops sending, so the next waits run out after
    ``wait_limit_ns``. ``(0, -1)`` restores normal operation."""
    _check(lib().exl3_encoder_test_cluster_wait(int(wait_limit_ns), int(stop_sends_at_step)))


class encoder_fault_check:
    """Context manager that raises :class:`EncoderFault` when the encoder's
    fault count on ``device`` grew inside the block. Reading the count
    synchronizes the device (at entry and at exit); a block that raised
    already is left alone. ``delta()`` reads the growth so far, for callers
    that combine it across ranks before raising."""

    def __init__(self, device=None):
        import torch

        self.device = torch.device(device) if device is not None else None
        self.start = 0

    def _count(self) -> int:
        import torch

        if self.device is None or self.device.type != "cuda":
            return 0
        with torch.cuda.device(self.device):
            return encoder_fault_count()

    def delta(self) -> int:
        return self._count() - self.start

    def __enter__(self):
        self.start = self._count()
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc_type is None:
            raise_on_faults(self.delta())
        return False


def raise_on_faults(delta: int) -> None:
    if delta > 0:
        raise EncoderFault(
            f"{delta} encoder CTA(s) gave up a bounded inter-CTA wait during this call; "
            "its trellis states and reconstructions are not valid")


def ext():
    """The PyTorch binding module (``exl3_b200_ext``)."""
    global _EXT
    if _EXT is not None:
        return _EXT
    import torch  # noqa: F401  (libtorch symbols must be loaded first)

    lib()
    with _LOCK:
        if _EXT is None:
            path = _build.extension_path()
            if not _build._stamp_ok(path, _build.extension_digest()):
                _build.build_extension()
            loader = importlib.machinery.ExtensionFileLoader(_build.EXT_NAME, str(path))
            spec = importlib.util.spec_from_file_location(_build.EXT_NAME, str(path), loader=loader)
            module = importlib.util.module_from_spec(spec)
            loader.exec_module(module)
            _EXT = module
    return _EXT


def require_cuda(device=None):
    """Raise unless a CUDA device is usable; returns a ``torch.device``."""
    import torch

    if not torch.cuda.is_available():
        raise NativeUnavailable(
            "no CUDA device: the EXL3 B200 kernels have no CPU fallback")
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    dev = torch.device(device)
    if dev.type != "cuda":
        raise NativeUnavailable(f"device {dev} is not a CUDA device")
    return dev
