"""Drop-in for an unmodified reference checkout (``exl3_quant``).

The reference's device path enters through one module:
``exl3_quant.xpu_quantizer`` (``XPUTrellisEncoder``, ``ScratchArena``,
``CB_MUL1``), which its ``ldlq.make_xpu_tile_encoder`` (ldlq.py:344-387) and
``layer_quant`` (layer_quant.py:44) import by name. Its Hessian capture adds
``X^T X`` in ``calibration.HessianCollector._accumulate``
(calibration.py:337-352). :func:`install` points both at this package, in
the running process only:

* ``sys.modules["exl3_quant.xpu_quantizer"]`` becomes
  :mod:`exl3_intel_arc_quantizer_b200.xpu_quantizer`, whose
  ``XPUTrellisEncoder`` keeps the reference's constructor, ``encode_tile``,
  ``encode_batch`` and ``encode_batch_detailed`` (bit-exact states and
  reconstructions), so the reference's own ``ldlq``, ``gss`` and
  ``quantize_linear_module`` run their loops with the B200 encoder;
* ``HessianCollector._accumulate`` adds fp16/bf16 activations on a CUDA
  device with the tcgen05 kernel (``hessian_accumulate_``; products of 16-bit
  values are exact in fp32, so only the summation order differs from the
  reference's fp32 GEMM); other inputs keep the reference's own code;
* with ``reference_encoder=True``, the reference's CPU-encoder factory
  ``make_reference_tile_encoder`` (ldlq.py:317-341, which its
  ``quantize_linear_module`` and ``quantize_decoder_layer`` use on every
  non-XPU device, so its ``convert_model`` too) also returns the B200
  encoder: it emits the same states and reconstructions bit for bit, on
  tiles of any device.

Call it before the reference imports ``exl3_quant.layer_quant`` (which binds
the encoder class at import time); ``ldlq.make_xpu_tile_encoder`` looks the
module up at each call. Nothing here renames this package or edits the
reference's files.
"""

from __future__ import annotations

import importlib
import sys
from typing import Optional

REFERENCE_PACKAGE = "exl3_quant"


def install(package: str = REFERENCE_PACKAGE, hessian: bool = True,
            reference_encoder: bool = False):
    """Route the reference package ``package`` (importable from ``sys.path``)
    to the B200 path; returns the reference package module. Idempotent."""
    from . import xpu_quantizer

    pkg = sys.modules.get(package) or importlib.import_module(package)
    sys.modules[f"{package}.xpu_quantizer"] = xpu_quantizer
    setattr(pkg, "xpu_quantizer", xpu_quantizer)
    if hessian:
        _patch_hessian(importlib.import_module(f"{package}.calibration"))
    if reference_encoder:
        _patch_reference_encoder(package)
    return pkg


def _b200_reference_encoder(K: int = 2):
    """``make_reference_tile_encoder``'s contract (MUL1 codebook; tiles on any
    device in, reconstruction and int16 states on that device out) served by
    the B200 encoder on the current CUDA device."""
    import torch

    from .ldlq import make_xpu_tile_encoder

    return make_xpu_tile_encoder(K=K, device_index=torch.cuda.current_device())


_b200_reference_encoder._exl3_b200 = True


def _patch_reference_encoder(package: str) -> None:
    for name in ("ldlq", "layer_quant"):
        mod = importlib.import_module(f"{package}.{name}")
        current = getattr(mod, "make_reference_tile_encoder", None)
        if current is None or getattr(current, "_exl3_b200", False):
            continue
        _b200_reference_encoder.__dict__.setdefault("reference", {})[mod.__name__] = current
        mod.make_reference_tile_encoder = _b200_reference_encoder


def installed(package: str = REFERENCE_PACKAGE) -> bool:
    from . import xpu_quantizer

    return sys.modules.get(f"{package}.xpu_quantizer") is xpu_quantizer


def _patch_hessian(calibration) -> None:
    cls = calibration.HessianCollector
    if getattr(cls._accumulate, "_exl3_b200", False):
        return
    reference_accumulate = cls._accumulate

    def _accumulate(self, key: str, x, _ref=reference_accumulate):
        import torch

        from .calibration import hessian_accumulate_

        dev = torch.device(self.device) if self.device is not None else x.device
        if (dev.type != "cuda" or self.dtype != torch.float32
                or x.dtype not in (torch.float16, torch.bfloat16)):
            return _ref(self, key, x)
        d = x.shape[-1]
        x_flat = x.reshape(-1, d).to(device=dev).contiguous()
        if key not in self.hessians:
            self.hessians[key] = torch.zeros((d, d), device=dev, dtype=torch.float32)
            self.token_counts[key] = 0
        hessian_accumulate_(self.hessians[key], x_flat)
        self.token_counts[key] += x_flat.shape[0]

    _accumulate._exl3_b200 = True
    _accumulate.reference = reference_accumulate
    cls._accumulate = _accumulate


def uninstall(package: str = REFERENCE_PACKAGE) -> None:
    """Undo :func:`install` (the reference's own module is imported again on
    next use)."""
    sys.modules.pop(f"{package}.xpu_quantizer", None)
    pkg: Optional[object] = sys.modules.get(package)
    if pkg is not None and hasattr(pkg, "xpu_quantizer"):
        delattr(pkg, "xpu_quantizer")
    cal = sys.modules.get(f"{package}.calibration")
    if cal is not None:
        acc = cal.HessianCollector._accumulate
        if getattr(acc, "_exl3_b200", False):
            cal.HessianCollector._accumulate = acc.reference
    saved = _b200_reference_encoder.__dict__.get("reference", {})
    for modname, original in list(saved.items()):
        mod = sys.modules.get(modname)
        if mod is not None and getattr(mod, "make_reference_tile_encoder", None) is \
                _b200_reference_encoder:
            mod.make_reference_tile_encoder = original
        del saved[modname]
