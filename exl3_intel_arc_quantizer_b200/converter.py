"""Layer conversion pipeline on one or more GPUs.

The per-layer steps of the reference's model loop
(``exl3_quant/converter.py:1452-1612``), without its file handling
(safetensors streaming, checkpoints, resume), which is outside the hot path:

1. capture the grouped Hessians of the layer on the current hidden states
   (``calibration.HessianCollector``, tensor-core accumulation);
2. quantize every projection (``layer_quant.quantize_modules``: batched
   global-scale search, one block-LDL per shared Hessian, interleaved LDLQ);
3. reload the quantized numerics (``w_hat``) into the layer
   (``converter.py:993-1003``);
4. re-forward the same pre-layer hidden states through the quantized layer
   to produce the next layer's inputs.

On several GPUs (a ``torch.distributed`` process group, one process per GPU)
each rank holds its own share of the calibration sequences: step 1 runs on
the local share and one NCCL all-reduce per Hessian group (plus the token
counts) gives every rank the Hessians of all tokens; step 2 shards every
module's columns over the ranks and all-gathers them; steps 3 and 4 are
local. Every rank ends with identical layer weights.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from .calibration import (
    DEFAULT_DAMPING_LAMBDA,
    DEFAULT_HEAD_DIM,
    DEFAULT_ZERO_CHANNEL_FLOOR,
    HessianCollector,
    enumerate_linear_modules,
    make_rotary_embeddings,
)
from .layer_quant import QuantizedModuleResult, quantize_modules
from .ldlq import DEFAULT_BLOCK_SIZE, DEFAULT_BUF_SIZE_K, make_xpu_tile_encoder
from .trellis_format import CB_MUL1


@dataclass
class LayerConversionTimings:
    calibrate_s: float = 0.0
    reduce_s: float = 0.0
    quantize_s: float = 0.0
    reload_reforward_s: float = 0.0
    total_s: float = 0.0
    local_tokens: int = 0
    tiles: int = 0
    damping: Dict[str, float] = field(default_factory=dict)


def default_layer_runner(layer: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """Llama-style forward with rotary embeddings (converter.py:1340-1346)."""
    hd = getattr(layer.self_attn, "head_dim", DEFAULT_HEAD_DIM)
    return layer(x, position_embeddings=make_rotary_embeddings(x.shape[1], hd, device=x.device))


def getattr_path(root, dotted: str):
    obj = root
    for part in dotted.split("."):
        obj = getattr(obj, part)
    return obj


def reload_quantized(layer: nn.Module, results: Dict[str, QuantizedModuleResult]) -> None:
    """Swap each module's quantized numerics into the layer: ``w_hat`` is
    (in, out); ``nn.Linear.weight`` is (out, in) (converter.py:993-1003)."""
    for name, res in results.items():
        module = getattr_path(layer, name)
        module.weight.data.copy_(res.w_hat.detach().T.contiguous().to(module.weight.dtype))


def _sync(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def convert_layer(layer: nn.Module, hidden_states: List[torch.Tensor], K: int = 2,
                  cb: int = CB_MUL1, device: Optional[torch.device] = None, group=None,
                  damping_lambda: float = DEFAULT_DAMPING_LAMBDA,
                  zero_floor: float = DEFAULT_ZERO_CHANNEL_FLOOR, skip_g_scale: bool = True,
                  buf_size_k: int = DEFAULT_BUF_SIZE_K, block_size: int = DEFAULT_BLOCK_SIZE,
                  module_names: Optional[List[str]] = None,
                  layer_runner: Optional[Callable[[nn.Module, torch.Tensor], torch.Tensor]] = None,
                  tile_encoder=None
                  ) -> Tuple[Dict[str, QuantizedModuleResult], List[torch.Tensor],
                             LayerConversionTimings]:
    """Convert one decoder layer in place; returns the module results, the
    next layer's hidden states (this rank's share) and phase timings."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("convert_layer needs a CUDA device (no CPU path)")
    runner = layer_runner or default_layer_runner
    tm = LayerConversionTimings()
    _sync(device)
    t0 = time.perf_counter()

    layer.eval()
    layer.to(device=device, dtype=torch.float16)
    col = HessianCollector(layer, device=device)
    try:
        with torch.no_grad():
            for x in hidden_states:
                x = x.to(device=device, dtype=torch.float16)
                tm.local_tokens += x.shape[0] * x.shape[1]
                runner(layer, x)
    finally:
        col.close()
    _sync(device)
    t1 = time.perf_counter()
    if group is not None:
        from .distributed import finalize_collector_distributed

        hessians, damping = finalize_collector_distributed(col, damping_lambda, zero_floor, group)
    else:
        hessians, damping = col.finalize(damping_lambda=damping_lambda, zero_floor=zero_floor)
    tm.damping = damping
    del col
    _sync(device)
    t2 = time.perf_counter()

    linears = enumerate_linear_modules(layer)
    names = list(linears) if module_names is None else list(module_names)
    missing = [nm for nm in names if nm not in linears or nm not in hessians]
    if missing:
        raise KeyError(f"modules without a linear or a Hessian: {missing}")
    if tile_encoder is None:
        tile_encoder = make_xpu_tile_encoder(K=K, device_index=device.index or 0)
    modules = {nm: (linears[nm].weight.data, hessians[nm]) for nm in names}
    results = quantize_modules(modules, K=K, cb=cb, tile_encoder=tile_encoder,
                               skip_g_scale=skip_g_scale, buf_size_k=buf_size_k,
                               block_size=block_size, group=group)
    tm.tiles = sum(r.encoded.shape[0] * r.encoded.shape[1] for r in results.values())
    del hessians
    _sync(device)
    t3 = time.perf_counter()

    reload_quantized(layer, results)
    with torch.no_grad():
        nxt = [runner(layer, x.to(device=device, dtype=torch.float16)) for x in hidden_states]
    _sync(device)
    t4 = time.perf_counter()
    tm.calibrate_s, tm.reduce_s, tm.quantize_s = t1 - t0, t2 - t1, t3 - t2
    tm.reload_reforward_s, tm.total_s = t4 - t3, t4 - t0
    return results, nxt, tm


def convert_layers(layers: List[nn.Module], hidden_states: List[torch.Tensor], K: int = 2,
                   **kwargs) -> Tuple[List[Dict[str, QuantizedModuleResult]],
                                      List[LayerConversionTimings]]:
    """The layer loop: layers in order, each on the previous one's outputs
    (converter.py:1452-1612, without its file handling)."""
    all_results, timings = [], []
    hs = hidden_states
    for layer in layers:
        res, hs, tm = convert_layer(layer, hs, K=K, **kwargs)
        all_results.append(res)
        timings.append(tm)
    return all_results, timings
