"""Hessian calibration (API of ``exl3_quant/calibration.py``).

``HessianCollector`` hooks one projection per shared input and accumulates
``H += X^T X`` in fp32 on the device, one Hessian per input group (q/k/v
share one, gate/up share one, o and down alone); ``finalize`` divides by the
token count, adds ``max(1e-8, lambda * mean(diag))`` to the diagonal and
floors near-zero diagonal entries, on the device (``exl3_hessian_finalize``).
``hessian_accumulate_`` is the accumulation kernel entry
(``exl3_hessian_accumulate``): fp16 / bf16 activations, fp32 sums.

The Llama-style ``TransformerDecoderLayer`` only drives calibration (it is
the reference's calibration model, not part of the encoder path).
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

DEFAULT_HIDDEN_SIZE = 4096
DEFAULT_INTERMEDIATE_SIZE = 14336
DEFAULT_NUM_ATTN_HEADS = 32
DEFAULT_NUM_KV_HEADS = 8
DEFAULT_HEAD_DIM = 128
DEFAULT_RMS_NORM_EPS = 1e-5
DEFAULT_DAMPING_LAMBDA = 0.01
DEFAULT_ZERO_CHANNEL_FLOOR = 1e-7


# ---------------------------------------------------------------------------
# Calibration model (drives the hooks)
# ---------------------------------------------------------------------------

class LlamaRMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = DEFAULT_RMS_NORM_EPS):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=torch.float16))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        h = x.to(torch.float32)
        h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + self.variance_epsilon)
        return self.weight * h.to(dt)


class LlamaMLP(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class LlamaAttention(nn.Module):
    def __init__(self, hidden_size: int = DEFAULT_HIDDEN_SIZE, num_heads: int = DEFAULT_NUM_ATTN_HEADS,
                 num_kv_heads: int = DEFAULT_NUM_KV_HEADS, head_dim: Optional[int] = None):
        super().__init__()
        self.num_heads, self.num_kv_heads = num_heads, num_kv_heads
        self.head_dim = head_dim or hidden_size // num_heads
        self.q_proj = nn.Linear(hidden_size, num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * self.head_dim, hidden_size, bias=False)

    @staticmethod
    def _rotate_half(x: torch.Tensor) -> torch.Tensor:
        h = x.shape[-1] // 2
        return torch.cat((-x[..., h:], x[..., :h]), dim=-1)

    def forward(self, x, position_embeddings=None, attention_mask=None):
        b, s, _ = x.shape
        q = self.q_proj(x).view(b, s, self.num_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(b, s, self.num_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, s, self.num_kv_heads, self.head_dim).transpose(1, 2)
        if position_embeddings is not None:
            cos, sin = position_embeddings
            q = q * cos + self._rotate_half(q) * sin
            k = k * cos + self._rotate_half(k) * sin
        rep = self.num_heads // self.num_kv_heads
        if rep > 1:
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        att = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(self.head_dim))
        if attention_mask is not None:
            att = att + attention_mask
        att = F.softmax(att, dim=-1, dtype=torch.float32).to(q.dtype)
        out = torch.matmul(att, v).transpose(1, 2).contiguous().view(b, s, -1)
        return self.o_proj(out)


class TransformerDecoderLayer(nn.Module):
    def __init__(self, hidden_size: int = DEFAULT_HIDDEN_SIZE,
                 intermediate_size: int = DEFAULT_INTERMEDIATE_SIZE,
                 num_heads: int = DEFAULT_NUM_ATTN_HEADS, num_kv_heads: int = DEFAULT_NUM_KV_HEADS,
                 rms_norm_eps: float = DEFAULT_RMS_NORM_EPS):
        super().__init__()
        self.hidden_size, self.intermediate_size = hidden_size, intermediate_size
        self.input_layernorm = LlamaRMSNorm(hidden_size, rms_norm_eps)
        self.self_attn = LlamaAttention(hidden_size, num_heads, num_kv_heads)
        self.post_attention_layernorm = LlamaRMSNorm(hidden_size, rms_norm_eps)
        self.mlp = LlamaMLP(hidden_size, intermediate_size)

    def forward(self, hidden_states, position_embeddings=None, attention_mask=None):
        h = hidden_states + self.self_attn(self.input_layernorm(hidden_states),
                                           position_embeddings, attention_mask)
        return h + self.mlp(self.post_attention_layernorm(h))


def make_rotary_embeddings(seq_len: int, head_dim: int = DEFAULT_HEAD_DIM, base: float = 500000.0,
                           device: Optional[torch.device] = None,
                           dtype: torch.dtype = torch.float16) -> Tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    fr = torch.outer(torch.arange(seq_len, dtype=torch.float32, device=device), inv)
    emb = torch.cat((fr, fr), dim=-1)
    return (emb.cos().to(dtype)[None, None], emb.sin().to(dtype)[None, None])


# ---------------------------------------------------------------------------
# Hessian accumulation
# ---------------------------------------------------------------------------

_ERR_FLAGS: Dict[int, torch.Tensor] = {}


def _err_flag(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    f = _ERR_FLAGS.get(idx)
    if f is None:
        f = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR_FLAGS[idx] = f
    return f


def hessian_accumulate_(H: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """In place ``H += x^T x`` for ``x`` of shape (tokens, d) on the CUDA
    device of ``H``: tensor-core products of fp16/bf16 activations, fp32 sums.
    fp32 activations are first rounded to the layer's fp16."""
    from ._ext import ext, require_cuda

    require_cuda(H.device)
    if H.dtype != torch.float32 or H.dim() != 2 or H.shape[0] != H.shape[1]:
        raise ValueError("H must be a square float32 matrix")
    if x.dim() != 2 or x.shape[1] != H.shape[0]:
        raise ValueError(f"x must be (tokens, {H.shape[0]}), got {tuple(x.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        x = x.to(torch.float16)
    ext().hessian_accumulate_(H, x.contiguous(), _err_flag(H.device))
    return H


def check_accumulate_errors(device: torch.device) -> None:
    """Raise if a tensor-core accumulation on ``device`` timed out (reads the
    device flag: synchronizes)."""
    f = _ERR_FLAGS.get(device.index if device.index is not None else torch.cuda.current_device())
    if f is not None and int(f.item()) != 0:
        f.zero_()
        raise RuntimeError("hessian_accumulate: a tensor-core completion wait timed out")


def hessian_finalize_(H: torch.Tensor, count: int, damping_lambda: float = DEFAULT_DAMPING_LAMBDA,
                      zero_floor: float = DEFAULT_ZERO_CHANNEL_FLOOR) -> float:
    """In place finalize on the device; returns the damping added."""
    from ._ext import ext, require_cuda

    require_cuda(H.device)
    damp = torch.empty(1, dtype=torch.float32, device=H.device)
    ext().hessian_finalize_(H, int(max(1, count)), float(damping_lambda), float(zero_floor), damp)
    return float(damp.item())


@dataclass
class CalibrationTelemetry:
    total_tokens: int
    batches_processed: int
    elapsed_time_seconds: float
    peak_allocated_bytes: int
    peak_reserved_bytes: int
    initial_memory: object
    final_memory: object
    operator_fallbacks: List[str] = field(default_factory=list)
    hessian_shapes: Dict[str, Tuple[int, int]] = field(default_factory=dict)
    hessian_dtypes: Dict[str, str] = field(default_factory=dict)
    damping_applied: Dict[str, float] = field(default_factory=dict)


def enumerate_linear_modules(layer: nn.Module) -> Dict[str, nn.Linear]:
    return {nm: m for nm, m in layer.named_modules() if isinstance(m, nn.Linear) and m.bias is None}


def hessian_groups(layer: nn.Module, modules: Optional[Dict[str, nn.Linear]] = None
                   ) -> Dict[str, List[str]]:
    """Projections that read the same input share one Hessian."""
    modules = enumerate_linear_modules(layer) if modules is None else modules
    groups: Dict[str, List[str]] = {}
    table = (("self_attn.input", ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj")),
             ("self_attn.o_proj", ("self_attn.o_proj",)),
             ("linear_attn.input", ("linear_attn.in_proj_qkv", "linear_attn.in_proj_z",
                                    "linear_attn.in_proj_b", "linear_attn.in_proj_a")),
             ("linear_attn.out_proj", ("linear_attn.out_proj",)),
             ("mlp.input", ("mlp.gate_proj", "mlp.up_proj")),
             ("mlp.down_proj", ("mlp.down_proj",)))
    for key, names in table:
        present = [nm for nm in names if nm in modules]
        if present:
            groups[key] = present
    assigned = {nm for v in groups.values() for nm in v}
    for nm in modules:
        if nm not in assigned:
            groups[nm] = [nm]
    return groups


class HessianCollector:
    def __init__(self, layer: nn.Module, device: torch.device, dtype: torch.dtype = torch.float32,
                 groups: Optional[Dict[str, List[str]]] = None):
        if dtype != torch.float32:
            raise ValueError("Hessians accumulate in float32")
        self.layer, self.device, self.dtype = layer, torch.device(device), dtype
        self.modules = enumerate_linear_modules(layer)
        self.groups = hessian_groups(layer, self.modules) if groups is None else groups
        for key, members in self.groups.items():
            if not members:
                raise ValueError(f"Hessian group {key!r} has no members")
            if members[0] not in self.modules:
                raise ValueError(f"Hessian group {key!r} representative {members[0]!r} is not a "
                                 "bias-free linear module of this layer")
        self.hessians: Dict[str, torch.Tensor] = {}
        self.token_counts: Dict[str, int] = {}
        self.handles = []
        for key, members in self.groups.items():
            def hook(module, inp, out, _key=key):
                if not inp:
                    raise RuntimeError(f"hooked module for group {_key!r} got no input")
                self._accumulate(_key, inp[0].detach())
            self.handles.append(self.modules[members[0]].register_forward_hook(hook))

    def _accumulate(self, key: str, x: torch.Tensor) -> None:
        d = x.shape[-1]
        tokens = x.numel() // d
        xf = x.reshape(-1, d).to(self.device)
        if key not in self.hessians:
            self.hessians[key] = torch.zeros((d, d), dtype=torch.float32, device=self.device)
            self.token_counts[key] = 0
        hessian_accumulate_(self.hessians[key], xf)
        self.token_counts[key] += tokens

    def close(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles.clear()

    def finalize(self, damping_lambda: float = DEFAULT_DAMPING_LAMBDA,
                 zero_floor: float = DEFAULT_ZERO_CHANNEL_FLOOR):
        out_map: Dict[str, torch.Tensor] = {}
        damp_map: Dict[str, float] = {}
        norm: Dict[str, Tuple[torch.Tensor, float]] = {}
        if self.hessians:
            check_accumulate_errors(next(iter(self.hessians.values())).device)
        for key, H in self.hessians.items():
            Hn = H.clone()
            damp = hessian_finalize_(Hn, self.token_counts.get(key, 1), damping_lambda, zero_floor)
            norm[key] = (Hn, damp)
        for key, members in self.groups.items():
            if key not in norm:
                continue
            Hn, damp = norm[key]
            for pos, nm in enumerate(members):
                out_map[nm] = Hn.clone() if pos < len(members) - 1 else Hn
                damp_map[nm] = damp
        return out_map, damp_map


def calibrate_layer(layer: nn.Module, calibration_data: List[torch.Tensor], device: torch.device,
                    damping_lambda: float = DEFAULT_DAMPING_LAMBDA, memory_policy=None,
                    zero_floor: float = DEFAULT_ZERO_CHANNEL_FLOOR,
                    layer_runner: Optional[Callable[[nn.Module, torch.Tensor], torch.Tensor]] = None,
                    hessian_groups: Optional[Dict[str, List[str]]] = None):
    from .memory_policy import capture_snapshot

    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("calibrate_layer needs a CUDA device (no CPU accumulation path)")
    di = device.index or 0
    init_mem = capture_snapshot(di)
    layer.eval()
    layer.to(device=device, dtype=torch.float16)
    col = HessianCollector(layer, device=device, groups=hessian_groups)
    t0 = time.time()
    total = batches = 0
    torch.cuda.reset_peak_memory_stats(di)
    try:
        with torch.no_grad():
            for batch in calibration_data:
                x = batch.to(device=device, dtype=torch.float16)
                b, s, _ = x.shape
                total += b * s
                batches += 1
                if layer_runner is not None:
                    layer_runner(layer, x)
                else:
                    hd = getattr(layer.self_attn, "head_dim", DEFAULT_HEAD_DIM)
                    layer(x, position_embeddings=make_rotary_embeddings(s, hd, device=device))
        torch.cuda.synchronize(di)
    finally:
        col.close()
    elapsed = time.time() - t0
    hessians, damping = col.finalize(damping_lambda=damping_lambda, zero_floor=zero_floor)
    tel = CalibrationTelemetry(
        total_tokens=total, batches_processed=batches, elapsed_time_seconds=elapsed,
        peak_allocated_bytes=int(torch.cuda.max_memory_allocated(di)),
        peak_reserved_bytes=int(torch.cuda.max_memory_reserved(di)),
        initial_memory=init_mem, final_memory=capture_snapshot(di),
        hessian_shapes={k: tuple(h.shape) for k, h in hessians.items()},
        hessian_dtypes={k: str(h.dtype) for k, h in hessians.items()}, damping_applied=damping)
    return hessians, tel
