"""Global-scale search (API of ``exl3_quant/gss.py``; upstream ``quantize.py:895-1076``).

Sample tiles along a wrapped diagonal of the tile grid plus the highest and
lowest RMS tiles; try a coarse grid of 10 scales (0.1 .. 1.9) on every third
sampled tile, then 5 scales at 0.075 spacing around the best one on all
sampled tiles, refined by a parabola through the best point and its
neighbours (offset clamped to +-0.5 step, result >= 0.01).

On B200 every (scale, tile) candidate of a stage goes to the encoder in one
call: the encoder chunks internally and the per-scale MSEs are one segmented
reduction on the device.
"""

from __future__ import annotations

from typing import Callable, List, Sequence, Tuple

import torch

from .trellis_format import tensor_core_perm

COARSE_START = 0.1
COARSE_STEP = 0.2
COARSE_POINTS = 10
FINE_POINTS = 5
FINE_STEP = 0.075
MIN_SCALE = 0.01
MAX_TILES_PER_CALL = 1 << 22

TileEncoder = Callable[[torch.Tensor], "tuple[torch.Tensor, torch.Tensor]"]


def sample_scale_tiles(weight_r: torch.Tensor, width: int = 3) -> torch.Tensor:
    """Tiles for the search, tensor-core order, ``(num_tiles, 256)`` (quantize.py:895-916)."""
    device = weight_r.device
    tk, tn = weight_r.shape[0] // 16, weight_r.shape[1] // 16
    w4 = weight_r.reshape(tk, 16, tn, 16)
    diag_len = max(tk, tn)
    ii = torch.arange(diag_len, device=device).repeat_interleave(width)
    ww = torch.arange(width, device=device).repeat(diag_len)
    kk, nn = ii % tk, (ii + ww) % tn
    num_x = max(8, (diag_len * width) // 16)
    tile_ms = w4.square().mean(dim=(1, 3)).flatten()
    num_x = min(num_x, (tile_ms.shape[0] + 1) // 2)
    hi = torch.topk(tile_ms, num_x).indices
    lo = torch.topk(tile_ms, num_x, largest=False).indices
    xk = torch.cat((hi, lo)) // tn
    xn = torch.cat((hi, lo)) % tn
    tiles = w4[torch.cat((kk, xk)), :, torch.cat((nn, xn)), :].reshape(-1, 256)
    perm = torch.as_tensor(tensor_core_perm(), dtype=torch.long, device=device)
    return tiles[:, perm].contiguous()


def select_refined_scale(fine_scales: List[float], fine_mses: List[float]) -> float:
    best = min(range(len(fine_mses)), key=lambda i: fine_mses[i])
    offset = 0.0
    if 0 < best < len(fine_scales) - 1:
        y0, y1, y2 = fine_mses[best - 1], fine_mses[best], fine_mses[best + 1]
        denom = y0 - 2.0 * y1 + y2
        offset = 0.5 * (y0 - y2) / denom if denom > 0 else 0.0
        offset = max(-0.5, min(0.5, offset))
    return max(fine_scales[best] + offset * FINE_STEP, MIN_SCALE)


def _eval(pairs: List[Tuple[int, float]], tile_sets: Sequence[torch.Tensor],
          encode_tiles: TileEncoder, max_tiles: int) -> torch.Tensor:
    """MSE of every (tensor, scale) pair; one encoder call per max_tiles."""
    device = tile_sets[0].device
    out = torch.empty(len(pairs), dtype=torch.float32, device=device)
    i = 0
    while i < len(pairs):
        j, tot = i, 0
        while j < len(pairs) and tot + tile_sets[pairs[j][0]].shape[0] <= max_tiles:
            tot += tile_sets[pairs[j][0]].shape[0]
            j += 1
        j = max(j, i + 1)
        batch = torch.cat([tile_sets[t] * s for t, s in pairs[i:j]])
        q, _ = encode_tiles(batch)
        off = 0
        for p, (t, s) in enumerate(pairs[i:j]):
            cnt = tile_sets[t].shape[0]
            out[i + p] = (q[off:off + cnt] / s - tile_sets[t]).square().mean()
            off += cnt
        i = j
    return out


def g_scale_search_batch(samples: Sequence[torch.Tensor], encode_tiles: TileEncoder,
                         max_tiles: int = MAX_TILES_PER_CALL) -> List[Tuple[float, float]]:
    n_t = len(samples)
    if n_t == 0:
        return []
    for t, s in enumerate(samples):
        if s.dim() != 2 or s.shape[1] != 256 or s.shape[0] < 1:
            raise ValueError(f"samples[{t}] must be (T, 256) tensor-core-order tiles, "
                             f"got {tuple(s.shape)}")
    coarse = [COARSE_START + COARSE_STEP * i for i in range(COARSE_POINTS)]
    subs = [s[::3] for s in samples]
    mse1 = _eval([(t, s) for t in range(n_t) for s in coarse], subs, encode_tiles,
                 max_tiles).reshape(n_t, len(coarse))
    centers = [coarse[c] for c in mse1.argmin(dim=1).tolist()]
    fine = [[c + FINE_STEP * (i - 2) for i in range(FINE_POINTS)] for c in centers]
    mse2 = _eval([(t, s) for t in range(n_t) for s in fine[t]], samples, encode_tiles,
                 max_tiles).reshape(n_t, FINE_POINTS).tolist()
    results = []
    for t in range(n_t):
        best = min(range(FINE_POINTS), key=lambda i: mse2[t][i])
        results.append((select_refined_scale(fine[t], mse2[t]), mse2[t][best]))
    return results


def g_scale_gss(weight_r: torch.Tensor, encode_tiles: TileEncoder, width: int = 3):
    return g_scale_search_batch([sample_scale_tiles(weight_r, width)], encode_tiles)[0]


def g_scale_fn_from_encoder(encode_tiles: TileEncoder, width: int = 3) -> Callable[[torch.Tensor], float]:
    def g_scale_fn(weight_r: torch.Tensor) -> float:
        return g_scale_gss(weight_r, encode_tiles, width)[0]
    return g_scale_fn
