"""EXL3 trellis format: codebooks, tile permutation, bitstream packing.

Same names and semantics as the reference module
``exl3_quant/trellis_format.py`` (alpha2beta/EXL3_Intel_Arc_quantizer), which
in turn transcribes upstream exllamav3 (codebook.cuh, pack.cu, quantize.py).
The host-side functions here are the format definition (NumPy). The encoder
path never calls them: it packs on the device (``pack_trellis_cuda`` and the
encoder's fused epilogue).
"""

from __future__ import annotations

import numpy as np

MUL1_MULT = 0x83DCD12D
MCG_MULT = 0xCBAC1FED
THREEINST_MULT = 89226354
THREEINST_ADD = 64248484

CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2

_MUL1_INV_BITS = 0x1EEE
_MUL1_BIAS_BITS = 0xC931


def _half(bits: int) -> float:
    return float(np.array([bits], dtype=np.uint16).view(np.float16)[0])


def codebook_lut(cb: int) -> np.ndarray:
    """fp16 value of each of the 65536 trellis states (trellis_format.py:41-81).

    MUL1: ``h = fp16(1024 + bytesum(s * 0x83DCD12D))``, value
    ``fma(h, fp16(0x1EEE), fp16(0xC931))`` rounded once.
    MCG / 3INST: ``x = (s * mult (+ add)) & 0x8FFF8FFF ^ 0x3B603B60``, value
    ``lo16(x) + hi16(x)`` rounded once.
    """
    if cb not in (CB_3INST, CB_MCG, CB_MUL1):
        raise ValueError(f"Unknown codebook {cb}")
    s = np.arange(65536, dtype=np.uint64)
    if cb == CB_MUL1:
        x = (s * MUL1_MULT) & 0xFFFFFFFF
        bsum = (x & 0xFF) + ((x >> 8) & 0xFF) + ((x >> 16) & 0xFF) + ((x >> 24) & 0xFF)
        h = (1024 + bsum).astype(np.float64)
        return (h * _half(_MUL1_INV_BITS) + _half(_MUL1_BIAS_BITS)).astype(np.float16)
    if cb == CB_3INST:
        x = (s * THREEINST_MULT + THREEINST_ADD) & 0xFFFFFFFF
    else:
        x = (s * MCG_MULT) & 0xFFFFFFFF
    x = ((x & 0x8FFF8FFF) ^ 0x3B603B60) & 0xFFFFFFFF
    lo = (x & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float64)
    hi = (x >> 16).astype(np.uint16).view(np.float16).astype(np.float64)
    return (lo + hi).astype(np.float16)


def tensor_core_perm() -> np.ndarray:
    """16x16 tile permutation: encoded element t is tile position perm[t]
    (trellis_format.py:88-108)."""
    perm = np.empty(256, dtype=np.int64)
    for t in range(32):
        r0, c0 = (t % 4) * 2, t // 4
        rows = (r0, r0 + 1, r0 + 8, r0 + 9)
        for j, c in enumerate((c0, c0 + 8)):
            for i, r in enumerate(rows):
                perm[t * 8 + 4 * j + i] = r * 16 + c
    return perm


def tensor_core_perm_inv() -> np.ndarray:
    return np.argsort(tensor_core_perm())


def pack_trellis(states: np.ndarray, K: int) -> np.ndarray:
    """Pack 256 states into ``16*K`` uint16 words: per 16-element span, the low
    K bits of each state, MSB-first (trellis_format.py:120-159)."""
    if not 1 <= K <= 8:
        raise ValueError(f"K must be in 1..8, got {K}")
    st = np.asarray(states, dtype=np.uint16)
    if st.size != 256:
        raise ValueError(f"Expected 256 states per tile, got {st.size}")
    sym = (st.reshape(16, 16).astype(np.uint32) & ((1 << K) - 1))
    out = np.zeros(16 * K, dtype=np.uint16)
    for span in range(16):
        acc, nb, j = 0, 0, K * span
        for v in sym[span]:
            acc = (acc << K) | int(v)
            nb += K
            if nb >= 16:
                out[j] = (acc >> (nb - 16)) & 0xFFFF
                nb -= 16
                acc &= (1 << nb) - 1
                j += 1
    return out


def swap16_storage(s_packed: np.ndarray) -> np.ndarray:
    """Exchange the two halves of every 32-bit word (pack.cu SWAP16)."""
    p = np.asarray(s_packed, dtype=np.uint16).reshape(-1, 2)
    return np.ascontiguousarray(p[:, ::-1]).reshape(-1)


def words_from_storage(t16: np.ndarray) -> np.ndarray:
    t16 = np.asarray(t16, dtype=np.uint16)
    return t16[0::2].astype(np.uint64) | (t16[1::2].astype(np.uint64) << 16)


def stream_from_words(words: np.ndarray) -> np.ndarray:
    shifts = np.arange(31, -1, -1, dtype=np.uint64)
    return ((np.asarray(words, dtype=np.uint64)[:, None] >> shifts[None, :]) & 1).reshape(-1)


def state_index(K: int) -> np.ndarray:
    """Bit positions of each element's 16-bit window, which ends at bit
    (t+1)*K of the circular tile stream."""
    nbits = 256 * K
    t = np.arange(256)
    b0 = (t * K + K - 16 + nbits) % nbits
    return (b0[:, None] + np.arange(16)[None, :]) % nbits


def decode_states(t16: np.ndarray, K: int) -> np.ndarray:
    """Packed tile (SWAP16 storage) -> the 256 16-bit states."""
    bits = stream_from_words(words_from_storage(t16))
    win = bits[state_index(K)]
    return (win * (1 << np.arange(15, -1, -1))[None, :]).sum(-1).astype(np.int64)


def decode_tile_values(t16: np.ndarray, K: int, cb: int = CB_MUL1) -> np.ndarray:
    """Packed tile -> 256 fp16 values scattered back to tile order."""
    vals = codebook_lut(cb)[decode_states(t16, K)]
    tile = np.empty(256, dtype=np.float16)
    tile[tensor_core_perm()] = vals
    return tile


# ---------------------------------------------------------------------------
# Device versions (CUDA kernels in libexl3k)
# ---------------------------------------------------------------------------

def codebook_lut_cuda(cb: int, device=None):
    """All 65536 codebook values decoded on the GPU (fp16 tensor)."""
    import torch

    from ._ext import ext, require_cuda

    dev = require_cuda(device)
    out = torch.empty(65536, dtype=torch.float16, device=dev)
    ext().decode_codebook(int(cb), out)
    return out


def pack_trellis_cuda(states, K: int):
    """(n, 256) int16 states on the GPU -> (n, 16*K) int16 container words in
    SWAP16 storage order (``swap16_storage(pack_trellis(...))`` per tile)."""
    import torch

    from ._ext import ext

    st = states.reshape(-1, 256).to(torch.int16).contiguous()
    out = torch.empty((st.shape[0], 16 * K), dtype=torch.int16, device=st.device)
    if st.shape[0]:
        ext().pack_trellis(st, out, int(K))
    return out
