"""CPU oracle for the EXL3 storage side — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` import this module, as the checker of the container unpack
and weight decode kernels. Restates, in NumPy:

* ``unpack_module_trellis`` (reference ``exl3_quant/serialization.py:65-84``):
  per tile, ``decode_states`` of the SWAP16 container;
* ``decode_weight_from_storage`` (``serialization.py:227-266``): codebook
  value of each state, inverse tensor-core permutation, tiles to the (k, n)
  matrix, then ``weight_from_quantized`` (``exl3_quant/hadamard.py:122-140``):
  H_l @ w on 128-row blocks, x su, w @ H_r on 128-column blocks, x sv, with
  H = Sylvester(128)/sqrt(128) in float32, as the reference computes it.
"""

from __future__ import annotations

import numpy as np

from .trellis_oracle import codebook_lut, decode_states, tensor_core_perm


def sylvester128() -> np.ndarray:
    idx = np.arange(128)
    bits = idx[:, None] & idx[None, :]
    parity = np.zeros_like(bits)
    while bits.any():
        parity ^= bits & 1
        bits = bits >> 1
    return ((1 - 2 * parity) / np.sqrt(128.0)).astype(np.float32)


def unpack_module_trellis(trellis: np.ndarray, K: int) -> np.ndarray:
    tk, tn, pd = trellis.shape
    assert pd == 16 * K
    words = np.asarray(trellis).view(np.uint16)
    out = np.empty((tk, tn, 256), dtype=np.int64)
    for i in range(tk):
        for j in range(tn):
            out[i, j] = decode_states(words[i, j], K)
    return out.astype(np.uint16).view(np.int16)


def w_hat_from_trellis(trellis: np.ndarray, K: int, cb: int) -> np.ndarray:
    tk, tn, _ = trellis.shape
    states = unpack_module_trellis(trellis, K).view(np.uint16).astype(np.int64)
    vals = codebook_lut(cb)[states].astype(np.float32)          # (tk, tn, 256)
    tiles = np.empty_like(vals)
    tiles[..., tensor_core_perm()] = vals
    return tiles.reshape(tk, tn, 16, 16).transpose(0, 2, 1, 3).reshape(tk * 16, tn * 16)


def weight_from_quantized(w_hat: np.ndarray, su: np.ndarray, sv: np.ndarray) -> np.ndarray:
    k, n = w_hat.shape
    H = sylvester128()
    work = w_hat.astype(np.float32).copy()
    for r in range(0, k, 128):
        work[r:r + 128] = H @ work[r:r + 128]
    work = work * su.astype(np.float32).reshape(k, 1)
    for c in range(0, n, 128):
        work[:, c:c + 128] = work[:, c:c + 128] @ H
    return work * sv.astype(np.float32).reshape(1, n)


def decode_weight_from_storage(trellis, suh, svh, K: int, cb: int) -> np.ndarray:
    return weight_from_quantized(w_hat_from_trellis(trellis, K, cb), suh, svh)
