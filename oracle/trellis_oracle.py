"""CPU oracle for the EXL3 trellis encoder — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, always as the checker. The product package
never imports it; its encoder path has no CPU fallback.

Two independent restatements of the reference encoder
(alpha2beta/EXL3_Intel_Arc_quantizer, ``exl3_quant/reference_encoder.py``):

* :class:`NumpyOracle` — vectorised NumPy, one array op per branch per step,
  the same formulation as the reference (``reference_encoder.py:130-324``);
* :class:`COracle` — the plain-C restatement in ``oracle/trellis_oracle.c``
  (built by ``oracle/Makefile``), multi-threaded over tiles; fast enough to be
  the checker at thousands of tiles and the timed CPU baseline.

Both are pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).

Format helpers restate ``exl3_quant/trellis_format.py``:
codebook (:41-81), tensor-core permutation (:88-113), pack (:120-159),
SWAP16 (:162-174), decode (:177-213).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path
from typing import Optional

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
H_INF_BITS = 0x7C00
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2


# ---------------------------------------------------------------------------
# Format (trellis_format.py)
# ---------------------------------------------------------------------------

def _h(bits: int) -> float:
    return float(np.array([bits], dtype=np.uint16).view(np.float16)[0])


def codebook_lut(cb: int) -> np.ndarray:
    """fp16 value of every 16-bit state (trellis_format.py:41-81)."""
    s = np.arange(65536, dtype=np.uint64)
    if cb == CB_MUL1:
        x = (s * 0x83DCD12D) & 0xFFFFFFFF
        bsum = sum(((x >> sh) & 0xFF) for sh in (0, 8, 16, 24))
        h = (1024 + bsum).astype(np.float64)       # exact in fp16 (<= 2044)
        return (h * _h(0x1EEE) + _h(0xC931)).astype(np.float16)
    if cb == CB_3INST:
        x = (s * 89226354 + 64248484) & 0xFFFFFFFF
    elif cb == CB_MCG:
        x = (s * 0xCBAC1FED) & 0xFFFFFFFF
    else:
        raise ValueError(f"unknown codebook {cb}")
    x = ((x & 0x8FFF8FFF) ^ 0x3B603B60) & 0xFFFFFFFF
    lo = (x & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float64)
    hi = (x >> 16).astype(np.uint16).view(np.float16).astype(np.float64)
    return (lo + hi).astype(np.float16)


def tensor_core_perm() -> np.ndarray:
    """Encoder element t is tile position perm[t] (trellis_format.py:88-108)."""
    t = np.arange(32)
    r0 = (t % 4) * 2
    c0 = t // 4
    rows = np.stack([r0, r0 + 1, r0 + 8, r0 + 9, r0, r0 + 1, r0 + 8, r0 + 9], axis=1)
    cols = np.stack([c0, c0, c0, c0, c0 + 8, c0 + 8, c0 + 8, c0 + 8], axis=1)
    return (rows * 16 + cols).reshape(-1).astype(np.int64)


def tensor_core_perm_inv() -> np.ndarray:
    return np.argsort(tensor_core_perm())


def pack_trellis(states: np.ndarray, K: int) -> np.ndarray:
    """Low K bits of each state, MSB-first, 16 spans of 16 (pre-SWAP16)."""
    st = np.asarray(states, dtype=np.uint16).reshape(16, 16).astype(np.uint64)
    sym = st & ((1 << K) - 1)
    bits = ((sym[:, :, None] >> np.arange(K - 1, -1, -1, dtype=np.uint64)) & 1)
    bits = bits.reshape(16, 16 * K).reshape(16, K, 16)          # K words per span
    words = (bits << np.arange(15, -1, -1, dtype=np.uint64)).sum(-1)
    return words.reshape(-1).astype(np.uint16)


def swap16_storage(packed: np.ndarray) -> np.ndarray:
    p = np.asarray(packed, dtype=np.uint16).reshape(-1, 2)
    return p[:, ::-1].reshape(-1).copy()


def decode_states(t16: np.ndarray, K: int) -> np.ndarray:
    """Packed (SWAP16 storage) tile -> 256 states; element t's 16-bit window
    ends at bit (t+1)*K of the circular stream (trellis_format.py:177-213)."""
    t16 = np.asarray(t16, dtype=np.uint16)
    words = t16[0::2].astype(np.uint64) | (t16[1::2].astype(np.uint64) << 16)
    stream = ((words[:, None] >> np.arange(31, -1, -1, dtype=np.uint64)) & 1).reshape(-1)
    nbits = 256 * K
    start = (np.arange(256) * K + K - 16) % nbits
    win = stream[(start[:, None] + np.arange(16)[None, :]) % nbits]
    return (win * (1 << np.arange(15, -1, -1))).sum(-1).astype(np.int64)


# ---------------------------------------------------------------------------
# NumPy restatement of the encoder (reference_encoder.py:130-324)
# ---------------------------------------------------------------------------

class NumpyOracle:
    """Two-pass tail-biting Viterbi encoder, vectorised over edges."""

    def __init__(self, K: int, cb: int = CB_MUL1, L: int = 256):
        if not 1 <= K <= 8:
            raise ValueError("K must be in 1..8")
        self.K, self.cb, self.L = K, cb, L
        self.S = 65536 >> K
        self.lut = codebook_lut(cb)
        e = np.arange(self.S, dtype=np.uint32)
        self.vals = []
        self.preds = []
        for k in range(1 << K):
            st = (np.uint32(k) << np.uint32(16 - K)) | e
            self.vals.append(self.lut[st])
            self.preds.append((st >> np.uint32(K)).astype(np.int64))

    def forward(self, w16: np.ndarray, roll: int, pre_state: int,
                edges: Optional[np.ndarray] = None) -> np.ndarray:
        inf = np.float16(np.inf)
        prev = None
        for i in range(self.L):
            ri = (i + roll) % self.L
            w = w16[ri]
            best = None
            bpred = None
            for k in range(1 << self.K):
                d = (self.vals[k] - w).astype(np.float64)          # fp16 subtract
                if prev is None:
                    err = (d * d).astype(np.float16)
                    if pre_state >= 0:
                        err = np.where(self.preds[k] != pre_state, inf, err).astype(np.float16)
                else:
                    err = (d * d + prev[self.preds[k]].astype(np.float64)).astype(np.float16)
                if k == 0:
                    best = err.copy()
                    bpred = self.preds[k].copy()
                else:
                    take = err < best
                    best[take] = err[take]
                    bpred[take] = self.preds[k][take]
            if edges is not None:
                edges[ri] = bpred
            prev = best
        return prev

    @staticmethod
    def argmin(costs: np.ndarray) -> int:
        if not np.any(np.isfinite(costs)) or np.all(costs == np.float16(np.inf)):
            return 0
        return int(np.argmin(costs))

    def encode(self, tile: np.ndarray) -> dict:
        """Encode one tile already in encoder order."""
        w16 = np.asarray(tile, dtype=np.float32).reshape(-1).astype(np.float16)
        L, K = self.L, self.K
        edges = np.zeros((L, self.S), dtype=np.int64)
        c1 = self.forward(w16, L // 2, -1, edges)
        e = self.argmin(c1)
        for i in range(L - 1, -1, -1):
            ri = (i + L // 2) % L
            e = int(edges[ri, e])
            if ri == 0:
                break
        end_state = e
        c2 = self.forward(w16, 0, end_state, edges)
        idx = np.zeros(L, dtype=np.uint16)
        for i in range(L - 1, -1, -1):
            prev = int(edges[i, e])
            idx[i] = (prev << K) | e
            e = prev
        out = {
            "indices": idx,
            "recon": self.lut[idx],
            "end_state": end_state,
            "path_cost": c2[end_state],
        }
        if L == 256:
            out["packed"] = swap16_storage(pack_trellis(idx, K))
        return out


# ---------------------------------------------------------------------------
# C restatement (oracle/trellis_oracle.c) through ctypes
# ---------------------------------------------------------------------------

_C_LOCK = threading.Lock()
_C_LIB = None


def _c_lib() -> ctypes.CDLL:
    global _C_LIB
    with _C_LOCK:
        if _C_LIB is None:
            so = ORACLE_DIR / "libtrellis_oracle.so"
            src = ORACLE_DIR / "trellis_oracle.c"
            if not so.exists() or so.stat().st_mtime < src.stat().st_mtime:
                subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
            lib = ctypes.CDLL(str(so))
            P = ctypes.c_void_p
            lib.ora_encode_batch.restype = ctypes.c_int
            lib.ora_encode_batch.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, P, P, P, P, P, ctypes.c_int]
            lib.ora_codebook.argtypes = [ctypes.c_int, P]
            lib.ora_forward.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int,
                                        ctypes.c_int, P, P]
            lib.ora_pack.argtypes = [P, ctypes.c_int, P]
            lib.ora_f32_to_h.restype = ctypes.c_uint16
            lib.ora_f32_to_h.argtypes = [ctypes.c_float]
            lib.ora_d_to_h.restype = ctypes.c_uint16
            lib.ora_d_to_h.argtypes = [ctypes.c_double]
            _C_LIB = lib
    return _C_LIB


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class COracle:
    """C restatement of the encoder, threads over tiles."""

    def __init__(self, K: int, cb: int = CB_MUL1, L: int = 256):
        self.K, self.cb, self.L = K, cb, L
        self.lib = _c_lib()

    def encode_batch(self, tiles: np.ndarray, threads: Optional[int] = None) -> dict:
        t = np.ascontiguousarray(np.asarray(tiles, dtype=np.float32).reshape(-1, self.L))
        n = t.shape[0]
        idx = np.zeros((n, self.L), dtype=np.uint16)
        recon = np.zeros((n, self.L), dtype=np.uint16)
        end_state = np.zeros(n, dtype=np.int32)
        cost = np.zeros(n, dtype=np.uint16)
        packed = np.zeros((n, 16 * self.K), dtype=np.uint16) if self.L == 256 else None
        if threads is None:
            threads = os.cpu_count() or 1
        used = self.lib.ora_encode_batch(_ptr(t), n, self.L, self.K, self.cb, _ptr(idx),
                                         _ptr(recon), _ptr(end_state), _ptr(cost),
                                         _ptr(packed) if packed is not None else None,
                                         int(threads))
        return {
            "indices": idx,
            "recon": recon.view(np.float16),
            "end_state": end_state,
            "path_cost": cost.view(np.float16),
            "packed": packed,
            "threads": used,
        }

    def codebook(self) -> np.ndarray:
        out = np.zeros(65536, dtype=np.uint16)
        self.lib.ora_codebook(self.cb, _ptr(out))
        return out.view(np.float16)

    def forward(self, w16: np.ndarray, roll: int, pre_state: int):
        """One forward pass; returns (edges (L, S) uint16, final costs (S,) fp16)."""
        w = np.ascontiguousarray(np.asarray(w16, dtype=np.float16).view(np.uint16))
        S = 65536 >> self.K
        lut = np.ascontiguousarray(codebook_lut(self.cb).view(np.uint16))
        edges = np.zeros((self.L, S), dtype=np.uint16)
        costs = np.zeros(S, dtype=np.uint16)
        self.lib.ora_forward(_ptr(w), self.L, self.K, _ptr(lut), roll, pre_state, _ptr(edges),
                             _ptr(costs))
        return edges, costs.view(np.float16)


def f32_to_f16_bits(x: float) -> int:
    return int(_c_lib().ora_f32_to_h(float(x)))


def f64_to_f16_bits(x: float) -> int:
    return int(_c_lib().ora_d_to_h(float(x)))
