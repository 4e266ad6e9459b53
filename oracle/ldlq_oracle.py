"""LDLQ loop with a fixed summation order — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs use this module, as the checker;
the product never imports it.

It restates the reference loop (``exl3_quant/ldlq.py:163-309``; the same step
order as ``module_oracle.ldlq``) with the two products done by
``oracle/ldlq_oracle.c`` in one fixed order (each output a sequential fmaf
chain from 0 over ascending contracted rows, added once to the cached
product) instead of the host BLAS's. Any tile encoder can be plugged in:
the C restatement of the encoder (``module_oracle.c_encoder``) for a fully
CPU run, or the device encoder, whose bit-exactness against that
restatement is pinned separately, for full-size runs.
"""

from __future__ import annotations

import ctypes
import subprocess
import threading
from typing import Callable, Tuple

import numpy as np
import torch

from .trellis_oracle import ORACLE_DIR, tensor_core_perm_inv

_LIB = None
_LOCK = threading.Lock()


def _lib() -> ctypes.CDLL:
    global _LIB
    with _LOCK:
        if _LIB is None:
            path = ORACLE_DIR / "libldlq_oracle.so"
            src = ORACLE_DIR / "ldlq_oracle.c"
            if not path.exists() or path.stat().st_mtime < src.stat().st_mtime:
                subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), "libldlq_oracle.so"],
                               check=True)
            lib = ctypes.CDLL(str(path))
            P, I = ctypes.c_void_p, ctypes.c_int64
            lib.ldlq_oracle_prep.argtypes = [P, P, P, P, I, I, I, I, I, P, P]
            lib.ldlq_oracle_prep.restype = None
            lib.ldlq_oracle_span.argtypes = [P, P, P, P, I, I, I, I, I]
            lib.ldlq_oracle_span.restype = None
            _LIB = lib
        return _LIB


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def ldlq_fixed_order(weight: torch.Tensor, L: torch.Tensor, encode: Callable,
                     buf: int = 128) -> Tuple[torch.Tensor, torch.Tensor]:
    """(weight_q (k, n) f32, encoded (k/16, n/16, 256) int16) of the LDLQ loop
    over CPU fp32 ``weight`` (k, n) and ``L`` (k, k). ``encode`` maps (tn, 256)
    f32 tiles in encoder order to (reconstruction f32, states int16)."""
    lib = _lib()
    W = np.ascontiguousarray(weight.detach().cpu().numpy(), dtype=np.float32)
    Lm = np.ascontiguousarray(L.detach().cpu().numpy(), dtype=np.float32)
    k, n = W.shape
    tn = n // 16
    inv = np.ascontiguousarray(np.asarray(tensor_core_perm_inv(), dtype=np.int16))
    prod = np.zeros((k, n), dtype=np.float32)
    wq = np.zeros((k, n), dtype=np.float32)
    enc = np.zeros((k // 16, tn, 256), dtype=np.int16)
    tiles = np.empty((tn, 256), dtype=np.float32)
    inv_l = inv.astype(np.int64)
    for span0 in range(k - buf, -1, -buf):
        for bi in range(buf - 16, -1, -16):
            r0 = span0 + bi
            lib.ldlq_oracle_prep(_p(W), _p(wq), _p(Lm), _p(prod), k, n, r0, r0 + 16,
                                 span0 + buf, _p(inv), _p(tiles))
            qw, qi = encode(torch.from_numpy(tiles.copy()))
            qw = np.asarray(qw.cpu().numpy() if isinstance(qw, torch.Tensor) else qw,
                            dtype=np.float32)
            qi = np.asarray(qi.cpu().numpy() if isinstance(qi, torch.Tensor) else qi)
            # encoder order -> tile position (r, c): position p holds qw[:, inv[p]]
            blk = qw[:, inv_l].reshape(tn, 16, 16).transpose(1, 0, 2).reshape(16, n)
            wq[r0:r0 + 16] = blk
            enc[r0 // 16] = (qi.astype(np.int64) & 0xFFFF).astype(np.uint16).view(np.int16)
        if span0 > 0:
            lib.ldlq_oracle_span(_p(W), _p(wq), _p(Lm), _p(prod), k, n, span0, buf, span0)
    return torch.from_numpy(wq), torch.from_numpy(enc)
