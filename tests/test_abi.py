"""The C-ABI library loads, exports every symbol its headers declare, and its
host-side argument checks return the documented status codes (no GPU work is
issued: validation happens before any CUDA call)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from exl3_intel_arc_quantizer_b200 import _build, _ext

REPO = Path(__file__).resolve().parent.parent
EINVAL, ENOMEM = -22, -12


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(exl3_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_builds_and_exports_every_declared_symbol():
    lib = _ext.lib()
    syms = declared_symbols()
    assert "exl3_quantize_tiles" in syms and "exl3_last_error" in syms
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"


def test_library_is_sm100a_only_build():
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.NVCC_FLAGS)
    assert _ext.lib().exl3_version().decode().endswith("(sm_100a)")


def test_workspace_size_formula():
    from exl3_intel_arc_quantizer_b200.scratch_estimator import b200_workspace_bytes

    lib = _ext.lib()
    for K in range(1, 9):
        for L in (256, 160):
            assert lib.exl3_quantize_tiles_ws_bytes(7, K, L) == b200_workspace_bytes(K, L, 7)
    # K=2: 127 pass-2 cost checkpoints of 16,384 {cost_A, cost_B} words per
    # tile pair, half per tile; tiles are encoded in pairs
    assert lib.exl3_quantize_tiles_ws_bytes(2, 2, 256) == 2 * (127 * 16384 * 4 // 2 + 8)
    assert lib.exl3_quantize_tiles_ws_bytes(1, 2, 256) == lib.exl3_quantize_tiles_ws_bytes(2, 2, 256)
    assert lib.exl3_quantize_tiles_ws_bytes(1, 9, 256) == 0
    assert lib.exl3_quantize_tiles_ws_bytes(1, 2, 128) == 0


def test_argument_errors_return_status_and_message():
    lib = _ext.lib()
    f = lib.exl3_quantize_tiles
    f.restype = ctypes.c_int
    P = ctypes.c_void_p
    f.argtypes = [P, P, P, P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                  ctypes.c_size_t, P]
    dummy = P(16)
    assert f(dummy, dummy, dummy, None, None, 4, 9, 2, 256, dummy, 1 << 20, None) == EINVAL
    assert b"K must be in 1..8" in lib.exl3_last_error()
    assert f(dummy, dummy, dummy, None, None, 4, 2, 1, 160, dummy, 1 << 20, None) == EINVAL
    assert b"L=160" in lib.exl3_last_error()
    assert f(dummy, dummy, dummy, None, None, 0, 2, 2, 256, dummy, 1 << 20, None) == EINVAL
    assert f(dummy, dummy, dummy, None, None, 4, 2, 2, 256, None, 1 << 20, None) == EINVAL
    assert f(dummy, dummy, dummy, dummy, None, 4, 2, 2, 160, dummy, 1 << 20, None) == EINVAL
    g = lib.exl3_decode_codebook
    g.restype = ctypes.c_int
    g.argtypes = [ctypes.c_int, P, P]
    assert g(3, dummy, None) == EINVAL
    assert lib.exl3_hessian_set_tile(3) == EINVAL
    assert b"tile mode" in lib.exl3_last_error()
    assert lib.exl3_hessian_set_tile(0) == 0


def test_torch_binding_loads_and_validates_on_cpu_tensors():
    import torch

    e = _ext.ext()
    for name in ("quantize_tiles", "quantize_tiles_forward_pass", "quantize_tiles_backward_pass",
                 "decode_codebook", "encode_tiles", "pack_trellis"):
        assert hasattr(e, name)
    x = torch.zeros((1, 256))
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        e.quantize_tiles(x, x, torch.zeros((1, 256), dtype=torch.int16),
                         torch.zeros((1, 2, 16384), dtype=torch.float16),
                         torch.zeros((1, 256, 16384), dtype=torch.int16), 2, False, True)
    with pytest.raises(RuntimeError, match="ambiguous codebook"):
        e.quantize_tiles(x, x, torch.zeros((1, 256), dtype=torch.int16),
                         torch.zeros((1, 2, 16384), dtype=torch.float16),
                         torch.zeros((1, 256, 16384), dtype=torch.int16), 2, True, True)


def test_product_has_no_cpu_encoder_path():
    """Without a CUDA device the encoder raises instead of computing on the host."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    import numpy as np

    from exl3_intel_arc_quantizer_b200.xpu_quantizer import XPUTrellisEncoder

    with pytest.raises(RuntimeError, match="no CUDA device"):
        XPUTrellisEncoder(K=2).encode_tile(np.zeros(256, np.float32))


class _LdlqJob(ctypes.Structure):
    _fields_ = [("W", ctypes.c_void_p), ("L", ctypes.c_void_p), ("W_q", ctypes.c_void_p),
                ("encoded", ctypes.c_void_p), ("k", ctypes.c_int64), ("n", ctypes.c_int64)]


def test_float_and_storage_entry_points_validate_arguments():
    """Argument checks of the LDLQ, storage, Hadamard and Hessian entry
    points: status codes and messages, no device work (no GPU needed)."""
    lib = _ext.lib()
    P = ctypes.c_void_p
    d = P(256)
    lib.exl3_ldlq_ws_bytes.restype = ctypes.c_size_t
    lib.exl3_ldlq_ws_bytes.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    lib.exl3_ldlq.restype = ctypes.c_int
    lib.exl3_ldlq.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                              ctypes.c_size_t, P]
    good = (_LdlqJob * 1)(_LdlqJob(256, 256, 256, 256, 256, 512))
    assert lib.exl3_ldlq_ws_bytes(good, 1, 2, 128) > 256 * 512 * 4
    for job, msg in (((256, 256, 256, 256, 200, 512), b"multiple of buf"),
                     ((256, 256, 256, 256, 256, 100), b"multiple of 128"),
                     ((None, 256, 256, 256, 256, 512), b"NULL pointer")):
        bad = (_LdlqJob * 1)(_LdlqJob(*job))
        assert lib.exl3_ldlq(bad, 1, 2, 2, 128, d, 1 << 30, None) == EINVAL
        assert msg in lib.exl3_last_error(), lib.exl3_last_error()
        assert lib.exl3_ldlq_ws_bytes(bad, 1, 2, 128) == 0
    assert lib.exl3_ldlq(good, 1, 2, 2, 24, d, 1 << 30, None) == EINVAL
    assert lib.exl3_ldlq(good, 0, 2, 2, 128, d, 1 << 30, None) == EINVAL
    assert lib.exl3_ldlq(good, 1, 9, 2, 128, d, 1 << 30, None) == EINVAL
    assert lib.exl3_ldlq(good, 1, 2, 2, 128, d, 16, None) == EINVAL
    assert b"smaller than" in lib.exl3_last_error()

    f = lib.exl3_decode_weight
    f.restype = ctypes.c_int
    f.argtypes = [P, P, P, ctypes.c_int, P, P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                  ctypes.c_int, P]
    assert f(d, d, d, 0, d, None, 4, 8, 2, 2, None) == EINVAL          # k = 64 not a 128-multiple
    assert b"multiples of 128" in lib.exl3_last_error()
    assert f(d, d, d, 2, d, None, 8, 8, 2, 2, None) == EINVAL          # scale dtype
    assert f(d, d, d, 0, d, None, 8, 8, 9, 2, None) == EINVAL          # K
    assert f(d, d, d, 0, d, None, 8, 8, 2, 3, None) == EINVAL          # codebook
    g = lib.exl3_unpack_trellis
    g.restype = ctypes.c_int
    g.argtypes = [P, P, ctypes.c_int64, ctypes.c_int, P]
    assert g(d, d, 4, 0, None) == EINVAL
    assert g(d, d, 0, 2, None) == 0                                     # empty is a no-op
    h = lib.exl3_hessian_accumulate
    h.restype = ctypes.c_int
    h.argtypes = [P, P, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, P, P]
    assert h(d, d, 1, 16, 100, d, None) == EINVAL                       # d % 8
    assert h(d, d, 2, 16, 128, d, None) == EINVAL                       # dtype
    assert h(d, P(8), 1, 16, 128, d, None) == EINVAL                    # X alignment
    assert h(d, d, 1, 0, 128, d, None) == 0                             # no tokens: no-op
    r = lib.exl3_had128_right
    r.restype = ctypes.c_int
    r.argtypes = [P, ctypes.c_int64, ctypes.c_int64, P]
    assert r(d, 4, 100, None) == EINVAL
