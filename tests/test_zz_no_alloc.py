"""The encoder entry point that allocates no device memory.

exl3_quantize_tiles_noalloc serves callers that cannot allocate GPU memory
themselves (their HBM belongs to another runtime's pool, or they are plain C
hosts without a device allocator that must not call the synchronizing
cudaMalloc). Its scratch is a fixed array inside the library, shared by every
call. This checks, through the C ABI, that two calls in a row give exactly
what the workspace-taking entry point gives on the same inputs (so contents
left by the previous call do not leak into the next), and that a call larger
than the array is refused with a clear message.

The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from exl3_intel_arc_quantizer_b200 import _ext  # noqa: E402

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


def _bind():
    lib = _ext.lib()
    f = lib.exl3_quantize_tiles
    f.restype = ctypes.c_int
    f.argtypes = [P, P, P, P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                  ctypes.c_size_t, P]
    g = lib.exl3_quantize_tiles_noalloc
    g.restype = ctypes.c_int
    g.argtypes = [P, P, P, P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    lib.exl3_quantize_tiles_ws_bytes.restype = ctypes.c_size_t
    lib.exl3_quantize_tiles_ws_bytes.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    return lib, f, g


def _outputs(n, K, dev):
    return (torch.empty((n, 256), dtype=torch.float32, device=dev),
            torch.empty((n, 256), dtype=torch.int16, device=dev),
            torch.empty((n, 16 * K), dtype=torch.int16, device=dev),
            torch.empty((n,), dtype=torch.float32, device=dev))


def _ptr(t):
    return P(t.data_ptr())


def test_no_alloc_entry_point_matches_workspace_entry_point():
    lib, with_ws, no_alloc = _bind()
    dev = torch.device("cuda", 0)
    stream = P(torch.cuda.current_stream(dev).cuda_stream)
    K, cb = 2, 2
    for call, n in enumerate((16, 11)):           # two calls in a row, 2nd one odd
        g = torch.Generator().manual_seed(100 + call)
        x = (torch.randn((n, 256), generator=g)
             * torch.exp(0.5 * torch.randn((n, 1), generator=g))).to(dev)
        ws = torch.empty(lib.exl3_quantize_tiles_ws_bytes(n, K, 256), dtype=torch.uint8, device=dev)
        ref = _outputs(n, K, dev)
        got = _outputs(n, K, dev)
        assert with_ws(_ptr(x), *map(_ptr, ref), n, K, cb, 256, _ptr(ws), ws.numel(), stream) == 0
        torch.cuda.synchronize(dev)
        free_before = torch.cuda.mem_get_info(dev)[0]
        assert no_alloc(_ptr(x), *map(_ptr, got), n, K, cb, 256, stream) == 0, \
            lib.exl3_last_error()
        torch.cuda.synchronize(dev)
        if call == 1:
            # the first call committed the scratch array; later calls take no memory
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        for a, b in zip(ref, got):
            assert torch.equal(a, b)              # bit-exact, the encoder tests' tolerance


def test_no_alloc_entry_point_rejects_oversized_calls():
    lib, _, no_alloc = _bind()
    dev = torch.device("cuda", 0)
    stream = P(torch.cuda.current_stream(dev).cuda_stream)
    x = torch.zeros((1, 256), device=dev)
    rc = no_alloc(_ptr(x), _ptr(x), _ptr(x), None, None, 17, 2, 2, 256, stream)
    assert rc == -22
    msg = lib.exl3_last_error().decode()
    assert "at most 16 tiles per call at K=2" in msg, msg
