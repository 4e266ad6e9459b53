"""Block-LDL preparation and the LDLQ error-feedback loop.

Same API and semantics as the reference ``exl3_quant/ldlq.py``
(upstream ``quantize.py:416-609``):

* :func:`block_ldl` — Cholesky of H with the audited retry schedule (first
  attempt undamped; on failure ``diag += 2 * sigma_reg * mean(diag)``, up to
  ``max_retries`` times), 16x16 diagonal-block inverses folded into their
  block columns, identity diagonal blocks. On CUDA the factorization is
  cuSOLVER (``torch.linalg.cholesky_ex``) and the fold one pass of the
  libexl3k kernel (``exl3_block_ldl_fold``: forward-substitution inverses of
  the 16x16 diagonal blocks and the block-column products); host tensors
  take the reference's op sequence (batched inverse, batched product).
* :func:`ldlq` — spans of ``buf_size_k`` rows bottom-up, 16-row blocks
  bottom-up inside a span; each block's target rows get the compensation
  ``L[i+bj:j, i+bi:i+bj]^T @ err_below`` added, are cut into 16x16 tiles in
  tensor-core order and encoded; after a span its residual is propagated
  through ``L[i:j]^T``. The op sequence is the reference's, so a run on CPU
  tensors reproduces the reference bit for bit given the same tile encoder.
* :func:`make_xpu_tile_encoder` — the B200 encoder as the loop's callback;
  on CUDA tensors it never leaves the device.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence, Tuple, List, Callable

import torch

from .trellis_format import tensor_core_perm, tensor_core_perm_inv

DEFAULT_BLOCK_SIZE = 16
DEFAULT_SIGMA_REG = 0.025
DEFAULT_MAX_RETRIES = 10
DEFAULT_BUF_SIZE_K = 128

TileEncoder = Callable[[torch.Tensor], "tuple[torch.Tensor, torch.Tensor]"]


@dataclass(frozen=True)
class BlockLDLResult:
    transformed: torch.Tensor
    cholesky: torch.Tensor
    block_inverses: torch.Tensor
    retries: int
    damping_applied: bool
    n: int
    block_size: int


def _validate_h(H: torch.Tensor, block_size: int) -> None:
    if H.dim() != 2 or H.shape[0] != H.shape[1]:
        raise ValueError(f"H must be a square 2-D tensor, got shape {tuple(H.shape)}")
    if H.dtype != torch.float32:
        raise ValueError(f"block_ldl requires float32 (the audited contract uses fp32); got {H.dtype}")
    if block_size <= 0:
        raise ValueError(f"block_size must be positive, got {block_size}")
    if block_size > H.shape[0]:
        raise ValueError(f"block_size {block_size} exceeds matrix size {H.shape[0]}")
    if H.shape[0] % block_size != 0:
        raise ValueError(f"matrix size {H.shape[0]} is not divisible by block_size {block_size}")


def block_ldl(H: torch.Tensor, block_size: int = DEFAULT_BLOCK_SIZE,
              sigma_reg: float = DEFAULT_SIGMA_REG,
              max_retries: int = DEFAULT_MAX_RETRIES) -> BlockLDLResult:
    _validate_h(H, block_size)
    if max_retries < 0:
        raise ValueError(f"max_retries must be non-negative, got {max_retries}")
    n = H.shape[0]
    work = H.clone()
    chol = None
    retries = 0
    for attempt in range(max_retries + 1):
        factor, info = torch.linalg.cholesky_ex(work)
        if int(info.item()) == 0:
            chol, retries = factor, attempt
            break
        if attempt == max_retries:
            raise torch.linalg.LinAlgError(
                f"cholesky failed after {max_retries} damping retries (info={int(info.item())})")
        work.diagonal().add_(2.0 * sigma_reg * work.diagonal().mean())
    m = n // block_size
    if H.is_cuda and block_size == 16:
        # the fold on the device (exl3_block_ldl_fold): one pass over the factor
        from ._ext import ext

        chol = chol.contiguous()
        transformed = torch.empty_like(chol)
        inverses = torch.empty((m, 16, 16), dtype=H.dtype, device=H.device)
        ext().block_ldl_fold(chol, transformed, inverses)
        return BlockLDLResult(transformed, chol, inverses, retries, retries > 0, n, block_size)
    cb = chol.reshape(m, block_size, m, block_size)
    diag_blocks = torch.diagonal(cb, dim1=0, dim2=2).permute(2, 0, 1).contiguous()
    inverses = torch.linalg.inv(diag_blocks)
    transformed = torch.einsum("rbi,bij->rbj", chol.reshape(n, m, block_size), inverses)
    transformed = transformed.reshape(n, n).contiguous()
    tb = transformed.reshape(m, block_size, m, block_size)
    eye = torch.eye(block_size, dtype=H.dtype, device=H.device)
    idx = torch.arange(m, device=H.device)
    tb[idx, :, idx, :] = eye
    return BlockLDLResult(transformed, chol, inverses, retries, retries > 0, n, block_size)


@dataclass
class LDLQResult:
    weight_q: torch.Tensor
    encoded: torch.Tensor
    tiles_k: int
    tiles_n: int
    buf_size_k: int


def _as_int16_states(indices: torch.Tensor) -> torch.Tensor:
    if indices.dtype == torch.int16:
        return indices
    v = indices.to(torch.int64) & 0xFFFF
    return torch.where(v >= 0x8000, v - 0x10000, v).to(torch.int16)


def _check_ldlq_args(weight: torch.Tensor, L: torch.Tensor, buf_size_k: int) -> int:
    if weight.dim() != 2:
        raise ValueError(f"weight must be 2-D, got shape {tuple(weight.shape)}")
    if weight.dtype != torch.float32:
        raise ValueError(f"weight must be float32, got {weight.dtype}")
    k, n = weight.shape
    if k % 16 != 0:
        raise ValueError(f"rows ({k}) must be a multiple of 16")
    if n % 128 != 0:
        raise ValueError(f"columns ({n}) must be a multiple of 128")
    if L.dim() != 2 or L.shape != (k, k):
        raise ValueError(f"L must have shape {(k, k)}, got {tuple(L.shape)}")
    if L.dtype != torch.float32:
        raise ValueError(f"L must be float32, got {L.dtype}")
    if L.device != weight.device:
        raise ValueError(f"L and weight must be on the same device, got {L.device} / {weight.device}")
    buf = int(buf_size_k)
    if buf < 16 or buf % 16 != 0:
        raise ValueError(f"buf_size_k must be a positive multiple of 16, got {buf_size_k}")
    if n % buf != 0:
        raise ValueError(f"columns ({n}) must be divisible by buf_size_k ({buf})")
    if k % buf != 0:
        raise ValueError(f"rows ({k}) must be divisible by buf_size_k ({buf}); "
                         "the bottom-up span walk assumes this")
    return buf


def _ldlq_steps(weight: torch.Tensor, L: torch.Tensor, buf: int):
    """The LDLQ loop (ldlq.py:163-309) as a generator: yields each 16-row
    block's tiles (tiles_n, 256) in encoder order and receives the encoder's
    ``(recon, states)`` for them; returns the ``LDLQResult``. The op order is
    the reference's: per span (bottom-up, ``buf`` rows) and 16-row block
    (bottom-up), ``rows = W + L_slab^T (W - W_q)_below + prod_cache``, encode,
    then the span's trailing ``prod_cache += L[span]^T (W - W_q)[span]``."""
    device = weight.device
    k, n = weight.shape
    tiles_k, tiles_n = k // 16, n // 16
    perm = torch.as_tensor(tensor_core_perm(), dtype=torch.long, device=device)
    inv_perm = torch.as_tensor(tensor_core_perm_inv(), dtype=torch.long, device=device)
    prod_cache = torch.zeros((k, n), dtype=torch.float32, device=device)
    weight_q = torch.zeros((k, n), dtype=torch.float32, device=device)
    encoded = torch.zeros((tiles_k, tiles_n, 256), dtype=torch.int16, device=device)

    for j in range(k, 0, -buf):
        i = j - buf
        b_weight, b_weight_q = weight[i:j], weight_q[i:j]
        b_encoded, b_prod, b_L = encoded[i // 16:j // 16], prod_cache[i:j], L[i:j]
        for bj in range(buf, 0, -16):
            bi = bj - 16
            err_below = b_weight[bj:] - b_weight_q[bj:]
            comp = b_prod[bi:bj]
            if err_below.shape[0] > 0:
                comp.addmm_(b_L[bj:, i + bi:i + bj].T, err_below, alpha=1.0, beta=1.0)
            rows = b_weight[bi:bj] + comp
            tiles = rows.reshape(16, tiles_n, 16).permute(1, 0, 2).reshape(tiles_n, 256)[:, perm]
            q_w, q_i = yield tiles
            if q_w.shape != (tiles_n, 256) or q_i.shape != (tiles_n, 256):
                raise ValueError("encode_tiles must return two (tiles_n, 256) tensors, got "
                                 f"{tuple(q_w.shape)} / {tuple(q_i.shape)}")
            q_w = q_w.to(device=device, dtype=torch.float32)[:, inv_perm]
            b_weight_q[bi:bj] = q_w.reshape(tiles_n, 16, 16).permute(1, 0, 2).reshape(16, n)
            b_encoded[bi // 16:bj // 16] = _as_int16_states(q_i.to(device=device)).unsqueeze(0)
        prod_cache.addmm_(b_L.T, b_weight - b_weight_q, alpha=1.0, beta=1.0)

    return LDLQResult(weight_q, encoded, tiles_k, tiles_n, buf)


def ldlq(weight: torch.Tensor, L: torch.Tensor, encode_tiles: TileEncoder,
         buf_size_k: int = DEFAULT_BUF_SIZE_K) -> LDLQResult:
    """LDLQ of one weight matrix (ldlq.py:163-309): one encoder call per
    16-row block."""
    return ldlq_batched([(weight, L)], encode_tiles, buf_size_k)[0]


def ldlq_batched(jobs: Sequence[Tuple[torch.Tensor, torch.Tensor]], encode_tiles: TileEncoder,
                 buf_size_k: int = DEFAULT_BUF_SIZE_K) -> List[LDLQResult]:
    """Several independent LDLQ loops advanced in lockstep: at every step the
    current 16-row blocks of all unfinished jobs go to the encoder as ONE
    batch. Each job's arithmetic is exactly its own ``ldlq`` (the encoder
    treats every tile independently), so the results equal separate runs;
    the GPU sees one large launch per step instead of one per module."""
    gens, cur, results = [], [], [None] * len(jobs)
    for weight, L in jobs:
        buf = _check_ldlq_args(weight, L, buf_size_k)
        gens.append(_ldlq_steps(weight, L, buf))
    for idx, g in enumerate(gens):
        cur.append(next(g))
    active = list(range(len(gens)))
    while active:
        batch = [cur[a] for a in active]
        sizes = [t.shape[0] for t in batch]
        tiles = batch[0] if len(batch) == 1 else torch.cat(batch, dim=0)
        q_w, q_i = encode_tiles(tiles)
        if q_w.shape != tiles.shape or q_i.shape != tiles.shape:
            raise ValueError("encode_tiles must return two (tiles_n, 256) tensors, got "
                             f"{tuple(q_w.shape)} / {tuple(q_i.shape)}")
        nxt = []
        off = 0
        for a, sz in zip(active, sizes):
            try:
                cur[a] = gens[a].send((q_w[off:off + sz], q_i[off:off + sz]))
                nxt.append(a)
            except StopIteration as stop:
                results[a] = stop.value
            off += sz
        active = nxt
    return results


def ldlq_native(jobs: Sequence[Tuple[torch.Tensor, torch.Tensor]], K: int, cb: int = 2,
                buf_size_k: int = DEFAULT_BUF_SIZE_K) -> List[LDLQResult]:
    """The LDLQ loop of every ``(weight, L)`` job on the GPU (``exl3_ldlq``):
    the same spans, blocks and feedback as :func:`ldlq` with the B200 encoder,
    without a host round trip per block; one encoder launch per step encodes
    the current block of every active job (the longest job runs throughout,
    the others start where :func:`ldlq_schedule` places them; results do not
    depend on the placement). The compensation and trailing products are the
    library's own fp32 kernels (fixed summation order), so results are close
    to, not bit-identical with, the cuBLAS products of :func:`ldlq`."""
    from ._ext import ext, require_cuda

    if not jobs:
        return []
    Ws, Ls, Wqs, encs = [], [], [], []
    for weight, L in jobs:
        buf = _check_ldlq_args(weight, L, buf_size_k)
        require_cuda(weight.device)
        k, n = weight.shape
        Ws.append(weight.contiguous())
        Ls.append(L.contiguous())
        Wqs.append(torch.empty_like(Ws[-1]))
        encs.append(torch.empty((k // 16, n // 16, 256), dtype=torch.int16, device=weight.device))
    ext().ldlq_(Ws, Ls, Wqs, encs, int(K), int(cb), int(buf))
    return [LDLQResult(wq, e, w.shape[0] // 16, w.shape[1] // 16, int(buf_size_k))
            for w, wq, e in zip(Ws, Wqs, encs)]


def ldlq_schedule(shapes: Sequence[Tuple[int, int]], K: int,
                  buf_size_k: int = DEFAULT_BUF_SIZE_K) -> List[int]:
    """First step of each ``(k, n)`` job in :func:`ldlq_native` on the current
    device (``exl3_ldlq_schedule``): longest first, then widest, each at the
    start that adds the least estimated encoder time."""
    import ctypes

    from ._ext import lib

    class _Job(ctypes.Structure):
        _fields_ = [("W", ctypes.c_void_p), ("L", ctypes.c_void_p), ("W_q", ctypes.c_void_p),
                    ("encoded", ctypes.c_void_p), ("k", ctypes.c_int64), ("n", ctypes.c_int64)]

    arr = (_Job * len(shapes))(*[_Job(None, None, None, None, int(k), int(n)) for k, n in shapes])
    out = (ctypes.c_int64 * len(shapes))()
    rc = lib().exl3_ldlq_schedule(arr, len(shapes), int(K), int(buf_size_k), out)
    if rc:
        raise ValueError(lib().exl3_last_error().decode())
    return [int(v) for v in out]


def make_xpu_tile_encoder(K: int = 2, device_index: int = 0, arena=None, sg_size: int = 32,
                          force_global_costs: bool = False,
                          traceback_mode: str = "gpu_resident") -> TileEncoder:
    """The B200 encoder as an LDLQ callback (ldlq.py:344-387).

    CUDA tiles stay on the device (no host round trip per 16-row block);
    tiles on another device are moved to ``cuda:device_index`` and the
    results moved back. The encoder and its arena are reused by every call.
    """
    from .xpu_quantizer import CB_MUL1, TRACEBACK_MODES, XPUTrellisEncoder

    if traceback_mode not in TRACEBACK_MODES:
        raise ValueError(f"Unknown traceback_mode {traceback_mode!r}")
    enc = XPUTrellisEncoder(K=K, cb=CB_MUL1, arena=arena, device_index=device_index,
                            sg_size=sg_size, force_global_costs=force_global_costs)

    def encode(tiles: torch.Tensor):
        src = tiles.device
        w, i, _, _ = enc.encode_device(tiles.detach(), want_packed=False)
        if src.type != "cuda" or src.index != device_index:
            return w.to(src), i.to(src)
        return w, i

    encode.K = K
    encode.cb = CB_MUL1
    encode.encoder = enc
    encode.native_ldlq = True   # quantize drivers may run the loop natively (ldlq_native)
    return encode


make_cuda_tile_encoder = make_xpu_tile_encoder
