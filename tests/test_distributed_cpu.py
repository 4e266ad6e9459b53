"""Multi-rank host logic on CPU: world size 2 over gloo (127.0.0.1).

Covers the sharding arithmetic, the token-sharded Hessian all-reduce
(identical to one rank holding every token), column-sharded LDLQ (identical
to the single-device loop with a device-agnostic tile encoder), module
assignment and the owner broadcast of module results.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from exl3_intel_arc_quantizer_b200 import distributed as xd
from exl3_intel_arc_quantizer_b200.ldlq import block_ldl, ldlq


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, ws, port, fn, q, received):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    try:
        dist.init_process_group("gloo", rank=rank, world_size=ws,
                                timeout=datetime.timedelta(seconds=60))
        q.put((rank, fn(rank, ws)))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, e))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
        # tensors cross the queue as shared-memory handles of this process:
        # stay alive until the parent has received them
        received.wait(timeout=120)


def _spawn_once(fn, ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    received = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, ws, port, fn, q, received)) for r in range(ws)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=120) for _ in range(ws))
    finally:
        received.set()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    return out


def spawn(fn, ws=2, attempts=2):
    """Run fn(rank, ws) on ws gloo ranks; a rendezvous failure (the free port
    taken by another process between probe and bind) is retried once on a
    new port."""
    for attempt in range(attempts):
        out = _spawn_once(fn, ws)
        errs = [v for v in out.values() if isinstance(v, Exception)]
        if errs and attempt + 1 < attempts and any(
                "address already in use" in str(e).lower() or "store" in str(e).lower()
                for e in errs):
            continue
        for v in errs:
            raise v
        return out


class GridEncoder:
    """Content-only states (a state never depends on where a tile sits in
    the batch), so sharded and unsharded runs are comparable."""

    def __call__(self, tiles):
        q = torch.round(tiles / 0.25)
        return q * 0.25, q.to(torch.int64) % 65536


def test_shard_range():
    for n, ws, al in ((65536, 8, 1), (1024, 3, 128), (256, 4, 128), (0, 2, 16)):
        parts = [xd.shard_range(n, ws, r, al) for r in range(ws)]
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
        assert all((e - s) % al == 0 for s, e in parts)
        sizes = [e - s for s, e in parts]
        assert max(sizes) - min(sizes) <= al
    with pytest.raises(ValueError):
        xd.shard_range(100, 2, 0, 16)
    with pytest.raises(ValueError):
        xd.shard_range(128, 2, 2)


def test_assign_modules_balances_tiles():
    shapes = {"q": (4096, 4096), "k": (4096, 1024), "v": (4096, 1024), "o": (4096, 4096),
              "gate": (4096, 12288), "up": (4096, 12288), "down": (12288, 4096)}
    own = xd.assign_modules(shapes, 4)
    assert own == xd.assign_modules(dict(reversed(list(shapes.items()))), 4)  # order-free
    load = [0] * 4
    for m, r in own.items():
        load[r] += shapes[m][0] * shapes[m][1]
    assert max(load) == 4096 * 12288
    assert set(xd.assign_modules(shapes, 1).values()) == {0}


def _hessian_body(rank, ws):
    g = torch.Generator().manual_seed(100 + rank)
    xs = {"a": torch.randn(50 + 10 * rank, 32, generator=g), "b": torch.randn(7 + rank, 16, generator=g)}
    H = {k: x.T @ x for k, x in xs.items()}
    counts = {k: x.shape[0] for k, x in xs.items()}
    tot = xd.all_reduce_hessians(H, counts)
    return H, tot, xs


def test_all_reduce_hessians_equals_single_rank_sum():
    out = spawn(_hessian_body)
    H0, tot0, xs0 = out[0]
    H1, tot1, xs1 = out[1]
    assert tot0 == tot1 == {"a": 50 + 60, "b": 7 + 8}
    for k in ("a", "b"):
        x = torch.cat([xs0[k], xs1[k]])
        assert torch.allclose(H0[k], x.T @ x, rtol=1e-5, atol=1e-4)
        assert torch.equal(H0[k], H1[k])


def _ldlq_body(rank, ws):
    torch.manual_seed(7)
    w = torch.randn(64, 384)
    a = torch.randn(64, 8)
    L = block_ldl(a @ a.T + 0.05 * torch.eye(64)).transformed
    return xd.ldlq_column_sharded(w, L, GridEncoder(), buf_size_k=32), w, L


def test_ldlq_column_sharded_equals_single_device():
    out = spawn(_ldlq_body)
    res, w, L = out[0]
    ref = ldlq(w, L, GridEncoder(), buf_size_k=32)
    assert torch.allclose(res.weight_q, ref.weight_q, atol=1e-5)
    assert torch.equal(res.encoded, ref.encoded)
    assert torch.equal(out[1][0].weight_q, res.weight_q)
    assert (res.tiles_k, res.tiles_n) == (4, 24)


def _layer_body(rank, ws):
    shapes = {"a": (128, 256), "b": (128, 128), "c": (256, 128)}
    g = torch.Generator().manual_seed(3)
    weights = {m: torch.randn(n, k, generator=g) for m, (k, n) in shapes.items()}
    hess = {m: torch.eye(k) for m, (k, n) in shapes.items()}
    calls = []

    class Res:
        pass

    def fake_quantize(name, W, H, K=2, **kw):
        calls.append(name)
        k = H.shape[0]
        r = Res()
        r.w_hat = W.T.contiguous() * 0.5
        r.encoded = torch.full((k // 16, W.shape[0] // 16, 256), len(name), dtype=torch.int16)
        r.su = torch.ones(k, 1) * 2
        r.sv = torch.ones(1, W.shape[0]) * 3
        r.cb = 2
        return r

    out = xd.quantize_layer_sharded(weights, hess, K=2, quantize_fn=fake_quantize)
    return {m: (r.owner, r.w_hat, r.encoded, float(r.su[0, 0]), float(r.sv[0, 0]), r.cb)
            for m, r in out.items()}, calls, weights


def test_quantize_layer_sharded_broadcasts_owner_results():
    out = spawn(_layer_body)
    (res0, calls0, weights), (res1, calls1, _) = out[0], out[1]
    assert sorted(calls0 + calls1) == ["a", "b", "c"] and not set(calls0) & set(calls1)
    for m in ("a", "b", "c"):
        owner, w_hat, enc, su, sv, cb = res0[m]
        assert res1[m][0] == owner and (m in (calls0, calls1)[owner])
        assert torch.equal(w_hat, weights[m].T * 0.5) and torch.equal(res1[m][1], w_hat)
        assert int(enc[0, 0, 0]) == 1 and torch.equal(res1[m][2], enc)
        assert (su, sv, cb) == (2.0, 3.0, 2) == res1[m][3:]
