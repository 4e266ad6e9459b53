"""Multi-GPU paths on B200s (2 ranks over NCCL, one process per GPU); skipped
with fewer than 2 GPUs.

* token-sharded Hessian: per-rank tcgen05 accumulation + NCCL all-reduce
  equals one GPU accumulating every token within the Hessian tolerance
  (max rel 1e-4: the tensor-core accumulation chains are split differently);
* column-sharded LDLQ with the B200 encoder: close to the single-GPU loop
  (rel Frobenius <= 1e-2; cuBLAS may round a narrower product differently,
  which can move a tile's path);
* module-sharded layer quantization: every rank ends with every module's
  result, bit-identical to what its owner computed;
* column-sharded batched modules: each module's metrics (and each distinct
  Hessian's factorization residual), summed over every rank's column slice
  and all-reduced, match what any rank recomputes whole from its gathered
  result (rtol 1e-4: fp64 partial sums against fp32 whole-matrix
  reductions; the residual, itself a rounding-error measure, within 2x).
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        from exl3_intel_arc_quantizer_b200 import distributed as xd
        from exl3_intel_arc_quantizer_b200.calibration import hessian_accumulate_
        from exl3_intel_arc_quantizer_b200.ldlq import block_ldl, ldlq, make_xpu_tile_encoder
        from exl3_intel_arc_quantizer_b200.layer_quant import quantize_linear_module

        # 1. token-sharded Hessian
        g = torch.Generator(device=dev).manual_seed(5)
        X = torch.randn(8192, 512, generator=g, device=dev, dtype=torch.bfloat16)
        t0, t1 = xd.shard_range(8192, ws, rank, 64)
        H = {"g": torch.zeros(512, 512, device=dev)}
        hessian_accumulate_(H["g"], X[t0:t1].contiguous())
        counts = xd.all_reduce_hessians(H, {"g": t1 - t0})
        Href = torch.zeros(512, 512, device=dev)
        hessian_accumulate_(Href, X)
        out["hess_rel"] = float((H["g"] - Href).abs().max() / Href.abs().max())
        out["count"] = counts["g"]

        # 2. column-sharded LDLQ with the B200 encoder
        gc = torch.Generator(device="cpu").manual_seed(9)
        W = torch.randn(256, 512, generator=gc).to(dev)
        A = torch.randn(256, 32, generator=gc).to(dev)
        L = block_ldl(A @ A.T / 32 + 0.1 * torch.eye(256, device=dev)).transformed
        enc = make_xpu_tile_encoder(K=2, device_index=rank)
        sh = xd.ldlq_column_sharded(W, L, enc, buf_size_k=128)
        ref = ldlq(W, L, enc, buf_size_k=128)
        out["ldlq_rel"] = float(torch.linalg.norm(sh.weight_q - ref.weight_q)
                                / torch.linalg.norm(ref.weight_q))
        out["ldlq_same"] = float((sh.encoded == ref.encoded).all(-1).float().mean())

        # 3. module-sharded layer
        weights = {"a": (torch.randn(256, 128, generator=gc) * 0.02).to(dev),
                   "b": (torch.randn(128, 256, generator=gc) * 0.02).to(dev)}
        hess = {}
        for m, w in weights.items():
            k = w.shape[1]
            x = torch.randn(1024, k, generator=gc).to(dev)
            hh = x.T @ x / 1024
            hh.diagonal().add_(0.01 * hh.diagonal().mean())
            hess[m] = hh
        res = xd.quantize_layer_sharded(weights, hess, K=2, tile_encoder=enc)
        own = {m: r.owner for m, r in res.items()}
        digest = {m: (float(r.w_hat.double().sum()), int(r.encoded.long().sum())) for m, r in res.items()}
        local = {}
        for m, r in res.items():
            if r.owner == rank:
                local[m] = float(torch.linalg.norm(r.result.w_hat - r.w_hat))
        out.update(owners=own, digest=digest, local=local)

        # 4. column-sharded batched modules: metrics summed over the ranks'
        #    column slices equal the ones every rank can recompute whole
        from exl3_intel_arc_quantizer_b200.layer_quant import (
            _ldl_of, _module_metrics, quantize_modules)

        mods = {"q": (weights["a"], hess["b"]), "k": (weights["a"] * 0.5, hess["b"]),
                "o": (weights["b"], hess["a"])}
        qm = quantize_modules(mods, K=2, tile_encoder=enc, group=dist.group.WORLD)
        met, again = {}, {}
        for m, r in qm.items():
            mt = r.metrics
            met[m] = (mt.mse, mt.relative_frobenius_error, mt.tile_distortion, mt.proxy_loss,
                      mt.normalized_proxy_loss, mt.factorization_residual)
            W = r.weight_orig
            reg = r.regularize_result
            redo = list(_module_metrics(W, mods[m][1].float(), reg, reg.weight, r.w_hat))
            redo[2] = mt.tile_distortion   # needs weight_q, which results do not keep
            again[m] = tuple(redo) + (_ldl_of(mods[m][1].float(), 16)[1],)
        out.update(mod_metrics=met, mod_again=again)
        torch.cuda.synchronize()
    except Exception as e:  # pragma: no cover
        out = e
    finally:
        dist.destroy_process_group()
    q.put((rank, out))


def test_two_gpu_sharded_paths():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r, v in res.items():
        if isinstance(v, Exception):
            raise v
    a, b = res[0], res[1]
    print(a, b)
    assert a["count"] == b["count"] == 8192
    assert a["hess_rel"] <= 1e-4 and b["hess_rel"] <= 1e-4
    assert a["ldlq_rel"] <= 1e-2 and b["ldlq_rel"] == a["ldlq_rel"]
    assert a["owners"] == b["owners"] and set(a["owners"].values()) == {0, 1}
    assert a["digest"] == b["digest"]
    assert all(v == 0.0 for v in list(a["local"].values()) + list(b["local"].values()))
    assert a["mod_metrics"] == b["mod_metrics"]
    for r in (a, b):
        for m, vals in r["mod_metrics"].items():
            again = r["mod_again"][m]
            for got, want in zip(vals[:5], again[:5]):
                assert abs(got - want) <= 1e-4 * max(abs(want), 1e-12), (m, vals, again)
            # the factorization residual measures fp32 rounding of L L^T itself,
            # so a column-sliced product only has to agree in size
            assert vals[5] <= 1e-5 and again[5] <= 1e-5 and 0.5 <= vals[5] / again[5] <= 2.0
