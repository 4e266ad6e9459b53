"""Multi-GPU paths on B200s (2 ranks over NCCL, one process per GPU); skipped
with fewer than 2 GPUs.

* token-sharded Hessian: per-rank tcgen05 accumulation + NCCL all-reduce
  equals one GPU accumulating every token within the Hessian tolerance
  (max rel 1e-4: the tensor-core accumulation chains are split differently);
* column-sharded LDLQ with the B200 encoder: bit-identical to the
  single-GPU native loop (its fixed per-output summation order does not
  depend on the slice's width);
* module-sharded layer quantization: every rank ends with every module's
  result, bit-identical to what its owner computed;
* convert_layer with one calibration batch per rank (Hessian all-reduce,
  column-sharded quantization, local re-forward) equals one GPU converting
  both batches bit for bit: every module's w_hat and trellis states and the
  next hidden states;
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


def _step(rank, what):
    print(f"[rank {rank}] {what}", flush=True)


def _worker(rank, ws, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=ws, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        from exl3_intel_arc_quantizer_b200 import distributed as xd
        from exl3_intel_arc_quantizer_b200.calibration import hessian_accumulate_
        from exl3_intel_arc_quantizer_b200.ldlq import block_ldl, ldlq_native, make_xpu_tile_encoder
        from exl3_intel_arc_quantizer_b200.layer_quant import quantize_linear_module

        _step(rank, "1 token-sharded Hessian")
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

        _step(rank, "2 column-sharded LDLQ")
        # 2. column-sharded LDLQ with the B200 encoder
        gc = torch.Generator(device="cpu").manual_seed(9)
        W = torch.randn(256, 512, generator=gc).to(dev)
        A = torch.randn(256, 32, generator=gc).to(dev)
        L = block_ldl(A @ A.T / 32 + 0.1 * torch.eye(256, device=dev)).transformed
        enc = make_xpu_tile_encoder(K=2, device_index=rank)
        sh = xd.ldlq_column_sharded(W, L, enc, buf_size_k=128)
        ref = ldlq_native([(W, L)], K=2, buf_size_k=128)[0]
        out["ldlq_rel"] = float(torch.linalg.norm(sh.weight_q - ref.weight_q)
                                / torch.linalg.norm(ref.weight_q))
        out["ldlq_same"] = float((sh.encoded == ref.encoded).all(-1).float().mean())

        _step(rank, "3 module-sharded layer")
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

        _step(rank, "4 column-sharded batched modules")
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

        _step(rank, "5 the same modules on one GPU")
        # 5. the same modules on one GPU: sharded == unsharded, bit for bit
        one = quantize_modules(mods, K=2, tile_encoder=enc)
        out["qm_equal"] = {m: bool(torch.equal(qm[m].w_hat, one[m].w_hat)
                                   and torch.equal(qm[m].encoded, one[m].encoded)) for m in mods}

        _step(rank, "6 convert_layer")
        # 6. convert_layer: one calibration batch per rank (Hessian all-reduce
        #    of the two partial sums), column-sharded quantization, local
        #    re-forward; against one GPU converting both batches
        import copy

        from exl3_intel_arc_quantizer_b200.calibration import TransformerDecoderLayer
        from exl3_intel_arc_quantizer_b200.converter import convert_layer

        torch.manual_seed(0)
        layer = TransformerDecoderLayer(256, 512, 4, 2)
        for prm in layer.parameters():
            if prm.dim() == 2:
                torch.nn.init.normal_(prm, std=0.02)
        layer1 = copy.deepcopy(layer)
        gh = torch.Generator(device="cpu").manual_seed(4)
        hs = [torch.randn(2, 64, 256, generator=gh).half().to(dev) for _ in range(ws)]
        res, nxt, tm = convert_layer(layer, [hs[rank]], K=2, device=dev, group=dist.group.WORLD)
        full, nxt1, _ = convert_layer(layer1, hs, K=2, device=dev)
        out["cl_equal"] = {m: bool(torch.equal(res[m].w_hat, full[m].w_hat)
                                   and torch.equal(res[m].encoded, full[m].encoded)) for m in res}
        out["cl_next_equal"] = bool(torch.equal(nxt[0], nxt1[rank]))
        out["cl_metric"] = {m: (res[m].metrics.relative_frobenius_error,
                                full[m].metrics.relative_frobenius_error) for m in res}
        out["cl_tokens"] = tm.local_tokens
        torch.cuda.synchronize()
        _step(rank, "done")
    except Exception as e:  # pragma: no cover
        import traceback

        traceback.print_exc()
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
    import queue

    try:
        res = dict(q.get(timeout=240) for _ in range(2))
    except queue.Empty:
        for p in procs:
            p.terminate()
        raise AssertionError("a rank did not report within 240 s (see its progress lines)")
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    for r, v in res.items():
        if isinstance(v, Exception):
            raise v
    a, b = res[0], res[1]
    print(a, b)
    assert a["count"] == b["count"] == 8192
    assert a["hess_rel"] <= 1e-4 and b["hess_rel"] <= 1e-4
    assert a["ldlq_rel"] == 0.0 and b["ldlq_rel"] == 0.0
    assert a["ldlq_same"] == 1.0 and b["ldlq_same"] == 1.0
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
    for r in (a, b):
        assert all(r["qm_equal"].values()), r["qm_equal"]
        # convert_layer over 2 GPUs == one GPU: identical Hessians (each rank's
        # one batch is one exact partial sum; the all-reduce adds the two),
        # identical quantized modules, identical next hidden states
        assert r["cl_tokens"] == 128
        assert all(r["cl_equal"].values()), r["cl_equal"]
        assert r["cl_next_equal"]
        for m, (got, want) in r["cl_metric"].items():
            assert abs(got - want) <= 1e-4 * want, (m, got, want)
