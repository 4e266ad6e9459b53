#!/usr/bin/env python3
"""Generate golden vectors from the reference implementation.

Run once in a container that holds the reference checkout
(alpha2beta/EXL3_Intel_Arc_quantizer); the outputs are committed next to this
script and the tests read only those files:

    python tests/golden/make_golden.py --reference /path/to/EXL3_Intel_Arc_quantizer

Every vector comes from the reference's own CPU code path:
  * encoder  — exl3_quant.reference_encoder.ReferenceTrellisEncoder.encode_tile
  * forward  — ReferenceTrellisEncoder.forward (edges hashed, final costs kept)
  * format   — exl3_quant.trellis_format (codebook_lut, pack_trellis, swap16)
  * ldlq     — exl3_quant.ldlq.block_ldl / ldlq with make_reference_tile_encoder
  * float    — hadamard / regularize / calibration.HessianCollector
  * storage  — exl3_quant.serialization (pack/unpack_module_trellis,
               build_layer_tensors, decode_weight_from_storage)
  * gss      — exl3_quant.gss (sample_scale_tiles, g_scale_search_batch with
               the reference encoder)

Inputs are seeded synthetic data with the shapes and distributions of the
reference's tests and of the benchmark configurations.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import multiprocessing as mp
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = None  # set in main()


def _ref_encoder(K, cb, L=256):
    from exl3_quant.reference_encoder import ReferenceTrellisEncoder
    return ReferenceTrellisEncoder(K=K, cb=cb, tile_len=L)


def _encode_job(args):
    sys.path.insert(0, REF)
    K, cb, L, tile, pre_permute = args
    r = _ref_encoder(K, cb, L).encode_tile(tile, pre_permute=pre_permute)
    return (r.output_indices.astype(np.uint16), r.reconstructed_perm.view(np.uint16).copy(),
            r.reconstructed.view(np.uint16).copy(),
            (r.packed.astype(np.uint16) if r.packed.size else np.zeros(0, np.uint16)),
            int(r.end_state), np.float16(r.path_cost).view(np.uint16).item(), float(r.distortion))


def encode_cases():
    """(name, K, cb, L, tiles (n, L) f32, pre_permute)"""
    CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2
    cases = []
    # 256 tiles N(0,1) fp16, seed 0, K=2, mul1, encoder order
    t = np.random.default_rng(0).standard_normal((256, 256), dtype=np.float32).astype(np.float16)
    cases.append(("cfg1_k2_mul1", 2, CB_MUL1, 256, t.astype(np.float32), False))
    # reference device-parity recipe (test_xpu_quantizer.py:88-115): seed 2026, N(0, 1.15)
    tile = np.random.default_rng(2026).normal(0.0, 1.15, size=256).astype(np.float32)
    for K in (1, 2, 3, 4):
        for cb in ((CB_MUL1,) if K == 1 else (CB_3INST, CB_MCG, CB_MUL1)):
            cases.append((f"parity_k{K}_cb{cb}", K, cb, 256, tile[None, :].copy(), True))
    # BASELINE config 2 distribution: N(0,1) x per-(tile,row) LogNormal(0, 0.5) scale
    for K in (1, 2, 3, 4, 5, 6, 7, 8):
        rng = np.random.default_rng(100 + K)
        n = 6 if K <= 6 else 3
        base = rng.standard_normal((n, 16, 16), dtype=np.float32)
        scale = np.exp(0.5 * rng.standard_normal((n, 16, 1))).astype(np.float32)
        cases.append((f"cfg2_k{K}_mul1", K, CB_MUL1, 256,
                      (base * scale).reshape(n, 256).astype(np.float16).astype(np.float32), False))
    for K in (5, 6, 8):
        for cb in (CB_3INST, CB_MCG):
            rng = np.random.default_rng(300 + 10 * K + cb)
            cases.append((f"cb{cb}_k{K}", K, cb, 256,
                          rng.normal(0, 1.24371088, size=(2, 256)).astype(np.float32), False))
    # edge cases (test_xpu_quantizer.py:160-205), pre-permuted like the reference test
    rng = np.random.default_rng(77)
    edge = np.stack([
        np.zeros(256, dtype=np.float32),
        np.full(256, 0.5, dtype=np.float32),
        np.where(np.arange(256) % 17 == 0, 25.0, rng.normal(0.0, 0.5, size=256)).astype(np.float32),
        np.tile(np.array([-1.5, 1.5], dtype=np.float32), 128),
    ])
    for K in (2, 4):
        cases.append((f"edge_k{K}", K, CB_MUL1, 256, edge.copy(), True))
    # fp16 saturation: path costs overflow to +inf and tie
    rng = np.random.default_rng(5)
    sat = (rng.standard_normal((3, 256)) * np.array([[40.0], [120.0], [400.0]])).astype(np.float32)
    for K in (2, 3):
        cases.append((f"saturate_k{K}", K, CB_MUL1, 256, sat.copy(), False))
    # tiny magnitudes (fp16 subnormal differences)
    tiny = (np.random.default_rng(6).standard_normal((2, 256)) * 1e-5).astype(np.float32)
    cases.append(("tiny_k2", 2, CB_MUL1, 256, tiny, False))
    # non-finite inputs
    nf = np.random.default_rng(7).standard_normal((5, 256)).astype(np.float32)
    nf[0, 17] = np.nan
    nf[1, :] = np.inf
    nf[2, 3] = -np.inf
    nf[2, 200] = np.inf
    nf[3, 0] = np.nan           # NaN at ring index 0 (pass 2 step 0, masked step)
    nf[4, 128] = np.nan         # NaN at pass 1 step 0
    for K in (2, 4, 7):
        cases.append((f"nonfinite_k{K}", K, CB_MUL1, 256, nf.copy(), False))
    # L = 160 rows, mul1 only (test_xpu_quantizer.py:117-131)
    t160 = np.random.default_rng(160).normal(0.0, 1.0, size=(2, 160)).astype(np.float32)
    cases.append(("l160_k3", 3, CB_MUL1, 160, t160, False))
    cases.append(("l160_k2", 2, CB_MUL1, 160, t160.copy(), False))
    # upstream test recipe (torch.manual_seed(0) randn * scale, encoder order)
    import torch
    for cb, scale in ((0, 1.24371088), (1, 1.24371088), (2, 1.0)):
        torch.manual_seed(0)
        tt = (torch.randn((1, 256)) * scale).numpy().astype(np.float32)
        for K in (2, 3, 4):
            cases.append((f"upstream_k{K}_cb{cb}", K, cb, 256, tt.copy(), False))
    return cases


def gen_encoder(pool, out):
    cases = encode_cases()
    jobs, spans = [], []
    for name, K, cb, L, tiles, pre in cases:
        start = len(jobs)
        for t in tiles:
            jobs.append((K, cb, L, t, pre))
        spans.append((name, K, cb, L, tiles, pre, start, len(jobs)))
    t0 = time.time()
    res = pool.map(_encode_job, jobs, chunksize=1)
    print(f"encoded {len(jobs)} tiles in {time.time() - t0:.1f}s", flush=True)
    arrays, meta = {}, []
    for name, K, cb, L, tiles, pre, a, b in spans:
        r = res[a:b]
        arrays[f"{name}/tiles"] = tiles.astype(np.float32)
        arrays[f"{name}/indices"] = np.stack([x[0] for x in r])
        arrays[f"{name}/recon_perm"] = np.stack([x[1] for x in r])
        arrays[f"{name}/recon"] = np.stack([x[2] for x in r])
        if L == 256:
            arrays[f"{name}/packed"] = np.stack([x[3] for x in r])
        arrays[f"{name}/end_state"] = np.array([x[4] for x in r], dtype=np.int32)
        arrays[f"{name}/path_cost"] = np.array([x[5] for x in r], dtype=np.uint16)
        arrays[f"{name}/distortion"] = np.array([x[6] for x in r], dtype=np.float64)
        meta.append({"name": name, "K": K, "cb": cb, "L": L, "n": int(b - a),
                     "pre_permute": bool(pre)})
    np.savez_compressed(out / "encoder_golden.npz", **arrays)
    return meta


def _forward_job(args):
    sys.path.insert(0, REF)
    K, roll, pre_state, tile = args
    enc = _ref_encoder(K, 2)
    edges = np.zeros((enc.L, enc.edges), dtype=np.uint16)
    costs = enc.forward(tile, roll=roll, pre_state=pre_state, temp_edges=edges)
    return hashlib.sha256(edges.tobytes()).hexdigest(), costs.view(np.uint16).copy(), edges[:4].copy()


def gen_forward(pool, out):
    """Forward-pass audits (test_forward_semantics.py:95-176)."""
    cases = []
    for K in (2, 3, 4):
        cases.append((f"unconstrained_k{K}", K, 0, -1,
                      np.random.default_rng(11 + K).normal(scale=0.5, size=256).astype(np.float16)))
    for K in (3, 4):
        enc_edges = 65536 >> K
        pre = int(np.random.default_rng(5).integers(0, enc_edges))
        cases.append((f"constrained_k{K}", K, 0, pre,
                      np.random.default_rng(21 + K).normal(scale=0.5, size=256).astype(np.float16)))
    cases.append(("rolled_k4", 4, 128, -1,
                  np.random.default_rng(31).normal(scale=0.5, size=256).astype(np.float16)))
    cases.append(("inf_k2", 2, 0, -1, np.full(256, np.inf, dtype=np.float16)))
    res = pool.map(_forward_job, [(K, roll, pre, t) for _, K, roll, pre, t in cases])
    arrays, meta = {}, []
    for (name, K, roll, pre, t), (h, costs, head) in zip(cases, res):
        arrays[f"{name}/w16"] = t.view(np.uint16).copy()
        arrays[f"{name}/costs"] = costs
        arrays[f"{name}/edges_head"] = head
        meta.append({"name": name, "K": K, "roll": roll, "pre_state": pre, "edges_sha256": h})
    np.savez_compressed(out / "forward_golden.npz", **arrays)
    return meta


def gen_format(out):
    sys.path.insert(0, REF)
    from exl3_quant import trellis_format as tf
    arrays, meta = {}, {}
    for cb in (0, 1, 2):
        lut = tf.codebook_lut(cb).view(np.uint16)
        meta[f"lut{cb}_sha256"] = hashlib.sha256(lut.tobytes()).hexdigest()
        arrays[f"lut{cb}_head"] = lut[:4096].copy()
    arrays["perm"] = tf.tensor_core_perm()
    for K in range(1, 9):
        st = np.random.default_rng(900 + K).integers(0, 65536, size=256).astype(np.uint16)
        arrays[f"pack_k{K}/states"] = st
        arrays[f"pack_k{K}/packed"] = tf.pack_trellis(st, K)
        arrays[f"pack_k{K}/stored"] = tf.swap16_storage(tf.pack_trellis(st, K))
        arrays[f"pack_k{K}/decoded"] = tf.decode_states(tf.swap16_storage(tf.pack_trellis(st, K)), K)
    np.savez_compressed(out / "format_golden.npz", **arrays)
    return meta


def gen_float(out):
    """Floating-point stages on small shapes (reference CPU torch fp32)."""
    sys.path.insert(0, REF)
    import torch
    from exl3_quant import hadamard as hd
    from exl3_quant import regularize as rg
    from exl3_quant import ldlq as lq
    from exl3_quant import calibration as cal

    arrays = {}
    g = torch.Generator().manual_seed(11)
    x = torch.randn(128, 256, generator=g)
    arrays["had/x"] = x.numpy()
    arrays["had/l"] = hd.preapply_had_l(x, 128).numpy()
    arrays["had/r"] = hd.preapply_had_r(x, 128).numpy()
    # regularize (test_regularize.py recipe)
    w = torch.randn(128, 256, generator=torch.Generator().manual_seed(11))
    su = torch.randn(128, generator=torch.Generator().manual_seed(5)).sign().reshape(128, 1)
    sv = torch.randn(256, generator=torch.Generator().manual_seed(9)).sign().reshape(1, 256)
    hdiag = torch.rand(128, generator=torch.Generator().manual_seed(4)) + 0.5
    reg = rg.regularize(w, su, sv, H_diag=hdiag, skip_g_scale=True)
    arrays["reg/w"], arrays["reg/su_in"], arrays["reg/sv_in"] = w.numpy(), su.numpy(), sv.numpy()
    arrays["reg/hdiag"] = hdiag.numpy()
    arrays["reg/weight"], arrays["reg/su"], arrays["reg/sv"] = reg.weight.numpy(), reg.su.numpy(), reg.sv.numpy()
    arrays["reg/flags"] = np.array([reg.apply_out_scales, reg.zeros], dtype=np.int8)
    # block_ldl
    A = torch.randn(128, 128, generator=torch.Generator().manual_seed(7))
    H = (A @ A.T / 128 + torch.eye(128)).float()
    b = lq.block_ldl(H, block_size=16)
    arrays["ldl/H"], arrays["ldl/L"] = H.numpy(), b.transformed.numpy()
    arrays["ldl/chol"] = b.cholesky.numpy()
    # Hessian accumulation + finalize (calibration.py:337-407) on raw activations
    X1 = torch.randn(3, 40, 128, generator=torch.Generator().manual_seed(21)).to(torch.float16)
    X2 = torch.randn(2, 24, 128, generator=torch.Generator().manual_seed(22)).to(torch.float16)
    X2[..., 5] = 0
    layer = torch.nn.Linear(128, 64, bias=False)
    hc = cal.HessianCollector.__new__(cal.HessianCollector)
    hc.device, hc.dtype = torch.device("cpu"), torch.float32
    hc.hessians, hc.token_counts = {}, {}
    hc.groups = {"g": ["g"]}
    hc._accumulate("g", X1)
    hc._accumulate("g", X2)
    arrays["hess/x1"], arrays["hess/x2"] = X1.numpy(), X2.numpy()
    arrays["hess/raw"] = hc.hessians["g"].numpy().copy()
    hf, damp = hc.finalize(damping_lambda=0.01, zero_floor=1e-7)
    arrays["hess/final"] = hf["g"].numpy()
    arrays["hess/damp"] = np.array([damp["g"]])
    np.savez_compressed(out / "float_golden.npz", **arrays)


def _ldlq_job(args):
    sys.path.insert(0, REF)
    import torch
    from exl3_quant import ldlq as lq
    K, k, n, buf, seed = args
    gen = torch.Generator().manual_seed(seed)
    weight = torch.randn(k, n, generator=gen) * 0.5
    a = torch.randn(k, 8, generator=gen)
    H = a @ a.T + 0.05 * torch.eye(k)
    L = lq.block_ldl(H).transformed
    res = lq.ldlq(weight, L, lq.make_reference_tile_encoder(K=K), buf_size_k=buf)
    return weight.numpy(), L.numpy(), res.weight_q.numpy(), res.encoded.numpy()


def gen_ldlq(pool, out):
    cases = [("k2_32x128", 2, 32, 128, 32, 17), ("k4_64x128", 4, 64, 128, 32, 23)]
    res = pool.map(_ldlq_job, [c[1:] for c in cases], chunksize=1)
    arrays = {}
    for (name, K, k, n, buf, seed), (w, L, wq, enc) in zip(cases, res):
        arrays[f"{name}/weight"], arrays[f"{name}/L"] = w, L
        arrays[f"{name}/weight_q"], arrays[f"{name}/encoded"] = wq, enc
        arrays[f"{name}/params"] = np.array([K, k, n, buf, seed])
    np.savez_compressed(out / "ldlq_golden.npz", **arrays)
    return [{"name": c[0], "K": c[1], "k": c[2], "n": c[3], "buf": c[4], "seed": c[5]} for c in cases]


def gen_module(out):
    """quantize_linear_module end to end (reference CPU path, reference encoder)."""
    sys.path.insert(0, REF)
    import torch
    from exl3_quant import layer_quant as lqm
    g = torch.Generator().manual_seed(31)
    k, n = 128, 256
    W = (torch.randn(n, k, generator=g) * 0.02)
    W[:, torch.randperm(k, generator=g)[:2]] *= 8.0
    X = torch.randn(512, k, generator=g)
    X[:, torch.randperm(k, generator=g)[:3]] *= 20.0
    H = (X.T @ X) / 512
    H.diagonal().add_(0.01 * H.diagonal().mean())
    res = lqm.quantize_linear_module("mod", W, H, K=2, skip_g_scale=True, buf_size_k=64)
    m = res.metrics
    np.savez_compressed(out / "module_golden.npz", W=W.numpy(), H=H.numpy(), w_hat=res.w_hat.numpy(),
                        encoded=res.encoded.numpy(), su=res.su.numpy(), sv=res.sv.numpy(),
                        reg_weight=res.regularize_result.weight.numpy(),
                        L=res.ldl_result.transformed.numpy(),
                        metrics=np.array([m.mse, m.relative_frobenius_error, m.tile_distortion,
                                          m.proxy_loss, m.normalized_proxy_loss]))
    return {"k": k, "n": n, "K": 2, "buf": 64, "seed": 31}


def gen_gss(pool, out):
    """gss.py: tile sampling and the two-stage global-scale search with the
    reference encoder (encode calls mapped over the process pool)."""
    sys.path.insert(0, REF)
    import torch
    from exl3_quant import gss

    class PoolEncoder:
        K = 2

        def __call__(self, tiles):
            arr = np.ascontiguousarray(tiles.detach().cpu().numpy(), dtype=np.float32)
            res = pool.map(_encode_job, [(2, 2, 256, t, False) for t in arr], chunksize=4)
            rec = np.stack([r[2] for r in res]).view(np.float16).astype(np.float32)
            idx = np.stack([r[0] for r in res]).view(np.int16)
            return torch.from_numpy(rec), torch.from_numpy(idx)

    g = torch.Generator().manual_seed(41)
    w = torch.randn(128, 256, generator=g) * 0.9
    w[:, 5] *= 4.0
    samples = gss.sample_scale_tiles(w, 3)
    scale, mse = gss.g_scale_search_batch([samples], PoolEncoder())[0]
    np.savez_compressed(out / "gss_golden.npz", weight_r=w.numpy(), samples=samples.numpy(),
                        result=np.array([scale, mse], dtype=np.float64))
    return {"shape": [128, 256], "K": 2, "tiles": int(samples.shape[0]),
            "scale": scale, "mse": mse}


def gen_storage(out):
    """serialization.py: module packing, unpacking and weight decode.

    * module: the module golden's encoded states and scales through
      pack_module_trellis, build_layer_tensors (keys/shapes/dtypes) and
      decode_weight_from_storage (fp16 stored scales);
    * rand_K{K}_{cb}: random container words (8x8 tiles, 128x128 weight),
      random positive scales, unpacked and decoded for every K and codebook.
    """
    sys.path.insert(0, REF)
    import torch
    from exl3_quant import serialization as ser
    from exl3_quant.layer_quant import QuantizedModuleResult

    arrays = {}
    gm = np.load(out / "module_golden.npz")
    enc = torch.from_numpy(gm["encoded"])
    trellis = ser.pack_module_trellis(enc, K=2)
    suh = torch.from_numpy(gm["su"]).flatten().to(torch.float16)
    svh = torch.from_numpy(gm["sv"]).flatten().to(torch.float16)
    arrays["module/trellis"] = trellis.numpy()
    arrays["module/unpacked"] = ser.unpack_module_trellis(trellis, K=2).numpy()
    arrays["module/decoded"] = ser.decode_weight_from_storage(trellis, suh, svh, K=2, cb=2).numpy()
    res = QuantizedModuleResult.__new__(QuantizedModuleResult)
    res.K, res.cb, res.encoded = 2, 2, enc
    res.su, res.sv = torch.from_numpy(gm["su"]), torch.from_numpy(gm["sv"])
    tensors, storage = ser.build_layer_tensors({"self_attn.o_proj": res}, layer_idx=3)
    keys = sorted(tensors)
    arrays["module/layer_keys"] = np.array(keys)
    arrays["module/layer_shapes"] = np.array([json.dumps(list(tensors[k].shape)) for k in keys])
    arrays["module/layer_dtypes"] = np.array([str(tensors[k].dtype) for k in keys])
    arrays["module/storage_json"] = np.array(json.dumps(storage, sort_keys=True))
    rng = np.random.default_rng(77)
    cases = []
    for K in range(1, 9):
        cb = (2, 1, 0)[K % 3]
        words = rng.integers(0, 65536, size=(8, 8, 16 * K), dtype=np.uint32).astype(np.uint16)
        tr = torch.from_numpy(words.view(np.int16).copy())
        su = torch.from_numpy(rng.uniform(0.5, 2.0, 128).astype(np.float16))
        sv = torch.from_numpy((rng.uniform(0.5, 2.0, 128) * rng.choice([-1, 1], 128))
                              .astype(np.float16))
        name = f"rand_K{K}_cb{cb}"
        arrays[f"{name}/trellis"] = tr.numpy()
        arrays[f"{name}/suh"], arrays[f"{name}/svh"] = su.numpy(), sv.numpy()
        arrays[f"{name}/unpacked"] = ser.unpack_module_trellis(tr, K=K).numpy()
        arrays[f"{name}/decoded"] = ser.decode_weight_from_storage(tr, su, sv, K=K, cb=cb).numpy()
        arrays[f"{name}/params"] = np.array([K, cb])
        cases.append(name)
    np.savez_compressed(out / "storage_golden.npz", **arrays)
    return {"module": "module_golden encoded K=2 mul1", "random": cases}


def main():
    global REF
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default="", help="comma list: encoder,forward,format,float,ldlq,module,storage,gss")
    ap.add_argument("--procs", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    REF = str(Path(args.reference).resolve())
    sys.path.insert(0, REF)
    os.environ["OMP_NUM_THREADS"] = "1"
    only = set(filter(None, args.only.split(",")))
    manifest_path = HERE / "MANIFEST.json"
    manifest = json.loads(manifest_path.read_text()) if manifest_path.exists() else {}
    ctx = mp.get_context("spawn")
    with ctx.Pool(args.procs, initializer=_init, initargs=(REF,)) as pool:
        if not only or "format" in only:
            manifest["format"] = gen_format(HERE)
        if not only or "forward" in only:
            manifest["forward"] = gen_forward(pool, HERE)
        if not only or "float" in only:
            gen_float(HERE)
            manifest["float"] = "float_golden.npz"
        if not only or "ldlq" in only:
            manifest["ldlq"] = gen_ldlq(pool, HERE)
        if not only or "encoder" in only:
            manifest["encoder"] = gen_encoder(pool, HERE)
        if not only or "module" in only:
            manifest["module"] = gen_module(HERE)
        if not only or "storage" in only:
            manifest["storage"] = gen_storage(HERE)
        if not only or "gss" in only:
            manifest["gss"] = gen_gss(pool, HERE)
    files = {}
    for f in sorted(HERE.glob("*.npz")):
        files[f.name] = hashlib.sha256(f.read_bytes()).hexdigest()
    manifest["sha256"] = files
    manifest["generator"] = "tests/golden/make_golden.py --reference <checkout>"
    manifest_path.write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", sorted(files))


def _init(ref):
    global REF
    REF = ref
    sys.path.insert(0, ref)
    os.environ["OMP_NUM_THREADS"] = "1"
    import torch
    torch.set_num_threads(1)


if __name__ == "__main__":
    main()
