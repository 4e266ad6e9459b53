#!/usr/bin/env python3
"""Benchmark of the EXL3 trellis encoder on B200.

Workload (the encoder sweep): 65,536 16x16 tiles per GPU of
N(0,1) weights scaled per (tile, row) by LogNormal(0, 0.5), K=2 (headline,
the reference's published 1,711.5 tiles/s on Arc B580 is for this K), mul1
codebook, tail-biting two-pass encode with packed output. One step encodes the
whole batch. Synthetic seeded data; the reference evaluates no dataset here.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs one rank per GPU under torch.distributed.run; every rank encodes
its own 65,536 tiles (weak scaling, no data-path collective); the reported
value is all ranks' tiles / the slowest rank's device time.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime as _dt
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "encoder tiles/s at K=2/4 (1/2/4/8 B200); seconds per 4096x4096 layer"
PUBLISHED_K2_TILES_PER_S = 1711.5     # the reference's published Arc B580 rate, K=2 mul1
ACS_PER_TILE = 2 * 256 * 65536        # candidate add-compare-selects per tile (both passes)
FP16_OPS_PER_ACS = 2                  # sub + fma per candidate on the fp16 FMA pipe
                                      # (the running min is an ALU-pipe op)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--K", type=int, default=2)
    ap.add_argument("--tiles", type=int, default=65536)
    ap.add_argument("--chunk", type=int, default=8192, help="tiles per workspace chunk")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-k4", action="store_true")
    ap.add_argument("--no-layer", action="store_true")
    ap.add_argument("--no-decoder-layer", action="store_true")
    ap.add_argument("--no-k-sweep", action="store_true")
    ap.add_argument("--no-hessian", action="store_true")
    ap.add_argument("--model-only", action="store_true",
                    help="convert the config-5 model (32 decoder layers, K=4) on all ranks and exit")
    ap.add_argument("--model-layers", type=int, default=32)
    ap.add_argument("--decoder-layer-only", action="store_true",
                    help="convert one config-4 decoder layer at K=2 and K=4 on all ranks and exit")
    ap.add_argument("--hessian-only", action="store_true",
                    help="time the Hessian accumulation on config 4 shapes and exit")
    ap.add_argument("--hessian-tokens", type=int, default=262144)
    ap.add_argument("--layer-only", action="store_true",
                    help="only the 4096x4096 K=4 layer measurement (config 3)")
    ap.add_argument("--storage-only", action="store_true",
                    help="time pack / unpack / weight decode on config-4 module shapes and exit")
    ap.add_argument("--small-call-only", action="store_true",
                    help="time one encoder call of --tiles tiles at --K (latency of an LDLQ "
                         "step) with --cluster CTAs per tile pair and exit")
    ap.add_argument("--cluster", type=int, default=0,
                    help="encoder cluster split for every mode: 0 automatic, 1 off, 2/4/8 forced")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_tiles(n, seed, device):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    base = torch.randn((n, 16, 16), generator=g)
    scale = torch.exp(0.5 * torch.randn((n, 16, 1), generator=g))
    return (base * scale).reshape(n, 256).to(device)


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "samples": len(rows), "reasons": sorted(reasons)}


def lib_timing():
    from exl3_intel_arc_quantizer_b200._ext import lib

    h = lib()
    h.exl3_timing_end.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]
    return h


def fp16x2_peak():
    import torch

    from exl3_intel_arc_quantizer_b200._ext import lib

    h = lib()
    h.exl3_probe_fp16x2_rate.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_void_p]
    best = 0.0
    for _ in range(3):
        v = ctypes.c_double(0.0)
        rc = h.exl3_probe_fp16x2_rate(ctypes.byref(v), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if rc == 0:
            best = max(best, v.value)
    return best


def cpu_baseline(K, threads=None, seconds_target=12.0, impl_tag="port"):
    """C oracle (plain-C restatement of the reference encoder), all host
    threads, on a bounded sample of the same workload."""
    import numpy as np

    from oracle.trellis_oracle import COracle

    threads = threads or os.cpu_count() or 1
    o = COracle(K, 2)
    probe = make_tiles(threads, 99, "cpu").numpy()
    t0 = time.perf_counter()
    o.encode_batch(probe, threads=threads)
    per_round = max(1e-3, time.perf_counter() - t0)
    rounds = max(1, int(seconds_target / per_round))
    n = threads * rounds
    tiles = make_tiles(n, 7, "cpu").numpy()
    t0 = time.perf_counter()
    r = o.encode_batch(tiles, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tiles/s", "cores": int(r["threads"]), "kind": impl_tag,
            "sample": f"{n} tiles of the config-2 distribution, K={K}, C restatement of the "
                      f"reference encoder (oracle/trellis_oracle.c), {dt:.1f}s"}


_REF_ENCODER = None


def _ref_worker_init(K):
    """Pool worker set-up: the reference's own encoder from the byte-compiled
    reference package (oracle/_ref)."""
    global _REF_ENCODER
    from oracle import build_ref

    build_ref.enable()
    from exl3_quant.reference_encoder import ReferenceTrellisEncoder

    _REF_ENCODER = ReferenceTrellisEncoder(K=K, cb=2)


def _ref_worker_encode(tile):
    return _REF_ENCODER.encode_tile(tile, pre_permute=False).end_state


class ReferenceEncoderPool:
    """The reference's CPU encoder (ReferenceTrellisEncoder.encode_tile,
    exl3_quant/reference_encoder.py:253-324, its NumPy code byte-compiled into
    oracle/_ref) in one spawned process per host core with OMP_NUM_THREADS=1,
    one tile per task. None when oracle/_ref was not built."""

    def __new__(cls, K, procs=None):
        from oracle import build_ref

        if not build_ref.available():
            return None
        return super().__new__(cls)

    def __init__(self, K, procs=None):
        import multiprocessing as mp

        from oracle import build_ref

        self.procs = procs or os.cpu_count() or 1
        old = os.environ.get("OMP_NUM_THREADS")
        os.environ["OMP_NUM_THREADS"] = "1"          # inherited by the spawned workers
        try:
            self.pool = mp.get_context("spawn").Pool(
                self.procs, initializer=_ref_worker_init, initargs=(K,))
        finally:
            if old is None:
                os.environ.pop("OMP_NUM_THREADS", None)
            else:
                os.environ["OMP_NUM_THREADS"] = old

    def encode(self, tiles):
        return self.pool.map(_ref_worker_encode, list(tiles), chunksize=1)

    def close(self):
        self.pool.close()
        self.pool.join()


def reference_cpu_baseline(K, tiles_per_core=2):
    """The reference's own CPU encoder on every host core (the line the
    reference's CPU path gives), on a bounded sample of the workload."""
    pool = ReferenceEncoderPool(K)
    if pool is None:
        return None
    try:
        pool.encode(make_tiles(pool.procs, 98, "cpu").numpy())       # imports, tables
        n = pool.procs * tiles_per_core
        tiles = make_tiles(n, 7, "cpu").numpy()
        t0 = time.perf_counter()
        pool.encode(tiles)
        dt = time.perf_counter() - t0
    finally:
        pool.close()
    return {"value": n / dt, "unit": "tiles/s", "cores": pool.procs, "kind": "reference",
            "sample": f"{n} tiles of the config-2 distribution, K={K}: the reference's "
                      "ReferenceTrellisEncoder.encode_tile (reference_encoder.py:253-324, "
                      f"byte-compiled), {pool.procs} spawned processes, OMP_NUM_THREADS=1, "
                      f"{dt:.1f}s"}


def run_reference(args):
    """Reference arm: the reference's own CPU encoder on every host core
    (ReferenceEncoderPool); the C restatement of oracle/ only when the
    compiled reference package is absent. Bounded samples per step."""
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    pool = ReferenceEncoderPool(args.K)
    if pool is not None:
        try:
            per_step = pool.procs
            tiles = make_tiles(per_step, 7, "cpu").numpy()
            for _ in range(args.warmup):
                pool.encode(tiles)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                pool.encode(tiles)
            dt = time.perf_counter() - t0
        finally:
            pool.close()
        value = per_step * args.steps / dt
        base = {"value": value, "unit": "tiles/s", "cores": pool.procs, "kind": "reference",
                "sample": f"{per_step} tiles/step x {args.steps} steps: the reference's "
                          "ReferenceTrellisEncoder.encode_tile (reference_encoder.py:253-324, "
                          "byte-compiled from its sources), one spawned process per core, "
                          "OMP_NUM_THREADS=1"}
        line = _reference_line(args, value, dt, per_step, base)
        line["cpu_baseline_port"] = cpu_baseline(args.K, seconds_target=6.0)
        print(json.dumps(line), flush=True)
        return 0
    from oracle.trellis_oracle import COracle

    o = COracle(args.K, 2)
    per_step = threads * 2
    tiles = make_tiles(per_step, 7, "cpu").numpy()
    for _ in range(args.warmup):
        o.encode_batch(tiles[:threads], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r = o.encode_batch(tiles, threads=threads)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    base = {"value": value, "unit": "tiles/s", "cores": int(r["threads"]), "kind": "port",
            "sample": f"{per_step} tiles/step x {args.steps} steps, C restatement of the "
                      "reference encoder (the compiled reference package is absent)"}
    print(json.dumps(_reference_line(args, value, dt, per_step, base)), flush=True)
    return 0


def _reference_line(args, value, dt, per_step, cpu):
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tiles/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"encoder sweep (config 2) K={args.K} mul1 L=256, "
                               f"{per_step} tiles per step (bounded sample)", "K": args.K},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tiles/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def layer_config3(device, seed=0):
    """W 4096x4096 bf16 N(0, 0.02^2) with 1% outlier
    columns x8; X 2048x4096 bf16 N(0,1) with 32 outlier channels x20."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    W = torch.randn(4096, 4096, generator=g) * 0.02
    W[:, torch.randperm(4096, generator=g)[:41]] *= 8.0
    X = torch.randn(2048, 4096, generator=g)
    X[:, torch.randperm(4096, generator=g)[:32]] *= 20.0
    return W.to(torch.bfloat16).to(device), X.to(torch.bfloat16).to(device)


def run_layer(device, K=4, reps=2, skip_g_scale=True):
    """Seconds per 4096x4096 linear layer: Hessian (X^T X, finalize) and
    quantize_linear_module (regularize, Hadamard, block-LDL, LDLQ with the
    B200 encoder, reconstruction, metrics), each timed end to end."""
    import torch

    from exl3_intel_arc_quantizer_b200.calibration import hessian_accumulate_, hessian_finalize_
    from exl3_intel_arc_quantizer_b200.layer_quant import quantize_linear_module
    from exl3_intel_arc_quantizer_b200.ldlq import make_xpu_tile_encoder

    W, X = layer_config3(device)
    enc = make_xpu_tile_encoder(K=K, device_index=device.index or 0)
    out = {}
    for rep in range(reps + 1):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        H = torch.zeros(4096, 4096, dtype=torch.float32, device=device)
        hessian_accumulate_(H, X)
        hessian_finalize_(H, X.shape[0], 0.01, 1e-7)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        res = quantize_linear_module("o_proj", W, H, K=K, tile_encoder=enc,
                                     skip_g_scale=skip_g_scale, buf_size_k=128, block_size=16)
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        if rep > 0:   # first repetition is warm-up
            out.setdefault("hessian_s", []).append(t1 - t0)
            out.setdefault("layer_s", []).append(t2 - t1)
            m = res.metrics
            out["relative_frobenius_error"] = m.relative_frobenius_error
            out["normalized_proxy_loss"] = m.normalized_proxy_loss
            out["retries"] = m.retries
            out["g_scale"] = m.g_scale
    enc.encoder.arena.release()
    gss = "skip_g_scale" if skip_g_scale else f"global-scale search (g={out['g_scale']:.4f})"
    return {
        "workload": f"config 3: 4096x4096 bf16 layer, K={K}, Hessian from 2048x4096 bf16, "
                    f"{gss}, buf 128, block 16",
        "seconds_per_layer": min(out["layer_s"]),
        "hessian_seconds": min(out["hessian_s"]),
        "tiles": 65536, "K": K,
        "relative_frobenius_error": out["relative_frobenius_error"],
        "normalized_proxy_loss": out["normalized_proxy_loss"],
        "reference_published_seconds": 43.0 if (K == 2 and not skip_g_scale) else None,
        "reference_published_note": "Arc B580, 4096x4096 o_proj, K=2 with global-scale search "
                                    "(reports/discrete_phase_c.md); no K=4 figure is published",
    }


def layer_cpu_baseline(K=4, crop=512, threads=None):
    """Config-3 layer on the host cores through the module oracle
    (oracle/module_oracle.py: the reference's float stages with torch on the
    CPU, the C restatement of the encoder on every host thread). The float
    stages run at full size with a rounding stand-in for the encoder; the
    encoder runs on a crop x crop corner of the layer (W and its Hessian), and
    its time is scaled to the layer's 65,536 tiles (extrapolated)."""
    import torch

    from oracle import module_oracle as mo

    threads = threads or os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        W, X = layer_config3("cpu")
        W, X = W.float(), X.float()
        t0 = time.perf_counter()
        H = mo.hessian(X)
        t_hess = time.perf_counter() - t0

        def rounding(tiles):
            return torch.round(tiles * 8.0) / 8.0, torch.zeros(tiles.shape, dtype=torch.int16)

        t_float = mo.quantize_module(W, H, K, encode=rounding).seconds
        Hc = mo.hessian(X[:, :crop])
        rc = mo.quantize_module(W[:crop, :crop].contiguous(), Hc, K,
                                encode=mo.c_encoder(K, 2, threads))
        tiles = crop * crop // 256
        est = t_hess + t_float + rc.seconds * (65536 / tiles)
        return {"value": est, "unit": "s per 4096x4096 layer (extrapolated)", "cores": threads,
                "kind": "port",
                "sample": f"Hessian {t_hess:.2f}s and float stages {t_float:.2f}s at full size "
                          f"(rounding stand-in encoder); module with the C encoder on the "
                          f"{crop}x{crop} corner ({tiles} tiles, {rc.seconds:.1f}s) scaled "
                          f"x{65536 // tiles} by tiles; K={K}, torch CPU + oracle/trellis_oracle.c"}
    finally:
        torch.set_num_threads(prev)


def run_storage(device, K=4, shapes=((4096, 4096), (12288, 4096)), reps=5):
    """Storage side on config-4/5 module shapes: pack (states -> container),
    unpack (container -> states) and the one-pass weight decode (container ->
    codebook -> both rotations -> fp32 weight), and the HBM-bound float
    stages on the same shapes (Hadamards, regularization, block-LDL fold). Each launch timed alone with
    CUDA events, L2 flushed before it (512 MiB write); bandwidth from the
    algorithmic bytes: decode K/8 B read + 4 B written per weight, pack
    2 B read + K/8 B written, unpack K/8 B read + 2 B written."""
    import torch

    from exl3_intel_arc_quantizer_b200._ext import ext

    peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) \
        if (REPO / "MEASURED_PEAKS.json").exists() else {}
    hbm = float(peaks.get("hbm_gbs") or 6650.0)
    e = ext()
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)
    out = []
    for k, n in shapes:
        g = torch.Generator(device=device).manual_seed(k + n)
        tk, tn = k // 16, n // 16
        # a random container is a valid trellis stream: unpack gives its states
        container = torch.randint(-32768, 32767, (tk * tn, 16 * K), generator=g, device=device,
                                  dtype=torch.int32).to(torch.int16)
        states = torch.empty((tk * tn, 256), dtype=torch.int16, device=device)
        e.unpack_trellis(container, states, K)
        packed = torch.empty_like(container)
        unpacked = torch.empty_like(states)
        su = (torch.rand(k, generator=g, device=device) + 0.5).half()
        sv = (torch.rand(n, generator=g, device=device) + 0.5).half()
        w = torch.empty((k, n), dtype=torch.float32, device=device)

        def timed(fn):
            best = []
            for r in range(reps + 1):
                flush.fill_(r & 0xFF)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                fn()
                e1.record()
                e1.synchronize()
                if r:
                    best.append(e0.elapsed_time(e1))
            return statistics.median(best)

        t_pack = timed(lambda: e.pack_trellis(states, packed, K))
        t_unpack = timed(lambda: e.unpack_trellis(packed.view(tk, tn, 16 * K),
                                                  unpacked.view(tk, tn, 256), K))
        t_dec = timed(lambda: e.decode_weight(packed.view(tk, tn, 16 * K), su, sv, w, None, K, 2))
        assert torch.equal(packed, container) and torch.equal(unpacked, states)
        # the floating-point stages on the same shape: in-place 128-block
        # Hadamards (8 B per weight), the device regularization (20 B per
        # weight: column sums, W/sv + right FWHT, work/su + left FWHT; timed
        # through the binding that leaves its four info words on the device,
        # so the host's wake-up from the read-back sync is not in the kernel
        # time) and the block-LDL fold of a (k, k) factor (4 B written per
        # element, 4 B read below the diagonal)
        t_hl = timed(lambda: e.had128_left_(w))
        t_hr = timed(lambda: e.had128_right_(w))
        W0 = torch.randn((k, n), generator=g, device=device) * 0.02
        ones_k = torch.ones(k, device=device)
        ones_n = torch.ones(n, device=device)
        hd = torch.rand(k, generator=g, device=device) + 0.5
        regs = [torch.empty_like(W0), torch.empty(k, device=device), torch.empty(n, device=device),
                torch.empty(n, device=device), torch.empty(k, device=device)]
        t_reg = timed(lambda: e.regularize_device_(W0, ones_k, ones_n, hd, -1, False, *regs))
        a = torch.randn((k, k // 2), generator=g, device=device)
        chol = torch.linalg.cholesky(a @ a.T / k + 0.05 * torch.eye(k, device=device)).contiguous()
        L = torch.empty_like(chol)
        inv = torch.empty((k // 16, 16, 16), device=device)
        del a
        t_fold = timed(lambda: e.block_ldl_fold(chol, L, inv))
        del W0, regs, chol, L, inv
        wts = k * n
        row = {"shape": [k, n], "K": K,
               "pack_ms": t_pack, "pack_gbs": wts * (2 + K / 8) / t_pack / 1e6,
               "unpack_ms": t_unpack, "unpack_gbs": wts * (K / 8 + 2) / t_unpack / 1e6,
               "decode_ms": t_dec, "decode_gbs": wts * (K / 8 + 4) / t_dec / 1e6,
               "had_left_ms": t_hl, "had_left_gbs": wts * 8 / t_hl / 1e6,
               "had_right_ms": t_hr, "had_right_gbs": wts * 8 / t_hr / 1e6,
               "regularize_ms": t_reg, "regularize_gbs": wts * 20 / t_reg / 1e6,
               "ldl_fold_ms": t_fold, "ldl_fold_gbs": k * k * 6 / t_fold / 1e6}
        for key in ("pack", "unpack", "decode", "had_left", "had_right", "regularize", "ldl_fold"):
            row[f"{key}_frac_of_measured_hbm"] = row[f"{key}_gbs"] / hbm
        out.append(row)
    # the weight decode at every K on the largest shape (MUL1 codebook, fp16
    # scales, random containers)
    k, n = shapes[-1]
    g = torch.Generator(device=device).manual_seed(17)
    su = (torch.rand(k, generator=g, device=device) + 0.5).half()
    sv = (torch.rand(n, generator=g, device=device) + 0.5).half()
    w = torch.empty((k, n), dtype=torch.float32, device=device)
    sweep = []
    for kk in range(1, 9):
        cont = torch.randint(-32768, 32767, (k // 16, n // 16, 16 * kk), generator=g,
                             device=device, dtype=torch.int32).to(torch.int16)
        ts = []
        for r in range(reps + 1):
            flush.fill_(r & 0xFF)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            e.decode_weight(cont, su, sv, w, None, kk, 2)
            e1.record()
            e1.synchronize()
            if r:
                ts.append(e0.elapsed_time(e1))
        t = statistics.median(ts)
        gbs = k * n * (kk / 8 + 4) / t / 1e6
        sweep.append({"K": kk, "ms": round(t, 4), "gbs": round(gbs, 1),
                      "frac_of_measured_hbm": round(gbs / hbm, 3)})
        del cont
    del flush, w
    return {"kernels": out, "decode_k_sweep": {"shape": [k, n], "rows": sweep},
            "hbm_peak_gbs": hbm,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (copy)" if peaks else "fallback 6650"}


def run_layer_sharded(device, world, rank, K=4, reps=2):
    """Config 3 on several GPUs: the 4096x4096 layer's calibration tokens
    sharded over the ranks (tensor-core X^T X of each shard, one NCCL
    all-reduce, finalize), then quantize_modules with the process group
    (column slices of the LDLQ per rank, one all-gather). Seconds are the
    max over ranks of the best repetition after a warm-up."""
    import torch
    import torch.distributed as dist

    from exl3_intel_arc_quantizer_b200.calibration import hessian_accumulate_, hessian_finalize_
    from exl3_intel_arc_quantizer_b200.distributed import shard_range
    from exl3_intel_arc_quantizer_b200.layer_quant import quantize_modules
    from exl3_intel_arc_quantizer_b200.ldlq import make_xpu_tile_encoder

    W, X = layer_config3(device)
    t0, t1 = shard_range(X.shape[0], world, rank, 64)
    Xs = X[t0:t1].contiguous()
    enc = make_xpu_tile_encoder(K=K, device_index=device.index or 0)
    best, rel = None, None
    for rep in range(reps + 1):
        dist.barrier()
        torch.cuda.synchronize()
        a = time.perf_counter()
        H = torch.zeros(4096, 4096, dtype=torch.float32, device=device)
        hessian_accumulate_(H, Xs)
        dist.all_reduce(H)
        hessian_finalize_(H, X.shape[0], 0.01, 1e-7)
        res = quantize_modules({"o_proj": (W, H)}, K=K, tile_encoder=enc, skip_g_scale=True,
                               buf_size_k=128, block_size=16, group=dist.group.WORLD)
        torch.cuda.synchronize()
        t = torch.tensor([time.perf_counter() - a], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rep > 0:
            best = float(t.item()) if best is None else min(best, float(t.item()))
        rel = res["o_proj"].metrics.relative_frobenius_error
    enc.encoder.arena.release()
    return {"workload": f"config 3: 4096x4096 bf16 layer, K={K}, Hessian from 2048x4096 bf16 "
                        f"(tokens sharded), skip_g_scale, LDLQ columns over {world} GPUs",
            "seconds_per_layer": best, "tiles": 65536, "K": K, "n_gpus": world,
            "relative_frobenius_error": rel}


def run_small_calls(device, Ks=(2, 4), sizes=(2, 16, 30, 32, 64), reps=10):
    """Latency of one encoder call of a few tiles (an LDLQ step of a
    column-sharded module), with the cluster-split ACS (automatic choice)
    and with one CTA per tile pair, in ms per call."""
    import torch

    from exl3_intel_arc_quantizer_b200._ext import set_encoder_cluster
    from exl3_intel_arc_quantizer_b200.xpu_quantizer import XPUTrellisEncoder

    out = []
    try:
        for K in Ks:
            enc = XPUTrellisEncoder(K=K, device_index=device.index or 0)
            for n in sizes:
                x = make_tiles(n, 900 + n, device)
                row = {"K": K, "tiles": n}
                for name, pol in (("cluster_auto_ms", 0), ("one_cta_per_pair_ms", 1)):
                    set_encoder_cluster(pol)
                    for _ in range(3):
                        enc.encode_device(x)
                    torch.cuda.synchronize()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record()
                    for _ in range(reps):
                        enc.encode_device(x)
                    e1.record()
                    e1.synchronize()
                    row[name] = e0.elapsed_time(e1) / reps
                out.append(row)
            enc.arena.release()
    finally:
        set_encoder_cluster(0)
    return out


def run_hessian(device, tokens=262144, dims=(4096, 12288), steps=3, warmup=2):
    """Hessian accumulation H += X^T X (tcgen05 kernel) on BASELINE config 4
    shapes: `tokens` bf16 activation rows, one group per width in `dims`.
    FLOPs are reported as 2*T*d^2 (full square; the kernel computes the upper
    triangle of 128x128 tiles and mirrors it, 2*T*d*(d+128)/2 MMA flops)."""
    import torch

    from exl3_intel_arc_quantizer_b200._ext import ext

    peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) \
        if (REPO / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("bf16_tflops", 1590.0)
    out = []
    for d in dims:
        g = torch.Generator(device=device).manual_seed(d)
        X = torch.randn(tokens, d, generator=g, device=device, dtype=torch.bfloat16)
        H = torch.zeros(d, d, dtype=torch.float32, device=device)
        err = torch.zeros(1, dtype=torch.int32, device=device)
        for _ in range(warmup):
            ext().hessian_accumulate_(H, X, err)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for e0, e1 in ev:
            e0.record()
            ext().hessian_accumulate_(H, X, err)
            e1.record()
        torch.cuda.synchronize()
        ms = min(e0.elapsed_time(e1) for e0, e1 in ev)
        nt = (d + 127) // 128
        mma_flops = 2.0 * tokens * (nt * (nt + 1) // 2) * 128 * 128
        full = 2.0 * tokens * d * d
        # accuracy spot check on a 256x256 corner against an fp32 product
        xs = X[:, :256].float()
        ref = (warmup + steps) * (xs.T @ xs)
        rel = float((H[:256, :256] - ref).abs().max() / ref.abs().max())
        out.append({"tokens": tokens, "d": d, "ms": ms,
                    "tflops_full_square": full / ms / 1e9,
                    "tflops_mma": mma_flops / ms / 1e9,
                    "frac_mma_of_measured_bf16": mma_flops / ms / 1e9 / peak,
                    "err_flag": int(err.item()), "corner_max_rel_err": rel})
        del X, H
        torch.cuda.empty_cache()
    return {"workload": "config 4 Hessian groups, bf16 activations, fp32 H",
            "peak_bf16_tflops_measured": peak, "groups": out}


_FULL_LAYER_WARM: list = []


def run_decoder_layer(device, world, rank, K, seqs_total=128, seq_len=2048, hidden=4096,
                      inter=12288, heads=32, kv_heads=8, batch_seqs=4):
    """one decoder layer of a 9B-class GQA transformer
    (hidden 4096, 32 q / 8 kv heads x 128, SwiGLU 12288), random-init bf16
    weights (std 0.02, identical on every rank), calibration on 128 x 2048
    synthetic N(0,1) tokens sharded over the ranks; all seven projections
    converted (calibrate -> Hessian all-reduce -> quantize with column
    sharding -> reload -> re-forward). Seconds are max over ranks."""
    import torch
    import torch.distributed as dist

    from exl3_intel_arc_quantizer_b200.calibration import TransformerDecoderLayer
    from exl3_intel_arc_quantizer_b200.converter import convert_layer

    group = dist.group.WORLD if world > 1 else None

    def build(h, it, nh, nkv, seed):
        # weights as a checkpoint would hold them (bf16), already on the GPU:
        # loading is outside the timed region
        torch.manual_seed(seed)
        layer = TransformerDecoderLayer(h, it, nh, nkv)
        with torch.no_grad():
            for p in layer.parameters():
                if p.dim() == 2:
                    p.normal_(0.0, 0.02)
        return layer.to(device=device, dtype=torch.bfloat16)

    def make_hidden(nseq, s, h, seed):
        g = torch.Generator(device=device).manual_seed(seed)
        return [torch.randn(min(batch_seqs, nseq - i), s, h, generator=g, device=device,
                            dtype=torch.float16) for i in range(0, nseq, batch_seqs)]

    # warm-up on a small layer (extension load, cuBLAS/cuSOLVER handles), then
    # once per process one untimed full-size layer (first-use allocations and
    # kernel set-up of the full shapes), so the timed layer is a steady-state
    # one like every layer after the first of a model conversion
    convert_layer(build(512, 1024, 4, 2, 1), make_hidden(2, 128, 512, 5 + rank), K=K,
                  device=device, group=group)
    per_rank = seqs_total // world
    if not _FULL_LAYER_WARM:
        convert_layer(build(hidden, inter, heads, kv_heads, 6),
                      make_hidden(per_rank, seq_len, hidden, 2000 + rank), K=K, device=device,
                      group=group)
        _FULL_LAYER_WARM.append(True)
    hs = make_hidden(per_rank, seq_len, hidden, 1000 + rank)
    layer = build(hidden, inter, heads, kv_heads, 7)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    t0 = time.perf_counter()
    res, nxt, tm = convert_layer(layer, hs, K=K, device=device, group=group)
    torch.cuda.synchronize()
    sec = time.perf_counter() - t0
    clk = clocks.stop()
    phases = [tm.calibrate_s, tm.reduce_s, tm.quantize_s, tm.reload_reforward_s, sec]
    if world > 1:
        t = torch.tensor(phases, device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        phases = t.tolist()
    rel = {m: r.metrics.relative_frobenius_error for m, r in res.items()}
    del res, nxt, hs, layer
    torch.cuda.empty_cache()
    return {"workload": f"config 4: decoder layer h{hidden}/i{inter}/{heads}q{kv_heads}kv x128, "
                        f"K={K}, {seqs_total}x{seq_len} calibration tokens over {world} GPU(s)",
            "K": K, "seconds_per_layer": phases[4], "tiles": tm.tiles,
            "tokens": seqs_total * seq_len,
            "phases_s": {"calibrate": phases[0], "hessian_allreduce_finalize": phases[1],
                         "quantize": phases[2], "reload_reforward": phases[3]},
            "tiles_per_s": tm.tiles / phases[2],
            "relative_frobenius_error": rel, "clocks": clk}


def run_model(device, world, rank, K=4, nlayers=32, seqs_total=128, seq_len=2048, hidden=4096,
              inter=12288, heads=32, kv_heads=8, batch_seqs=4):
    """a 32-layer model of the config-4 decoder shape
    converted layer by layer (calibrate on the current hidden states,
    Hessian all-reduce, quantize with column sharding, reload, re-forward),
    calibration tokens sharded over the ranks. Random-init bf16 weights
    (std 0.02, identical on every rank), synthetic N(0,1) hidden states in
    place of the (unquantized) embedding output. Seconds are max over ranks."""
    import torch
    import torch.distributed as dist

    from exl3_intel_arc_quantizer_b200.calibration import TransformerDecoderLayer
    from exl3_intel_arc_quantizer_b200.converter import convert_layers

    group = dist.group.WORLD if world > 1 else None
    layers = []
    for li in range(nlayers):
        torch.manual_seed(1000 + li)
        with torch.device(device):
            layer = TransformerDecoderLayer(hidden, inter, heads, kv_heads)
        with torch.no_grad():
            for p in layer.parameters():
                if p.dim() == 2:
                    p.normal_(0.0, 0.02)
        layers.append(layer.to(torch.bfloat16))
    per_rank = seqs_total // world
    g = torch.Generator(device=device).manual_seed(7 + rank)
    hs = [torch.randn(min(batch_seqs, per_rank - i), seq_len, hidden, generator=g, device=device,
                      dtype=torch.float16) for i in range(0, per_rank, batch_seqs)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    results, timings = convert_layers(layers, hs, K=K, device=device, group=group)
    torch.cuda.synchronize()
    sec = time.perf_counter() - t0
    tiles = sum(t.tiles for t in timings)
    if world > 1:
        t = torch.tensor([sec], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t.item())
    rel = [sum(r.metrics.relative_frobenius_error for r in res.values()) / len(res)
           for res in results]
    return {"workload": f"config 5: {nlayers} decoder layers h{hidden}/i{inter}/{heads}q{kv_heads}kv, "
                        f"K={K}, {seqs_total}x{seq_len} calibration tokens over {world} GPU(s)",
            "K": K, "layers": nlayers, "seconds": sec, "seconds_per_layer": sec / nlayers,
            "tiles": tiles, "tiles_per_s_per_gpu": tiles / sec / world,
            "mean_relative_frobenius_error_first_last": [rel[0], rel[-1]]}


def run_b200(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=_dt.timedelta(seconds=300), device_id=device)

    from exl3_intel_arc_quantizer_b200._ext import ext
    from exl3_intel_arc_quantizer_b200.xpu_quantizer import ScratchArena, XPUTrellisEncoder

    K, n = args.K, args.tiles
    if args.cluster:
        from exl3_intel_arc_quantizer_b200._ext import set_encoder_cluster

        set_encoder_cluster(args.cluster)   # encoder cluster split for every mode below
    if args.model_only:
        out = {"model": run_model(device, world, rank, K=4, nlayers=args.model_layers)}
        if rank == 0:
            print(json.dumps(out), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.decoder_layer_only:
        out = {"decoder_layer": [run_decoder_layer(device, world, rank, k) for k in (2, 4)]}
        if rank == 0:
            print(json.dumps(out), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.hessian_only:
        if rank == 0:
            print(json.dumps({"hessian": run_hessian(device, tokens=args.hessian_tokens)}),
                  flush=True)
        return 0
    if args.storage_only:
        if rank == 0:
            print(json.dumps({"storage": run_storage(device)}), flush=True)
        return 0
    if args.small_call_only:
        if rank == 0:
            from exl3_intel_arc_quantizer_b200._ext import set_encoder_cluster

            set_encoder_cluster(args.cluster)
            try:
                enc = XPUTrellisEncoder(K=K, cb=2, device_index=local)
                x = make_tiles(n, 4321, device)
                for _ in range(args.warmup):
                    enc.encode_device(x)
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(args.steps):
                    enc.encode_device(x)
                e1.record()
                e1.synchronize()
                print(json.dumps({"small_call": {"K": K, "tiles": n, "cluster": args.cluster,
                                                 "ms_per_call": e0.elapsed_time(e1) / args.steps}}),
                      flush=True)
                enc.arena.release()
            finally:
                set_encoder_cluster(0)
        return 0
    if args.layer_only:
        if world > 1:
            out = {"layer_sharded": run_layer_sharded(device, world, rank)}
            if rank == 0:
                print(json.dumps(out), flush=True)
            dist.barrier()
            dist.destroy_process_group()
            return 0
        if rank == 0:
            print(json.dumps({"layer": run_layer(device),
                              "layer_k2_gss": run_layer(device, K=2, skip_g_scale=False)}),
                  flush=True)
        return 0
    enc = XPUTrellisEncoder(K=K, cb=2, device_index=local,
                            arena=ScratchArena(device_index=local, default_cap_b=args.chunk))
    x = make_tiles(n, 1234 + rank, device)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)  # > L2 (126 MB)

    for _ in range(args.warmup):
        enc.encode_device(x)
    torch.cuda.synchronize()

    timing = lib_timing()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    timing.exl3_timing_begin()
    step_ms = []
    for _ in range(args.steps):
        flush.zero_()                         # evict L2 between timed steps
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        enc.encode_device(x)
        e1.record()
        e1.synchronize()
        step_ms.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    acs_ms, tb_ms = ctypes.c_double(), ctypes.c_double()
    acs_n, total_n = ctypes.c_int64(), ctypes.c_int64()
    timing.exl3_timing_end(ctypes.byref(acs_ms), ctypes.byref(tb_ms), ctypes.byref(acs_n),
                           ctypes.byref(total_n))
    clk = clocks.stop()
    total_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([total_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        dist.barrier()
    value = world * n * args.steps / (total_ms / 1e3)

    # secondary: the config-2 K sweep (same workload, same timing rules);
    # K=4 is also reported on its own
    def encoder_rate(Kx, reps):
        ex = XPUTrellisEncoder(K=Kx, cb=2, device_index=local,
                               arena=ScratchArena(device_index=local, default_cap_b=args.chunk))
        for _ in range(2):
            ex.encode_device(x)
        ms = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            ex.encode_device(x)
            e1.record()
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        tx = sum(ms)
        if world > 1:
            t = torch.tensor([tx], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            tx = float(t.item())
        ex.arena.release()
        return world * n * len(ms) / (tx / 1e3)

    k4 = None
    if not args.no_k4 and K != 4:
        k4 = encoder_rate(4, max(2, args.steps // 2))
    ksweep = None
    if not args.no_k_sweep:
        ksweep = {str(kx): (value if kx == K else (k4 if (kx == 4 and k4) else
                                                    encoder_rate(kx, 2)))
                  for kx in (1, 2, 3, 4, 5, 6, 8)}

    # e2e through the op binding with pinned host buffers
    e2e = None
    if not args.no_e2e:
        host_in = x.cpu().pin_memory()
        h_w = torch.empty((n, 256), dtype=torch.float32).pin_memory()
        h_i = torch.empty((n, 256), dtype=torch.int16).pin_memory()
        h_p = torch.empty((n, 16 * K), dtype=torch.int16).pin_memory()
        d_in = torch.empty_like(x)
        d_w = torch.empty_like(x)
        d_i = torch.empty((n, 256), dtype=torch.int16, device=device)
        d_p = torch.empty((n, 16 * K), dtype=torch.int16, device=device)
        ws, per, adm = enc.arena.acquire(K, 256, args.chunk)
        e = ext()
        # chunks of the workspace's size go through three streams: pinned
        # host -> device copies, the encoder (op binding, current stream),
        # device -> pinned host copies; per chunk, events order each stage
        # after the one before and after the previous step's use of the buffers
        comp = torch.cuda.current_stream(device)
        s_in, s_out = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
        chunks = [(c, min(c + args.chunk, n)) for c in range(0, n, args.chunk)]
        ev_in = [torch.cuda.Event() for _ in chunks]
        ev_c = [torch.cuda.Event() for _ in chunks]
        ev_out = [torch.cuda.Event() for _ in chunks]

        def one():
            for q, (a, b) in enumerate(chunks):
                s_in.wait_event(ev_c[q])        # the last step's encode has read d_in[a:b]
                with torch.cuda.stream(s_in):
                    d_in[a:b].copy_(host_in[a:b], non_blocking=True)
                    ev_in[q].record(s_in)
                comp.wait_event(ev_in[q])
                comp.wait_event(ev_out[q])      # the last step's outputs have left
                e.encode_tiles(d_in[a:b], d_w[a:b], d_i[a:b], d_p[a:b], None, ws, K, 2)
                ev_c[q].record(comp)
                s_out.wait_event(ev_c[q])
                with torch.cuda.stream(s_out):
                    h_w[a:b].copy_(d_w[a:b], non_blocking=True)
                    h_i[a:b].copy_(d_i[a:b], non_blocking=True)
                    h_p[a:b].copy_(d_p[a:b], non_blocking=True)
                    ev_out[q].record(s_out)

        for _ in range(2):
            one()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        s_in.wait_event(e0)
        for _ in range(args.steps):
            one()
        for ev in ev_out:
            comp.wait_event(ev)
        e1.record(comp)
        e1.synchronize()
        t_e2e = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([t_e2e], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        e2e = {"value": world * n * args.steps / (t_e2e / 1e3), "unit": "tiles/s",
               "h2d_bytes_per_step": int(host_in.numel() * 4),
               "d2h_bytes_per_step": int(h_w.numel() * 4 + h_i.numel() * 2 + h_p.numel() * 2)}

    peak = fp16x2_peak()
    tiles_timed = n * args.steps
    achieved = tiles_timed * ACS_PER_TILE * FP16_OPS_PER_ACS / (acs_ms.value / 1e3)
    traffic = None
    tfile = REPO / "profiles" / f"encoder_k{K}_dram_per_launch.json"
    if tfile.exists():
        prof = json.loads(tfile.read_text())
        per = prof.get("dram_bytes_per_tile_per_pass")
        if per is not None and prof.get("layout") == "cost checkpoints, bulk copies":
            # one ACS launch = one pass over a chunk; per-tile bytes from an
            # ncu capture of smaller launches, scaled by the chunk's tiles
            traffic = per * min(args.chunk, n)
    roofline = {
        "bound": "fp16_fma_pipe",
        "achieved": achieved / 1e9, "peak": peak / 1e9, "unit": "Gop/s",
        "frac": achieved / peak if peak else None,
        "peak_source": "measured live: exl3_probe_fp16x2_rate (fma.rn.f16x2 at full occupancy)",
        "work": f"{ACS_PER_TILE} candidate ACS/tile x {FP16_OPS_PER_ACS} fp16 ops on the FMA "
                "pipe (sub, fma; the min is on the ALU pipe)",
        "kernel": "exl3::acs_pair_kernel (pass 1 + pass 2)" if K >= 2 else
                  "exl3::acs_kernel (pass 1 + pass 2)",
        "acs_share_of_step": acs_ms.value / max(1e-9, sum(step_ms)),
        "traffic": traffic,
        "traffic_unit": "bytes per ACS launch (ncu dram read+write per tile of a smaller "
                        "launch, scaled to the chunk)",
    }
    from exl3_intel_arc_quantizer_b200.scratch_estimator import b200_hbm_bytes_written_per_tile

    ck_bytes_per_tile = b200_hbm_bytes_written_per_tile(K)   # both passes' checkpoints
    roofline["trellis_bytes_written_per_tile"] = ck_bytes_per_tile
    roofline["hbm_trellis_write_gbs"] = (tiles_timed * ck_bytes_per_tile
                                         / (acs_ms.value / 1e3) / 1e9)

    # the headline encoder's workspace is not used by the sections below
    enc.arena.release()
    cpu = cpu_port = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_port = cpu_baseline(K)
        cpu = reference_cpu_baseline(K) or cpu_port
    small = run_small_calls(device) if rank == 0 else None
    storage = run_storage(device) if rank == 0 else None
    layer = layer2 = None
    if rank == 0 and not args.no_layer:
        layer = run_layer(device)
        if world == 1 and not args.no_cpu_baseline:
            layer["cpu_baseline"] = layer_cpu_baseline(K=4)
        layer2 = run_layer(device, K=2, skip_g_scale=False)
    if world > 1:
        dist.barrier()
    layer_sh = None
    if world > 1 and not args.no_layer:
        layer_sh = run_layer_sharded(device, world, rank)
    declayer = None
    if not args.no_decoder_layer:
        declayer = [run_decoder_layer(device, world, rank, k) for k in (2, 4)]
    hessian = None
    if rank == 0 and not args.no_hessian:
        hessian = run_hessian(device)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tiles/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (value / PUBLISHED_K2_TILES_PER_S) if K == 2 else None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"encoder sweep (config 2): {n} tiles/GPU of N(0,1) x "
                                   f"LogNormal(0,0.5) row scales, K={K}, mul1, L=256, "
                                   "tail-biting 2-pass + packed output",
                       "K": K, "tiles_per_gpu": n, "chunk_tiles": args.chunk,
                       "l2": "flushed between timed steps (512 MiB write)",
                       "parallelism": f"tiles sharded, {world} rank(s), no collective"},
            "k4_tiles_per_s": k4,
            "k_sweep_tiles_per_s": ksweep,
            "layer": layer,
            "layer_k2_gss": layer2,
            "layer_sharded": layer_sh,
            "decoder_layer": declayer,
            "small_calls": small,
            "storage": storage,
            "roofline": roofline,
            "hessian": hessian,
            "cpu_baseline": cpu,
            "cpu_baseline_port": cpu_port,
            "e2e": e2e,
            "gpu_launches": int(total_n.value),
            "clocks": clk,
        }
        # last key: a short digest of the sections above, so that the end of
        # the line (what a log tail keeps) carries the layer-level numbers
        line["summary"] = summarize(line)
        print(json.dumps(line), flush=True)
    enc.arena.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def summarize(line):
    def r(v, nd=4):
        return None if v is None else float(f"{v:.{nd}g}")

    out = {"encoder_k2_tiles_per_s": r(line["value"], 6),
           "e2e_tiles_per_s": r((line.get("e2e") or {}).get("value"), 6),
           "acs_roofline_frac": r((line.get("roofline") or {}).get("frac"), 3)}
    if line.get("layer"):
        out["config3_layer_k4_s"] = r(line["layer"]["seconds_per_layer"])
    if line.get("layer_k2_gss"):
        out["config3_layer_k2_gss_s"] = r(line["layer_k2_gss"]["seconds_per_layer"])
    if line.get("layer_sharded"):
        out["config3_layer_sharded_s"] = r(line["layer_sharded"].get("seconds_per_layer"))
    for d in line.get("decoder_layer") or []:
        out[f"config4_layer_k{d['K']}_s"] = r(d["seconds_per_layer"])
        out[f"config4_layer_k{d['K']}_phases_s"] = {k: r(v, 3) for k, v in d["phases_s"].items()}
    for row in (line.get("storage") or {}).get("kernels", [])[-1:]:   # the largest shape
        tag = "x".join(str(v) for v in row["shape"])
        for key in ("decode", "had_left", "regularize", "ldl_fold"):
            if f"{key}_frac_of_measured_hbm" in row:
                out[f"{key}_{tag}_frac_hbm"] = r(row[f"{key}_frac_of_measured_hbm"], 3)
    for g in (line.get("hessian") or {}).get("groups", []):
        out[f"hessian_d{g['d']}_ms"] = r(g["ms"])
        out[f"hessian_d{g['d']}_frac_bf16"] = r(g["frac_mma_of_measured_bf16"], 3)
    for key, tag in (("cpu_baseline", "cpu_reference"), ("cpu_baseline_port", "cpu_port")):
        c = line.get(key)
        if c:
            out[f"{tag}_tiles_per_s"] = r(c["value"])
            out[f"{tag}_cores"] = c["cores"]
    out["n_gpus"] = line["n_gpus"]
    return out


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
