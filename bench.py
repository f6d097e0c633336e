"""Benchmark: 8B-shaped Q4_0 greedy decode on the cuda-b200 backend.

Workload (the headline configuration): a Llama-3-8B-shaped model, 32
layers, hidden 4096, 32 query / 8 KV heads of 128, FFN 14336, vocab
128256; layer matrices Q4_0, embedding and lm head Q8_0; weights N(0, 0.02)
from a seed; a 512-token seeded prompt, then greedy decode steps with an
fp16 KV cache, batch 1 (``--batch 8`` for eight independent sequences).
A step is one decoded token per sequence through every layer and the lm
head. ``value`` is decode tokens/s with everything resident in HBM
(CUDA-graph replays timed by CUDA events); ``e2e`` is the same through
the C ABI's host-buffer call (``pai_b200_session_step``: token H2D, step,
next-token D2H each step). The model's 4.5 GB of weights exceed the
126 MB L2, so no flush is needed between steps.

``--impl reference`` times the reference's own CPU implementation of the
path instead (see ``reference_arm``).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG_8B = dict(n_layer=32, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=14336,
              vocab=128256, eps=1e-5, rope_theta=500000.0, wtype=2, etype=8)
PROMPT = 512
SEED = 20261201
# DRAM bytes per launch of the 32-layer persistent layer kernel, batch 1: ncu's
# dram__bytes_read.sum + dram__bytes_write.sum of a 4-layer launch x 8
# (profiles/k_decode_q4_0_8b.md)
K_DECODE_TRAFFIC = 4176 * 10 ** 6
METRIC = "Q4_0 8B-shape decode tok/s"
UNIT = "tokens/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """bf16 dense TFLOP/s: the measured burst figure (a kernel timed alone)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def prefill_gemm(dev, iters=12, ms=(16, 128, 512, 2048), shards=1, t=2):
    """Config 2: the Q4_0 prefill GEMM Y[M,14336] = X[M,4096] . W^T on the
    tcgen05 tensor cores (X f32 -> bf16 tiles, W dequantised to bf16 in
    shared memory, fp32 accumulate in TMEM), for M in 16/128/512/2048.
    Rotates over 4 distinct weight copies (4 x 33 MB > L2) so every launch
    streams its weights from HBM, as successive layers of a prefill do.
    Timed with CUDA events; the time covers the X conversion kernel and
    the GEMM (the whole call)."""
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Buffer
    L = _native.load()
    # with shards > 1 this rank holds a column shard (N / shards output rows);
    # t: the weights' block type (Q4_0 is config 2's; Q8_0 and Q4_K run the same GEMM)
    n, k = CFG_8B["n_ff"] // shards, CFG_8B["n_embd"]
    tname = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K"}[t]
    rb = L.pai_b200_block_bytes(t, k)
    copies = 4 * shards
    tmp = dev.alloc(n * k * 4)
    blk = dev.alloc(n * rb)
    offs = dev.put(np.arange(n, dtype=np.uint64) * rb)
    mats = []
    for c in range(copies):
        _native.check(L.pai_b200_synth_blocks(dev.ctx, t, n, k, SEED + 2000 + c, 0.02, tmp.ptr,
                                              blk.ptr), "synth")
        w = Buffer(dev, L.pai_b200_packed_bytes(t, n, k))
        _native.check(L.pai_b200_pack(dev.ctx, t, n, k, blk.ptr, offs.ptr, w.ptr), "pack")
        mats.append(w)
    tmp.free()
    blk.free()
    peak, kind = tensor_peak()
    out = {"workload": f"{tname} GEMM N={n} K=4096 (config 2{', column shard' if shards > 1 else ''}), "
                       "bf16 tiles, fp32 accumulate",
           "kernel": f"k_gemm<{tname}> (tcgen05.mma kind::f16, TMEM accumulators) + k_gemm_xprep",
           "peak_tflops": peak, "peak_kind": kind,
           "l2": f"{copies} rotating weight copies ({copies * n * rb / 1e6:.0f} MB)",
           "by_m": {}}
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    for m in ms:
        x = dev.put(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32))
        y = dev.alloc(m * n * 4)
        for i in range(4):
            _native.check(L.pai_b200_gemm_f32(dev.ctx, t, m, n, k, x.ptr, mats[i % copies].ptr, y.ptr), "gemm")
        dev.sync()
        L.pai_b200_event_record(dev.ctx, e0)
        for i in range(iters):
            L.pai_b200_gemm_f32(dev.ctx, t, m, n, k, x.ptr, mats[i % copies].ptr, y.ptr)
        L.pai_b200_event_record(dev.ctx, e1)
        ms = C.c_float()
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        dev.sync()
        per = ms.value / iters
        tf = 2.0 * m * n * k / (per * 1e-3) / 1e12
        out["by_m"][str(m)] = {"us": round(per * 1e3, 2), "tflops": round(tf, 1),
                               "frac": round(tf / peak, 4)}
        x.free()
        y.free()
    for w in mats:
        w.free()
    return out


class Clocks:
    """Sample nvidia-smi clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
                self.lines = [l for l in out.splitlines() if l.strip()]
            except Exception:
                pass

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def gemv_roofline(dev, hbm_peak, peak_kind, iters=40):
    """Time the dominant kernel alone: the Q4_0 GEMV of one layer's fused
    gate|up matrix (28672 x 4096), rotating over 8 distinct copies
    (8 x 66 MB > L2) so every launch streams its weights from HBM.
    Back-to-back launches under programmatic dependent launch, as inside
    the decode step (each launch's weight prefetch overlaps the previous
    launch's tail); the plain-launch time is reported beside it."""
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Buffer
    L = _native.load()
    n, k, t = 2 * CFG_8B["n_ff"], CFG_8B["n_embd"], 2
    rb = L.pai_b200_block_bytes(t, k)
    copies = 8
    tmp = dev.alloc(n * k * 4)
    blk = dev.alloc(n * rb)
    offs = dev.put(np.arange(n, dtype=np.uint64) * rb)
    mats = []
    for c in range(copies):
        _native.check(L.pai_b200_synth_blocks(dev.ctx, t, n, k, SEED + 1000 + c, 0.02, tmp.ptr,
                                              blk.ptr), "synth")
        pk = Buffer(dev, L.pai_b200_packed_bytes(t, n, k))
        _native.check(L.pai_b200_pack(dev.ctx, t, n, k, blk.ptr, offs.ptr, pk.ptr), "pack")
        mats.append(pk)
    tmp.free()
    blk.free()
    x = dev.put(np.random.default_rng(1).standard_normal(k).astype(np.float32))
    xq = C.c_void_p()
    _native.check(L.pai_b200_alloc(dev.ctx, L.pai_b200_xq_bytes(1, k), C.byref(xq)), "alloc xq")
    _native.check(L.pai_b200_prepare_x_f32(dev.ctx, 1, k, x.ptr, xq), "prepare_x")
    y = dev.alloc(n * 4)
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    per = {}
    for mode in (0, 1):
        _native.check(L.pai_b200_set_pdl(dev.ctx, mode), "set_pdl")
        for i in range(6):
            _native.check(L.pai_b200_gemv_prepared_f32(dev.ctx, t, 1, n, k, mats[i % copies].ptr, xq,
                                                       None, y.ptr), "gemv")
        dev.sync()
        L.pai_b200_event_record(dev.ctx, e0)
        for i in range(iters):  # k_gemv launches only: x was prepared once
            L.pai_b200_gemv_prepared_f32(dev.ctx, t, 1, n, k, mats[i % copies].ptr, xq, None, y.ptr)
        L.pai_b200_event_record(dev.ctx, e1)
        ms = C.c_float()
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        dev.sync()
        per[mode] = ms.value / iters
    _native.check(L.pai_b200_set_pdl(dev.ctx, 0), "set_pdl")
    alg = n * rb + k * 4 + n * 4  # weights + x (f32) + y (f32, plain store)
    achieved = alg / (per[1] * 1e-3) / 1e9
    for mat in mats:
        mat.free()
    L.pai_b200_free(dev.ctx, xq)
    return {"kernel": "k_gemv<Q4_0> gate|up 28672x4096, batch 1 (plain-store epilogue)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(alg), "avg_launch_ms": round(per[1], 5),
            "launch_mode": "back-to-back, programmatic dependent launch (as in the decode step)",
            "plain_launch": {"avg_launch_ms": round(per[0], 5),
                             "achieved": round(alg / (per[0] * 1e-3) / 1e9, 1)},
            # DRAM bytes of one launch of this kernel on this workload, from one ncu
            # capture (profiles/k_gemv_q4_0_gateup.md: dram__bytes_read.sum 66.18 MB
            # + dram__bytes_write.sum 0.47 MB), not measured by this run
            "traffic": 66650000, "traffic_source": "one ncu capture (profiles/k_gemv_q4_0_gateup.md)"}


def layer_kernel_roofline(dev, model, sess, hbm_peak, peak_kind, reps=20):
    """The dominant kernel of the step: the persistent layer kernel (every
    layer of one decode step in one cooperative launch), timed alone with
    CUDA events on its stream over `reps` back-to-back launches. Algorithmic
    bytes per launch: every layer's packed weights (read once), the K/V cache
    rows attended over, one embedding row and the new K/V rows. The position
    does not advance between these launches (pai_b200_session_run_layers)."""
    from prosperoai_b200 import _native
    L = _native.load()
    c = model.cfg
    if sess.step_kernels != 4:
        return None
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    sess.run_layers(3)  # warm-up
    dev.sync()
    L.pai_b200_event_record(dev.ctx, e0)
    sess.run_layers(reps)
    L.pai_b200_event_record(dev.ctx, e1)
    ms = C.c_float()
    _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
    per_ms = ms.value / reps
    E, vocab = c["n_embd"], c["vocab"]
    lm_head = L.pai_b200_block_bytes(c["etype"], vocab * E)
    emb_row = L.pai_b200_block_bytes(c["etype"], E)
    layer_w = model.step_weight_bytes() - lm_head - emb_row
    npos = sess.pos + 1
    kv = c["n_layer"] * c["n_head_kv"] * c["head_dim"] * 2 * 2 * npos * sess.batch
    alg = layer_w + kv + emb_row
    achieved = alg / (per_ms * 1e-3) / 1e9
    return {"kernel": "k_decode<Q4_0> (persistent: embedding row, 32 layers, final RMSNorm; 148 CTAs, "
                      "cooperative launch)",
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(alg),
            "bytes_breakdown": {"layer_weights": int(layer_w), "kv_cache": int(kv), "embedding_row": int(emb_row)},
            "positions_attended": npos, "avg_launch_ms": round(per_ms, 5), "launches_timed": reps,
            # ncu dram__bytes_read.sum + dram__bytes_write.sum of a 4-layer launch of the same
            # kernel (profiles/k_decode_q4_0_8b.md), scaled to 32 layers (batch 1 only)
            "traffic": K_DECODE_TRAFFIC if sess.batch == 1 and c["n_layer"] == 32 else None,
            "traffic_source": "profiles/k_decode_q4_0_8b.md: ncu DRAM bytes of a 4-layer launch x 32/4"}


def gemv_sweep(dev, hbm_peak, peak_kind, iters=30):
    """Configs 1 and 3: the Q8_0 4096x4096 GEMV and the Q4_K GEMV shapes,
    batch 1, x prepared once; each shape rotates over enough distinct
    copies to exceed 2x the L2 (every launch streams from HBM). Timed with
    CUDA events over back-to-back launches under programmatic dependent
    launch (as in the decode step) and plainly."""
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Buffer
    L = _native.load()
    shapes = [("config 1", 8, 4096, 4096)] + [("config 3", 12, n_, k_) for n_, k_ in
                                             ((4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336),
                                              (128256, 4096))]
    out = []
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    for cfg_name, t, n, k in shapes:
        rb = L.pai_b200_block_bytes(t, k)
        copies = max(2, int(2 * 126e6 // (n * rb)) + 1)
        tmp = dev.alloc(n * k * 4)
        blk = dev.alloc(n * rb)
        offs = dev.put(np.arange(n, dtype=np.uint64) * rb)
        mats = []
        for c in range(copies):
            _native.check(L.pai_b200_synth_blocks(dev.ctx, t, n, k, SEED + 3000 + c, 0.02, tmp.ptr, blk.ptr),
                          "synth")
            pk = Buffer(dev, L.pai_b200_packed_bytes(t, n, k))
            _native.check(L.pai_b200_pack(dev.ctx, t, n, k, blk.ptr, offs.ptr, pk.ptr), "pack")
            mats.append(pk)
        tmp.free()
        blk.free()
        offs.free()
        x = dev.put(np.random.default_rng(2).standard_normal(k).astype(np.float32))
        xq = C.c_void_p()
        _native.check(L.pai_b200_alloc(dev.ctx, L.pai_b200_xq_bytes(1, k), C.byref(xq)), "alloc xq")
        _native.check(L.pai_b200_prepare_x_f32(dev.ctx, 1, k, x.ptr, xq), "prepare_x")
        y = dev.alloc(n * 4)
        per = {}
        for mode in (0, 1):
            _native.check(L.pai_b200_set_pdl(dev.ctx, mode), "set_pdl")
            for i in range(4):
                _native.check(L.pai_b200_gemv_prepared_f32(dev.ctx, t, 1, n, k, mats[i % copies].ptr, xq,
                                                           None, y.ptr), "gemv")
            dev.sync()
            L.pai_b200_event_record(dev.ctx, e0)
            for i in range(iters):
                L.pai_b200_gemv_prepared_f32(dev.ctx, t, 1, n, k, mats[i % copies].ptr, xq, None, y.ptr)
            L.pai_b200_event_record(dev.ctx, e1)
            ms = C.c_float()
            _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
            dev.sync()
            per[mode] = ms.value / iters
        _native.check(L.pai_b200_set_pdl(dev.ctx, 0), "set_pdl")
        alg = n * (k // (256 if t == 12 else 32)) * (144 if t == 12 else 34) + 4 * k + 4 * n
        gbs = alg / (per[1] * 1e-3) / 1e9
        out.append({"config": cfg_name, "type": "Q4_K" if t == 12 else "Q8_0", "n": n, "k": k,
                    "algorithmic_bytes": int(alg), "us": round(per[1] * 1e3, 2), "gbs": round(gbs, 1),
                    "frac": round(gbs / hbm_peak, 4), "plain_us": round(per[0] * 1e3, 2)})
        for m_ in mats:
            m_.free()
        y.free()
        x.free()
        L.pai_b200_free(dev.ctx, xq)
    return {"peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
            "launch_mode": "back-to-back, programmatic dependent launch; plain_us: plain launches",
            "shapes": out}


def v0_sweep(dev, hbm_peak, peak_kind, iters=40):
    """The v0 grouped-scale GEMMs at the config-1 shape (4096x4096, one
    activation row): the registered w8/w4 ops (scales per (k-group,
    column)) and .pai blobs (scales per 32 flat elements), each rotating
    over enough distinct weight copies to exceed 2x the L2. Device time:
    CUDA events around graph replays of the calls (one graph of `iters`
    calls, so host launch cost is not in the device time); plain_us: the
    same calls launched one by one from Python."""
    from prosperoai_b200 import _native
    L = _native.load()
    n = k = 4096
    g = 32
    rng = np.random.default_rng(SEED + 77)
    a = dev.put(rng.standard_normal(k).astype(np.float32))
    c = dev.alloc(n * 4)
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    out = []
    for name, bits, form in (("gemm_w8_f32", 8, "op"), ("gemm_w4_f32", 4, "op"),
                             ("gemm_v0_f32 q8", 8, "pai"), ("gemm_v0_f32 q4", 4, "pai")):
        vbytes = n * k if bits == 8 else n * k // 2
        sbytes = 4 * (n * k // g)
        copies = int(2 * 126e6 // (vbytes + sbytes)) + 1
        bufs = []
        for _ in range(copies):
            v = rng.integers(-128, 128, vbytes, dtype=np.int8).view(np.uint8)
            sc = (rng.uniform(0.5, 1.5, n * k // g) / 127).astype(np.float32).view(np.uint8)
            bufs.append((dev.put(v), dev.put(sc)) if form == "op" else (dev.put(np.concatenate([v, sc])),))

        def call(i):
            b = bufs[i % copies]
            if form == "op":
                fn = L.pai_b200_gemm_w8_f32 if bits == 8 else L.pai_b200_gemm_w4_f32
                return fn(dev.ctx, 1, n, k, a.ptr, b[0].ptr, b[1].ptr, g, c.ptr)
            return L.pai_b200_gemm_v0_f32(dev.ctx, bits, g, 1, n, k, a.ptr, b[0].ptr, c.ptr)

        for i in range(4):
            _native.check(call(i), name)
        dev.sync()
        # plain launches: one ctypes call each, host-bound at this size
        L.pai_b200_event_record(dev.ctx, e0)
        for i in range(iters):
            call(i)
        L.pai_b200_event_record(dev.ctx, e1)
        ms = C.c_float()
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        dev.sync()
        plain_us = ms.value / iters * 1e3
        # device time: the same calls captured in one CUDA graph and replayed
        graph = C.c_void_p()
        _native.check(L.pai_b200_graph_begin(dev.ctx), "graph_begin")
        for i in range(iters):
            _native.check(call(i), name)
        _native.check(L.pai_b200_graph_end(dev.ctx, C.byref(graph)), "graph_end")
        for _ in range(3):
            _native.check(L.pai_b200_graph_launch(dev.ctx, graph), "graph_launch")
        dev.sync()
        reps = 5
        L.pai_b200_event_record(dev.ctx, e0)
        for _ in range(reps):
            L.pai_b200_graph_launch(dev.ctx, graph)
        L.pai_b200_event_record(dev.ctx, e1)
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        dev.sync()
        L.pai_b200_graph_destroy(graph)
        us = ms.value / (reps * iters) * 1e3
        alg = vbytes + sbytes + 4 * k + 4 * n
        gbs = alg / (us * 1e-6) / 1e9
        out.append({"op": name, "scales": "per (32-row group, column)" if form == "op"
                    else "per 32 flat elements (.pai blob)", "n": n, "k": k, "rows": 1,
                    "algorithmic_bytes": int(alg), "us": round(us, 2), "gbs": round(gbs, 1),
                    "frac": round(gbs / hbm_peak, 4), "plain_us": round(plain_us, 2), "copies": copies})
        for b in bufs:
            for x in b:
                x.free()
    a.free()
    c.free()
    return {"peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s", "shapes": out}


def layer_config4(dev, hbm_peak, peak_kind, steps=30, warmup=5):
    """Config 4: one Q4_0 decoder layer of the 8B shape, fp16 KV cache with
    4096 past positions, batch 1, one token appended per step. Built as a
    one-layer model with a 512-row Q8_0 embedding/lm head; the 4096 past
    positions are written by a prefill of seeded token ids (the cache
    values, not their distribution, are what the step reads). Timed with
    CUDA events over graph-replayed steps; the step also runs the embedding
    row, the final norm, the 2.2 MB lm head and the argmax."""
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Model, Session
    L = _native.load()
    cfg = dict(CFG_8B, n_layer=1, vocab=512)
    past = 4096
    m = Model(dev, cfg)
    m.synthesize(SEED + 4)
    sess = Session(m, 1, past + warmup + steps + 8)
    sess.prefill(np.random.default_rng(SEED + 4).integers(0, cfg["vocab"], (1, past)).astype(np.int32))
    sess.run(warmup)
    dev.sync()
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    pos0 = sess.pos
    L.pai_b200_event_record(dev.ctx, e0)
    sess.run(steps)
    L.pai_b200_event_record(dev.ctx, e1)
    ms = C.c_float()
    _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
    dev.sync()
    kern_us = None
    if sess.step_kernels == 4:  # the persistent layer kernel of this one-layer model, timed alone
        sess.run_layers(3)
        L.pai_b200_event_record(dev.ctx, e0)
        sess.run_layers(steps)
        L.pai_b200_event_record(dev.ctx, e1)
        ms_k = C.c_float()
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms_k)), "elapsed")
        kern_us = ms_k.value / steps * 1e3
    sess.close()
    m.close()
    us = ms.value / steps * 1e3
    E, F, hd, H, HK = cfg["n_embd"], cfg["n_ff"], cfg["head_dim"], cfg["n_head"], cfg["n_head_kv"]
    weights = ((H + 2 * HK) * hd * E + E * H * hd + 3 * F * E) * 18 // 32  # Q4_0 bytes of the layer
    kv = HK * (pos0 + steps // 2) * hd * 2 * 2  # K and V read at the middle timed position
    alg = weights + kv + 4 * (E + F) * 2
    gbs = alg / (us * 1e-6) / 1e9
    out = {"workload": "config 4: one Q4_0 decoder layer (8B shape), fp16 KV cache, batch 1",
           "past_positions": past, "positions_timed": [pos0, pos0 + steps - 1], "us_per_step": round(us, 2),
           "layer_steps_per_s": round(1e6 / us, 1), "algorithmic_bytes": int(alg), "gbs": round(gbs, 1),
           "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind,
           "note": "the step also runs an embedding row, final norm, a 512-row Q8_0 lm head and argmax"}
    if kern_us is not None:
        kg = alg / (kern_us * 1e-6) / 1e9
        out["layer_kernel"] = {"us_per_launch": round(kern_us, 2), "gbs": round(kg, 1),
                               "frac": round(kg / hbm_peak, 4),
                               "what": "the persistent layer kernel alone (embedding row, the layer, final "
                                       "norm; one cooperative launch each, position not advanced)"}
    return out


def prefill_timing(dev, sess, prompts, reps=3, pg=None):
    """Time-to-first-token of the config-5 prompt through
    pai_b200_session_prefill (tokens from host memory, the next token read
    back), against stepping the prompt one decode step per position.
    CUDA events around each call; the best of `reps` after one warm-up."""
    from prosperoai_b200 import _native
    L = _native.load()
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    times = []
    for i in range(reps + 1):
        sess.reset()
        dev.sync()
        L.pai_b200_event_record(dev.ctx, e0)
        sess.prefill(prompts)
        L.pai_b200_event_record(dev.ctx, e1)
        ms = C.c_float()
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        if i:
            times.append(ms.value)
    best = min(times)
    if pg is not None:  # the job's time: the slowest rank
        import torch
        t = torch.tensor([best], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        best = float(t.item())
    B, P = prompts.shape
    return {"api": "pai_b200_session_prefill", "sequences": B, "positions": P, "ms": round(best, 3),
            "tokens_per_s": round(B * P / (best * 1e-3), 1),
            "path": "Q4_0 layers: tcgen05 GEMM over all prompt rows; attention over the fp16 cache"
                    + ("; row-parallel outputs summed by NCCL all-reduce, max over ranks" if pg is not None else "")}


def cpu_baseline_port(dev, steps=3, prompt=24):
    """The CPU restatement (oracle/, bit-identical to the reference ops)
    on a bounded sample of the same decode: one 8B-shaped layer plus 1/32
    of the lm-head rows, fed a short prompt, then `steps` timed tokens on
    all host cores. tokens/s for the full model = 1 / (32 x sample time)."""
    from oracle import py_oracle as po
    from prosperoai_b200 import _native
    L = _native.load()
    cfg = dict(CFG_8B, n_layer=1, vocab=CFG_8B["vocab"] // 32)
    E, qd, kd, ff = cfg["n_embd"], 4096, 1024, cfg["n_ff"]
    shapes = {"wq": (qd, E, 2, 3), "wk": (kd, E, 2, 4), "wv": (kd, E, 2, 5), "wo": (E, qd, 2, 6),
              "wgate": (ff, E, 2, 7), "wup": (ff, E, 2, 8), "wdown": (E, ff, 2, 9),
              "tok_embd": (cfg["vocab"], E, 8, 0), "output": (cfg["vocab"], E, 8, 1)}
    w = {}
    for name, (rows, cols, t, kind) in shapes.items():
        tmp = dev.alloc(rows * cols * 4)
        blk = dev.alloc(rows * L.pai_b200_block_bytes(t, cols))
        _native.check(L.pai_b200_synth_blocks(dev.ctx, t, rows, cols,
                                              L.pai_b200_tensor_seed(SEED, kind, 0), 0.02, tmp.ptr,
                                              blk.ptr), "synth")
        b = blk.download(np.uint8)
        w[name] = b if name in ("tok_embd", "output") else [b]
        tmp.free()
        blk.free()
    w["attn_norm"] = [np.ones(E, np.float32)]
    w["ffn_norm"] = [np.ones(E, np.float32)]
    w["output_norm"] = np.ones(E, np.float32)
    threads = os.cpu_count() or 1
    s = po.Session(cfg, w, prompt + steps + 2, threads=threads)
    tok = 1
    for i in range(prompt):
        tok = s.step(i % cfg["vocab"])
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = s.step(tok)
    dt = (time.perf_counter() - t0) / steps
    s.close()
    return {"value": round(1.0 / (32 * dt), 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"oracle C restatement, 1 of 32 layers + 1/32 of lm-head rows at the 8B shape, "
                       f"positions {prompt}..{prompt + steps - 1}, {steps} tokens timed; "
                       f"full-model tok/s = 1/(32 x {dt * 1e3:.1f} ms)")}


def path_session(model, batch, max_ctx, persistent):
    """A session whose step runs the layers as the persistent kernel
    (PAI_B200_PERSISTENT=1) or as one launch per op."""
    from prosperoai_b200.api import Session
    os.environ["PAI_B200_PERSISTENT"] = "1" if persistent else "0"
    try:
        return Session(model, batch, max_ctx)
    finally:
        os.environ.pop("PAI_B200_PERSISTENT", None)


def decode_variant(dev, model, batch, prompt, steps=20, warmup=3, persistent=None):
    """Decode tok/s of one more session of the same model: `batch`
    independent sequences after a `prompt`-token seeded prompt (appended by
    pai_b200_session_prefill), CUDA-graph steps timed with CUDA events (as
    the headline line). persistent: True/False picks the step's path
    (persistent layer kernel or one launch per op), None the default."""
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Session
    L = _native.load()
    if persistent is None:
        sess = Session(model, batch, prompt + warmup + steps + 8)
    else:
        sess = path_session(model, batch, prompt + warmup + steps + 8, persistent)
    kernels = sess.step_kernels
    ids = np.random.default_rng(SEED + batch).integers(0, CFG_8B["vocab"], (batch, prompt)).astype(np.int32)
    sess.prefill(ids)
    sess.run(warmup)
    dev.sync()
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    pos0 = sess.pos
    L.pai_b200_event_record(dev.ctx, e0)
    sess.run(steps)
    L.pai_b200_event_record(dev.ctx, e1)
    ms = C.c_float()
    _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
    out = {"batch": batch, "prompt": prompt, "positions_timed": [pos0, pos0 + steps - 1],
           "ms_per_step": round(ms.value / steps, 4), "value": round(batch * steps / (ms.value * 1e-3), 3),
           "unit": UNIT, "launches_per_step": kernels,
           "path": "one launch per op" if kernels != 4 else "persistent layer kernel"}
    if kernels == 4:
        # the layer kernel alone: per-layer time and bytes inside the 32-layer launch
        sess.run_layers(2)
        L.pai_b200_event_record(dev.ctx, e0)
        sess.run_layers(10)
        L.pai_b200_event_record(dev.ctx, e1)
        _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
        c = model.cfg
        per_layer_us = ms.value / 10 * 1e3 / c["n_layer"]
        E, F, hd, H, HK = c["n_embd"], c["n_ff"], c["head_dim"], c["n_head"], c["n_head_kv"]
        lw = ((H + 2 * HK) * hd * E + E * H * hd + 3 * F * E) * 18 // 32  # Q4_0 bytes of one layer
        kv = HK * (sess.pos + 1) * hd * 2 * 2 * batch
        gbs = (lw + kv) / (per_layer_us * 1e-6) / 1e9
        hbm, kind = peaks()
        out["layer_in_model"] = {"us_per_layer": round(per_layer_us, 2), "bytes_per_layer": int(lw + kv),
                                 "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4), "peak_kind": kind,
                                 "what": "persistent layer kernel timed alone / layers"}
    sess.close()
    return out


def gpu_arm(args):
    from prosperoai_b200 import _native
    from prosperoai_b200.api import Device, Model, Session, TPComm
    rank, world, local = dist_env()
    pg = None
    if world > 1:
        import torch.distributed as dist
        # host-side plumbing only (barriers, timing max, the communicator id)
        dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=180))
        pg = dist
    tp = world > 1 and not args.replicas
    if tp:
        # the exchanges are 16 KB per sequence: no NVLink multicast (NVLS) objects
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    if world > 1 and os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        # NCCL's version banner goes to stdout, where rank 0 prints the one JSON line
        os.environ["NCCL_DEBUG"] = "WARN"
    L = _native.load()
    dev = Device(local)
    cfg = dict(CFG_8B)
    B, K, W = args.batch, args.steps, args.warmup
    # tensor parallel: rank r holds 1/world of every matrix (column-parallel
    # q/k/v/gate/up, row-parallel o/down, vocab-sharded lm head); the row
    # exchanges after o/down and the argmax merge go over NVLink peer memory
    # (IPC-mapped buffers whose handles NCCL exchanges once at setup)
    model = Model(dev, cfg, tp_rank=rank if tp else 0, tp_size=world if tp else 1)
    model.synthesize(SEED)
    comm = None
    if tp:
        comm = TPComm.over_group(dev, rank, world)
        model.set_tp(comm)
    P = args.prompt
    max_ctx = P + W + 2 * K + 8
    sess = Session(model, B, max_ctx)
    prompts = np.random.default_rng(SEED).integers(0, cfg["vocab"], (B, P)).astype(np.int32)
    # nvidia-smi needs about a second to start sampling and the timed steps
    # take a fraction of one, so sampling spans the prompt, warm-up and
    # timed steps (the same kernels throughout)
    clk = Clocks(local).__enter__()
    prefill = None
    if not args.no_roofline and (tp or world == 1):
        prefill = prefill_timing(dev, sess, prompts, pg=pg)  # collective under tensor parallelism
        sess.reset()  # the stepped prompt below overwrites the cache from position 0
    for p in range(P):  # prompt positions, untimed
        sess.set_tokens(prompts[:, p])
        sess.run(1)
    sess.run(W)  # warm-up greedy steps
    dev.sync()
    if pg:
        pg.barrier()
    launches0 = dev.launches()
    e0, e1 = C.c_void_p(), C.c_void_p()
    L.pai_b200_event_create(dev.ctx, C.byref(e0))
    L.pai_b200_event_create(dev.ctx, C.byref(e1))
    pos0 = sess.pos
    dev.sync()
    if args.nvtx:  # lets a profiler select the timed steps (ncu --nvtx --nvtx-include decode_timed/)
        import torch.cuda.nvtx as nvtx
        nvtx.range_push("decode_timed")
    L.pai_b200_event_record(dev.ctx, e0)
    sess.run(K)
    L.pai_b200_event_record(dev.ctx, e1)
    dev.sync()
    if args.nvtx:
        nvtx.range_pop()
    clk.__exit__(None, None, None)
    ms = C.c_float()
    _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms)), "elapsed")
    launches = dev.launches() - launches0
    t_dev = ms.value
    # e2e: the same steps through the host-buffer C ABI call
    tok = sess.tokens()
    dev.sync()
    if pg:
        # every rank starts the e2e loop together: the clock sampler's exit above
        # takes a variable fraction of a second per rank, and under tensor
        # parallelism a rank's first step waits for the last rank to begin
        pg.barrier()
    L.pai_b200_event_record(dev.ctx, e0)
    w0 = time.perf_counter()
    for _ in range(K):
        tok = sess.step(tok)
    wall = (time.perf_counter() - w0) * 1e3
    L.pai_b200_event_record(dev.ctx, e1)
    ms2 = C.c_float()
    _native.check(L.pai_b200_event_elapsed(e0, e1, C.byref(ms2)), "elapsed")
    t_e2e = max(ms2.value, wall)
    if pg:
        import torch
        t = torch.tensor([t_dev, t_e2e], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        t_dev, t_e2e = float(t[0]), float(t[1])
    hbm, kind = peaks()
    # bytes one decode step reads: weights + the KV cache up to the mean position
    mean_pos = pos0 + K / 2.0
    kv_bytes = cfg["n_layer"] * cfg["n_head_kv"] * cfg["head_dim"] * 2 * 2 * mean_pos * B
    # whole job: every rank reads its shard (equal shards), the KV heads split
    step_bytes = model.step_weight_bytes() * (world if tp else 1) + kv_bytes
    step_gbs = step_bytes / (t_dev / K * 1e-3) / 1e9
    step_peak_gpus = world if tp else 1
    result = None
    gemm = None
    if tp and not args.no_roofline:
        # config 2 column-sharded over the ranks: every rank times its shard,
        # the job's time per M is the maximum over ranks
        import torch
        part = prefill_gemm(dev, shards=world)
        ms_list = sorted(int(m) for m in part["by_m"])
        t = torch.tensor([part["by_m"][str(m)]["us"] for m in ms_list], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        peak_tf = part["peak_tflops"]
        gemm = {"workload": f"Q4_0 GEMM N=14336 K=4096 (config 2), column-sharded over {world} GPUs "
                            f"({CFG_8B['n_ff'] // world} rows each), bf16 tiles, fp32 accumulate",
                "kernel": part["kernel"], "peak_tflops": peak_tf * world, "peak_kind": part["peak_kind"],
                "timing": "max over ranks of each rank's CUDA-event time", "by_m": {}}
        for i, m in enumerate(ms_list):
            tf = 2.0 * m * CFG_8B["n_ff"] * CFG_8B["n_embd"] / (float(t[i]) * 1e-6) / 1e12
            gemm["by_m"][str(m)] = {"us": round(float(t[i]), 2), "tflops": round(tf, 1),
                                    "frac": round(tf / (peak_tf * world), 4)}
    if rank == 0:
        layer_roof = None
        if not args.no_roofline and not tp:
            # the persistent layer kernel timed alone, from a session on that path
            psess = sess if sess.step_kernels == 4 else path_session(model, B, max_ctx, True)
            if psess is not sess:
                psess.prefill(prompts)
            layer_roof = layer_kernel_roofline(dev, model, psess, hbm, kind)
            if psess is not sess:
                psess.close()
        gemv_roof = None if args.no_roofline else gemv_roofline(dev, hbm, kind)
        # the dominant kernel of the step the headline measures
        roof = layer_roof if sess.step_kernels == 4 else gemv_roof
        if gemm is None and not args.no_roofline:
            gemm = prefill_gemm(dev)
            # the same GEMM with the other layer block types (prefill of Q8_0 / Q4_K models)
            gemm["other_types"] = [prefill_gemm(dev, ms=(128, 512, 2048), t=t) for t in (8, 12)]
        sweep = None if args.no_roofline else gemv_sweep(dev, hbm, kind)
        v0 = None if args.no_roofline else v0_sweep(dev, hbm, kind)
        cpu = None if args.no_cpu_baseline else cpu_baseline_port(dev)
        variants = None
        if world == 1 and not args.no_roofline:
            # configs 4-5 also name 8 independent sequences and a 4096-position cache
            variants = [decode_variant(dev, model, 8, P), decode_variant(dev, model, 1, 4096),
                        decode_variant(dev, model, 1, P, persistent=sess.step_kernels != 4)]
            variants.append(layer_config4(dev, hbm, kind))
        jobs = 1 if tp else world  # sequences advanced per step: TP ranks share one job
        value = jobs * B * K / (t_dev * 1e-3)
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(t_dev / K, 4), "higher_is_better": True,
            "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "q4_0 weights, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, seeded prompt ids)",
            "config": {"workload": "Llama-3-8B-shaped Q4_0 decode (config 5)", "batch": B,
                       "prompt": P, "positions_timed": [pos0, pos0 + K - 1],
                       "layers": cfg["n_layer"], "hidden": cfg["n_embd"], "vocab": cfg["vocab"],
                       "kv_cache": "fp16",
                       "parallelism": ("single GPU" if world == 1 else
                                       (f"tp{world}: rows exchanged over NVLink peer memory inside the "
                                        f"persistent layer kernel after o and down, vocab-sharded lm head, "
                                        f"argmax merged over peer memory (no collective library call per step)"
                                        if sess.step_kernels == 3 else
                                        f"tp{world}: peer-memory exchange kernel after o/down, NCCL all-gather "
                                        f"for the argmax")
                                       if tp else f"{world} independent replicas"),
                       "l2": "no flush: 4.5 GB of weights per step exceed the 126 MB L2"},
            "e2e": {"value": round(jobs * B * K / (t_e2e * 1e-3), 3), "unit": UNIT,
                    "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
            "gpu_launches": int(launches),
            "decode_path": (f"persistent layer kernel + lm head GEMV + argmax + token feedback "
                            f"({sess.step_kernels} launches per step, one CUDA graph)"
                            if sess.step_kernels <= 4 else
                            f"one launch per op ({sess.step_kernels} per step, one CUDA graph)"),
            "roofline": roof,
            "gemv_roofline": gemv_roof if roof is not gemv_roof else None,
            "layer_kernel_roofline": layer_roof if roof is not layer_roof else None,
            "prefill_gemm": gemm,
            "prompt_prefill": prefill,
            "decode_variants": variants,
            "gemv_configs": sweep,
            "v0_gemm": v0,
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved": round(step_gbs, 1),
                              "peak": round(hbm * step_peak_gpus, 1), "unit": "GB/s",
                              "frac": round(step_gbs / (hbm * step_peak_gpus), 4), "peak_kind": kind,
                              "gpus": step_peak_gpus},
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
    if pg:
        pg.barrier()  # no rank leaves while another may still run collectives
    sess.close()  # releases the graph that holds the NCCL calls first
    if comm:
        comm.close()
    model.close()
    dev.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return result


def reference_arm(args):
    """The reference's own CPU code for one decode token, on a bounded sample.

    oracle/_ref/libpai_ref.so is the reference's cpu/reference, cpu/optimized
    and adapters/llama sources compiled unmodified. Its session keeps
    weights as f32 after dequantising them once (models/model.c:246-290),
    so the sample does that with the reference's dequant_block and then
    runs one 8B-shaped layer per token with the reference's fastest GEMV
    (pai_opt_gemv_f32, AVX2+FMA) on disjoint row slices over all host
    threads, the reference's rmsnorm/rope/silu/vecmul/vecadd, and decode
    attention over 512 cached positions (the last-row loop of
    pai_ref_attention_f32, restated in oracle/ because the reference only
    offers the full-sequence form), plus 1/32 of the lm head.
    tok/s = 1 / (32 x sample time).
    """
    from concurrent.futures import ThreadPoolExecutor

    from oracle import py_oracle as po
    R = po.ref()
    kind = "reference"
    if R is None:
        kind = "port"
    E, ff, qd, kd, hd = 4096, 14336, 4096, 1024, 128
    vocab_s = CFG_8B["vocab"] // 32
    rng = np.random.default_rng(SEED)
    threads = os.cpu_count() or 1

    def dq(t, rows, cols):
        w = (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02))
        blocks = po.quantize(t, w)
        out = np.empty(rows * cols, np.float32)
        if R is not None:
            assert R.pai_refshim_dequant(t, blocks, out, out.size) == 0
        else:
            out[:] = po.dequant(t, blocks, out.size)
        return out.reshape(rows, cols)

    mats = {"q": dq(2, qd, E), "k": dq(2, kd, E), "v": dq(2, kd, E), "o": dq(2, E, qd),
            "gate": dq(2, ff, E), "up": dq(2, ff, E), "down": dq(2, E, ff), "lm": dq(8, vocab_s, E)}
    pool = ThreadPoolExecutor(threads)
    gemv_fn = R.pai_opt_gemv_f32 if R is not None else po.lib().po_gemv_f32

    def gemv(W, x):
        n, k = W.shape
        y = np.empty(n, np.float32)
        bounds = np.linspace(0, n, threads + 1).astype(int)

        def part(i):
            a, b = bounds[i], bounds[i + 1]
            if b > a:
                yv = y[a:b]
                gemv_fn(b - a, k, np.ascontiguousarray(W[a:b]), x, yv)
        list(pool.map(part, range(threads)))
        return y

    P = PROMPT
    kc = rng.standard_normal((8, P + 1, hd)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((8, P + 1, hd)).astype(np.float16).view(np.uint16)
    cos_t, sin_t = po.rope_tables(P + 1, hd // 2, 500000.0)
    ones = np.ones(E, np.float32)
    x = rng.standard_normal(E).astype(np.float32)

    def ref_call(fn, *a):
        if R is not None:
            getattr(R, "pai_ref_" + fn)(*a)
        else:
            getattr(po.lib(), "po_" + fn)(*a)

    def one_token(x):
        xn = np.empty(E, np.float32)
        ref_call("rmsnorm_gamma_f32", x, xn, E, ones, 1e-5)
        q, k, v = gemv(mats["q"], xn), gemv(mats["k"], xn), gemv(mats["v"], xn)
        qr, kr = np.empty_like(q), np.empty_like(k)
        po.lib().po_rope_at_f32(q, 32, hd, P, cos_t, sin_t, hd // 2, qr)
        po.lib().po_rope_at_f32(k, 8, hd, P, cos_t, sin_t, hd // 2, kr)
        kc[:, P] = kr.reshape(8, hd).astype(np.float16).view(np.uint16)
        vc[:, P] = v.reshape(8, hd).astype(np.float16).view(np.uint16)
        att = po.attention_decode_f16(32, 8, hd, P + 1, P + 1, qr, kc, vc)
        o = gemv(mats["o"], att)
        x1 = np.empty(E, np.float32)
        ref_call("vecadd_f32", x, o, x1, E)
        ref_call("rmsnorm_gamma_f32", x1, xn, E, ones, 1e-5)
        g, u = gemv(mats["gate"], xn), gemv(mats["up"], xn)
        sg, h = np.empty_like(g), np.empty_like(g)
        ref_call("silu_f32", g, sg, ff)
        ref_call("vecmul_f32", sg, u, h, ff)
        d = gemv(mats["down"], h)
        x2 = np.empty(E, np.float32)
        ref_call("vecadd_f32", x1, d, x2, E)
        gemv(mats["lm"], x2)
        return x2

    for _ in range(args.warmup):
        one_token(x)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_token(x)
    dt = (time.perf_counter() - t0) / args.steps
    value = 1.0 / (32 * dt)
    sample = (f"reference cpu/optimized pai_opt_gemv_f32 (AVX2) on row slices x {threads} threads + "
              f"cpu/reference elementwise ops, 1 of 32 layers + 1/32 of the lm head per step, "
              f"f32 weights dequantised by the reference's dequant_block, attention over {P + 1} "
              f"cached positions; tok/s = 1/(32 x {dt * 1e3:.1f} ms)")
    # n_gpus: the launch's N (the reference path runs on the host cores; its GPUs stay idle)
    return {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(32 * dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (weights dequantised from Q4_0/Q8_0)", "data": "synthetic",
            "config": {"workload": "Llama-3-8B-shaped Q4_0 decode (config 5)", "batch": 1,
                       "prompt": PROMPT, "device": f"host CPU, {threads} threads"},
            "impl": "reference",
            "caveats": [
                "a bounded sample: 1 of 32 layers and 1/32 of the lm-head rows per token, scaled x32",
                "the reference's fastest GEMV (cpu/optimized pai_opt_gemv_f32) rather than the "
                "pai_ref_gemm_f32 its executor calls, and split over all host threads by this harness "
                "(the reference executor runs a step on one thread): the reference's best case",
                "weights held as f32 after dequantisation, as the reference session keeps them "
                "(models/model.c:246-290): 4x-8x the bytes of the quantised blocks",
                "RoPE at one position and the last-row decode attention are the oracle's restatements "
                "(the reference offers only the full-sequence forms); all other ops are the reference's",
            ],
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1, choices=[1, 2, 4, 8])
    ap.add_argument("--replicas", action="store_true",
                    help="with several GPUs: independent replicas instead of tensor parallelism")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-roofline", action="store_true",
                    help="skip the standalone GEMV timing (profiling runs)")
    ap.add_argument("--prompt", type=int, default=PROMPT,
                    help="prompt length fed before timing (profiling runs use a short one)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the dominant GEMV (28672x4096 Q4_0) and print its roofline line")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the config-2 prefill GEMM and print its line")
    ap.add_argument("--gemm-m", type=int, action="append",
                    help="with --gemm-only: token counts to time (repeatable; default 16 128 512 2048)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="time only the config-5 prompt prefill (with --nvtx: one prefill inside the range prefill)")
    ap.add_argument("--v0-only", action="store_true",
                    help="time only the v0 grouped-scale GEMMs (w8/w4 ops and .pai blobs)")
    ap.add_argument("--nvtx", action="store_true",
                    help="wrap the timed decode steps in the NVTX range decode_timed")
    ap.add_argument("--profile-layers", type=int, default=0,
                    help="profiling only: the persistent layer kernel of an N-layer model with the 8B layer "
                         "shapes (a few GB on the device), launched --steps times after --warmup; prints "
                         "its CUDA-event time per launch, not a bench line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local = dist_env()
    if args.gemm_only:
        from prosperoai_b200.api import Device
        dev = Device(local)
        print(json.dumps(prefill_gemm(dev, ms=tuple(args.gemm_m or (16, 128, 512, 2048)))), flush=True)
        dev.close()
        return
    if args.prefill_only:
        # config-5 prompt prefill alone: one untimed prefill, then (inside the
        # NVTX range "prefill" with --nvtx) the timed ones
        from prosperoai_b200.api import Device, Model, Session
        dev = Device(local)
        model = Model(dev, dict(CFG_8B))
        model.synthesize(SEED)
        sess = Session(model, 1, PROMPT + 8)
        prompts = np.random.default_rng(SEED).integers(0, CFG_8B["vocab"], (1, PROMPT)).astype(np.int32)
        sess.prefill(prompts)
        sess.reset()
        dev.sync()
        if args.nvtx:
            import torch.cuda.nvtx as nvtx
            nvtx.range_push("prefill")
            sess.prefill(prompts)
            nvtx.range_pop()
            sess.reset()
            dev.sync()
        print(json.dumps(prefill_timing(dev, sess, prompts)), flush=True)
        sess.close()
        model.close()
        dev.close()
        return
    if args.profile_layers:
        # a small-memory stand-in for ncu captures of k_decode: N layers of the
        # config-5 shape after a 512-token prefill
        from prosperoai_b200.api import Device, Model, Session
        dev = Device(local)
        cfg = dict(CFG_8B, n_layer=args.profile_layers)
        model = Model(dev, cfg)
        model.synthesize(SEED)
        sess = Session(model, args.batch, PROMPT + args.warmup + 8)
        prompts = np.random.default_rng(SEED).integers(0, cfg["vocab"], (args.batch, PROMPT)).astype(np.int32)
        sess.prefill(prompts)
        sess.run(args.warmup)
        dev.sync()
        L = __import__("prosperoai_b200._native", fromlist=["load"]).load()
        e0, e1 = C.c_void_p(), C.c_void_p()
        L.pai_b200_event_create(dev.ctx, C.byref(e0))
        L.pai_b200_event_create(dev.ctx, C.byref(e1))
        L.pai_b200_event_record(dev.ctx, e0)
        sess.run_layers(args.steps)
        L.pai_b200_event_record(dev.ctx, e1)
        ms = C.c_float()
        L.pai_b200_event_elapsed(e0, e1, C.byref(ms))
        print(json.dumps({"profile": "k_decode", "layers": args.profile_layers, "batch": args.batch,
                          "launches": args.steps, "ms_per_launch": round(ms.value / args.steps, 4)}), flush=True)
        sess.close()
        model.close()
        dev.close()
        return
    if args.v0_only:
        from prosperoai_b200.api import Device
        dev = Device(local)
        hbm, kind = peaks()
        print(json.dumps(v0_sweep(dev, hbm, kind)), flush=True)
        dev.close()
        return
    if args.kernel_only:
        from prosperoai_b200.api import Device
        dev = Device(local)
        hbm, kind = peaks()
        print(json.dumps(gemv_roofline(dev, hbm, kind)), flush=True)
        dev.close()
        return
    if args.impl == "reference":
        if rank != 0:
            return
        args.steps = min(args.steps, 8)
        print(json.dumps(reference_arm(args)), flush=True)
        return
    res = gpu_arm(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
