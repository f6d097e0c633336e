"""Generate tests/golden/*.npz from the reference's own code.

Run in a checkout where the reference sources are available, after
``make -C oracle`` has built ``oracle/_ref/libpai_ref.so`` from them:

    python tests/golden/make_golden.py

Inputs are (a) the known-answer cases of the reference's own tests
(tests/test_gguf.c:284-331,451-490 and tests/test_ref_ops.c:113-119,
224-351, restated here as data) and (b) seeded random cases. Every output
is computed by the reference functions (pai_refshim_dequant = gguf.c's
dequant_block, pai_ref_*), so the fixtures pin the CPU restatement in
oracle/ and, through it, the CUDA path.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import py_oracle as po  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
Q4_0, Q8_0, Q4_K = po.Q4_0, po.Q8_0, po.Q4_K


def f16(v: float) -> bytes:
    return np.array([v], np.float16).tobytes()


def known_blocks():
    """Block bytes of the reference's dequant known-answer tests."""
    q8 = f16(1.0) + bytes((i - 16) & 0xFF for i in range(32))                  # test_gguf.c:284-297
    q4 = f16(1.0) + bytes(j | ((j ^ 8) << 4) for j in range(16))               # :317-331
    q4k = f16(1.0) + f16(0.0) + b"\x01" * 12 + b"\x12" * 128                   # :451-469
    q4k_min = f16(1.0) + f16(0.5) + b"\x01" * 12 + b"\x12" * 128               # :471-490
    exp8 = np.arange(32, dtype=np.float32) - 16
    exp4 = np.concatenate([np.arange(16) - 8, (np.arange(16) ^ 8) - 8]).astype(np.float32)
    e = np.arange(256)
    expk = np.where(e & 32, 1.0, 2.0).astype(np.float32)
    expk_min = (expk - np.where(e < 128, 0.5, 0.0)).astype(np.float32)
    return [("q8_0", Q8_0, q8, exp8), ("q4_0", Q4_0, q4, exp4), ("q4_k", Q4_K, q4k, expk),
            ("q4_k_min", Q4_K, q4k_min, expk_min)]


def random_blocks(rng, wtype, nblocks):
    el, nb = po.BLOCK[wtype]
    raw = rng.integers(0, 256, size=(nblocks, nb), dtype=np.uint8)
    # finite fp16 scales: random magnitude in [2^-14, 2^3], random sign
    nscale = 2 if wtype == Q4_K else 1
    for s in range(nscale):
        v = (rng.uniform(-14, 3, nblocks)).astype(np.float64)
        h = (np.exp2(v) * rng.choice([-1, 1], nblocks)).astype(np.float16).view(np.uint8)
        raw[:, 2 * s:2 * s + 2] = h.reshape(nblocks, 2)
    return raw.ravel()


def ref_dequant(R, wtype, blocks, numel):
    out = np.empty(numel, np.float32)
    assert R.pai_refshim_dequant(wtype, np.ascontiguousarray(blocks, np.uint8), out, numel) == 0
    return out


def ref_gemv(R, wtype, n, k, blocks, x):
    w = ref_dequant(R, wtype, blocks, n * k)
    y = np.empty(n, np.float32)
    assert R.pai_ref_gemv_f32(n, k, w, np.ascontiguousarray(x, np.float32), y) == 0
    return y


def main():
    po.build()
    R = po.ref()
    if R is None:
        sys.exit("oracle/_ref/libpai_ref.so is missing: build it from the reference first")
    rng = np.random.default_rng(20261201)
    g = {}

    # dequant known answers + reference output for the same bytes
    for name, t, raw, expect in known_blocks():
        b = np.frombuffer(raw, np.uint8).copy()
        g[f"dq_known_{name}_blocks"] = b
        g[f"dq_known_{name}_expect"] = expect
        g[f"dq_known_{name}_ref"] = ref_dequant(R, t, b, expect.size)

    # dequant of seeded random blocks
    for name, t in (("q4_0", Q4_0), ("q8_0", Q8_0), ("q4_k", Q4_K)):
        b = random_blocks(rng, t, 64)
        g[f"dq_rand_{name}_blocks"] = b
        g[f"dq_rand_{name}_ref"] = ref_dequant(R, t, b, 64 * po.BLOCK[t][0])

    # quantised GEMV on quantiser output (N(0,0.02) weights, N(0,1) x)
    for name, t, n, k in (("q4_0", Q4_0, 64, 256), ("q8_0", Q8_0, 64, 256), ("q4_k", Q4_K, 64, 256)):
        w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
        blocks = po.quantize(t, w)
        x = rng.standard_normal(k).astype(np.float32)
        g[f"gemv_{name}_blocks"] = blocks
        g[f"gemv_{name}_x"] = x
        g[f"gemv_{name}_ref"] = ref_gemv(R, t, n, k, blocks, x)

    # rmsnorm: ref_ops test (a = 1..4, unit gain) and a 4096 row with gains
    a4 = np.array([1, 2, 3, 4], np.float32)
    o = np.empty(4, np.float32)
    R.pai_ref_rmsnorm_gamma_f32(a4, o, 4, np.ones(4, np.float32), 0.0)
    g["rms_small_a"], g["rms_small_ref"] = a4, o
    a = rng.standard_normal(4096).astype(np.float32)
    gam = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
    o = np.empty(4096, np.float32)
    R.pai_ref_rmsnorm_gamma_f32(a, o, 4096, gam, 1e-5)
    g["rms_a"], g["rms_gamma"], g["rms_ref"] = a, gam, o

    # rope: ref_ops test (ctx 2, r2 2, base 1e4, x = 1,3,2,4,10,30,20,40) + LLaMA-shaped case
    c = np.empty(4, np.float32)
    s = np.empty(4, np.float32)
    R.pai_ref_rope_cossin_f32(2, 2, 10000.0, c, s)
    x2 = np.array([1, 3, 2, 4, 10, 30, 20, 40], np.float32)
    o = np.empty(8, np.float32)
    R.pai_ref_rope_f32(x2, 2, 4, 2, 1, c, s, 2, o)
    g["rope_small_cos"], g["rope_small_sin"], g["rope_small_x"], g["rope_small_ref"] = c, s, x2, o
    ctx, r2, heads, seq = 64, 64, 4, 5
    c = np.empty(ctx * r2, np.float32)
    s = np.empty(ctx * r2, np.float32)
    R.pai_ref_rope_cossin_f32(ctx, r2, 500000.0, c, s)
    xr = rng.standard_normal(seq * heads * 128).astype(np.float32)
    o = np.empty_like(xr)
    R.pai_ref_rope_f32(xr, seq * heads, 128, seq, heads, c, s, r2, o)
    g["rope_cos"], g["rope_sin"], g["rope_x"], g["rope_ref"] = c, s, xr, o

    # attention: ref_ops MHA case (test_ref_ops.c:327-351) and a GQA case
    q = np.array([1, 2, 0, 0, 3, 0, 1, 0, 2, 1, 0, 0, 0, 4, 0, 1], np.float32)
    k = np.array([1, 0, 0, 0, 0, 2, 0, 0, 0, 1, 0, 0, 1, 0, 0, 0], np.float32)
    v = np.arange(1, 17, dtype=np.float32)
    o = np.empty(16, np.float32)
    R.pai_ref_attention_f32(2, 2, 2, 4, q, k, v, o)
    g["attn_small_q"], g["attn_small_k"], g["attn_small_v"], g["attn_small_ref"] = q, k, v, o
    h, hk, seq, hd = 8, 2, 9, 128
    q = rng.standard_normal(seq * h * hd).astype(np.float32)
    k = rng.standard_normal(seq * hk * hd).astype(np.float32)
    v = rng.standard_normal(seq * hk * hd).astype(np.float32)
    o = np.empty_like(q)
    R.pai_ref_attention_f32(h, hk, seq, hd, q, k, v, o)
    g["attn_q"], g["attn_k"], g["attn_v"], g["attn_ref"] = q, k, v, o

    # silu * up
    gt = (rng.standard_normal(2048) * 3).astype(np.float32)
    up = rng.standard_normal(2048).astype(np.float32)
    sg = np.empty_like(gt)
    R.pai_ref_silu_f32(gt, sg, gt.size)
    hh = np.empty_like(gt)
    R.pai_ref_vecmul_f32(sg, up, hh, gt.size)
    g["silu_gate"], g["silu_up"], g["silu_ref"] = gt, up, hh

    # greedy sampler with a tie: first index of the maximum (sampler.c:89-99)
    lg = rng.standard_normal(1000).astype(np.float32)
    lg[[17, 400, 999]] = lg.max() + 1.0

    class Sampler(C.Structure):
        _fields_ = [("seed", C.c_uint64), ("temperature", C.c_float), ("top_k", C.c_uint32),
                    ("top_p", C.c_float)]

    smp = Sampler(1, 0.0, 0, 1.0)
    tok = C.c_uint32()
    assert R.pai_sampler_sample_logits(C.byref(smp), lg, lg.size, C.byref(tok)) == 0
    g["argmax_logits"], g["argmax_ref"] = lg, np.array([tok.value], np.int64)

    path = os.path.join(OUT, "golden.npz")
    np.savez_compressed(path, **g)
    print(f"wrote {path}: {len(g)} arrays, {os.path.getsize(path)} bytes")

    v0 = v0_cases(R)
    path = os.path.join(OUT, "golden_v0.npz")
    np.savez_compressed(path, **v0)
    print(f"wrote {path}: {len(v0)} arrays, {os.path.getsize(path)} bytes")


def ref_quant_v0(R, bits, gs, w):
    """pai_quantize_f32 (models/quantize.c:74-143) on w: (values, scales)."""
    w = np.ascontiguousarray(w, np.float32).ravel()
    sch = po.QuantScheme(bits, 1, gs)
    q = np.empty(po.v0_value_bytes(bits, w.size), np.int8)
    s = np.empty(po.v0_groups(w.size, gs), np.float32)
    ng = po.U64()
    assert R.pai_quantize_f32(w, w.size, C.byref(sch), q, s, C.byref(ng)) == 0
    assert ng.value == s.size
    return q, s


def per_column_quant(R, bits, gs, w, k, n):
    """The reference test's per-column quantisation of a [k][n] weight with
    the scales scattered to [k/g][n] (tests/test_quantize.c:155-180,
    201-230): what pai_ref_gemm_w8_f32 / _w4_f32 take."""
    g = k if gs == 0 else gs
    ng = (k + g - 1) // g
    vals = np.zeros((k, n), np.int32)
    scales = np.empty((ng, n), np.float32)
    for j in range(n):
        q, sc = ref_quant_v0(R, bits, gs, w[:, j])
        if bits == 8:
            vals[:, j] = q
        else:
            b = q.view(np.uint8).astype(np.int32)
            nib = np.stack([b & 15, b >> 4], 1).ravel()[:k]
            vals[:, j] = np.where(nib & 8, nib - 16, nib)
        scales[:, j] = sc
    flat = vals.ravel()
    if bits == 8:
        packed = flat.astype(np.int8)
    else:
        nib = (flat & 15).astype(np.uint8)
        if nib.size % 2:
            nib = np.append(nib, 0)
        packed = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8).view(np.int8)
    return packed, scales


def v0_cases(R):
    """v0 grouped-scale formats. (a) the registered w8/w4 GEMMs on the
    reference test's shapes (tests/test_quantize.c:135-271: m 3, n 5, k 8,
    group 4 and per-tensor) and on a larger ragged shape; (b) .pai blobs
    ([values][scales] of pai_quantize_f32 over the flat [k][n] tensor) with
    the reference's dequantise-then-GEMM result (models/model.c:259-290,
    ref_ops.c:428-444), including an odd element count whose scales start
    at an unaligned offset."""
    rng = np.random.default_rng(20261202)
    g = {}
    for name, bits, (m, n, k), gs in (("w8_g4", 8, (3, 5, 8), 4), ("w4_g4", 4, (3, 5, 8), 4),
                                      ("w8_g0", 8, (3, 5, 8), 0), ("w8_g32", 8, (4, 37, 96), 32),
                                      ("w4_g32", 4, (4, 37, 96), 32), ("w4_g0", 4, (2, 24, 40), 0)):
        a = rng.standard_normal((m, k)).astype(np.float32)
        w = rng.standard_normal((k, n)).astype(np.float32)
        wq, sc = per_column_quant(R, bits, gs, w, k, n)
        c = np.empty(m * n, np.float32)
        fn = R.pai_ref_gemm_w8_f32 if bits == 8 else R.pai_ref_gemm_w4_f32
        assert fn(m, n, k, a, wq, sc, gs, c) == 0
        g[f"{name}_shape"] = np.array([m, n, k, gs], np.int64)
        g[f"{name}_a"], g[f"{name}_wq"], g[f"{name}_scales"], g[f"{name}_ref"] = a, wq, sc.ravel(), c
    for name, bits, (m, n, k), gs in (("pai8_g32", 8, (1, 48, 64), 32), ("pai4_g32", 4, (2, 48, 64), 32),
                                      ("pai8_g0", 8, (3, 40, 24), 0), ("pai4_g12", 4, (1, 20, 30), 12),
                                      ("pai4_odd", 4, (2, 5, 7), 3)):
        a = rng.standard_normal((m, k)).astype(np.float32)
        w = (rng.standard_normal((k, n)) * 0.05).astype(np.float32)
        q, sc = ref_quant_v0(R, bits, gs, w)
        deq = np.empty(k * n, np.float32)
        assert R.pai_dequantize_f32(q, sc, k * n, C.byref(po.QuantScheme(bits, 1, gs)), deq) == 0
        c = np.empty(m * n, np.float32)
        assert R.pai_ref_gemm_f32(m, n, k, a, deq, c) == 0
        g[f"{name}_shape"] = np.array([m, n, k, gs, bits], np.int64)
        g[f"{name}_a"], g[f"{name}_w"] = a, w
        g[f"{name}_blob"] = np.concatenate([q.view(np.uint8), sc.view(np.uint8)])
        g[f"{name}_deq"], g[f"{name}_ref"] = deq, c
    return g


if __name__ == "__main__":
    main()
