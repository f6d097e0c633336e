"""Pin the CPU restatement (oracle/) to the reference's own outputs.

Fixtures in tests/golden/golden.npz were produced by the reference code
itself (tests/golden/make_golden.py); the restatement must reproduce
them bit for bit. When the reference build (oracle/_ref) is present the
same comparison also runs live on fresh seeded inputs.
"""
import os

import numpy as np
import pytest

from oracle import py_oracle as po

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
TYPES = {"q4_0": po.Q4_0, "q8_0": po.Q8_0, "q4_k": po.Q4_K}


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("name,t", [("q8_0", po.Q8_0), ("q4_0", po.Q4_0), ("q4_k", po.Q4_K),
                                    ("q4_k_min", po.Q4_K)])
def test_dequant_known_answers(name, t):
    blocks = G[f"dq_known_{name}_blocks"]
    expect = G[f"dq_known_{name}_expect"]
    got = po.dequant(t, blocks, expect.size)
    assert same_bits(got, G[f"dq_known_{name}_ref"])
    np.testing.assert_array_equal(got, expect)  # the hand-computed values of the reference tests


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_random_blocks(name):
    t = TYPES[name]
    ref = G[f"dq_rand_{name}_ref"]
    assert same_bits(po.dequant(t, G[f"dq_rand_{name}_blocks"], ref.size), ref)


@pytest.mark.parametrize("name", list(TYPES))
def test_gemv_matches_reference(name):
    t = TYPES[name]
    ref = G[f"gemv_{name}_ref"]
    x = G[f"gemv_{name}_x"]
    got = po.gemv_q(t, ref.size, x.size, G[f"gemv_{name}_blocks"], x, threads=3)
    assert same_bits(got, ref)


def test_rmsnorm_matches_reference():
    a = G["rms_small_a"]
    assert same_bits(po.rmsnorm_gamma(a, np.ones_like(a), 0.0), G["rms_small_ref"])
    assert same_bits(po.rmsnorm_gamma(G["rms_a"], G["rms_gamma"], 1e-5), G["rms_ref"])


def test_rope_matches_reference():
    c, s = po.rope_tables(2, 2, 10000.0)
    assert same_bits(c, G["rope_small_cos"]) and same_bits(s, G["rope_small_sin"])
    out = po.rope(G["rope_small_x"], 1, 4, c, s, 2)
    assert same_bits(out, G["rope_small_ref"])
    c, s = po.rope_tables(64, 64, 500000.0)
    assert same_bits(c, G["rope_cos"]) and same_bits(s, G["rope_sin"])
    assert same_bits(po.rope(G["rope_x"], 4, 128, c, s, 64), G["rope_ref"])


def test_attention_matches_reference():
    out = po.attention(2, 2, 2, 4, G["attn_small_q"], G["attn_small_k"], G["attn_small_v"])
    assert same_bits(out, G["attn_small_ref"])
    out = po.attention(8, 2, 9, 128, G["attn_q"], G["attn_k"], G["attn_v"])
    assert same_bits(out, G["attn_ref"])


def test_decode_attention_is_the_last_row():
    """The fp16-cache decode restatement equals the last row of the full
    reference attention when k/v are fp16-exact."""
    rng = np.random.default_rng(5)
    h, hk, seq, hd, cap = 8, 2, 13, 128, 16
    q = rng.standard_normal((seq, h, hd)).astype(np.float32)
    k = rng.standard_normal((seq, hk, hd)).astype(np.float16)
    v = rng.standard_normal((seq, hk, hd)).astype(np.float16)
    full = po.attention(h, hk, seq, hd, q, k.astype(np.float32), v.astype(np.float32))
    kc = np.zeros((hk, cap, hd), np.float16)
    vc = np.zeros((hk, cap, hd), np.float16)
    kc[:, :seq] = k.transpose(1, 0, 2)
    vc[:, :seq] = v.transpose(1, 0, 2)
    last = po.attention_decode_f16(h, hk, hd, seq, cap, q[-1], kc.view(np.uint16),
                                   vc.view(np.uint16))
    assert same_bits(last, full.reshape(seq, h * hd)[-1])


def test_silu_mul_matches_reference():
    assert same_bits(po.silu_mul(G["silu_gate"], G["silu_up"]), G["silu_ref"])


def test_argmax_first_of_ties():
    assert po.argmax(G["argmax_logits"]) == int(G["argmax_ref"][0]) == 17


def test_f16_conversion_matches_ieee():
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.standard_normal(2000) * 10, rng.standard_normal(500) * 1e-5,
                        [0.0, -0.0, 65504.0, 65520.0, 1e6, 6e-8, 3e-8, 2.98e-8]]).astype(np.float32)
    assert np.array_equal(po.f32_to_f16_bits(v), v.astype(np.float16).view(np.uint16))
    bits = np.arange(0, 65536, 97, dtype=np.uint16)
    bits = bits[(bits & 0x7C00) != 0x7C00]
    got = np.array([po.lib().po_f16_to_f32(int(b)) for b in bits], np.float32)
    assert same_bits(got, bits.view(np.float16).astype(np.float32))


ref = po.ref()


@pytest.mark.skipif(ref is None, reason="reference build oracle/_ref not present")
@pytest.mark.parametrize("name", list(TYPES))
def test_live_dequant_and_gemv_against_reference(name):
    t = TYPES[name]
    rng = np.random.default_rng(hash(name) & 0xFFFF)
    el, nb = po.BLOCK[t]
    n, k = 37, el * 6
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    blocks = po.quantize(t, w)
    x = rng.standard_normal(k).astype(np.float32)
    dq = np.empty(n * k, np.float32)
    assert ref.pai_refshim_dequant(t, blocks, dq, n * k) == 0
    assert same_bits(po.dequant(t, blocks, n * k), dq)
    y = np.empty(n, np.float32)
    ref.pai_ref_gemv_f32(n, k, dq, x, y)
    assert same_bits(po.gemv_q(t, n, k, blocks, x, threads=4), y)


@pytest.mark.skipif(ref is None, reason="reference build oracle/_ref not present")
def test_live_q8_0_maps_onto_reference_w8_gemm():
    """Q8_0 is exactly the reference's gemm_w8 with group 32 and
    b_scales = (float)d (cpu/reference/ref_ops.c:447-468)."""
    rng = np.random.default_rng(8)
    n, k = 24, 128
    blocks = po.quantize(po.Q8_0, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    b = blocks.reshape(n, k // 32, 34)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32).reshape(n, k // 32)
    q = b[:, :, 2:].copy().view(np.int8).reshape(n, k)
    wq = np.ascontiguousarray(q.T)                   # [k][n]
    sc = np.ascontiguousarray(d.T)                   # [k/32][n]
    x = rng.standard_normal(k).astype(np.float32)
    c = np.empty(n, np.float32)
    assert ref.pai_ref_gemm_w8_f32(1, n, k, x, wq, sc, 32, c) == 0
    np.testing.assert_allclose(c, po.gemv_q(po.Q8_0, n, k, blocks, x), rtol=1e-5, atol=1e-6)


# ---- v0 grouped-scale formats (models/quantize.c, ref_ops.c:447-499) ------------------

V0 = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_v0.npz"))
WQ_CASES = ["w8_g4", "w4_g4", "w8_g0", "w8_g32", "w4_g32", "w4_g0"]
PAI_CASES = ["pai8_g32", "pai4_g32", "pai8_g0", "pai4_g12", "pai4_odd"]


@pytest.mark.parametrize("name", WQ_CASES)
def test_gemm_wq_matches_reference(name):
    m, n, k, gs = (int(v) for v in V0[f"{name}_shape"])
    bits = 8 if name.startswith("w8") else 4
    got = po.gemm_wq(bits, m, n, k, V0[f"{name}_a"], V0[f"{name}_wq"], V0[f"{name}_scales"], gs)
    assert same_bits(got.ravel(), V0[f"{name}_ref"])


@pytest.mark.parametrize("name", PAI_CASES)
def test_v0_blob_quantise_dequantise_gemm_match_reference(name):
    m, n, k, gs, bits = (int(v) for v in V0[f"{name}_shape"])
    q, s = po.quant_v0(bits, gs, V0[f"{name}_w"])
    blob = V0[f"{name}_blob"]
    assert np.array_equal(np.concatenate([q.view(np.uint8), s.view(np.uint8)]), blob)
    deq = po.dequant_v0(bits, gs, q, s, n * k)
    assert same_bits(deq, V0[f"{name}_deq"])
    assert same_bits(po.gemm_f32(m, n, k, V0[f"{name}_a"], deq).ravel(), V0[f"{name}_ref"])


def test_v0_known_answers():
    """The reference's own round-trip cases (tests/test_quantize.c:62-116)."""
    rng = np.random.default_rng(5)
    src = rng.uniform(-1, 1, 256).astype(np.float32)
    q, s = po.quant_v0(8, 64, src)
    assert s.size == 4 and np.abs(po.dequant_v0(8, 64, q, s, 256) - src).max() < 0.02
    exact = np.array([0, 100, -100, 100], np.float32)
    q, s = po.quant_v0(8, 0, exact)
    assert np.abs(po.dequant_v0(8, 0, q, s, 4) - exact).max() < 1e-4
    exact = np.array([0, 2, -2, 1], np.float32)
    q, s = po.quant_v0(4, 0, exact)
    d = po.dequant_v0(4, 0, q, s, 4)
    assert q.size == 2 and np.abs(d[:3] - exact[:3]).max() < 1e-4 and abs(d[3] - 1) < 0.2
    odd = np.array([4, -4, 4], np.float32)
    q, s = po.quant_v0(4, 0, odd)
    assert q.size == 2 and np.abs(po.dequant_v0(4, 0, q, s, 3) - odd).max() < 1e-4
    assert q.view(np.uint8)[1] >> 4 == 0  # the padding nibble stays zero


@pytest.mark.skipif(po.ref() is None, reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("bits,gs", [(8, 0), (8, 7), (4, 32), (4, 5)])
def test_v0_live_against_reference(bits, gs):
    import ctypes as C
    R = po.ref()
    rng = np.random.default_rng(bits * 100 + gs)
    w = (rng.standard_normal(777) * 0.1).astype(np.float32)
    q, s = po.quant_v0(bits, gs, w)
    q2, s2 = np.empty_like(q), np.empty_like(s)
    ng = po.U64()
    sch = po.QuantScheme(bits, 1, gs)
    assert R.pai_quantize_f32(w, w.size, C.byref(sch), q2, s2, C.byref(ng)) == 0
    assert np.array_equal(q, q2) and same_bits(s, s2)
    m, n, k = 2, 21, 37
    a = rng.standard_normal(m * k).astype(np.float32)
    g = gs or k
    wq = rng.integers(-128, 128, n * k if bits == 8 else (n * k + 1) // 2).astype(np.int8)
    sc = rng.standard_normal((k + g - 1) // g * n).astype(np.float32)
    c2 = np.empty(m * n, np.float32)
    fn = R.pai_ref_gemm_w8_f32 if bits == 8 else R.pai_ref_gemm_w4_f32
    assert fn(m, n, k, a, wq, sc, gs, c2) == 0
    assert same_bits(po.gemm_wq(bits, m, n, k, a, wq, sc, gs).ravel(), c2)
