"""GPU parity of every hot-path op against the CPU restatement (oracle/).

Bars: bit-exact for dequantisation, embedding rows, RMSNorm, RoPE, the
residual add and argmax (the same IEEE operations in the same order);
max-abs-rel error <= 1e-3 for the fp32-accumulated GEMVs and attention,
where max-abs-rel = max|gpu - ref| / max|ref| over the output.
"""
import os

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200.api import PackedMatrix, quantize

pytestmark = pytest.mark.gpu

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
TYPES = {"q4_0": po.Q4_0, "q8_0": po.Q8_0, "q4_k": po.Q4_K}
TOL = 1e-3


def maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_bit_exact_against_golden(dev, name):
    t = TYPES[name]
    el = po.BLOCK[t][0]
    for key in (f"dq_rand_{name}", f"dq_known_{name}"):
        blocks = G[f"{key}_blocks"]
        ref = G[f"{key}_ref"]
        n = ref.size // el
        w = PackedMatrix(dev, t, n, el, blocks)
        out = dev.alloc(ref.nbytes)
        dev.dequant(w, out)
        assert np.array_equal(bits(out.download(np.float32)), bits(ref)), key


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("n,k", [(64, 256), (4096, 4096), (1000, 2048), (4128, 1024)])
def test_dequant_bit_exact_quantiser_output(dev, name, n, k):
    t = TYPES[name]
    rng = np.random.default_rng(n + k)
    blocks = quantize(t, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    w = PackedMatrix(dev, t, n, k, blocks)
    out = dev.alloc(n * k * 4)
    dev.dequant(w, out)
    assert np.array_equal(bits(out.download(np.float32)), bits(po.dequant(t, blocks, n * k)))


@pytest.mark.parametrize("name", list(TYPES))
def test_gemv_golden(dev, name):
    t = TYPES[name]
    ref = G[f"gemv_{name}_ref"]
    x = G[f"gemv_{name}_x"]
    w = PackedMatrix(dev, t, ref.size, x.size, G[f"gemv_{name}_blocks"])
    y = dev.alloc(ref.nbytes)
    dev.gemv(w, dev.put(x), y)
    assert maxrel(y.download(np.float32), ref) <= TOL


# The benchmark shapes (Q8_0 4096^2; Q4_K sweep; Q4_0 layer matrices) plus
# ragged row counts and short K that exercise the split-K and padding paths.
SHAPES = [
    (po.Q8_0, 4096, 4096), (po.Q4_K, 4096, 4096), (po.Q4_K, 1024, 4096),
    (po.Q4_K, 14336, 4096), (po.Q4_K, 4096, 14336), (po.Q4_0, 14336, 4096),
    (po.Q4_0, 4096, 14336), (po.Q4_0, 6144, 4096), (po.Q4_0, 1, 32), (po.Q4_0, 33, 64),
    (po.Q8_0, 1000, 512), (po.Q4_K, 7, 256), (po.Q8_0, 16032, 4096),
]


@pytest.mark.parametrize("t,n,k", SHAPES)
def test_gemv_against_oracle(dev, t, n, k):
    rng = np.random.default_rng(n * 7 + k)
    blocks = quantize(t, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal(k).astype(np.float32)
    w = PackedMatrix(dev, t, n, k, blocks)
    y = dev.alloc(n * 4)
    dev.gemv(w, dev.put(x), y)
    got = y.download(np.float32)
    ref = po.gemv_q(t, n, k, blocks, x, threads=8)
    assert maxrel(got, ref) <= TOL
    # second launch reuses the split-K counters: identical result
    dev.gemv(w, dev.put(x), y)
    assert np.array_equal(bits(y.download(np.float32)), bits(got))


@pytest.mark.parametrize("t", [po.Q4_0, po.Q8_0, po.Q4_K])
@pytest.mark.parametrize("batch", [2, 4, 8])
def test_gemv_batched_with_residual(dev, t, batch):
    n, k = 2048, 4096
    rng = np.random.default_rng(batch)
    blocks = quantize(t, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((batch, k)).astype(np.float32)
    res = rng.standard_normal((batch, n)).astype(np.float32)
    w = PackedMatrix(dev, t, n, k, blocks)
    y = dev.put(res)
    dev.gemv(w, dev.put(x), y, batch=batch, residual=y)
    got = y.download(np.float32).reshape(batch, n)
    for b in range(batch):
        ref = res[b] + po.gemv_q(t, n, k, blocks, x[b])
        assert maxrel(got[b], ref) <= TOL


@pytest.mark.parametrize("t", [po.Q4_0, po.Q8_0, po.Q4_K])
@pytest.mark.parametrize("batch", [1, 3])
def test_gemv_prepared_equals_gemv(dev, t, batch):
    """x prepared once and reused by several matrices gives gemv's bits."""
    rng = np.random.default_rng(40 + batch)
    k = 4096
    x = dev.put(rng.standard_normal((batch, k)).astype(np.float32))
    xq = dev.prepare_x(x, k, batch)
    for n in (4096, 1040):
        blocks = quantize(t, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
        w = PackedMatrix(dev, t, n, k, blocks)
        res = dev.put(rng.standard_normal((batch, n)).astype(np.float32))
        y0, y1 = dev.alloc(batch * n * 4), dev.alloc(batch * n * 4)
        dev.gemv(w, x, y0, batch=batch, residual=res)
        dev.gemv_prepared(w, xq, y1, batch=batch, residual=res)
        assert np.array_equal(bits(y0.download(np.float32)), bits(y1.download(np.float32)))


@pytest.mark.parametrize("t", [po.Q4_0, po.Q8_0, po.Q4_K])
@pytest.mark.parametrize("batch,k", [(1, 4096), (3, 2048), (8, 4096)])
def test_gemv_rmsnorm_against_oracle(dev, t, batch, k):
    """RMSNorm computed inside the GEMV: the oracle's rmsnorm_gamma then gemv."""
    rng = np.random.default_rng(7 * batch + k)
    n = 1552  # not a multiple of the 128-row group
    blocks = quantize(t, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = (rng.standard_normal((batch, k)) * 3.0).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    res = rng.standard_normal((batch, n)).astype(np.float32)
    w = PackedMatrix(dev, t, n, k, blocks)
    y = dev.alloc(batch * n * 4)
    dev.gemv_rmsnorm(w, dev.put(x), dev.put(gamma), 1e-5, y, batch=batch, residual=dev.put(res))
    got = y.download(np.float32).reshape(batch, n)
    for b in range(batch):
        xn = po.rmsnorm_gamma(x[b][None, :], gamma, 1e-5).reshape(k)
        ref = res[b] + po.gemv_q(t, n, k, blocks, xn)
        assert maxrel(got[b], ref) <= TOL


def test_gemv_rejects_bad_shapes(dev):
    from prosperoai_b200 import PaiError
    blocks = quantize(po.Q4_K, np.zeros(256 * 4, np.float32))
    w = PackedMatrix(dev, po.Q4_K, 4, 256, blocks)
    w.k = 300  # not a whole number of super-blocks
    with pytest.raises(PaiError) as e:
        dev.gemv(w, dev.put(np.zeros(300, np.float32)), dev.alloc(16))
    assert e.value.status == -6


def test_rmsnorm_bit_exact(dev):
    a, gam, ref = G["rms_a"], G["rms_gamma"], G["rms_ref"]
    c = dev.alloc(a.nbytes)
    dev.rmsnorm_gamma(1, a.size, dev.put(a), dev.put(gam), 1e-5, c)
    assert np.array_equal(bits(c.download(np.float32)), bits(ref))
    rng = np.random.default_rng(2)
    rows = rng.standard_normal((8, 4096)).astype(np.float32) * 3
    c = dev.alloc(rows.nbytes)
    dev.rmsnorm_gamma(8, 4096, dev.put(rows), dev.put(np.ones(4096, np.float32)), 0.0, c)
    got = c.download(np.float32).reshape(8, 4096)
    ref = po.rmsnorm_gamma(rows, np.ones(4096, np.float32), 1e-5)
    assert np.array_equal(bits(got), bits(ref))


def test_rope_bit_exact(dev):
    c, s = G["rope_cos"], G["rope_sin"]
    x = G["rope_x"]
    out = dev.alloc(x.nbytes)
    dev.rope(dev.put(x), x.size // 128, 128, 5, 4, dev.put(c), dev.put(s), 64, out)
    assert np.array_equal(bits(out.download(np.float32)), bits(G["rope_ref"]))
    x2 = G["rope_small_x"]
    out = dev.alloc(x2.nbytes)
    dev.rope(dev.put(x2), 2, 4, 2, 1, dev.put(G["rope_small_cos"]), dev.put(G["rope_small_sin"]), 2, out)
    assert np.array_equal(bits(out.download(np.float32)), bits(G["rope_small_ref"]))


def test_silu_mul_and_vecadd(dev):
    g, u = G["silu_gate"], G["silu_up"]
    out = dev.alloc(g.nbytes)
    dev.silu_mul(dev.put(g), dev.put(u), out, g.size)
    got = out.download(np.float32)
    ref = G["silu_ref"]
    # expf may differ from glibc's in the last bit
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)) <= 1e-6
    a = np.random.default_rng(0).standard_normal(10001).astype(np.float32)
    out = dev.alloc(a.nbytes)
    dev.vecadd(dev.put(a), dev.put(a[::-1].copy()), out, a.size)
    assert np.array_equal(out.download(np.float32), a + a[::-1])


def test_attention_prefill(dev):
    for tag, (h, hk, seq, hd) in (("attn_small", (2, 2, 2, 4)), ("attn", (8, 2, 9, 128))):
        q, k, v = G[f"{tag}_q"], G[f"{tag}_k"], G[f"{tag}_v"]
        out = dev.alloc(q.nbytes)
        dev.attention(h, hk, seq, hd, dev.put(q), dev.put(k), dev.put(v), out)
        assert maxrel(out.download(np.float32), G[f"{tag}_ref"]) <= 1e-5


@pytest.mark.parametrize("h,hk,npos", [(32, 8, 1), (32, 8, 37), (32, 8, 4097), (8, 8, 300), (16, 2, 1000)])
def test_attn_decode_f16kv(dev, h, hk, npos):
    rng = np.random.default_rng(npos)
    hd, cap = 128, npos + 5
    q = rng.standard_normal((h, hd)).astype(np.float32)
    kc = rng.standard_normal((hk, cap, hd)).astype(np.float16)
    vc = rng.standard_normal((hk, cap, hd)).astype(np.float16)
    out = dev.alloc(q.nbytes)
    dev.attn_decode_f16kv(h, hk, hd, npos, cap, dev.put(q), dev.put(kc), dev.put(vc), out)
    ref = po.attention_decode_f16(h, hk, hd, npos, cap, q, kc.view(np.uint16), vc.view(np.uint16))
    assert maxrel(out.download(np.float32), ref) <= TOL


def test_argmax_first_of_ties(dev):
    lg = G["argmax_logits"]
    rows = np.stack([lg, lg[::-1], np.full(lg.size, -3.0, np.float32)])
    out = dev.alloc(12)
    dev.argmax(3, lg.size, dev.put(rows), out)
    got = out.download(np.int32)
    assert list(got) == [int(G["argmax_ref"][0]), po.argmax(lg[::-1].copy()), 0]
    big = np.random.default_rng(9).standard_normal(128256).astype(np.float32)
    out = dev.alloc(4)
    dev.argmax(1, big.size, dev.put(big), out)
    assert out.download(np.int32)[0] == po.argmax(big)
    # equal maxima in different slices of the multi-CTA scan: the first wins,
    # and a repeat call (counters left at zero) agrees
    tie = big.copy()
    tie[[70001, 3003, 128255]] = 9.0
    out = dev.alloc(8)
    rows2 = np.stack([tie, tie[::-1].copy()])
    for _ in range(2):
        dev.argmax(2, tie.size, dev.put(rows2), out)
        assert list(out.download(np.int32)) == [3003, po.argmax(tie[::-1].copy())]
