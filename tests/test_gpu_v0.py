"""GPU parity of the v0 grouped-scale GEMMs (csrc/kernels/k_v0.cu).

- pai_b200_gemm_w8_f32 / _w4_f32 against the reference's own
  pai_ref_gemm_w8_f32 / _w4_f32 outputs (tests/golden/golden_v0.npz, the
  reference test's shapes included) and against the oracle restatement at
  sizes that take the vector path (several k-splits, 1 to 11 rows);
- pai_b200_gemm_v0_f32 on .pai blobs against the reference's
  dequantise-then-GEMM result, including per-tensor scales, groups that are
  not a multiple of 8, an odd element count (scales at an unaligned offset)
  and a blob at an unaligned address;
- repeated calls are bit-identical; bad arguments give the reference's codes.

Bar: max|gpu - ref| / max|ref| <= 1e-4 (fp32 accumulation in a different
order; the products carry the same two roundings as the reference's).
"""
import os

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import _native

pytestmark = pytest.mark.gpu

TOL = 1e-4
V0 = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_v0.npz"))


def maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def run_wq(dev, bits, m, n, k, a, wq, sc, gs):
    c = dev.alloc(m * n * 4)
    dev.gemm_wq(bits, m, n, k, dev.put(a), dev.put(wq), dev.put(sc), gs, c)
    return c.download(np.float32).reshape(m, n)


def run_v0(dev, bits, gs, m, n, k, a, blob, offset=0):
    buf = dev.alloc(blob.nbytes + 64)
    if offset:
        buf.upload(np.concatenate([np.zeros(offset, np.uint8), blob]))
    else:
        buf.upload(blob)
    c = dev.alloc(m * n * 4)
    dev.gemm_v0(bits, gs, m, n, k, dev.put(a), buf, c, blob_offset=offset)
    return c.download(np.float32).reshape(m, n)


@pytest.mark.parametrize("name", ["w8_g4", "w4_g4", "w8_g0", "w8_g32", "w4_g32", "w4_g0"])
def test_gemm_wq_golden(dev, name):
    m, n, k, gs = (int(v) for v in V0[f"{name}_shape"])
    bits = 8 if name.startswith("w8") else 4
    got = run_wq(dev, bits, m, n, k, V0[f"{name}_a"], V0[f"{name}_wq"], V0[f"{name}_scales"], gs)
    assert maxrel(got.ravel(), V0[f"{name}_ref"]) <= TOL


@pytest.mark.parametrize("name", ["pai8_g32", "pai4_g32", "pai8_g0", "pai4_g12", "pai4_odd"])
@pytest.mark.parametrize("offset", [0, 4])
def test_gemm_v0_golden(dev, name, offset):
    m, n, k, gs, bits = (int(v) for v in V0[f"{name}_shape"])
    got = run_v0(dev, bits, gs, m, n, k, V0[f"{name}_a"], V0[f"{name}_blob"], offset)
    assert maxrel(got.ravel(), V0[f"{name}_ref"]) <= TOL


def random_wq(rng, bits, n, k, gs):
    g = k if gs == 0 or gs > k else gs
    nbytes = n * k if bits == 8 else (n * k + 1) // 2
    wq = rng.integers(-128, 128, nbytes).astype(np.int8)
    sc = (rng.uniform(0.5, 1.5, (k + g - 1) // g * n) / 127).astype(np.float32)
    return wq, sc


@pytest.mark.parametrize("bits,m,n,k,gs", [
    (8, 1, 4096, 4096, 32),    # config-1 shape: wide strips, 74 k-splits per strip
    (8, 2, 2560, 1000, 32),    # wide: a partial second strip, ragged last split
    (4, 8, 4096, 512, 16),     # wide, nibbles, 8 rows, split length one box
    (4, 3, 1024, 2048, 64),
    (8, 11, 512, 256, 0),      # two row passes (8 + 3), one group over k
    (4, 8, 264, 1000, 100),    # ragged strip and split ends
    (8, 1, 262144, 64, 16),    # one split: results stored directly
    (4, 2, 37, 300, 7),        # n % 8 != 0: element-wise path
])
def test_gemm_wq_against_oracle(dev, bits, m, n, k, gs):
    rng = np.random.default_rng(bits + m + n + k + gs)
    a = rng.standard_normal((m, k)).astype(np.float32)
    wq, sc = random_wq(rng, bits, n, k, gs)
    got = run_wq(dev, bits, m, n, k, a, wq, sc, gs)
    want = po.gemm_wq(bits, m, n, k, a, wq, sc, gs)
    assert maxrel(got, want) <= TOL
    again = run_wq(dev, bits, m, n, k, a, wq, sc, gs)
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))


@pytest.mark.parametrize("bits,m,n,k,gs", [
    (8, 1, 4096, 4096, 32),    # a q8 .pai tensor of the config-1 shape
    (4, 1, 4096, 4096, 32),
    (4, 2, 2048, 1024, 0),     # per-tensor scale
    (8, 5, 1024, 520, 4096),   # groups spanning rows
    (4, 1, 64, 64, 12),        # groups not a multiple of 8: element-wise path
])
def test_gemm_v0_against_oracle(dev, bits, m, n, k, gs):
    rng = np.random.default_rng(7 * bits + m + n + k + gs)
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    q, s = po.quant_v0(bits, gs, w)
    blob = np.concatenate([q.view(np.uint8), s.view(np.uint8)])
    assert blob.nbytes == _native.load().pai_b200_v0_blob_bytes(bits, gs, n * k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    got = run_v0(dev, bits, gs, m, n, k, a, blob)
    want = po.gemm_f32(m, n, k, a, po.dequant_v0(bits, gs, q, s, n * k))
    assert maxrel(got, want) <= TOL


def test_v0_argument_errors(dev):
    a = dev.put(np.ones(8, np.float32))
    w = dev.put(np.ones(64, np.int8))
    s = dev.put(np.ones(16, np.float32))
    c = dev.alloc(64 * 4)
    with pytest.raises(_native.PaiError) as e:
        dev.gemm_wq(8, 0, 8, 8, a, w, s, 4, c)
    assert e.value.status == -1  # PAI_ERR_INVALID_ARG, as ref_ops.c:450-452
    with pytest.raises(_native.PaiError) as e:
        dev.gemm_v0(2, 0, 1, 8, 8, a, w, c)
    assert e.value.status == -3  # PAI_ERR_UNSUPPORTED: v0 runs q8 and q4 only
    assert _native.load().pai_b200_v0_blob_bytes(2, 0, 64) == 0


@pytest.mark.parametrize("n", [1024, 4096])
def test_graph_capture_replays_the_op(dev, n):
    """pai_b200_graph_begin/end/launch: two ops captured once, replayed,
    give the bits of the direct calls (n = 4096: the wide-strip form, a
    cooperative launch whose strips share their k-split reduction)."""
    import ctypes as C
    L = _native.load()
    rng = np.random.default_rng(9)
    m, k = 2, 512
    a = dev.put(rng.standard_normal((m, k)).astype(np.float32))
    wq, sc = random_wq(rng, 8, n, k, 32)
    w, s = dev.put(wq), dev.put(sc)
    c1, c2 = dev.alloc(m * n * 4), dev.alloc(m * n * 4)
    dev.gemm_wq(8, m, n, k, a, w, s, 32, c1)
    direct = c1.download(np.float32)
    g = C.c_void_p()
    _native.check(L.pai_b200_graph_begin(dev.ctx), "graph_begin")
    dev.gemm_wq(8, m, n, k, a, w, s, 32, c2)
    dev.gemm_wq(8, m, n, k, a, w, s, 32, c1)
    _native.check(L.pai_b200_graph_end(dev.ctx, C.byref(g)), "graph_end")
    before = L.pai_b200_launch_count(dev.ctx)
    for _ in range(3):
        _native.check(L.pai_b200_graph_launch(dev.ctx, g), "graph_launch")
    dev.sync()
    assert L.pai_b200_launch_count(dev.ctx) - before == 3 * 2
    L.pai_b200_graph_destroy(g)
    assert np.array_equal(c2.download(np.float32).view(np.uint32), direct.view(np.uint32))
    assert np.array_equal(c1.download(np.float32).view(np.uint32), direct.view(np.uint32))
