"""The allocation-free decode attention entry point.

pai_b200_attn_decode_f16kv_noalloc exists for callers that cannot allocate
device memory where they run attention (a runtime that already reserved
the GPU's memory for its own arena, code inside CUDA-graph capture, a
latency-critical loop). It must give the same result as the regular entry
point, pai_b200_attn_decode_f16kv, whose scratch is allocated on demand.

This file is named so pytest collects it last; it also works on its own
in a fresh process (it creates its own device context).
"""
import ctypes as C

import numpy as np
import pytest

from prosperoai_b200 import _native

pytestmark = pytest.mark.gpu


def _run(L, ctx, fn, h, hk, hd, npos, cap, bufs, out_nbytes):
    q, kc, vc, out = bufs
    # poison the output first: a call that launched nothing, or returned
    # early, leaves NaN behind instead of the previous call's answer
    poison = np.full(out_nbytes // 4, np.nan, np.float32)
    _native.check(L.pai_b200_memcpy_h2d(ctx, out, poison.ctypes.data, out_nbytes), "h2d")
    _native.check(fn(ctx, h, hk, hd, npos, cap, q, kc, vc, out), fn.__name__)
    host = np.empty(out_nbytes // 4, np.float32)
    _native.check(L.pai_b200_memcpy_d2h(ctx, host.ctypes.data, out, out_nbytes), "d2h")
    _native.check(L.pai_b200_sync(ctx), "sync")
    return host


@pytest.mark.parametrize("h,hk,npos", [(32, 8, 1), (32, 8, 700), (32, 8, 4097), (16, 2, 1000)])
def test_noalloc_matches_regular_entry_point(h, hk, npos):
    L = _native.load()
    ctx = C.c_void_p()
    _native.check(L.pai_b200_init(0, C.byref(ctx)), "init")
    rng = np.random.default_rng(npos + h)
    hd, cap = 128, npos + 3
    arrays = [rng.standard_normal((h, hd)).astype(np.float32),
              rng.standard_normal((hk, cap, hd)).astype(np.float16),
              rng.standard_normal((hk, cap, hd)).astype(np.float16)]
    ptrs = []
    for a in arrays + [np.zeros((h, hd), np.float32)]:
        p = C.c_void_p()
        _native.check(L.pai_b200_alloc(ctx, a.nbytes, C.byref(p)), "alloc")
        _native.check(L.pai_b200_memcpy_h2d(ctx, p, a.ctypes.data, a.nbytes), "h2d")
        ptrs.append(p)
    nbytes = h * hd * 4
    try:
        ref = _run(L, ctx, L.pai_b200_attn_decode_f16kv, h, hk, hd, npos, cap, ptrs, nbytes)
        assert np.all(np.isfinite(ref))
        for _ in range(2):  # two calls in a row share the fixed scratch array
            got = _run(L, ctx, L.pai_b200_attn_decode_f16kv_noalloc, h, hk, hd, npos, cap, ptrs,
                       nbytes)
            # same kernels, same chunking, same order: the same bits
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    finally:
        for p in ptrs:
            L.pai_b200_free(ctx, p)
        L.pai_b200_shutdown(ctx)


def test_noalloc_rejects_sizes_beyond_its_array():
    L = _native.load()
    ctx = C.c_void_p()
    _native.check(L.pai_b200_init(0, C.byref(ctx)), "init")
    try:
        # 4096 heads over a long context need more than the 2^20-float array
        st = L.pai_b200_attn_decode_f16kv_noalloc(ctx, 4096, 4096, 128, 100000, 100000,
                                                  C.c_void_p(16), C.c_void_p(16), C.c_void_p(16),
                                                  C.c_void_p(16))
        assert st == -3  # PAI_ERR_UNSUPPORTED, before any launch
        assert b"fixed" in L.pai_b200_last_error()
    finally:
        L.pai_b200_shutdown(ctx)
