"""Failure detection without a GPU fault: a bounded device wait that runs out.

The tensor-parallel exchange (pai_b200_tp_allreduce_add_f32) waits for every
rank's arrival stamp. Here it runs as rank 0 of 2 with both exchange buffers
on this GPU and no rank 1: the stamp never comes, the wait gives up after the
context's limit (pai_b200_set_wait_limit, the counterpart of the reference's
pai_gpu_wait_label timeout, gpu/hal/hal.h:106-108), the next sync reports
PAI_ERR_TIMEOUT, and the context keeps working: a GEMV run afterwards still
matches the oracle. Nothing faults, traps or hangs; the kernel that waits is
the only one running.
"""
import ctypes as C
import time

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import _native
from prosperoai_b200.api import PackedMatrix, quantize

pytestmark = pytest.mark.gpu

PAI_ERR_TIMEOUT = -5


def _xbuf(L, ctx, cap):
    buf = C.c_void_p()
    handle = (C.c_uint8 * 64)()
    _native.check(L.pai_b200_tp_xbuf_create(ctx, cap, C.byref(buf), handle), "tp_xbuf_create")
    return buf


def test_exchange_with_one_rank_sums_its_slot(dev):
    """rank 0 of 1: the stamp it waits for is its own; x += slot 0."""
    L = _native.load()
    cap, n = 4096, 4000
    a = _xbuf(L, dev.ctx, cap)
    try:
        part = np.arange(n, dtype=np.float32) * 0.5
        slot = L.pai_b200_tp_xbuf_slot(a, 0, cap)
        _native.check(L.pai_b200_memcpy_h2d(dev.ctx, slot, part.ctypes.data, part.nbytes), "h2d")
        x0 = np.full(n, 2.0, np.float32)
        x = dev.put(x0)
        bufs = (C.c_void_p * 1)(a.value)
        for _ in range(3):  # repeated calls advance the stamps in step
            _native.check(L.pai_b200_tp_allreduce_add_f32(dev.ctx, bufs, 0, 1, 0, cap, x.ptr, n), "exchange")
        dev.sync()
        np.testing.assert_array_equal(x.download(np.float32, n), x0 + 3 * part)
    finally:
        L.pai_b200_tp_xbuf_release(dev.ctx, a, 1)


def test_exchange_wait_runs_out_and_context_stays_usable(dev):
    L = _native.load()
    cap, n = 4096, 4096
    a, b = _xbuf(L, dev.ctx, cap), _xbuf(L, dev.ctx, cap)
    limit_ns = 50_000_000  # 50 ms
    _native.check(L.pai_b200_set_wait_limit(dev.ctx, limit_ns), "set_wait_limit")
    try:
        x = dev.put(np.ones(n, np.float32))
        bufs = (C.c_void_p * 2)(a.value, b.value)
        _native.check(L.pai_b200_tp_allreduce_add_f32(dev.ctx, bufs, 0, 2, 0, cap, x.ptr, n), "exchange")
        t0 = time.perf_counter()
        st = L.pai_b200_sync(dev.ctx)
        waited = time.perf_counter() - t0
        assert st == PAI_ERR_TIMEOUT, (st, L.pai_b200_last_error())
        assert waited < 5.0
        assert L.pai_b200_sync(dev.ctx) == 0  # the error is reported once
        # the context still runs work: a GEMV against the oracle
        _native.check(L.pai_b200_set_wait_limit(dev.ctx, 0), "set_wait_limit")
        rng = np.random.default_rng(5)
        rows, k = 512, 4096
        blocks = quantize(po.Q4_0, (rng.standard_normal(rows * k) * 0.02).astype(np.float32))
        xv = rng.standard_normal(k).astype(np.float32)
        w = PackedMatrix(dev, po.Q4_0, rows, k, blocks)
        y = dev.alloc(rows * 4)
        dev.gemv(w, dev.put(xv), y)
        got = y.download(np.float32)
        ref = po.gemv_q(po.Q4_0, rows, k, blocks, xv)
        assert np.max(np.abs(got - ref)) <= 1e-3 * np.max(np.abs(ref))
    finally:
        L.pai_b200_set_wait_limit(dev.ctx, 0)
        L.pai_b200_tp_xbuf_release(dev.ctx, a, 1)
        L.pai_b200_tp_xbuf_release(dev.ctx, b, 1)


def test_wait_limit_range(dev):
    L = _native.load()
    assert L.pai_b200_set_wait_limit(dev.ctx, 10) == -1  # below 1 ms
    assert L.pai_b200_set_wait_limit(dev.ctx, 120_000_000_000) == -1  # above 60 s
    assert L.pai_b200_set_wait_limit(dev.ctx, 0) == 0  # default
