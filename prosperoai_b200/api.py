"""Host-side API over the C ABI, shaped like the reference's op interface.

Each op takes the arguments of its ``pai_ref_*`` twin (cpu/reference/ref_ops.h)
with device buffers in place of host arrays, and raises ``PaiError`` carrying
the reference status code (pai/error.h) when the C call fails.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._native import (Q4_0, Q4_K, Q8_0, GgufInfo, ModelCfg, OpRegistry, PaiError, check, load)

__all__ = ["Device", "Buffer", "PackedMatrix", "Model", "Session", "PaiError",
           "Q4_0", "Q8_0", "Q4_K", "block_bytes", "quantize", "rope_tables", "gguf_inspect",
           "pai_from_gguf", "pai_inspect"]

BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256}


def block_bytes(wtype: int, numel: int) -> int:
    return int(load().pai_b200_block_bytes(wtype, numel))


def quantize(wtype: int, w: np.ndarray) -> np.ndarray:
    """Host ggml block quantiser (pai_b200_quantize)."""
    w = np.ascontiguousarray(w, np.float32).ravel()
    out = np.empty(block_bytes(wtype, w.size), np.uint8)
    check(load().pai_b200_quantize(wtype, w.ctypes.data, w.size, out.ctypes.data), "quantize")
    return out


def rope_tables(ctx_len: int, r2: int, base: float):
    c = np.empty(ctx_len * r2, np.float32)
    s = np.empty(ctx_len * r2, np.float32)
    check(load().pai_b200_rope_cossin_f32(ctx_len, r2, base, c.ctypes.data, s.ctypes.data),
          "rope_cossin")
    return c, s


class Buffer:
    """Device allocation owned by a Device."""

    def __init__(self, dev: "Device", nbytes: int):
        self.dev = dev
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        check(load().pai_b200_alloc(dev.ctx, max(self.nbytes, 1), C.byref(p)), "alloc")
        self.ptr = p.value

    def upload(self, arr: np.ndarray) -> "Buffer":
        a = np.ascontiguousarray(arr)
        assert a.nbytes <= self.nbytes
        check(load().pai_b200_memcpy_h2d(self.dev.ctx, self.ptr, a.ctypes.data, a.nbytes), "h2d")
        return self

    def download(self, dtype, count: int | None = None) -> np.ndarray:
        dtype = np.dtype(dtype)
        n = self.nbytes // dtype.itemsize if count is None else count
        out = np.empty(n, dtype)
        check(load().pai_b200_memcpy_d2h(self.dev.ctx, out.ctypes.data, self.ptr, out.nbytes), "d2h")
        self.dev.sync()
        return out

    def free(self):
        if self.ptr and self.dev.ctx:
            load().pai_b200_free(self.dev.ctx, self.ptr)
        self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class PackedMatrix:
    """An n x k matrix of ggml blocks in the device GEMV layout."""

    def __init__(self, dev: "Device", wtype: int, n: int, k: int, blocks: np.ndarray):
        self.dev, self.wtype, self.n, self.k = dev, wtype, n, k
        self.buf = dev.alloc(int(load().pai_b200_packed_bytes(wtype, n, k)))
        b = np.ascontiguousarray(blocks, np.uint8)
        assert b.nbytes == block_bytes(wtype, n * k)
        check(load().pai_b200_upload_matrix(dev.ctx, wtype, n, k, b.ctypes.data, self.buf.ptr),
              "upload_matrix")

    @property
    def ptr(self):
        return self.buf.ptr


class Device:
    """One CUDA device context (pai_b200_init)."""

    def __init__(self, device: int = 0):
        L = load()
        ctx = C.c_void_p()
        check(L.pai_b200_init(device, C.byref(ctx)), "init")
        self.ctx = ctx.value
        self.device = device

    def close(self):
        if self.ctx:
            load().pai_b200_shutdown(self.ctx)
            self.ctx = None

    def sync(self):
        check(load().pai_b200_sync(self.ctx), "sync")

    def alloc(self, nbytes: int) -> Buffer:
        return Buffer(self, nbytes)

    def put(self, arr: np.ndarray) -> Buffer:
        a = np.ascontiguousarray(arr)
        return Buffer(self, a.nbytes).upload(a)

    def launches(self) -> int:
        return int(load().pai_b200_launch_count(self.ctx))

    # --- ops ------------------------------------------------------------------------------
    def gemv(self, w: PackedMatrix, x: Buffer, y: Buffer, batch: int = 1,
             residual: Buffer | None = None):
        check(load().pai_b200_gemv_f32(self.ctx, w.wtype, batch, w.n, w.k, w.ptr, x.ptr,
                                       residual.ptr if residual else None, y.ptr), "gemv")

    def prepare_x(self, x: Buffer, k: int, batch: int = 1) -> Buffer:
        """x[batch][k] in the GEMV operand format, for several gemv_prepared calls."""
        xq = Buffer(self, int(load().pai_b200_xq_bytes(batch, k)))
        check(load().pai_b200_prepare_x_f32(self.ctx, batch, k, x.ptr, xq.ptr), "prepare_x")
        return xq

    def gemv_prepared(self, w: PackedMatrix, xq: Buffer, y: Buffer, batch: int = 1,
                      residual: Buffer | None = None):
        check(load().pai_b200_gemv_prepared_f32(self.ctx, w.wtype, batch, w.n, w.k, w.ptr, xq.ptr,
                                                residual.ptr if residual else None, y.ptr),
              "gemv_prepared")

    def gemv_rmsnorm(self, w: PackedMatrix, x: Buffer, gamma: Buffer, eps: float, y: Buffer,
                     batch: int = 1, residual: Buffer | None = None):
        check(load().pai_b200_gemv_rmsnorm_f32(self.ctx, w.wtype, batch, w.n, w.k, w.ptr, x.ptr,
                                               gamma.ptr, eps, residual.ptr if residual else None,
                                               y.ptr), "gemv_rmsnorm")

    def gemm_q4_0(self, w: PackedMatrix, x: Buffer, y: Buffer, m: int):
        """Y[m][n] = X[m][k] . W^T on the tensor cores (bf16 tiles, fp32 accumulate)."""
        check(load().pai_b200_gemm_q4_0_f32(self.ctx, m, w.n, w.k, x.ptr, w.ptr, y.ptr), "gemm_q4_0")

    def gemm(self, w: PackedMatrix, x: Buffer, y: Buffer, m: int):
        """The same GEMM for a packed Q4_0, Q8_0 or Q4_K matrix."""
        check(load().pai_b200_gemm_f32(self.ctx, w.wtype, m, w.n, w.k, x.ptr, w.ptr, y.ptr), "gemm")

    def gemm_wq(self, bits: int, m: int, n: int, k: int, a: Buffer, w_q: Buffer, scales: Buffer,
                group_size: int, c: Buffer):
        """pai_ref_gemm_w8_f32 / _w4_f32 semantics on the GPU ([k][n] int8 or nibbles)."""
        fn = load().pai_b200_gemm_w8_f32 if bits == 8 else load().pai_b200_gemm_w4_f32
        check(fn(self.ctx, m, n, k, a.ptr, w_q.ptr, scales.ptr, group_size, c.ptr), f"gemm_w{bits}")

    def gemm_v0(self, bits: int, group_size: int, m: int, n: int, k: int, a: Buffer, blob: Buffer,
                c: Buffer, blob_offset: int = 0):
        """A v0 .pai quantized [k][n] tensor ([values][f32 scales]) read in place."""
        check(load().pai_b200_gemm_v0_f32(self.ctx, bits, group_size, m, n, k, a.ptr,
                                          blob.ptr + blob_offset, c.ptr), "gemm_v0")

    def dequant(self, w: PackedMatrix, out: Buffer):
        check(load().pai_b200_dequant(self.ctx, w.wtype, w.n, w.k, w.ptr, out.ptr), "dequant")

    def rmsnorm_gamma(self, rows: int, n: int, a: Buffer, gamma: Buffer, eps: float, c: Buffer):
        check(load().pai_b200_rmsnorm_gamma_f32(self.ctx, rows, n, a.ptr, gamma.ptr, eps, c.ptr),
              "rmsnorm_gamma")

    def silu_mul(self, gate: Buffer, up: Buffer, out: Buffer, n: int):
        check(load().pai_b200_silu_mul_f32(self.ctx, gate.ptr, up.ptr, out.ptr, n), "silu_mul")

    def vecadd(self, a: Buffer, b: Buffer, c: Buffer, n: int):
        check(load().pai_b200_vecadd_f32(self.ctx, a.ptr, b.ptr, c.ptr, n), "vecadd")

    def rope(self, x: Buffer, rows, hd, seq, heads, cos_t: Buffer, sin_t: Buffer, r2, out: Buffer):
        check(load().pai_b200_rope_f32(self.ctx, x.ptr, rows, hd, seq, heads, cos_t.ptr, sin_t.ptr,
                                       r2, out.ptr), "rope")

    def attention(self, h, hk, seq, hd, q: Buffer, k: Buffer, v: Buffer, out: Buffer):
        check(load().pai_b200_attention_f32(self.ctx, h, hk, seq, hd, q.ptr, k.ptr, v.ptr, out.ptr),
              "attention")

    def attn_decode_f16kv(self, h, hk, hd, npos, cap, q: Buffer, kc: Buffer, vc: Buffer,
                          out: Buffer):
        check(load().pai_b200_attn_decode_f16kv(self.ctx, h, hk, hd, npos, cap, q.ptr, kc.ptr,
                                                vc.ptr, out.ptr), "attn_decode_f16kv")

    def argmax(self, rows: int, n: int, logits: Buffer, out: Buffer):
        check(load().pai_b200_argmax_f32(self.ctx, rows, n, logits.ptr, out.ptr), "argmax")

    def register_ops(self, registry: OpRegistry):
        check(load().pai_b200_register_ops(C.byref(registry)), "register_ops")


TP_ID_BYTES = 128


def share_tp_id(rank: int, make_id, group=None) -> bytes:
    """Rank 0 makes a communicator id with `make_id()`, every rank of the
    torch.distributed `group` (gloo is enough) receives the same bytes."""
    import torch
    import torch.distributed as dist
    t = torch.zeros(TP_ID_BYTES, dtype=torch.uint8)
    if rank == 0:
        t[:] = torch.frombuffer(bytearray(make_id()), dtype=torch.uint8)
    dist.broadcast(t, src=0, group=group)
    return bytes(t.tolist())


class TPComm:
    """Tensor-parallel communicator of one rank (pai_b200_tp_*: NCCL over
    NVLink). Every rank of the group constructs it with the same id."""

    def __init__(self, dev: Device, rank: int, size: int, uid: bytes):
        if len(uid) != TP_ID_BYTES:
            raise ValueError(f"communicator id must be {TP_ID_BYTES} bytes")
        self.dev, self.rank, self.size = dev, rank, size
        buf = (C.c_uint8 * TP_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        check(load().pai_b200_tp_create(dev.ctx, buf, rank, size, C.byref(h)), "tp_create")
        self.h = h.value

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * TP_ID_BYTES)()
        check(load().pai_b200_tp_unique_id(buf), "tp_unique_id")
        return bytes(buf)

    @classmethod
    def over_group(cls, dev: Device, rank: int, size: int, group=None) -> "TPComm":
        """Create the communicator of a torch.distributed group (id from rank 0)."""
        return cls(dev, rank, size, share_tp_id(rank, cls.unique_id, group))

    def allreduce(self, buf: Buffer, n: int):
        check(load().pai_b200_tp_allreduce_f32(self.h, buf.ptr, n), "tp_allreduce")

    def close(self):
        if self.h:
            load().pai_b200_tp_destroy(self.h)
            self.h = None


def _info_dict(info: "GgufInfo") -> dict:
    c = info.cfg
    cfg = {f: getattr(c, f) for f, _ in ModelCfg._fields_}
    return {"cfg": cfg, "version": info.version, "context_length": info.context_length,
            "n_rot": info.n_rot, "tied_output": bool(info.tied_output),
            "tensor_count": info.tensor_count, "weight_bytes": info.weight_bytes,
            "architecture": info.architecture.decode()}


def gguf_inspect(path: str) -> dict:
    """Parse a GGUF file's header, metadata and tensor table (no GPU needed)."""
    info = GgufInfo()
    check(load().pai_b200_gguf_inspect(os.fsencode(path), C.byref(info)), "gguf_inspect")
    return _info_dict(info)


def pai_from_gguf(gguf_path: str, pai_path: str) -> None:
    """Convert a LLaMA-family GGUF file into a version-2 .pai container that
    keeps the ggml blocks as stored (pai_b200_pai_from_gguf; no GPU needed)."""
    check(load().pai_b200_pai_from_gguf(os.fsencode(gguf_path), os.fsencode(pai_path)), "pai_from_gguf")


def pai_inspect(path: str) -> dict:
    """Parse and validate a version-2 .pai container (no GPU needed)."""
    info = GgufInfo()
    check(load().pai_b200_pai_inspect(os.fsencode(path), C.byref(info)), "pai_inspect")
    return _info_dict(info)


class Model:
    """LLaMA-shaped decoder resident on one device (one tensor-parallel rank)."""

    def __init__(self, dev: Device, cfg: dict, tp_rank: int = 0, tp_size: int = 1):
        self.dev = dev
        self.cfg = dict(cfg)
        c = ModelCfg(cfg["n_layer"], cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"],
                     cfg["head_dim"], cfg["n_ff"], cfg["vocab"], cfg["eps"], cfg["rope_theta"],
                     cfg["wtype"], cfg["etype"])
        h = C.c_void_p()
        check(load().pai_b200_model_create(dev.ctx, C.byref(c), tp_rank, tp_size, C.byref(h)),
              "model_create")
        self.h = h.value

    @classmethod
    def from_gguf(cls, dev: Device, path: str, tp_rank: int = 0, tp_size: int = 1) -> "Model":
        """Load a LLaMA-family GGUF file's blocks as stored (pai_b200_model_load_gguf)."""
        info = GgufInfo()
        h = C.c_void_p()
        check(load().pai_b200_model_load_gguf(dev.ctx, os.fsencode(path), tp_rank, tp_size, C.byref(h),
                                              C.byref(info)), "model_load_gguf")
        self = cls.__new__(cls)
        self.dev = dev
        self.cfg = _info_dict(info)["cfg"]
        self.h = h.value
        return self

    @classmethod
    def from_pai(cls, dev: Device, path: str, tp_rank: int = 0, tp_size: int = 1) -> "Model":
        """Load a version-2 .pai container's blocks as stored (pai_b200_model_load_pai)."""
        info = GgufInfo()
        h = C.c_void_p()
        check(load().pai_b200_model_load_pai(dev.ctx, os.fsencode(path), tp_rank, tp_size, C.byref(h),
                                             C.byref(info)), "model_load_pai")
        self = cls.__new__(cls)
        self.dev = dev
        self.cfg = _info_dict(info)["cfg"]
        self.h = h.value
        return self

    def set_tensor(self, kind: int, layer: int, host: np.ndarray):
        a = np.ascontiguousarray(host)
        check(load().pai_b200_model_set_tensor(self.h, kind, layer, a.ctypes.data), "set_tensor")

    def synthesize(self, seed: int):
        check(load().pai_b200_model_synthesize(self.h, seed), "synthesize")

    def step_weight_bytes(self) -> int:
        return int(load().pai_b200_model_step_weight_bytes(self.h))

    def set_tp(self, comm: "TPComm | None"):
        """Attach the rank's communicator (needed before a tensor-parallel session)."""
        check(load().pai_b200_model_set_tp(self.h, comm.h if comm else None), "model_set_tp")

    def close(self):
        if self.h:
            load().pai_b200_model_destroy(self.h)
            self.h = None


class KvInfo(C.Structure):
    """pai_b200_kv_info_t."""
    _fields_ = [("capacity_tokens", C.c_uint32), ("positions", C.c_uint32),
                ("block_tokens", C.c_uint32), ("n_layer", C.c_uint32), ("batch", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("layer_stride", C.c_uint64),
                ("seq_stride", C.c_uint64), ("head_stride", C.c_uint64),
                ("stats_blocks", C.c_uint64), ("k", C.c_void_p), ("v", C.c_void_p)]


class Session:
    """Greedy decode session (pai_b200_session_*)."""

    def __init__(self, model: Model, batch: int, max_ctx: int):
        self.model, self.batch = model, batch
        h = C.c_void_p()
        check(load().pai_b200_session_create(model.h, batch, max_ctx, C.byref(h)),
              "session_create")
        self.h = h.value

    def step(self, tokens, want_logits: bool = False):
        t = np.ascontiguousarray(tokens, np.int32)
        nxt = np.empty(self.batch, np.int32)
        logits = (np.empty(self.batch * self.model.cfg["vocab"], np.float32)
                  if want_logits else None)
        check(load().pai_b200_session_step(self.h, t.ctypes.data, nxt.ctypes.data,
                                           logits.ctypes.data if want_logits else None),
              "session_step")
        return (nxt, logits) if want_logits else nxt

    def run(self, steps: int):
        check(load().pai_b200_session_run(self.h, steps), "session_run")

    def prefill(self, tokens) -> np.ndarray:
        """Append a prompt ([batch][n] token ids) in one pass per layer; returns
        the greedy next token of every sequence (pai_b200_session_prefill)."""
        t = np.ascontiguousarray(tokens, np.int32).reshape(self.batch, -1)
        nxt = np.empty(self.batch, np.int32)
        check(load().pai_b200_session_prefill(self.h, t.ctypes.data, t.shape[1], nxt.ctypes.data),
              "session_prefill")
        return nxt

    def set_tokens(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        check(load().pai_b200_session_set_tokens(self.h, t.ctypes.data), "set_tokens")

    def tokens(self) -> np.ndarray:
        out = np.empty(self.batch, np.int32)
        check(load().pai_b200_session_get_tokens(self.h, out.ctypes.data), "get_tokens")
        return out

    @property
    def pos(self) -> int:
        return int(load().pai_b200_session_pos(self.h))

    def reset(self):
        check(load().pai_b200_session_reset(self.h), "session_reset")

    @property
    def step_kernels(self) -> int:
        """Kernels one decode step launches (4 on the persistent path)."""
        return int(load().pai_b200_session_step_kernels(self.h))

    def run_layers(self, reps: int = 1):
        """Launch only the persistent layer kernel (timing; the position does not advance)."""
        check(load().pai_b200_session_run_layers(self.h, reps), "session_run_layers")

    def kv_info(self) -> dict:
        info = KvInfo()
        check(load().pai_b200_session_kv_info(self.h, C.byref(info)), "session_kv_info")
        return {f: getattr(info, f) for f, _ in KvInfo._fields_}

    def kv_reserve(self, tokens: int) -> int:
        """pai_kv_cache_reserve semantics: the first of `tokens` new positions."""
        pos = C.c_uint32()
        check(load().pai_b200_session_kv_reserve(self.h, tokens, C.byref(pos)), "session_kv_reserve")
        return int(pos.value)

    def write_kv(self, layer: int, seq: int, k: np.ndarray, v: np.ndarray, pos0: int = 0) -> None:
        """Copy host fp16 rows [kv_head][positions][head_dim] into the cache of
        one layer and sequence at positions pos0.. (this rank's kv heads)."""
        info = self.kv_info()
        L = load()
        for base, a in ((info["k"], k), (info["v"], v)):
            a = np.ascontiguousarray(a, np.float16)
            hk, npos, hd = a.shape
            assert hk == info["kv_heads"] and hd == info["head_dim"]
            assert pos0 + npos <= info["capacity_tokens"]
            for h in range(hk):
                off = (layer * info["layer_stride"] + seq * info["seq_stride"] + h * info["head_stride"]
                       + pos0 * hd) * 2
                check(L.pai_b200_memcpy_h2d(self.model.dev.ctx, C.c_void_p(base + off), a[h].ctypes.data,
                                            a[h].nbytes), "h2d")
        self.model.dev.sync()

    def hidden(self) -> np.ndarray:
        p = load().pai_b200_session_hidden(self.h)
        n = self.batch * self.model.cfg["n_embd"]
        out = np.empty(n, np.float32)
        check(load().pai_b200_memcpy_d2h(self.model.dev.ctx, out.ctypes.data, p, out.nbytes), "d2h")
        self.model.dev.sync()
        return out

    def close(self):
        if self.h:
            load().pai_b200_session_destroy(self.h)
            self.h = None
