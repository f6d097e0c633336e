"""ctypes bindings to the CPU checkers (test infrastructure only).

``lib()`` is the C restatement (``oracle/build/liboracle.so``, built from
``oracle/pai_oracle.c``). ``ref()`` is the reference's own hot-path code
compiled in place from its sources (``oracle/_ref/libpai_ref.so``, see
``oracle/Makefile``); it is present wherever the reference checkout was
available at build time and ``None`` otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
Q4_0, Q8_0, Q4_K = 2, 8, 12
BLOCK = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144)}

_lib = None
_ref = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
U64 = C.c_uint64


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def reference_dir() -> str:
    """Location of the reference checkout: PAI_REFERENCE_DIR, else the
    default that oracle/Makefile names (its only written copy)."""
    env = os.environ.get("PAI_REFERENCE_DIR")
    if env:
        return env
    r = subprocess.run(["make", "-s", "-C", HERE, "print-ref"], capture_output=True, text=True)
    return r.stdout.strip()


def _sig(fn, res, *args):
    fn.restype = res
    fn.argtypes = list(args)
    return fn


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "build", "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        _sig(L.po_f16_to_f32, C.c_float, C.c_uint16)
        _sig(L.po_f32_to_f16, C.c_uint16, C.c_float)
        _sig(L.po_type_bytes, U64, C.c_uint32, U64)
        _sig(L.po_dequant, C.c_int, C.c_uint32, u8p, f32p, U64)
        _sig(L.po_quantize, C.c_int, C.c_uint32, f32p, u8p, U64)
        _sig(L.po_gemv_f32, None, U64, U64, f32p, f32p, f32p)
        _sig(L.po_gemv_q, C.c_int, C.c_uint32, U64, U64, u8p, f32p, f32p, C.c_int)
        _sig(L.po_gemm_f32, None, U64, U64, U64, f32p, f32p, f32p)
        _sig(L.po_quant_v0, U64, C.c_uint32, U64, f32p, U64, i8p, f32p)
        _sig(L.po_dequant_v0, C.c_int, C.c_uint32, U64, i8p, f32p, U64, f32p)
        _sig(L.po_gemm_wq_f32, C.c_int, C.c_uint32, U64, U64, U64, f32p, i8p, f32p, U64,
             f32p)
        _sig(L.po_rmsnorm_gamma_f32, None, f32p, f32p, U64, f32p, C.c_float)
        _sig(L.po_silu_f32, None, f32p, f32p, U64)
        _sig(L.po_vecmul_f32, None, f32p, f32p, f32p, U64)
        _sig(L.po_vecadd_f32, None, f32p, f32p, f32p, U64)
        _sig(L.po_rope_f32, None, f32p, U64, U64, U64, f32p, f32p, U64, f32p)
        _sig(L.po_rope_at_f32, None, f32p, U64, U64, U64, f32p, f32p, U64, f32p)
        _sig(L.po_rope_cossin_f32, None, U64, U64, C.c_float, f32p, f32p)
        _sig(L.po_attention_f32, C.c_int, U64, U64, U64, U64, f32p, f32p, f32p, f32p)
        _sig(L.po_attention_decode_f16, C.c_int, U64, U64, U64, U64, U64, f32p,
             u16p, u16p, f32p)
        _sig(L.po_argmax_f32, C.c_uint32, f32p, U64)
        _sig(L.po_fill_normal, None, f32p, U64, U64, C.c_double, C.c_double)
        _sig(L.po_session_create, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32,
             C.c_int)
        _sig(L.po_session_destroy, None, C.c_void_p)
        _sig(L.po_session_step, C.c_int64, C.c_void_p, C.c_uint32, C.c_void_p)
        _sig(L.po_session_hidden, C.POINTER(C.c_float), C.c_void_p)
        _sig(L.po_session_kv, C.POINTER(C.c_uint16), C.c_void_p, C.c_uint32, C.c_int)
        _sig(L.po_session_seek, C.c_int, C.c_void_p, C.c_uint32)
        _lib = L
    return _lib


class GgufTensor(C.Structure):
    """pai_gguf_tensor_t (adapters/llama/gguf.h:55-61)."""
    _fields_ = [("name", C.c_char * 128), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("type", C.c_uint32), ("offset", C.c_uint64)]


class Gguf(C.Structure):
    """pai_gguf_t (adapters/llama/gguf.h:64-74)."""
    _fields_ = [("data", C.c_void_p), ("size", C.c_uint64), ("version", C.c_uint32),
                ("tensor_count", C.c_uint64), ("kv_count", C.c_uint64), ("alignment", C.c_uint64),
                ("kv_start", C.c_void_p), ("data_start", C.c_void_p),
                ("tensors", C.POINTER(GgufTensor))]


class QuantScheme(C.Structure):
    """pai_quant_scheme_t (models/quantize.h:35-39)."""
    _fields_ = [("bit_width", C.c_uint8), ("is_signed", C.c_uint8), ("group_size", C.c_uint16)]


def ref():
    """The reference's own code built from its sources, or None."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libpai_ref.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        _sig(R.pai_refshim_dequant, C.c_int32, C.c_uint32, u8p, f32p, U64)
        _sig(R.pai_refshim_type_bytes, U64, C.c_uint32, U64)
        _sig(R.pai_ref_gemv_f32, C.c_int32, U64, U64, f32p, f32p, f32p)
        _sig(R.pai_ref_rmsnorm_gamma_f32, C.c_int32, f32p, f32p, U64, f32p, C.c_float)
        _sig(R.pai_ref_silu_f32, C.c_int32, f32p, f32p, U64)
        _sig(R.pai_ref_vecmul_f32, C.c_int32, f32p, f32p, f32p, U64)
        _sig(R.pai_ref_vecadd_f32, C.c_int32, f32p, f32p, f32p, U64)
        _sig(R.pai_ref_rope_f32, C.c_int32, f32p, U64, U64, U64, U64, f32p, f32p,
             U64, f32p)
        _sig(R.pai_ref_rope_cossin_f32, C.c_int32, U64, U64, C.c_float, f32p, f32p)
        _sig(R.pai_ref_attention_f32, C.c_int32, U64, U64, U64, U64, f32p, f32p,
             f32p, f32p)
        _sig(R.pai_ref_gemm_f32, C.c_int32, U64, U64, U64, f32p, f32p, f32p)
        _sig(R.pai_ref_gemm_w8_f32, C.c_int32, U64, U64, U64, f32p, i8p, f32p, U64,
             f32p)
        _sig(R.pai_ref_gemm_w4_f32, C.c_int32, U64, U64, U64, f32p, i8p, f32p, U64,
             f32p)
        _sig(R.pai_opt_gemv_f32, C.c_int32, U64, U64, f32p, f32p, f32p)
        _sig(R.pai_gguf_open, C.c_int32, C.c_char_p, U64, C.POINTER(Gguf))
        _sig(R.pai_gguf_close, None, C.POINTER(Gguf))
        _sig(R.pai_gguf_get_u32, C.c_int32, C.POINTER(Gguf), C.c_char_p, C.POINTER(C.c_uint32))
        _sig(R.pai_gguf_get_f32, C.c_int32, C.POINTER(Gguf), C.c_char_p, C.POINTER(C.c_float))
        _sig(R.pai_gguf_get_string, C.c_int32, C.POINTER(Gguf), C.c_char_p, C.c_char_p, U64)
        _sig(R.pai_gguf_get_string_array, C.c_int32, C.POINTER(Gguf), C.c_char_p,
             C.POINTER(C.POINTER(C.c_char_p)), C.POINTER(U64))
        _sig(R.pai_gguf_find_tensor, C.POINTER(GgufTensor), C.POINTER(Gguf), C.c_char_p)
        _sig(R.pai_gguf_dequant, C.c_int32, C.POINTER(Gguf), C.POINTER(GgufTensor),
             C.POINTER(C.POINTER(C.c_float)), C.POINTER(U64))
        _sig(R.pai_quantize_f32, C.c_int32, f32p, U64, C.POINTER(QuantScheme), i8p, f32p,
             C.POINTER(U64))
        _sig(R.pai_quant_weights_bytes, U64, U64, C.POINTER(QuantScheme))
        _sig(R.pai_dequantize_f32, C.c_int32, i8p, f32p, U64, C.POINTER(QuantScheme), f32p)
        _sig(R.pai_opt_gemm_f32, C.c_int32, U64, U64, U64, f32p, f32p, f32p)
        _sig(R.pai_opt_gemm_w8_f32, C.c_int32, U64, U64, U64, f32p, i8p, f32p, U64,
             f32p)
        _sig(R.pai_opt_backend_name, C.c_char_p)
        _sig(R.pai_sampler_sample_logits, C.c_int32, C.c_void_p, f32p, C.c_uint32,
             C.POINTER(C.c_uint32))
        _sig(R.refdisp_run, C.c_int32, C.c_char_p, C.c_int32, C.c_uint32, U64, U64, U64, u8p,
             f32p, f32p, f32p, f32p, f32p, C.POINTER(DispatchReport))
        _ref = R
    return _ref


class DispatchReport(C.Structure):
    """refdisp_report_t (oracle/ref_dispatch.c)."""
    _fields_ = [("gate_cpu_ref", C.c_int32), ("gate_b200_ref_map", C.c_int32),
                ("gate_b200", C.c_int32), ("cpu_status", C.c_int32), ("gpu_status", C.c_int32),
                ("num_steps", C.c_uint32), ("gpu_steps", C.c_uint32),
                ("kernel_ids", C.c_int32 * 4), ("devices", C.c_uint8 * 4),
                ("error", C.c_char * 256)]


def dispatch_slice(backend_so: str, run_gpu: bool, wtype: int, m: int, n: int, k: int,
                   blocks: np.ndarray, x: np.ndarray, gamma: np.ndarray, res: np.ndarray):
    """The decoder slice rmsnorm -> projection -> residual add, built with the
    reference's graph builder, planned by its scheduler and run by its executor
    on the host; with run_gpu, also through the executor's cuda-b200 branch
    (oracle/ref_dispatch.c), which loads backend_so. Returns
    (report, out_cpu [m][n], out_gpu [m][n])."""
    R = ref()
    assert R is not None, "oracle/_ref/libpai_ref.so is not built"
    rep = DispatchReport()
    out_cpu = np.zeros(m * n, np.float32)
    out_gpu = np.zeros(m * n, np.float32)
    rc = R.refdisp_run(backend_so.encode(), int(run_gpu), wtype, m, n, k,
                       np.ascontiguousarray(blocks, np.uint8).ravel(),
                       np.ascontiguousarray(x, np.float32).ravel(),
                       np.ascontiguousarray(gamma, np.float32).ravel(),
                       np.ascontiguousarray(res, np.float32).ravel(), out_cpu, out_gpu,
                       C.byref(rep))
    assert rc == 0, rep.error.decode()
    return rep, out_cpu.reshape(m, n), out_gpu.reshape(m, n)


# ---- convenience wrappers (numpy in, numpy out) ---------------------------------

def row_bytes(wtype: int, k: int) -> int:
    elems, nbytes = BLOCK[wtype]
    assert k % elems == 0
    return k // elems * nbytes


def dequant(wtype: int, blocks: np.ndarray, numel: int) -> np.ndarray:
    out = np.empty(numel, np.float32)
    rc = lib().po_dequant(wtype, np.ascontiguousarray(blocks, np.uint8).ravel(), out, numel)
    assert rc == 0
    return out


def quantize(wtype: int, w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32).ravel()
    out = np.empty(row_bytes(wtype, w.size), np.uint8)
    rc = lib().po_quantize(wtype, w, out, w.size)
    assert rc == 0
    return out


def gemv_q(wtype: int, n: int, k: int, blocks: np.ndarray, x: np.ndarray,
           threads: int = 8) -> np.ndarray:
    y = np.empty(n, np.float32)
    rc = lib().po_gemv_q(wtype, n, k, np.ascontiguousarray(blocks, np.uint8).ravel(),
                         np.ascontiguousarray(x, np.float32), y, threads)
    assert rc == 0
    return y


def gemm_f32(m: int, n: int, k: int, a, b) -> np.ndarray:
    c = np.empty(m * n, np.float32)
    lib().po_gemm_f32(m, n, k, np.ascontiguousarray(a, np.float32).ravel(),
                      np.ascontiguousarray(b, np.float32).ravel(), c)
    return c.reshape(m, n)


def v0_value_bytes(bits: int, n: int) -> int:
    return n if bits == 8 else (n + 1) // 2


def v0_groups(n: int, gs: int) -> int:
    gs = gs or n
    return (n + gs - 1) // gs


def quant_v0(bits: int, gs: int, w) -> tuple[np.ndarray, np.ndarray]:
    """models/quantize.c:74-143 restated: (packed values, f32 scales)."""
    w = np.ascontiguousarray(w, np.float32).ravel()
    q = np.empty(v0_value_bytes(bits, w.size), np.int8)
    s = np.empty(v0_groups(w.size, gs), np.float32)
    assert lib().po_quant_v0(bits, gs, w, w.size, q, s) == s.size
    return q, s


def dequant_v0(bits: int, gs: int, q, scales, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    assert lib().po_dequant_v0(bits, gs, np.ascontiguousarray(q, np.int8),
                               np.ascontiguousarray(scales, np.float32), n, out) == 0
    return out


def gemm_wq(bits: int, m: int, n: int, k: int, a, w_q, scales, g: int) -> np.ndarray:
    """ref_ops.c:447-499 restated (pai_ref_gemm_w8_f32 / _w4_f32)."""
    c = np.empty(m * n, np.float32)
    assert lib().po_gemm_wq_f32(bits, m, n, k, np.ascontiguousarray(a, np.float32).ravel(),
                                np.ascontiguousarray(w_q, np.int8).ravel(),
                                np.ascontiguousarray(scales, np.float32).ravel(), g, c) == 0
    return c.reshape(m, n)


def rmsnorm_gamma(a, gamma, eps=1e-5):
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty_like(a)
    rows = a.reshape(-1, a.shape[-1])
    o = out.reshape(-1, a.shape[-1])
    g = np.ascontiguousarray(gamma, np.float32)
    for r in range(rows.shape[0]):
        row = np.ascontiguousarray(rows[r])
        orow = np.empty_like(row)
        lib().po_rmsnorm_gamma_f32(row, orow, row.size, g, eps)
        o[r] = orow
    return out


def silu_mul(gate, up):
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    g = np.empty_like(gate)
    lib().po_silu_f32(gate, g, gate.size)
    h = np.empty_like(gate)
    lib().po_vecmul_f32(g, up, h, gate.size)
    return h


def rope_tables(ctx: int, r2: int, base: float):
    c = np.empty(ctx * r2, np.float32)
    s = np.empty(ctx * r2, np.float32)
    lib().po_rope_cossin_f32(ctx, r2, base, c, s)
    return c, s


def rope(x, heads: int, hd: int, cos_t, sin_t, r2: int):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    rows = x.size // hd
    lib().po_rope_f32(x.ravel(), rows, hd, heads, cos_t, sin_t, r2, out.ravel())
    return out


def attention(h, hk, seq, hd, q, k, v):
    out = np.empty(seq * h * hd, np.float32)
    rc = lib().po_attention_f32(h, hk, seq, hd, np.ascontiguousarray(q, np.float32).ravel(),
                                np.ascontiguousarray(k, np.float32).ravel(),
                                np.ascontiguousarray(v, np.float32).ravel(), out)
    assert rc == 0
    return out


def attention_decode_f16(h, hk, hd, npos, cap, q, kc, vc):
    out = np.empty(h * hd, np.float32)
    rc = lib().po_attention_decode_f16(h, hk, hd, npos, cap,
                                       np.ascontiguousarray(q, np.float32).ravel(),
                                       np.ascontiguousarray(kc, np.uint16).ravel(),
                                       np.ascontiguousarray(vc, np.uint16).ravel(), out)
    assert rc == 0
    return out


def argmax(logits) -> int:
    return int(lib().po_argmax_f32(np.ascontiguousarray(logits, np.float32), logits.size))


def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().po_fill_normal(out, n, seed, mean, std)
    return out


def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    f = lib().po_f32_to_f16
    return np.array([f(float(v)) for v in np.ravel(a)], np.uint16)


# ---- composed decode ---------------------------------------------------------------

class _Cfg(C.Structure):
    _fields_ = [("n_layer", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("n_ff", C.c_uint32),
                ("vocab", C.c_uint32), ("eps", C.c_float), ("rope_theta", C.c_float),
                ("wtype", C.c_uint32), ("etype", C.c_uint32)]


_PP = C.POINTER(C.c_void_p)


class _W(C.Structure):
    _fields_ = [("tok_embd", C.c_void_p), ("output", C.c_void_p),
                ("output_norm", C.c_void_p),
                ("wq", _PP), ("wk", _PP), ("wv", _PP), ("wo", _PP), ("wgate", _PP),
                ("wup", _PP), ("wdown", _PP), ("attn_norm", _PP), ("ffn_norm", _PP)]


class Session:
    """The composed reference decode (llama.c:669-797 op order) on CPU.

    ``weights`` is a dict of numpy arrays in ggml row-major blocks:
    tok_embd, output, output_norm and per-layer lists wq, wk, wv, wo,
    wgate, wup, wdown, attn_norm, ffn_norm.
    """

    def __init__(self, cfg: dict, weights: dict, max_ctx: int, threads: int = 8):
        self.cfg = _Cfg(cfg["n_layer"], cfg["n_embd"], cfg["n_head"], cfg["n_head_kv"],
                        cfg["head_dim"], cfg["n_ff"], cfg["vocab"], cfg["eps"],
                        cfg["rope_theta"], cfg["wtype"], cfg["etype"])
        self._keep = []

        def ptr(a):
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a.ctypes.data

        def plist(name):
            arr = (C.c_void_p * cfg["n_layer"])(*[ptr(a) for a in weights[name]])
            self._keep.append(arr)
            return C.cast(arr, _PP)

        self.w = _W(ptr(weights["tok_embd"]), ptr(weights["output"]),
                    ptr(weights["output_norm"]),
                    *[plist(n) for n in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown",
                                         "attn_norm", "ffn_norm")])
        self.vocab = cfg["vocab"]
        self.n_embd = cfg["n_embd"]
        self.max_ctx = max_ctx
        self.h = lib().po_session_create(C.byref(self.cfg), C.byref(self.w), max_ctx, threads)
        assert self.h, "oracle session allocation failed"

    def step(self, token: int, want_logits: bool = False):
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        tok = lib().po_session_step(self.h, token,
                                    logits.ctypes.data if want_logits else None)
        assert tok >= 0
        return (int(tok), logits) if want_logits else int(tok)

    def hidden(self) -> np.ndarray:
        p = lib().po_session_hidden(self.h)
        return np.ctypeslib.as_array(p, (self.n_embd,)).copy()

    def set_kv(self, layer: int, k: np.ndarray, v: np.ndarray) -> None:
        """Cache rows of one layer, [kv_head][positions][head_dim] fp16 bits
        (positions <= max_ctx), from position 0."""
        for which, a in ((0, k), (1, v)):
            a = np.ascontiguousarray(a, np.uint16)
            hk, npos, hd = a.shape
            dst = np.ctypeslib.as_array(lib().po_session_kv(self.h, layer, which),
                                        (hk, self.max_ctx, hd))
            dst[:, :npos, :] = a

    def seek(self, pos: int) -> None:
        assert lib().po_session_seek(self.h, pos) == 0

    def close(self):
        if self.h:
            lib().po_session_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
