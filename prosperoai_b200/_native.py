"""ctypes binding of ``libpai_b200.so`` (the C ABI declared in include/pai_b200.h).

Loading fails loudly when the library has not been built: there is no
CPU fallback behind this package.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libpai_b200.so")

Q4_0, Q8_0, Q4_K = 2, 8, 12

# status codes (pai/error.h:13-23)
PAI_OK = 0
STATUS_NAMES = {0: "PAI_OK", -1: "PAI_ERR_INVALID_ARG", -2: "PAI_ERR_NOMEM",
                -3: "PAI_ERR_UNSUPPORTED", -4: "PAI_ERR_CAPABILITY", -5: "PAI_ERR_TIMEOUT",
                -6: "PAI_ERR_MISMATCH", -7: "PAI_ERR_IO", -8: "PAI_ERR_INIT",
                -9: "PAI_ERR_INTERNAL"}

# tensor kinds of pai_b200_model_set_tensor
T_TOK_EMBD, T_OUTPUT, T_OUTPUT_NORM, T_WQ, T_WK, T_WV, T_WO, T_WGATE, T_WUP, T_WDOWN, \
    T_ATTN_NORM, T_FFN_NORM = range(12)


class PaiError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}: {detail}")
        self.status = status


class ModelCfg(C.Structure):
    _fields_ = [("n_layer", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("head_dim", C.c_uint32), ("n_ff", C.c_uint32),
                ("vocab", C.c_uint32), ("eps", C.c_float), ("rope_theta", C.c_float),
                ("wtype", C.c_uint32), ("etype", C.c_uint32)]


class GgufInfo(C.Structure):
    """pai_b200_gguf_info_t."""
    _fields_ = [("cfg", ModelCfg), ("version", C.c_uint32), ("context_length", C.c_uint32),
                ("n_rot", C.c_uint32), ("tied_output", C.c_uint32), ("tensor_count", C.c_uint64),
                ("weight_bytes", C.c_uint64), ("architecture", C.c_char * 64)]


class OpDescriptor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("version", C.c_uint32), ("num_inputs", C.c_uint32),
                ("num_outputs", C.c_uint32), ("in_dtype", C.c_int32), ("out_dtype", C.c_int32),
                ("caps", C.c_uint32), ("ref_fn", C.c_void_p), ("kernel_id", C.c_int32),
                ("reserved", C.c_uint32 * 2)]


class OpRegistry(C.Structure):
    _fields_ = [("version", C.c_uint32), ("count", C.c_uint32),
                ("ops", C.POINTER(OpDescriptor) * 64)]


_lib = None
V, P, U64, U32, I32, F32 = C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_int32, C.c_float
PP = C.POINTER(C.c_void_p)

# name -> (restype, argtypes)
SIGNATURES = {
    "pai_b200_init": (I32, [C.c_int, PP]),
    "pai_b200_shutdown": (I32, [P]),
    "pai_b200_device_count": (I32, [C.POINTER(C.c_int)]),
    "pai_b200_last_error": (C.c_char_p, []),
    "pai_b200_version": (C.c_char_p, []),
    "pai_b200_alloc": (I32, [P, U64, PP]),
    "pai_b200_free": (I32, [P, P]),
    "pai_b200_host_alloc": (I32, [P, U64, PP]),
    "pai_b200_host_free": (I32, [P, P]),
    "pai_b200_memcpy_h2d": (I32, [P, P, P, U64]),
    "pai_b200_memcpy_d2h": (I32, [P, P, P, U64]),
    "pai_b200_memcpy_d2d": (I32, [P, P, P, U64]),
    "pai_b200_memset": (I32, [P, P, C.c_int, U64]),
    "pai_b200_sync": (I32, [P]),
    "pai_b200_set_pdl": (I32, [P, I32]),
    "pai_b200_set_wait_limit": (I32, [P, U64]),
    "pai_b200_tp_xbuf_create": (I32, [P, U64, PP, P]),
    "pai_b200_tp_xbuf_open": (I32, [P, P, PP]),
    "pai_b200_tp_xbuf_release": (I32, [P, P, C.c_int]),
    "pai_b200_tp_xbuf_slot": (P, [P, U32, U64]),
    "pai_b200_tp_allreduce_add_f32": (I32, [P, P, U32, U32, U32, U64, P, U64]),
    "pai_b200_event_create": (I32, [P, PP]),
    "pai_b200_event_destroy": (I32, [P, P]),
    "pai_b200_event_record": (I32, [P, P]),
    "pai_b200_event_elapsed": (I32, [P, P, C.POINTER(C.c_float)]),
    "pai_b200_launch_count": (U64, [P]),
    "pai_b200_graph_begin": (I32, [P]),
    "pai_b200_graph_end": (I32, [P, PP]),
    "pai_b200_graph_launch": (I32, [P, P]),
    "pai_b200_graph_destroy": (I32, [P]),
    "pai_b200_block_bytes": (U64, [U32, U64]),
    "pai_b200_quantize": (I32, [U32, P, U64, P]),
    "pai_b200_packed_bytes": (U64, [U32, U64, U64]),
    "pai_b200_pack": (I32, [P, U32, U64, U64, P, P, P]),
    "pai_b200_upload_matrix": (I32, [P, U32, U64, U64, P, P]),
    "pai_b200_dequant": (I32, [P, U32, U64, U64, P, P]),
    "pai_b200_gemv_q8_0_f32": (I32, [P, U64, U64, P, P, P]),
    "pai_b200_gemv_q4_0_f32": (I32, [P, U64, U64, P, P, P]),
    "pai_b200_gemv_q4_k_f32": (I32, [P, U64, U64, P, P, P]),
    "pai_b200_gemv_f32": (I32, [P, U32, U64, U64, U64, P, P, P, P]),
    "pai_b200_xq_bytes": (U64, [U64, U64]),
    "pai_b200_prepare_x_f32": (I32, [P, U64, U64, P, P]),
    "pai_b200_gemv_prepared_f32": (I32, [P, U32, U64, U64, U64, P, P, P, P]),
    "pai_b200_gemv_rmsnorm_f32": (I32, [P, U32, U64, U64, U64, P, P, P, F32, P, P]),
    "pai_b200_gemm_q4_0_f32": (I32, [P, U64, U64, U64, P, P, P]),
    "pai_b200_gemm_f32": (I32, [P, U32, U64, U64, U64, P, P, P]),
    "pai_b200_gemm_w8_f32": (I32, [P, U64, U64, U64, P, P, P, U64, P]),
    "pai_b200_gemm_w4_f32": (I32, [P, U64, U64, U64, P, P, P, U64, P]),
    "pai_b200_gemm_v0_f32": (I32, [P, U32, U32, U64, U64, U64, P, P, P]),
    "pai_b200_v0_blob_bytes": (U64, [U32, U32, U64]),
    "pai_b200_rmsnorm_gamma_f32": (I32, [P, U64, U64, P, P, F32, P]),
    "pai_b200_silu_mul_f32": (I32, [P, P, P, P, U64]),
    "pai_b200_vecadd_f32": (I32, [P, P, P, P, U64]),
    "pai_b200_rope_f32": (I32, [P, P, U64, U64, U64, U64, P, P, U64, P]),
    "pai_b200_rope_cossin_f32": (I32, [U64, U64, F32, P, P]),
    "pai_b200_attention_f32": (I32, [P, U64, U64, U64, U64, P, P, P, P]),
    "pai_b200_attn_decode_f16kv": (I32, [P, U64, U64, U64, U64, U64, P, P, P, P]),
    "pai_b200_attn_decode_f16kv_noalloc": (I32, [P, U64, U64, U64, U64, U64, P, P, P, P]),
    "pai_b200_argmax_f32": (I32, [P, U64, U64, P, P]),
    "pai_b200_register_ops": (I32, [P]),
    "pai_b200_op_count": (U32, []),
    "pai_b200_op": (C.POINTER(OpDescriptor), [U32]),
    "pai_b200_model_create": (I32, [P, C.POINTER(ModelCfg), U32, U32, PP]),
    "pai_b200_model_set_tp": (I32, [P, P]),
    "pai_b200_tp_unique_id": (I32, [P]),
    "pai_b200_tp_create": (I32, [P, P, U32, U32, PP]),
    "pai_b200_tp_destroy": (I32, [P]),
    "pai_b200_tp_rank": (U32, [P]),
    "pai_b200_tp_size": (U32, [P]),
    "pai_b200_tp_allreduce_f32": (I32, [P, P, U64]),
    "pai_b200_model_destroy": (I32, [P]),
    "pai_b200_gguf_inspect": (I32, [C.c_char_p, C.POINTER(GgufInfo)]),
    "pai_b200_model_load_gguf": (I32, [P, C.c_char_p, U32, U32, PP, C.POINTER(GgufInfo)]),
    "pai_b200_pai_from_gguf": (I32, [C.c_char_p, C.c_char_p]),
    "pai_b200_pai_inspect": (I32, [C.c_char_p, C.POINTER(GgufInfo)]),
    "pai_b200_model_load_pai": (I32, [P, C.c_char_p, U32, U32, PP, C.POINTER(GgufInfo)]),
    "pai_b200_ir_quant_ggml": (I32, [U32, C.c_void_p]),
    "pai_b200_ir_quant_ggml_type": (I32, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "pai_b200_model_set_tensor": (I32, [P, U32, U32, P]),
    "pai_b200_model_synthesize": (I32, [P, U64]),
    "pai_b200_tensor_seed": (U64, [U64, U32, U32]),
    "pai_b200_synth_blocks": (I32, [P, U32, U64, U64, U64, F32, P, P]),
    "pai_b200_model_weight_bytes": (U64, [P]),
    "pai_b200_model_step_weight_bytes": (U64, [P]),
    "pai_b200_session_create": (I32, [P, U32, U32, PP]),
    "pai_b200_session_destroy": (I32, [P]),
    "pai_b200_session_pos": (U32, [P]),
    "pai_b200_session_reset": (I32, [P]),
    "pai_b200_session_step": (I32, [P, P, P, P]),
    "pai_b200_session_run": (I32, [P, U32]),
    "pai_b200_session_prefill": (I32, [P, P, U32, P]),
    "pai_b200_session_set_tokens": (I32, [P, P]),
    "pai_b200_session_get_tokens": (I32, [P, P]),
    "pai_b200_session_hidden": (P, [P]),
    "pai_b200_session_kv_info": (I32, [P, P]),
    "pai_b200_session_step_kernels": (U32, [P]),
    "pai_b200_session_run_layers": (I32, [P, U32]),
    "pai_b200_session_kv_reserve": (I32, [P, U32, P]),
}


def load():
    """Load the built library; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C prosperoai_b200/csrc` "
                "(or __graft_entry__.build()); prosperoai_b200 has no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, what: str) -> None:
    if status != PAI_OK:
        raise PaiError(status, what, load().pai_b200_last_error().decode())
