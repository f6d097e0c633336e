"""Host-side checks of libpai_b200.so that need no GPU.

The library must load and export every function include/pai_b200.h
declares; the host quantiser must produce the same ggml bytes as the CPU
restatement of the quantisation formulas; the op descriptors must be
layout-compatible with the reference's pai_op_descriptor_t.
"""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import _native
from prosperoai_b200.api import quantize, rope_tables

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pai_b200.h")
REF = po.reference_dir()


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pai_b200_\w+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    L = _native.load()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    assert set(declared_functions()) <= set(_native.SIGNATURES), "ctypes signature table incomplete"
    assert b"sm_100a" in L.pai_b200_version()


def test_library_exports_only_the_declared_abi():
    """Dynamic symbol table of libpai_b200.so: the declared pai_b200_* entry
    points and nothing else (internal helpers, kernel templates and the
    statically linked CUDA runtime stay local)."""
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    assert exported == set(declared_functions()), sorted(exported ^ set(declared_functions()))


def test_host_quantiser_matches_restated_formulas():
    rng = np.random.default_rng(11)
    for t in (po.Q4_0, po.Q8_0, po.Q4_K):
        el = po.BLOCK[t][0]
        w = (rng.standard_normal(el * 300) * 0.02).astype(np.float32)
        w[:el] = 0.0                    # an all-zero block
        w[el:2 * el] = np.abs(w[el:2 * el])  # all-positive block
        w[2 * el:3 * el] = -np.abs(w[2 * el:3 * el])
        assert np.array_equal(quantize(t, w), po.quantize(t, w)), t


# Q8_0: half a step plus the fp16 rounding of d (127 * 2^-11 steps);
# Q4_0: the extreme of the opposite sign clamps at +7, up to one step.
@pytest.mark.parametrize("t,step", [(po.Q8_0, 0.6 / 127), (po.Q4_0, 1.01 / 8), (po.Q4_K, 1.0)])
def test_quantise_round_trip_error_bound(t, step):
    rng = np.random.default_rng(3)
    el = po.BLOCK[t][0]
    w = (rng.standard_normal(el * 200) * 0.02).astype(np.float32)
    back = po.dequant(t, quantize(t, w), w.size)
    err = np.abs(back - w).reshape(-1, el)
    amax = np.abs(w).reshape(-1, el).max(axis=1)
    if t == po.Q4_K:
        bound = (w.reshape(-1, 32).max(1) - np.minimum(0, w.reshape(-1, 32).min(1)))
        assert (np.abs(back - w).reshape(-1, 32).max(1) <= bound / 15 * 1.3 + 1e-6).all()
    else:
        assert (err.max(axis=1) <= amax * step + 1e-7).all()


def test_quantise_rejects_ragged_input():
    with pytest.raises(_native.PaiError) as e:
        quantize(po.Q4_0, np.zeros(33, np.float32))
    assert e.value.status == -6  # PAI_ERR_MISMATCH


def test_rope_tables_match_reference_formula():
    c1, s1 = rope_tables(100, 64, 500000.0)
    c2, s2 = po.rope_tables(100, 64, 500000.0)
    assert np.array_equal(c1, c2) and np.array_equal(s1, s2)


def test_registry_registration():
    reg = _native.OpRegistry()
    reg.version, reg.count = 1, 28  # a registry already holding the 28 builtin ops
    L = _native.load()
    _native.check(L.pai_b200_register_ops(C.byref(reg)), "register_ops")
    n = L.pai_b200_op_count()
    assert reg.count == 28 + n
    names = {reg.ops[28 + i].contents.name.decode() for i in range(n)}
    assert {"gemv_q4_0_f32", "gemv_q8_0_f32", "gemv_q4_k_f32", "attention_decode_f16kv"} <= names
    for i in range(n):
        d = reg.ops[28 + i].contents
        assert d.caps == 1 << 3 and 14 <= d.kernel_id <= 30
    full = _native.OpRegistry()
    full.count = 60
    assert L.pai_b200_register_ops(C.byref(full)) == -2  # PAI_ERR_NOMEM: 64-op cap


def test_init_without_gpu_reports_error():
    L = _native.load()
    n = C.c_int(-1)
    assert L.pai_b200_device_count(C.byref(n)) == 0
    if n.value > 0:
        pytest.skip("a GPU is present")
    ctx = C.c_void_p()
    assert L.pai_b200_init(0, C.byref(ctx)) == -8  # PAI_ERR_INIT
    assert b"no CUDA device" in L.pai_b200_last_error()


@pytest.mark.skipif(not os.path.exists(f"{REF}/sdk/include/pai/op.h"),
                    reason="reference headers not present")
def test_descriptor_layout_matches_reference(tmp_path):
    """Compile the reference's pai/op.h and this header separately and
    compare sizes and field offsets."""
    probe = r"""
#include <stdio.h>
#include <stddef.h>
#include HDR
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu\n", sizeof(pai_op_descriptor_t),
         offsetof(pai_op_descriptor_t, caps), offsetof(pai_op_descriptor_t, ref_fn),
         offsetof(pai_op_descriptor_t, kernel_id), offsetof(pai_op_descriptor_t, reserved),
         sizeof(pai_op_registry_t), offsetof(pai_op_registry_t, ops));
  return 0;
}
"""
    src = tmp_path / "probe.c"
    src.write_text(probe)
    outs = []
    for hdr, inc in (("<pai/op.h>", f"-I{REF}/sdk/include"), ('"pai_b200.h"', f"-I{ROOT}/include")):
        exe = tmp_path / f"probe{len(outs)}"
        subprocess.run(["gcc", "-std=c11", inc, f"-DHDR={hdr}", str(src), "-o", str(exe)], check=True)
        outs.append(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert outs[0] == outs[1], outs


@pytest.mark.skipif(po.ref() is None, reason="reference build (oracle/_ref) not present")
def test_v0_blob_bytes_match_reference():
    """pai_b200_v0_blob_bytes is the reference's pai_quant_weights_bytes
    (models/quantize.c:53-72): packed values plus one f32 scale per group."""
    L = _native.load()
    R = po.ref()
    for bits in (8, 4):
        for gs in (0, 1, 7, 32, 4096, 65535):
            for n in (1, 2, 33, 1000, 4096 * 4096):
                want = R.pai_quant_weights_bytes(n, C.byref(po.QuantScheme(bits, 1, gs)))
                assert L.pai_b200_v0_blob_bytes(bits, gs, n) == want, (bits, gs, n)


@pytest.mark.skipif(po.ref() is None, reason="reference build (oracle/_ref) not present")
def test_ops_register_into_the_reference_registry():
    """The reference's own registry code (runtime/op_registry.c, compiled in
    oracle/_ref): pai_op_registry_builtin, then pai_b200_register_ops on the
    same registry; the reference's lookups then find this backend's ops by
    name and by kernel id, the builtins are untouched, the capability gate
    pai_op_supports sees PAI_OP_CAP_CUDA_B200, and the reference's eager
    CPU path refuses them (no CPU fallback: ref_fn is NULL)."""
    from prosperoai_b200._native import OpDescriptor, OpRegistry
    L = _native.load()
    R = po.ref()
    DP = C.POINTER(OpDescriptor)
    R.pai_op_registry_builtin.restype = C.c_int32
    R.pai_op_registry_lookup.restype = DP
    R.pai_op_registry_lookup.argtypes = [C.c_void_p, C.c_char_p]
    R.pai_op_registry_lookup_kernel.restype = DP
    R.pai_op_registry_lookup_kernel.argtypes = [C.c_void_p, C.c_int32]
    R.pai_op_supports.restype = C.c_uint32
    R.pai_op_supports.argtypes = [DP, C.c_uint32]
    R.pai_op_eval_f32.restype = C.c_int32
    R.pai_op_eval_f32.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_uint32, C.c_void_p,
                                  C.c_uint32, C.c_void_p, C.c_uint32]
    reg = OpRegistry()
    assert R.pai_op_registry_builtin(C.byref(reg)) == 0
    builtin = reg.count
    matmul = R.pai_op_registry_lookup(C.byref(reg), b"matmul_f32")
    assert L.pai_b200_register_ops(C.byref(reg)) == 0
    assert reg.count == builtin + L.pai_b200_op_count()
    cuda_b200 = 1 << 3
    for name, kid, wfmt, warg in ((b"gemv_q4_0_f32", 15, 2, 1), (b"gemv_q8_0_f32", 14, 8, 1),
                                  (b"gemv_q4_k_f32", 16, 12, 1), (b"gemm_q4_0_f32", 17, 2, 2),
                                  (b"gemm_q8_0_f32", 29, 8, 2), (b"gemm_q4_k_f32", 30, 12, 2),
                                  (b"attention_decode_f16kv", 20, 0, 0)):
        d = R.pai_op_registry_lookup(C.byref(reg), name)
        assert d, name
        assert d.contents.name == name and d.contents.kernel_id == kid
        assert tuple(d.contents.reserved) == (wfmt, warg)  # the quantized weight operand
        assert R.pai_op_supports(d, cuda_b200) == 1 and R.pai_op_supports(d, 1) == 0
        k = R.pai_op_registry_lookup_kernel(C.byref(reg), kid)
        assert C.addressof(k.contents) == C.addressof(d.contents)
        # the reference's eager path: a vocabulary-only entry for it
        assert R.pai_op_eval_f32(C.byref(reg), name, None, d.contents.num_inputs, None,
                                 d.contents.num_outputs, None, 0) == -3  # PAI_ERR_UNSUPPORTED
    after = R.pai_op_registry_lookup(C.byref(reg), b"matmul_f32")
    assert (not matmul and not after) or C.addressof(after.contents) == C.addressof(matmul.contents)


def slice_inputs(wtype, m, n, k, seed):
    rng = np.random.default_rng(seed)
    blocks = quantize(wtype, (rng.standard_normal(n * k) * 0.05).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    res = rng.standard_normal((m, n)).astype(np.float32)
    return blocks, x, gamma, res


@pytest.mark.parametrize("wtype,m,k", [(po.Q4_0, 1, 256), (po.Q8_0, 1, 256), (po.Q4_K, 1, 512),
                                       (po.Q4_0, 8, 256), (po.Q4_K, 4, 256)])
def test_reference_scheduler_plans_gates_and_runs_the_slice(wtype, m, k):
    """The reference's graph builder, memory planner, scheduler, registry and
    executor (graph.c, planner.c, scheduler.c, op_registry.c compiled from its
    sources into oracle/_ref) over rmsnorm -> projection -> residual add, each
    op hinted to the GPU. The reference's own gate pai_kernel_plan_check passes
    for PAI_OP_CAP_CPU_REF and refuses PAI_OP_CAP_CUDA_B200 (its name map,
    scheduler.c:647-682, picks the f32 builtins); the gate over the name map
    extended with the quantized names passes once this backend is registered.
    The executor's host result is rmsnorm, the dense product with the
    reference-dequantised weights, and the add."""
    R = po.ref()
    if R is None:
        pytest.skip("reference checkout not built into oracle/_ref")
    n = 96
    blocks, x, gamma, res = slice_inputs(wtype, m, n, k, seed=m * 7 + k + wtype)
    rep, cpu, _ = po.dispatch_slice(_native.LIB_PATH, False, wtype, m, n, k, blocks, x, gamma, res)
    assert rep.num_steps == 3 and rep.gpu_steps == 3, rep.error
    assert list(rep.devices[:3]) == [2, 2, 2]  # PAI_SCHED_DEV_GPU
    assert rep.gate_cpu_ref == 0
    assert rep.gate_b200_ref_map == -3  # PAI_ERR_UNSUPPORTED
    assert rep.gate_b200 == 0
    assert rep.cpu_status == 0 and rep.gpu_status == 1  # the GPU branch did not run
    w = po.dequant(wtype, blocks, n * k).reshape(n, k).astype(np.float64)
    want = po.rmsnorm_gamma(x, gamma).astype(np.float64) @ w.T + res
    assert np.max(np.abs(cpu - want)) <= 1e-4 * max(1.0, float(np.max(np.abs(want))))


def test_b200_gate_refuses_a_block_type_without_a_kernel():
    """Q5_0 weights (ggml type 6): the reference executor still runs the slice
    on the host, and the cuda-b200 gate refuses the plan (no descriptor)."""
    R = po.ref()
    if R is None:
        pytest.skip("reference checkout not built into oracle/_ref")
    m, n, k = 1, 64, 128
    rng = np.random.default_rng(5)
    blocks = rng.integers(0, 256, n * k // 32 * 22, dtype=np.uint8)
    blocks.reshape(-1, 22)[:, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    x = rng.standard_normal(k).astype(np.float32)
    rep, cpu, _ = po.dispatch_slice(_native.LIB_PATH, False, 6, m, n, k, blocks, x,
                                    np.ones(k, np.float32), np.zeros(n, np.float32))
    assert rep.gate_cpu_ref == 0 and rep.cpu_status == 0
    assert rep.gate_b200 == -3 and rep.gate_b200_ref_map == -3
    assert np.all(np.isfinite(cpu))
