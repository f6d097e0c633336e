"""GPU: the reference's graph executor dispatching into this backend.

oracle/ref_dispatch.c (compiled into oracle/_ref/libpai_ref.so with the
reference's graph builder, memory planner, scheduler and op registry) builds
the decoder slice rmsnorm -> projection -> residual add, plans it with the
reference's pai_sched_build (every op placed on the GPU), registers this
backend next to the builtins, and runs each GPU-placed step through the
executor's cuda-b200 branch: the descriptor selected by name, checked for
PAI_OP_CAP_CUDA_B200 and its declared quantized operand, then dispatched on
its kernel_id into libpai_b200.so (loaded by dlopen) over a device copy of
the reference memory plan's region. The same plan also runs in the
reference executor on the host with the reference-dequantised weights.
Bar: the projection part (out - res) within 1e-3 max-abs-rel for the GEMV
(decode) and 2e-2 for the bf16-tile GEMM (prompt), the bars of the op tests.
"""
import numpy as np
import pytest

from oracle import py_oracle as po
from prosperoai_b200 import _native
from test_host_lib import slice_inputs

pytestmark = pytest.mark.gpu

KID = {("gemv", po.Q4_0): 15, ("gemv", po.Q8_0): 14, ("gemv", po.Q4_K): 16,
       ("gemm", po.Q4_0): 17, ("gemm", po.Q8_0): 29, ("gemm", po.Q4_K): 30}
RMSNORM, VECADD = 18, 23


def maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("wtype,m,n,k", [(po.Q4_0, 1, 1024, 4096), (po.Q8_0, 1, 512, 4096),
                                         (po.Q4_K, 1, 768, 2048), (po.Q4_0, 16, 512, 1024),
                                         (po.Q8_0, 33, 256, 512), (po.Q4_K, 8, 256, 1024)])
def test_executor_dispatches_by_kernel_id(wtype, m, n, k):
    if po.ref() is None:
        pytest.skip("oracle/_ref/libpai_ref.so is not built")
    blocks, x, gamma, res = slice_inputs(wtype, m, n, k, seed=m * 13 + n + k + wtype)
    rep, cpu, gpu = po.dispatch_slice(_native.LIB_PATH, True, wtype, m, n, k, blocks, x,
                                      gamma, res)
    assert rep.gate_cpu_ref == 0 and rep.gate_b200_ref_map == -3 and rep.gate_b200 == 0
    assert rep.cpu_status == 0, rep.error
    assert rep.gpu_status == 0, rep.error
    op = "gemv" if m == 1 else "gemm"
    assert list(rep.kernel_ids[:3]) == [RMSNORM, KID[(op, wtype)], VECADD]
    tol = 1e-3 if m == 1 else 2e-2
    for r in range(m):
        proj_gpu = gpu[r].astype(np.float64) - res[r]
        proj_cpu = cpu[r].astype(np.float64) - res[r]
        assert maxrel(proj_gpu, proj_cpu) <= tol, (r, maxrel(proj_gpu, proj_cpu))
