"""The C ABI used from C, the reference's host language, with no Python in
between: a program that includes only include/pai_b200.h and links
libpai_b200.so compiles as ISO C11 and runs the calls a ProsperoAI host
makes before it has a GPU (no GPU needed):

- op registration into a registry already holding the 28 builtin ops
  (runtime/op_registry.c:367-377), and the descriptors' capability bit;
- the v0 blob size of a quantized .pai tensor (models/quantize.c:53-72);
- GGUF inspection status codes (a missing file: PAI_ERR_IO);
- pai_b200_init reporting the absence of a device with PAI_ERR_INIT.
"""
import os
import subprocess

import pytest

from prosperoai_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "pai_b200.h"

int main(void) {
  static pai_op_registry_t reg;
  reg.version = 1;
  reg.count = 28; /* the builtin table */
  if (pai_b200_register_ops(&reg) != PAI_OK) return 1;
  if (reg.count != 28 + pai_b200_op_count()) return 2;
  for (uint32_t i = 28; i < reg.count; i++)
    if (!(reg.ops[i]->caps & PAI_OP_CAP_CUDA_B200)) return 3;
  /* q8, 32 per group, a 4096 x 4096 tensor: values + one f32 scale per group */
  if (pai_b200_v0_blob_bytes(8, 32, 4096ull * 4096ull) != 4096ull * 4096ull + 4096ull * 4096ull / 32 * 4) return 4;
  pai_b200_gguf_info_t info;
  if (pai_b200_gguf_inspect("/nonexistent/model.gguf", &info) != PAI_ERR_IO) return 5;
  int n = -1;
  if (pai_b200_device_count(&n) != PAI_OK) return 6;
  if (n == 0) {
    pai_b200_ctx_t *ctx = NULL;
    if (pai_b200_init(0, &ctx) != PAI_ERR_INIT || ctx != NULL) return 7;
  }
  printf("ok %u ops\n", pai_b200_op_count());
  return 0;
}
"""


def test_c_program_uses_the_abi(tmp_path):
    lib_dir = os.path.dirname(_native.LIB_PATH)
    if not os.path.exists(_native.LIB_PATH):
        pytest.fail(f"{_native.LIB_PATH} is missing: build the library first")
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                    "-L", lib_dir, "-lpai_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok ")
