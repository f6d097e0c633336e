"""cuda-b200 backend of the ProsperoAI quantized-weights hot path.

The product is ``lib/libpai_b200.so`` (C ABI: include/pai_b200.h): C host
code plus hand-written sm_100a kernels. This package is its Python
binding for tests and benchmarks.
"""
from ._native import LIB_PATH, PaiError, Q4_0, Q4_K, Q8_0, load  # noqa: F401
