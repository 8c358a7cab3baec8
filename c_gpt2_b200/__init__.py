"""B200-native (sm_100a) W8A8 inference path for GPT-2.

Native pieces (built in-tree by ``python -m c_gpt2_b200.build``):
  lib/libgpt2_w8a8.so            kernels + C host engine, C ABI in include/
  lib/libcuda_kernels_<size>.so  drop-in for the reference's cuda_kernels.h

Python modules: ``ops`` (torch front end of the kernel ABI), ``engine``
(batched generation), ``quant8`` (the reference's weight formats),
``synthetic`` (seeded workloads).
"""
from .quant8 import DIMS, GPT2Dims  # noqa: F401

__all__ = ["DIMS", "GPT2Dims"]
