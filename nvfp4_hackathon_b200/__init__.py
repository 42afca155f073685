"""B200-native (sm_100a) NVFP4 block-scaled GEMM and grouped GEMM.

Drop-in modules mirroring the reference's entry points:
``nvfp4_hackathon_b200.gemm`` (custom_kernel / compile_kernel of
kernels/gemm/submission.py) and ``nvfp4_hackathon_b200.group_gemm``
(kernels/group_gemm/submission.py).  The compute path is the in-tree C-ABI
library ``libnvfp4_b200.so``; there is no other backend.
"""
from . import layout, inputs  # noqa: F401

__all__ = ["gemm", "group_gemm", "layout", "inputs", "sharding"]
