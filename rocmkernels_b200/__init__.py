"""B200 (sm_100a) FP32 attention: the ROCmKernels attention entry points on NVIDIA Blackwell.

The product is the C-ABI library ``librocmkernels_attention.so`` (declared in
``include/rocmkernels_attention.h``); this package builds it (:mod:`.build`), binds it with
ctypes under the reference's names (:mod:`.attention`) and plans multi-GPU shards
(:mod:`.sharding`).
"""
from .attention import (  # noqa: F401
    ENTRY_POINTS,
    HipError,
    Strides,
    build_info,
    lib,
    strides_of,
)
from .attention import *  # noqa: F401,F403
