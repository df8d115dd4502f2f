"""kda-b200: B200-native (sm_100a) fused operators with the reference's signatures.

    import kda
    y = kda.silu(x)                      # x: fp32 CUDA tensor
    out = kda.rmsnorm_matmul(x, w, g, 1e-6)

All work runs in hand-written CUDA kernels in ``libkda.so`` (C ABI in
``include/kda.h``); importing this package loads that library and fails if it
has not been built (``python kda-for-trainium_b200/build.py``).  Importing it
also registers the operators as ``torch.ops.kda.<op>`` (``kda.library``) and
provides the numpy-in / numpy-out shim ``kda.compat.<op>``.
"""

from ._lib import KdaError, lib as _load_lib
from .ops import (  # noqa: F401
    adamw, adamw_multi, add_rmsnorm_matmul, bmm, bmm_softmax, device_error, gqa_full, gqa_full_backward,
    gqa_full_lse, lora,
    mamba, matmul, matmul_add_rmsnorm, rmsnorm_matmul, rmsnorm_matmul_backward, rope_single_freq_apply, silu, swiglu,
    swiglu_backward, swiglu_gu, transpose_matmul,
)

OPS = ("silu", "rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "swiglu", "matmul",
       "transpose_matmul", "bmm", "bmm_softmax", "gqa_full", "rope_single_freq_apply", "lora", "adamw",
       "mamba")

_load_lib()

from . import compat, library  # noqa: E402,F401  (torch.ops.kda.<op> and the numpy shim)

__all__ = list(OPS) + ["adamw_multi", "rmsnorm_matmul_backward", "swiglu_backward", "gqa_full_backward",
                       "gqa_full_lse", "swiglu_gu", "KdaError", "device_error"]
