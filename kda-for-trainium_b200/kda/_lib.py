"""ctypes binding of libkda.so (the C ABI declared in include/kda.h).

The library is built in-tree by ``kda-for-trainium_b200/build.py``.  There is
no fallback: if the shared library is missing, importing ``kda`` fails with an
error that says how to build it.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("KDA_LIB", Path(__file__).resolve().parent / "libkda.so"))

KDA_OK = 0
STATUS_NAMES = {0: "KDA_OK", 1: "KDA_INVALID_ARG", 2: "KDA_UNSUPPORTED", 3: "KDA_CUDA_ERROR",
                4: "KDA_TIMEOUT"}

P = C.c_void_p
I64 = C.c_int64
F = C.c_float
INT = C.c_int
SZ = C.c_size_t
D = C.c_double

# name -> (restype, argtypes); mirrors include/kda.h one to one
PROTOTYPES = {
    "kda_abi_version": (INT, []),
    "kda_status_string": (C.c_char_p, [INT]),
    "kda_last_error": (C.c_char_p, []),
    "kda_device_error": (INT, [C.POINTER(C.c_uint), INT]),
    "kda_silu_f32": (INT, [P, P, I64, P]),
    "kda_rope_single_freq_apply_f32": (INT, [P, P, P, P, I64, I64, P]),
    "kda_adamw_f32": (INT, [P, P, P, P, P, I64, INT, P]),
    "kda_mamba_scan_workspace_size": (SZ, [I64, I64, I64, I64]),
    "kda_mamba_scan": (INT, [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                             INT, INT, P, SZ, P]),
    "kda_mamba_scan_noalloc": (INT, [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64,
                                     INT, INT, P]),
    "kda_matmul_bf16": (INT, [P, P, P, I64, I64, I64, P]),
    "kda_matmul_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_matmul_f32": (INT, [P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_transpose_matmul_bf16": (INT, [P, P, P, I64, I64, I64, P]),
    "kda_transpose_matmul_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_transpose_matmul_f32": (INT, [P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_bmm_bf16": (INT, [P, P, P, I64, I64, I64, I64, P]),
    "kda_bmm_f32_workspace_size": (SZ, [I64, I64, I64, I64]),
    "kda_bmm_f32": (INT, [P, P, P, I64, I64, I64, I64, P, SZ, P]),
    "kda_bmm_softmax_bf16": (INT, [P, P, P, I64, I64, I64, I64, P]),
    "kda_rmsnorm_matmul_workspace_size": (SZ, [I64, I64, I64]),
    "kda_rmsnorm_matmul_bf16": (INT, [P, P, P, F, P, I64, I64, I64, P, SZ, P]),
    "kda_add_rmsnorm_matmul_workspace_size": (SZ, [I64, I64, I64]),
    "kda_add_rmsnorm_matmul_bf16": (INT, [P, P, F, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_matmul_add_rmsnorm_workspace_size": (SZ, [I64, I64, I64]),
    "kda_matmul_add_rmsnorm_bf16": (INT, [P, P, F, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_swiglu_workspace_size": (SZ, [I64, I64, I64]),
    "kda_swiglu_bf16": (INT, [P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_lora_workspace_size": (SZ, [I64, I64, I64, I64]),
    "kda_lora_bf16": (INT, [P, P, P, P, P, I64, I64, I64, I64, P, SZ, P]),
    "kda_gqa_full_workspace_size": (SZ, [I64, I64, I64, I64, I64, F]),
    "kda_gqa_full_bf16": (INT, [P, P, P, P, I64, I64, I64, I64, I64, INT, F, INT, P, SZ, P]),
    "kda_gqa_full_lse_bf16": (INT, [P, P, P, P, P, I64, I64, I64, I64, I64, INT, F, INT, P, SZ, P]),
    "kda_bmm_softmax_f32_workspace_size": (SZ, [I64, I64, I64, I64]),
    "kda_bmm_softmax_f32": (INT, [P, P, P, I64, I64, I64, I64, P, SZ, P]),
    "kda_rmsnorm_matmul_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_rmsnorm_matmul_f32": (INT, [P, P, P, F, P, I64, I64, I64, P, SZ, P]),
    "kda_add_rmsnorm_matmul_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_add_rmsnorm_matmul_f32": (INT, [P, P, F, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_matmul_add_rmsnorm_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_matmul_add_rmsnorm_f32": (INT, [P, P, F, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_swiglu_f32_workspace_size": (SZ, [I64, I64, I64]),
    "kda_swiglu_f32": (INT, [P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_lora_f32_workspace_size": (SZ, [I64, I64, I64, I64]),
    "kda_lora_f32": (INT, [P, P, P, P, P, I64, I64, I64, I64, P, SZ, P]),
    "kda_rmsnorm_matmul_backward_workspace_size": (SZ, [I64, I64, I64]),
    "kda_rmsnorm_matmul_backward_bf16": (INT, [P, P, P, P, F, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_swiglu_backward_workspace_size": (SZ, [I64, I64, I64]),
    "kda_swiglu_backward_bf16": (INT, [P, P, P, P, P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_swiglu_gu_workspace_size": (SZ, [I64, I64, I64]),
    "kda_swiglu_gu_bf16": (INT, [P, P, P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_swiglu_backward_saved_workspace_size": (SZ, [I64, I64, I64]),
    "kda_swiglu_backward_saved_bf16": (INT, [P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "kda_gqa_full_backward_workspace_size": (SZ, [I64, I64, I64, I64, I64, F]),
    "kda_gqa_full_backward_bf16": (INT, [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, INT, F, P, SZ, P]),
    "kda_gqa_full_backward_saved_workspace_size": (SZ, [I64, I64, I64, I64, I64, F]),
    "kda_gqa_full_backward_saved_bf16": (INT, [P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, INT, F, P, SZ,
                                               P]),
    "kda_adamw_multi_f32": (INT, [P, P, P, P, P, INT, D, D, D, D, D, I64, P]),
    "kda_ipc_handle_size": (SZ, []),
    "kda_ipc_export": (INT, [P, P, P]),
    "kda_ipc_open": (INT, [P, I64, P]),
    "kda_ipc_close": (INT, [P, I64]),
    "kda_zero1_adamw_f32": (INT, [P, P, INT, INT, I64, I64, P, P, D, D, D, D, D, I64, P]),
    "kda_gqa_full_f32_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
    "kda_gqa_full_f32": (INT, [P, P, P, P, I64, I64, I64, I64, I64, INT, F, INT, P, SZ, P]),
}


class KdaError(RuntimeError):
    """A libkda entry point returned a non-OK status."""

    def __init__(self, fn: str, status: int, detail: str):
        self.status = status
        super().__init__(f"{fn} -> {STATUS_NAMES.get(status, status)}: {detail}")


_lib = None


def lib():
    """Load libkda.so once (prototypes are attached on first use of each symbol)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"libkda.so not found at {LIB_PATH}; build it with "
                f"`python kda-for-trainium_b200/build.py` (nvcc, sm_100a)")
        h = C.CDLL(str(LIB_PATH))
        for name in ("kda_abi_version", "kda_status_string", "kda_last_error", "kda_device_error"):
            _attach(h, name)
        _lib = h
    return _lib


_attached = set()


def _attach(h, name):
    fn = getattr(h, name)
    if name not in _attached:
        res, args = PROTOTYPES[name]
        fn.restype = res
        fn.argtypes = args
        _attached.add(name)
    return fn


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise KdaError on a non-OK status."""
    h = lib()
    st = _attach(h, name)(*args)
    if st != KDA_OK:
        detail = h.kda_last_error().decode(errors="replace")
        if st == 1:
            raise ValueError(f"{name}: {detail}")
        raise KdaError(name, st, detail)


def device_error(clear: bool = True) -> int:
    """OR of the kernels' device error words on the current device (0 = none)."""
    w = C.c_uint(0)
    lib().kda_device_error(C.byref(w), int(clear))
    return int(w.value)
