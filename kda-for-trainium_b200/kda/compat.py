"""numpy in, numpy out: the reference forwards' calling convention.

The reference scores each operator through a numpy ``forward`` whose
parameters come from ``get_numpy_inputs()`` as a dict keyed by the forward's
parameter names (``adapter/nkibench_case.py:147-155``) and returns a float32
array.  ``kda.compat.<op>(**get_numpy_inputs())`` is that call on a B200: the
arrays are uploaded to the current CUDA device, the library's operator runs,
and the result comes back as a float32 numpy array.

Precision: by default the matrix operands of the contractions are rounded to
bf16 (round to nearest even) on upload and the bf16 tensor-core path runs --
the library's bf16 policy.  ``strict_fp32=True`` uploads them as fp32 and runs
each contraction's fp32-accuracy path (bf16 hi + lo split operands), whose
results meet the reference's own fp32 gate.  silu, rope, adamw and mamba are
fp32 operators either way.  Scalars (eps) pass through unchanged.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import ops

# matrix operands uploaded as bf16 on the default path (gamma vectors stay fp32)
_BF16_ARGS = {
    "matmul": ("lhs", "rhs"),
    "transpose_matmul": ("lhs", "rhs"),
    "bmm": ("lhs", "rhs"),
    "bmm_softmax": ("lhs", "rhs"),
    "rmsnorm_matmul": ("x", "w"),
    "add_rmsnorm_matmul": ("x", "w", "z"),
    "matmul_add_rmsnorm": ("x", "w", "z"),
    "swiglu": ("x", "w_up", "w_down", "w_gate"),
    "lora": ("x", "w", "a", "b"),
    "gqa_full": ("q", "k", "v"),
}


def _run(op: str, arrays: dict, strict_fp32: bool, device, **kw) -> np.ndarray:
    for name, v in arrays.items():
        if not (v is None or isinstance(v, (np.ndarray, int, float))):
            raise TypeError(f"{op}: argument {name!r} must be a numpy array or a number, got {type(v).__name__}")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    bf = () if strict_fp32 else _BF16_ARGS.get(op, ())
    args = {}
    for name, v in arrays.items():
        if isinstance(v, np.ndarray):
            t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(dev)
            args[name] = t.to(torch.bfloat16) if name in bf else t
        else:
            args[name] = v
    out = getattr(ops, op)(**args, **kw)
    return out.float().cpu().numpy()


def silu(x, *, device=None) -> np.ndarray:
    return _run("silu", {"x": x}, False, device)


def rope_single_freq_apply(x_in, cos, sin, *, device=None) -> np.ndarray:
    return _run("rope_single_freq_apply", {"x_in": x_in, "cos": cos, "sin": sin}, False, device)


def adamw(theta, g, m, v, *, device=None) -> np.ndarray:
    return _run("adamw", {"theta": theta, "g": g, "m": m, "v": v}, False, device)


def mamba(delta, u, a, b, c, D=None, *, device=None) -> np.ndarray:
    return _run("mamba", {"delta": delta, "u": u, "a": a, "b": b, "c": c, "D": D}, False, device)


def matmul(lhs, rhs, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("matmul", {"lhs": lhs, "rhs": rhs}, strict_fp32, device)


def transpose_matmul(lhs, rhs, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("transpose_matmul", {"lhs": lhs, "rhs": rhs}, strict_fp32, device)


def bmm(lhs, rhs, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("bmm", {"lhs": lhs, "rhs": rhs}, strict_fp32, device)


def bmm_softmax(lhs, rhs, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("bmm_softmax", {"lhs": lhs, "rhs": rhs}, strict_fp32, device)


def rmsnorm_matmul(x, w, g=None, eps: float = 0.0, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("rmsnorm_matmul", {"x": x, "w": w, "g": g, "eps": float(eps)}, strict_fp32, device)


def add_rmsnorm_matmul(x, w, eps, z, g, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("add_rmsnorm_matmul", {"x": x, "w": w, "eps": float(eps), "z": z, "g": g}, strict_fp32, device)


def matmul_add_rmsnorm(x, w, eps, z, g, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("matmul_add_rmsnorm", {"x": x, "w": w, "eps": float(eps), "z": z, "g": g}, strict_fp32, device)


def swiglu(x, w_up, w_down, w_gate, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("swiglu", {"x": x, "w_up": w_up, "w_down": w_down, "w_gate": w_gate}, strict_fp32, device)


def lora(x, w, a, b, *, strict_fp32: bool = False, device=None) -> np.ndarray:
    return _run("lora", {"x": x, "w": w, "a": a, "b": b}, strict_fp32, device)


def gqa_full(q, k, v, causal: bool = False, rope_theta: Optional[float] = None, *, strict_fp32: bool = False,
             device=None) -> np.ndarray:
    """Returns the reference order (B, QH, S, D)."""
    return _run("gqa_full", {"q": q, "k": k, "v": v, "causal": bool(causal), "rope_theta": rope_theta},
                strict_fp32, device)


OPS = ("silu", "rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "swiglu", "matmul",
       "transpose_matmul", "bmm", "bmm_softmax", "gqa_full", "rope_single_freq_apply", "lora", "adamw",
       "mamba")
