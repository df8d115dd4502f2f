"""The fourteen operators as ``torch.library`` custom ops: ``torch.ops.kda.<op>``.

Each op calls the same ``kda.ops`` function (and so the same libkda.so entry
point, with the same host checks raising ``ValueError`` before any launch) and
has a fake (meta) implementation that gives the output's shape and dtype
without running anything, so the ops trace under ``FakeTensorMode`` and
``torch.compile`` / ``torch.export`` see them as opaque calls.  Positional
parameters keep the reference forwards' names and order; the keyword
extensions of ``kda.ops`` that select semantics (gamma / eps, causal, RoPE,
output layout and dtype) are schema arguments with the same defaults.
Buffers (``out=``, ``workspace=``) are not part of the schema: the custom ops
allocate their outputs and scratch through torch's caching allocator.

Reference forwards: ``prompts/_gen_prompts.py:19-254`` and
``workspaces/<op>/runs/offline_*_sim.py`` (cited per op in ``kda.ops``).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops

_f32 = torch.float32
_bf16 = torch.bfloat16


def _contraction_dtype(t: torch.Tensor) -> torch.dtype:
    # fp32 operands take the fp32-accuracy path and return fp32; otherwise bf16
    return _f32 if t.dtype == _f32 else _bf16


# ----------------------------------------------------------------- elementwise
@torch.library.custom_op("kda::silu", mutates_args=())
def silu(x: torch.Tensor) -> torch.Tensor:
    return ops.silu(x)


@silu.register_fake
def _(x):
    return torch.empty_like(x, dtype=_f32)


@torch.library.custom_op("kda::rope_single_freq_apply", mutates_args=())
def rope_single_freq_apply(x_in: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return ops.rope_single_freq_apply(x_in, cos, sin)


@rope_single_freq_apply.register_fake
def _(x_in, cos, sin):
    return torch.empty_like(x_in, dtype=_f32)


@torch.library.custom_op("kda::adamw", mutates_args=())
def adamw(theta: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return ops.adamw(theta, g, m, v)


@adamw.register_fake
def _(theta, g, m, v):
    return torch.empty_like(theta, dtype=_f32)


@torch.library.custom_op("kda::mamba", mutates_args=())
def mamba(delta: torch.Tensor, u: torch.Tensor, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor,
          D: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    return ops.mamba(delta, u, a, b, c, D, out_dtype=out_dtype)


@mamba.register_fake
def _(delta, u, a, b, c, D=None, out_dtype=None):
    return delta.new_empty(delta.shape, dtype=out_dtype or u.dtype)


# ---------------------------------------------------------------- contractions
@torch.library.custom_op("kda::matmul", mutates_args=())
def matmul(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    return ops.matmul(lhs, rhs)


@matmul.register_fake
def _(lhs, rhs):
    return lhs.new_empty((lhs.shape[0], rhs.shape[1]), dtype=_contraction_dtype(lhs))


@torch.library.custom_op("kda::transpose_matmul", mutates_args=())
def transpose_matmul(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    return ops.transpose_matmul(lhs, rhs)


@transpose_matmul.register_fake
def _(lhs, rhs):
    return lhs.new_empty((lhs.shape[1], rhs.shape[1]), dtype=_contraction_dtype(lhs))


@torch.library.custom_op("kda::bmm", mutates_args=())
def bmm(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    return ops.bmm(lhs, rhs)


@bmm.register_fake
def _(lhs, rhs):
    return lhs.new_empty((lhs.shape[0], lhs.shape[1], rhs.shape[2]), dtype=_contraction_dtype(lhs))


@torch.library.custom_op("kda::bmm_softmax", mutates_args=())
def bmm_softmax(lhs: torch.Tensor, rhs: torch.Tensor) -> torch.Tensor:
    return ops.bmm_softmax(lhs, rhs)


@bmm_softmax.register_fake
def _(lhs, rhs):
    return lhs.new_empty((lhs.shape[0], lhs.shape[1], rhs.shape[2]), dtype=_contraction_dtype(lhs))


@torch.library.custom_op("kda::rmsnorm_matmul", mutates_args=())
def rmsnorm_matmul(x: torch.Tensor, w: torch.Tensor, g: Optional[torch.Tensor] = None,
                   eps: float = 0.0) -> torch.Tensor:
    return ops.rmsnorm_matmul(x, w, g, eps)


@rmsnorm_matmul.register_fake
def _(x, w, g=None, eps=0.0):
    return x.new_empty((x.shape[0], w.shape[1]), dtype=_contraction_dtype(x))


@torch.library.custom_op("kda::add_rmsnorm_matmul", mutates_args=())
def add_rmsnorm_matmul(x: torch.Tensor, w: torch.Tensor, eps: float, z: torch.Tensor,
                       g: torch.Tensor) -> torch.Tensor:
    return ops.add_rmsnorm_matmul(x, w, eps, z, g)


@add_rmsnorm_matmul.register_fake
def _(x, w, eps, z, g):
    return x.new_empty((x.shape[0], w.shape[1]), dtype=_contraction_dtype(x))


@torch.library.custom_op("kda::matmul_add_rmsnorm", mutates_args=())
def matmul_add_rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, z: torch.Tensor,
                       g: torch.Tensor) -> torch.Tensor:
    return ops.matmul_add_rmsnorm(x, w, eps, z, g)


@matmul_add_rmsnorm.register_fake
def _(x, w, eps, z, g):
    return x.new_empty((x.shape[0], w.shape[1]), dtype=_contraction_dtype(x))


@torch.library.custom_op("kda::swiglu", mutates_args=())
def swiglu(x: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, w_gate: torch.Tensor) -> torch.Tensor:
    return ops.swiglu(x, w_up, w_down, w_gate)


@swiglu.register_fake
def _(x, w_up, w_down, w_gate):
    return x.new_empty((x.shape[0], w_down.shape[1]), dtype=_contraction_dtype(x))


@torch.library.custom_op("kda::lora", mutates_args=())
def lora(x: torch.Tensor, w: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return ops.lora(x, w, a, b)


@lora.register_fake
def _(x, w, a, b):
    return x.new_empty((x.shape[0], w.shape[1]), dtype=_contraction_dtype(x))


@torch.library.custom_op("kda::gqa_full", mutates_args=())
def gqa_full(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
             rope_theta: Optional[float] = None, out_layout: str = "bhsd") -> torch.Tensor:
    return ops.gqa_full(q, k, v, causal, rope_theta, out_layout=out_layout)


@gqa_full.register_fake
def _(q, k, v, causal=False, rope_theta=None, out_layout="bhsd"):
    B, S, QH, D = q.shape
    shape = (B, QH, S, D) if out_layout == "bhsd" else (B, S, QH, D)
    return q.new_empty(shape, dtype=_contraction_dtype(q))


OPS = ("silu", "rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "swiglu", "matmul",
       "transpose_matmul", "bmm", "bmm_softmax", "gqa_full", "rope_single_freq_apply", "lora", "adamw",
       "mamba")
