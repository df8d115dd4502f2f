"""Autograd bindings: the library's forward and backward kernels as one
differentiable op for training code.

    y = kda.autograd.rmsnorm_matmul(x, w, g, 1e-6)   # bf16 x, w; fp32 g (or None)
    y.backward(dy)                                   # x.grad, w.grad, g.grad from the kernels
    y = kda.autograd.swiglu(x, w_up, w_down, w_gate)  # bf16; all four gradients from the kernels
    o = kda.autograd.gqa_full(q, k, v, causal=True, rope_theta=1e4)  # bf16; dq, dk, dv from the kernels
"""

from __future__ import annotations

import torch

from . import ops


class _RMSNormMatmul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, g, eps):
        ctx.save_for_backward(x, w, g)
        ctx.eps = float(eps)
        return ops.rmsnorm_matmul(x, w, g, eps)

    @staticmethod
    def backward(ctx, dy):
        x, w, g = ctx.saved_tensors
        dx, dw, dg = ops.rmsnorm_matmul_backward(dy.to(torch.bfloat16).contiguous(), x, w, g, ctx.eps)
        return dx, dw, dg, None


def rmsnorm_matmul(x, w, g=None, eps=0.0):
    """Differentiable ``kda.rmsnorm_matmul``: gradients for x, w and g come
    from ``kda.rmsnorm_matmul_backward``."""
    return _RMSNormMatmul.apply(x, w, g, eps)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_up, w_down, w_gate):
        # the forward keeps g = x w_gate and u = x w_up, so the backward does
        # not recompute them
        out, g, u = ops.swiglu_gu(x, w_up, w_down, w_gate)
        ctx.save_for_backward(x, w_up, w_down, w_gate, g, u)
        return out

    @staticmethod
    def backward(ctx, dout):
        x, w_up, w_down, w_gate, g, u = ctx.saved_tensors
        return ops.swiglu_backward(dout.to(torch.bfloat16).contiguous(), x, w_up, w_down, w_gate, g=g, u=u)


def swiglu(x, w_up, w_down, w_gate):
    """Differentiable ``kda.swiglu`` (bf16): the forward (``kda.swiglu_gu``) keeps
    g and u, the gradients come from ``kda.swiglu_backward`` on them."""
    return _SwiGLU.apply(x, w_up, w_down, w_gate)


class _GQA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, rope_theta):
        # the forward keeps its output and row log2-sum-exp, so the backward
        # does not run it again
        out, lse = ops.gqa_full_lse(q, k, v, causal=causal, rope_theta=rope_theta)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.rope_theta = bool(causal), rope_theta
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = ops.gqa_full_backward(dout.to(torch.bfloat16).contiguous(), q, k, v, causal=ctx.causal,
                                           rope_theta=ctx.rope_theta, fwd_out=out, lse=lse)
        return dq, dk, dv, None, None


def gqa_full(q, k, v, causal=False, rope_theta=None):
    """Differentiable ``kda.gqa_full`` (bf16; output in the reference order
    (B, QH, S, D)): the forward keeps its row log2-sum-exp, the gradients come
    from ``kda.gqa_full_backward`` on the saved forward."""
    return _GQA.apply(q, k, v, causal, rope_theta)
