"""The operator API: one function per reference operator ``forward``.

Positional parameters keep the names and order of the reference's per-operator
numpy ``forward`` functions (the NKIBench case files the reference drives,
restated in ``workspaces/<op>/runs/offline_*_sim.py``); keyword arguments extend
them to the north-star configurations with defaults that reproduce the
reference semantics.  Inputs are CUDA tensors in natural (untiled) row-major
layout; contractions take bf16, elementwise / scan ops fp32 (the scan's x may
be bf16).  Violations raise ``ValueError`` before any launch.  Every op runs a
hand-written sm_100a kernel in libkda.so through its C ABI -- there is no CPU
or PyTorch fallback.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib

_bf16 = torch.bfloat16
_f32 = torch.float32


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _p(t: Optional[torch.Tensor]):
    return C.c_void_p(0 if t is None else t.data_ptr())


def _check(t, name, dtypes, ndim=None, shape=None, device=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not isinstance(dtypes, tuple):
        dtypes = (dtypes,)
    if t.dtype not in dtypes:
        raise ValueError(f"{name} must have dtype {' or '.join(map(str, dtypes))}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _out(out, shape, dtype, device, name="out"):
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    _check(out, name, dtype, shape=shape, device=device)
    return out


def _workspace(ws, nbytes, device):
    """The caller's workspace (checked: on `device`, at least `nbytes`), or a
    fresh one when none was given."""
    if ws is None:
        return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)
    if ws.device != device:
        raise ValueError(f"workspace is on {ws.device}, the operands on {device}")
    if ws.numel() * ws.element_size() < nbytes:
        raise ValueError(f"workspace of {int(nbytes)} bytes required, got {ws.numel() * ws.element_size()}")
    return ws


class _on:
    """Make ``t``'s device current for the duration of a library call."""

    def __init__(self, t):
        self.ctx = torch.cuda.device(t.device)

    def __enter__(self):
        self.ctx.__enter__()

    def __exit__(self, *exc):
        return self.ctx.__exit__(*exc)


# ----------------------------------------------------------------- elementwise
def silu(x, *, out=None):
    """y = x / (1 + exp(-x)), fp32 (reference silu ``forward(x)``)."""
    _check(x, "x", _f32)
    y = _out(out, x.shape, _f32, x.device)
    with _on(x):
        _lib.call("kda_silu_f32", _p(x), _p(y), x.numel(), _stream(x))
    return y


def rope_single_freq_apply(x_in, cos, sin, *, out=None):
    """Half-split RoPE over the leading axis: x_in (D, S), cos/sin (D/2, S)."""
    _check(x_in, "x_in", _f32, ndim=2)
    D, S = x_in.shape
    if D % 2:
        raise ValueError(f"x_in leading dim {D} must be even")
    _check(cos, "cos", _f32, shape=(D // 2, S), device=x_in.device)
    _check(sin, "sin", _f32, shape=(D // 2, S), device=x_in.device)
    y = _out(out, x_in.shape, _f32, x_in.device)
    with _on(x_in):
        _lib.call("kda_rope_single_freq_apply_f32", _p(x_in), _p(cos), _p(sin), _p(y), D, S, _stream(x_in))
    return y


def adamw(theta, g, m, v, *, inplace_state=False, out=None):
    """One AdamW step (reference constants); returns theta'.

    ``inplace_state=True`` also writes m' and v' into ``m`` and ``v``.
    """
    _check(theta, "theta", _f32)
    for n, t in (("g", g), ("m", m), ("v", v)):
        _check(t, n, _f32, shape=theta.shape, device=theta.device)
    y = _out(out, theta.shape, _f32, theta.device)
    with _on(theta):
        _lib.call("kda_adamw_f32", _p(theta), _p(g), _p(m), _p(v), _p(y), theta.numel(),
                  int(bool(inplace_state)), _stream(theta))
    return y


# --------------------------------------------------------------------- scan
def adamw_multi(params, grads, exp_avgs, exp_avg_sqs, *, lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                weight_decay=1e-2, step=1):
    """AdamW over lists of fp32 CUDA tensors, in place (params, exp_avgs,
    exp_avg_sqs): one kernel launch per 48 tensors, each tensor cut into
    4096-element blocks.  Decoupled weight decay and bias correction at
    ``step``; the defaults (step 1) give exactly ``adamw``'s update."""
    n = len(params)
    if not (len(grads) == len(exp_avgs) == len(exp_avg_sqs) == n):
        raise ValueError("params, grads, exp_avgs and exp_avg_sqs must have the same length")
    if n == 0:
        return
    if int(step) < 1:
        raise ValueError(f"step must be >= 1, got {step}")
    dev = params[0].device if isinstance(params[0], torch.Tensor) else None
    ptrs = [[], [], [], []]
    sizes = []
    for i in range(n):
        ts = (params[i], grads[i], exp_avgs[i], exp_avg_sqs[i])
        for name, t in zip(("params", "grads", "exp_avgs", "exp_avg_sqs"), ts):
            _check(t, f"{name}[{i}]", _f32, device=dev)
            if t.numel() != ts[0].numel():
                raise ValueError(f"{name}[{i}] has {t.numel()} elements, params[{i}] {ts[0].numel()}")
        for j, t in enumerate(ts):
            ptrs[j].append(t.data_ptr())
        sizes.append(ts[0].numel())
    arrs = [(C.c_void_p * n)(*p) for p in ptrs]
    b1, b2 = betas
    with _on(params[0]):
        _lib.call("kda_adamw_multi_f32", *arrs, (C.c_int64 * n)(*sizes), n, float(lr), float(b1), float(b2),
                  float(eps), float(weight_decay), int(step), _stream(params[0]))


def mamba(delta, u, a, b, c, D=None, *, out_dtype=None, out=None, workspace=None):
    """Selective scan with fp32 state (d_state 16).

    Reference 2-D layout: delta, u (C, M); a (C, S); b, c (S, M) -> (C, M).
    Batched channels-last: delta (dt) fp32 and u (x) fp32/bf16 (B, L, D);
    a (A) (D, 16); b, c (B, L, 16); optional D (D,) -> y (B, L, D).
    ``out_dtype`` defaults to u's dtype.
    """
    _check(delta, "delta", _f32)
    dev = delta.device
    _check(u, "u", (_f32, _bf16), shape=delta.shape, device=dev)
    if delta.dim() == 2:
        Cn, M = delta.shape
        _check(a, "a", _f32, ndim=2, device=dev)
        S = a.shape[1]
        _check(a, "a", _f32, shape=(Cn, S))
        _check(b, "b", _f32, shape=(S, M), device=dev)
        _check(c, "c", _f32, shape=(S, M), device=dev)
        batch, L, Dm = 1, M, Cn
        ld = (Cn * M, 1, M)
        bc = (S * M, 1, M)
    elif delta.dim() == 3:
        batch, L, Dm = delta.shape
        _check(a, "a", _f32, ndim=2, device=dev)
        S = a.shape[1]
        _check(a, "a", _f32, shape=(Dm, S))
        _check(b, "b", _f32, shape=(batch, L, S), device=dev)
        _check(c, "c", _f32, shape=(batch, L, S), device=dev)
        ld = (L * Dm, Dm, 1)
        bc = (L * S, S, 1)
    else:
        raise ValueError(f"delta must be 2-D (C, M) or 3-D (B, L, D), got {tuple(delta.shape)}")
    if D is not None:
        _check(D, "D", _f32, shape=(Dm,), device=dev)
    odt = out_dtype or u.dtype
    if odt not in (_f32, _bf16):
        raise ValueError(f"out_dtype must be float32 or bfloat16, got {odt}")
    y = _out(out, delta.shape, odt, dev)
    nb = _ws_size("kda_mamba_scan_workspace_size", batch, L, Dm, S)
    ws = _workspace(workspace, nb, dev) if nb else None
    with _on(delta):
        _lib.call("kda_mamba_scan", _p(delta), _p(u), _p(a), _p(b), _p(c), _p(D), _p(y), batch, L, Dm, S,
                  *ld, *bc, int(u.dtype == _bf16), int(odt == _bf16), _p(ws), nb, _stream(delta))
    return y


# ------------------------------------------------------------- contractions
def matmul(lhs, rhs, *, out=None, workspace=None):
    """lhs (M,K) @ rhs (K,N), fp32 accumulate: bf16 in -> bf16 out; fp32 in ->
    fp32 out at fp32 accuracy (bf16 hi + lo split of both operands on the
    tensor core, hi.hi + hi.lo + lo.hi; needs a workspace, allocated when not given)."""
    if getattr(lhs, "dtype", None) == _f32:
        return _matmul_f32(lhs, rhs, out=out, workspace=workspace)
    _check(lhs, "lhs", _bf16, ndim=2)
    M, K = lhs.shape
    _check(rhs, "rhs", _bf16, ndim=2, device=lhs.device)
    if rhs.shape[0] != K:
        raise ValueError(f"rhs must be ({K}, N), got {tuple(rhs.shape)}")
    N = rhs.shape[1]
    y = _out(out, (M, N), _bf16, lhs.device)
    with _on(lhs):
        _lib.call("kda_matmul_bf16", _p(lhs), _p(rhs), _p(y), M, K, N, _stream(lhs))
    return y


def _matmul_f32(lhs, rhs, *, out=None, workspace=None):
    _check(lhs, "lhs", _f32, ndim=2)
    M, K = lhs.shape
    _check(rhs, "rhs", _f32, ndim=2, device=lhs.device)
    if rhs.shape[0] != K:
        raise ValueError(f"rhs must be ({K}, N), got {tuple(rhs.shape)}")
    N = rhs.shape[1]
    y = _out(out, (M, N), _f32, lhs.device)
    nb = _ws_size("kda_matmul_f32_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, lhs.device)
    with _on(lhs):
        _lib.call("kda_matmul_f32", _p(lhs), _p(rhs), _p(y), M, K, N, _p(ws), nb, _stream(lhs))
    return y


def transpose_matmul(lhs, rhs, *, out=None, workspace=None):
    """lhs.T @ rhs with lhs stored (K, M): bf16 in -> bf16 out; fp32 in -> fp32
    out at fp32 accuracy (the bf16 hi + lo split of ``matmul``; needs a
    workspace, allocated when not given)."""
    if getattr(lhs, "dtype", None) == _f32:
        _check(lhs, "lhs", _f32, ndim=2)
        K, M = lhs.shape
        _check(rhs, "rhs", _f32, ndim=2, device=lhs.device)
        if rhs.shape[0] != K:
            raise ValueError(f"rhs must be ({K}, N), got {tuple(rhs.shape)}")
        N = rhs.shape[1]
        y = _out(out, (M, N), _f32, lhs.device)
        nb = _ws_size("kda_transpose_matmul_f32_workspace_size", M, K, N)
        ws = _workspace(workspace, nb, lhs.device)
        with _on(lhs):
            _lib.call("kda_transpose_matmul_f32", _p(lhs), _p(rhs), _p(y), M, K, N, _p(ws), nb, _stream(lhs))
        return y
    _check(lhs, "lhs", _bf16, ndim=2)
    K, M = lhs.shape
    _check(rhs, "rhs", _bf16, ndim=2, device=lhs.device)
    if rhs.shape[0] != K:
        raise ValueError(f"rhs must be ({K}, N), got {tuple(rhs.shape)}")
    N = rhs.shape[1]
    y = _out(out, (M, N), _bf16, lhs.device)
    with _on(lhs):
        _lib.call("kda_transpose_matmul_bf16", _p(lhs), _p(rhs), _p(y), M, K, N, _stream(lhs))
    return y


def _bmm_shapes(lhs, rhs, dtype=_bf16):
    _check(lhs, "lhs", dtype, ndim=3)
    Bn, M, K = lhs.shape
    _check(rhs, "rhs", dtype, ndim=3, device=lhs.device)
    if rhs.shape[0] != Bn or rhs.shape[1] != K:
        raise ValueError(f"rhs must be ({Bn}, {K}, N), got {tuple(rhs.shape)}")
    return Bn, M, K, rhs.shape[2]


def bmm(lhs, rhs, *, out=None, workspace=None):
    """out[b] = lhs[b] @ rhs[b]: bf16 in -> bf16 out; fp32 in -> fp32 out at
    fp32 accuracy (bf16 hi + lo split; needs a workspace, allocated when not
    given)."""
    if getattr(lhs, "dtype", None) == _f32:
        Bn, M, K, N = _bmm_shapes(lhs, rhs, _f32)
        y = _out(out, (Bn, M, N), _f32, lhs.device)
        nb = _ws_size("kda_bmm_f32_workspace_size", Bn, M, K, N)
        ws = _workspace(workspace, nb, lhs.device)
        with _on(lhs):
            _lib.call("kda_bmm_f32", _p(lhs), _p(rhs), _p(y), Bn, M, K, N, _p(ws), nb, _stream(lhs))
        return y
    Bn, M, K, N = _bmm_shapes(lhs, rhs)
    y = _out(out, (Bn, M, N), _bf16, lhs.device)
    with _on(lhs):
        _lib.call("kda_bmm_bf16", _p(lhs), _p(rhs), _p(y), Bn, M, K, N, _stream(lhs))
    return y


def bmm_softmax(lhs, rhs, *, out=None, workspace=None):
    """softmax over axis 2 of lhs @ rhs (max-shifted): bf16 in -> bf16 out;
    fp32 in -> fp32 out at fp32 accuracy (workspace allocated when not given)."""
    if getattr(lhs, "dtype", None) == _f32:  # fp32 in / out at fp32 accuracy
        Bn, M, K, N = _bmm_shapes(lhs, rhs, _f32)
        y = _out(out, (Bn, M, N), _f32, lhs.device)
        nb = _ws_size("kda_bmm_softmax_f32_workspace_size", Bn, M, K, N)
        ws = _workspace(workspace, nb, lhs.device)
        with _on(lhs):
            _lib.call("kda_bmm_softmax_f32", _p(lhs), _p(rhs), _p(y), Bn, M, K, N, _p(ws), nb, _stream(lhs))
        return y
    Bn, M, K, N = _bmm_shapes(lhs, rhs)
    y = _out(out, (Bn, M, N), _bf16, lhs.device)
    with _on(lhs):
        _lib.call("kda_bmm_softmax_bf16", _p(lhs), _p(rhs), _p(y), Bn, M, K, N, _stream(lhs))
    return y


def _kind(t):
    """(dtype, workspace-query suffix) of an operator's path: fp32 operands run
    the fp32-accuracy path, anything else the bf16 path (whose checks then
    reject a wrong dtype)."""
    if getattr(t, "dtype", None) == _f32:
        return _f32, "_f32"
    return _bf16, ""


def _dt_name(dt):
    return "f32" if dt == _f32 else "bf16"


def _ws_size(name, *dims):
    h = _lib.lib()
    return int(_lib._attach(h, name)(*dims))


def rmsnorm_matmul(x, w, g=None, eps=0.0, *, out=None, workspace=None):
    """(x / sqrt(mean_k x^2 + eps) * g) @ w; g=None, eps=0 is the reference.
    bf16 x, w -> bf16 out; fp32 x, w -> fp32 out at fp32 accuracy."""
    dt, sfx = _kind(x)
    _check(x, "x", dt, ndim=2)
    M, K = x.shape
    _check(w, "w", dt, ndim=2, device=x.device)
    if w.shape[0] != K:
        raise ValueError(f"w must be ({K}, N), got {tuple(w.shape)}")
    N = w.shape[1]
    if g is not None:
        _check(g, "g", _f32, shape=(K,), device=x.device)
    y = _out(out, (M, N), dt, x.device)
    nb = _ws_size(f"kda_rmsnorm_matmul{sfx}_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call(f"kda_rmsnorm_matmul_{_dt_name(dt)}", _p(x), _p(w), _p(g), float(eps), _p(y), M, K, N, _p(ws),
                  nb, _stream(x))
    return y


def rmsnorm_matmul_backward(dy, x, w, g=None, eps=0.0, *, workspace=None):
    """Gradients of ``rmsnorm_matmul(x, w, g, eps)`` given dy (M,N) bf16:
    returns (dx bf16 (M,K), dw bf16 (K,N), dg fp32 (K,) or None when g is None)."""
    _check(x, "x", _bf16, ndim=2)
    M, K = x.shape
    _check(w, "w", _bf16, ndim=2, device=x.device)
    if w.shape[0] != K:
        raise ValueError(f"w must be ({K}, N), got {tuple(w.shape)}")
    N = w.shape[1]
    _check(dy, "dy", _bf16, shape=(M, N), device=x.device)
    if g is not None:
        _check(g, "g", _f32, shape=(K,), device=x.device)
    dx = torch.empty(M, K, dtype=_bf16, device=x.device)
    dw = torch.empty(K, N, dtype=_bf16, device=x.device)
    dg = torch.empty(K, dtype=_f32, device=x.device) if g is not None else None
    nb = _ws_size("kda_rmsnorm_matmul_backward_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call("kda_rmsnorm_matmul_backward_bf16", _p(dy), _p(x), _p(w), _p(g), float(eps), _p(dx), _p(dw),
                  _p(dg), M, K, N, _p(ws), nb, _stream(x))
    return dx, dw, dg


def add_rmsnorm_matmul(x, w, eps, z, g, *, out=None, workspace=None):
    """a = x + z; (a / sqrt(mean_k a^2 + eps) * g) @ w.
    bf16 x, z, w -> bf16 out; fp32 x, z, w -> fp32 out at fp32 accuracy."""
    dt, sfx = _kind(x)
    _check(x, "x", dt, ndim=2)
    M, K = x.shape
    _check(w, "w", dt, ndim=2, device=x.device)
    if w.shape[0] != K:
        raise ValueError(f"w must be ({K}, N), got {tuple(w.shape)}")
    N = w.shape[1]
    _check(z, "z", dt, shape=(M, K), device=x.device)
    _check(g, "g", _f32, shape=(K,), device=x.device)
    y = _out(out, (M, N), dt, x.device)
    nb = _ws_size(f"kda_add_rmsnorm_matmul{sfx}_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call(f"kda_add_rmsnorm_matmul_{_dt_name(dt)}", _p(x), _p(w), float(eps), _p(z), _p(g), _p(y), M, K,
                  N, _p(ws), nb, _stream(x))
    return y


def matmul_add_rmsnorm(x, w, eps, z, g, *, out=None, workspace=None):
    """y = x @ w + z; y * g / sqrt(mean_n y^2 + eps).
    bf16 x, w, z -> bf16 out; fp32 x, w, z -> fp32 out at fp32 accuracy."""
    dt, sfx = _kind(x)
    _check(x, "x", dt, ndim=2)
    M, K = x.shape
    _check(w, "w", dt, ndim=2, device=x.device)
    if w.shape[0] != K:
        raise ValueError(f"w must be ({K}, N), got {tuple(w.shape)}")
    N = w.shape[1]
    _check(z, "z", dt, shape=(M, N), device=x.device)
    _check(g, "g", _f32, shape=(N,), device=x.device)
    y = _out(out, (M, N), dt, x.device)
    nb = _ws_size(f"kda_matmul_add_rmsnorm{sfx}_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call(f"kda_matmul_add_rmsnorm_{_dt_name(dt)}", _p(x), _p(w), float(eps), _p(z), _p(g), _p(y), M, K,
                  N, _p(ws), nb, _stream(x))
    return y


def swiglu(x, w_up, w_down, w_gate, *, out=None, workspace=None):
    """(silu(x @ w_gate) * (x @ w_up)) @ w_down; x (M,K), w_up/w_gate (K,N), w_down (N,K).
    bf16 in -> bf16 out (h stored bf16); fp32 in -> fp32 out at fp32 accuracy (fp32 h)."""
    dt, sfx = _kind(x)
    _check(x, "x", dt, ndim=2)
    M, K = x.shape
    _check(w_up, "w_up", dt, ndim=2, device=x.device)
    if w_up.shape[0] != K:
        raise ValueError(f"w_up must be ({K}, N), got {tuple(w_up.shape)}")
    N = w_up.shape[1]
    _check(w_gate, "w_gate", dt, shape=(K, N), device=x.device)
    _check(w_down, "w_down", dt, shape=(N, K), device=x.device)
    y = _out(out, (M, K), dt, x.device)
    nb = _ws_size(f"kda_swiglu{sfx}_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call(f"kda_swiglu_{_dt_name(dt)}", _p(x), _p(w_up), _p(w_down), _p(w_gate), _p(y), M, K, N, _p(ws),
                  nb, _stream(x))
    return y


def _swiglu_shapes(x, w_up, w_down, w_gate):
    _check(x, "x", _bf16, ndim=2)
    M, K = x.shape
    _check(w_up, "w_up", _bf16, ndim=2, device=x.device)
    if w_up.shape[0] != K:
        raise ValueError(f"w_up must be ({K}, N), got {tuple(w_up.shape)}")
    N = w_up.shape[1]
    _check(w_gate, "w_gate", _bf16, shape=(K, N), device=x.device)
    _check(w_down, "w_down", _bf16, shape=(N, K), device=x.device)
    return M, K, N


def swiglu_gu(x, w_up, w_down, w_gate, *, workspace=None):
    """``swiglu`` for a training step (bf16): returns (out, g, u) with
    g = x @ w_gate and u = x @ w_up (M, N) kept for
    ``swiglu_backward(..., g=g, u=u)``.  Unfused (h = silu(g) * u from the
    bf16 g, u), so out can differ from ``swiglu``'s in the last bf16 bit."""
    M, K, N = _swiglu_shapes(x, w_up, w_down, w_gate)
    out = torch.empty((M, K), dtype=_bf16, device=x.device)
    g = torch.empty((M, N), dtype=_bf16, device=x.device)
    u = torch.empty_like(g)
    nb = _ws_size("kda_swiglu_gu_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call("kda_swiglu_gu_bf16", _p(x), _p(w_up), _p(w_down), _p(w_gate), _p(out), _p(g), _p(u), M, K, N,
                  _p(ws), nb, _stream(x))
    return out, g, u


def swiglu_backward(dout, x, w_up, w_down, w_gate, *, g=None, u=None, workspace=None):
    """Gradients of ``swiglu(x, w_up, w_down, w_gate)`` given dout (M,K) bf16:
    returns (dx, dw_up, dw_down, dw_gate), bf16, shaped like x, w_up, w_down, w_gate.

    With ``g`` and ``u`` from ``swiglu_gu`` (same x and weights) the two GEMMs
    that recompute them are skipped."""
    M, K, N = _swiglu_shapes(x, w_up, w_down, w_gate)
    _check(dout, "dout", _bf16, shape=(M, K), device=x.device)
    if (g is None) != (u is None):
        raise ValueError("g and u must be given together")
    saved = g is not None
    if saved:
        _check(g, "g", _bf16, shape=(M, N), device=x.device)
        _check(u, "u", _bf16, shape=(M, N), device=x.device)
    dx, dwu, dwd, dwg = (torch.empty_like(t) for t in (x, w_up, w_down, w_gate))
    name = "kda_swiglu_backward_saved" if saved else "kda_swiglu_backward"
    nb = _ws_size(name + "_workspace_size", M, K, N)
    ws = _workspace(workspace, nb, x.device)
    extra = (_p(g), _p(u)) if saved else ()
    with _on(x):
        _lib.call(name + "_bf16", _p(dout), _p(x), _p(w_up), _p(w_down), _p(w_gate), *extra, _p(dx), _p(dwu),
                  _p(dwd), _p(dwg), M, K, N, _p(ws), nb, _stream(x))
    return dx, dwu, dwd, dwg


def lora(x, w, a, b, *, out=None, workspace=None):
    """x @ w + (x @ a) @ b: bf16 in -> bf16 out; fp32 in -> fp32 out at fp32
    accuracy (fp32 t = x @ a)."""
    dt, sfx = _kind(x)
    _check(x, "x", dt, ndim=2)
    M, K = x.shape
    _check(w, "w", dt, ndim=2, device=x.device)
    if w.shape[0] != K:
        raise ValueError(f"w must be ({K}, N), got {tuple(w.shape)}")
    N = w.shape[1]
    _check(a, "a", dt, ndim=2, device=x.device)
    if a.shape[0] != K:
        raise ValueError(f"a must be ({K}, R), got {tuple(a.shape)}")
    R = a.shape[1]
    _check(b, "b", dt, shape=(R, N), device=x.device)
    y = _out(out, (M, N), dt, x.device)
    nb = _ws_size(f"kda_lora{sfx}_workspace_size", M, K, N, R)
    ws = _workspace(workspace, nb, x.device)
    with _on(x):
        _lib.call(f"kda_lora_{_dt_name(dt)}", _p(x), _p(w), _p(a), _p(b), _p(y), M, K, N, R, _p(ws), nb,
                  _stream(x))
    return y


def gqa_full(q, k, v, causal=False, rope_theta=None, *, out_layout="bhsd", out=None, workspace=None):
    """Grouped-query attention (head_dim 128), q (B,S,QH,D), k/v (B,S,KH,D).

    Returns the reference order (B, QH, S, D) by default; ``out_layout="bshd"``
    returns (B, S, QH, D).  ``causal`` masks keys after the query position;
    ``rope_theta`` applies half-split RoPE to q and k first.  fp32 q, k, v
    run the fp32-accuracy path (head by head, any head_dim that is a multiple
    of 32, no RoPE) and return fp32.
    """
    dt, _ = _kind(q)
    _check(q, "q", dt, ndim=4)
    B, S, QH, D = q.shape
    _check(k, "k", dt, ndim=4, device=q.device)
    KH = k.shape[2]
    _check(k, "k", dt, shape=(B, S, KH, D))
    _check(v, "v", dt, shape=(B, S, KH, D), device=q.device)
    if KH == 0 or QH % KH:
        raise ValueError(f"query heads {QH} must be a multiple of kv heads {KH}")
    if out_layout not in ("bhsd", "bshd"):
        raise ValueError(f"out_layout must be 'bhsd' or 'bshd', got {out_layout!r}")
    shape = (B, QH, S, D) if out_layout == "bhsd" else (B, S, QH, D)
    y = _out(out, shape, dt, q.device)
    theta = float(rope_theta) if rope_theta else 0.0
    if dt == _f32:
        if theta > 0:
            raise ValueError("rope_theta is not supported with fp32 q, k, v")
        nb = _ws_size("kda_gqa_full_f32_workspace_size", B, S, QH, KH, D)
        ws = _workspace(workspace, nb, q.device)
        with _on(q):
            _lib.call("kda_gqa_full_f32", _p(q), _p(k), _p(v), _p(y), B, S, QH, KH, D, int(bool(causal)),
                      0.0, int(out_layout == "bshd"), _p(ws), nb, _stream(q))
        return y
    nb = _ws_size("kda_gqa_full_workspace_size", B, S, QH, KH, D, theta)
    ws = _workspace(workspace, nb, q.device) if nb else None
    with _on(q):
        _lib.call("kda_gqa_full_bf16", _p(q), _p(k), _p(v), _p(y), B, S, QH, KH, D, int(bool(causal)),
                  theta, int(out_layout == "bshd"), _p(ws), nb, _stream(q))
    return y


def gqa_full_lse(q, k, v, causal=False, rope_theta=None, *, workspace=None):
    """``gqa_full`` (bf16, head_dim 128) that also returns each query row's
    log2-sum-exp of the scaled scores: (out (B, QH, S, D) bf16 in the reference
    order, lse (B, QH, S) fp32) -- the forward of a training step, whose two
    outputs ``gqa_full_backward(..., fwd_out=out, lse=lse)`` takes instead of
    recomputing the forward."""
    _check(q, "q", _bf16, ndim=4)
    B, S, QH, D = q.shape
    _check(k, "k", _bf16, ndim=4, device=q.device)
    KH = k.shape[2]
    _check(k, "k", _bf16, shape=(B, S, KH, D))
    _check(v, "v", _bf16, shape=(B, S, KH, D), device=q.device)
    if KH == 0 or QH % KH:
        raise ValueError(f"query heads {QH} must be a multiple of kv heads {KH}")
    y = torch.empty((B, QH, S, D), dtype=_bf16, device=q.device)
    lse = torch.empty((B, QH, S), dtype=torch.float32, device=q.device)
    theta = float(rope_theta) if rope_theta else 0.0
    nb = _ws_size("kda_gqa_full_workspace_size", B, S, QH, KH, D, theta)
    ws = _workspace(workspace, nb, q.device) if nb else None
    with _on(q):
        _lib.call("kda_gqa_full_lse_bf16", _p(q), _p(k), _p(v), _p(y), _p(lse), B, S, QH, KH, D, int(bool(causal)),
                  theta, 0, _p(ws), nb, _stream(q))
    return y, lse


def gqa_full_backward(dout, q, k, v, causal=False, rope_theta=None, *, fwd_out=None, lse=None, workspace=None):
    """Gradients of ``gqa_full(q, k, v, causal, rope_theta)`` given dout in the
    reference order (B, QH, S, D) bf16: returns (dq, dk, dv) shaped like q, k, v.

    With ``fwd_out`` and ``lse`` from ``gqa_full_lse`` (same q, k, v, causal,
    rope_theta) the forward is not run again."""
    _check(q, "q", _bf16, ndim=4)
    B, S, QH, D = q.shape
    _check(k, "k", _bf16, ndim=4, device=q.device)
    KH = k.shape[2]
    _check(k, "k", _bf16, shape=(B, S, KH, D))
    _check(v, "v", _bf16, shape=(B, S, KH, D), device=q.device)
    if KH == 0 or QH % KH:
        raise ValueError(f"query heads {QH} must be a multiple of kv heads {KH}")
    _check(dout, "dout", _bf16, shape=(B, QH, S, D), device=q.device)
    if (fwd_out is None) != (lse is None):
        raise ValueError("fwd_out and lse must be given together")
    saved = fwd_out is not None
    if saved:
        _check(fwd_out, "fwd_out", _bf16, shape=(B, QH, S, D), device=q.device)
        _check(lse, "lse", torch.float32, shape=(B, QH, S), device=q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    theta = float(rope_theta) if rope_theta else 0.0
    name = "kda_gqa_full_backward_saved" if saved else "kda_gqa_full_backward"
    nb = _ws_size(name + "_workspace_size", B, S, QH, KH, D, theta)
    ws = _workspace(workspace, nb, q.device)
    extra = (_p(fwd_out), _p(lse)) if saved else ()
    with _on(q):
        _lib.call(name + "_bf16", _p(dout), _p(q), _p(k), _p(v), *extra, _p(dq), _p(dk), _p(dv), B, S, QH, KH,
                  D, int(bool(causal)), theta, _p(ws), nb, _stream(q))
    return dq, dk, dv


def device_error(clear: bool = True) -> int:
    """Device error word of the current device (0 = no kernel wait expired)."""
    return _lib.device_error(clear)
