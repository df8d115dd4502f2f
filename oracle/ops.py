"""numpy restatements of the reference operator forwards (TEST INFRASTRUCTURE).

Each function takes numpy arrays whose values are already in the dtype the
GPU path consumes (bf16 inputs arrive as fp32 arrays holding bf16-rounded
values, see ``oracle.bf16``) and computes in fp32 with float64 row reductions,
so a parity test measures kernel error, not input-quantisation error.
Positional parameters keep the reference ``forward``'s names and order;
keyword extensions default to the reference (NKIBench) semantics.

Citations are paths inside the reference project (Jerry2423/kda-for-trainium).
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


# --------------------------------------------------------------------------- #
# elementwise / bandwidth-bound
# --------------------------------------------------------------------------- #
def silu(x):
    """y = x / (1 + exp(-x)).

    Spec: ``prompts/_gen_prompts.py:25`` ("SiLU / swish: y = x / (1 + exp(-x))");
    the same expression is the swiglu helper at
    ``workspaces/swiglu/runs/offline_bf16_split_sim.py:87-89``.
    """
    x = np.asarray(x, dtype=f32)
    with np.errstate(over="ignore"):
        return (x / (f32(1.0) + np.exp(-x))).astype(f32)


def rope_single_freq_apply(x_in, cos, sin):
    """Half-split rotation over the leading (D) axis.

    x_in (D, S), cos/sin (D/2, S):
        out[:D/2] = x0*cos - x1*sin ; out[D/2:] = x0*sin + x1*cos
    Spec: ``workspaces/rope_single_freq_apply/runs/rope_v1.py:5-8`` and
    ``prompts/_gen_prompts.py:143-144``; layout (identity transform)
    ``workspaces/rope_single_freq_apply/docs/draft-phase1.md:36-49``.
    """
    x_in = np.asarray(x_in, dtype=f32)
    h = x_in.shape[0] // 2
    x0, x1 = x_in[:h], x_in[h:]
    out0 = x0 * cos - x1 * sin
    out1 = x0 * sin + x1 * cos
    return np.concatenate([out0, out1], axis=0).astype(f32)


def adamw(theta, g, m, v):
    """One AdamW step with the reference's literal constants; returns theta'.

    m' = 0.9 m + 0.1 g ; v' = 0.999 v + 0.001 g^2 ;
    theta' = theta - 1e-5 theta - 0.01 m' / (sqrt(1000 v') + 1e-8)
    Spec: ``prompts/_gen_prompts.py:227-228``; ``workspaces/adamw/runs/adamw_v1.py:5-11``.
    (The reference kernel folds constants and drops eps; this keeps the formula.)
    """
    theta, g, m, v = (np.asarray(a, dtype=f32) for a in (theta, g, m, v))
    theta_t = theta - f32(1e-5) * theta
    m_t = f32(0.9) * m + f32(0.1) * g
    v_t = f32(0.999) * v + f32(0.001) * g * g
    v_hat = v_t * f32(1000.0)
    return (theta_t - f32(0.01) * m_t / (np.sqrt(v_hat) + f32(1e-8))).astype(f32)


def adamw_state(theta, g, m, v):
    """(theta', m', v') -- the in-place-state variant's three outputs."""
    g, m, v = (np.asarray(a, dtype=f32) for a in (g, m, v))
    m_t = (f32(0.9) * m + f32(0.1) * g).astype(f32)
    v_t = (f32(0.999) * v + f32(0.001) * g * g).astype(f32)
    return adamw(theta, g, m, v), m_t, v_t


def adamw_step(theta, g, m, v, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, step=1):
    """(theta', m', v') of AdamW with decoupled weight decay and bias
    correction, in fp32 with the scalars folded in float64:
    theta' = (theta - lr*wd*theta) - lr/(1-b1^t) * m' / (sqrt(v' / (1-b2^t)) + eps).
    At lr 1e-3, betas (0.9, 0.999), eps 1e-8, wd 1e-2, t = 1 this is ``adamw``
    (``workspaces/adamw/runs/adamw_v1.py:5-11``), the step the reference's
    operator performs."""
    theta, g, m, v = (np.asarray(a, dtype=f32) for a in (theta, g, m, v))
    b1, b2 = betas
    m_t = (f32(b1) * m + f32(1.0 - b1) * g).astype(f32)
    v_t = (f32(b2) * v + f32(1.0 - b2) * g * g).astype(f32)
    step_size = f32(lr / (1.0 - b1 ** step))
    bc2 = f32(1.0 / (1.0 - b2 ** step))
    th = (theta - f32(lr * weight_decay) * theta) - step_size * m_t / (np.sqrt(v_t * bc2) + f32(eps))
    return th.astype(f32), m_t, v_t


# --------------------------------------------------------------------------- #
# selective scan
# --------------------------------------------------------------------------- #
def mamba(delta, u, a, b, c, D=None):
    """Selective-scan SSM with fp32 state, h_0 = 0.

    NKIBench layout (2-D): delta, u (C, M); a (C, S); b, c (S, M) -> out (C, M)
        dA = exp(delta*a), dBu = delta*b*u, s_i = dA_i s_{i-1} + dBu_i,
        out = sum_S c*s
    (``workspaces/mamba/docs/draft-phase1.md:22-29``, ``prompts/_gen_prompts.py:244-246``,
    kernel semantics ``workspaces/mamba/runs/mamba_v1.py:8-84``).

    Batched channels-last layout (3-D): delta = dt, u = x (B, L, D);
    a = A (D, N); b, c = B, C (B, L, N); optional D (D,) skip term:
        h_t = exp(dt_t*A) h_{t-1} + dt_t B_t x_t ; y_t = C_t . h_t + D x_t
    The loop runs over the sequence axis with an (…, D, N) fp32 state and
    never materialises the (B, L, D, N) tensor.
    """
    delta = np.asarray(delta, dtype=f32)
    u = np.asarray(u, dtype=f32)
    a = np.asarray(a, dtype=f32)
    b = np.asarray(b, dtype=f32)
    c = np.asarray(c, dtype=f32)
    if delta.ndim == 2:
        # (C, M) channel-major -> (1, M, C) channels-last, b/c (S, M) -> (1, M, S)
        y = mamba(delta.T[None], u.T[None], a, b.T[None], c.T[None], D)
        return np.ascontiguousarray(y[0].T)
    Bt, L, Dm = delta.shape
    N = a.shape[1]
    h = np.zeros((Bt, Dm, N), dtype=f32)
    y = np.empty((Bt, L, Dm), dtype=f32)
    for t in range(L):
        dt = delta[:, t, :]                                    # (B, D)
        dA = np.exp(dt[:, :, None] * a[None, :, :])            # (B, D, N)
        dBx = (dt * u[:, t, :])[:, :, None] * b[:, t, None, :]  # (B, D, N)
        h = dA * h + dBx
        y[:, t, :] = np.einsum("bdn,bn->bd", h, c[:, t, :])
    if D is not None:
        y = y + np.asarray(D, dtype=f32)[None, None, :] * u
    return y.astype(f32)


# --------------------------------------------------------------------------- #
# contractions
# --------------------------------------------------------------------------- #
def _mm(a, b):
    return np.matmul(np.asarray(a, dtype=f32), np.asarray(b, dtype=f32)).astype(f32)


def matmul(lhs, rhs):
    """lhs @ rhs.  ``workspaces/matmul/runs/offline_bf16_split_sim.py:137-139``."""
    return _mm(lhs, rhs)


def transpose_matmul(lhs, rhs):
    """lhs.T @ rhs, lhs stored (K, M).
    ``workspaces/transpose_matmul/runs/offline_bf16_split_sim.py:101-104``."""
    return _mm(np.asarray(lhs, dtype=f32).T, rhs)


def bmm(lhs, rhs):
    """out[b] = lhs[b] @ rhs[b].  ``workspaces/bmm/runs/offline_bf16_split_sim.py:102-104``
    (its fp32 control reproduces the reference)."""
    return _mm(lhs, rhs)


def _softmax_lastaxis(s):
    s = s - np.max(s, axis=-1, keepdims=True)
    e = np.exp(s).astype(f32)
    return (e / np.sum(e, axis=-1, keepdims=True, dtype=np.float64)).astype(f32)


def bmm_softmax(lhs, rhs):
    """softmax over axis 2 of lhs@rhs, max-shifted.
    Spec ``prompts/_gen_prompts.py:176-177``; per-row algorithm
    ``workspaces/bmm_softmax/runs/bmm_softmax_v4.py:20-27``."""
    lhs = np.asarray(lhs, dtype=f32)
    rhs = np.asarray(rhs, dtype=f32)
    out = np.empty(lhs.shape[:2] + rhs.shape[2:], dtype=f32)
    for i in range(lhs.shape[0]):
        out[i] = _softmax_lastaxis(_mm(lhs[i], rhs[i]))
    return out


def _row_inv_rms(a, eps, denom):
    ss = np.sum(np.square(a.astype(np.float64)), axis=-1, keepdims=True)
    return (1.0 / np.sqrt(ss / denom + eps)).astype(f32)


def rmsnorm_matmul(x, w, g=None, eps=0.0):
    """out = (x / sqrt(mean_k x^2 + eps) * g) @ w.

    NKIBench (g=None, eps=0): divide-by-K inside the sum, sqrt, divide, matmul
    (``workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:83-93``).
    g and eps extend it to the RMSNorm->GEMM configuration.
    """
    x = np.asarray(x, dtype=f32)
    a = x * _row_inv_rms(x, eps, x.shape[-1])
    if g is not None:
        a = a * np.asarray(g, dtype=f32)
    return _mm(a, w)


def rmsnorm_matmul_backward(dy, x, w, g=None, eps=0.0):
    """(dx, dw, dg) of ``rmsnorm_matmul`` given dy, in float64 (dg None when g is):
    xn = x r, r = 1/sqrt(mean_k x^2 + eps); dA = dy w^T; dw = (xn g)^T dy;
    dg = sum_m dA xn; dx = r (dA g - xn mean_k(dA g xn)).  The derivative of the
    forward at ``workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:83-93``
    (the reference itself has no backward)."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    dy = np.asarray(dy, dtype=np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    xn = x * r
    gg = np.ones(x.shape[-1]) if g is None else np.asarray(g, dtype=np.float64)
    dA = dy @ w.T
    dw = (xn * gg).T @ dy
    dxn = dA * gg
    dx = r * (dxn - xn * np.mean(dxn * xn, axis=-1, keepdims=True))
    dg = None if g is None else np.sum(dA * xn, axis=0)
    return dx, dw, dg


def add_rmsnorm_matmul(x, w, eps, z, g):
    """a = x + z ; out = (a / sqrt(mean_k a^2 + eps) * g) @ w.
    ``workspaces/add_rmsnorm_matmul/runs/offline_bf16_split_sim.py:97-106``."""
    a = (np.asarray(x, dtype=f32) + np.asarray(z, dtype=f32)).astype(f32)
    a = a * _row_inv_rms(a, float(eps), a.shape[-1]) * np.asarray(g, dtype=f32)
    return _mm(a, w)


def matmul_add_rmsnorm(x, w, eps, z, g):
    """y = x@w + z ; out = y * g / sqrt(mean_n y^2 + eps).
    ``workspaces/matmul_add_rmsnorm/runs/offline_bf16_split_sim.py:111-115``."""
    y = (_mm(x, w) + np.asarray(z, dtype=f32)).astype(f32)
    return (y * np.asarray(g, dtype=f32) * _row_inv_rms(y, float(eps), y.shape[-1])).astype(f32)


def swiglu(x, w_up, w_down, w_gate, h_round=None):
    """out = (silu(x@w_gate) * (x@w_up)) @ w_down.
    ``workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97``.

    ``h_round`` optionally rounds the intermediate h (e.g. ``to_bf16_rne``) to
    model an implementation that stores h in bf16; None keeps the reference's
    fp32 h.
    """
    up = _mm(x, w_up)
    gate = _mm(x, w_gate)
    h = (silu(gate) * up).astype(f32)
    if h_round is not None:
        h = h_round(h)
    return _mm(h, w_down)


def swiglu_backward(dout, x, w_up, w_down, w_gate):
    """(dx, dw_up, dw_down, dw_gate) of ``swiglu`` given dout, in float64:
    g = x w_gate, u = x w_up, h = silu(g) u; dh = dout w_down^T;
    dg = dh u silu'(g), silu'(g) = s (1 + g (1 - s)), s = sigmoid(g); du = dh silu(g);
    dw_down = h^T dout, dw_gate = x^T dg, dw_up = x^T du, dx = dg w_gate^T + du w_up^T.
    The derivative of the forward at ``workspaces/swiglu/runs/offline_bf16_split_sim.py:87-97``
    (the reference itself has no backward)."""
    x, wu, wd, wg, dout = (np.asarray(t, dtype=np.float64) for t in (x, w_up, w_down, w_gate, dout))
    g = x @ wg
    u = x @ wu
    s = 1.0 / (1.0 + np.exp(-g))
    silu_g = g * s
    h = silu_g * u
    dh = dout @ wd.T
    dg = dh * u * s * (1.0 + g * (1.0 - s))
    du = dh * silu_g
    return dg @ wg.T + du @ wu.T, x.T @ du, h.T @ dout, x.T @ dg


def lora(x, w, a, b):
    """x@w + (x@a)@b.  ``workspaces/lora/runs/offline_lora_bf16_split_sim.py:175-180``."""
    return (_mm(x, w) + _mm(_mm(x, a), b)).astype(f32)


# --------------------------------------------------------------------------- #
# attention
# --------------------------------------------------------------------------- #
def rope_tables(seq_len, head_dim, theta=10000.0):
    """cos/sin (S, D/2) for the half-split convention: angle = pos * theta^(-2i/D)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv_freq = theta ** (-2.0 * i / head_dim)
    ang = np.arange(seq_len, dtype=np.float64)[:, None] * inv_freq[None, :]
    return np.cos(ang).astype(f32), np.sin(ang).astype(f32)


def apply_rope_bshd(x, theta):
    """RoPE on (B, S, H, D) with the half-split rotation of rope_single_freq_apply."""
    x = np.asarray(x, dtype=f32)
    S, D = x.shape[1], x.shape[3]
    cos, sin = rope_tables(S, D, theta)
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    x0, x1 = x[..., : D // 2], x[..., D // 2:]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).astype(f32)


def gqa_head(q_h, k_h, v_h, causal=False, scale=None):
    """One (query-head, kv-head) pair: softmax(q k^T * scale [+mask]) v, fp32.
    ``workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:108-124``."""
    D = q_h.shape[-1]
    scale = f32(1.0 / np.sqrt(D)) if scale is None else f32(scale)
    s = (_mm(q_h, np.asarray(k_h, dtype=f32).T) * scale).astype(f32)
    if causal:
        n_q, n_k = s.shape
        mask = np.triu(np.ones((n_q, n_k), dtype=bool), k=1 + (n_k - n_q))
        s[mask] = -np.inf
    return _mm(_softmax_lastaxis(s), v_h)


def gqa_full_backward(dout, q, k, v, causal=False, rope_theta=None):
    """(dq, dk, dv) of ``gqa_full`` given dout (B, QH, S, D), float64:
    per query head h with kv head g = h // n_rep: P = softmax(q_h k_g^T s), s = 1/sqrt(D);
    dv_g += P^T dout_h; dP = dout_h v_g^T; dS = P (dP - rowsum(P dP)) s;
    dq_h = dS k_g; dk_g += dS^T q_h.  With RoPE the same on the rotated q, k,
    and dq, dk rotated back by the negated angle.  The derivative of the forward at
    ``workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124`` (the reference
    has no backward)."""
    if rope_theta:
        dq, dk, dv = gqa_full_backward(dout, apply_rope_bshd(q, rope_theta), apply_rope_bshd(k, rope_theta), v,
                                       causal)
        return _rope_inverse_bshd(dq, rope_theta), _rope_inverse_bshd(dk, rope_theta), dv
    q, k, v, dout = (np.asarray(t, dtype=np.float64) for t in (q, k, v, dout))
    B, S, QH, D = q.shape
    KH = k.shape[2]
    rep = QH // KH
    sc = 1.0 / np.sqrt(D)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    for b in range(B):
        for h in range(QH):
            g = h // rep
            qh, kg, vg, do = q[b, :, h], k[b, :, g], v[b, :, g], dout[b, h]
            s = qh @ kg.T * sc
            if causal:
                s = np.where(np.triu(np.ones((S, S), dtype=bool), k=1), -np.inf, s)
            p = np.exp(s - s.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            dv[b, :, g] += p.T @ do
            dp = do @ vg.T
            ds = p * (dp - np.sum(p * dp, -1, keepdims=True)) * sc
            dq[b, :, h] = ds @ kg
            dk[b, :, g] += ds.T @ qh
    return dq, dk, dv


def _rope_inverse_bshd(x, theta):
    """The transpose of ``apply_rope_bshd``'s rotation (by the negated angle), float64."""
    S, D = x.shape[1], x.shape[3]
    cos, sin = (t.astype(np.float64)[None, :, None, :] for t in rope_tables(S, D, theta))
    x0, x1 = x[..., : D // 2], x[..., D // 2:]
    return np.concatenate([x0 * cos + x1 * sin, -x0 * sin + x1 * cos], axis=-1)


def gqa_full(q, k, v, causal=False, rope_theta=None, out_layout="bhsd", heads=None):
    """Grouped-query attention; kv head of query head qh is qh // n_rep.

    q (B, S, QH, D), k/v (B, S, KH, D).  Reference forward: kv-repeat,
    score / sqrt(D), max-shifted softmax over keys, @ v
    (``workspaces/gqa_full/runs/offline_score_bf16_split_sim.py:100-124``,
    index maps ``workspaces/gqa_full/runs/gqa_full_v1.py:25-35``), returned in
    NKIBench order (B, QH, S, D) (``gqa_full_v1.py:30-31``); ``out_layout="bshd"``
    returns (B, S, QH, D).  ``causal`` and ``rope_theta`` extend it to the GQA
    causal + RoPE configuration.  ``heads`` optionally restricts the work to a
    list of (b, qh) pairs (others are left zero) so large shapes can be
    spot-checked.
    """
    q = np.asarray(q, dtype=f32)
    k = np.asarray(k, dtype=f32)
    v = np.asarray(v, dtype=f32)
    if rope_theta is not None:
        q = apply_rope_bshd(q, rope_theta)
        k = apply_rope_bshd(k, rope_theta)
    B, S, QH, D = q.shape
    KH = k.shape[2]
    n_rep = QH // KH
    out = np.zeros((B, QH, S, D), dtype=f32)
    todo = heads if heads is not None else [(b, h) for b in range(B) for h in range(QH)]
    for b, h in todo:
        out[b, h] = gqa_head(q[b, :, h, :], k[b, :, h // n_rep, :], v[b, :, h // n_rep, :],
                             causal=causal)
    if out_layout == "bshd":
        return np.ascontiguousarray(out.transpose(0, 2, 1, 3))
    return out
