"""Seeded synthetic inputs (oracle / test infrastructure).

Two families:

* ``nkibench(op, seed, **shape)`` -- the reference's natural-layout draws:
  ``np.random.seed(seed)`` once, then ``np.random.normal(0, 1, shape)`` fp32 for
  each ``forward`` argument in the reference draw order (python floats such as
  eps do not advance the RNG).  Orders follow the ``draw_inputs`` functions of
  the reference's offline simulations, e.g.
  ``workspaces/add_rmsnorm_matmul/runs/offline_bf16_split_sim.py:81-95``
  (x, w, [eps], z, g) and ``workspaces/swiglu/runs/offline_bf16_split_sim.py:77-84``
  (x, w_up, w_down, w_gate).  adamw's v is |N(0,1)| (``workspaces/adamw/runs/adamw_v1.py:19``).
  The mamba draw distribution is not recorded by the reference; the scan's
  configuration distributions (below) are used so the recurrence stays stable.

* ``config(name, seed, scale=1)`` -- the five north-star configurations with
  their distributions: N(0, 0.02) weights, gamma = 1 + 0.1 N(0,1),
  dt = softplus(N(0,1) - 3), A = -exp(N(0, 0.5)), D = 1.  ``scale`` shrinks
  the leading (row/batch/sequence) extent for fast tests.

bf16 tensors are drawn in fp32 and rounded RNE (``oracle.bf16.to_bf16_rne``);
the returned dict says which names are bf16 via ``BF16_ARGS``.
"""

from __future__ import annotations

import numpy as np

from .bf16 import to_bf16_rne

f32 = np.float32

# forward-parameter order per op (reference order), and default NKIBench shapes
# (``baselines.json`` kernel names / ``prompts/_gen_prompts.py:19-254``).
NKIBENCH_SHAPES = {
    "silu": dict(M=4096, N=7168),
    "matmul": dict(M=4096, K=5120, N=12288),
    "rmsnorm_matmul": dict(M=4096, K=1024, N=2048),
    "add_rmsnorm_matmul": dict(M=4096, K=1024, N=2048),
    "matmul_add_rmsnorm": dict(M=4096, K=2048, N=2048),
    "swiglu": dict(M=4096, K=1024, N=3072),
    "transpose_matmul": dict(M=4096, K=2048, N=10944),
    "bmm": dict(B=16, M=4096, K=64, N=4096),
    "bmm_softmax": dict(B=16, M=4096, K=64, N=4096),
    "lora": dict(M=4096, K=5120, N=12288, R=128),
    "gqa_full": dict(B=1, S=4096, QH=16, KH=8, D=128),
    "rope_single_freq_apply": dict(D=128, S=262144),
    "adamw": dict(M=10944, N=2048),
    "mamba": dict(C=256, M=7168, S=16),
}

# arguments the GPU path consumes as bf16 (contractions); everything else fp32
BF16_ARGS = {
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


def _n(shape, scale=1.0):
    return (np.random.normal(0.0, scale, size=shape)).astype(f32)


def softplus(x):
    return np.logaddexp(0.0, x).astype(f32)


def nkibench(op: str, seed: int = 42, bf16: bool = True, **shape):
    """Reference-order draws for ``op`` (dict keyed by forward parameter names)."""
    s = dict(NKIBENCH_SHAPES[op])
    s.update(shape)
    np.random.seed(seed)
    if op == "silu":
        d = {"x": _n((s["M"], s["N"]))}
    elif op == "matmul":
        d = {"lhs": _n((s["M"], s["K"])), "rhs": _n((s["K"], s["N"]))}
    elif op == "rmsnorm_matmul":
        d = {"x": _n((s["M"], s["K"])), "w": _n((s["K"], s["N"]))}
    elif op == "add_rmsnorm_matmul":
        x = _n((s["M"], s["K"]))
        w = _n((s["K"], s["N"]))
        z = _n((s["M"], s["K"]))
        g = _n((s["K"],))
        d = {"x": x, "w": w, "eps": 1e-5, "z": z, "g": g}
    elif op == "matmul_add_rmsnorm":
        x = _n((s["M"], s["K"]))
        w = _n((s["K"], s["N"]))
        z = _n((s["M"], s["N"]))
        g = _n((s["N"],))
        d = {"x": x, "w": w, "eps": 1e-5, "z": z, "g": g}
    elif op == "swiglu":
        x = _n((s["M"], s["K"]))
        w_up = _n((s["K"], s["N"]))
        w_down = _n((s["N"], s["K"]))
        w_gate = _n((s["K"], s["N"]))
        d = {"x": x, "w_up": w_up, "w_down": w_down, "w_gate": w_gate}
    elif op == "transpose_matmul":
        d = {"lhs": _n((s["K"], s["M"])), "rhs": _n((s["K"], s["N"]))}
    elif op in ("bmm", "bmm_softmax"):
        d = {"lhs": _n((s["B"], s["M"], s["K"])), "rhs": _n((s["B"], s["K"], s["N"]))}
    elif op == "lora":
        x = _n((s["M"], s["K"]))
        w = _n((s["K"], s["N"]))
        a = _n((s["K"], s["R"]))
        b = _n((s["R"], s["N"]))
        d = {"x": x, "w": w, "a": a, "b": b}
    elif op == "gqa_full":
        q = _n((s["B"], s["S"], s["QH"], s["D"]))
        k = _n((s["B"], s["S"], s["KH"], s["D"]))
        v = _n((s["B"], s["S"], s["KH"], s["D"]))
        d = {"q": q, "k": k, "v": v}
    elif op == "rope_single_freq_apply":
        d = {"x_in": _n((s["D"], s["S"])), "cos": _n((s["D"] // 2, s["S"])),
             "sin": _n((s["D"] // 2, s["S"]))}
    elif op == "adamw":
        theta = _n((s["M"], s["N"]))
        g = _n((s["M"], s["N"]))
        m = _n((s["M"], s["N"]))
        v = np.abs(_n((s["M"], s["N"])))
        d = {"theta": theta, "g": g, "m": m, "v": v}
    elif op == "mamba":
        C, M, S = s["C"], s["M"], s["S"]
        delta = softplus(_n((C, M)) - f32(3.0))
        u = _n((C, M))
        a = (-np.exp(_n((C, S), 0.5))).astype(f32)
        b = _n((S, M))
        c = _n((S, M))
        d = {"delta": delta, "u": u, "a": a, "b": b, "c": c}
    else:
        raise KeyError(op)
    if bf16:
        for k in BF16_ARGS.get(op, ()):
            d[k] = to_bf16_rne(d[k])
    return d


# --------------------------------------------------------------------------- #
# north-star configurations
# --------------------------------------------------------------------------- #
CONFIGS = {
    "silu": "SiLU fp32 x[4096,8192] ~ N(0,1)",
    "rmsnorm_matmul": "RMSNorm->GEMM X[4096,4096] bf16, gamma fp32, eps 1e-6, W[4096,11008] bf16",
    "matmul_add_rmsnorm": "GEMM+residual->RMSNorm A,B,R [4096,4096] bf16, gamma fp32, eps 1e-6",
    "swiglu": "SwiGLU X[8192,4096] bf16, W_gate/W_up [4096,14336], W_down [14336,4096]",
    "gqa_full": "GQA causal+RoPE B8 S4096 QH32 KH8 D128 bf16, theta 1e4",
    "mamba": "Mamba scan B8 L4096 D4096 N16: x bf16, dt/A/B/C/D fp32",
}


def config(name: str, seed: int = 42, scale: int = 1):
    """Inputs of a north-star configuration; ``scale`` divides the leading extent."""
    np.random.seed(seed)
    if name == "silu":
        return {"x": _n((4096 // scale, 8192))}
    if name == "rmsnorm_matmul":
        M, K, N = 4096 // scale, 4096, 11008
        x = to_bf16_rne(_n((M, K)))
        g = (f32(1.0) + f32(0.1) * _n((K,))).astype(f32)
        w = to_bf16_rne(_n((K, N), 0.02))
        return {"x": x, "w": w, "g": g, "eps": 1e-6}
    if name == "matmul_add_rmsnorm":
        M, K, N = 4096 // scale, 4096, 4096
        x = to_bf16_rne(_n((M, K)))
        g = (f32(1.0) + f32(0.1) * _n((N,))).astype(f32)
        w = to_bf16_rne(_n((K, N), 0.02))
        z = to_bf16_rne(_n((M, N)))
        return {"x": x, "w": w, "eps": 1e-6, "z": z, "g": g}
    if name == "swiglu":
        M, K, N = 8192 // scale, 4096, 14336
        x = to_bf16_rne(_n((M, K)))
        w_gate = to_bf16_rne(_n((K, N), 0.02))
        w_up = to_bf16_rne(_n((K, N), 0.02))
        w_down = to_bf16_rne(_n((N, K), 0.02))
        return {"x": x, "w_up": w_up, "w_down": w_down, "w_gate": w_gate}
    if name == "gqa_full":
        B, S, QH, KH, D = 8, 4096 // scale, 32, 8, 128
        q = to_bf16_rne(_n((B, S, QH, D)))
        k = to_bf16_rne(_n((B, S, KH, D)))
        v = to_bf16_rne(_n((B, S, KH, D)))
        return {"q": q, "k": k, "v": v}
    if name == "mamba":
        B, L, Dm, N = 8, 4096 // scale, 4096, 16
        x = to_bf16_rne(_n((B, L, Dm)))
        dt = softplus(_n((B, L, Dm)) - f32(3.0))
        A = (-np.exp(_n((Dm, N), 0.5))).astype(f32)
        Bm = _n((B, L, N))
        Cm = _n((B, L, N))
        Dv = np.ones((Dm,), dtype=f32)
        return {"delta": dt, "u": x, "a": A, "b": Bm, "c": Cm, "D": Dv}
    raise KeyError(name)
