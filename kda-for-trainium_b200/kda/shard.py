"""Natural partitioning of every operator across GPUs (no collective needed).

Each operator splits into independent units, so a multi-GPU run gives each
device (or each torch.distributed rank) a contiguous range of units and
concatenates -- or simply keeps -- the per-device outputs:

  silu, adamw                flat: leading-axis row ranges
  rope_single_freq_apply     flat: column ranges of (D, S) (the S axis)
  rmsnorm_matmul, add_rmsnorm_matmul, matmul_add_rmsnorm, matmul, lora, swiglu
                             row blocks of the activation (weights replicated)
  transpose_matmul           column blocks of lhs (K, M) = output row blocks
  bmm, bmm_softmax           batch ranges
  gqa_full                   (batch, kv-head) units; each carries its query heads
  mamba                      batch ranges (channels-last) / channel ranges (2-D)

``split(op, args, world)`` returns one argument dict per part;
``merge(op, outs, args)`` reassembles a full output for verification.  The
functions are array-type agnostic (numpy or torch) and do no device work.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

ROW_OPS = ("rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "matmul", "lora", "swiglu")


def ranges(n: int, world: int) -> List[range]:
    """Split [0, n) into `world` contiguous ranges whose sizes differ by at most one."""
    if world < 1:
        raise ValueError("world must be >= 1")
    base, rem = divmod(n, world)
    out, start = [], 0
    for r in range(world):
        size = base + (1 if r < rem else 0)
        out.append(range(start, start + size))
        start += size
    return out


def _cat(parts, axis):
    first = parts[0]
    if hasattr(first, "dim"):  # torch
        import torch
        return torch.cat(list(parts), dim=axis)
    import numpy as np
    return np.concatenate(list(parts), axis=axis)


def split(op: str, args: Dict, world: int) -> List[Dict]:
    """Per-part argument dicts (keys = the op's forward parameter names)."""
    a = dict(args)
    parts: List[Dict] = []
    if op in ("silu",):
        for r in ranges(a["x"].shape[0], world):
            parts.append({"x": a["x"][r.start:r.stop]})
    elif op == "adamw":
        for r in ranges(a["theta"].shape[0], world):
            parts.append({k: a[k][r.start:r.stop] for k in ("theta", "g", "m", "v")})
    elif op == "rope_single_freq_apply":
        for r in ranges(a["x_in"].shape[1], world):
            parts.append({k: a[k][:, r.start:r.stop] for k in ("x_in", "cos", "sin")})
    elif op in ROW_OPS:
        row_keys = {"rmsnorm_matmul": ("x",), "add_rmsnorm_matmul": ("x", "z"),
                    "matmul_add_rmsnorm": ("x", "z"), "matmul": ("lhs",), "lora": ("x",),
                    "swiglu": ("x",)}[op]
        for r in ranges(a[row_keys[0]].shape[0], world):
            d = dict(a)
            for k in row_keys:
                d[k] = a[k][r.start:r.stop]
            parts.append(d)
    elif op == "transpose_matmul":
        for r in ranges(a["lhs"].shape[1], world):
            parts.append({"lhs": a["lhs"][:, r.start:r.stop], "rhs": a["rhs"]})
    elif op in ("bmm", "bmm_softmax"):
        for r in ranges(a["lhs"].shape[0], world):
            parts.append({"lhs": a["lhs"][r.start:r.stop], "rhs": a["rhs"][r.start:r.stop]})
    elif op == "gqa_full":
        B, KH = a["k"].shape[0], a["k"].shape[2]
        rep = a["q"].shape[2] // KH
        units = [(b, g) for b in range(B) for g in range(KH)]
        for r in ranges(len(units), world):
            mine = units[r.start:r.stop]
            parts.append({"units": mine, "rep": rep, **a})
    elif op == "mamba":
        if a["delta"].ndim == 3:
            for r in ranges(a["delta"].shape[0], world):
                d = dict(a)
                for k in ("delta", "u", "b", "c"):
                    d[k] = a[k][r.start:r.stop]
                parts.append(d)
        else:
            for r in ranges(a["delta"].shape[0], world):
                d = dict(a)
                for k in ("delta", "u", "a"):
                    d[k] = a[k][r.start:r.stop]
                parts.append(d)
    else:
        raise KeyError(op)
    return parts


def gqa_unit_args(part: Dict, b: int, g: int) -> Dict:
    """(q, k, v) of one (batch, kv-head) unit: k/v head g and its query heads."""
    rep = part["rep"]
    q = part["q"][b:b + 1, :, g * rep:(g + 1) * rep]
    k = part["k"][b:b + 1, :, g:g + 1]
    v = part["v"][b:b + 1, :, g:g + 1]
    return {"q": q, "k": k, "v": v}


def merge(op: str, outs: Sequence, args: Dict):
    """Reassemble a full output from per-part outputs (verification only)."""
    if op in ("silu", "adamw") or op in ROW_OPS or op == "transpose_matmul":
        return _cat(outs, 0)
    if op == "rope_single_freq_apply":
        return _cat(outs, 1)
    if op in ("bmm", "bmm_softmax"):
        return _cat(outs, 0)
    if op == "mamba":
        return _cat(outs, 0)
    raise KeyError(f"merge({op}) is per-unit; use gqa_unit_args")
