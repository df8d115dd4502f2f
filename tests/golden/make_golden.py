"""Generate the golden fixtures in this directory from the reference itself.

Run once in a container that has the reference checkout (read-only) at
``$KDA_REFERENCE_ROOT`` (default: the ``reference`` directory next to the repo
root).  It imports the reference's own numpy offline simulations
(``workspaces/<op>/runs/offline_*_sim.py``) -- the reference's verbatim
restatements of the NKIBench ``forward`` functions -- shrinks their module
shape constants, and records for each case:

  * the seed and shapes,
  * a SHA-256 of every input array the reference's ``draw_inputs(seed)``
    produced (pins the oracle's draw order and distributions),
  * the reference forward's fp32 output.

Nothing here is needed at test time: the tests regenerate the inputs with
``oracle.inputs.nkibench`` and compare against the stored digests/outputs.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("KDA_REFERENCE_ROOT", REPO.parent / "reference"))

# op -> (sim file, module constants to set, forward-arg names in draw order,
#        output function name)
CASES = [
    ("matmul", "matmul/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("lhs", "rhs"), "reference_forward"),
    ("transpose_matmul", "transpose_matmul/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("lhs", "rhs"), "reference_forward"),
    ("bmm", "bmm/runs/offline_bf16_split_sim.py",
     dict(B=2, M=136, K=64, N=144), ("lhs", "rhs"), "mm_fp32"),
    ("rmsnorm_matmul", "rmsnorm_matmul/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("x", "w"), "reference_forward"),
    ("add_rmsnorm_matmul", "add_rmsnorm_matmul/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("x", "w", "z", "g"), "reference_forward"),
    ("matmul_add_rmsnorm", "matmul_add_rmsnorm/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("x", "w", "z", "g"), "reference_forward"),
    ("swiglu", "swiglu/runs/offline_bf16_split_sim.py",
     dict(M=136, K=200, N=144), ("x", "w_up", "w_down", "w_gate"), "reference_forward"),
    ("lora", "lora/runs/offline_lora_bf16_split_sim.py",
     dict(M=136, K=200, N=144, R=128), ("x", "w", "a", "b"), "reference_forward"),
    ("gqa_full", "gqa_full/runs/offline_score_bf16_split_sim.py",
     dict(B=1, N=160, QH=4, KH=2, D=128, N_REP=2), ("q", "k", "v"), "output_fp32"),
]
SEEDS = (42, 0)


def _load(rel):
    path = REF / "workspaces" / rel
    spec = importlib.util.spec_from_file_location("refsim_" + path.parent.parent.name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


def main() -> int:
    if not REF.is_dir():
        print(f"reference checkout not found at {REF}", file=sys.stderr)
        return 1
    meta = {}
    for op, rel, consts, names, fn in CASES:
        mod = _load(rel)
        for k, v in consts.items():
            setattr(mod, k, v)
        for seed in SEEDS:
            arrs = mod.draw_inputs(seed)
            out = getattr(mod, fn)(*arrs)
            if op == "gqa_full":            # (QH, N, D) for batch 0 -> (B, QH, N, D)
                out = out[None]
            key = f"{op}_s{seed}"
            np.save(HERE / f"{key}.npy", np.asarray(out, dtype=np.float32))
            meta[key] = {
                "op": op, "seed": seed, "source": f"workspaces/{rel}:{fn}",
                "shape": {k: v for k, v in consts.items() if k != "N_REP"},
                "input_sha256": {n: _digest(a) for n, a in zip(names, arrs)},
                "out_shape": list(np.shape(out)),
            }
            print(key, np.shape(out))
    # the reference's bf16 RNE known-answer asserts
    # (workspaces/matmul_add_rmsnorm/runs/offline_bf16_split_sim.py:178-190)
    sim = _load("matmul_add_rmsnorm/runs/offline_bf16_split_sim.py")
    probes = np.array([1.0, 1.0 + 2.0 ** -8, 1.0 + 3.0 * 2.0 ** -9, -2.5, 3.14159265,
                       1e-30, 65504.0, 1.0 + 2.0 ** -7 + 2.0 ** -8], dtype=np.float32)
    meta["bf16_rne"] = {"in": probes.tolist(),
                        "out": sim.to_bf16_rne(probes).astype(np.float32).tolist()}
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
