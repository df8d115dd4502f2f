"""The reference's correctness metric (oracle / test infrastructure).

relative-L2 = ||v_k - v_r||_2 / ||v_r||_2 over the flattened output, computed
in float64 -- the gate quantity of ``verify.py:44-45`` and the ``rel_l2``
helpers of the offline simulations (e.g.
``workspaces/rmsnorm_matmul/runs/offline_bf16_split_sim.py:102-106``).
"""

from __future__ import annotations

import numpy as np

# Gates named by the build's north star: fp32 operators 1e-5, bf16 operators 1e-2.
GATE_FP32 = 1e-5
GATE_BF16 = 1e-2


def rel_l2(v_k, v_r) -> float:
    v_k = np.asarray(v_k, dtype=np.float64).ravel()
    v_r = np.asarray(v_r, dtype=np.float64).ravel()
    num = np.linalg.norm(v_k - v_r)
    den = np.linalg.norm(v_r)
    if den == 0.0:
        return float(num)
    return float(num / den)
