"""Multi-process paths on CPU (gloo, world size 2): the natural shard plans
reassemble the full result, and the bench's rank plumbing (barrier, max over
ranks, reference arm on rank 0 only) works without a GPU."""

import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import PKG_ROOT, REPO
from oracle import inputs, ops as ref

sys.path.insert(0, str(PKG_ROOT))
from kda import shard  # noqa: E402  (pure host code; loads no library)


def test_ranges_cover_exactly():
    for n in (0, 1, 7, 16, 33):
        for w in (1, 2, 3, 8):
            rs = shard.ranges(n, w)
            assert len(rs) == w
            assert [i for r in rs for i in r] == list(range(n))
            assert max(len(r) for r in rs) - min(len(r) for r in rs) <= 1


CASES = {
    "silu": dict(M=9, N=5),
    "adamw": dict(M=7, N=6),
    "rope_single_freq_apply": dict(D=8, S=13),
    "rmsnorm_matmul": dict(M=11, K=16, N=8),
    "add_rmsnorm_matmul": dict(M=11, K=16, N=8),
    "matmul_add_rmsnorm": dict(M=11, K=16, N=8),
    "matmul": dict(M=9, K=8, N=8),
    "lora": dict(M=9, K=16, N=8, R=8),
    "swiglu": dict(M=9, K=8, N=16),
    "transpose_matmul": dict(M=10, K=8, N=8),
    "bmm": dict(B=5, M=4, K=8, N=8),
    "bmm_softmax": dict(B=5, M=4, K=8, N=8),
    "mamba": dict(C=6, M=20, S=4),
}


@pytest.mark.parametrize("op", sorted(CASES))
@pytest.mark.parametrize("world", [2, 3])
def test_shard_plans_reassemble_the_oracle(op, world):
    d = inputs.nkibench(op, 3, bf16=False, **CASES[op])
    full = getattr(ref, op)(**d)
    outs = [getattr(ref, op)(**part) for part in shard.split(op, d, world)]
    np.testing.assert_allclose(shard.merge(op, outs, d), full, rtol=1e-5, atol=1e-5)


def test_gqa_units_cover_all_heads():
    d = inputs.nkibench("gqa_full", 2, B=2, S=16, QH=4, KH=2, D=8)
    full = ref.gqa_full(**d, causal=True, out_layout="bshd")
    got = np.zeros_like(full)
    for part in shard.split("gqa_full", d, 3):
        for b, g in part["units"]:
            u = shard.gqa_unit_args(part, b, g)
            o = ref.gqa_full(u["q"], u["k"], u["v"], causal=True, out_layout="bshd")
            got[b:b + 1, :, g * 2:(g + 1) * 2] = o
    np.testing.assert_allclose(got, full, rtol=1e-6, atol=1e-6)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


WORKER = textwrap.dedent("""
    import os, sys
    sys.path.insert(0, {repo!r})
    import numpy as np
    import torch.distributed as dist
    import bench
    from oracle import inputs, ops as ref
    sys.path.insert(0, {pkg!r})
    from kda import shard
    d = bench.Dist()
    d.init("gloo")
    # rank plumbing used by bench.py: barrier and max over ranks
    d.barrier()
    m = d.max(float(d.rank + 1))
    assert m == float(d.world), m
    assert d.sum(float(d.rank + 1)) == d.world * (d.world + 1) / 2
    # each rank computes its shard of a row-partitioned op; gather on rank 0
    args = inputs.nkibench("rmsnorm_matmul", 5, bf16=False, M=10, K=16, N=8)
    part = shard.split("rmsnorm_matmul", args, d.world)[d.rank]
    mine = ref.rmsnorm_matmul(**part)
    gathered = [None] * d.world
    dist.all_gather_object(gathered, mine)
    if d.rank == 0:
        full = ref.rmsnorm_matmul(**args)
        np.testing.assert_allclose(np.concatenate(gathered, 0), full, rtol=1e-5, atol=1e-5)
        print("OK", m)
    d.close()
""")


def test_gloo_two_ranks_bench_plumbing(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(repo=str(REPO), pkg=str(PKG_ROOT)))
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE="2",
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
        assert p.returncode == 0, out
    assert "OK 2.0" in outs[0]


def test_reference_arm_rank0_only(tmp_path):
    """--impl reference under a 2-rank launch: rank 0 prints one line on every
    host core (the launcher's OMP_NUM_THREADS=1 notwithstanding), rank 1 exits quietly."""
    outs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE="2", OMP_NUM_THREADS="1")
        r = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                            "--warmup", "3"], env=env, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        outs.append(r.stdout.strip())
    import json
    line = json.loads(outs[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["cpu_baseline"]["cores"] == os.cpu_count()
    assert outs[1] == ""
