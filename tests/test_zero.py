"""The ZeRO-1 AdamW step (kda.zero) and the multi-tensor AdamW it runs on.

CPU (gloo, world size 2 and 3): the sharding, the collective sequence and the
padding reproduce a single-process AdamW on the rank-averaged gradients (the
per-shard update is the CPU oracle, injected: no CUDA kernel runs on CPU).
GPU: the multi-tensor kernel against the oracle; on 2+ GPUs the fused
reduce-scatter -> AdamW -> all-gather kernel over NVLink peer memory against
the same single-process result and against the collective path.
"""

import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import PKG_ROOT, REPO
from oracle import ops as ref
from oracle.metrics import GATE_FP32, rel_l2

sys.path.insert(0, str(PKG_ROOT))


def test_shard_bounds():
    from kda.zero import shard_bounds
    for n in (0, 1, 5, 16, 1000003):
        for w in (1, 2, 3, 8):
            padded, sl = shard_bounds(n, w)
            assert padded >= n and padded == sl * w and sl % 4 == 0 and padded - n < 4 * w + 4 * w


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run_ranks(script, world, extra_env=None, timeout=240):
    port = _free_port()
    procs = []
    for rank in range(world):
        env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), **(extra_env or {}))
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for p, out in zip(procs, outs):
        assert p.returncode == 0, out
    return outs


# The single-process result every configuration must reproduce: AdamW on the
# mean of the ranks' gradients, three steps.
EXPECT = textwrap.dedent("""
    def expected(numel, world, steps, hp):
        theta = np.random.default_rng(1).normal(size=numel).astype(np.float32)
        m = np.zeros(numel, np.float32)
        v = np.zeros(numel, np.float32)
        for t in range(1, steps + 1):
            gs = [np.random.default_rng(100 * t + r).normal(size=numel).astype(np.float32) for r in range(world)]
            g = (np.sum(gs, axis=0, dtype=np.float32) * np.float32(1.0 / world)).astype(np.float32)
            theta, m, v = ref.adamw_step(theta, g, m, v, step=t, **hp)
        return theta
""")

CPU_WORKER = textwrap.dedent("""
    import os, sys, datetime
    sys.path.insert(0, {repo!r}); sys.path.insert(0, {pkg!r})
    import numpy as np, torch, torch.distributed as dist
    from oracle import ops as ref
    from kda.zero import Zero1AdamW
    {expect}
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    hp = dict(lr=1e-2, betas=(0.8, 0.99), eps=1e-8, weight_decay=0.1)
    numel = 1001

    def update(p, g, m, v, *, step, **kw):   # the CPU oracle stands in for the kernel
        th, m2, v2 = ref.adamw_step(p.numpy(), g.numpy(), m.numpy(), v.numpy(), step=step, **kw)
        p.copy_(torch.from_numpy(th)); m.copy_(torch.from_numpy(m2)); v.copy_(torch.from_numpy(v2))

    opt = Zero1AdamW(numel, update=update, fused=False, **hp)
    opt.param[:numel] = torch.from_numpy(np.random.default_rng(1).normal(size=numel).astype(np.float32))
    for t in range(1, 4):
        opt.grad[:numel] = torch.from_numpy(np.random.default_rng(100 * t + rank).normal(size=numel)
                                            .astype(np.float32))
        opt.step()
    want = expected(numel, world, 3, hp)
    np.testing.assert_allclose(opt.param[:numel].numpy(), want, rtol=1e-5, atol=1e-6)
    assert not opt.param[numel:].any()        # the padding stays zero
    print("OK", rank, flush=True)
    dist.destroy_process_group()
""")


VIEWS_WORKER = textwrap.dedent("""
    import os, sys, datetime
    sys.path.insert(0, {repo!r}); sys.path.insert(0, {pkg!r})
    import numpy as np, torch, torch.distributed as dist
    from oracle import ops as ref
    from kda.zero import Zero1AdamW
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    shapes = [(3, 5), (7,), (2, 2, 3)]
    rng = np.random.default_rng(3)
    params = [torch.from_numpy(rng.normal(size=s).astype(np.float32)) for s in shapes]

    def update(p, g, m, v, *, step, **kw):
        th, m2, v2 = ref.adamw_step(p.numpy(), g.numpy(), m.numpy(), v.numpy(), step=step, **kw)
        p.copy_(torch.from_numpy(th)); m.copy_(torch.from_numpy(m2)); v.copy_(torch.from_numpy(v2))

    opt, pv, gv = Zero1AdamW.for_tensors(params, update=update, fused=False)
    for p, t in zip(pv, params):
        assert torch.equal(p, t)
    grads = [np.random.default_rng(10 + rank + 7 * i).normal(size=s).astype(np.float32) for i, s in enumerate(shapes)]
    for g, x in zip(gv, grads):
        g.copy_(torch.from_numpy(x))
    opt.step()
    all_g = [None] * world
    dist.all_gather_object(all_g, grads)
    for i, (p, t) in enumerate(zip(pv, params)):
        mean = (np.sum([ag[i] for ag in all_g], axis=0, dtype=np.float32) * np.float32(1.0 / world)).astype(np.float32)
        want, _, _ = ref.adamw_step(t.numpy(), mean, np.zeros_like(mean), np.zeros_like(mean))
        np.testing.assert_allclose(p.numpy(), want, rtol=1e-5, atol=1e-6)
    print("OK", rank, flush=True)
    dist.destroy_process_group()
""")


def test_zero1_views_over_model_tensors_gloo(tmp_path):
    script = tmp_path / "zero_views.py"
    script.write_text(VIEWS_WORKER.format(repo=str(REPO), pkg=str(PKG_ROOT)))
    outs = _run_ranks(script, 2)
    for r, out in enumerate(outs):
        assert f"OK {r}" in out, out


@pytest.mark.parametrize("world", [2, 3])
def test_zero1_collective_path_gloo(tmp_path, world):
    script = tmp_path / "zero_cpu.py"
    script.write_text(CPU_WORKER.format(repo=str(REPO), pkg=str(PKG_ROOT), expect=EXPECT))
    outs = _run_ranks(script, world)
    for r, out in enumerate(outs):
        assert f"OK {r}" in out, out


# ------------------------------------------------------------------- GPU
torch = pytest.importorskip("torch")


@pytest.mark.gpu
def test_adamw_multi_matches_oracle():
    import kda
    rng = np.random.default_rng(0)
    sizes = [0, 1, 3, 4, 4097, 10000, 40961, 3 * 4096]
    hp = dict(lr=1e-2, betas=(0.8, 0.99), eps=1e-8, weight_decay=0.1)
    host = [[rng.normal(size=n).astype(np.float32) for n in sizes] for _ in range(4)]
    host[3] = [np.abs(x) for x in host[3]]
    dev = [[torch.from_numpy(x.copy()).cuda() for x in lst] for lst in host]
    th, g, m, v = (list(x) for x in host)
    for t in (1, 2, 3):
        kda.adamw_multi(dev[0], dev[1], dev[2], dev[3], step=t, **hp)
        for i in range(len(sizes)):
            th[i], m[i], v[i] = ref.adamw_step(th[i], g[i], m[i], v[i], step=t, **hp)
    torch.cuda.synchronize()
    for i, n in enumerate(sizes):
        if n:
            assert rel_l2(dev[0][i].cpu().numpy(), th[i]) <= GATE_FP32
            assert rel_l2(dev[2][i].cpu().numpy(), m[i]) <= GATE_FP32
            assert rel_l2(dev[3][i].cpu().numpy(), v[i]) <= GATE_FP32
    assert kda.device_error() == 0


@pytest.mark.gpu
def test_adamw_multi_defaults_are_the_adamw_operator():
    """Default hyperparameters at step 1 give the adamw operator's update, on
    many tensors at once (including an unaligned view: scalar path)."""
    import kda
    rng = np.random.default_rng(3)
    base = [torch.from_numpy(rng.normal(size=(4, 8193)).astype(np.float32)).cuda() for _ in range(4)]
    base[3] = base[3].abs()
    views = [t.reshape(-1)[1:] for t in base]          # 4-byte offset
    a = [[t.clone() for t in base], [t.clone() for t in views]]
    for lst in a:
        want = kda.adamw(lst[0], lst[1], lst[2].clone(), lst[3].clone())
        kda.adamw_multi([lst[0]], [lst[1]], [lst[2]], [lst[3]])
        assert rel_l2(lst[0].cpu().numpy(), want.cpu().numpy()) <= 1e-6
    x = [torch.empty(0, device="cuda") for _ in range(4)]
    kda.adamw_multi(*([t] for t in x))                  # empty tensors: no launch
    with pytest.raises(ValueError):
        kda.adamw_multi([base[0]], [base[1][:1]], [base[2]], [base[3]])
    with pytest.raises(ValueError):
        kda.adamw_multi([base[0]], [base[1]], [base[2]], [base[3]], step=0)


GPU_WORKER = textwrap.dedent("""
    import os, sys, datetime
    sys.path.insert(0, {repo!r}); sys.path.insert(0, {pkg!r})
    import numpy as np, torch, torch.distributed as dist
    from oracle import ops as ref
    from oracle.metrics import rel_l2
    import kda
    from kda.zero import Zero1AdamW
    {expect}
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    hp = dict(lr=1e-2, betas=(0.8, 0.99), eps=1e-8, weight_decay=0.1)
    numel = 1000003
    want = expected(numel, world, 3, hp)
    res = {{}}
    for fused in (True, False):
        opt = Zero1AdamW(numel, device=f"cuda:{{rank}}", fused=fused, **hp)
        opt.param[:numel] = torch.from_numpy(np.random.default_rng(1).normal(size=numel).astype(np.float32)).cuda()
        for t in range(1, 4):
            opt.grad[:numel] = torch.from_numpy(np.random.default_rng(100 * t + rank).normal(size=numel)
                                                .astype(np.float32)).cuda()
            opt.step()
        torch.cuda.synchronize()
        got = opt.param[:numel].cpu().numpy()
        res[fused] = got
        err = rel_l2(got, want)
        assert err <= 1e-5, (fused, err)
        assert not opt.param[numel:].any()
        opt.close()
    # the fused and collective paths agree (each rank holds the same replica)
    assert rel_l2(res[True], res[False]) <= 1e-6
    assert kda.device_error() == 0
    dist.barrier()
    dist.destroy_process_group()
    print("OK", rank, flush=True)
""")


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_zero1_fused_two_gpus(tmp_path):
    script = tmp_path / "zero_gpu.py"
    script.write_text(GPU_WORKER.format(repo=str(REPO), pkg=str(PKG_ROOT), expect=EXPECT))
    outs = _run_ranks(script, 2, extra_env={"NCCL_NVLS_ENABLE": "0"}, timeout=300)
    for r, out in enumerate(outs):
        assert f"OK {r}" in out, out
