"""Benchmark: per-op latency and roofline fraction of the kda-b200 operators.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {kda,reference}]
                    [--op NAME] [--no-ops-table]

Headline workload (the JSON line's ``metric`` / ``value``): the fused
RMSNorm->GEMM configuration -- X bf16 [4096, 4096], gamma fp32 [4096], eps
1e-6, W bf16 [4096, 11008] -> Y bf16 [4096, 11008], 369.37 GFLOP -- one step =
one ``kda.rmsnorm_matmul`` call.  With N GPUs (torchrun, one process per GPU)
the ONE configuration is partitioned by row blocks of X (M/N rows per GPU, W
and gamma replicated; row norms are row-local, so there is no collective on
the data path): ``value`` is the whole configuration's TFLOP/s over the max-
over-ranks step time (strong scaling).  L2 (126 MB) is flushed before every
timed step by writing a 256 MB buffer and then reading another 256 MB (so no
dirty flush lines are written back inside the timed step).

The line also carries, for the same run:
  roofline     -- the dominant kernel (the tcgen05 GEMM) at this rank's shape
                  timed alone with CUDA events, against MEASURED_PEAKS.json's
                  bf16 peak; traffic from the committed ncu summary.
  cpu_baseline -- the numpy oracle (test infrastructure, oracle/) on a bounded
                  row sample, on this host's cores (N=1 only).
  e2e          -- the same metric through the public API from pinned host
                  buffers: each rank uploads its X rows and 1/N of W's rows,
                  the W parts are all-gathered over NVLink (NCCL; N > 1), the
                  op runs and each rank reads its Y rows back -- all inside the
                  timed step.
  ops          -- every operator at its configuration, partitioned over the
                  N GPUs as it shards naturally (row blocks, batch, batch x
                  kv-head, flat): [p50 ms (max over ranks), fraction of N x
                  the measured roofline, numpy oracle ms on the host cores
                  (N=1 only)]; details on stderr.
  zero1_adamw  -- (N > 1) the fused ZeRO-1 AdamW step against NCCL
                  reduce-scatter + AdamW + all-gather, with their difference.
  clocks       -- nvidia-smi SM clock / throttle reasons sampled during timing.

``--impl reference`` times the reference's own algorithm on the host cores
instead (the numpy restatement in oracle/; the reference's NKI kernels need
Trainium hardware), on the same metric and configuration, with a bounded row
sample per step and every host core (rank 0 only under torchrun).
"""

import os
import sys


def _reference_arm_requested(argv) -> bool:
    for i, a in enumerate(argv):
        if a == "--impl=reference" or (a == "--impl" and i + 1 < len(argv) and argv[i + 1] == "reference"):
            return True
    return False


if _reference_arm_requested(sys.argv[1:]):
    # torchrun sets OMP_NUM_THREADS=1 for every rank; the reference arm runs on
    # rank 0 alone and uses every host core, so size the BLAS pool before numpy
    # (and its OpenBLAS) is imported
    for _v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_v] = str(os.cpu_count() or 1)

import argparse  # noqa: E402
import json  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import threading  # noqa: E402
import time  # noqa: E402
from pathlib import Path  # noqa: E402

import numpy as np  # noqa: E402

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "kda-for-trainium_b200"))

METRIC = "per-op p50 latency + % of roofline (TC or HBM) at 1/2/4/8 B200 vs CPU numpy ref"
HEAD_M, HEAD_K, HEAD_N = 4096, 4096, 11008
HEAD_FLOP = 2.0 * HEAD_M * HEAD_N * HEAD_K
IDLE_S = 0.3  # idle gap before each op of the per-op table
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def cpu_cores():
    try:
        from threadpoolctl import threadpool_info
        n = max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
        return int(n)
    except Exception:
        return os.cpu_count() or 1


# --------------------------------------------------------------------------- #
# distributed plumbing
# --------------------------------------------------------------------------- #
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl"):
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
            self.pg = dist

    def barrier(self):
        if self.pg:
            import torch
            if self.pg.get_backend() == "nccl":
                self.pg.barrier(device_ids=[torch.cuda.current_device()])
            else:
                self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        dev = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        dev = "cuda" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# --------------------------------------------------------------------------- #
# clocks sampling (nvidia-smi during the timed region)
# --------------------------------------------------------------------------- #
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def count(self):
        return len(self.lines)

    def stop(self, first=0):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[first:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                smax.append(float(parts[2].split()[0]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- #
# kda arm
# --------------------------------------------------------------------------- #
class L2Flush:
    """Evicts L2 (126 MB) before a timed step: write 256 MB, then read another
    256 MB so the written lines are also written back before the timer starts
    (otherwise their write-back would land inside the timed kernel)."""

    def __init__(self, torch, dev):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 << 20, dtype=torch.float32, device=dev)
        self.acc = torch.empty((), dtype=torch.float32, device=dev)

    def fill_(self, v=1):
        self.w.fill_(v)
        self.acc.copy_(self.r.sum())


def _flush_buf(torch, dev):
    return L2Flush(torch, dev)


def time_steps(torch, fn, steps, warmup, flush, stream):
    """Per-step device time (ms) with CUDA events on `stream`; L2 flushed before each step."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        if flush is not None:
            flush.fill_(1)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return times


def as_graph(torch, fn):
    """Capture one call of `fn` in a CUDA graph and return its replay (device
    time without the host's per-call Python and launch overhead, which can
    outlast the L2 flush queued before a step and leave the GPU idle inside
    the timed region); None if the call cannot be captured."""
    try:
        fn()
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        torch.cuda.synchronize()
        return graph.replay  # the bound method keeps the graph alive while it is timed
    except Exception:
        torch.cuda.synchronize()
        return None


def head_inputs(torch, dev, seed=42):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(HEAD_M, HEAD_K, device=dev, generator=g).to(torch.bfloat16)
    gam = (1.0 + 0.1 * torch.randn(HEAD_K, device=dev, generator=g)).float()
    w = (0.02 * torch.randn(HEAD_K, HEAD_N, device=dev, generator=g)).to(torch.bfloat16)
    return x, gam, w


def ops_table(torch, kda, dev, pk, flush, dist=None, iters=10, only=None, small=False):
    """Every operator at its configuration: p50 ms, achieved, roofline fraction.

    With ``dist.world`` > 1 each rank runs its part of the configuration, split
    the way the operator shards naturally (``kda.shard``): row blocks of the
    activation for the GEMM family (weights replicated), output-row blocks
    (lhs columns) for transpose_matmul, batch for bmm / bmm_softmax / mamba,
    batch x kv-head for gqa_full, flat ranges for silu / adamw / rope.  Every
    rank times its part after a barrier; an op's time is the max over ranks of
    the per-rank p50, its throughput the whole configuration's work over that
    time, and its fraction that throughput over world x the measured peak.
    The backward and fp32-accuracy rows run at N = 1 only.
    ``only`` restricts the table to one operator (``bench.py --op NAME``);
    ``small`` runs the scan on 512 of its 4096 steps (a profiling case with the
    configuration's kernel and layout)."""
    from kda.shard import ranges
    bf = torch.bfloat16
    world = dist.world if dist is not None else 1
    rank = dist.rank if dist is not None else 0
    hbm = pk["hbm_gbs"] * world
    tc = pk["bf16_tflops"] * world
    g = torch.Generator(device=dev)
    g.manual_seed(0)

    def part(n):
        """This rank's share of n units (contiguous, sizes differ by at most one)."""
        return len(ranges(n, world)[rank])

    def rn(*s, dtype=torch.float32, scale=1.0):
        return (scale * torch.randn(*s, device=dev, generator=g)).to(dtype)

    rows = {}

    def exp_bound(name, exps):
        """Second bound for exponential-heavy ops: exponentials per second
        against the ex2 throughput (16 per clock per SM, measured) at the
        maximum SM clock, times the GPU count."""
        r = rows.get(name)
        if not r or "p50_ms" not in r:
            return
        peak = 16 * 148 * 1.965e9 * world
        got = exps / (r["p50_ms"] * 1e-3)
        r["exp_bound"] = {"exps": exps, "achieved_per_s": round(got / 1e12, 3), "peak_per_s": round(peak / 1e12, 3),
                          "unit": "T exp/s", "frac": round(got / peak, 3),
                          "note": "ex2 pipe: 16 per clock per SM x 148 SMs x 1.965 GHz per GPU"}

    def want(name, single_only=False):
        if only is not None:
            return name == only
        return not (single_only and world > 1)

    def run(name, fn, work, bound, launches, note=""):
        """Time ``fn`` (this rank's part); ``work`` is the whole configuration's."""
        err = None
        p50 = float("inf")
        timing = ""
        try:
            replay = as_graph(torch, fn)
            timing = "CUDA graph replay" if replay is not None else "direct calls"
            # every op starts from an idle GPU: right after a long tensor-core op
            # (swiglu) the 1 kW power cap keeps the next op ~15 % slower for a
            # few hundred ms, which would make each row depend on the one before
            torch.cuda.synchronize()
            time.sleep(IDLE_S)
            timing += f", after {IDLE_S} s idle"
        except Exception as e:  # an op that fails is reported, not hidden
            err, replay = e, None
        if dist is not None:
            dist.barrier()
        if err is None:
            try:
                p50 = statistics.median(time_steps(torch, replay or fn, iters, 3, flush,
                                                   torch.cuda.current_stream()))
            except Exception as e:
                err = e
        p50 = dist.max(p50) if dist is not None else p50   # every rank joins, even after a failure
        if err is not None or p50 == float("inf"):
            rows[name] = {"error": str(err)[:200] if err is not None else "failed on another rank"}
            return
        if bound == "hbm":
            ach = work / (p50 * 1e-3) / 1e9
            rows[name] = {"p50_ms": round(p50, 4), "achieved": round(ach, 1), "unit": "GB/s",
                          "frac": round(ach / hbm, 3), "bound": "hbm", "algorithmic_bytes": work,
                          "kernels": launches}
        else:
            ach = work / (p50 * 1e-3) / 1e12
            rows[name] = {"p50_ms": round(p50, 4), "achieved": round(ach, 1), "unit": "TFLOP/s",
                          "frac": round(ach / tc, 3), "bound": "tensor", "flops": work, "kernels": launches}
        rows[name]["timing"] = timing
        if note:
            rows[name]["config"] = note

    def ws_for(fn_name, *dims):
        return torch.empty(max(1, kda.ops._ws_size(fn_name, *dims)), dtype=torch.uint8, device=dev)

    if want("silu"):
        x = rn(part(4096), 8192)
        run("silu", lambda: kda.silu(x), 2 * 4096 * 8192 * 4, "hbm", 1, "x fp32 [4096,8192]")
        del x
    # GEMM family: row blocks of the activation, weights replicated
    Mr = part(HEAD_M)
    if want("rmsnorm_matmul") or want("rmsnorm_matmul_backward", True) or want("matmul_add_rmsnorm"):
        X, gam, W = head_inputs(torch, dev)
        X = X[:Mr].contiguous()
        if want("rmsnorm_matmul"):
            ws = ws_for("kda_rmsnorm_matmul_workspace_size", Mr, 4096, 11008)
            run("rmsnorm_matmul", lambda: kda.rmsnorm_matmul(X, W, gam, 1e-6, workspace=ws), HEAD_FLOP, "tc", 2,
                "X[4096,4096] W[4096,11008] bf16")
            del ws
        if want("rmsnorm_matmul_backward", True):
            dY = rn(Mr, 11008, dtype=bf)
            wsb = ws_for("kda_rmsnorm_matmul_backward_workspace_size", Mr, 4096, 11008)
            run("rmsnorm_matmul_backward", lambda: kda.rmsnorm_matmul_backward(dY, X, W, gam, 1e-6, workspace=wsb),
                2 * HEAD_FLOP, "tc", 7, "dY[4096,11008] -> dX, dW, dgamma (two GEMMs: dY W^T fp32, a^T dY)")
            del dY, wsb
        del W
        if want("matmul_add_rmsnorm"):
            B = rn(4096, 4096, dtype=bf, scale=0.02)
            R = rn(Mr, 4096, dtype=bf)
            ws2 = ws_for("kda_matmul_add_rmsnorm_workspace_size", Mr, 4096, 4096)
            run("matmul_add_rmsnorm", lambda: kda.matmul_add_rmsnorm(X, B, 1e-6, R, gam, workspace=ws2),
                2.0 * 4096 ** 3, "tc", 2, "A,B,R [4096,4096] bf16")
            del B, R, ws2
        del X
    if want("add_rmsnorm_matmul"):
        x = rn(Mr, 1024, dtype=bf)
        z = rn(Mr, 1024, dtype=bf)
        w = rn(1024, 2048, dtype=bf, scale=0.02)
        g1 = 1 + 0.1 * rn(1024)
        ws = ws_for("kda_add_rmsnorm_matmul_workspace_size", Mr, 1024, 2048)
        run("add_rmsnorm_matmul", lambda: kda.add_rmsnorm_matmul(x, w, 1e-5, z, g1, workspace=ws),
            2.0 * 4096 * 1024 * 2048, "tc", 2, "x,z[4096,1024] w[1024,2048]")
        del x, z, w, ws
    if want("swiglu") or want("swiglu_backward", True) or want("swiglu_gu", True) or \
            want("swiglu_backward_saved", True):
        Ms = part(8192)
        x = rn(Ms, 4096, dtype=bf)
        wg = rn(4096, 14336, dtype=bf, scale=0.02)
        wu = rn(4096, 14336, dtype=bf, scale=0.02)
        wd = rn(14336, 4096, dtype=bf, scale=0.02)
        if want("swiglu"):
            ws3 = ws_for("kda_swiglu_workspace_size", Ms, 4096, 14336)
            run("swiglu", lambda: kda.swiglu(x, wu, wd, wg, workspace=ws3), 2.0 * 8192 * 4096 * 14336 * 3, "tc",
                2, "X[8192,4096] d_ff 14336")
            del ws3
        if want("swiglu_backward", True):
            dO = rn(Ms, 4096, dtype=bf)
            wsb = ws_for("kda_swiglu_backward_workspace_size", Ms, 4096, 14336)
            run("swiglu_backward", lambda: kda.swiglu_backward(dO, x, wu, wd, wg, workspace=wsb),
                2.0 * 8192 * 4096 * 14336 * 8, "tc", 10,
                "dout[8192,4096] -> dx, dw_up, dw_down, dw_gate (8 GEMM-equivalents incl. the g/u recompute)")
            del dO, wsb
        if want("swiglu_gu", True) or want("swiglu_backward_saved", True):
            # the training-step pair: a forward that keeps g, u and the backward on them
            wsf = ws_for("kda_swiglu_gu_workspace_size", Ms, 4096, 14336)
            run("swiglu_gu", lambda: kda.swiglu_gu(x, wu, wd, wg, workspace=wsf), 2.0 * 8192 * 4096 * 14336 * 3,
                "tc", 4, "X[8192,4096] d_ff 14336, unfused, g and u kept (g, u GEMMs, silu*mul, down GEMM)")
            _, gk, uk = kda.swiglu_gu(x, wu, wd, wg, workspace=wsf)
            dO = rn(Ms, 4096, dtype=bf)
            wss = ws_for("kda_swiglu_backward_saved_workspace_size", Ms, 4096, 14336)
            run("swiglu_backward_saved", lambda: kda.swiglu_backward(dO, x, wu, wd, wg, g=gk, u=uk, workspace=wss),
                2.0 * 8192 * 4096 * 14336 * 6, "tc", 8,
                "dout[8192,4096] -> dx, dw_up, dw_down, dw_gate from the kept g, u (6 GEMM-equivalents)")
            del wsf, gk, uk, dO, wss
        del x, wg, wu, wd
    if want("matmul") or want("matmul_f32", True) or want("lora"):
        a = rn(Mr, 5120, dtype=bf)
        b = rn(5120, 12288, dtype=bf, scale=0.02)
        if want("matmul"):
            run("matmul", lambda: kda.matmul(a, b), 2.0 * 4096 * 5120 * 12288, "tc", 1,
                "(4096,5120)@(5120,12288)")
        if want("matmul_f32", True):
            # fp32 in / fp32 out at fp32 accuracy: bf16 hi + lo split, three bf16 passes
            a32, b32 = a.float(), b.float()
            ws32 = ws_for("kda_matmul_f32_workspace_size", Mr, 5120, 12288)
            run("matmul_f32", lambda: kda.matmul(a32, b32, workspace=ws32), 2.0 * 4096 * 5120 * 12288, "tc", 3,
                "(4096,5120)@(5120,12288) fp32 in/out, bf16x3 (3 tensor-core passes + hi/lo split)")
            del a32, b32, ws32
        if want("lora"):
            la = rn(5120, 128, dtype=bf, scale=0.02)
            lb = rn(128, 12288, dtype=bf, scale=0.02)
            ws4 = ws_for("kda_lora_workspace_size", Mr, 5120, 12288, 128)
            run("lora", lambda: kda.lora(a, b, la, lb, workspace=ws4),
                2.0 * 4096 * 5120 * 12288 + 2.0 * 4096 * 5120 * 128 + 2.0 * 4096 * 128 * 12288, "tc", 3,
                "x[4096,5120] w[5120,12288] R=128")
            del la, lb, ws4
        del a, b
    if want("transpose_matmul") or want("transpose_matmul_f32", True):
        Mt = part(4096)          # this rank's columns of lhs (K, M) = its output rows
        lt = rn(2048, Mt, dtype=bf)
        rt = rn(2048, 10944, dtype=bf, scale=0.02)
        if want("transpose_matmul"):
            run("transpose_matmul", lambda: kda.transpose_matmul(lt, rt), 2.0 * 4096 * 2048 * 10944, "tc", 1,
                "lhs(2048,4096).T @ (2048,10944)")
        if want("transpose_matmul_f32", True):
            lt32, rt32 = lt.float(), rt.float()
            wst = ws_for("kda_transpose_matmul_f32_workspace_size", Mt, 2048, 10944)
            run("transpose_matmul_f32", lambda: kda.transpose_matmul(lt32, rt32, workspace=wst),
                2.0 * 4096 * 2048 * 10944, "tc", 3, "lhs(2048,4096).T @ (2048,10944) fp32 in/out, bf16x3")
            del lt32, rt32, wst
        del lt, rt
    bmm_bytes = (16 * 4096 * 64 * 2 + 16 * 4096 * 4096) * 2
    if want("bmm") or want("bmm_softmax") or want("bmm_f32", True) or want("bmm_softmax_f32", True):
        Bb = part(16)
        l3 = rn(Bb, 4096, 64, dtype=bf)
        r3 = rn(Bb, 64, 4096, dtype=bf)
        if want("bmm"):
            run("bmm", lambda: kda.bmm(l3, r3), bmm_bytes, "hbm", 1, "B16 M4096 K64 N4096")
        if want("bmm_softmax"):
            run("bmm_softmax", lambda: kda.bmm_softmax(l3, r3), bmm_bytes, "hbm", 1, "B16 M4096 K64 N4096")
            exp_bound("bmm_softmax", 2 * 16 * 4096 * 4096)  # statistics pass + output pass
        if want("bmm_f32", True) or want("bmm_softmax_f32", True):
            l32, r32 = l3.float(), r3.float()
            if want("bmm_f32", True):
                wsb = ws_for("kda_bmm_f32_workspace_size", Bb, 4096, 64, 4096)
                run("bmm_f32", lambda: kda.bmm(l32, r32, workspace=wsb), 2 * bmm_bytes, "hbm", 18,
                    "B16 M4096 K64 N4096 fp32 in/out, bf16x3 (split + one GEMM per batch entry)")
                del wsb
            if want("bmm_softmax_f32", True):
                wss = ws_for("kda_bmm_softmax_f32_workspace_size", Bb, 4096, 64, 4096)
                run("bmm_softmax_f32", lambda: kda.bmm_softmax(l32, r32, workspace=wss), 2 * bmm_bytes, "hbm",
                    19, "B16 M4096 K64 N4096 fp32 in/out, three-way split (6 products, one K-extended GEMM per "
                    "entry) + row softmax")
                del wss
            del l32, r32
        del l3, r3
    if want("gqa_full"):
        # (batch, kv-head) units in batch-major order: at 1/2/4/8 GPUs a rank's
        # contiguous range is whole batch entries, each with all 8 kv heads
        Bq = part(8)
        q = rn(Bq, 4096, 32, 128, dtype=bf)
        k = rn(Bq, 4096, 8, 128, dtype=bf)
        v = rn(Bq, 4096, 8, 128, dtype=bf)
        causal_flops = 4.0 * 8 * 32 * 128 * (4096 * 4097 / 2)
        wsa = ws_for("kda_gqa_full_workspace_size", Bq, 4096, 32, 8, 128, 10000.0)
        run("gqa_full", lambda: kda.gqa_full(q, k, v, causal=True, rope_theta=10000.0, out_layout="bshd",
                                             workspace=wsa),
            causal_flops, "tc", 5,
            "B8 S4096 QH32 KH8 D128 causal RoPE (rope table + q/k rotation + V transpose + attention)")
        del q, k, v, wsa
    if want("gqa_full_backward") or want("gqa_full_backward_saved"):
        # backward at the NKIBench shape (B1 S4096 QH16 KH8, non-causal, no RoPE): five
        # products of 2 S^2 D per query head counted (the forward it reruns for the rows'
        # log2-sum-exp and out is not); P and dS stay in shared memory (flash-style).
        # With N GPUs each takes whole kv groups (its kv heads and their query heads):
        # no exchange, as in the forward
        KHr = part(8)
        QHr = 2 * KHr
        qb = rn(1, 4096, QHr, 128, dtype=bf)
        kb_ = rn(1, 4096, KHr, 128, dtype=bf)
        vb = rn(1, 4096, KHr, 128, dtype=bf)
        dob = rn(1, QHr, 4096, 128, dtype=bf)
        wsg = ws_for("kda_gqa_full_backward_workspace_size", 1, 4096, QHr, KHr, 128, 0.0)
        run("gqa_full_backward", lambda: kda.gqa_full_backward(dob, qb, kb_, vb, workspace=wsg),
            5 * 2.0 * 16 * 4096 * 4096 * 128, "tc", 5,
            "B1 S4096 QH16 KH8 D128 non-causal: dq, dk, dv (forward, row sums, flash-style backward kernel)")
        # the training-step backward: the forward's output and lse kept by gqa_full_lse
        ob, lseb = kda.gqa_full_lse(qb, kb_, vb)
        wss = ws_for("kda_gqa_full_backward_saved_workspace_size", 1, 4096, QHr, KHr, 128, 0.0)
        run("gqa_full_backward_saved",
            lambda: kda.gqa_full_backward(dob, qb, kb_, vb, fwd_out=ob, lse=lseb, workspace=wss),
            5 * 2.0 * 16 * 4096 * 4096 * 128, "tc", 3,
            "same, from the saved forward (out, lse of gqa_full_lse): row sums, flash-style backward kernel")
        del qb, kb_, vb, dob, wsg, ob, lseb, wss
    if want("rope_single_freq_apply"):
        Sr = part(262144)
        xr = rn(128, Sr)
        c = rn(64, Sr)
        s = rn(64, Sr)
        run("rope_single_freq_apply", lambda: kda.rope_single_freq_apply(xr, c, s),
            4 * (2 * 128 * 262144 + 64 * 262144 * 2), "hbm", 1, "x[128,262144] cos/sin[64,262144]")
        del xr, c, s
    if want("adamw"):
        Ma = part(10944)
        th = rn(Ma, 2048)
        gr = rn(Ma, 2048)
        m = rn(Ma, 2048)
        vv = rn(Ma, 2048).abs()
        run("adamw", lambda: kda.adamw(th, gr, m, vv), 5 * 10944 * 2048 * 4, "hbm", 1, "theta,g,m,v [10944,2048]")
        del th, gr, m, vv
    if want("mamba"):
        Bm_ = part(8)
        Ls = 512 if small else 4096
        dt = torch.nn.functional.softplus(rn(Bm_, Ls, 4096) - 3.0)
        xx = rn(Bm_, Ls, 4096, dtype=bf)
        A = -torch.exp(0.5 * rn(4096, 16))
        Bm = rn(Bm_, Ls, 16)
        Cm = rn(Bm_, Ls, 16)
        Dv = torch.ones(4096, device=dev)
        wsm = ws_for("kda_mamba_scan_workspace_size", Bm_, Ls, 4096, 16)
        mamba_bytes = 8 * Ls * 4096 * (4 + 2 + 2) + 4096 * 16 * 4 + 2 * 8 * Ls * 16 * 4 + 4096 * 4
        run("mamba", lambda: kda.mamba(dt, xx, A, Bm, Cm, Dv, workspace=wsm), mamba_bytes, "hbm", 1,
            f"B8 L{Ls} D4096 N16, y bf16")
        exp_bound("mamba", 8 * Ls * 4096 * 16)  # one exp(dt * A) per (t, channel, state)
        del dt, xx, A, Bm, Cm, Dv, wsm
    return rows


def cpu_ops(budget_s=1.0):
    """The numpy oracle (the reference's algorithm restated; test
    infrastructure) for every operator on this host's cores: a bounded sample
    of each configuration (whole configuration where it runs in about a
    second, else a slice along an axis the work is linear in), best of up to
    three runs, scaled to the whole configuration.  Returns
    {op: (ms, sample description)}."""
    from oracle import ops as ref
    from oracle.bf16 import to_bf16_rne
    rng = np.random.default_rng(0)

    def n(*s, scale=1.0):
        return (scale * rng.standard_normal(s, dtype=np.float32)).astype(np.float32)

    def b(*s, scale=1.0):
        return to_bf16_rne(n(*s, scale=scale))

    def timed(fn):
        best, total, reps = float("inf"), 0.0, 0
        while reps < 3 and (reps == 0 or total < budget_s):
            t0 = time.perf_counter()
            fn()
            dt = time.perf_counter() - t0
            best, total, reps = min(best, dt), total + dt, reps + 1
        return best * 1e3

    out = {}

    def add(name, fn, scale, sample):
        try:
            out[name] = (round(timed(fn) * scale, 3), sample)
        except Exception as e:  # reported, not hidden
            out[name] = (None, f"failed: {str(e)[:80]}")

    x = n(4096, 8192)
    add("silu", lambda: ref.silu(x), 1, "whole")
    del x
    w = b(4096, 11008, scale=0.02)
    gam = 1 + 0.1 * n(4096)
    x = b(512, 4096)
    add("rmsnorm_matmul", lambda: ref.rmsnorm_matmul(x, w, gam, 1e-6), 8, "512 of 4096 rows")
    dy = b(128, 11008)
    add("rmsnorm_matmul_backward", lambda: ref.rmsnorm_matmul_backward(dy, x[:128], w, gam, 1e-6), 32,
        "128 of 4096 rows, float64")
    del w, dy
    w2, z = b(4096, 4096, scale=0.02), b(512, 4096)
    add("matmul_add_rmsnorm", lambda: ref.matmul_add_rmsnorm(x, w2, 1e-6, z, gam), 8, "512 of 4096 rows")
    del w2, z, x
    x, z, w, g1 = b(4096, 1024), b(4096, 1024), b(1024, 2048, scale=0.02), 1 + 0.1 * n(1024)
    add("add_rmsnorm_matmul", lambda: ref.add_rmsnorm_matmul(x, w, 1e-5, z, g1), 1, "whole")
    del x, z, w
    x = b(256, 4096)
    wg, wu, wd = b(4096, 14336, scale=0.02), b(4096, 14336, scale=0.02), b(14336, 4096, scale=0.02)
    add("swiglu", lambda: ref.swiglu(x, wu, wd, wg), 32, "256 of 8192 rows")
    add("swiglu_gu", lambda: ref.swiglu(x, wu, wd, wg), 32, "256 of 8192 rows (the restatement keeps no g, u)")
    do = b(64, 4096)
    add("swiglu_backward", lambda: ref.swiglu_backward(do, x[:64], wu, wd, wg), 128, "64 of 8192 rows, float64")
    add("swiglu_backward_saved", lambda: ref.swiglu_backward(do, x[:64], wu, wd, wg), 128,
        "64 of 8192 rows, float64 (the restatement recomputes g, u)")
    del x, wg, wu, wd, do
    a, w = b(512, 5120), b(5120, 12288, scale=0.02)
    add("matmul", lambda: ref.matmul(a, w), 8, "512 of 4096 rows")
    la, lb = b(5120, 128, scale=0.02), b(128, 12288, scale=0.02)
    add("lora", lambda: ref.lora(a, w, la, lb), 8, "512 of 4096 rows")
    del a, w, la, lb
    lt, rt = b(2048, 1024), b(2048, 10944, scale=0.02)
    add("transpose_matmul", lambda: ref.transpose_matmul(lt, rt), 4, "1024 of 4096 output rows")
    del lt, rt
    l3, r3 = b(2, 4096, 64), b(2, 64, 4096)
    add("bmm", lambda: ref.bmm(l3, r3), 8, "2 of 16 batch entries")
    add("bmm_softmax", lambda: ref.bmm_softmax(l3, r3), 8, "2 of 16 batch entries")
    del l3, r3
    q, k, v = b(1, 4096, 4, 128), b(1, 4096, 1, 128), b(1, 4096, 1, 128)
    add("gqa_full", lambda: ref.gqa_full(q, k, v, causal=True, rope_theta=10000.0), 64,
        "1 of 64 (batch, kv-head) units")
    q, k, v, do = b(1, 4096, 2, 128), b(1, 4096, 1, 128), b(1, 4096, 1, 128), b(1, 2, 4096, 128)
    add("gqa_full_backward", lambda: ref.gqa_full_backward(do, q, k, v), 8, "1 of 8 kv groups, float64")
    add("gqa_full_backward_saved", lambda: ref.gqa_full_backward(do, q, k, v), 8,
        "1 of 8 kv groups, float64 (the restatement computes its own forward)")
    del q, k, v, do
    xr, c, s = n(128, 65536), n(64, 65536), n(64, 65536)
    add("rope_single_freq_apply", lambda: ref.rope_single_freq_apply(xr, c, s), 4, "65536 of 262144 columns")
    del xr, c, s
    th, gr, m, vv = n(10944, 2048), n(10944, 2048), n(10944, 2048), np.abs(n(10944, 2048))
    add("adamw", lambda: ref.adamw(th, gr, m, vv), 1, "whole")
    del th, gr, m, vv
    dt = np.logaddexp(0, n(1, 4096, 256) - 3).astype(np.float32)
    xx, A = b(1, 4096, 256), (-np.exp(0.5 * n(256, 16))).astype(np.float32)
    Bm, Cm, Dv = n(1, 4096, 16), n(1, 4096, 16), np.ones(256, dtype=np.float32)
    add("mamba", lambda: ref.mamba(dt, xx, A, Bm, Cm, Dv), 128, "1 of 8 batch entries x 256 of 4096 channels")
    # the fp32-accuracy rows compute the same fp32 numpy forward
    for f32_name, base in (("matmul_f32", "matmul"), ("transpose_matmul_f32", "transpose_matmul"),
                           ("bmm_f32", "bmm"), ("bmm_softmax_f32", "bmm_softmax")):
        out[f32_name] = out[base]
    return out


def traffic_from_profiles(key: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary (or None)."""
    p = REPO / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        parts = ln.split()
        if len(parts) >= 2 and parts[0] == key:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


def cpu_sample_rmsnorm_matmul(budget_s=10.0):
    """Time the numpy oracle on a bounded row sample of the headline workload."""
    from oracle import ops as ref
    try:  # every host core, whatever the launcher set (the env above covers OpenBLAS at load)
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count() or 1)
    except Exception:
        pass
    rng = np.random.default_rng(42)
    w = (0.02 * rng.standard_normal((HEAD_K, HEAD_N), dtype=np.float32))
    gam = (1 + 0.1 * rng.standard_normal(HEAD_K, dtype=np.float32)).astype(np.float32)
    rows = 64
    x = rng.standard_normal((rows, HEAD_K), dtype=np.float32)
    t0 = time.perf_counter()
    ref.rmsnorm_matmul(x, w, gam, 1e-6)
    dt = time.perf_counter() - t0
    rows = int(min(HEAD_M, max(64, rows * (budget_s / 3) / max(dt, 1e-6))))
    x = rng.standard_normal((rows, HEAD_K), dtype=np.float32)
    reps, total = 0, 0.0
    while total < budget_s / 1.5 or reps < 2:
        t0 = time.perf_counter()
        ref.rmsnorm_matmul(x, w, gam, 1e-6)
        total += time.perf_counter() - t0
        reps += 1
        if reps >= 20:
            break
    flops = 2.0 * rows * HEAD_N * HEAD_K * reps
    return {"value": round(flops / total / 1e12, 4), "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port",
            "sample": f"{reps} x numpy oracle rmsnorm_matmul on {rows} of {HEAD_M} rows "
                      f"({total:.1f} s, fp32 on bf16-valued inputs)"}


def run_kda(args, dist: Dist):
    import torch
    torch.cuda.set_device(dist.local)
    dist.init("nccl")
    import kda
    from kda.shard import ranges
    dev = torch.device("cuda", dist.local)
    pk, pk_kind = peaks()
    stream = torch.cuda.current_stream()
    flush = _flush_buf(torch, dev)
    world, rank = dist.world, dist.rank

    # this rank's row block of the one configuration (every rank draws the same
    # X and keeps its rows; W and gamma are replicated)
    rr = ranges(HEAD_M, world)[rank]
    Mr = len(rr)
    X, gam, W = head_inputs(torch, dev)
    X = X[rr.start:rr.stop].contiguous()
    Y = torch.empty(Mr, HEAD_N, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(kda.ops._ws_size("kda_rmsnorm_matmul_workspace_size", Mr, HEAD_K, HEAD_N),
                     dtype=torch.uint8, device=dev)

    def step_call():
        kda.rmsnorm_matmul(X, W, gam, 1e-6, out=Y, workspace=ws)

    # one step = the pre-pass + GEMM launches, replayed from a CUDA graph
    step_replay = as_graph(torch, step_call)
    step = step_replay or step_call
    step_timing = "CUDA graph replay of one step" if step_replay is not None else "direct calls"

    clocks = Clocks(dist.local)
    clocks.start()

    def keep_busy(n_new, limit_s):
        """Run untimed steps until the sampler has n_new more readings under load
        (every rank runs the same number of rounds: the stop decision is rank 0's)."""
        n = clocks.count()
        t_end = time.time() + limit_s
        while True:
            stop = clocks.count() >= n + n_new or time.time() >= t_end
            if dist.pg:
                stop = dist.max(1.0 if stop else 0.0) > 0.5
            if stop:
                break
            for _ in range(8):
                flush.fill_(1)
                step()
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    first_loaded = clocks.count()
    keep_busy(2, 5.0)
    dist.barrier()
    torch.cuda.synchronize()
    times = time_steps(torch, step, args.steps, 0, flush, stream)
    torch.cuda.synchronize()
    keep_busy(1, 3.0)
    dist.barrier()
    clk = clocks.stop(first_loaded)
    clk["note"] = "sampled every 50 ms while the headline step ran (warm-up, timed steps, trailing steps)"
    step_ms = dist.max(statistics.mean(times))
    p50_ms = dist.max(statistics.median(times))
    value = HEAD_FLOP / (step_ms * 1e-3) / 1e12

    # dominant kernel alone: the tcgen05 GEMM on this rank's normalized rows
    A = torch.empty(Mr, HEAD_K, dtype=torch.bfloat16, device=dev)
    A.copy_(ws[: Mr * HEAD_K * 2].view(torch.bfloat16).view(Mr, HEAD_K))
    g_call = lambda: kda.matmul(A, W, out=Y)  # noqa: E731
    gtimes = time_steps(torch, as_graph(torch, g_call) or g_call, args.steps, 2, flush, stream)
    g_ms = statistics.mean(gtimes)
    g_flop = 2.0 * Mr * HEAD_N * HEAD_K
    g_ach = g_flop / (g_ms * 1e-3) / 1e12
    peak = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    # per launch, from the ncu capture of the full-size launch (N = 1)
    traffic = traffic_from_profiles("gemm_bf16_256x4_rmsnorm_matmul") if world == 1 else None
    roofline = {"bound": "tensor", "kernel": "kda::gemm::gemm_kernel<256,K-major A,MN-major B,bf16 out,2-SM pair>",
                "achieved": round(g_ach, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(g_ach / peak, 3),
                "peak_kind": f"{pk_kind} burst bf16 (cuBLAS)", "traffic": traffic,
                "algorithmic_flops": g_flop, "kernel_ms": round(g_ms, 4)}

    # end to end through the public API from pinned host buffers.  Each rank
    # uploads its X rows and its 1/N of W's rows; with N > 1 the W parts are
    # all-gathered over NVLink (NCCL) into the full W every rank multiplies
    # by; the op runs and each rank reads its Y rows back.  Steps are pipelined
    # over an upload, a compute and a read-back stream with two device buffer
    # sets (step i's read-back and step i+1's upload use the two directions of
    # the PCIe link at once); the time runs from the first upload to the last
    # read-back, max over ranks.
    nbuf = 2
    wr = ranges(HEAD_K, world)
    even_w = all(len(r) == len(wr[0]) for r in wr)  # all_gather_into_tensor needs equal parts
    wpart = wr[rank] if (world > 1 and even_w) else range(0, HEAD_K)
    hX = X.cpu().pin_memory()
    hW = W[wpart.start:wpart.stop].cpu().pin_memory()
    hg = gam.cpu().pin_memory()
    hY = [torch.empty(Mr, HEAD_N, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    dX = [torch.empty_like(X) for _ in range(nbuf)]
    dW = [torch.empty_like(W) for _ in range(nbuf)]
    dWp = [torch.empty(len(wpart), HEAD_N, dtype=torch.bfloat16, device=dev) for _ in range(nbuf)]
    dg = [torch.empty_like(gam) for _ in range(nbuf)]
    dY = [torch.empty_like(Y) for _ in range(nbuf)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_c = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    gather = world > 1 and even_w

    def e2e_run(n):
        for i in range(n):
            k = i % nbuf
            if i >= nbuf:
                s_in.wait_event(ev_c[k])  # step i - nbuf has finished reading buffer set k
            with torch.cuda.stream(s_in):
                dX[k].copy_(hX, non_blocking=True)
                if gather:
                    dWp[k].copy_(hW, non_blocking=True)
                    dist.pg.all_gather_into_tensor(dW[k], dWp[k])
                else:
                    dW[k].copy_(hW, non_blocking=True)
                dg[k].copy_(hg, non_blocking=True)
                ev_in[k].record(s_in)
            stream.wait_event(ev_in[k])
            if i >= nbuf:
                stream.wait_event(ev_out[k])  # ... and its Y has been read back
            with torch.cuda.stream(stream):
                kda.rmsnorm_matmul(dX[k], dW[k], dg[k], 1e-6, out=dY[k], workspace=ws)
                ev_c[k].record(stream)
            s_out.wait_event(ev_c[k])
            with torch.cuda.stream(s_out):
                hY[k].copy_(dY[k], non_blocking=True)
                ev_out[k].record(s_out)

    e2e_run(nbuf + 1)  # warm-up
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e_steps = max(6, args.steps)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(s_in)
    e2e_run(e_steps)
    s_in.wait_stream(stream)
    s_in.wait_stream(s_out)
    t_end.record(s_in)
    t_end.synchronize()
    e_ms = dist.max(t_start.elapsed_time(t_end) / e_steps)
    torch.cuda.synchronize()
    h2d = hX.numel() * 2 + hW.numel() * 2 + hg.numel() * 4
    d2h = hY[0].numel() * 2
    h2d_all = dist.sum(h2d)
    d2h_all = dist.sum(d2h)
    e2e = {"value": round(HEAD_FLOP / (e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": int(h2d_all), "d2h_bytes_per_step": int(d2h_all), "ms_per_step": round(e_ms, 4),
           "steps": e_steps,
           "pipeline": "upload / compute / read-back streams, 2 buffer sets"
                       + ("; W rows uploaded 1/N per rank + NCCL all-gather" if gather else "")}
    del hX, hW, hY, dX, dW, dWp, dg, dY, A

    ops = None
    if not args.no_ops_table:
        del X, W, Y, ws
        torch.cuda.empty_cache()
        ops = ops_table(torch, kda, dev, pk, flush, dist=dist)

    zero1 = None
    if world > 1 and not args.no_ops_table:
        torch.cuda.empty_cache()
        zero1 = zero1_run(torch, dist, args.steps, args.warmup)

    dist.barrier()
    line = None
    if rank == 0:
        cpu = cpu_sample_rmsnorm_matmul() if world == 1 else None
        cpu_table = cpu_ops() if (world == 1 and ops is not None) else {}
        if ops is not None:
            # full details on stderr; the JSON line keeps [p50 ms, frac, cpu ms]
            detail = {k: dict(v, cpu_ms=cpu_table.get(k, (None, None))[0],
                              cpu_sample=cpu_table.get(k, (None, None))[1]) for k, v in ops.items()}
            print(json.dumps({"ops_detail": detail, "n_gpus": world}), file=sys.stderr, flush=True)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
            "p50_ms": round(p50_ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) X, N(0,0.02) W, 1+0.1N(0,1) gamma)",
            "config": {"workload": "rmsnorm_matmul X[4096,4096] W[4096,11008] bf16, gamma fp32, eps 1e-6",
                       "parallelism": f"row blocks x{world}: X[{Mr},4096] per GPU, W replicated",
                       "l2": "flushed before every timed step (256 MB write + 256 MB read)",
                       "timing": step_timing},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": 2 * args.steps, "clocks": clk,
        }
        if ops is not None:
            line["ops_cols"] = ["p50_ms", "frac_of_roofline", "cpu_numpy_ms"]
            # compact, so the whole line stays inside a 3 KB log tail: CPU ms to
            # three significant figures
            def _cpu(k):
                c = cpu_table.get(k, (None, None))[0]
                return None if c is None else float(f"{c:.3g}")
            line["ops"] = {k: ([v.get("p50_ms"), v.get("frac"), _cpu(k)]
                               if "p50_ms" in v else [None, None, v.get("error", "")[:60]])
                           for k, v in ops.items()}
            line["ops_exp_frac"] = {k: v["exp_bound"]["frac"] for k, v in ops.items() if "exp_bound" in v}
            if world == 1:
                line["cpu_cores"] = cpu_cores()
        if zero1 is not None:
            line["zero1_adamw"] = zero1
    dist.close()
    return line


# --------------------------------------------------------------------------- #
# reference arm: the reference's algorithm (numpy restatement) on host cores
# --------------------------------------------------------------------------- #
def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return None
    from oracle import ops as ref
    try:  # every host core, whatever the launcher set (the env above covers OpenBLAS at load)
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count() or 1)
    except Exception:
        pass
    rng = np.random.default_rng(42)
    w = (0.02 * rng.standard_normal((HEAD_K, HEAD_N), dtype=np.float32))
    gam = (1 + 0.1 * rng.standard_normal(HEAD_K, dtype=np.float32)).astype(np.float32)
    rows = 256
    x = rng.standard_normal((rows, HEAD_K), dtype=np.float32)
    for _ in range(args.warmup):
        ref.rmsnorm_matmul(x[:64], w, gam, 1e-6)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.rmsnorm_matmul(x, w, gam, 1e-6)
        times.append(time.perf_counter() - t0)
    step_s = statistics.mean(times)
    value = 2.0 * rows * HEAD_N * HEAD_K / step_s / 1e12
    cores = cpu_cores()
    sample = (f"numpy restatement of the reference forward (oracle/), {rows} of {HEAD_M} rows per step, "
              f"fp32; the reference's NKI kernels need Trainium")
    return {"metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "rmsnorm_matmul X[4096,4096] W[4096,11008] bf16, gamma fp32, eps 1e-6",
                       "parallelism": f"host cores of rank 0 ({cores} threads), {rows}-row sample per step"},
            "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def zero1_run(torch, dist, steps, warmup, numel=1 << 28):
    """ZeRO-1 AdamW step over a flat fp32 buffer of ``numel`` parameters
    replicated on every rank (torchrun, one process per GPU, process group
    already initialised): the fused kernel (peer loads of every rank's
    gradient shard, AdamW, peer stores of the new parameters) against the
    collective path (NCCL reduce-scatter, multi-tensor AdamW, NCCL all-gather).
    Each step's device time includes its two one-element barriers (fused) or
    its collectives; max over ranks.  Before timing, one step of each path
    from the same parameters, gradients and zero moments is compared (max
    absolute difference of the parameters, max over ranks).  Roofline: the
    bytes one rank must move over NVLink per direction, 2 (world-1) shard x 4 B
    (gradient shards read from peers + parameter shards stored to peers), at
    the measured 770 GB/s peer-copy rate, against the rank's local HBM traffic
    (2 world + 5) shard x 4 B at the measured copy peak."""
    from kda.zero import Zero1AdamW
    dev = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=dev)
    res, after = {}, {}
    for fused in (True, False):
        opt = Zero1AdamW(numel, device=dev, fused=fused)
        gen.manual_seed(1234)                      # same parameters on every rank
        opt.param.normal_(generator=gen)
        gen.manual_seed(99 + dist.rank)            # each rank's own gradients
        opt.grad.normal_(generator=gen)
        opt.step()
        torch.cuda.synchronize()
        after[fused] = opt.param[: opt.numel].clone()
        for _ in range(warmup):
            opt.step()
        times = []
        for _ in range(steps):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            dist.barrier()
            torch.cuda.synchronize()
            s.record()
            opt.step()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        res[fused] = dist.max(statistics.median(times))
        opt.close()
        del opt
        torch.cuda.empty_cache()
    diff = dist.max(float((after[True] - after[False]).abs().max().item()))
    scale = dist.max(float(after[False].abs().max().item()))
    del after
    dist.barrier()
    world = dist.world
    shard = numel // world
    nvl_bytes = 2 * (world - 1) * shard * 4
    hbm_bytes = (2 * world + 5) * shard * 4
    pk, kind = peaks()
    t_nvl = nvl_bytes / 770e9
    t_hbm = hbm_bytes / (pk["hbm_gbs"] * 1e9)
    bound = max(t_nvl, t_hbm)
    return {"params": numel, "fused_ms": round(res[True], 4), "collective_ms": round(res[False], 4),
            "speedup": round(res[False] / res[True], 3), "bound": "nvlink" if t_nvl >= t_hbm else "hbm",
            "frac": round(bound * 1e3 / res[True], 3), "max_abs_diff": diff, "max_abs_param": round(scale, 3)}


def zero1_bench(args, dist, numel=1 << 28):
    """``bench.py --op zero1_adamw``: the ZeRO-1 comparison on its own, one line."""
    import torch
    torch.cuda.set_device(dist.local)
    dist.init("nccl")
    r = zero1_run(torch, dist, args.steps, args.warmup, numel)
    line = {"op": "zero1_adamw", "n_gpus": dist.world, "dtype": "f32", "steps": args.steps, **r} \
        if dist.rank == 0 else None
    dist.close()
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["kda", "reference"], default="kda")
    ap.add_argument("--no-ops-table", action="store_true", help="skip the per-operator table")
    ap.add_argument("--op", default=None,
                    help="time only this operator at its configuration (per-op table entry; used for profiling)")
    ap.add_argument("--small", action="store_true",
                    help="with --op mamba: 512 of the 4096 steps (a profiling case, same kernel and layout)")
    ap.add_argument("--partition", type=int, default=1,
                    help="with --op: time rank 0's part of the configuration split N ways, on one GPU "
                         "(the shape one rank of an N-GPU run gets; used for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    dist = Dist()
    if args.op == "zero1_adamw" and args.impl == "kda":
        line = zero1_bench(args, dist)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    if args.op and args.impl == "kda":
        import torch
        import kda
        dev = torch.device("cuda", dist.local)
        torch.cuda.set_device(dev)
        pk, _ = peaks()
        part = None
        if args.partition > 1:  # rank 0 of N, without a process group (no collectives)
            part = Dist()
            part.world, part.rank = args.partition, 0
        rows = ops_table(torch, kda, dev, pk, _flush_buf(torch, dev), dist=part, iters=args.steps, only=args.op,
                         small=args.small)
        if args.op not in rows:
            ap.error(f"unknown --op {args.op!r}")
        print(json.dumps({"op": args.op, **rows[args.op]}), flush=True)
        return 0
    if args.impl == "reference":
        line = run_reference(args, dist)
    else:
        line = run_kda(args, dist)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
