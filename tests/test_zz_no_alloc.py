"""The allocation-free scan entry point, called through the C ABI.

kda_mamba_scan_noalloc serves callers that cannot allocate device memory (a
host binding handed only its inputs and outputs, or code that must not call
cudaMalloc because it can synchronise the device): its chunk summaries live in
a fixed array inside the library instead of a caller workspace.  Its output
must match the workspace entry point's on the reference's chunked case, on two
calls in a row (the shared array keeps the previous call's contents), and a
shape that needs more than the array holds must be refused before any launch.

This file sorts last so that a run stopping at its first failure has already
run every other test.
"""

import ctypes as C

import numpy as np
import pytest

from oracle import inputs
from oracle.metrics import GATE_FP32, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _args(d):
    g = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items()}
    Cn, M = g["delta"].shape
    S = g["a"].shape[1]
    return g, Cn, M, S


def _call_noalloc(lib, fn, g, y, Cn, M, S):
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    # reference 2-D layout: batch 1, ld_t = 1, ld_d = M, bc_ld_t = 1, bc_ld_n = M
    return fn(ptr(g["delta"]), ptr(g["u"]), ptr(g["a"]), ptr(g["b"]), ptr(g["c"]), C.c_void_p(0), ptr(y),
              1, M, Cn, S, Cn * M, 1, M, S * M, 1, M, 0, 0, stream)


def test_mamba_scan_noalloc_matches_workspace_entry_point():
    import kda
    from kda import _lib

    lib = _lib.lib()
    fn = _lib._attach(lib, "kda_mamba_scan_noalloc")
    d = inputs.nkibench("mamba", 42)                 # C=256, M=7168: the chunked path
    g, Cn, M, S = _args(d)
    assert kda.ops._ws_size("kda_mamba_scan_workspace_size", 1, M, Cn, S) > 0
    want = kda.mamba(g["delta"], g["u"], g["a"], g["b"], g["c"])   # workspace entry point
    torch.cuda.synchronize()
    for _ in range(2):
        y = torch.full_like(want, float("nan"))
        st = _call_noalloc(lib, fn, g, y, Cn, M, S)
        assert st == 0, lib.kda_last_error().decode()
        torch.cuda.synchronize()
        assert rel_l2(y.cpu().numpy(), want.cpu().numpy()) <= GATE_FP32
    assert kda.device_error() == 0


def test_mamba_scan_noalloc_rejects_oversized_scratch():
    from kda import _lib

    lib = _lib.lib()
    fn = _lib._attach(lib, "kda_mamba_scan_noalloc")
    d = inputs.nkibench("mamba", 1, C=1024, M=8192)  # 32 chunks x 1024 channels: > 1 MiB of summaries
    g, Cn, M, S = _args(d)
    y = torch.empty_like(g["delta"])
    st = _call_noalloc(lib, fn, g, y, Cn, M, S)
    assert st == 2  # KDA_UNSUPPORTED, refused on the host before any launch
    assert "built-in array" in lib.kda_last_error().decode()
