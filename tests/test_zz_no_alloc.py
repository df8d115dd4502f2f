"""The allocation-free scan entry point, called through the C ABI.

kda_mamba_scan_noalloc serves callers that cannot allocate device memory: a
host binding (cgo, JNI, a plugin) that its framework hands only the input and
output buffers, with no way to ask that framework's allocator for a workspace,
or code that must not call cudaMalloc because it can synchronise the device
and stall work queued on other streams.  Its chunk summaries live in a fixed
array inside the library instead of a caller workspace.

Each case calls it twice in a row (the shared array keeps the previous call's
contents) and compares the output with the workspace entry point's and with the
CPU oracle: the reference's chunked 2-D case, a single-chunk channels-last
shape (no scratch used), a bf16 batch-2 chunked shape, and a smaller chunked
shape right after a larger one.  A shape that needs more than the array holds
must be refused before any launch.

This file sorts last so that a run stopping at its first failure has already
run every other test.
"""

import ctypes as C

import numpy as np
import pytest

from oracle import inputs, ops as ref
from oracle.metrics import GATE_BF16, GATE_FP32, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _lib_fn():
    from kda import _lib
    lib = _lib.lib()
    return lib, _lib._attach(lib, "kda_mamba_scan_noalloc")


def _to_gpu(d, u_bf16=False):
    g = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items() if isinstance(v, np.ndarray)}
    if u_bf16:
        g["u"] = g["u"].to(torch.bfloat16)
    return g


def _call_noalloc(g, y):
    """kda_mamba_scan_noalloc with the strides kda.mamba passes for the same tensors."""
    lib, fn = _lib_fn()
    delta = g["delta"]
    S = g["a"].shape[1]
    if delta.dim() == 2:                      # reference layout: (C, M) channel-major
        Cn, M = delta.shape
        batch, L, Dm = 1, M, Cn
        ld, bc = (Cn * M, 1, M), (S * M, 1, M)
    else:                                     # channels-last (B, L, D)
        batch, L, Dm = delta.shape
        ld, bc = (L * Dm, Dm, 1), (L * S, S, 1)
    ptr = lambda t: C.c_void_p(0 if t is None else t.data_ptr())  # noqa: E731
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = fn(ptr(delta), ptr(g["u"]), ptr(g["a"]), ptr(g["b"]), ptr(g["c"]), ptr(g.get("D")), ptr(y),
            batch, L, Dm, S, *ld, *bc, int(g["u"].dtype == torch.bfloat16), int(y.dtype == torch.bfloat16),
            stream)
    return st, lib


def _check_case(d, u_bf16=False, y_dtype=torch.float32, want=None):
    import kda

    g = _to_gpu(d, u_bf16)
    ws_entry = kda.mamba(g["delta"], g["u"], g["a"], g["b"], g["c"], g.get("D"), out_dtype=y_dtype)
    if want is None:
        want = ref.mamba(d["delta"], d["u"], d["a"], d["b"], d["c"], d.get("D"))
    gate = GATE_BF16 if y_dtype == torch.bfloat16 else GATE_FP32
    torch.cuda.synchronize()
    for _ in range(2):
        y = torch.full_like(ws_entry, float("nan"))
        st, lib = _call_noalloc(g, y)
        assert st == 0, lib.kda_last_error().decode()
        torch.cuda.synchronize()
        got = y.float().cpu().numpy()
        assert rel_l2(got, ws_entry.float().cpu().numpy()) <= gate
        assert rel_l2(got, want) <= gate
    assert kda.device_error() == 0


def _ws_bytes(batch, L, Dm):
    import kda
    return kda.ops._ws_size("kda_mamba_scan_workspace_size", batch, L, Dm, 16)


def test_noalloc_reference_chunked_case():
    d = inputs.nkibench("mamba", 42)                 # C=256, M=7168: the chunked path
    assert _ws_bytes(1, 7168, 256) > 0
    _check_case(d)


def test_noalloc_single_chunk_channels_last():
    d = inputs.config("mamba", 7, scale=16)          # B8, L256, D4096: one chunk, no scratch
    for k in ("delta", "u", "b", "c"):
        d[k] = np.ascontiguousarray(d[k][:, :200])
    assert _ws_bytes(8, 200, 4096) == 0
    _check_case(d, u_bf16=True, y_dtype=torch.bfloat16)


def test_noalloc_bf16_batch2_chunked():
    # the configuration's distributions at B2, L2048, D256 (16 chunks)
    from oracle.bf16 import to_bf16_rne
    rng = np.random.default_rng(11)
    B, L, Dm, N = 2, 2048, 256, 16
    n = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    d = {"delta": np.logaddexp(0, n(B, L, Dm) - 3).astype(np.float32), "u": to_bf16_rne(n(B, L, Dm)),
         "a": (-np.exp(0.5 * n(Dm, N))).astype(np.float32), "b": n(B, L, N), "c": n(B, L, N),
         "D": np.ones(Dm, dtype=np.float32)}
    assert _ws_bytes(B, L, Dm) > 0
    _check_case(d, u_bf16=True, y_dtype=torch.bfloat16)


def test_noalloc_small_after_large():
    """A smaller chunked shape right after a larger one: the shared array still
    holds the larger call's summaries when the smaller call starts."""
    big = inputs.nkibench("mamba", 3)                # C=256, M=7168
    small = inputs.nkibench("mamba", 4, C=64, M=1000)
    assert _ws_bytes(1, 1000, 64) > 0
    _check_case(big)
    _check_case(small)


def test_mamba_scan_noalloc_rejects_oversized_scratch():
    d = inputs.nkibench("mamba", 1, C=1024, M=8192)  # 32 chunks x 1024 channels: > 1 MiB of summaries
    g = _to_gpu(d)
    y = torch.empty_like(g["delta"])
    st, lib = _call_noalloc(g, y)
    assert st == 2  # KDA_UNSUPPORTED, refused on the host before any launch
    assert "built-in array" in lib.kda_last_error().decode()
