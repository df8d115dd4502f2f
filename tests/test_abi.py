"""The C ABI library: loads without a GPU, exports every declared symbol, and
rejects bad arguments on the host before any launch (no GPU needed)."""

import ctypes as C
import re
from pathlib import Path

import pytest

from conftest import REPO

HEADER = REPO / "include" / "kda.h"


def declared_functions():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kda_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from kda import _lib
    return _lib.lib()


def test_header_declares_all_ops():
    names = declared_functions()
    for op in ("silu_f32", "rope_single_freq_apply_f32", "adamw_f32", "mamba_scan", "matmul_bf16",
               "transpose_matmul_bf16", "bmm_bf16", "bmm_softmax_bf16", "rmsnorm_matmul_bf16",
               "add_rmsnorm_matmul_bf16", "matmul_add_rmsnorm_bf16", "swiglu_bf16", "lora_bf16",
               "gqa_full_bf16"):
        assert f"kda_{op}" in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared in kda.h but not exported: {missing}"


def test_bindings_cover_header():
    from kda import _lib
    assert set(declared_functions()) == set(_lib.PROTOTYPES)


def test_abi_version_and_status_strings(lib):
    from kda import _lib
    assert lib.kda_abi_version() == 1
    for code, name in _lib.STATUS_NAMES.items():
        assert lib.kda_status_string(code).decode() == name


@pytest.mark.parametrize("fn,args", [
    ("kda_silu_f32", (None, None, 16, None)),
    ("kda_silu_f32", (None, None, -1, None)),
    ("kda_adamw_f32", (None, None, None, None, None, 8, 0, None)),
    ("kda_rope_single_freq_apply_f32", (None, None, None, None, 3, 8, None)),
    ("kda_matmul_bf16", (None, None, None, 16, 16, 16, None)),
    ("kda_matmul_bf16", (1, 1, 1, 0, 16, 16, None)),
    ("kda_bmm_bf16", (None, None, None, 0, 16, 16, 16, None)),
    ("kda_bmm_f32", (None, None, None, 1, 16, 16, 16, None, 0, None)),
    ("kda_transpose_matmul_f32", (None, None, None, 16, 16, 16, None, 0, None)),
    ("kda_gqa_full_bf16", (None, None, None, None, 1, 16, 2, 1, 128, 0, 0.0, 0, None, 0, None)),
    ("kda_gqa_full_lse_bf16", (16, 16, 16, 16, None, 1, 16, 2, 1, 128, 0, 0.0, 0, None, 0, None)),
    ("kda_swiglu_gu_bf16", (16, 16, 16, 16, 16, None, 16, 16, 16, 16, None, 0, None)),
    ("kda_swiglu_backward_saved_bf16", (16, 16, 16, 16, 16, None, None, 16, 16, 16, 16, 16, 16, 16, None, 0,
                                        None)),
    ("kda_gqa_full_backward_saved_bf16", (16, 16, 16, 16, None, None, 16, 16, 16, 1, 16, 2, 1, 128, 0, 0.0,
                                          None, 0, None)),
])
def test_invalid_arguments_rejected_on_host(lib, fn, args):
    from kda import _lib
    f = _lib._attach(lib, fn)
    assert f(*args) == 1  # KDA_INVALID_ARG, before any CUDA call
    assert lib.kda_last_error().decode()


def test_unsupported_shapes_rejected_on_host(lib):
    from kda import _lib
    f = _lib._attach(lib, "kda_matmul_bf16")
    # K not a multiple of 8 violates the TMA 16-byte stride rule
    assert f(16, 16, 16, 16, 12, 16, None) == 2
    assert "multiples of 8" in lib.kda_last_error().decode()


def test_workspace_queries(lib):
    from kda import _lib
    q = _lib._attach(lib, "kda_rmsnorm_matmul_workspace_size")
    assert q(4096, 4096, 11008) >= 4096 * 4096 * 2
    q = _lib._attach(lib, "kda_transpose_matmul_f32_workspace_size")
    assert q(4096, 2048, 10944) == 2 * 4096 * 2048 * 2 + 2 * 2048 * 10944 * 2   # hi + lo of both operands
    q = _lib._attach(lib, "kda_bmm_f32_workspace_size")
    assert q(16, 4096, 64, 4096) == 2 * 16 * 4096 * 64 * 2 * 2
    assert q(0, 16, 16, 16) == 0
    q = _lib._attach(lib, "kda_mamba_scan_workspace_size")
    assert q(8, 4096, 4096, 16) == 0          # enough channels: no chunking
    assert q(1, 7168, 256, 16) > 0            # few channels: chunked scan
    q = _lib._attach(lib, "kda_swiglu_workspace_size")
    assert q(8192, 4096, 14336) >= 8192 * 14336 * 2
    q = _lib._attach(lib, "kda_lora_workspace_size")
    t = 4096 * 128 * 2                            # t = x @ a (bf16)
    assert q(4096, 5120, 12288, 128) == t + 4 * 4096 * 128 * 4   # K split in 4: fp32 partials
    assert q(520, 200, 264, 16) == 520 * 16 * 2                  # 4 k-blocks: no split
    assert q(4096, 5120, 12288, 256) == 4096 * 256 * 2           # R > 128: no split
    q = _lib._attach(lib, "kda_gqa_full_workspace_size")
    vt = 2 * 8 * 128 * 4096 * 2                   # transposed v (B=2, KH=8, S=4096)
    assert q(2, 4096, 32, 8, 128, 0.0) == vt
    assert q(2, 4096, 32, 8, 128, 10000.0) > vt   # + rotated q, k and the table
    assert q(1, 13, 2, 1, 128, 0.0) == 128 * 16 * 2  # keys padded to a multiple of 8
    assert q(1, 16, 2, 1, 64, 0.0) == 0           # head_dim other than 128 is unsupported
    full = _lib._attach(lib, "kda_gqa_full_backward_workspace_size")
    saved = _lib._attach(lib, "kda_gqa_full_backward_saved_workspace_size")
    for theta in (0.0, 10000.0):
        # the saved-forward backward needs no room for the forward's output, lse and workspace
        fwd = 1 * 16 * 4096 * 128 * 2 + 1 * 16 * 4096 * 4 + q(1, 4096, 16, 8, 128, theta)
        assert full(1, 4096, 16, 8, 128, theta) == saved(1, 4096, 16, 8, 128, theta) + fwd
    assert saved(1, 4096, 16, 8, 128, 0.0) == 16 * 4096 * 4 + 16 * 4096 * 128 * 4   # di + fp32 dq
    assert saved(1, 16, 3, 2, 128, 0.0) == 0      # query heads not a multiple of kv heads
    full = _lib._attach(lib, "kda_swiglu_backward_workspace_size")
    saved = _lib._attach(lib, "kda_swiglu_backward_saved_workspace_size")
    # the saved-activation backward needs no room for g and u
    assert full(8192, 4096, 14336) == saved(8192, 4096, 14336) + 2 * 8192 * 14336 * 2
    assert _lib._attach(lib, "kda_swiglu_gu_workspace_size")(8192, 4096, 14336) == 8192 * 14336 * 2  # h


def test_ops_reject_cpu_tensors():
    import torch
    import kda
    with pytest.raises(ValueError):
        kda.silu(torch.zeros(4))
    with pytest.raises((ValueError, TypeError)):
        kda.matmul(torch.zeros(4, 4), torch.zeros(4, 4))


def test_plain_c_caller(tmp_path):
    """The library from a plain C program (what a cgo / JNI / N-API binding
    links against): compiled with gcc against include/kda.h and run without a GPU."""
    import shutil
    import subprocess
    from kda import _lib
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    exe = tmp_path / "abi_host_check"
    libdir = _lib.LIB_PATH.parent
    r = subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-I", str(REPO / "include"),
                        str(REPO / "tests" / "c" / "abi_host_check.c"), "-o", str(exe), f"-L{libdir}", "-lkda",
                        f"-Wl,-rpath,{libdir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "OK" in r.stdout
