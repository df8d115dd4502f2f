"""GPU parity: every operator through the C ABI vs the CPU oracle.

Gates (north star): relative-L2 <= 1e-5 for the fp32 operators (silu, rope,
adamw, mamba with fp32 output) and <= 1e-2 for the bf16 operators.  Inputs are
the reference's seeded draws (``oracle.inputs``); bf16 inputs are rounded RNE
before both the kernel and the oracle see them, so the gate measures kernel
error.  The golden-vector cases additionally compare against the reference's
own outputs (``tests/golden``), computed from the unrounded fp32 inputs.
"""

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import inputs, ops as ref
from oracle.metrics import GATE_BF16, GATE_FP32, rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def kda():
    import kda as k
    return k


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    return t.float().cpu().numpy()


def gpu_args(op, d):
    out = {}
    for k, v in d.items():
        if isinstance(v, np.ndarray):
            out[k] = dev(v, torch.bfloat16 if k in inputs.BF16_ARGS.get(op, ()) else torch.float32)
        else:
            out[k] = v
    return out


@pytest.fixture(autouse=True)
def no_device_error(kda):
    yield
    torch.cuda.synchronize()
    assert kda.device_error() == 0, "a kernel reported an expired bounded wait"


# --------------------------------------------------------------- elementwise
@pytest.mark.parametrize("shape", [(4096, 8192), (3, 5), (1,), (0,), (1000003,)])
def test_silu(kda, shape):
    x = np.random.default_rng(0).normal(size=shape).astype(np.float32) * 4
    y = kda.silu(dev(x))
    if x.size:
        assert rel_l2(host(y), ref.silu(x)) <= GATE_FP32


def test_silu_unaligned_view(kda):
    x = dev(np.random.default_rng(1).normal(size=4099).astype(np.float32))
    xs = x[1:]          # 4-byte offset: scalar path
    y = kda.silu(xs)
    assert rel_l2(host(y), ref.silu(host(xs))) <= GATE_FP32


def test_silu_extremes(kda):
    x = np.array([-1e4, -90, -20, -1e-30, 0, 1e-30, 20, 90, 1e4], dtype=np.float32)
    y = host(kda.silu(dev(x)))
    assert np.all(np.isfinite(y))
    np.testing.assert_allclose(y, ref.silu(x), rtol=1e-6, atol=1e-30)


@pytest.mark.parametrize("D,S", [(128, 262144), (128, 4096), (4, 6), (64, 1001)])
def test_rope(kda, D, S):
    d = inputs.nkibench("rope_single_freq_apply", 42, D=D, S=S)
    y = kda.rope_single_freq_apply(*gpu_args("rope_single_freq_apply", d).values())
    assert rel_l2(host(y), ref.rope_single_freq_apply(**d)) <= GATE_FP32


@pytest.mark.parametrize("M,N", [(10944, 2048), (7, 9), (1, 1)])
def test_adamw(kda, M, N):
    d = inputs.nkibench("adamw", 42, M=M, N=N)
    a = gpu_args("adamw", d)
    y = kda.adamw(**a)
    assert rel_l2(host(y), ref.adamw(**d)) <= GATE_FP32


def test_adamw_inplace_state(kda):
    d = inputs.nkibench("adamw", 3, M=33, N=64)
    a = gpu_args("adamw", d)
    y = kda.adamw(**a, inplace_state=True)
    th, m, v = ref.adamw_state(**d)
    assert rel_l2(host(y), th) <= GATE_FP32
    assert rel_l2(host(a["m"]), m) <= GATE_FP32
    assert rel_l2(host(a["v"]), v) <= GATE_FP32


# ------------------------------------------------------------------- mamba
@pytest.mark.parametrize("C,M", [(256, 7168), (16, 40), (130, 1000)])
def test_mamba_reference_layout(kda, C, M):
    d = inputs.nkibench("mamba", 42, C=C, M=M)
    y = kda.mamba(**gpu_args("mamba", d))
    assert y.dtype == torch.float32
    assert rel_l2(host(y), ref.mamba(**d)) <= GATE_FP32


@pytest.mark.parametrize("ydt", ["f32", "bf16"])
def test_mamba_batched_config_scaled(kda, ydt):
    d = inputs.config("mamba", 42, scale=16)        # B8, L256, D4096, N16
    d["u"] = d["u"][:, :, :512].copy()
    d["delta"] = d["delta"][:, :, :512].copy()
    d["a"] = d["a"][:512].copy()
    d["D"] = d["D"][:512].copy()
    g = {k: dev(v) for k, v in d.items()}
    g["u"] = g["u"].to(torch.bfloat16)
    out_dtype = torch.float32 if ydt == "f32" else torch.bfloat16
    y = kda.mamba(g["delta"], g["u"], g["a"], g["b"], g["c"], g["D"], out_dtype=out_dtype)
    want = ref.mamba(d["delta"], d["u"], d["a"], d["b"], d["c"], d["D"])
    gate = GATE_FP32 if ydt == "f32" else GATE_BF16
    assert rel_l2(host(y), want) <= gate


def cuda_kernels_launched(fn):
    """Names of the CUDA kernels ``fn`` launches (torch profiler, CUPTI)."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    names = {e.key for e in prof.key_averages()}
    return out, names


_MAMBA_CL_WANT = {}


def _mamba_cl_case(L):
    """The north-star scan at full width (B8, D4096: batch x channels = 32768,
    one chunk, the channels-last kernel) and L steps, with its oracle output."""
    d = inputs.config("mamba", 42, scale=8)          # B8, L512, D4096, N16
    for k in ("delta", "u", "b", "c"):
        d[k] = np.ascontiguousarray(d[k][:, :L])
    if L not in _MAMBA_CL_WANT:
        _MAMBA_CL_WANT[L] = ref.mamba(d["delta"], d["u"], d["a"], d["b"], d["c"], d["D"])
    return d, _MAMBA_CL_WANT[L]


@pytest.mark.parametrize("L", [512, 500])            # 500: not a multiple of the 32-step tile
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
@pytest.mark.parametrize("ydt", ["f32", "bf16"])
def test_mamba_channels_last_full_width(kda, L, xdt, ydt):
    """The kernel the north-star configuration runs (scan_cl_kernel) against the
    oracle, at the configuration's full batch and channel count."""
    d, want = _mamba_cl_case(L)
    g = {k: dev(v) for k, v in d.items()}
    if xdt == "bf16":
        g["u"] = g["u"].to(torch.bfloat16)
    out_dtype = torch.float32 if ydt == "f32" else torch.bfloat16
    y, names = cuda_kernels_launched(
        lambda: kda.mamba(g["delta"], g["u"], g["a"], g["b"], g["c"], g["D"], out_dtype=out_dtype))
    assert any("scan_cl_kernel" in n for n in names), f"channels-last kernel not launched: {sorted(names)}"
    assert not any("carry_kernel" in n for n in names)
    assert y.dtype == out_dtype and tuple(y.shape) == (8, L, 4096)
    gate = GATE_FP32 if ydt == "f32" else GATE_BF16
    assert rel_l2(host(y), want) <= gate


@pytest.mark.parametrize("nb", [4, 2, 1])             # 16384 / 8192 / 4096 channels: 2 / 4 / 4 lanes each
@pytest.mark.parametrize("ydt", ["f32", "bf16"])
def test_mamba_channels_last_fewer_batches(kda, nb, ydt):
    """The batch entries one GPU gets when the configuration is split over 2 /
    4 / 8 GPUs: the channels-last kernel with several lanes per channel."""
    d, want = _mamba_cl_case(500)
    g = {k: dev(v) for k, v in d.items()}
    for k in ("delta", "u", "b", "c"):
        g[k] = g[k][:nb].contiguous()
    g["u"] = g["u"].to(torch.bfloat16)
    out_dtype = torch.float32 if ydt == "f32" else torch.bfloat16
    y, names = cuda_kernels_launched(
        lambda: kda.mamba(g["delta"], g["u"], g["a"], g["b"], g["c"], g["D"], out_dtype=out_dtype))
    assert any("scan_cl_kernel" in n for n in names), f"channels-last kernel not launched: {sorted(names)}"
    assert not any("carry_kernel" in n for n in names)
    gate = GATE_FP32 if ydt == "f32" else GATE_BF16
    assert rel_l2(host(y), want[:nb]) <= gate


# ------------------------------------------------------------ contractions
GOLDEN_OPS = ["matmul", "transpose_matmul", "bmm", "rmsnorm_matmul", "add_rmsnorm_matmul",
              "matmul_add_rmsnorm", "swiglu", "lora"]


def golden_case(op, seed, golden_meta):
    meta = golden_meta[f"{op}_s{seed}"]
    shape = dict(meta["shape"])
    if op == "gqa_full":
        shape["S"] = shape.pop("N")
    d = inputs.nkibench(op, seed, bf16=True, **shape)
    return d, np.load(GOLDEN / f"{op}_s{seed}.npy")


@pytest.mark.parametrize("op", GOLDEN_OPS)
@pytest.mark.parametrize("seed", [42, 0])
def test_contraction_vs_reference_golden(kda, op, seed, golden_meta):
    d, want = golden_case(op, seed, golden_meta)
    out = getattr(kda, op)(**gpu_args(op, d))
    got = host(out)
    assert got.shape == want.shape
    assert rel_l2(got, want) <= GATE_BF16            # vs the reference's fp32 output
    assert rel_l2(got, getattr(ref, op)(**d)) <= GATE_BF16


@pytest.mark.parametrize("M,K,N", [(1, 8, 8), (128, 64, 256), (129, 72, 264), (300, 1000, 520),
                                   (256, 4096, 128), (1024, 512, 2048)])
def test_matmul_shapes(kda, M, K, N):
    d = inputs.nkibench("matmul", 1, M=M, K=K, N=N)
    out = kda.matmul(**gpu_args("matmul", d))
    assert rel_l2(host(out), ref.matmul(**d)) <= GATE_BF16


FP32_GATE_REF = 2e-5  # the reference's own fp32 relative-L2 gate


@pytest.mark.parametrize("seed", [42, 0])
def test_matmul_f32_vs_reference_golden(kda, seed, golden_meta):
    """fp32 in / fp32 out (bf16 hi + lo split on the tensor core) against the
    reference's own fp32 outputs, from the unrounded fp32 draws, at its gate."""
    meta = golden_meta[f"matmul_s{seed}"]
    d = inputs.nkibench("matmul", seed, bf16=False, **dict(meta["shape"]))
    want = np.load(GOLDEN / f"matmul_s{seed}.npy")
    got = host(kda.matmul(dev(d["lhs"]), dev(d["rhs"])))
    assert rel_l2(got, want) <= FP32_GATE_REF


@pytest.mark.parametrize("M,K,N", [(1, 8, 8), (128, 64, 256), (129, 72, 264), (300, 1000, 520),
                                   (1024, 5120, 1536), (4096, 5120, 12288)])
def test_matmul_f32_shapes(kda, M, K, N):
    d = inputs.nkibench("matmul", 3, bf16=False, M=M, K=K, N=N)
    out = kda.matmul(dev(d["lhs"]), dev(d["rhs"]))
    assert out.dtype == torch.float32
    got = host(out)
    if M * N > 1e7:            # full NKIBench shape: a row sample of the oracle
        rows = slice(0, M, 97)
        assert rel_l2(got[rows], ref.matmul(d["lhs"][rows], d["rhs"])) <= FP32_GATE_REF
    else:
        assert rel_l2(got, ref.matmul(**d)) <= FP32_GATE_REF


@pytest.mark.parametrize("op", ["transpose_matmul", "bmm"])
@pytest.mark.parametrize("seed", [42, 0])
def test_split_f32_vs_reference_golden(kda, op, seed, golden_meta):
    """transpose_matmul / bmm with fp32 operands against the reference's own
    fp32 outputs from the unrounded draws, at the reference's fp32 gate."""
    meta = golden_meta[f"{op}_s{seed}"]
    d = inputs.nkibench(op, seed, bf16=False, **dict(meta["shape"]))
    want = np.load(GOLDEN / f"{op}_s{seed}.npy")
    out = getattr(kda, op)(dev(d["lhs"]), dev(d["rhs"]))
    assert out.dtype == torch.float32
    assert rel_l2(host(out), want) <= FP32_GATE_REF


@pytest.mark.parametrize("M,K,N", [(8, 8, 8), (136, 200, 264), (520, 1000, 264), (4096, 2048, 10944)])
def test_transpose_matmul_f32_shapes(kda, M, K, N):
    d = inputs.nkibench("transpose_matmul", 3, bf16=False, M=M, K=K, N=N)
    out = kda.transpose_matmul(dev(d["lhs"]), dev(d["rhs"]))
    got = host(out)
    if M * N > 1e7:            # full NKIBench shape: a row sample of the oracle
        rows = slice(0, M, 97)
        assert rel_l2(got[rows], ref.matmul(d["lhs"][:, rows].T, d["rhs"])) <= FP32_GATE_REF
    else:
        assert rel_l2(got, ref.transpose_matmul(**d)) <= FP32_GATE_REF


@pytest.mark.parametrize("B,M,K,N", [(16, 4096, 64, 4096), (3, 130, 64, 264), (2, 64, 512, 64)])
def test_bmm_f32_shapes(kda, B, M, K, N):
    d = inputs.nkibench("bmm", 3, bf16=False, B=B, M=M, K=K, N=N)
    out = kda.bmm(dev(d["lhs"]), dev(d["rhs"]))
    got = host(out)
    if B * M * N > 1e8:      # full NKIBench shape: a row sample of two batches
        rows = slice(0, M, 61)
        for b in (0, B - 1):
            assert rel_l2(got[b][rows], ref.matmul(d["lhs"][b][rows], d["rhs"][b])) <= FP32_GATE_REF
    else:
        assert rel_l2(got, ref.bmm(**d)) <= FP32_GATE_REF


@pytest.mark.parametrize("M,K,N", [(8, 8, 8), (136, 200, 264), (512, 2048, 1024)])
def test_transpose_matmul_shapes(kda, M, K, N):
    d = inputs.nkibench("transpose_matmul", 1, M=M, K=K, N=N)
    out = kda.transpose_matmul(**gpu_args("transpose_matmul", d))
    assert rel_l2(host(out), ref.transpose_matmul(**d)) <= GATE_BF16


@pytest.mark.parametrize("B,M,K,N", [(16, 4096, 64, 4096), (3, 130, 64, 264), (2, 64, 128, 64)])
def test_bmm_shapes(kda, B, M, K, N):
    d = inputs.nkibench("bmm", 1, B=B, M=M, K=K, N=N)
    out = kda.bmm(**gpu_args("bmm", d))
    got = host(out)
    if B * M * N > 1e8:      # spot-check a few batches at full size
        for b in (0, B - 1):
            assert rel_l2(got[b], ref.matmul(d["lhs"][b], d["rhs"][b])) <= GATE_BF16
    else:
        assert rel_l2(got, ref.bmm(**d)) <= GATE_BF16


def test_rmsnorm_matmul_config_scaled(kda):
    d = inputs.config("rmsnorm_matmul", 42, scale=16)     # M=256 of 4096
    g = gpu_args("rmsnorm_matmul", d)
    out = kda.rmsnorm_matmul(g["x"].to(torch.bfloat16), g["w"].to(torch.bfloat16), g["g"], d["eps"])
    assert rel_l2(host(out), ref.rmsnorm_matmul(**d)) <= GATE_BF16


@pytest.mark.parametrize("M,K,N", [(257, 256, 2048), (130, 512, 8192), (200, 136, 4104)])
def test_matmul_add_rmsnorm_row_widths(kda, M, K, N):
    """The in-place row normalisation: two rows per CTA for N = 2048 * {1, 4}
    (odd M: a last CTA with one row), one row per CTA otherwise."""
    d = inputs.nkibench("matmul_add_rmsnorm", 8, M=M, K=K, N=N)
    out = kda.matmul_add_rmsnorm(**gpu_args("matmul_add_rmsnorm", d))
    assert rel_l2(host(out), ref.matmul_add_rmsnorm(**d)) <= GATE_BF16


@pytest.mark.parametrize("M,K,N", [(1024, 1024, 2056), (4096, 4096, 4096)])
def test_matmul_add_rmsnorm_tail_split(kda, M, K, N):
    """Shapes whose last wave of pair tiles is split along K: the part that
    arrives last adds z and the row's sum of squares (ragged N: the scalar z
    loads; the full configuration: 34 of 256 tiles in two parts)."""
    d = inputs.nkibench("matmul_add_rmsnorm", 9, M=M, K=K, N=N)
    out = kda.matmul_add_rmsnorm(**gpu_args("matmul_add_rmsnorm", d))
    assert rel_l2(host(out), ref.matmul_add_rmsnorm(**d)) <= GATE_BF16


def test_matmul_add_rmsnorm_config_scaled(kda):
    d = inputs.config("matmul_add_rmsnorm", 42, scale=16)
    g = {k: (dev(v) if isinstance(v, np.ndarray) else v) for k, v in d.items()}
    out = kda.matmul_add_rmsnorm(g["x"].to(torch.bfloat16), g["w"].to(torch.bfloat16), d["eps"],
                                 g["z"].to(torch.bfloat16), g["g"])
    assert rel_l2(host(out), ref.matmul_add_rmsnorm(**d)) <= GATE_BF16


def test_swiglu_config_scaled(kda):
    d = inputs.config("swiglu", 42, scale=32)              # M=256 of 8192
    g = {k: dev(v, torch.bfloat16) for k, v in d.items()}
    out = kda.swiglu(g["x"], g["w_up"], g["w_down"], g["w_gate"])
    assert rel_l2(host(out), ref.swiglu(**d)) <= GATE_BF16


def test_lora_nkibench_rank(kda):
    d = inputs.nkibench("lora", 5, M=256, K=1024, N=768, R=128)
    out = kda.lora(**gpu_args("lora", d))
    assert rel_l2(host(out), ref.lora(**d)) <= GATE_BF16


@pytest.mark.parametrize("M,K,N,R", [(1024, 5120, 512, 128), (300, 1096, 392, 64), (520, 200, 264, 16)])
def test_lora_split_k(kda, M, K, N, R):
    """t = x @ a with K split over 8 / 2 parts (fp32 partials summed to bf16),
    including a partial last k-block and R < 128, and an unsplit small K."""
    d = inputs.nkibench("lora", 6, M=M, K=K, N=N, R=R)
    out = kda.lora(**gpu_args("lora", d))
    assert rel_l2(host(out), ref.lora(**d)) <= GATE_BF16


@pytest.mark.parametrize("op", ["rmsnorm_matmul", "add_rmsnorm_matmul"])
@pytest.mark.parametrize("K", [256, 512, 1024, 2048, 4096, 8192, 1280])
def test_rms_prepass_widths(kda, op, K):
    """Every row-statistics pre-pass variant (warp per register-resident row,
    CTA per row, general two-read kernel) against the oracle."""
    d = inputs.nkibench(op, 11, M=72, K=K, N=136)
    out = getattr(kda, op)(**gpu_args(op, d))
    assert rel_l2(host(out), getattr(ref, op)(**d)) <= GATE_BF16


@pytest.mark.parametrize("op", ["rmsnorm_matmul", "add_rmsnorm_matmul"])
@pytest.mark.parametrize("M,K,N", [(300, 1288, 392), (256, 4096, 520), (520, 256, 136), (1024, 2048, 1024),
                                   (3000, 1024, 264), (2600, 256, 136)])
def test_rms_pair_gemm(kda, op, M, K, N):
    """Row-statistics pre-pass + CTA-pair GEMM: ragged M / N, K not a multiple
    of the 64-wide k-block, several tiles per CTA pair; M > 2368 takes the
    two-rows-per-warp pre-pass (with a ragged last CTA)."""
    d = inputs.nkibench(op, 13, M=M, K=K, N=N)
    out = getattr(kda, op)(**gpu_args(op, d))
    assert rel_l2(host(out), getattr(ref, op)(**d)) <= GATE_BF16


@pytest.mark.parametrize("op", ["rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm"])
@pytest.mark.parametrize("M,K,N", [(1024, 2048, 5120), (1100, 1288, 4104)])
def test_rms_gemm_repeat_call(kda, op, M, K, N):
    """A partial last wave of pair tiles (80 / 85 tiles on 74 SM pairs), ragged
    M and N, K of 21 k-blocks: two calls on one workspace agree with the
    oracle and with each other -- bit for bit where the op is deterministic
    (matmul_add_rmsnorm sums each row's squares with float atomics over its
    column tiles, so its last bits may differ between calls)."""
    d = inputs.nkibench(op, 21, M=M, K=K, N=N)
    g = gpu_args(op, d)
    ws = torch.empty(kda.ops._ws_size(f"kda_{op}_workspace_size", M, K, N), dtype=torch.uint8, device="cuda")
    a = getattr(kda, op)(**g, workspace=ws).clone()
    b = getattr(kda, op)(**g, workspace=ws)
    want = getattr(ref, op)(**d)
    assert rel_l2(host(a), want) <= GATE_BF16
    assert rel_l2(host(b), want) <= GATE_BF16
    if op == "matmul_add_rmsnorm":
        assert rel_l2(host(a), host(b)) <= 1e-3
    else:
        assert torch.equal(a, b)


def test_rms_pair_gemm_with_gamma(kda):
    d = inputs.config("rmsnorm_matmul", 7, scale=8)  # M=512 of 4096, gamma and eps
    g = gpu_args("rmsnorm_matmul", d)
    out = kda.rmsnorm_matmul(g["x"].to(torch.bfloat16), g["w"].to(torch.bfloat16), g["g"], d["eps"])
    assert rel_l2(host(out), ref.rmsnorm_matmul(**d)) <= GATE_BF16


@pytest.mark.parametrize("M", [512, 1024, 4096])
def test_rms_gemm_tail_split(kda, M):
    """The configuration's row blocks at 8 / 4 / 1 GPUs (86 / 172 / 688 pair
    tiles on 74 CTA pairs): the last partial wave is split along K into 6 / 3 /
    3 parts whose fp32 partials the last-arriving part sums.  The workspace
    starts as garbage (the pre-pass zeroes the part counters) and two calls
    agree bit for bit."""
    d = inputs.config("rmsnorm_matmul", 5, scale=4096 // M)
    g = gpu_args("rmsnorm_matmul", d)
    x, w = g["x"].to(torch.bfloat16), g["w"].to(torch.bfloat16)
    ws = torch.full((kda.ops._ws_size("kda_rmsnorm_matmul_workspace_size", M, 4096, 11008),), 255,
                    dtype=torch.uint8, device="cuda")
    a = kda.rmsnorm_matmul(x, w, g["g"], d["eps"], workspace=ws).clone()
    b = kda.rmsnorm_matmul(x, w, g["g"], d["eps"], workspace=ws)
    assert torch.equal(a, b)
    assert rel_l2(host(a), ref.rmsnorm_matmul(**d)) <= GATE_BF16


def test_too_small_workspace_is_rejected(kda):
    d = inputs.nkibench("rmsnorm_matmul", 9, M=200, K=256, N=136)
    g = gpu_args("rmsnorm_matmul", d)
    with pytest.raises(ValueError, match="workspace"):
        kda.rmsnorm_matmul(g["x"], g["w"], workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))


def test_workspace_reuse_is_stateless(kda):
    """Two calls sharing one workspace give identical results (no hidden state)."""
    d = inputs.nkibench("rmsnorm_matmul", 9, M=200, K=256, N=136)
    g = gpu_args("rmsnorm_matmul", d)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    a = kda.rmsnorm_matmul(g["x"], g["w"], workspace=ws).clone()
    b = kda.rmsnorm_matmul(g["x"], g["w"], workspace=ws)
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,M,K,N", [
    (2, 136, 64, 144), (16, 4096, 64, 4096), (1, 8, 16, 40), (3, 200, 128, 520),
    # row blocks of 4, 9 (odd: the pair's second CTA gets one tile fewer, K of
    # two k-blocks), 12 and 33 column tiles split over a CTA pair
    (2, 136, 64, 1000), (1, 264, 128, 2056), (2, 128, 64, 3072), (1, 136, 64, 8200),
])
def test_bmm_softmax(kda, B, M, K, N):
    d = inputs.nkibench("bmm_softmax", 2, B=B, M=M, K=K, N=N)
    got = host(kda.bmm_softmax(**gpu_args("bmm_softmax", d)))
    if B * M * N > 1e8:      # spot-check batches at full size; rows still sum to one
        for b in (0, B - 1):
            want = ref.bmm_softmax(d["lhs"][b:b + 1], d["rhs"][b:b + 1])[0]
            assert rel_l2(got[b], want) <= GATE_BF16
    else:
        assert rel_l2(got, ref.bmm_softmax(**d)) <= GATE_BF16
    np.testing.assert_allclose(got.sum(-1), 1.0, atol=2e-2)


# --------------------------------------------------------------- attention
@pytest.mark.parametrize("seed", [42, 0])
def test_gqa_vs_reference_golden(kda, seed, golden_meta):
    d, want = golden_case("gqa_full", seed, golden_meta)
    got = host(kda.gqa_full(**gpu_args("gqa_full", d)))          # reference order (B, QH, S, D)
    assert got.shape == want.shape
    assert rel_l2(got, want) <= GATE_BF16
    assert rel_l2(got, ref.gqa_full(**d)) <= GATE_BF16


@pytest.mark.parametrize("B,S,QH,KH,causal,theta", [
    (2, 384, 8, 2, True, 10000.0), (1, 200, 4, 4, True, None), (1, 200, 4, 1, False, 10000.0),
    (2, 256, 4, 2, False, None), (1, 1, 2, 1, True, 10000.0), (1, 1000, 2, 1, True, 500.0)])
def test_gqa_shapes(kda, B, S, QH, KH, causal, theta):
    d = inputs.nkibench("gqa_full", 11, B=B, S=S, QH=QH, KH=KH, D=128)
    a = gpu_args("gqa_full", d)
    got = host(kda.gqa_full(a["q"], a["k"], a["v"], causal=causal, rope_theta=theta, out_layout="bshd"))
    want = ref.gqa_full(**d, causal=causal, rope_theta=theta, out_layout="bshd")
    assert rel_l2(got, want) <= GATE_BF16


def test_gqa_config_full_size_sampled_heads(kda):
    """North-star configuration (B8 S4096 QH32 KH8, causal, RoPE 1e4): every
    output checked for finiteness, four (batch, head) slices against the oracle."""
    d = inputs.config("gqa_full", 42)
    a = {k: dev(v, torch.bfloat16) for k, v in d.items()}
    out = kda.gqa_full(a["q"], a["k"], a["v"], causal=True, rope_theta=10000.0, out_layout="bshd")
    assert bool(torch.isfinite(out).all())
    heads = [(0, 0), (3, 17), (7, 31), (5, 8)]
    want = ref.gqa_full(**d, causal=True, rope_theta=10000.0, out_layout="bshd", heads=heads)
    got = host(out)
    for b, h in heads:
        assert rel_l2(got[b, :, h], want[b, :, h]) <= GATE_BF16


def test_gqa_config_full_size_every_head(kda):
    """North-star configuration, every (batch, head) slice against a float32 torch
    restatement of the oracle's forward (same RoPE tables, kv head h // n_rep,
    scores / sqrt(D), causal mask, max-shifted softmax, @ v), one batch entry at a
    time on the GPU; the sampled-heads test above pins this restatement to the oracle."""
    d = inputs.config("gqa_full", 42)
    a = {k: dev(v, torch.bfloat16) for k, v in d.items()}
    out = kda.gqa_full(a["q"], a["k"], a["v"], causal=True, rope_theta=10000.0, out_layout="bshd")
    torch.cuda.synchronize()
    B, S, QH, D = a["q"].shape
    rep = QH // a["k"].shape[2]
    cos, sin = (torch.from_numpy(t).cuda()[None, :, None, :] for t in ref.rope_tables(S, D, 10000.0))

    def rope(x):
        x0, x1 = x[..., : D // 2], x[..., D // 2:]
        return torch.cat([x0 * cos - x1 * sin, x0 * sin + x1 * cos], dim=-1)

    mask = torch.ones(S, S, dtype=torch.bool, device="cuda").triu(1)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        worst = 0.0
        for b in range(B):
            q = rope(a["q"][b:b + 1].float())[0].transpose(0, 1)                       # (QH, S, D)
            k = rope(a["k"][b:b + 1].float())[0].transpose(0, 1).repeat_interleave(rep, 0)
            v = a["v"][b].float().transpose(0, 1).repeat_interleave(rep, 0)
            s = (q @ k.transpose(1, 2)) * (1.0 / D ** 0.5)
            s.masked_fill_(mask, float("-inf"))
            want = torch.softmax(s, dim=-1) @ v                                        # (QH, S, D)
            del s
            got = out[b].float().transpose(0, 1)
            err = ((got - want).norm(dim=(1, 2)) / want.norm(dim=(1, 2))).max().item()
            worst = max(worst, err)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert worst <= GATE_BF16, worst
    assert kda.device_error() == 0


# ------------------------------------------- fp32-accuracy contraction paths
F32_GOLDEN_OPS = ["rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "swiglu", "lora", "gqa_full"]


def f32_args(d):
    return {k: (dev(v) if isinstance(v, np.ndarray) else v) for k, v in d.items()}


@pytest.mark.parametrize("op", F32_GOLDEN_OPS)
@pytest.mark.parametrize("seed", [42, 0])
def test_fused_f32_vs_reference_golden(kda, op, seed, golden_meta):
    """fp32 operands (unrounded draws) against the reference's own fp32 outputs
    and the oracle, at the reference's fp32 gate."""
    shape = dict(golden_meta[f"{op}_s{seed}"]["shape"])
    if op == "gqa_full":
        shape["S"] = shape.pop("N")
    d = inputs.nkibench(op, seed, bf16=False, **shape)
    want = np.load(GOLDEN / f"{op}_s{seed}.npy")
    out = getattr(kda, op)(**f32_args(d))
    assert out.dtype == torch.float32
    got = host(out)
    assert got.shape == want.shape
    assert rel_l2(got, want) <= FP32_GATE_REF
    assert rel_l2(got, getattr(ref, op)(**d)) <= FP32_GATE_REF


@pytest.mark.parametrize("op,shape", [
    ("rmsnorm_matmul", dict(M=4096, K=1024, N=2048)), ("rmsnorm_matmul", dict(M=130, K=264, N=200)),
    ("add_rmsnorm_matmul", dict(M=4096, K=1024, N=2048)), ("add_rmsnorm_matmul", dict(M=8, K=8, N=8)),
    ("matmul_add_rmsnorm", dict(M=4096, K=2048, N=2048)), ("matmul_add_rmsnorm", dict(M=300, K=72, N=520)),
    ("swiglu", dict(M=4096, K=1024, N=3072)), ("swiglu", dict(M=129, K=64, N=264)),
])
def test_fused_f32_shapes(kda, op, shape):
    d = inputs.nkibench(op, 5, bf16=False, **shape)
    got = host(getattr(kda, op)(**f32_args(d)))
    assert rel_l2(got, getattr(ref, op)(**d)) <= FP32_GATE_REF


def test_rmsnorm_matmul_f32_gamma_eps(kda):
    d = inputs.nkibench("rmsnorm_matmul", 6, bf16=False, M=520, K=512, N=264)
    g = (1 + 0.1 * np.random.default_rng(6).normal(size=512)).astype(np.float32)
    got = host(kda.rmsnorm_matmul(dev(d["x"]), dev(d["w"]), dev(g), 1e-6))
    assert rel_l2(got, ref.rmsnorm_matmul(d["x"], d["w"], g, 1e-6)) <= FP32_GATE_REF


@pytest.mark.parametrize("M,K,N,R", [(4096, 5120, 12288, 128), (136, 200, 144, 16), (264, 512, 520, 256)])
def test_lora_f32_shapes(kda, M, K, N, R):
    d = inputs.nkibench("lora", 4, bf16=False, M=M, K=K, N=N, R=R)
    got = host(kda.lora(**f32_args(d)))
    if M * N > 1e7:            # full NKIBench shape: a row sample of the oracle
        rows = slice(0, M, 97)
        assert rel_l2(got[rows], ref.lora(d["x"][rows], d["w"], d["a"], d["b"])) <= FP32_GATE_REF
    else:
        assert rel_l2(got, ref.lora(**d)) <= FP32_GATE_REF


@pytest.mark.parametrize("B,M,K,N", [(2, 136, 64, 144), (16, 4096, 64, 4096), (3, 200, 128, 520),
                                     (1, 9, 16, 16384)])   # long rows, few of them
def test_bmm_softmax_f32(kda, B, M, K, N):
    """Three-way operand split (six products): the error left is the oracle's
    own fp32 rounding, well inside the reference's gate."""
    tol = 5e-6
    d = inputs.nkibench("bmm_softmax", 2, bf16=False, B=B, M=M, K=K, N=N)
    out = kda.bmm_softmax(dev(d["lhs"]), dev(d["rhs"]))
    assert out.dtype == torch.float32
    got = host(out)
    if B * M * N > 1e8:      # full NKIBench shape: two batches
        for b in (0, B - 1):
            want = ref.bmm_softmax(d["lhs"][b:b + 1], d["rhs"][b:b + 1])[0]
            assert rel_l2(got[b], want) <= tol
    else:
        assert rel_l2(got, ref.bmm_softmax(**d)) <= tol
    np.testing.assert_allclose(got.sum(-1), 1.0, atol=1e-5)


@pytest.mark.parametrize("B,S,QH,KH,D,causal,layout", [
    (1, 4096, 16, 8, 128, False, "bhsd"),     # NKIBench shape: sampled heads
    (2, 384, 8, 2, 128, True, "bshd"), (1, 200, 4, 4, 64, False, "bshd"), (1, 8, 2, 1, 32, True, "bhsd")])
def test_gqa_f32(kda, B, S, QH, KH, D, causal, layout):
    d = inputs.nkibench("gqa_full", 12, bf16=False, B=B, S=S, QH=QH, KH=KH, D=D)
    out = kda.gqa_full(dev(d["q"]), dev(d["k"]), dev(d["v"]), causal=causal, out_layout=layout)
    assert out.dtype == torch.float32
    got = host(out)
    if S >= 4096:
        heads = [(0, 0), (0, 7), (0, 15)]
        want = ref.gqa_full(**d, causal=causal, out_layout=layout, heads=heads)
        for b, h in heads:
            assert rel_l2(got[b, h], want[b, h]) <= FP32_GATE_REF
    else:
        assert rel_l2(got, ref.gqa_full(**d, causal=causal, out_layout=layout)) <= FP32_GATE_REF


def test_gqa_f32_rejects_rope(kda):
    d = inputs.nkibench("gqa_full", 12, bf16=False, B=1, S=16, QH=2, KH=1, D=128)
    with pytest.raises(ValueError, match="rope"):
        kda.gqa_full(dev(d["q"]), dev(d["k"]), dev(d["v"]), rope_theta=10000.0)


# ------------------------------------------------ rmsnorm_matmul backward
@pytest.mark.parametrize("M,K,N,with_g", [(136, 256, 264, True), (4096, 1024, 2048, False), (520, 4096, 1024, True),
                                          (8, 8, 8, True), (300, 72, 520, False), (256, 2048, 512, False),
                                          (136, 8192, 256, True)])
def test_rmsnorm_matmul_backward(kda, M, K, N, with_g):
    rng = np.random.default_rng(M + K)
    from oracle.bf16 import to_bf16_rne
    x = to_bf16_rne(rng.normal(size=(M, K)).astype(np.float32))
    w = to_bf16_rne((0.02 * rng.normal(size=(K, N))).astype(np.float32))
    dy = to_bf16_rne(rng.normal(size=(M, N)).astype(np.float32))
    g = (1 + 0.1 * rng.normal(size=K)).astype(np.float32) if with_g else None
    dx, dw, dg = kda.rmsnorm_matmul_backward(dev(dy, torch.bfloat16), dev(x, torch.bfloat16), dev(w, torch.bfloat16),
                                             None if g is None else dev(g), 1e-6)
    wdx, wdw, wdg = ref.rmsnorm_matmul_backward(dy, x, w, g, 1e-6)
    assert rel_l2(host(dx), wdx) <= GATE_BF16
    assert rel_l2(host(dw), wdw) <= GATE_BF16
    if with_g:
        assert rel_l2(host(dg), wdg) <= GATE_BF16
    else:
        assert dg is None


def test_rmsnorm_matmul_autograd(kda):
    import kda.autograd as ka
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(136, 256, device="cuda", generator=gen).to(torch.bfloat16).requires_grad_()
    w = (0.02 * torch.randn(256, 264, device="cuda", generator=gen)).to(torch.bfloat16).requires_grad_()
    g = (1 + 0.1 * torch.randn(256, device="cuda", generator=gen)).requires_grad_()
    y = ka.rmsnorm_matmul(x, w, g, 1e-6)
    assert torch.equal(y, kda.rmsnorm_matmul(x.detach(), w.detach(), g.detach(), 1e-6))
    dy = torch.randn(y.shape, device="cuda", generator=gen).to(torch.bfloat16)
    y.backward(dy)
    dx, dw, dg = kda.rmsnorm_matmul_backward(dy, x.detach(), w.detach(), g.detach(), 1e-6)
    assert torch.equal(x.grad, dx) and torch.equal(w.grad, dw) and torch.equal(g.grad, dg)


# ---------------------------------------------------------- swiglu backward
@pytest.mark.parametrize("M,K,N", [(136, 200, 144), (4096, 1024, 3072), (8, 8, 8), (520, 512, 264)])
def test_swiglu_backward(kda, M, K, N):
    from oracle.bf16 import to_bf16_rne
    rng = np.random.default_rng(M + N)
    x = to_bf16_rne(rng.normal(size=(M, K)).astype(np.float32))
    wu, wg = (to_bf16_rne((0.05 * rng.normal(size=(K, N))).astype(np.float32)) for _ in range(2))
    wd = to_bf16_rne((0.05 * rng.normal(size=(N, K))).astype(np.float32))
    dout = to_bf16_rne(rng.normal(size=(M, K)).astype(np.float32))
    b = torch.bfloat16
    got = kda.swiglu_backward(dev(dout, b), dev(x, b), dev(wu, b), dev(wd, b), dev(wg, b))
    want = ref.swiglu_backward(dout, x, wu, wd, wg)
    for name, gt, wt in zip(("dx", "dw_up", "dw_down", "dw_gate"), got, want):
        assert gt.shape == wt.shape, name
        assert rel_l2(host(gt), wt) <= GATE_BF16, name


@pytest.mark.parametrize("M,K,N", [(128, 128, 192), (520, 200, 264), (136, 256, 1024)])
def test_swiglu_backward_from_saved_forward(kda, M, K, N):
    """swiglu_gu keeps g = x w_gate and u = x w_up; the backward on them gives
    the standalone backward's gradients bit for bit (it recomputes the same g, u)."""
    rng = np.random.default_rng(M + N)
    b = torch.bfloat16
    x = dev(rng.normal(size=(M, K)).astype(np.float32), b)
    wu, wg = (dev(0.05 * rng.normal(size=(K, N)).astype(np.float32), b) for _ in range(2))
    wd = dev(0.05 * rng.normal(size=(N, K)).astype(np.float32), b)
    dout = dev(rng.normal(size=(M, K)).astype(np.float32), b)
    out, g, u = kda.swiglu_gu(x, wu, wd, wg)
    assert torch.equal(g, kda.matmul(x, wg)) and torch.equal(u, kda.matmul(x, wu))
    want_out = ref.swiglu(host(x), host(wu), host(wd), host(wg))
    assert rel_l2(host(out), want_out) <= GATE_BF16
    assert rel_l2(host(out), host(kda.swiglu(x, wu, wd, wg))) <= 1e-2
    saved = kda.swiglu_backward(dout, x, wu, wd, wg, g=g, u=u)
    full = kda.swiglu_backward(dout, x, wu, wd, wg)
    for name, gs, gf in zip(("dx", "dw_up", "dw_down", "dw_gate"), saved, full):
        assert torch.equal(gs, gf), name
    with pytest.raises(ValueError):
        kda.swiglu_backward(dout, x, wu, wd, wg, g=g)
    assert kda.device_error() == 0


def test_swiglu_autograd(kda):
    import kda.autograd as ka
    gen = torch.Generator(device="cuda").manual_seed(1)
    b = torch.bfloat16
    x = torch.randn(136, 200, device="cuda", generator=gen).to(b).requires_grad_()
    ws = [(0.05 * torch.randn(*s, device="cuda", generator=gen)).to(b).requires_grad_()
          for s in ((200, 144), (144, 200), (200, 144))]
    y = ka.swiglu(x, *ws)
    dout = torch.randn(y.shape, device="cuda", generator=gen).to(b)
    y.backward(dout)
    want = kda.swiglu_backward(dout, x.detach(), *(w.detach() for w in ws))
    for t, w in zip([x] + ws, want):
        assert torch.equal(t.grad, w)


# ------------------------------------------------------- gqa_full backward
@pytest.mark.parametrize("B,S,QH,KH,causal,theta", [
    (1, 256, 4, 2, False, None), (1, 256, 4, 2, True, None), (2, 136, 4, 4, True, None), (1, 8, 2, 1, False, None),
    (1, 1024, 8, 2, True, None), (2, 384, 8, 2, True, 10000.0), (1, 200, 4, 1, False, 500.0)])
def test_gqa_backward(kda, B, S, QH, KH, causal, theta):
    from oracle.bf16 import to_bf16_rne
    rng = np.random.default_rng(S + QH)
    q = to_bf16_rne(rng.normal(size=(B, S, QH, 128)).astype(np.float32))
    k = to_bf16_rne(rng.normal(size=(B, S, KH, 128)).astype(np.float32))
    v = to_bf16_rne(rng.normal(size=(B, S, KH, 128)).astype(np.float32))
    dout = to_bf16_rne(rng.normal(size=(B, QH, S, 128)).astype(np.float32))
    b = torch.bfloat16
    got = kda.gqa_full_backward(dev(dout, b), dev(q, b), dev(k, b), dev(v, b), causal=causal, rope_theta=theta)
    want = ref.gqa_full_backward(dout, q, k, v, causal=causal, rope_theta=theta)
    for name, gt, wt in zip(("dq", "dk", "dv"), got, want):
        assert gt.shape == wt.shape, name
        assert rel_l2(host(gt), wt) <= GATE_BF16, name


@pytest.mark.parametrize("B,S,QH,KH,causal,theta", [
    (1, 256, 4, 2, False, None), (2, 136, 4, 4, True, None), (1, 1024, 8, 2, True, None),
    (2, 384, 8, 2, True, 10000.0), (1, 200, 4, 1, False, 500.0)])
def test_gqa_backward_from_saved_forward(kda, B, S, QH, KH, causal, theta):
    """The forward's output and lse from gqa_full_lse replace the backward's own
    forward: same output as gqa_full, lse = log2-sum-exp of the scaled scores,
    and the same gradients as the standalone backward."""
    from oracle.bf16 import to_bf16_rne
    rng = np.random.default_rng(3 * S + QH)
    q = to_bf16_rne(rng.normal(size=(B, S, QH, 128)).astype(np.float32))
    k = to_bf16_rne(rng.normal(size=(B, S, KH, 128)).astype(np.float32))
    v = to_bf16_rne(rng.normal(size=(B, S, KH, 128)).astype(np.float32))
    dout = to_bf16_rne(rng.normal(size=(B, QH, S, 128)).astype(np.float32))
    b = torch.bfloat16
    qd, kd, vd, dod = dev(q, b), dev(k, b), dev(v, b), dev(dout, b)
    out, lse = kda.gqa_full_lse(qd, kd, vd, causal=causal, rope_theta=theta)
    assert torch.equal(out, kda.gqa_full(qd, kd, vd, causal=causal, rope_theta=theta))
    if theta is None:
        # lse against float64 scores of the same bf16 inputs (no RoPE)
        rep = QH // KH
        qh = q.astype(np.float64).transpose(0, 2, 1, 3)                       # B, QH, S, D
        kh = np.repeat(k.astype(np.float64).transpose(0, 2, 1, 3), rep, 1)    # B, QH, S, D
        sc = np.einsum("bhqd,bhkd->bhqk", qh, kh) / np.sqrt(128.0)
        if causal:
            sc = np.where(np.tril(np.ones((S, S), dtype=bool)), sc, -np.inf)
        m = sc.max(-1, keepdims=True)
        want = (m[..., 0] + np.log(np.exp(sc - m).sum(-1))) / np.log(2.0)
        np.testing.assert_allclose(host(lse), want, rtol=0, atol=2e-3)
    saved = kda.gqa_full_backward(dod, qd, kd, vd, causal=causal, rope_theta=theta, fwd_out=out, lse=lse)
    full = kda.gqa_full_backward(dod, qd, kd, vd, causal=causal, rope_theta=theta)
    want = ref.gqa_full_backward(dout, q, k, v, causal=causal, rope_theta=theta)
    for name, gs, gf, wt in zip(("dq", "dk", "dv"), saved, full, want):
        # dk and dv are summed in a fixed order; dq adds the key blocks'
        # contributions in the order they arrive
        assert rel_l2(host(gs), host(gf)) <= 1e-3, name
        assert rel_l2(host(gs), wt) <= GATE_BF16, name
    assert kda.device_error() == 0


def test_gqa_backward_saved_rejects_half_the_saved_state(kda):
    t = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(1, 16, 1, 128, dtype=torch.bfloat16, device="cuda")
    dout = torch.zeros(1, 2, 16, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kda.gqa_full_backward(dout, t, kv, kv, fwd_out=dout)


def test_gqa_autograd(kda):
    import kda.autograd as ka
    gen = torch.Generator(device="cuda").manual_seed(2)
    b = torch.bfloat16
    q = torch.randn(1, 136, 4, 128, device="cuda", generator=gen).to(b).requires_grad_()
    k = torch.randn(1, 136, 2, 128, device="cuda", generator=gen).to(b).requires_grad_()
    v = torch.randn(1, 136, 2, 128, device="cuda", generator=gen).to(b).requires_grad_()
    o = ka.gqa_full(q, k, v, causal=True, rope_theta=10000.0)
    assert torch.equal(o, kda.gqa_full(q.detach(), k.detach(), v.detach(), causal=True, rope_theta=10000.0))
    dout = torch.randn(o.shape, device="cuda", generator=gen).to(b)
    o.backward(dout)
    want = kda.gqa_full_backward(dout, q.detach(), k.detach(), v.detach(), causal=True, rope_theta=10000.0)
    for t, w in zip((q, k, v), want):
        assert torch.equal(t.grad, w)
