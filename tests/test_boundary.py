"""The Python boundary: ``torch.ops.kda.<op>`` custom ops and the numpy
``kda.compat.<op>`` shim keep the reference forwards' parameter names and
order (``adapter/nkibench_case.py:147-155`` calls ``forward(**get_numpy_inputs())``),
propagate shapes without a GPU, and pass the host checks' ``ValueError``
through.  The GPU half compares both against the CPU oracle."""

import inspect

import numpy as np
import pytest

from oracle import inputs, ops as ref
from oracle.metrics import GATE_BF16, GATE_FP32, rel_l2

torch = pytest.importorskip("torch")

OPS = ["silu", "rmsnorm_matmul", "add_rmsnorm_matmul", "matmul_add_rmsnorm", "swiglu", "matmul",
       "transpose_matmul", "bmm", "bmm_softmax", "gqa_full", "rope_single_freq_apply", "lora", "adamw", "mamba"]
FP32_OPS = {"silu", "rope_single_freq_apply", "adamw", "mamba"}

# small cases of every operator (NKIBench parameter names)
SMALL = {
    "silu": dict(M=64, N=1000), "matmul": dict(M=264, K=256, N=272),
    "rmsnorm_matmul": dict(M=136, K=256, N=264), "add_rmsnorm_matmul": dict(M=136, K=1024, N=264),
    "matmul_add_rmsnorm": dict(M=136, K=256, N=264), "swiglu": dict(M=128, K=128, N=192),
    "transpose_matmul": dict(M=264, K=256, N=272), "bmm": dict(B=3, M=136, K=64, N=264),
    "bmm_softmax": dict(B=2, M=128, K=64, N=512), "lora": dict(M=264, K=256, N=272, R=64),
    "gqa_full": dict(B=1, S=256, QH=4, KH=2, D=128), "rope_single_freq_apply": dict(D=16, S=256),
    "adamw": dict(M=17, N=64), "mamba": dict(C=64, M=300),
}


@pytest.fixture(scope="module")
def kda():
    import kda as k
    return k


def forward_names(op):
    """The reference forward's parameters, in order (the oracle's draw dict)."""
    return list(inputs.nkibench(op, 0, **SMALL[op]).keys())


@pytest.mark.parametrize("op", OPS)
def test_custom_op_registered_with_forward_names(kda, op):
    schema = getattr(torch.ops.kda, op).default._schema
    names = [a.name for a in schema.arguments]
    assert names[:len(forward_names(op))] == forward_names(op)


@pytest.mark.parametrize("op", OPS)
def test_compat_signature_is_the_forward(kda, op):
    params = [p.name for p in inspect.signature(getattr(kda.compat, op)).parameters.values()
              if p.kind == p.POSITIONAL_OR_KEYWORD]
    assert params[:len(forward_names(op))] == forward_names(op)


def _meta(d, bf16_args=()):
    return {k: (torch.empty(v.shape, device="meta",
                            dtype=torch.bfloat16 if k in bf16_args else torch.float32)
                if isinstance(v, np.ndarray) else v) for k, v in d.items()}


@pytest.mark.parametrize("op", OPS)
def test_fake_kernels_propagate_shapes(kda, op):
    """Meta tensors in, the oracle's output shape and the op's dtype out, nothing run."""
    d = inputs.nkibench(op, 0, **SMALL[op])
    want = getattr(ref, op)(**d)
    out = getattr(torch.ops.kda, op)(**_meta(d, inputs.BF16_ARGS.get(op, ())))
    assert out.device.type == "meta"
    assert tuple(out.shape) == want.shape
    assert out.dtype == (torch.float32 if op in FP32_OPS else torch.bfloat16)


def test_fake_kernels_fp32_contraction_and_layouts(kda):
    q = torch.empty(2, 64, 8, 128, device="meta")
    k = torch.empty(2, 64, 2, 128, device="meta")
    assert torch.ops.kda.gqa_full(q, k, k).dtype == torch.float32
    assert tuple(torch.ops.kda.gqa_full(q, k, k, out_layout="bshd").shape) == (2, 64, 8, 128)
    assert tuple(torch.ops.kda.gqa_full(q, k, k).shape) == (2, 8, 64, 128)
    dt = torch.empty(2, 10, 32, device="meta")
    u = torch.empty(2, 10, 32, device="meta", dtype=torch.bfloat16)
    a = torch.empty(32, 16, device="meta")
    bc = torch.empty(2, 10, 16, device="meta")
    assert torch.ops.kda.mamba(dt, u, a, bc, bc).dtype == torch.bfloat16
    assert torch.ops.kda.mamba(dt, u, a, bc, bc, None, torch.float32).dtype == torch.float32


def test_host_checks_raise_value_error_through_the_custom_op(kda):
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.kda.silu(torch.ones(4))
    with pytest.raises(ValueError, match="CUDA"):
        torch.ops.kda.matmul(torch.ones(4, 4, dtype=torch.bfloat16), torch.ones(4, 4, dtype=torch.bfloat16))


def test_compat_rejects_non_array_arguments(kda):
    with pytest.raises(TypeError, match="numpy array"):
        kda.compat.silu([1.0, 2.0])


# ---------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("op", OPS)
def test_compat_matches_oracle(kda, op):
    """forward(**get_numpy_inputs()) through the shim: numpy in, float32 numpy out."""
    d = inputs.nkibench(op, 42, **SMALL[op])
    got = getattr(kda.compat, op)(**d)
    assert isinstance(got, np.ndarray) and got.dtype == np.float32
    want = getattr(ref, op)(**d)
    assert got.shape == want.shape
    assert rel_l2(got, want) <= (GATE_FP32 if op in FP32_OPS else GATE_BF16)


@pytest.mark.gpu
@pytest.mark.parametrize("op", sorted(set(OPS) - FP32_OPS))
def test_compat_strict_fp32_meets_reference_gate(kda, op):
    """Unrounded fp32 draws on the fp32-accuracy path, at the reference's own fp32 gate."""
    d = inputs.nkibench(op, 42, bf16=False, **SMALL[op])
    got = getattr(kda.compat, op)(**d, strict_fp32=True)
    assert rel_l2(got, getattr(ref, op)(**d)) <= 2e-5


@pytest.mark.gpu
@pytest.mark.parametrize("op", OPS)
def test_custom_op_equals_python_op(kda, op):
    d = inputs.nkibench(op, 7, **SMALL[op])
    bf = inputs.BF16_ARGS.get(op, ())
    g = {k: (torch.from_numpy(np.ascontiguousarray(v)).cuda().to(torch.bfloat16 if k in bf else torch.float32)
             if isinstance(v, np.ndarray) else v) for k, v in d.items()}
    a = getattr(torch.ops.kda, op)(**g)
    b = getattr(kda, op)(**g)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert kda.device_error() == 0
