"""Pin the CPU oracle against the reference's own golden vectors (no GPU)."""

import hashlib

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import bf16, inputs, ops
from oracle.metrics import rel_l2

GOLDEN_OPS = ["matmul", "transpose_matmul", "bmm", "rmsnorm_matmul", "add_rmsnorm_matmul",
              "matmul_add_rmsnorm", "swiglu", "lora", "gqa_full"]


def golden_inputs(meta):
    shape = dict(meta["shape"])
    if meta["op"] == "gqa_full":
        shape["S"] = shape.pop("N")
    return inputs.nkibench(meta["op"], meta["seed"], bf16=False, **shape)


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


@pytest.mark.parametrize("op", GOLDEN_OPS)
@pytest.mark.parametrize("seed", [42, 0])
def test_oracle_matches_reference_golden(op, seed, golden_meta):
    meta = golden_meta[f"{op}_s{seed}"]
    d = golden_inputs(meta)
    # the draw order / distributions match the reference's draw_inputs bit for bit
    for name, digest in meta["input_sha256"].items():
        assert _sha(d[name]) == digest, f"{op}: input {name} differs from the reference draw"
    fn = getattr(ops, op)
    out = fn(**d)
    want = np.load(GOLDEN / f"{op}_s{seed}.npy")
    assert out.shape == want.shape
    assert rel_l2(out, want) < 2e-6


def test_bf16_rne_known_answers(golden_meta):
    kat = golden_meta["bf16_rne"]
    got = bf16.to_bf16_rne(np.array(kat["in"], dtype=np.float32))
    np.testing.assert_array_equal(got, np.array(kat["out"], dtype=np.float32))
    # the reference's asserts, restated (offline_bf16_split_sim.py:178-190)
    assert bf16.to_bf16_rne(np.float32(1.0)) == 1.0
    assert bf16.to_bf16_rne(np.float32(1.0 + 2.0 ** -8)) == 1.0
    assert bf16.to_bf16_rne(np.float32(1.0 + 3.0 * 2.0 ** -9)) == np.float32(1.0 + 2.0 ** -7)


def test_bf16_rne_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(1).normal(size=4096).astype(np.float32) * 100
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(bf16.to_bf16_rne(x), t)


def test_mamba_2d_equals_3d_layout():
    d = inputs.nkibench("mamba", 3, C=16, M=40, S=4)
    y2 = ops.mamba(**d)
    y3 = ops.mamba(d["delta"].T[None], d["u"].T[None], d["a"], d["b"].T[None], d["c"].T[None])
    np.testing.assert_allclose(y2, y3[0].T, rtol=1e-6, atol=1e-6)


def test_mamba_matches_sequential_definition():
    """Independent scalar restatement of the recurrence (spec draft-phase1.md:22-29)."""
    d = inputs.nkibench("mamba", 5, C=3, M=17, S=4)
    C, M = d["delta"].shape
    S = d["a"].shape[1]
    want = np.zeros((C, M))
    for ch in range(C):
        for s in range(S):
            st = 0.0
            for i in range(M):
                dl = float(d["delta"][ch, i])
                st = np.exp(dl * d["a"][ch, s]) * st + dl * d["b"][s, i] * d["u"][ch, i]
                want[ch, i] += d["c"][s, i] * st
    assert rel_l2(ops.mamba(**d), want) < 1e-6


def test_bmm_softmax_rows_sum_to_one():
    d = inputs.nkibench("bmm_softmax", 1, B=2, M=8, K=16, N=32)
    out = ops.bmm_softmax(**d)
    np.testing.assert_allclose(out.sum(-1), 1.0, rtol=1e-5)
    ref = ops.bmm(**d)
    e = np.exp(ref - ref.max(-1, keepdims=True))
    np.testing.assert_allclose(out, e / e.sum(-1, keepdims=True), rtol=1e-5, atol=1e-7)


def test_rope_rotation_preserves_pair_norm():
    d = inputs.nkibench("rope_single_freq_apply", 2, D=8, S=32)
    ang = np.random.default_rng(0).uniform(-3, 3, size=(4, 32)).astype(np.float32)
    d["cos"], d["sin"] = np.cos(ang), np.sin(ang)
    out = ops.rope_single_freq_apply(**d)
    n_in = d["x_in"][:4] ** 2 + d["x_in"][4:] ** 2
    n_out = out[:4] ** 2 + out[4:] ** 2
    np.testing.assert_allclose(n_in, n_out, rtol=1e-5)


def test_adamw_literal_formula():
    d = inputs.nkibench("adamw", 4, M=3, N=5)
    th, g, m, v = (d[k].astype(np.float64) for k in ("theta", "g", "m", "v"))
    mt = 0.9 * m + 0.1 * g
    vt = 0.999 * v + 0.001 * g * g
    want = th - 1e-5 * th - 0.01 * mt / (np.sqrt(vt * 1000) + 1e-8)
    assert rel_l2(ops.adamw(**d), want) < 1e-6


def test_gqa_causal_first_row_is_v0():
    d = inputs.nkibench("gqa_full", 7, B=1, S=16, QH=2, KH=1, D=8)
    out = ops.gqa_full(**d, causal=True, out_layout="bshd")
    np.testing.assert_allclose(out[0, 0, 0], d["v"][0, 0, 0], rtol=1e-6)


def test_silu_spec():
    x = np.array([-20.0, -1.0, 0.0, 1.0, 20.0], dtype=np.float32)
    np.testing.assert_allclose(ops.silu(x), x / (1 + np.exp(-x.astype(np.float64))), rtol=1e-6)


@pytest.mark.parametrize("with_g", [True, False])
def test_rmsnorm_matmul_backward_matches_autograd(with_g):
    """The backward restatement against torch autograd of the forward (float64, CPU)."""
    import torch
    rng = np.random.default_rng(5)
    x, w, dy = rng.normal(size=(6, 16)), rng.normal(size=(16, 8)), rng.normal(size=(6, 8))
    g = 1 + 0.1 * rng.normal(size=16) if with_g else None
    tx, tw = torch.tensor(x, requires_grad=True), torch.tensor(w, requires_grad=True)
    tg = torch.tensor(g, requires_grad=True) if with_g else None
    a = tx / torch.sqrt((tx * tx).mean(-1, keepdim=True) + 1e-6)
    if with_g:
        a = a * tg
    (a @ tw).backward(torch.tensor(dy))
    dx, dw, dg = ops.rmsnorm_matmul_backward(dy, x, w, g, 1e-6)
    np.testing.assert_allclose(dx, tx.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dw, tw.grad.numpy(), rtol=1e-10, atol=1e-12)
    if with_g:
        np.testing.assert_allclose(dg, tg.grad.numpy(), rtol=1e-10, atol=1e-12)
    else:
        assert dg is None


def test_adamw_step_defaults_are_adamw():
    d = inputs.nkibench("adamw", 4, M=3, N=5)
    th, m, v = ops.adamw_step(**d)
    assert rel_l2(th, ops.adamw(**d)) < 1e-6
    _, m2, v2 = ops.adamw_state(**d)
    assert rel_l2(m, m2) < 1e-7 and rel_l2(v, v2) < 1e-7


def test_swiglu_backward_matches_autograd():
    import torch
    rng = np.random.default_rng(6)
    x, wu, wd, wg = (rng.normal(size=s) for s in ((5, 8), (8, 12), (12, 8), (8, 12)))
    dout = rng.normal(size=(5, 8))
    t = [torch.tensor(a, requires_grad=True) for a in (x, wu, wd, wg)]
    g, u = t[0] @ t[3], t[0] @ t[1]
    ((torch.nn.functional.silu(g) * u) @ t[2]).backward(torch.tensor(dout))
    got = ops.swiglu_backward(dout, x, wu, wd, wg)
    for a, b in zip(got, [t[0].grad, t[1].grad, t[2].grad, t[3].grad]):
        np.testing.assert_allclose(a, b.numpy(), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("causal", [False, True])
def test_gqa_backward_rope_matches_autograd(causal):
    """With RoPE: autograd through the oracle's own rotation (float64)."""
    import torch
    rng = np.random.default_rng(8)
    q, k, v = rng.normal(size=(1, 6, 4, 8)), rng.normal(size=(1, 6, 2, 8)), rng.normal(size=(1, 6, 2, 8))
    dout = rng.normal(size=(1, 4, 6, 8))
    cos, sin = (torch.tensor(t.astype(np.float64))[None, :, None, :] for t in ops.rope_tables(6, 8, 500.0))

    def rot(x):
        x0, x1 = x[..., :4], x[..., 4:]
        return torch.cat([x0 * cos - x1 * sin, x0 * sin + x1 * cos], -1)

    t = [torch.tensor(a, requires_grad=True) for a in (q, k, v)]
    qh = rot(t[0]).permute(0, 2, 1, 3)
    kh = rot(t[1]).permute(0, 2, 1, 3).repeat_interleave(2, dim=1)
    vh = t[2].permute(0, 2, 1, 3).repeat_interleave(2, dim=1)
    s = qh @ kh.transpose(-1, -2) / np.sqrt(8)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(6, 6, dtype=torch.bool), 1), float("-inf"))
    (torch.softmax(s, -1) @ vh).backward(torch.tensor(dout))
    got = ops.gqa_full_backward(dout, q, k, v, causal=causal, rope_theta=500.0)
    for a, b in zip(got, t):
        np.testing.assert_allclose(a, b.grad.numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("causal", [False, True])
def test_gqa_backward_matches_autograd(causal):
    import torch
    rng = np.random.default_rng(7)
    q, k, v = rng.normal(size=(1, 6, 4, 8)), rng.normal(size=(1, 6, 2, 8)), rng.normal(size=(1, 6, 2, 8))
    dout = rng.normal(size=(1, 4, 6, 8))
    t = [torch.tensor(a, requires_grad=True) for a in (q, k, v)]
    qh = t[0].permute(0, 2, 1, 3)
    kh = t[1].permute(0, 2, 1, 3).repeat_interleave(2, dim=1)
    vh = t[2].permute(0, 2, 1, 3).repeat_interleave(2, dim=1)
    s = qh @ kh.transpose(-1, -2) / np.sqrt(8)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(6, 6, dtype=torch.bool), 1), float("-inf"))
    (torch.softmax(s, -1) @ vh).backward(torch.tensor(dout))
    got = ops.gqa_full_backward(dout, q, k, v, causal=causal)
    for a, b in zip(got, t):
        np.testing.assert_allclose(a, b.grad.numpy(), rtol=1e-9, atol=1e-12)
