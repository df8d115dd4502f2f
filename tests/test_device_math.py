"""CPU checks of the device-side numerics (no GPU needed).

exp2_poly2_lp (csrc/common.cuh) computes 2^x on the FMA pipe for softmax
weights; here the same float32 steps are emulated with numpy, using the
coefficients parsed from the header, and the relative error is checked
against the bound the header states.  The fp32-accuracy paths' bf16 operand
splits are emulated in float64 and checked against the error budget they
are designed to.
"""

import re

import numpy as np

from conftest import PKG_ROOT


def _lp_coefficients():
    src = (PKG_ROOT / "csrc" / "common.cuh").read_text()
    body = src[src.index("float2 exp2_poly2_lp(float2 x)"):]
    body = body[:body.index("\n}\n")]
    consts = re.findall(r"make_float2\(([0-9.e+-]+)f, \1f\)", body)
    # 1.5 * 2^23 (twice, +/-), -1, then c3 and the three Horner constants c2, c1, c0
    poly = [float(c) for c in consts if abs(float(c)) < 2.0 and float(c) != -1.0]
    assert len(poly) == 4, consts
    return [np.float32(c) for c in poly]  # c3, c2, c1, c0


def _fma32(a, b, c):
    # a*b is exact in float64 for float32 inputs; one rounding to float32 after the add
    return (a.astype(np.float64) * b.astype(np.float64) + np.float64(c)).astype(np.float32)


def _exp2_poly2_lp(x):
    c3, c2, c1, c0 = _lp_coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    n = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x - n).astype(np.float32)  # exact: |f| <= 0.5
    q = np.full_like(f, c3)
    for c in (c2, c1, c0):
        q = _fma32(q, f, c)
    bits = (q.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << np.uint64(23)))
    return (bits & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)


def test_exp2_poly2_lp_relative_error():
    # the normal range of the result (below x = -125 the result is only "tiny":
    # adding n to the exponent of a q just under 1 reaches the subnormals)
    x = np.concatenate([np.linspace(-125.0, 8.0, 400001, dtype=np.float32),
                        np.float32(-1.0) * np.random.default_rng(0).random(100000, dtype=np.float32) * 20])
    got = _exp2_poly2_lp(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() <= 7.6e-5, rel.max()


def test_exp2_poly2_lp_clamps_far_negative_to_tiny():
    got = _exp2_poly2_lp(np.array([-200.0, -np.inf, -126.0], dtype=np.float32))
    assert np.all(got >= 0) and np.all(got < 2e-38)


# --------------------------------------------------------------------------
# The fp32-accuracy paths' operand splits (csrc/gemm_f32.cu), emulated in
# float64 on the CPU: two-term hi + lo for the GEMMs (hi.lo + lo.hi + hi.hi,
# lo.lo dropped), three-term hi + mid + lo for bmm_softmax, whose softmax
# turns an absolute score error into a relative probability error.
def _bf(x):
    from oracle.bf16 import to_bf16_rne
    return to_bf16_rne(np.asarray(x, dtype=np.float32)).astype(np.float64)


def _split2_mm(a, b):
    ah, bh = _bf(a), _bf(b)
    al, bl = _bf(a - ah), _bf(b - bh)
    return ah @ bl + al @ bh + ah @ bh


def _split3_mm(a, b):
    ah, bh = _bf(a), _bf(b)
    am, bm = _bf(a - ah), _bf(b - bh)
    al, bl = _bf(a - ah - am), _bf(b - bh - bm)
    return ah @ bm + am @ bh + ah @ bl + al @ bh + am @ bm + ah @ bh


def _softmax(s):
    s = s.astype(np.float32)
    e = np.exp(s - s.max(-1, keepdims=True)).astype(np.float32)
    return (e / e.sum(-1, keepdims=True, dtype=np.float64)).astype(np.float32)


def test_two_term_split_gemm_meets_the_fp32_gate():
    from oracle.metrics import rel_l2
    rng = np.random.default_rng(0)
    a = rng.normal(size=(64, 2048)).astype(np.float32)
    b = rng.normal(size=(2048, 96)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    err = rel_l2(_split2_mm(a, b), exact)
    assert 1e-6 < err < 1e-5     # ~2^-17 per product: well inside 2e-5, far from fp32 rounding


def test_three_term_split_for_the_row_softmax():
    """Scores of N(0,1) operands at K = 64 are ~8: the two-term split leaves the
    softmax at ~80 % of the 2e-5 gate; the three-term split reaches the fp32
    rounding floor."""
    from oracle.metrics import rel_l2
    rng = np.random.default_rng(42)
    a = rng.normal(size=(256, 64)).astype(np.float32)
    b = rng.normal(size=(64, 1024)).astype(np.float32)
    want = _softmax(a.astype(np.float64) @ b.astype(np.float64))
    e2 = rel_l2(_softmax(_split2_mm(a, b)), want)
    e3 = rel_l2(_softmax(_split3_mm(a, b)), want)
    assert 1.0e-5 < e2 < 2e-5
    assert e3 < 2e-6
