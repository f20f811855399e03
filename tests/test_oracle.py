"""CPU: pin the oracle against the reference's known answers and its own code.

These tests run without a GPU. They establish that the oracle -- the checker
every GPU parity test compares against -- reproduces MatcoreDSL's arithmetic:
  * strict f32 pair: the answers the reference's tests state outright;
  * bf16 conversion / bf16 GEMM / int8 GEMM: bit-for-bit against the
    reference's own cpu_numeric_reference.cpp compiled into oracle/_ref;
  * FP8 codecs: exhaustive round trips against the OCP format definition and
    ml_dtypes' independent implementation.
"""
import numpy as np
import pytest

from tests import reference_cases as rc


def test_two_gemm_example(orc):
    a, b, d, c_exp, e_exp = rc.two_gemm_example()
    c = orc.strict_gemm(a, b)
    assert rc.same_bits(c, c_exp)
    assert rc.same_bits(orc.strict_gemm(d, c), e_exp)


@pytest.mark.parametrize("case", rc.known_answers(), ids=lambda c: c[0])
def test_strict_pair_known_answers(orc, case):
    name, a, b, d, expected = case
    e = orc.strict_fused_pair(a, b, d)
    assert rc.same_bits(e, expected), (name, e, expected)


def test_strict_pair_fma_would_differ(orc):
    # The discriminator only means something if an FMA gives another answer.
    eps = rc.EPS
    fused = np.float32(np.float64(1 + eps) * np.float64(1 - eps) - 1.0)
    e = orc.strict_fused_pair(np.array([[-1, 1 + eps]], np.float32),
                              np.array([[1], [1 - eps]], np.float32), np.ones((1, 1), np.float32))
    assert fused != e[0, 0]


def test_strict_pair_equals_two_strict_gemms(orc):
    for name, a, b, d in rc.execution_cases(include_sweep=False):
        if a.shape[0] == 0 or d.shape[1] == 0:
            continue
        e = orc.strict_fused_pair(a, b, d)
        e2 = orc.strict_gemm(orc.strict_gemm(a, b), d)
        assert rc.same_bits(e, e2), name


def test_strict_pair_threads_bit_identical(orc):
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (67, 33)).astype(np.float32)
    b = rng.uniform(-1, 1, (33, 45)).astype(np.float32)
    d = rng.uniform(-1, 1, (45, 19)).astype(np.float32)
    assert rc.same_bits(orc.strict_fused_pair(a, b, d), orc.strict_fused_pair(a, b, d, threads=4))


def test_physical_case_generator_matches_reference_draws():
    # First tiny/tail case with data: m=1,k=1,n=1,p=1 draws after the empty ones.
    cases = rc.physical_cases()
    assert len(cases) == 10 * 4 * 4 * 3 + 32 + 7 + 21 + 5 + 3 + 1
    for name, a, b, d in cases:
        if not name.startswith(("tiny/tail", "seeded-mixed", "work-cap")):
            continue
        for x in (a, b, d):
            # (r % 129 - 64) / 32: multiples of 1/32 in [-2, 2]
            assert np.all(np.abs(x) <= 2.0) and np.all((x * 32) == np.round(x * 32)), name


def _ref():
    import oracle
    r = oracle.ref_lib()
    if r is None:
        pytest.skip("oracle/_ref not built (needs the MatcoreDSL sources)")
    return r


def test_bf16_conversion_matches_reference(orc):
    R = _ref()
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 2 ** 32, 200000, dtype=np.uint64).astype(np.uint32)
    specials = np.array([0, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0x7f800001,
                         0xffffffff, 0x7f7fffff, 0x00000001, 0x3f808000, 0x3f818000,
                         0x3f807fff], np.uint32)
    x = np.concatenate([bits, specials]).view(np.float32)
    mine = orc.bf16_from_f32(x)
    ref = np.empty_like(mine)
    R.ref_bf16_from_f32(x, ref, x.size)
    assert np.array_equal(mine, ref)
    back, ref_back = orc.bf16_to_f32(mine), np.empty(mine.shape, np.float32)
    R.ref_bf16_to_f32(mine, ref_back, mine.size)
    assert np.array_equal(back.view(np.uint32), ref_back.view(np.uint32))


def test_bf16_gemm_matches_reference(orc):
    R = _ref()
    rng = np.random.default_rng(2)
    a = orc.bf16_from_f32(rng.normal(size=(37, 53)).astype(np.float32))
    b = orc.bf16_from_f32(rng.normal(size=(53, 29)).astype(np.float32))
    mine = orc.gemm_bf16_f32_fma(a, b)
    ref = np.empty_like(mine)
    assert R.ref_gemm_bf16_f32(a, b, ref, 37, 53, 29) == 0
    assert np.array_equal(mine.view(np.uint32), ref.view(np.uint32))


def test_i8_gemm_matches_reference(orc):
    R = _ref()
    rng = np.random.default_rng(3)
    a = rng.integers(-128, 128, (19, 300), dtype=np.int8)
    b = rng.integers(-128, 128, (300, 23), dtype=np.int8)
    mine = orc.gemm_i8_i32(a, b)
    ref = np.empty_like(mine)
    assert R.ref_gemm_i8_i32(a, b, ref, 19, 300, 23) == 0
    assert np.array_equal(mine, ref)


def test_quantized_i8_reference_case(orc):
    """The reference's quantized int8 plan and matmul cases
    (tests/test_plan_quantization.py:22-25,32-43; tests/test_matmul.py:60-70):
    2x3 @ 3x2 with zero point 2 on both operands equals (A - 2) @ (B - 2)."""
    lhs = np.array([[4, -3, 2], [1, 0, -2]], dtype=np.int8)
    rhs = np.array([[2, -1], [3, 4], [-2, 1]], dtype=np.int8)
    expected = (lhs.astype(np.int32) - 2) @ (rhs.astype(np.int32) - 2)
    assert np.array_equal(orc.gemm_i8_i32_zp(lhs, rhs, 2, 2), expected)
    assert np.array_equal(expected, [[-5, -16], [14, 3]])


@pytest.mark.parametrize("za,zb", [(0, 0), (2, 2), (-7, 0), (0, 113), (2 ** 30 + 3, -2 ** 31)])
def test_quantized_i8_wraps_like_int32(orc, za, zb):
    """Zero points 0 give the plain int8 GEMM; any others give the exact sum
    reduced modulo 2^32 (int32 wrap-around, as linalg.quantized_matmul)."""
    rng = np.random.default_rng(abs(za) + abs(zb))
    a = rng.integers(-128, 128, (13, 70), dtype=np.int8)
    b = rng.integers(-128, 128, (70, 11), dtype=np.int8)
    exact = (a.astype(object) - za).dot(b.astype(object) - zb)
    wrapped = np.array([[((int(v) + 2 ** 31) % 2 ** 32) - 2 ** 31 for v in row] for row in exact],
                       dtype=np.int64).astype(np.int32)
    got = orc.gemm_i8_i32_zp(a, b, za, zb)
    assert np.array_equal(got, wrapped)
    if za == 0 and zb == 0:
        assert np.array_equal(got, orc.gemm_i8_i32(a, b))


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_codec_exhaustive(orc, fmt):
    ml = pytest.importorskip("ml_dtypes")
    codes = np.arange(256, dtype=np.uint8)
    vals = orc.fp8_decode(codes, fmt)
    mlt = ml.float8_e4m3fn if fmt == "e4m3" else ml.float8_e5m2
    ref = codes.view(mlt).astype(np.float32)
    assert np.array_equal(np.isnan(vals), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert np.array_equal(vals[fin], ref[fin])
    # decode -> encode is the identity on every non-NaN code (saturation aside)
    enc = orc.fp8_encode(vals[fin], fmt)
    dec2 = orc.fp8_decode(enc, fmt)
    finite = np.isfinite(vals[fin])
    assert np.array_equal(dec2[finite], vals[fin][finite])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_fp8_encode_matches_ml_dtypes_rne(orc, fmt):
    ml = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(4)
    mx = 448.0 if fmt == "e4m3" else 57344.0
    x = np.concatenate([rng.normal(scale=mx / 8, size=100000),
                        rng.uniform(-mx, mx, 100000),
                        rng.normal(scale=1e-3, size=20000)]).astype(np.float32)
    mine = orc.fp8_decode(orc.fp8_encode(x, fmt), fmt)
    mlt = ml.float8_e4m3fn if fmt == "e4m3" else ml.float8_e5m2
    ref = x.astype(mlt).astype(np.float32)  # in range: RNE, no saturation needed
    assert np.array_equal(mine, ref)


def test_fp8_saturates(orc):
    q = orc.fp8_encode(np.array([1e6, -1e6, np.inf, 460.0], np.float32), "e4m3")
    assert list(orc.fp8_decode(q, "e4m3")) == [448.0, -448.0, 448.0, 448.0]


def test_blockwise_quantisation_recovers_values(orc):
    rng = np.random.default_rng(5)
    x = rng.normal(size=(300, 260)).astype(np.float32)
    q, s = orc.fp8_quantize_blockwise(x, 128, "e4m3")
    assert s.shape == (3, 3)
    deq = orc.fp8_decode(q, "e4m3") * np.repeat(np.repeat(s, 128, 0), 128, 1)[:300, :260]
    assert orc.rel_frobenius(deq, x) < 0.04
    # every block's absmax maps onto the e4m3 maximum
    assert np.isclose(np.abs(deq[:128, :128]).max(), np.abs(x[:128, :128]).max(), rtol=1e-6)


def test_fp8_gemm_oracle_is_dequantised_product(orc):
    rng = np.random.default_rng(6)
    a = rng.normal(size=(130, 256)).astype(np.float32)
    bt = rng.normal(size=(70, 256)).astype(np.float32)
    qa, sa = orc.fp8_quantize_blockwise(a, 128)
    qb, sb = orc.fp8_quantize_blockwise(bt, 128)
    c = orc.gemm_fp8_blockscaled(qa, sa, qb, sb)
    f64 = np.float64
    da = orc.fp8_decode(qa).astype(f64) * np.repeat(np.repeat(sa.astype(f64), 128, 0), 128, 1)[:130, :256]
    db = orc.fp8_decode(qb).astype(f64) * np.repeat(np.repeat(sb.astype(f64), 128, 0), 128, 1)[:70, :256]
    assert np.allclose(c, da @ db.T, rtol=1e-9, atol=1e-9)
    assert orc.rel_frobenius(c, a.astype(np.float64) @ bt.astype(np.float64).T) < 0.06


def test_gemm_epilogue_oracle_gelu_formula(orc):
    rng = np.random.default_rng(7)
    x = rng.normal(size=(16, 32)).astype(np.float32)
    w = rng.normal(size=(32, 24)).astype(np.float32)
    b = rng.normal(size=24).astype(np.float32)
    y = orc.gemm_epilogue(x, w, b, bias_mode="row", act="gelu_tanh")
    c = x.astype(np.float64) @ w.astype(np.float64) + b
    ref = 0.5 * c * (1 + np.tanh(0.7978845608 * (c + 0.044715 * c ** 3)))
    assert np.allclose(y, ref, rtol=1e-12, atol=1e-12)
    rows = np.array([3, 0, 15])
    assert np.array_equal(orc.gemm_epilogue(x, w, b, bias_mode="row", act="gelu_tanh", rows=rows),
                          y[rows])


def test_msm_oracle_is_row_softmax(orc):
    rng = np.random.default_rng(8)
    q = rng.normal(size=(9, 6)).astype(np.float32)
    k = rng.normal(size=(14, 6)).astype(np.float32)
    v = rng.normal(size=(14, 5)).astype(np.float32)
    o = orc.msm(q, k, v, 0.5)
    s = 0.5 * (q.astype(np.float64) @ k.astype(np.float64).T)
    p = np.exp(s - s.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert np.allclose(o, p @ v.astype(np.float64), rtol=1e-12, atol=1e-12)
