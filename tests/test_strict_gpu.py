"""GPU: the strict f32 GEMM and fused pair are bit-exact with the oracle.

Cases are the reference's own strict test suites regenerated from the same
mt19937 draws (tests/reference_cases.py), the stated known answers, and
BASELINE config 1 at full size. All calls go through the C ABI.
"""
import numpy as np
import pytest

from tests import reference_cases as rc

pytestmark = pytest.mark.gpu


def _check_pair(mcb, orc, name, a, b, d):
    got = mcb.strict_fused_pair(a, b, d)
    exp = orc.strict_fused_pair(a, b, d)
    assert rc.same_bits(got, exp), name


def test_known_answers(mcb, orc):
    for name, a, b, d, expected in rc.known_answers():
        got = mcb.strict_fused_pair(a, b, d)
        assert rc.same_bits(got, expected), (name, got, expected)


def test_two_gemm_example(mcb):
    a, b, d, c_exp, e_exp = rc.two_gemm_example()
    c = mcb.strict_gemm(a, b)
    assert rc.same_bits(c, c_exp)
    assert rc.same_bits(mcb.strict_gemm(d, c), e_exp)


def test_physical_suite_bit_exact(mcb, orc):
    for name, a, b, d in rc.physical_cases():
        if a.shape[0] == 0 or d.shape[1] == 0:
            continue  # empty E: nothing to launch, nothing to compare
        _check_pair(mcb, orc, name, a, b, d)


def test_execution_suite_bit_exact(mcb, orc):
    for name, a, b, d in rc.execution_cases():
        if a.shape[0] == 0 or d.shape[1] == 0:
            continue
        _check_pair(mcb, orc, name, a, b, d)


def test_large_n_two_pass(mcb, orc):
    """N far beyond a shared-memory panel: C goes through device memory."""
    rng = np.random.default_rng(11)
    a = rng.uniform(-1, 1, (37, 5)).astype(np.float32)
    b = rng.uniform(-1, 1, (5, 70001)).astype(np.float32)
    d = rng.uniform(-1, 1, (70001, 3)).astype(np.float32)
    got = mcb.strict_fused_pair(a, b, d)
    assert mcb.api.last_result.route == "strict_f32_simt_pair_two_pass"
    assert rc.same_bits(got, orc.strict_fused_pair(a, b, d))


def test_strict_gemm_bit_exact(mcb, orc):
    rng = np.random.default_rng(12)
    for m, k, n in [(1, 1, 1), (7, 0, 5), (33, 65, 129), (300, 257, 513), (1024, 64, 1024),
                    (700, 31, 600)]:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        assert rc.same_bits(mcb.strict_gemm(a, b), orc.strict_gemm(a, b)), (m, k, n)


@pytest.mark.parametrize("m,k,n", [(2048, 96, 2048), (2000, 100, 1992), (1664, 20, 1536)])
def test_strict_gemm_large_tiles_bit_exact(mcb, orc, m, k, n):
    """Problems of at least one 128x128 tile per SM run 8x8 chains per thread
    (edge tiles, K not a multiple of the 16-deep slice); still bit-exact, with
    IEEE specials in A and B."""
    import torch
    rng = np.random.default_rng(m + k + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    a[3, 5] = np.inf
    a[10, :] = -0.0
    b[7, 11] = np.nan
    b[:, 13] = 1e-39  # subnormal
    c = mcb.strict_gemm(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    r = mcb.api.last_result
    assert r.route == "strict_f32_simt_gemm_tiled" and r.tile[:2] == (128, 128)
    assert rc.same_bits(c.cpu().numpy(), orc.strict_gemm(a, b))


def _config1():
    a = np.random.default_rng(0).uniform(-1, 1, (512, 256)).astype(np.float32)
    b = np.random.default_rng(1).uniform(-1, 1, (256, 384)).astype(np.float32)
    d = np.random.default_rng(2).uniform(-1, 1, (384, 128)).astype(np.float32)
    return a, b, d


def test_config1_bit_exact_host_and_device(mcb, orc):
    import torch
    a, b, d = _config1()
    exp = orc.strict_fused_pair(a, b, d)
    assert rc.same_bits(mcb.strict_fused_pair(a, b, d), exp)
    ta, tb, td = (torch.from_numpy(x).cuda() for x in (a, b, d))
    te = mcb.strict_fused_pair(ta, tb, td)
    torch.cuda.synchronize()
    assert rc.same_bits(te.cpu().numpy(), exp)


def test_strided_device_operands(mcb, orc):
    import torch
    a, b, d = _config1()
    big = torch.zeros(512, 300, device="cuda")
    big[:, 10:266] = torch.from_numpy(a).cuda()
    ta = big[:, 10:266]  # row stride 300, offset base
    te = mcb.strict_fused_pair(ta, torch.from_numpy(b).cuda(), torch.from_numpy(d).cuda())
    torch.cuda.synchronize()
    assert rc.same_bits(te.cpu().numpy(), orc.strict_fused_pair(a, b, d))


@pytest.mark.parametrize("m,k,n,p", [(9, 8, 12, 8), (5, 4, 4, 1024), (64, 36, 200, 4)])
def test_staged_route_bit_exact(mcb, orc, m, k, n, p):
    """Small 16-byte aligned pairs (M*N < 16384, N, P <= 1024) take the fused
    shared-memory staged kernel: tail panels and a short last K chunk."""
    rng = np.random.default_rng(m + k + n + p)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    d = rng.uniform(-1, 1, (n, p)).astype(np.float32)
    got = mcb.strict_fused_pair(a, b, d)
    assert mcb.api.last_result.route == "strict_f32_simt_pair_staged"
    assert rc.same_bits(got, orc.strict_fused_pair(a, b, d))


@pytest.mark.parametrize("m,k,n,p", [(512, 256, 384, 128), (301, 68, 100, 12),
                                     (600, 512, 1024, 1024), (301, 67, 101, 13),
                                     (1000, 3, 17, 250), (130, 0, 128, 8), (800, 40, 500, 36)])
def test_two_pass_bit_exact(mcb, orc, m, k, n, p):
    """Larger pairs run as two tiled strict GEMMs through a binary32 C: tile
    edges in M, N and P, 16-byte and 4-byte copy paths, K = 0 (E = +0 * D)."""
    rng = np.random.default_rng(m + 3 * k + 5 * n + 7 * p)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    d = rng.uniform(-1, 1, (n, p)).astype(np.float32)
    if k == 0:
        d[3, 2] = np.inf  # +0 * inf = NaN must reach E
    got = mcb.strict_fused_pair(a, b, d)
    assert mcb.api.last_result.route == "strict_f32_simt_pair_two_pass"
    assert mcb.api.last_result.kernel_launches == 2
    assert rc.same_bits(got, orc.strict_fused_pair(a, b, d))


@pytest.mark.parametrize("shape", [(9, 8, 12, 8), (130, 8, 128, 8)])
def test_ieee_specials_both_routes(mcb, orc, shape):
    """Signed zeros, subnormals, infinities and NaNs through the staged and the
    two-pass routes."""
    m, k, n, p = shape
    rng = np.random.default_rng(99)
    pool = np.array([0.0, -0.0, 1e-40, -3e-39, np.inf, -np.inf, np.nan, 1.5, -2.25, 3e38,
                     -1e-45, 0.1], np.float32)
    a, b, d = (rng.choice(pool, size=sh).astype(np.float32)
               for sh in ((m, k), (k, n), (n, p)))
    got = mcb.strict_fused_pair(a, b, d)
    assert mcb.api.last_result.route == ("strict_f32_simt_pair_staged" if m * n < 16384
                                         else "strict_f32_simt_pair_two_pass")
    assert rc.same_bits(got, orc.strict_fused_pair(a, b, d))
