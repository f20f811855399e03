"""GPU: the legacy quantized int8 matmul with zero points,
C = sum_k (A - za)(B - zb) in wrapping int32 (src/mlir_engine.cpp:944-958),
through mcb_gemm_i8_i32_zp_v1 and the plan layer, bit for bit against the
oracle. On tcgen05 the raw codes are multiplied and the epilogue adds
K*za*zb - zb*rowsum(A) - za*colsum(B); on CUDA cores the zero points are
subtracted per product."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF_LHS = np.array([[4, -3, 2], [1, 0, -2]], dtype=np.int8)
REF_RHS = np.array([[2, -1], [3, 4], [-2, 1]], dtype=np.int8)


def _launches(n_direct, za, zb, simt=False):
    """Kernel launches of one call: [B^T transpose] [row sums of A when zb]
    [column sums of B when za] GEMM."""
    if simt:
        return 1
    return (0 if n_direct else 1) + (1 if zb else 0) + (1 if za else 0) + 1


@pytest.mark.parametrize("on_device", [True, False])
def test_reference_case(mcb, orc, on_device):
    """The reference's 2x3 @ 3x2 case with zero point 2
    (tests/test_plan_quantization.py:32-43, tests/test_matmul.py:60-70)."""
    import torch
    a, b = REF_LHS, REF_RHS
    if on_device:
        c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(),
                            a_zero_point=2, b_zero_point=2).cpu().numpy()
    else:
        c = mcb.gemm_i8_i32(a, b, a_zero_point=2, b_zero_point=2)
    assert mcb.api.last_result.route == "simt_i8_gemm"
    assert np.array_equal(c, (a.astype(np.int32) - 2) @ (b.astype(np.int32) - 2))
    assert np.array_equal(c, orc.gemm_i8_i32_zp(a, b, 2, 2))


# (M, K, N), zero points, tile rows. N % 16 != 0 sends B through the
# transpose (its column sums are then the row sums of B^T); M >= 256 runs
# the SM-pair kernel.
@pytest.mark.parametrize("shape,za,zb,tile_m", [
    ((256, 512, 384), 2, 2, 256),
    ((300, 1024, 520), -7, 0, 256),
    ((129, 48, 264), 0, 113, 128),
    ((200, 80, 208), 2 ** 30 + 3, -2 ** 31, 128),
    ((1024, 2048, 1024), -128, 127, 256),
    ((520, 112, 272), 1, -1, 256)])
def test_tcgen05_zero_points_bit_exact(mcb, orc, shape, za, zb, tile_m):
    import torch
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(),
                        a_zero_point=za, b_zero_point=zb)
    r = mcb.api.last_result
    assert r.route == "tcgen05_i8_gemm" and r.tile[0] == tile_m
    assert r.kernel_launches == _launches(n % 16 == 0, za, zb)
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32_zp(a, b, za, zb))


def test_cuda_core_zero_points(mcb, orc):
    """A rows not 16-byte aligned: the CUDA-core kernel subtracts the zero
    points per product."""
    import torch
    rng = np.random.default_rng(77)
    a = rng.integers(-128, 128, (77, 100), dtype=np.int8)
    b = rng.integers(-128, 128, (100, 33), dtype=np.int8)
    c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(),
                        a_zero_point=5, b_zero_point=-3)
    assert mcb.api.last_result.route == "simt_i8_gemm"
    assert mcb.api.last_result.kernel_launches == 1
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32_zp(a, b, 5, -3))


@pytest.mark.parametrize("ldb,n", [(400, 337), (400, 384), (344, 336)])
def test_strided_views(mcb, orc, ldb, n):
    """Row-strided A, B and C views. ldb = 400 is read in place: N = 337
    leaves a ragged last group of the 4-column sums (C's rows padded to 340
    int32 keep them 16-byte aligned); ldb = 344 goes through B^T."""
    import torch
    m, k = 300, 144
    rng = np.random.default_rng(ldb + n)
    a_big = rng.integers(-128, 128, (m, 160), dtype=np.int8)
    b_big = rng.integers(-128, 128, (k, ldb), dtype=np.int8)
    a, b = np.ascontiguousarray(a_big[:, :k]), np.ascontiguousarray(b_big[:, :n])
    out = torch.empty((m, (n + 3) // 4 * 4), dtype=torch.int32, device="cuda")[:, :n]
    c = mcb.gemm_i8_i32(torch.from_numpy(a_big).cuda()[:, :k],
                        torch.from_numpy(b_big).cuda()[:, :n], out=out, a_zero_point=-3,
                        b_zero_point=9)
    r = mcb.api.last_result
    assert r.route == "tcgen05_i8_gemm"
    assert r.kernel_launches == _launches(ldb % 16 == 0, -3, 9)
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32_zp(a, b, -3, 9))


def test_wraps_modulo_2_32(mcb):
    """K large enough for the exact sum to leave int32: every output is
    K * (-128 - za) * (-128 - zb) reduced modulo 2^32."""
    import torch
    m, k, n = 128, 135168, 256
    za, zb = 3, -1
    a = torch.full((m, k), -128, dtype=torch.int8, device="cuda")
    b = torch.full((k, n), -128, dtype=torch.int8, device="cuda")
    c = mcb.gemm_i8_i32(a, b, a_zero_point=za, b_zero_point=zb)
    exact = k * (-128 - za) * (-128 - zb)
    wrapped = ((exact + 2 ** 31) % 2 ** 32) - 2 ** 31
    assert exact != wrapped
    assert bool((c == wrapped).all())


def test_zero_points_zero_is_plain_gemm(mcb, orc):
    import torch
    rng = np.random.default_rng(8)
    a = rng.integers(-128, 128, (256, 256), dtype=np.int8)
    b = rng.integers(-128, 128, (256, 256), dtype=np.int8)
    c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(),
                        a_zero_point=0, b_zero_point=0)
    assert mcb.api.last_result.kernel_launches == 1
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32(a, b))


@pytest.mark.parametrize("graph", [False, True])
def test_plan_with_zero_points(mcb, orc, graph):
    """Shape-locked plan (create_plan / execute_plan) with frozen zero points,
    replayed on new data; zero points that differ from the plan's are
    rejected like the reference's "quantization mismatch"
    (tests/test_plan_quantization.py:46-64)."""
    import torch
    m, k, n = 256, 384, 200   # N % 16 != 0: B^T and both sums in the plan's workspace
    rng = np.random.default_rng(31)
    a = torch.empty((m, k), dtype=torch.int8, device="cuda")
    b = torch.empty((k, n), dtype=torch.int8, device="cuda")
    c = torch.empty((m, n), dtype=torch.int32, device="cuda")
    plan = mcb.Plan("gemm_i8_i32", c, a, b, graph=graph, a_zero_point=2, b_zero_point=-5)
    for _ in range(2):
        ah = rng.integers(-128, 128, (m, k), dtype=np.int8)
        bh = rng.integers(-128, 128, (k, n), dtype=np.int8)
        a.copy_(torch.from_numpy(ah))
        b.copy_(torch.from_numpy(bh))
        plan.execute(c, a, b)
        torch.cuda.synchronize()
        assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32_zp(ah, bh, 2, -5))
    plan.execute(c, a, b, a_zero_point=2, b_zero_point=-5)   # matching metadata: accepted
    with pytest.raises(RuntimeError, match="quantization mismatch"):
        plan.execute(c, a, b, a_zero_point=1)
    plan.close()
