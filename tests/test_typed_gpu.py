"""GPU: typed isolated GEMMs, bit-exact with the reference's typed references
(compiler/lib/runtime/cpu_numeric_reference.cpp): int8 x int8 -> int32 modulo
2^32 on tcgen05 (kind::i8) and CUDA cores, and bf16 x bf16 -> f32 with one
fma per k in increasing order. Compared bit for bit with the oracle and, when
it was compiled here, with the reference's own code (oracle/_ref)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref_i8(a, b):
    import oracle
    r = oracle.ref_lib()
    if r is None:
        return None
    c = np.empty((a.shape[0], b.shape[1]), np.int32)
    assert r.ref_gemm_i8_i32(np.ascontiguousarray(a), np.ascontiguousarray(b), c,
                             a.shape[0], a.shape[1], b.shape[1]) == 0
    return c


# (shape, route, launches, tile rows): B with 16-byte aligned rows is read
# MN-major in place (one launch); other B go through a transpose pass (two
# launches). M >= 256 runs on SM pairs (256-row tiles).
@pytest.mark.parametrize("shape,route,launches,tile_m", [
    ((256, 512, 384), "tcgen05_i8_gemm", 1, 256),
    ((300, 1024, 520), "tcgen05_i8_gemm", 2, 256),
    ((129, 48, 264), "tcgen05_i8_gemm", 2, 128),
    ((200, 80, 208), "tcgen05_i8_gemm", 1, 128),
    ((1024, 2048, 1024), "tcgen05_i8_gemm", 1, 256),
    ((520, 112, 272), "tcgen05_i8_gemm", 1, 256),
    ((77, 100, 33), "simt_i8_gemm", 1, None)])
def test_i8_gemm_bit_exact(mcb, orc, shape, route, launches, tile_m):
    import torch
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    r = mcb.api.last_result
    assert r.route == route and r.kernel_launches == launches
    if tile_m is not None:
        assert r.tile[0] == tile_m
    got = c.cpu().numpy()
    assert np.array_equal(got, orc.gemm_i8_i32(a, b))
    ref = _ref_i8(a, b)
    if ref is not None:
        assert np.array_equal(got, ref)


@pytest.mark.parametrize("ldb,launches", [(400, 1), (344, 2)])
def test_i8_gemm_strided_operands(mcb, orc, ldb, launches):
    """Row-strided A and B views: an aligned B stride is read in place, an
    unaligned one is transposed first; both stay bit-exact."""
    import torch
    m, k, n = 300, 144, 336
    rng = np.random.default_rng(ldb)
    a_big = rng.integers(-128, 128, (m, 160), dtype=np.int8)
    b_big = rng.integers(-128, 128, (k, ldb), dtype=np.int8)
    a, b = a_big[:, :k], b_big[:, :n]
    c = mcb.gemm_i8_i32(torch.from_numpy(a_big).cuda()[:, :k], torch.from_numpy(b_big).cuda()[:, :n])
    r = mcb.api.last_result
    assert r.route == "tcgen05_i8_gemm" and r.kernel_launches == launches
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32(np.ascontiguousarray(a),
                                                           np.ascontiguousarray(b)))


def test_i8_gemm_wraps_modulo_2_32(mcb, orc):
    """K large enough for the exact sum to leave int32: the result wraps."""
    import torch
    m, k, n = 128, 135168, 256
    a = np.full((m, k), -128, np.int8)
    b = np.full((k, n), -128, np.int8)
    c = mcb.gemm_i8_i32(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    exact = 128 * 128 * k  # 2.2e9 > 2^31 - 1
    assert np.all(c.cpu().numpy() == np.int32(np.int64(exact) - 2 ** 32))
    assert np.array_equal(c.cpu().numpy()[:2, :3], orc.gemm_i8_i32(a[:2], b[:, :3]))


def test_i8_gemm_host_operands(mcb, orc):
    rng = np.random.default_rng(5)
    a = rng.integers(-128, 128, (64, 96), dtype=np.int8)
    b = rng.integers(-128, 128, (96, 80), dtype=np.int8)
    assert np.array_equal(mcb.gemm_i8_i32(a, b), orc.gemm_i8_i32(a, b))


@pytest.mark.parametrize("shape,route", [
    ((37, 53, 29), "simt_bf16_f32_fma_gemm"),          # unaligned rows: one thread per output
    ((256, 1000, 300), "simt_bf16_f32_fma_gemm"),      # N % 8 != 0
    ((256, 1000, 304), "simt_bf16_f32_fma_gemm_tiled"),
    ((1030, 72, 520), "simt_bf16_f32_fma_gemm_tiled"),
    ((700, 264, 1024), "simt_bf16_f32_fma_gemm_tiled"),
    ((2048, 64, 1280), "simt_bf16_f32_fma_gemm_128x128"),
    ((1500, 200, 1608), "simt_bf16_f32_fma_gemm_128x128")])  # edge tiles, K % 16 == 8
def test_bf16_f32_fma_bit_exact(mcb, orc, shape, route):
    import torch
    from tests import gpu_util as gu
    m, k, n = shape
    rng = np.random.default_rng(sum(shape))
    ah, _ = gu.bf16_pair(rng.standard_normal((m, k), dtype=np.float32))
    bh, _ = gu.bf16_pair(rng.standard_normal((k, n), dtype=np.float32))
    c = mcb.gemm_bf16_f32_fma(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh))
    assert mcb.api.last_result.route == route
    got = c.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), orc.gemm_bf16_f32_fma(ah, bh).view(np.uint32))
    import oracle
    r = oracle.ref_lib()
    if r is not None:
        ref = np.empty((m, n), np.float32)
        assert r.ref_gemm_bf16_f32(ah, bh, ref, m, k, n) == 0
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert c.dtype == torch.float32
