"""GPU: matmul-softmax-matmul (Family C) against the fp64 oracle.

* The reference's own Family C cases (tests/test_family_c.py:102-179): f32,
  unscaled softmax, N(0, 0.65) inputs from default_rng(seed), max-abs
  tolerance 2e-3 -- M != N, V width != QK width, and the D=64 route.
* bf16 batched [B,H,S,D] at D=64 and D=128 (tensor cores): relative
  Frobenius error <= 1e-2.
"""
import numpy as np
import pytest

from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

FAMILY_C = [  # (name, M, N, qk_width, v_width, seed)
    ("unscaled 16x16x8", 16, 16, 8, 8, 1001),
    ("rectangular 9x14x6", 9, 14, 6, 6, 1002),
    ("value width 10x12x7->5", 10, 12, 7, 5, 1003),
    ("swapped args 12x12x6->4", 12, 12, 6, 4, 1004),
    ("small 16x16x8", 16, 16, 8, 8, 1005),
    ("dtile64 8x12x64", 8, 12, 64, 64, 1006),
]


def _family_c_inputs(m, n, dqk, dv, seed):
    rng = np.random.default_rng(seed)
    q = rng.normal(0.0, 0.65, size=(m, dqk)).astype(np.float32)
    k = rng.normal(0.0, 0.65, size=(n, dqk)).astype(np.float32)
    v = rng.normal(0.0, 0.65, size=(n, dv)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("case", FAMILY_C, ids=lambda c: c[0])
def test_family_c_reference_cases(mcb, orc, case):
    _, m, n, dqk, dv, seed = case
    q, k, v = _family_c_inputs(m, n, dqk, dv, seed)
    o = mcb.msm(q, k, v)
    ref = orc.msm(q, k, v, 1.0)
    assert np.max(np.abs(o - ref)) < 2e-3
    # the inputs distinguish scaled from unscaled softmax, as the reference requires
    if seed == 1001:
        assert np.max(np.abs(ref - orc.msm(q, k, v, 1 / np.sqrt(dqk)))) > 5e-2


def _bf16_case(shape, seed, kv_len=None, k_growth=0.0):
    b, h, s, d = shape
    n = kv_len or s
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((b, h, s, d), dtype=np.float32)
    k = rng.standard_normal((b, h, n, d), dtype=np.float32)
    v = rng.standard_normal((b, h, n, d), dtype=np.float32)
    if k_growth:  # later key tiles score higher: forces the running max to grow
        k *= (1.0 + k_growth * (np.arange(n) // 128))[None, None, :, None].astype(np.float32)
    return [gu.bf16_pair(x) for x in (q, k, v)]


def _check_msm(mcb, orc, pairs, scale, route, pairs_to_check=None):
    import torch
    (qh, qf), (kh, kf), (vh, vf) = pairs
    o = mcb.msm(gu.to_dev_bf16(qh), gu.to_dev_bf16(kh), gu.to_dev_bf16(vh), scale)
    assert mcb.api.last_result.route == route
    if route == "tcgen05_bf16_msm":
        m = qh.shape[2]  # 256-row query blocks (two tiles per CTA) unless that wastes too much
        two = m % 256 == 0 or m % 256 > 128 or m >= 2048
        assert mcb.api.last_result.tile[0] == (256 if two else 128)
    assert o.dtype == torch.bfloat16
    got = gu.from_dev(o)
    b, h = qh.shape[:2]
    todo = pairs_to_check or [(bi, hi) for bi in range(b) for hi in range(h)]
    for bi, hi in todo:
        ref = orc.msm(qf[bi, hi], kf[bi, hi], vf[bi, hi], scale)
        assert orc.rel_frobenius(got[bi, hi], ref) < 1e-2, (bi, hi)


@pytest.mark.parametrize("shape,route", [
    ((1, 2, 256, 128), "tcgen05_bf16_msm"),
    ((2, 3, 384, 128), "tcgen05_bf16_msm"),
    ((1, 1, 128, 128), "tcgen05_bf16_msm"),
    ((3, 5, 768, 128), "tcgen05_bf16_msm"),
    ((1, 2, 512, 128), "tcgen05_bf16_msm"),
    ((2, 3, 1536, 128), "tcgen05_bf16_msm"),
    ((1, 1, 200, 128), "tcgen05_bf16_msm"),   # ragged M: one partial 256-row block
    ((2, 3, 1000, 128), "tcgen05_bf16_msm"),  # ragged M, two-tile units
    ((1, 2, 300, 128), "tcgen05_bf16_msm"),   # ragged M, single-tile units
    ((2, 2, 128, 64), "tcgen05_bf16_msm"),    # D = 64: one 64-column chunk per tile
    ((2, 3, 1536, 64), "tcgen05_bf16_msm"),
    ((1, 1, 200, 64), "tcgen05_bf16_msm"),
    ((2, 3, 1000, 64), "tcgen05_bf16_msm"),
    ((1, 2, 300, 64), "tcgen05_bf16_msm"),
    ((1, 3, 200, 32), "simt_tiled_online_softmax_msm"),
    ((1, 2, 100, 96), "simt_online_softmax_msm"),         # other widths: row-per-warp kernel
])
def test_bf16_batched(mcb, orc, shape, route):
    _check_msm(mcb, orc, _bf16_case(shape, sum(shape)), shape[-1] ** -0.5, route)


def test_tcgen05_rescale_path(mcb, orc):
    """Key tiles with growing scores make the running max jump several times."""
    _check_msm(mcb, orc, _bf16_case((1, 2, 256, 128), 5, kv_len=1024, k_growth=0.6),
               128 ** -0.5, "tcgen05_bf16_msm")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("rows", [128, 256, 512])
def test_tcgen05_rescale_path_by_route(mcb, orc, rows, d):
    """Growing key tiles with one and two 256-row units per (b, h), and
    single-tile (128-row) units."""
    _check_msm(mcb, orc, _bf16_case((1, 2, rows, d), 15, kv_len=768, k_growth=0.6),
               d ** -0.5, "tcgen05_bf16_msm")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("rows,kv", [(256, 333), (129, 1), (517, 130), (1000, 1001)])
def test_tcgen05_ragged_keys(mcb, orc, rows, kv, d):
    """N not a multiple of 128: the partial last key tile is masked (its
    zero-filled keys must not enter the softmax); M ragged as well."""
    _check_msm(mcb, orc, _bf16_case((1, 2, rows, d), rows + kv, kv_len=kv), d ** -0.5,
               "tcgen05_bf16_msm")


@pytest.mark.parametrize("rows", [256, 512])
def test_tcgen05_unscaled_reference_semantics(mcb, orc, rows):
    """scale = 1 (the reference's mc.softmax(Q @ K.T)): scores of std ~11."""
    _check_msm(mcb, orc, _bf16_case((1, 1, rows, 128), 6, kv_len=640), 1.0, "tcgen05_bf16_msm")


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("s,n", [(256, 640), (512, 640), (300, 601)])
def test_tcgen05_rectangular_and_strided(mcb, orc, s, n, d):
    """M != N, and Q/K/V as strided views of a packed [B, S, 3, H, D] tensor
    (TMA stores of O clipped at a ragged M, a masked partial key tile)."""
    import torch
    b, h = 2, 2
    rng = np.random.default_rng(9)
    packed = rng.standard_normal((b, n, 3, h, d), dtype=np.float32)
    ph, pf = gu.bf16_pair(packed)
    t = gu.to_dev_bf16(ph)
    q = t[:, :s, 0].permute(0, 2, 1, 3)   # [B, H, S, D] with row stride 3*H*D
    k = t[:, :, 1].permute(0, 2, 1, 3)
    v = t[:, :, 2].permute(0, 2, 1, 3)
    o = mcb.msm(q, k, v, d ** -0.5)
    assert mcb.api.last_result.route == "tcgen05_bf16_msm"
    got = gu.from_dev(o)
    for bi in range(b):
        for hi in range(h):
            ref = orc.msm(pf[bi, :s, 0, hi], pf[bi, :, 1, hi], pf[bi, :, 2, hi], d ** -0.5)
            assert orc.rel_frobenius(got[bi, hi], ref) < 1e-2


def config3_pairs(bh_subset):
    """Q, K, V [8,32,4096,128] ~ N(0,1), seed 20, drawn Q, K, V."""
    rng = np.random.default_rng(20)
    shape = (8, 32, 4096, 128)
    return [rng.standard_normal(shape, dtype=np.float32) for _ in range(3)]


def test_config3_full_size_sampled(mcb, orc):
    q, k, v = config3_pairs(None)
    pairs = [gu.bf16_pair(x) for x in (q, k, v)]
    del q, k, v
    sample = [(0, 0), (3, 17), (5, 31), (7, 9)]
    _check_msm(mcb, orc, pairs, 128 ** -0.5, "tcgen05_bf16_msm", sample)
    assert mcb.device_status(0) == 0


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(1, 2, 300, 1000, 128), (2, 1, 64, 65, 64), (1, 1, 1, 1, 32),
                                   (1, 1, 70, 7, 64)])
def test_tiled_cuda_core_msm(mcb, orc, dtype, shape):
    """The tiled CUDA-core kernel (f32 and bf16 inputs, D in {32, 64, 128}):
    ragged M and N (zero-filled rows, masked keys), single keys, single
    queries. f32 at the reference's max-abs 2e-3; bf16 at 1e-2 rel. Frobenius.
    bf16 operands are row-padded views (row stride D + 2, not 16-byte
    aligned), which the tensor-core kernels do not take."""
    import torch
    b, h, m, n, d = shape
    rng = np.random.default_rng(sum(shape))
    q = rng.normal(0.0, 0.65, size=(b, h, m, d)).astype(np.float32)
    k = rng.normal(0.0, 0.65, size=(b, h, n, d)).astype(np.float32)
    v = rng.normal(0.0, 1.0, size=(b, h, n, d)).astype(np.float32)
    if dtype == "bf16":
        (qh, qf), (kh, kf), (vh, vf) = (gu.bf16_pair(x) for x in (q, k, v))
        pad = [(0, 0)] * 3 + [(0, 2)]
        args = [gu.to_dev_bf16(np.pad(x, pad))[..., :d] for x in (qh, kh, vh)]
    else:
        qf, kf, vf = q, k, v
        args = [torch.from_numpy(x).cuda() for x in (q, k, v)]
    o = mcb.msm(*args, d ** -0.5)
    assert mcb.api.last_result.route == "simt_tiled_online_softmax_msm"
    got = gu.from_dev(o)
    for bi in range(b):
        for hi in range(h):
            ref = orc.msm(qf[bi, hi], kf[bi, hi], vf[bi, hi], d ** -0.5)
            if dtype == "f32":
                assert np.max(np.abs(got[bi, hi] - ref)) < 2e-3
            else:
                assert orc.rel_frobenius(got[bi, hi], ref) < 1e-2



@pytest.mark.parametrize("scale", [-0.125, -1.0, 0.0])
@pytest.mark.parametrize("shape,route", [
    ((1, 2, 256, 128), "tcgen05_bf16_msm"),
    ((1, 2, 300, 64), "tcgen05_bf16_msm"),      # single-tile units, ragged M
    ((2, 2, 1000, 128), "tcgen05_bf16_msm"),    # two-tile units, ragged M and keys
    ((1, 3, 200, 32), "simt_tiled_online_softmax_msm"),
    ((1, 2, 100, 96), "simt_online_softmax_msm"),
])
def test_non_positive_scale(mcb, orc, scale, shape, route):
    """softmax(scale * Q K^T) for scale <= 0 on every route: a negative scale
    turns the smallest score into the largest exponent (the tensor-core
    kernels negate Q inside the S MMA and keep |scale|), and scale = 0 gives
    uniform weights, i.e. the mean of V's rows."""
    _check_msm(mcb, orc, _bf16_case(shape, 31 + sum(shape)), scale, route)
    assert mcb.device_status(0) == 0


def test_scale_not_finite_in_f32_rejected(mcb):
    import torch
    q = torch.zeros((1, 1, 128, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(mcb.McbError) as ei:
        mcb.msm(q, q, q, 1e300)
    assert "INVALID_ARGUMENT" in str(ei.value)
