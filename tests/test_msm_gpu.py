"""GPU: matmul-softmax-matmul (Family C) against the fp64 oracle.

* The reference's own Family C cases (tests/test_family_c.py:102-179): f32,
  unscaled softmax, N(0, 0.65) inputs from default_rng(seed), max-abs
  tolerance 2e-3 -- M != N, V width != QK width, and the D=64 route.
* bf16 batched [B,H,S,D] at D=128: relative Frobenius error <= 1e-2.
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


@pytest.mark.parametrize("shape", [(1, 2, 256, 128), (2, 3, 384, 128), (1, 1, 200, 128),
                                   (2, 2, 128, 64)])
def test_bf16_batched(mcb, orc, shape):
    import torch
    b, h, s, d = shape
    rng = np.random.default_rng(sum(shape))
    qh, qf = gu.bf16_pair(rng.standard_normal(shape, dtype=np.float32))
    kh, kf = gu.bf16_pair(rng.standard_normal(shape, dtype=np.float32))
    vh, vf = gu.bf16_pair(rng.standard_normal(shape, dtype=np.float32))
    scale = d ** -0.5
    o = mcb.msm(gu.to_dev_bf16(qh), gu.to_dev_bf16(kh), gu.to_dev_bf16(vh), scale)
    assert o.dtype == torch.bfloat16
    got = gu.from_dev(o)
    for bi in range(b):
        for hi in range(h):
            ref = orc.msm(qf[bi, hi], kf[bi, hi], vf[bi, hi], scale)
            assert orc.rel_frobenius(got[bi, hi], ref) < 1e-2, (bi, hi)
