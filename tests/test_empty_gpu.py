"""GPU: empty dimensions on every entry point. M = 0 or N = 0 launch nothing
and leave the (empty) output alone; K = 0 makes every GEMM sum empty, so the
output is the epilogue of a zero accumulator (bias and activation only) or
plain zeros, exactly as the oracle computes it."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("m,k,n", [(0, 64, 32), (48, 64, 0), (48, 0, 32)])
def test_gemm_epilogue_empty(mcb, orc, m, k, n):
    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((k, n)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    y = mcb.gemm_epilogue(_dev(x), _dev(w), _dev(b), bias_mode="row", act="gelu_tanh")
    assert tuple(y.shape) == (m, n)
    ref = orc.gemm_epilogue(x, w, b, bias_mode="row", act="gelu_tanh")
    assert np.allclose(y.cpu().numpy(), ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("m,k,n", [(0, 16, 8), (8, 16, 0), (8, 0, 8)])
def test_typed_gemms_empty(mcb, orc, m, k, n):
    from tests import gpu_util as gu
    rng = np.random.default_rng(7)
    a = rng.integers(-128, 128, (m, k), dtype=np.int8)
    b = rng.integers(-128, 128, (k, n), dtype=np.int8)
    c = mcb.gemm_i8_i32(_dev(a), _dev(b))
    assert np.array_equal(c.cpu().numpy(), orc.gemm_i8_i32(a, b))
    ah, _ = gu.bf16_pair(rng.standard_normal((m, k)).astype(np.float32))
    bh, _ = gu.bf16_pair(rng.standard_normal((k, n)).astype(np.float32))
    f = mcb.gemm_bf16_f32_fma(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh))
    assert np.array_equal(f.cpu().numpy().view(np.uint32),
                          orc.gemm_bf16_f32_fma(ah, bh).view(np.uint32))


def test_msm_empty_queries_and_no_keys(mcb):
    """No queries: nothing to compute. No keys: a softmax over an empty row is
    undefined, so the call is refused with INVALID_SHAPE and O is untouched."""
    import torch
    from matcoredsl_b200 import _abi
    rng = np.random.default_rng(3)
    k = rng.standard_normal((16, 32)).astype(np.float32)
    v = rng.standard_normal((16, 32)).astype(np.float32)
    o = torch.empty((0, 32), device="cuda")
    mcb.msm(_dev(np.zeros((0, 32), np.float32)), _dev(k), _dev(v), out=o)
    q = rng.standard_normal((16, 32)).astype(np.float32)
    o = torch.full((16, 32), 7.0, device="cuda")
    with pytest.raises(mcb.McbError) as err:
        mcb.msm(_dev(q), _dev(k[:0]), _dev(v[:0]), out=o)
    assert err.value.code == _abi.STATUS_CODE["INVALID_SHAPE"]
    assert torch.all(o == 7.0)
    assert mcb.device_status(0) == 0
