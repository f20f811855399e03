"""block_attn_res, the reference's region op (tests/test_block_attn_res.py).

CPU: the oracle reproduces the golden fixtures that the reference's own two
tests accepted (tests/golden/block_attn_res.npz), and the argument rules of
matcore/frontend.py:1734-1765 are enforced without a GPU.
GPU: the CUDA kernels match the fixtures and the oracle at the reference's
tolerance (rtol = atol = 1e-4) on its test shapes and its benchmark shapes
([MAX_BLOCKS, B, T, D] = [8,4,512,128] ... [16,8,2048,128]), plus the shapes
that select each kernel (warp per row for D = 128/256 with more sources than
its register cache, 8 lanes per row for D = 32/64, the general kernel
otherwise) and row counts that leave partial CTAs.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _cases():
    z = np.load(os.path.join(HERE, "golden", "block_attn_res.npz"))
    index = json.loads(bytes(z["index"]).decode())
    return [(m, [z[f"c{i}_in{j}"] for j in range(m["inputs"])], z[f"c{i}_out"],
             z[f"c{i}_expected"]) for i, m in enumerate(index)]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0]["name"])
def test_oracle_reproduces_golden(orc, case):
    meta, (blocks, partial, query), stored, ref_expected = case
    got = orc.block_attn_res(blocks, partial, query, meta["block_count"], meta["has_partial"],
                             meta["eps"])
    np.testing.assert_allclose(got, stored, rtol=1e-6, atol=1e-6)
    # the reference test's own numpy expectation (tests/test_block_attn_res.py:16-39)
    np.testing.assert_allclose(got, ref_expected, rtol=1e-6, atol=1e-6)


def test_argument_rules_enforced_without_gpu(mcb):
    blocks = np.zeros((33, 1, 2, 4), np.float32)
    partial = np.zeros((1, 2, 4), np.float32)
    query = np.zeros(4, np.float32)
    for kwargs in ({"block_count": 1, "eps": 1e-5},):
        with pytest.raises(mcb.McbError) as e:  # MAX_BLOCKS > 32
            mcb.block_attn_res(blocks, partial, query, **kwargs)
        assert e.value.name == "INVALID_SHAPE"
    with pytest.raises(mcb.McbError) as e:  # eps must be positive
        mcb.block_attn_res(blocks[:4], partial, query, block_count=1, eps=0.0)
    assert e.value.name == "INVALID_ARGUMENT"
    with pytest.raises(mcb.McbError) as e:  # block_count in [0, MAX_BLOCKS]
        mcb.block_attn_res(blocks[:4], partial, query, block_count=5, eps=1e-5)
    assert e.value.name == "INVALID_ARGUMENT"


@pytest.mark.gpu
@pytest.mark.parametrize("case", _cases(), ids=lambda c: c[0]["name"])
def test_cuda_matches_golden(mcb, case):
    meta, (blocks, partial, query), _, expected = case  # the reference test's expectation
    got = mcb.block_attn_res(blocks, partial, query, block_count=meta["block_count"],
                             has_partial=meta["has_partial"], eps=meta["eps"])
    assert mcb.api.last_result.route == "block_attn_res"
    np.testing.assert_allclose(got, expected, rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(8, 4, 512, 128), (8, 8, 1024, 128), (16, 8, 1024, 128),
                                   (8, 4, 1024, 256), (16, 8, 2048, 128), (5, 2, 33, 7),
                                   (32, 2, 33, 128), (12, 1, 17, 256), (6, 3, 40, 64),
                                   (4, 2, 30, 32)])
@pytest.mark.parametrize("block_count,has_partial", [("all", True), ("half", False), (0, True),
                                                     (0, False)])
def test_cuda_matches_oracle(mcb, orc, shape, block_count, has_partial):
    import torch
    maxb, b, t, d = shape
    bc = {"all": maxb, "half": maxb // 2}.get(block_count, block_count)
    rng = np.random.default_rng(sum(shape))
    blocks = rng.normal(size=shape).astype(np.float32)
    partial = rng.normal(size=(b, t, d)).astype(np.float32)
    query = rng.normal(size=(d,)).astype(np.float32)
    dev = [torch.from_numpy(x).cuda() for x in (blocks, partial, query)]
    got = mcb.block_attn_res(*dev, block_count=bc, has_partial=has_partial, eps=1e-6)
    ref = orc.block_attn_res(blocks, partial, query, bc, has_partial, 1e-6)
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)
