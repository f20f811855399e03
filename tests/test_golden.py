"""Golden fixtures produced by the reference's own Family A/B/C tests
(tests/golden/make_golden.py): every stored output was accepted by the
reference's assertion (max-abs 1e-3 / 1e-2 / 2e-3).

CPU: the oracle reproduces every stored output.
GPU: the CUDA path reproduces them within the reference's own tolerances.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
TOL = {"a": 1e-3, "b": 1e-2, "c": 2e-3}  # tests/test_family_{a,b,c}.py


def _cases(family):
    path = os.path.join(HERE, "golden", f"family_{family}.npz")
    z = np.load(path)
    index = json.loads(bytes(z["index"]).decode())
    out = []
    for i, meta in enumerate(index):
        ins = [z[f"c{i}_in{j}"] for j in range(meta["inputs"])]
        out.append((meta, ins, z[f"c{i}_out"]))
    return out


def _a_args(meta, ins):
    x, w = ins[0], ins[1]
    bias = ins[2] if meta["bias_mode"] == "full" else None
    return x, w, bias


@pytest.mark.parametrize("family", ["a", "b", "c"])
def test_fixture_files_present(family):
    assert len(_cases(family)) >= 4


@pytest.mark.parametrize("case", _cases("a"), ids=lambda c: c[0]["name"])
def test_oracle_reproduces_family_a(orc, case):
    meta, ins, expected = case
    x, w, bias = _a_args(meta, ins)
    # `sub` with the accumulator on the left was folded into an add of -bias
    got = orc.gemm_epilogue(x, w, bias, bias_mode=meta["bias_mode"], bias_op=meta["bias_op"],
                            act=meta["act"]).astype(np.float32)
    assert np.max(np.abs(got - expected)) <= 1e-6


@pytest.mark.parametrize("case", _cases("c"), ids=lambda c: c[0]["name"])
def test_oracle_reproduces_family_c(orc, case):
    meta, ins, expected = case
    q, k, v = _qkv(meta, ins)
    assert np.max(np.abs(orc.msm(q, k, v, 1.0).astype(np.float32) - expected)) <= 1e-6


def _qkv(meta, ins):
    # graph inputs in argument order; the swapped case binds (K, Q, V)
    if "swapped" in meta["name"]:
        k, q, v = ins
    else:
        q, k, v = ins
    return q, k, v


@pytest.mark.gpu
@pytest.mark.parametrize("case", _cases("a"), ids=lambda c: c[0]["name"])
def test_cuda_family_a_matches_golden(mcb, case):
    meta, ins, expected = case
    x, w, bias = _a_args(meta, ins)
    got = mcb.gemm_epilogue(x, w, bias, bias_mode=meta["bias_mode"], bias_op=meta["bias_op"],
                            act=meta["act"])
    assert np.max(np.abs(got - expected)) < TOL["a"]


def _b_args(meta, ins):
    a, b = ins[0], ins[1]
    if meta["bias_mode"] == "full":
        return a, b, ins[2], ins[3]
    return a, b, None, ins[2]


@pytest.mark.parametrize("case", _cases("b"), ids=lambda c: c[0]["name"])
def test_oracle_reproduces_family_b(orc, case):
    meta, ins, expected = case
    a, b, bnd, w = _b_args(meta, ins)
    mid = orc.gemm_epilogue(a, b, bnd, bias_mode=meta["bias_mode"], bias_op=meta["bias_op"],
                            act=meta["act"]).astype(np.float32)
    got = orc.gemm_epilogue(mid, w).astype(np.float32)
    assert np.max(np.abs(got - expected)) <= 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("case", _cases("b"), ids=lambda c: c[0]["name"])
def test_cuda_family_b_matches_golden(mcb, case):
    meta, ins, expected = case
    a, b, bnd, w = _b_args(meta, ins)
    got = mcb.gemm_chain(a, b, w, bnd, bias_mode=meta["bias_mode"], bias_op=meta["bias_op"],
                         act=meta["act"])
    assert mcb.api.last_result.kernel_launches == 2
    assert np.max(np.abs(got - expected)) < TOL["b"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", _cases("c"), ids=lambda c: c[0]["name"])
def test_cuda_family_c_matches_golden(mcb, case):
    meta, ins, expected = case
    q, k, v = _qkv(meta, ins)
    got = mcb.msm(q, k, v, 1.0)
    assert np.max(np.abs(got - expected)) < TOL["c"]
