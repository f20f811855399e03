"""Golden fixtures produced by the reference's own Family A/B/C and
block_attn_res tests (tests/golden/make_golden.py): every stored output was
accepted by the reference's assertion (max-abs 1e-3 / 1e-2 / 2e-3 / 1e-4),
and beside it is the reference test's own numpy expectation (`expected`).

CPU: the oracle reproduces every stored output, and it equals the reference's
own expectation to within 1e-6 relative to the largest value (100x tighter
than the reference's tolerances; in practice one f32 ulp).
GPU: the CUDA path reproduces the reference's expectation within the
reference's own tolerances.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
TOL = {"a": 1e-3, "b": 1e-2, "c": 2e-3}  # tests/test_family_{a,b,c}.py


def _load(name, with_expected=False):
    z = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    index = json.loads(bytes(z["index"]).decode())
    out = []
    for i, meta in enumerate(index):
        ins = [z[f"c{i}_in{j}"] for j in range(meta["inputs"])]
        if with_expected:
            out.append((meta, ins, z[f"c{i}_out"], z[f"c{i}_expected"]))
        else:
            out.append((meta, ins, z[f"c{i}_out"]))
    return out


def _cases(family):
    return _load(f"family_{family}")


ALL_WITH_EXPECTED = [(f, c) for f in ("family_a", "family_b", "family_c", "block_attn_res")
                     for c in _load(f, with_expected=True)]


@pytest.mark.parametrize("fam_case", ALL_WITH_EXPECTED, ids=lambda fc: fc[1][0]["name"])
def test_oracle_equals_reference_expectation(fam_case):
    """The stored oracle output against the reference test's own numpy
    expectation for the same inputs: within 1e-6 of the largest |value|."""
    _, (meta, _ins, out, expected) = fam_case
    assert out.shape == expected.shape
    scale = max(1.0, float(np.max(np.abs(expected))))
    assert np.max(np.abs(out.astype(np.float64) - expected.astype(np.float64))) <= 1e-6 * scale


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
@pytest.mark.parametrize("case", _load("family_a", True), ids=lambda c: c[0]["name"])
def test_cuda_family_a_matches_golden(mcb, case):
    meta, ins, _, expected = case
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
@pytest.mark.parametrize("case", _load("family_b", True), ids=lambda c: c[0]["name"])
def test_cuda_family_b_matches_golden(mcb, case):
    meta, ins, _, expected = case
    a, b, bnd, w = _b_args(meta, ins)
    got = mcb.gemm_chain(a, b, w, bnd, bias_mode=meta["bias_mode"], bias_op=meta["bias_op"],
                         act=meta["act"])
    # one launch; the f32 intermediate stays in shared memory (as the
    # reference keeps it in f32, src/fusion_emitter_family_b.cpp:231-383)
    assert mcb.api.last_result.kernel_launches == 1
    assert mcb.api.last_result.route == "simt_chain_fused"
    assert np.max(np.abs(got - expected)) < TOL["b"]


@pytest.mark.gpu
@pytest.mark.parametrize("case", _load("family_c", True), ids=lambda c: c[0]["name"])
def test_cuda_family_c_matches_golden(mcb, case):
    meta, ins, _, expected = case
    q, k, v = _qkv(meta, ins)
    got = mcb.msm(q, k, v, 1.0)
    assert np.max(np.abs(got - expected)) < TOL["c"]


def _tc_case():
    z = np.load(os.path.join(HERE, "golden", "family_c_tc.npz"))
    return z["q_bf16"], z["k_bf16"], z["v_bf16"], float(z["scale"]), z["expected"]


def test_oracle_equals_reference_expectation_tensor_core_size(orc):
    """256x256x128 with the 128^-0.5 scale: the oracle against the reference
    test module's own _attention_ref on the same bf16-representable inputs."""
    qb, kb, vb, scale, expected = _tc_case()
    q, k, v = (orc.bf16_to_f32(b) for b in (qb, kb, vb))
    got = orc.msm(q, k, v, scale)
    assert np.max(np.abs(got - expected)) <= 1e-6


@pytest.mark.gpu
def test_cuda_tcgen05_msm_matches_reference_expectation(mcb, orc):
    """The tcgen05 MSM kernel (bf16 output) against the reference's numpy
    expectation: relative Frobenius error <= 1e-2 (the north-star bf16 bar)
    and the reference Family C max-abs tolerance scaled for a bf16 output."""
    from tests import gpu_util as gu
    qb, kb, vb, scale, expected = _tc_case()
    dev = [gu.to_dev_bf16(b.reshape(1, 1, 256, 128)) for b in (qb, kb, vb)]
    o = mcb.msm(*dev, scale)
    assert mcb.api.last_result.route == "tcgen05_bf16_msm"
    got = gu.from_dev(o)[0, 0]
    assert orc.rel_frobenius(got, expected) < 1e-2
    assert np.max(np.abs(got - expected)) < 1e-2
