"""GPU: f16 operands, the reference's float16 matmul signature (f16 x f16 ->
f16 or f32, src/mlir_engine.cpp:140-145), on tcgen05 (kind::f16 with the f16
operand format) and on the CUDA-core kernel for unaligned shapes. Checked at
the tolerances of the reference's own f16 tests
(tests/test_subtile_correctness.py, tests/test_multiwarp_correctness.py,
tests/test_graph_mode.py) and, tighter, against the fp64 oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rel_frobenius(got, ref):
    got = np.asarray(got, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


@pytest.mark.parametrize("n", [16, 32, 48, 64, 128, 256, 384, 448, 512, 640, 768])
def test_reference_f16_matmul_sizes(mcb, orc, n):
    """The reference's square f16 cases: sub-tile sizes 16..256 (atol < 1) and
    the multi-warp sizes 384..768 (atol < max(1, 0.005 N)), C = A @ B in f16."""
    import torch
    rng = np.random.default_rng(n)
    a = rng.standard_normal((n, n)).astype(np.float16)
    b = rng.standard_normal((n, n)).astype(np.float16)
    c = mcb.gemm_epilogue(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    assert c.dtype == torch.float16
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    got = c.float().cpu().numpy()
    expected = (a.astype(np.float32) @ b.astype(np.float32)).astype(np.float16)
    tol = 1.0 if n <= 256 else max(1.0, n * 0.005)
    assert np.max(np.abs(got - expected.astype(np.float32))) < tol
    ref = orc.gemm_epilogue(a.astype(np.float32), b.astype(np.float32))
    assert _rel_frobenius(got, ref) < 1e-3


@pytest.mark.parametrize("out", ["f16", "f32"])
@pytest.mark.parametrize("shape", [(256, 512, 384), (100, 136, 264), (1000, 72, 520)])
def test_f16_epilogue(mcb, orc, shape, out):
    """Row bias (f16) + GELU-tanh on the CTA-pair (M >= 256) and single-SM
    kernels, ragged M, f16 or f32 output."""
    import torch
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    x = (rng.standard_normal((m, k)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((k, n)) * 0.5).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16)
    dev = [torch.from_numpy(t).cuda() for t in (x, w, bias)]
    y = mcb.gemm_epilogue(*dev, act="gelu_tanh", out_dtype=out)
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    assert y.dtype == (torch.float16 if out == "f16" else torch.float32)
    ref = orc.gemm_epilogue(x.astype(np.float32), w.astype(np.float32), bias.astype(np.float32),
                            bias_mode="row", act="gelu_tanh")
    assert _rel_frobenius(y.float().cpu().numpy(), ref) < 2e-3


def test_f16_full_bias_rsub_transposed_w(mcb, orc):
    """Exact-shape f16 boundary, reverse subtract, W given as W^T [N, K]."""
    import torch
    m, k, n = 384, 256, 320
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((m, k)) * 0.5).astype(np.float16)
    wt = (rng.standard_normal((n, k)) * 0.5).astype(np.float16)
    bnd = rng.standard_normal((m, n)).astype(np.float16)
    dev = [torch.from_numpy(t).cuda() for t in (x, wt, bnd)]
    y = mcb.gemm_epilogue(*dev, bias_op="rsub", act="relu", w_transposed=True)
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    ref = orc.gemm_epilogue(x.astype(np.float32), np.ascontiguousarray(wt.T).astype(np.float32),
                            bnd.astype(np.float32), bias_mode="full", bias_op="rsub", act="relu")
    assert _rel_frobenius(y.float().cpu().numpy(), ref) < 2e-3


def test_f16_unaligned_cuda_cores(mcb, orc):
    """K = 53 (rows not 16-byte aligned): the CUDA-core kernel reads and
    writes f16."""
    import torch
    rng = np.random.default_rng(4)
    x = rng.standard_normal((37, 53)).astype(np.float16)
    w = rng.standard_normal((53, 29)).astype(np.float16)
    bias = rng.standard_normal(29).astype(np.float16)
    y = mcb.gemm_epilogue(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                          torch.from_numpy(bias).cuda(), act="tanh")
    assert mcb.api.last_result.route.startswith("simt")
    assert y.dtype == torch.float16
    ref = orc.gemm_epilogue(x.astype(np.float32), w.astype(np.float32), bias.astype(np.float32),
                            bias_mode="row", act="tanh")
    assert _rel_frobenius(y.float().cpu().numpy(), ref) < 2e-3


def test_f16_host_operands(mcb, orc):
    """numpy float16 operands staged by the library."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((300, 128)).astype(np.float16)
    w = rng.standard_normal((128, 96)).astype(np.float16)
    y = mcb.gemm_epilogue(x, w)
    assert y.dtype == np.float16
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    ref = orc.gemm_epilogue(x.astype(np.float32), w.astype(np.float32))
    assert _rel_frobenius(y, ref) < 1e-3


def test_f16_graph_plan(mcb, orc):
    """The reference's graph-mode case: a shape-locked f16 plan captured once
    and replayed (tests/test_graph_mode.py:17-52); a moved buffer is rejected
    (:55-78)."""
    import torch
    n = 64
    rng = np.random.default_rng(6)
    a = rng.standard_normal((n, n)).astype(np.float16)
    b = rng.standard_normal((n, n)).astype(np.float16)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.zeros((n, n), dtype=torch.float16, device="cuda")
    plan = mcb.Plan("gemm_epilogue", dc, da, db, None, graph=True)
    expected = (a.astype(np.float32) @ b.astype(np.float32)).astype(np.float16).astype(np.float32)
    for _ in range(2):
        plan.execute(dc, da, db, None)
        torch.cuda.synchronize()
        assert np.max(np.abs(dc.float().cpu().numpy() - expected)) < 1.0
        dc.zero_()
    with pytest.raises(mcb.McbError):
        plan.execute(dc, da.clone(), db, None)
    plan.close()


def test_reference_staging_case(mcb):
    """The reference's staging case: f16 [16,16] @ [16,8] from
    default_rng(42/43), compared at atol 1e-2 + rtol 1e-1
    (tests/test_gpu_staging.py)."""
    lhs = np.random.default_rng(42).standard_normal((16, 16), dtype=np.float32).astype(np.float16)
    rhs = np.random.default_rng(43).standard_normal((16, 8), dtype=np.float32).astype(np.float16)
    out = np.zeros((16, 8), dtype=np.float16)
    mcb.gemm_epilogue(lhs, rhs, out=out)
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    expected = lhs.astype(np.float32) @ rhs.astype(np.float32)
    np.testing.assert_allclose(out.astype(np.float32), expected, atol=1e-2, rtol=1e-1)


def test_reference_graph_minimal(mcb):
    """The reference's minimal graph case (tests/test_graph_minimal.py): a
    normal plan, then a graph plan captured and replayed, N = 16 f16."""
    import torch
    n = 16
    rng = np.random.default_rng(16)
    a = rng.standard_normal((n, n)).astype(np.float16)
    b = rng.standard_normal((n, n)).astype(np.float16)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.zeros((n, n), dtype=torch.float16, device="cuda")
    expected = (a.astype(np.float32) @ b.astype(np.float32)).astype(np.float16).astype(np.float32)
    for graph in (False, True, True):
        dc.zero_()
        plan = mcb.Plan("gemm_epilogue", dc, da, db, None, graph=graph)
        plan.execute(dc, da, db, None)
        if graph:
            dc.zero_()
            plan.execute(dc, da, db, None)   # replay
        torch.cuda.synchronize()
        assert np.max(np.abs(dc.float().cpu().numpy() - expected)) < 1.0
        plan.close()


def test_f16_mixed_dtypes_rejected(mcb):
    """Mixed operand types and a bf16 output for f16 inputs are not signatures
    of the reference's matmul."""
    import torch
    a16 = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    abf = torch.zeros((64, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(mcb.McbError):
        mcb.gemm_epilogue(a16, abf)
    with pytest.raises(mcb.McbError):
        mcb.gemm_epilogue(a16, a16, out=torch.empty((64, 64), dtype=torch.bfloat16,
                                                     device="cuda"))
