"""GPU: general Family A epilogue chains (mcb_gemm_epilogue_chain_v1), the
chains FusionMlirEmitter::emitFamilyA accepts (src/fusion_emitter_family_a.cpp:
149-220): any sequence of unary ops and binary ops against exact-shape [M,N]
boundaries, with the running value on either side. Compared with the fp64
oracle (oracle.gemm_epilogue_chain), NaN positions included."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

UNARY = ["relu", "exp", "log", "tanh", "sqrt", "neg", "abs", "sin", "cos", "rsqrt", "sigmoid",
         "gelu_tanh"]


def _close(got, ref, tol):
    got = np.asarray(got, np.float64)
    nan_g, nan_r = np.isnan(got), np.isnan(ref)
    assert np.array_equal(nan_g, nan_r)
    inf_r = np.isinf(ref)
    assert np.array_equal(got[inf_r], ref[inf_r])
    ok = ~(nan_r | inf_r)
    g, r = got[ok], ref[ok]
    assert np.linalg.norm(g - r) <= tol * max(np.linalg.norm(r), 1e-30)


def _inputs(m, k, n, dt, seed, scale=0.3):
    import torch
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    w = (rng.standard_normal((k, n)) * scale).astype(np.float32)
    td = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dt]
    xd, wd = torch.from_numpy(x).cuda().to(td), torch.from_numpy(w).cuda().to(td)
    # the oracle sees exactly the rounded operands
    return xd, wd, xd.float().cpu().numpy(), wd.float().cpu().numpy()


@pytest.mark.parametrize("op", UNARY)
@pytest.mark.parametrize("dt,route", [("bf16", "tcgen05_bf16_gemm_epilogue"),
                                      ("f32", "simt_f32_gemm_epilogue")])
def test_each_unary_op(mcb, orc, op, dt, route):
    """Every unary kind alone, f32 output (log / sqrt / rsqrt of negative
    values give NaN in the same places as the oracle). Tolerance 1e-3: log,
    sqrt and rsqrt of sums that cancel to near zero amplify the GEMM's
    summation-order differences (a wrong op is off by O(1))."""
    xd, wd, x, w = _inputs(256, 128, 264, dt, 11)
    y = mcb.gemm_epilogue(xd, wd, chain=[op], out_dtype="f32")
    assert mcb.api.last_result.route == route
    _close(y.cpu().numpy(), orc.gemm_epilogue_chain(x, w, [op]), 1e-3)


def test_reference_activation_chain_f16(mcb, orc):
    """The reference's 'chaos' epilogue sigmoid(tanh(gelu(relu(A @ B))))
    (tests/benchmark_absurd_activation.py:35-38), f16 in and out."""
    xd, wd, x, w = _inputs(512, 256, 384, "f16", 12)
    chain = ["relu", "gelu", "tanh", "sigmoid"]
    y = mcb.gemm_epilogue(xd, wd, chain=chain)
    assert mcb.api.last_result.route == "tcgen05_f16_gemm_epilogue"
    _close(y.float().cpu().numpy(), orc.gemm_epilogue_chain(x, w, chain), 2e-3)


def test_reference_rsqrt_f16(mcb, orc):
    """rsqrt(A @ B) (tests/benchmark_rsqrt_sin_softmax.py:47-49): NaN where the
    product is negative, as in the reference's math.rsqrt."""
    xd, wd, x, w = _inputs(256, 64, 256, "f16", 13)
    y = mcb.gemm_epilogue(xd, wd, chain=["rsqrt"])
    _close(y.float().cpu().numpy(), orc.gemm_epilogue_chain(x, w, ["rsqrt"]), 2e-3)


@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("m", [384, 300, 100])
def test_binary_chain_two_boundaries(mcb, orc, m, out):
    """relu -> * c -> min(d) -> d - v -> / c with two boundaries (f32 and
    bf16), ragged M on the pair and single-SM kernels."""
    import torch
    n, k = 264, 192
    xd, wd, x, w = _inputs(m, k, n, "bf16", m)
    rng = np.random.default_rng(m + 1)
    c = torch.from_numpy((rng.random((m, n)) + 0.5).astype(np.float32)).cuda()
    d = torch.from_numpy(rng.standard_normal((m, n)).astype(np.float32)).cuda().to(torch.bfloat16)
    chain = ["relu", ("mul", c), ("min", d), ("sub", d, "right"), ("div", c)]
    y = mcb.gemm_epilogue(xd, wd, chain=chain, out_dtype=out)
    assert mcb.api.last_result.route == "tcgen05_bf16_gemm_epilogue"
    ref_chain = ["relu", ("mul", c.cpu().numpy()), ("min", d.float().cpu().numpy()),
                 ("sub", d.float().cpu().numpy(), "right"), ("div", c.cpu().numpy())]
    tol = 1e-2 if out == "bf16" else 1e-4
    _close(y.float().cpu().numpy(), orc.gemm_epilogue_chain(x, w, ref_chain), tol)


def test_strided_boundary_and_max(mcb, orc):
    """A row-strided boundary view and max with the value on the right."""
    import torch
    m, k, n = 256, 128, 256
    xd, wd, x, w = _inputs(m, k, n, "bf16", 21)
    big = torch.randn(m, n + 8, device="cuda")
    b = big[:, :n]
    chain = [("max", b, "right"), "neg", ("add", b)]
    y = mcb.gemm_epilogue(xd, wd, chain=chain, out_dtype="f32")
    bn = b.cpu().numpy()
    _close(y.cpu().numpy(),
           orc.gemm_epilogue_chain(x, w, [("max", bn, "right"), "neg", ("add", bn)]), 1e-4)


def test_host_operands_chain(mcb, orc):
    """numpy operands and boundary, staged by the library."""
    rng = np.random.default_rng(22)
    x = rng.standard_normal((300, 64)).astype(np.float32)
    w = rng.standard_normal((64, 40)).astype(np.float32)
    b = rng.standard_normal((300, 40)).astype(np.float32)
    chain = ["tanh", ("mul", b), "abs", "sqrt"]
    y = mcb.gemm_epilogue(x, w, chain=chain)
    _close(y, orc.gemm_epilogue_chain(x, w, chain), 1e-3)


def test_chain_argument_errors(mcb):
    import ctypes

    import torch
    from matcoredsl_b200 import _abi
    xd, wd, _, _ = _inputs(64, 64, 64, "bf16", 23)
    with pytest.raises(ValueError):
        mcb.gemm_epilogue(xd, wd, chain=["relu"] * 9)
    with pytest.raises(mcb.McbError):   # boundary shape must be exactly [M, N]
        mcb.gemm_epilogue(xd, wd, chain=[("add", torch.zeros(64, 32, device="cuda"))])
    with pytest.raises(mcb.McbError):   # boundary dtype
        mcb.gemm_epilogue(xd, wd, chain=[("add", torch.zeros(64, 64, dtype=torch.int32,
                                                            device="cuda"))])
    # unknown kind and an out-of-range boundary index, straight through the C ABI
    lib = _abi.load()
    y = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    from matcoredsl_b200.api import _desc, _exec
    ty, tx, tw = (_desc(t, "t")[0] for t in (y, xd, wd))
    ops = (_abi.EpilogueOp * 1)()
    ex = _exec(True, -1, 0, _abi.make_report(), None)
    for kind, bnd in ((13, 0), (99, 0), (_abi.EW["add"], 0)):
        ops[0].kind, ops[0].boundary = kind, bnd
        code = lib.mcb_gemm_epilogue_chain_v1(ctypes.byref(ty), ctypes.byref(tx),
                                              ctypes.byref(tw), None, 0, ops, 1, 0,
                                              ctypes.byref(ex))
        assert _abi.STATUS.get(code) == "INVALID_ARGUMENT"
