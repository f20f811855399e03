"""GPU: Family A (GEMM + fused epilogue) against the fp64 oracle.

* bf16 inputs run the tcgen05 kernel. With an f32 output the only error is
  f32 accumulation, so it is held to 1e-5 relative Frobenius error (this
  catches any descriptor/layout mistake); with a bf16 output the north-star
  tolerance of 1e-2 relative Frobenius error applies.
* f32 inputs run the CUDA-core kernel at the reference's own Family A test
  shapes and tolerance (max-abs 1e-3, tests/test_family_a.py).
* BASELINE config 2 (8192x4096x4096, GELU_tanh(X W + b)) at full size, checked
  on a row sample covering every 128-row tile.
"""
import numpy as np
import pytest

from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

REL_F32_OUT = 1e-5
REL_BF16 = 1e-2


def _inputs(m, k, n, seed, wscale=None):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(m, k)).astype(np.float32)
    w = rng.normal(scale=wscale or 1.0 / np.sqrt(k), size=(k, n)).astype(np.float32)
    b = rng.normal(scale=0.02, size=n).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("shape", [(128, 64, 256), (256, 1024, 512), (300, 264, 520),
                                   (1000, 4096, 1032), (128, 8, 8), (129, 16, 264),
                                   (2048, 256, 2560)])
@pytest.mark.parametrize("w_transposed", [False, True])
def test_tcgen05_f32_out_exact_accumulation(mcb, orc, shape, w_transposed):
    import torch
    m, k, n = shape
    x, w, _ = _inputs(m, k, n, seed=m + k + n)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    tx = gu.to_dev_bf16(xh)
    tw = gu.to_dev_bf16(np.ascontiguousarray(wh.T) if w_transposed else wh)
    y = torch.empty(m, n, dtype=torch.float32, device="cuda")
    mcb.gemm_epilogue(tx, tw, out=y, w_transposed=w_transposed)
    r = mcb.api.last_result
    assert r.route == "tcgen05_bf16_gemm_epilogue"
    # M >= 256 runs on SM pairs (256-row tiles), shorter problems on single SMs.
    assert r.tile[0] == (256 if m >= 256 else 128) and r.ctas % (2 if m >= 256 else 1) == 0
    ref = orc.gemm_epilogue(xf, wf)
    assert orc.rel_frobenius(gu.from_dev(y), ref) < REL_F32_OUT


@pytest.mark.parametrize("act", ["none", "relu", "gelu_tanh", "exp", "sigmoid", "tanh"])
@pytest.mark.parametrize("bias_mode,bias_op", [("none", "add"), ("row", "add"), ("full", "add"),
                                               ("full", "rsub"), ("row", "rsub")])
def test_tcgen05_epilogues_bf16_out(mcb, orc, act, bias_mode, bias_op):
    import torch
    m, k, n = 256, 512, 384
    x, w, b = _inputs(m, k, n, seed=7)
    if act == "exp":
        w *= 0.25
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    bias_np = None
    bias_dev = None
    if bias_mode == "row":
        bh, bias_np = gu.bf16_pair(b)
        bias_dev = gu.to_dev_bf16(bh)
    elif bias_mode == "full":
        full = np.random.default_rng(8).normal(scale=0.5, size=(m, n)).astype(np.float32)
        bias_np = full
        bias_dev = gu.to_dev_f32(full)
    y = mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), bias_dev, bias_mode=bias_mode,
                          bias_op=bias_op, act=act, out_dtype="bf16")
    assert mcb.api.last_result.route == "tcgen05_bf16_gemm_epilogue"
    ref = orc.gemm_epilogue(xf, wf, bias_np, bias_mode=bias_mode, bias_op=bias_op, act=act)
    assert orc.rel_frobenius(gu.from_dev(y), ref) < REL_BF16
    assert y.dtype == torch.bfloat16


@pytest.mark.parametrize("act", ["none", "relu", "gelu_tanh", "exp", "sigmoid", "tanh"])
@pytest.mark.parametrize("bias_mode,bias_op", [("none", "add"), ("row", "add"), ("full", "rsub")])
@pytest.mark.parametrize("m", [200, 512])
def test_tcgen05_epilogues_f32_out(mcb, orc, act, bias_mode, bias_op, m):
    """bf16 operands, f32 output: the activations must be the accurate ones
    (the hardware tanh/exp approximations are ~2^-11 relative, far above
    f32), so every activation and bias mode is held to 1e-5 relative
    Frobenius error and to the reference's Family A max-abs bar of 1e-3
    (tests/test_family_a.py). m = 200 runs the single-SM kernel, 512 the
    CTA-pair kernel."""
    import torch
    k, n = 512, 384
    x, w, b = _inputs(m, k, n, seed=11)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w * 2.0)   # pre-activations ~N(0, 4): tanh/GELU saturation regions too
    bias_np = bias_dev = None
    if bias_mode == "row":
        bh, bias_np = gu.bf16_pair(b)
        bias_dev = gu.to_dev_bf16(bh)
    elif bias_mode == "full":
        bias_np = np.random.default_rng(12).normal(scale=0.5, size=(m, n)).astype(np.float32)
        bias_dev = gu.to_dev_f32(bias_np)
    y = torch.empty(m, n, dtype=torch.float32, device="cuda")
    mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), bias_dev, bias_mode=bias_mode,
                      bias_op=bias_op, act=act, out=y)
    r = mcb.api.last_result
    assert r.route == "tcgen05_bf16_gemm_epilogue"
    assert r.tile[0] == (256 if m >= 256 else 128)
    ref = orc.gemm_epilogue(xf, wf, bias_np, bias_mode=bias_mode, bias_op=bias_op, act=act)
    got = gu.from_dev(y)
    assert orc.rel_frobenius(got, ref) < REL_F32_OUT
    assert np.max(np.abs(got - ref) / np.maximum(1.0, np.abs(ref))) < 1e-3


@pytest.mark.parametrize("act", ["gelu_tanh", "exp", "sigmoid", "tanh"])
def test_tcgen05_epilogues_f16_out(mcb, orc, act):
    """f16 output (10 mantissa bits) takes the accurate activations too: the
    error is the f16 rounding alone, under one f16 half-ulp (2^-11) relative
    per element for normal results."""
    import torch
    m, k, n = 512, 512, 384
    x, w, _ = _inputs(m, k, n, seed=13)
    x16 = torch.from_numpy(x).half().cuda()
    w16 = torch.from_numpy(w * 2.0).half().cuda()
    y = torch.empty(m, n, dtype=torch.float16, device="cuda")
    mcb.gemm_epilogue(x16, w16, act=act, out=y)
    assert mcb.api.last_result.route.startswith("tcgen05")
    ref = orc.gemm_epilogue(x16.float().cpu().numpy(), w16.float().cpu().numpy(), act=act)
    got = y.float().cpu().numpy()
    # half an f16 ulp (2^-11 relative for normal results) plus 1e-5 for the
    # f32 accumulation error where the pre-activation cancels near zero
    assert np.all(np.abs(got - ref) <= 2.0 ** -11 * 1.01 * np.abs(ref) + 1e-5)
    assert orc.rel_frobenius(got, ref) < 5e-4


# The reference's Family A GPU tests (tests/test_family_a.py:34-154): f32,
# M=N=64, K=32, max-abs tolerance 1e-3; exp uses inputs scaled by 0.1.
FAMILY_A = [
    ("gemm_relu", "relu", "none", "add", 1.0),
    ("gemm_gelu", "gelu_tanh", "none", "add", 1.0),
    ("gemm_exp", "exp", "none", "add", 0.1),
    ("gemm_add", "none", "full", "add", 1.0),
    ("gemm_add_relu", "relu", "full", "add", 1.0),
    ("bias_minus_gemm", "none", "full", "rsub", 1.0),
]


@pytest.mark.parametrize("case", FAMILY_A, ids=lambda c: c[0])
def test_family_a_f32_reference_shapes(mcb, orc, case):
    name, act, bias_mode, bias_op, scale = case
    m, n, k = (32, 32, 16) if name == "gemm_exp" else (64, 64, 32)
    rng = np.random.default_rng(abs(hash(name)) % 2 ** 32)
    a = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    b = (rng.standard_normal((k, n)) * scale).astype(np.float32)
    bias = rng.standard_normal((m, n)).astype(np.float32) if bias_mode == "full" else None
    y = mcb.gemm_epilogue(a, b, bias, bias_mode=bias_mode, bias_op=bias_op, act=act)
    assert mcb.api.last_result.route == "simt_f32_gemm_epilogue"
    ref = orc.gemm_epilogue(a, b, bias, bias_mode=bias_mode, bias_op=bias_op, act=act)
    assert np.max(np.abs(y - ref)) < 1e-3


@pytest.mark.parametrize("shape,act,bias_mode,bias_op,out_dtype", [
    ((2048, 512, 1536), "gelu_tanh", "row", "add", "f32"),
    ((2000, 300, 1540), "relu", "full", "rsub", "f32"),   # edge tiles, K % 16 != 0
    ((1920, 256, 1408), "exp", "none", "add", "bf16"),
])
def test_f32_large_tile_kernel(mcb, orc, shape, act, bias_mode, bias_op, out_dtype):
    """f32 operands large enough for 128x128 tiles (8x8 per thread): same
    epilogue semantics and the reference's max-abs tolerance (1e-3; bf16
    output at 1e-2 relative Frobenius)."""
    import torch
    m, k, n = shape
    rng = np.random.default_rng(m + k + n)
    scale = 0.05 if act == "exp" else 1.0
    a = (rng.standard_normal((m, k)) * scale).astype(np.float32)
    b = (rng.standard_normal((k, n)) * scale / np.sqrt(k)).astype(np.float32)
    bias = None
    if bias_mode == "row":
        bias = rng.standard_normal(n).astype(np.float32)
    elif bias_mode == "full":
        bias = rng.standard_normal((m, n)).astype(np.float32)
    dev = lambda t: None if t is None else torch.from_numpy(t).cuda()  # noqa: E731
    y = mcb.gemm_epilogue(dev(a), dev(b), dev(bias), bias_mode=bias_mode, bias_op=bias_op,
                          act=act, out_dtype=out_dtype)
    r = mcb.api.last_result
    assert r.route == "simt_f32_gemm_epilogue" and r.tile[:2] == (128, 128)
    ref = orc.gemm_epilogue(a, b, bias, bias_mode=bias_mode, bias_op=bias_op, act=act)
    got = gu.from_dev(y)
    if out_dtype == "f32":
        assert np.max(np.abs(got - ref)) < 1e-3
    else:
        assert orc.rel_frobenius(got, ref) < 1e-2


def test_host_operands_e2e_path(mcb, orc):
    """Host-resident bf16 operands are staged through the C ABI and match."""
    ml = pytest.importorskip("ml_dtypes")
    m, k, n = 256, 256, 256
    x, w, b = _inputs(m, k, n, seed=3)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    bh, bf = gu.bf16_pair(b)
    y = mcb.gemm_epilogue(xh.view(ml.bfloat16), wh.view(ml.bfloat16), bh.view(ml.bfloat16),
                          act="gelu_tanh", out_dtype="bf16")
    r = mcb.api.last_result
    assert r.route == "tcgen05_bf16_gemm_epilogue" and r.h2d_bytes == (m * k + k * n + n) * 2
    assert r.d2h_bytes == m * n * 2
    ref = orc.gemm_epilogue(xf, wf, bf, bias_mode="row", act="gelu_tanh")
    assert orc.rel_frobenius(y.astype(np.float32), ref) < REL_BF16


def config2_inputs():
    """X ~ N(0,1), W ~ N(0,1/4096), b ~ N(0,0.02), seed 10 (X, W, b)."""
    rng = np.random.default_rng(10)
    x = rng.standard_normal((8192, 4096), dtype=np.float32)
    w = (rng.standard_normal((4096, 4096), dtype=np.float32) * np.float32(1 / 64))
    b = (rng.standard_normal(4096, dtype=np.float32) * np.float32(0.02))
    return x, w, b


def test_config2_full_size_sampled(mcb, orc):
    x, w, b = config2_inputs()
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    bh, bf = gu.bf16_pair(b)
    y = mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), gu.to_dev_bf16(bh),
                          act="gelu_tanh", out_dtype="bf16")
    assert mcb.api.last_result.route == "tcgen05_bf16_gemm_epilogue"
    rows = gu.sample_rows(8192)
    ref = orc.gemm_epilogue(xf, wf, bf, bias_mode="row", act="gelu_tanh", rows=rows)
    got = gu.from_dev(y)[rows]
    assert orc.rel_frobenius(got, ref) < REL_BF16
    assert mcb.device_status(0) == 0


@pytest.mark.parametrize("act,bias_mode,bias_op", [("relu", "none", "add"), ("exp", "none", "add"),
                                                   ("none", "full", "add"),
                                                   ("gelu_tanh", "full", "rsub"),
                                                   ("relu", "row", "add")])
def test_family_b_chain_tcgen05(mcb, orc, act, bias_mode, bias_op):
    """E = glue(A B) W in one tcgen05 kernel: the intermediate stays in TMEM
    (f32) and shared memory (bf16 operand of the second GEMM), never in HBM."""
    import torch
    m, k, n1, n2 = 256, 256, 256, 192
    rng = np.random.default_rng(21)
    a = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.5)
    b = rng.standard_normal((k, n1), dtype=np.float32) / np.float32(np.sqrt(k))
    w = rng.standard_normal((n1, n2), dtype=np.float32) / np.float32(np.sqrt(n1))
    (ah, af), (bh, bf), (wh, wf) = gu.bf16_pair(a), gu.bf16_pair(b), gu.bf16_pair(w)
    bnd_np = bnd_dev = None
    if bias_mode == "full":
        bnd_np = rng.standard_normal((m, n1), dtype=np.float32) * np.float32(0.3)
        bnd_dev = gu.to_dev_f32(bnd_np)
    elif bias_mode == "row":
        bnd_np = rng.standard_normal(n1, dtype=np.float32) * np.float32(0.3)
        bnd_dev = gu.to_dev_f32(bnd_np)
    e = mcb.gemm_chain(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh), gu.to_dev_bf16(wh), bnd_dev,
                       bias_mode=bias_mode, bias_op=bias_op, act=act, out_dtype="f32")
    r = mcb.api.last_result
    assert r.route == "tcgen05_bf16_chain_fused" and r.kernel_launches == 1
    mid = orc.gemm_epilogue(af, bf, bnd_np, bias_mode=bias_mode, bias_op=bias_op, act=act)
    ref = orc.gemm_epilogue(mid.astype(np.float32), wf)
    assert orc.rel_frobenius(gu.from_dev(e), ref) < REL_BF16
    assert e.dtype == torch.float32


@pytest.mark.parametrize("shape,out_dtype,act,bias_mode,fused", [
    ((200, 72, 200, 24), "f32", "gelu_tanh", "row", True),     # ragged M, K, N1; N2 < 64
    ((130, 520, 264, 136), "bf16", "exp", "none", True),        # N1 chunks 128+128+8
    ((256, 512, 256, 448), "f32", "tanh", "row", True),         # two E tiles (256 + 192)
    ((8192, 256, 512, 64), "bf16", "relu", "full", True),       # K <= 256, many rows
    ((1024, 1024, 1024, 256), "bf16", "relu", "full", False),   # two GEMMs (faster here)
    ((256, 4096, 512, 64), "f32", "sigmoid", "none", False),
])
def test_family_b_fused_shapes(mcb, orc, shape, out_dtype, act, bias_mode, fused):
    """The chain at ragged and larger shapes on both tensor-core routes: in
    the fused kernel values past N1 and M are masked to 0 before the second
    GEMM, so they contribute nothing."""
    import torch
    m, k, n1, n2 = shape
    rng = np.random.default_rng(m + k + n1 + n2)
    a = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.5)
    b = rng.standard_normal((k, n1), dtype=np.float32) / np.float32(np.sqrt(k))
    w = rng.standard_normal((n1, n2), dtype=np.float32) / np.float32(np.sqrt(n1))
    if act == "exp":
        b *= np.float32(0.5)
    (ah, af), (bh, bf), (wh, wf) = gu.bf16_pair(a), gu.bf16_pair(b), gu.bf16_pair(w)
    bnd_np = bnd_dev = None
    if bias_mode == "full":
        bnd_np = rng.standard_normal((m, n1), dtype=np.float32) * np.float32(0.3)
        bnd_dev = gu.to_dev_bf16(gu.bf16_pair(bnd_np)[0])
        bnd_np = gu.bf16_pair(bnd_np)[1]
    elif bias_mode == "row":
        bnd_np = rng.standard_normal(n1, dtype=np.float32) * np.float32(0.3)
        bnd_dev = gu.to_dev_f32(bnd_np)
    for _ in range(2):
        e = mcb.gemm_chain(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh), gu.to_dev_bf16(wh), bnd_dev,
                           bias_mode=bias_mode, act=act, out_dtype=out_dtype)
        r = mcb.api.last_result
        if fused:
            assert r.route == "tcgen05_bf16_chain_fused" and r.kernel_launches == 1
        else:
            assert r.route == "chain:tcgen05_bf16_gemm_epilogue" and r.kernel_launches == 2
    rows = gu.sample_rows(m, seed=4) if m > 2048 else np.arange(m)
    bnd_rows = bnd_np[rows] if bias_mode == "full" else bnd_np
    mid = orc.gemm_epilogue(af[rows], bf, bnd_rows, bias_mode=bias_mode, act=act)
    ref = orc.gemm_epilogue(mid.astype(np.float32), wf)
    assert orc.rel_frobenius(gu.from_dev(e)[rows], ref) < REL_BF16
    assert e.dtype == (torch.bfloat16 if out_dtype == "bf16" else torch.float32)
    assert mcb.device_status(0) == 0


def test_family_b_large_takes_two_launches(mcb, orc):
    """A above 2^22 elements: two tcgen05 GEMMs through scratch (faster than
    the fused kernel, which re-reads A for every 128 intermediate columns)."""
    m, k, n1, n2 = 4096, 2048, 256, 64
    rng = np.random.default_rng(6)
    a = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.5)
    b = rng.standard_normal((k, n1), dtype=np.float32) / np.float32(np.sqrt(k))
    w = rng.standard_normal((n1, n2), dtype=np.float32) / np.float32(np.sqrt(n1))
    (ah, af), (bh, bf), (wh, wf) = gu.bf16_pair(a), gu.bf16_pair(b), gu.bf16_pair(w)
    e = mcb.gemm_chain(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh), gu.to_dev_bf16(wh), act="relu",
                       out_dtype="f32")
    r = mcb.api.last_result
    assert r.route == "chain:tcgen05_bf16_gemm_epilogue" and r.kernel_launches == 2
    rows = gu.sample_rows(m, seed=2)
    ref = orc.gemm_epilogue(orc.gemm_epilogue(af[rows], bf, act="relu").astype(np.float32), wf)
    assert orc.rel_frobenius(gu.from_dev(e)[rows], ref) < REL_BF16


def test_family_b_unaligned_takes_two_launches(mcb, orc):
    """K not a multiple of 8 (no TMA rows): the two-GEMM route through scratch."""
    m, k, n1, n2 = 256, 60, 128, 64
    rng = np.random.default_rng(5)
    a, b, w = (rng.standard_normal(sh, dtype=np.float32) * np.float32(0.2)
               for sh in ((m, k), (k, n1), (n1, n2)))
    (ah, af), (bh, bf), (wh, wf) = gu.bf16_pair(a), gu.bf16_pair(b), gu.bf16_pair(w)
    e = mcb.gemm_chain(gu.to_dev_bf16(ah), gu.to_dev_bf16(bh), gu.to_dev_bf16(wh), act="relu",
                       out_dtype="f32")
    assert mcb.api.last_result.kernel_launches == 2
    ref = orc.gemm_epilogue(orc.gemm_epilogue(af, bf, act="relu").astype(np.float32), wf)
    assert orc.rel_frobenius(gu.from_dev(e), ref) < REL_BF16


# ---- stream-K route of the CTA-pair kernel (opt-in: MCB_GEMM_STREAM_K=1) --------
# Shapes whose whole tiles would leave clusters idle split the K-block ranges
# of tiles over all clusters; a tile's parts are summed in f32 by whichever
# CTA arrives last. Checked at the f32-output bar (1e-5) against the fp64
# oracle, twice in a row (the arrival counters must be back at zero).
@pytest.fixture
def stream_k(monkeypatch):
    monkeypatch.setenv("MCB_GEMM_STREAM_K", "1")  # read by the library at every launch

@pytest.mark.parametrize("shape,w_transposed", [
    ((1024, 4096, 4096), False),   # config 2 rows per GPU at 8 GPUs: 64 tiles
    ((2048, 4096, 4096), False),   # 4 GPUs: 128 tiles, all stream-K
    ((4096, 2048, 4096), False),   # 2 GPUs: whole-tile waves, then stream-K
    ((1000, 4096, 1032), True),    # ragged M and N: 20 tiles in chains of one
    ((512, 8192, 768), False),     # long K: 6 tiles, 12 clusters
    ((256, 4096, 256), False),     # one tile, split over two clusters
    ((4096, 1000, 4096), False),   # K not a multiple of 64: the last K block is ragged
])
def test_stream_k_f32_out(mcb, orc, stream_k, shape, w_transposed):
    import torch
    m, k, n = shape
    x, w, b = _inputs(m, k, n, seed=m + n)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    tx = gu.to_dev_bf16(xh)
    tw = gu.to_dev_bf16(np.ascontiguousarray(wh.T) if w_transposed else wh)
    bh, bf = gu.bf16_pair(b)
    rows = gu.sample_rows(m, seed=3)
    ref = orc.gemm_epilogue(xf[rows], wf, bf, bias_mode="row", act="gelu_tanh")
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        mcb.gemm_epilogue(tx, tw, gu.to_dev_bf16(bh), bias_mode="row", act="gelu_tanh", out=y,
                          w_transposed=w_transposed)
        r = mcb.api.last_result
        assert r.route == "tcgen05_bf16_gemm_epilogue" and r.stream_k
        got = gu.from_dev(y)
        assert not np.isnan(got).any()
        assert orc.rel_frobenius(got[rows], ref) < REL_F32_OUT
    assert mcb.device_status(0) == 0


def test_stream_k_bf16_out_matches_whole_tile_run(mcb, orc, stream_k):
    """bf16 output at config 2's 1024-row shard: stream-K against the oracle
    at the bf16 bar, and the headline 8192-row shape keeps whole tiles."""
    import torch
    m, k, n = 1024, 4096, 4096
    x, w, b = _inputs(m, k, n, seed=10)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    bh, bf = gu.bf16_pair(b)
    y = mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), gu.to_dev_bf16(bh),
                          bias_mode="row", act="gelu_tanh")
    assert mcb.api.last_result.stream_k
    ref = orc.gemm_epilogue(xf, wf, bf, bias_mode="row", act="gelu_tanh")
    assert orc.rel_frobenius(gu.from_dev(y), ref) < REL_BF16
    big = torch.zeros(8192, 4096, dtype=torch.bfloat16, device="cuda")
    mcb.gemm_epilogue(big, gu.to_dev_bf16(wh), gu.to_dev_bf16(bh), bias_mode="row",
                      act="gelu_tanh")
    assert not mcb.api.last_result.stream_k  # 512 tiles: 6.9 waves, whole tiles


def test_stream_k_on_two_streams(mcb, orc, stream_k):
    """Stream-K launches from two streams share the device workspace: the
    library orders them, so interleaved calls stay exact."""
    import torch
    m, k, n = 1024, 2048, 4096
    cases = []
    for seed in (21, 22):
        x, w, _ = _inputs(m, k, n, seed=seed)
        xh, xf = gu.bf16_pair(x)
        wh, wf = gu.bf16_pair(w)
        cases.append((gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), orc.gemm_epilogue(xf[:64], wf)))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty(m, n, dtype=torch.float32, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    for _ in range(5):
        for i in (0, 1):
            with torch.cuda.stream(streams[i]):
                mcb.gemm_epilogue(cases[i][0], cases[i][1], out=outs[i])
                assert mcb.api.last_result.stream_k
    torch.cuda.synchronize()
    for i in (0, 1):
        assert orc.rel_frobenius(gu.from_dev(outs[i])[:64], cases[i][2]) < REL_F32_OUT


def test_stream_k_default_policy(mcb, orc, monkeypatch):
    """By default stream-K splits only a last wave that fills at most 70% of
    the 74 clusters: 1024, 2048 and 8192 rows (64, 54 and 68 tiles in the
    last wave) keep whole tiles, 4096 rows (34) splits them, and the result
    matches the whole-tile run (MCB_GEMM_STREAM_K=0) to f32 rounding."""
    import torch
    monkeypatch.delenv("MCB_GEMM_STREAM_K", raising=False)
    w = torch.zeros(4096, 4096, dtype=torch.bfloat16, device="cuda")
    for rows in (1024, 2048, 8192):
        mcb.gemm_epilogue(torch.zeros(rows, 4096, dtype=torch.bfloat16, device="cuda"), w)
        assert not mcb.api.last_result.stream_k
    x, wn, _ = _inputs(4096, 4096, 4096, seed=77)
    tx, tw = gu.to_dev_bf16(gu.bf16_pair(x)[0]), gu.to_dev_bf16(gu.bf16_pair(wn)[0])
    y = mcb.gemm_epilogue(tx, tw, out=torch.empty(4096, 4096, device="cuda"))
    assert mcb.api.last_result.stream_k
    monkeypatch.setenv("MCB_GEMM_STREAM_K", "0")
    y0 = mcb.gemm_epilogue(tx, tw, out=torch.empty(4096, 4096, device="cuda"))
    assert not mcb.api.last_result.stream_k
    assert orc.rel_frobenius(gu.from_dev(y), gu.from_dev(y0).astype(np.float64)) < 1e-6
    assert mcb.device_status(0) == 0


@pytest.mark.parametrize("out_dtype", ["bf16", "f16"])
@pytest.mark.parametrize("rows", [1000, 4096])  # whole tiles; a stream-K last wave
def test_tma_stored_output_into_a_strided_view(mcb, orc, out_dtype, rows):
    """16-bit outputs of the CTA-pair kernel go out through shared memory and
    TMA stores whose tensor map has the view's row stride: a column slice of
    a wider buffer gets exactly its own columns (ragged N and M included),
    and the padding columns keep their bytes."""
    import torch
    m, k, n, pad = rows, 512, 1000, 24
    x, w, b = _inputs(m, k, n, seed=rows + len(out_dtype))
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    bh, bf = gu.bf16_pair(b)
    tdt = torch.bfloat16 if out_dtype == "bf16" else torch.float16
    big = torch.full((m, n + pad), -3.0, dtype=tdt, device="cuda")
    view = big[:, :n]
    assert view.stride(0) == n + pad
    xd = gu.to_dev_bf16(xh)
    if out_dtype == "f16":
        xd, wd, bd = (torch.from_numpy(v).cuda().to(torch.float16) for v in (xf, wf, bf))
    else:
        wd, bd = gu.to_dev_bf16(wh), gu.to_dev_bf16(bh)
    mcb.gemm_epilogue(xd, wd, bd, bias_mode="row", act="gelu_tanh", out=view)
    assert mcb.api.last_result.route == f"tcgen05_{out_dtype}_gemm_epilogue"
    ref = orc.gemm_epilogue(xf, wf, bf, bias_mode="row", act="gelu_tanh")
    assert orc.rel_frobenius(view.float().cpu().numpy(), ref) < REL_BF16
    assert torch.all(big[:, n:] == -3.0)
    assert mcb.device_status(0) == 0
