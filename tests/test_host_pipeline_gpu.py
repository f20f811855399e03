"""GPU: host-operand row pipeline of mcb_gemm_epilogue_v1.

With operands in host memory (and no MCB_EXEC_TIME), the library moves X, a
full bias and Y in row chunks, overlapping uploads, GEMM launches and
downloads on separate streams. These tests check that the chunked path gives
the same bytes as the single-launch path (MCB_EXEC_TIME keeps the serial
staging), matches the fp64 oracle, reports the bytes it moved, and writes only
the output's own columns of a padded host output.
"""
import numpy as np
import pytest

from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

ml = pytest.importorskip("ml_dtypes")


def _bf16_host(bits):
    return np.ascontiguousarray(bits).view(ml.bfloat16)


def test_bf16_full_bias_padded_output(mcb, orc):
    from matcoredsl_b200 import _abi
    m, k, n = 2600, 4096, 264  # 8 KiB rows of X: 1024-row chunks, 3 launches
    rng = np.random.default_rng(5)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32) / np.float32(64)
    bias = rng.standard_normal((m, n), dtype=np.float32) * np.float32(0.3)
    (xh, xf), (wh, wf) = gu.bf16_pair(x), gu.bf16_pair(w)
    big = np.full((m, n + 24), -7.0, np.float32)
    out = big[:, :n]
    mcb.gemm_epilogue(_bf16_host(xh), _bf16_host(wh), bias, bias_mode="full", bias_op="rsub",
                      act="tanh", out=out)
    r = mcb.api.last_result
    assert r.route == "tcgen05_bf16_gemm_epilogue" and r.kernel_launches == 3
    assert r.h2d_bytes == m * k * 2 + k * n * 2 + m * n * 4
    assert r.d2h_bytes == m * n * 4
    assert np.all(big[:, n:] == -7.0), "padding of the host output was overwritten"
    ref = orc.gemm_epilogue(xf, wf, bias, bias_mode="full", bias_op="rsub", act="tanh")
    assert orc.rel_frobenius(out, ref) < 1e-5
    # The serial staging path (timed calls, one launch) agrees to f32
    # rounding: its 22 tiles and the chunks' 8 each are split differently by
    # stream-K, so the two sum the K blocks of some tiles in a different
    # order. The same call twice gives the same bytes.
    serial = np.empty((m, n), np.float32)
    mcb.gemm_epilogue(_bf16_host(xh), _bf16_host(wh), bias, bias_mode="full", bias_op="rsub",
                      act="tanh", out=serial, flags=_abi.EXEC_TIME)
    assert mcb.api.last_result.kernel_launches == 1
    assert orc.rel_frobenius(serial, out.astype(np.float64)) < 1e-5
    again = np.empty((m, n), np.float32)
    mcb.gemm_epilogue(_bf16_host(xh), _bf16_host(wh), bias, bias_mode="full", bias_op="rsub",
                      act="tanh", out=again)
    np.testing.assert_array_equal(out, again)


def test_bf16_row_bias_bf16_output_many_chunks(mcb, orc):
    m, k, n = 4100, 2048, 512  # 4 KiB rows: 2048-row chunks, 3 launches (last one 4 rows)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32) / np.float32(np.sqrt(k))
    b = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    (xh, xf), (wh, wf), (bh, bf) = gu.bf16_pair(x), gu.bf16_pair(w), gu.bf16_pair(b)
    y = mcb.gemm_epilogue(_bf16_host(xh), _bf16_host(wh), _bf16_host(bh), act="gelu_tanh",
                          out_dtype="bf16")
    r = mcb.api.last_result
    assert r.kernel_launches == 3 and r.d2h_bytes == m * n * 2
    rows = gu.sample_rows(m)
    ref = orc.gemm_epilogue(xf, wf, bf, bias_mode="row", act="gelu_tanh", rows=rows)
    assert orc.rel_frobenius(y.astype(np.float32)[rows], ref) < 1e-2


def test_f32_cuda_core_path_pipelined(mcb, orc):
    m, k, n = 4200, 1024, 96  # f32 X rows of 4 KiB: 2048-row chunks on the CUDA-core kernel
    rng = np.random.default_rng(7)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.standard_normal((k, n), dtype=np.float32) / np.float32(32)
    b = rng.standard_normal(n, dtype=np.float32)
    y = mcb.gemm_epilogue(x, w, b, bias_mode="row", act="relu")
    r = mcb.api.last_result
    assert r.route == "simt_f32_gemm_epilogue" and r.kernel_launches == 3
    ref = orc.gemm_epilogue(x, w, b, bias_mode="row", act="relu")
    assert np.max(np.abs(y - ref)) < 1e-3
