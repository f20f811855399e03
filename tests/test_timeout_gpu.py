"""GPU: a bounded device wait that runs out returns an error instead of hanging.

Every pipeline wait in the tensor-core kernels gives up after a bounded number
of clock64 cycles, records a bit in the per-device status word and aborts its
CTA (the device-side counterpart of the reference adapter's poison domain,
compiler/lib/runtime/closed_cuda_candidate_v1.cpp:86-120). The self-test
entry point runs one GEMM tile whose loads are never issued with a short
limit (10^6 cycles, about half a millisecond): the kernel must return, the
call must report MCB_STATUS_DEVICE_TIMEOUT with the "producer data never
arrived" bit, and the context must stay usable for the next call. No fault,
trap or hang is involved: the wait on a flag nothing sets simply runs out.
"""
import numpy as np
import pytest

from matcoredsl_b200 import _abi
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

TIMEOUT_FULL = 1 << 0
TIMEOUT_PEER = 1 << 5


def test_stalled_pipeline_returns_timeout_and_context_survives(mcb, orc):
    import torch
    lib = _abi.load()
    mcb.device_status(0, clear=True)
    for _ in range(2):  # twice: the second run starts from a cleared word again
        code = lib.mcb_device_timeout_selftest_v1(0, 1_000_000)
        assert code == _abi.STATUS_CODE["DEVICE_TIMEOUT"], _abi.STATUS.get(code, code)
        word = mcb.device_status(0, clear=True)
        assert word & TIMEOUT_FULL
        assert mcb.device_status(0) == 0
    # the same device then runs a normal call correctly
    rng = np.random.default_rng(3)
    x = rng.standard_normal((256, 512)).astype(np.float32)
    w = (rng.standard_normal((512, 384)) / 16).astype(np.float32)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    y = torch.empty(256, 384, dtype=torch.float32, device="cuda")
    mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), out=y, act="gelu_tanh")
    assert mcb.api.last_result.route == "tcgen05_bf16_gemm_epilogue"
    assert orc.rel_frobenius(gu.from_dev(y), orc.gemm_epilogue(xf, wf, act="gelu_tanh")) < 1e-5
    assert mcb.device_status(0) == 0


def test_selftest_rejects_out_of_range_limits(mcb):
    lib = _abi.load()
    assert lib.mcb_device_timeout_selftest_v1(0, 10) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    assert lib.mcb_device_timeout_selftest_v1(0, 10 ** 10) == _abi.STATUS_CODE["INVALID_ARGUMENT"]


def test_stream_k_owner_wait_for_a_flag_nothing_sets_returns_timeout(mcb, orc):
    """The one wait on another CTA cluster: a stream-K owner's producer waits
    for the flag of its tile's tail part. In the self-test the tails never
    raise it, so every owner's wait must run out (10^6 cycles), the kernel
    must return with the "stream-K partial never arrived" bit set, and a
    stream-K call afterwards must be correct."""
    import torch
    lib = _abi.load()
    mcb.device_status(0, clear=True)
    for _ in range(2):
        code = lib.mcb_device_peer_timeout_selftest_v1(0, 1_000_000)
        assert code == _abi.STATUS_CODE["DEVICE_TIMEOUT"], _abi.STATUS.get(code, code)
        word = mcb.device_status(0, clear=True)
        assert word & TIMEOUT_PEER
        assert mcb.device_status(0) == 0
    assert lib.mcb_device_peer_timeout_selftest_v1(0, 10) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    # a real stream-K launch (two tiles over four clusters) on the same device
    rng = np.random.default_rng(4)
    x = rng.standard_normal((256, 4096)).astype(np.float32)
    w = (rng.standard_normal((4096, 512)) / 64).astype(np.float32)
    xh, xf = gu.bf16_pair(x)
    wh, wf = gu.bf16_pair(w)
    y = torch.empty(256, 512, dtype=torch.float32, device="cuda")
    mcb.gemm_epilogue(gu.to_dev_bf16(xh), gu.to_dev_bf16(wh), out=y)
    assert mcb.api.last_result.stream_k
    assert orc.rel_frobenius(gu.from_dev(y), orc.gemm_epilogue(xf, wf)) < 1e-5
    assert mcb.device_status(0) == 0
