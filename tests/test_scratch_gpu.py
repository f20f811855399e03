"""GPU: device scratch of calls that need it (the strict pair's binary32 C,
the int8 B^T copy for unaligned B rows). Without a caller workspace it comes
from the library's stream-ordered pool and the call stays asynchronous;
calls queued on two streams at once must each see their own scratch. With a
workspace the same results come out of the caller's memory."""
import numpy as np
import pytest

from tests import reference_cases as rc

pytestmark = pytest.mark.gpu


def _pair_inputs(seed, m=320, k=96, n=200, p=72):
    rng = np.random.default_rng(seed)
    return (rng.uniform(-1, 1, (m, k)).astype(np.float32),
            rng.uniform(-1, 1, (k, n)).astype(np.float32),
            rng.uniform(-1, 1, (n, p)).astype(np.float32))


def test_strict_pair_concurrent_streams(mcb, orc):
    import torch
    cases = [_pair_inputs(s) for s in range(6)]
    dev = [[torch.from_numpy(x).cuda() for x in c] for c in cases]
    outs = [torch.empty(c[0].shape[0], c[2].shape[1], device="cuda") for c in cases]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for i, (a, b, d) in enumerate(dev):
        with torch.cuda.stream(streams[i % 2]):
            for _ in range(3):  # repeated calls reuse the pool's memory
                mcb.strict_fused_pair(a, b, d, out=outs[i])
    assert mcb.api.last_result.route == "strict_f32_simt_pair_two_pass"
    torch.cuda.synchronize()
    for (a, b, d), e in zip(cases, outs):
        assert rc.same_bits(e.cpu().numpy(), orc.strict_fused_pair(a, b, d))


def test_strict_pair_caller_workspace(mcb, orc):
    import torch
    a, b, d = _pair_inputs(11)
    ws = torch.full((a.shape[0] * b.shape[1],), float("nan"), device="cuda")
    e = mcb.strict_fused_pair(*(torch.from_numpy(x).cuda() for x in (a, b, d)), workspace=ws)
    assert mcb.api.last_result.route == "strict_f32_simt_pair_two_pass"
    assert rc.same_bits(e.cpu().numpy(), orc.strict_fused_pair(a, b, d))
    # C went through the workspace: it now holds A*B in binary32.
    assert rc.same_bits(ws.view(a.shape[0], b.shape[1]).cpu().numpy(), orc.strict_gemm(a, b))


@pytest.mark.parametrize("use_ws", [False, True])
def test_i8_transposed_b_scratch(mcb, orc, use_ws):
    import torch
    m, k, n, ldb = 300, 144, 336, 344  # B rows of 344 bytes: not 16-byte aligned
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    cases, outs = [], []
    for s in range(4):
        rng = np.random.default_rng(100 + s)
        a = rng.integers(-128, 128, (m, k), dtype=np.int8)
        b_big = rng.integers(-128, 128, (k, ldb), dtype=np.int8)
        cases.append((a, b_big))
    keep = []  # operands and workspaces stay alive until the streams are drained
    torch.cuda.synchronize()
    for s, (a, b_big) in enumerate(cases):
        with torch.cuda.stream(streams[s % 2]):
            ws = torch.empty(n * k, dtype=torch.int8, device="cuda") if use_ws else None
            da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b_big).cuda()
            keep.append((ws, da, db))
            outs.append(mcb.gemm_i8_i32(da, db[:, :n], workspace=ws))
        assert mcb.api.last_result.kernel_launches == 2
    torch.cuda.synchronize()
    for (a, b_big), c in zip(cases, outs):
        assert np.array_equal(c.cpu().numpy(),
                              orc.gemm_i8_i32(a, np.ascontiguousarray(b_big[:, :n])))


def test_strict_pair_pool_scratch_captured_in_graph(mcb, orc):
    """A call whose scratch comes from the pool can be captured into a CUDA
    graph (the allocation becomes a graph memory node) and replayed."""
    import torch
    a, b, d = _pair_inputs(21)
    da, db, dd = (torch.from_numpy(x).cuda() for x in (a, b, d))
    e = torch.empty(a.shape[0], d.shape[1], device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        mcb.strict_fused_pair(da, db, dd, out=e)  # pool created outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        mcb.strict_fused_pair(da, db, dd, out=e)
    assert mcb.api.last_result.route == "strict_f32_simt_pair_two_pass"
    e.zero_()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert rc.same_bits(e.cpu().numpy(), orc.strict_fused_pair(a, b, d))
    del g


def test_host_threads_on_their_own_streams(mcb, orc):
    """Calls from several host threads at once (ctypes releases the GIL), each
    on its own stream: strict pairs with pool scratch and GEMMs with an
    epilogue. Every result must match what a lone call gives."""
    import threading

    import torch
    from tests import gpu_util as gu
    rng = np.random.default_rng(31)
    x = rng.standard_normal((512, 256), dtype=np.float32)
    w = rng.standard_normal((256, 384), dtype=np.float32) / np.float32(16)
    (xh, _), (wh, _) = gu.bf16_pair(x), gu.bf16_pair(w)
    dx, dw = gu.to_dev_bf16(xh), gu.to_dev_bf16(wh)
    pairs = [[torch.from_numpy(t).cuda() for t in _pair_inputs(40 + i)] for i in range(4)]
    ref_y = mcb.gemm_epilogue(dx, dw, act="gelu_tanh").float()
    ref_e = [mcb.strict_fused_pair(*p) for p in pairs]
    torch.cuda.synchronize()
    errors = []

    def worker(i):
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                for _ in range(20):
                    e = mcb.strict_fused_pair(*pairs[i])
                    y = mcb.gemm_epilogue(dx, dw, act="gelu_tanh")
                s.synchronize()
            if not torch.equal(e, ref_e[i]) or not torch.equal(y.float(), ref_y):
                errors.append(f"thread {i}: result differs")
        except Exception as exc:  # noqa: BLE001 - reported below
            errors.append(f"thread {i}: {exc!r}")

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in threads), "a worker thread did not finish"
    assert not errors, errors
