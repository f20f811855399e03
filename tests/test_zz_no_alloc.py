"""GPU: the allocation-free strict fused pair matches the regular entry point.

mcb_strict_fused_pair_f32_noalloc_v1 exists for callers that cannot call
cudaMalloc (a framework that owns all device memory through its own pool, a
latency-critical path that must not hit cudaMalloc's implicit device-wide
synchronisation, or code that must not fail for lack of memory mid-run). It
keeps its intermediate panel in a fixed array inside the library instead of
allocating scratch. These tests call it through the C ABI, twice in a row on
each input, and require its output to equal mcb_strict_fused_pair_f32_v1's
bit for bit (the strict path's tolerance). This file is named so that pytest
collects it last; it also passes when run on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from tests import reference_cases as rc

pytestmark = pytest.mark.gpu

CAPACITY_FLOATS = 1 << 21  # the fixed panel array, 8 MiB


def _t(abi, x):
    return abi.make_tensor(x.data_ptr(), "f32", x.shape, x.stride(), x.is_cuda)


def _call(name, e, a, b, d, sync=True):
    import torch
    from matcoredsl_b200 import _abi
    lib = _abi.load()
    rep = _abi.make_report()
    ex = _abi.make_exec(device=torch.cuda.current_device(),
                        stream=torch.cuda.current_stream().cuda_stream,
                        flags=_abi.EXEC_SYNC if sync else 0, report=rep)
    descs = [_t(_abi, x) for x in (e, a, b, d)]
    code = getattr(lib, name)(*[ctypes.byref(t) for t in descs], ctypes.byref(ex))
    return code, rep


def _inputs(m, k, n, p, seed):
    import torch
    rng = np.random.default_rng(seed)
    mk = lambda r, c: torch.from_numpy(rng.uniform(-1, 1, (r, c)).astype(np.float32)).cuda()  # noqa
    return mk(m, k), mk(k, n), mk(n, p)


@pytest.mark.parametrize("shape", [
    (512, 256, 384, 128),
    (3000, 17, 4096, 9),    # all panels exceed the array: several launches
    (5, 3, 1, 4),
    (1, 0, 70, 3),          # K = 0: E = +0 * D
    (7, 4, 0, 5),           # N = 0: E = +0
])
def test_noalloc_matches_regular_entry_twice(mcb, shape):
    import torch
    m, k, n, p = shape
    a, b, d = _inputs(m, k, n, p, seed=sum(shape))
    ref = torch.full((m, p), float("nan"), device="cuda")
    code, _ = _call("mcb_strict_fused_pair_f32_v1", ref, a, b, d)
    assert code == 0
    expected = ref.cpu().numpy()
    for _ in range(2):  # the array keeps the previous call's contents
        out = torch.full((m, p), float("nan"), device="cuda")
        code, rep = _call("mcb_strict_fused_pair_f32_noalloc_v1", out, a, b, d)
        assert code == 0, code
        assert rc.same_bits(out.cpu().numpy(), expected)
        if n > 0:
            assert rep.route.decode() == "strict_f32_simt_pair_fixed_scratch"
    if shape[1:] == (17, 4096, 9):
        assert rep.kernel_launches > 1


def test_noalloc_config1_matches_oracle(mcb, orc):
    import torch
    a = np.random.default_rng(0).uniform(-1, 1, (512, 256)).astype(np.float32)
    b = np.random.default_rng(1).uniform(-1, 1, (256, 384)).astype(np.float32)
    d = np.random.default_rng(2).uniform(-1, 1, (384, 128)).astype(np.float32)
    out = torch.empty(512, 128, device="cuda")
    code, _ = _call("mcb_strict_fused_pair_f32_noalloc_v1", out,
                    *(torch.from_numpy(x).cuda() for x in (a, b, d)))
    assert code == 0
    assert rc.same_bits(out.cpu().numpy(), orc.strict_fused_pair(a, b, d))


def test_noalloc_rejects_panel_larger_than_array(mcb):
    import torch
    from matcoredsl_b200 import _abi
    n = CAPACITY_FLOATS + 1
    a, b, d = torch.zeros(2, 1, device="cuda"), torch.zeros(1, n, device="cuda"), \
        torch.zeros(n, 1, device="cuda")
    out = torch.empty(2, 1, device="cuda")
    code, _ = _call("mcb_strict_fused_pair_f32_noalloc_v1", out, a, b, d)
    assert code == _abi.STATUS_CODE["INSUFFICIENT_WORKSPACE"]
    # exactly at the limit is accepted
    b2, d2 = torch.zeros(1, CAPACITY_FLOATS, device="cuda"), torch.zeros(CAPACITY_FLOATS, 1,
                                                                         device="cuda")
    code, _ = _call("mcb_strict_fused_pair_f32_noalloc_v1", out, a, b2, d2)
    assert code == 0


def test_noalloc_rejects_host_operands(mcb):
    from matcoredsl_b200 import _abi
    lib = _abi.load()
    x = np.ones((2, 2), np.float32)
    y = np.empty((2, 2), np.float32)
    t = [_abi.make_tensor(z.ctypes.data, "f32", z.shape, [2, 1], False) for z in (y, x, x, x)]
    ex = _abi.make_exec()
    code = lib.mcb_strict_fused_pair_f32_noalloc_v1(*[ctypes.byref(z) for z in t], ctypes.byref(ex))
    assert code == _abi.STATUS_CODE["UNSUPPORTED_MEMORY_SPACE"]


def test_noalloc_allocates_nothing(mcb):
    """The property the entry point exists for: after a first call has done
    the per-device set-up, repeated calls (config 1 and the multi-launch
    shape) change neither the device's free memory nor torch's allocator
    statistics."""
    import torch
    cases = []
    for shape in [(512, 256, 384, 128), (3000, 17, 4096, 9)]:
        m, k, n, p = shape
        a, b, d = _inputs(m, k, n, p, seed=5 + sum(shape))
        cases.append((torch.empty(m, p, device="cuda"), a, b, d))
    for out, a, b, d in cases:  # first call: set-up (symbol address lookup)
        assert _call("mcb_strict_fused_pair_f32_noalloc_v1", out, a, b, d)[0] == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    stats0 = torch.cuda.memory_stats()
    for _ in range(3):
        for out, a, b, d in cases:
            assert _call("mcb_strict_fused_pair_f32_noalloc_v1", out, a, b, d, sync=False)[0] == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    stats1 = torch.cuda.memory_stats()
    assert free1 == free0
    for key in ("allocation.all.allocated", "reserved_bytes.all.current",
                "allocated_bytes.all.current"):
        assert stats1.get(key, 0) == stats0.get(key, 0), key
