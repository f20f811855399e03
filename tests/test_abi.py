"""CPU: the C-ABI library loads, exports every declared entry point, and its
host-only logic behaves; no kernel is launched here."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "mcb.h")).read()
    return sorted(set(re.findall(r"MCB_API\s+[\w\s\*]+?\b(mcb_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared_symbols()
    for required in ("mcb_strict_fused_pair_f32_v1", "mcb_strict_gemm_f32_v1",
                     "mcb_gemm_epilogue_v1", "mcb_msm_v1", "mcb_gemm_fp8_blockscaled_v1",
                     "mcb_attn_block_region_v1", "mcb_device_alloc"):
        assert required in names


def test_library_exports_every_declared_symbol(mcb):
    from matcoredsl_b200 import _abi
    lib = ctypes.CDLL(_abi.LIB_PATH)
    missing = [n for n in _declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes mirror declares exactly the header's set
    assert sorted(_abi.SIGNATURES) == _declared_symbols()


def test_abi_struct_layouts_match_c_compiler(mcb, tmp_path):
    """The ctypes mirror and a C compiler agree on every struct's size and offsets."""
    import shutil
    import subprocess
    from matcoredsl_b200 import _abi
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"mcb_tensor": _abi.Tensor, "mcb_exec": _abi.Exec, "mcb_report": _abi.Report,
               "mcb_epilogue": _abi.Epilogue, "mcb_buffer": _abi.Buffer,
               "mcb_fp8_tile_config": _abi.Fp8TileConfig, "mcb_shard": _abi.Shard,
               "mcb_plan_desc": _abi.PlanDesc, "mcb_comm_id": _abi.CommId,
               "mcb_epilogue_op": _abi.EpilogueOp, "mcb_ipc_handle": _abi.IpcHandle}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "mcb.h"', "int main(void){"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                 check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(out[cname]) == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(out[f"{cname}.{f}"]) == getattr(py, f).offset, (cname, f)


def test_status_messages(mcb):
    lib = mcb.load()
    assert lib.mcb_status_message(0) == b"ok"
    assert b"sm_100" in lib.mcb_status_message(42)
    assert lib.mcb_status_message(9999) == b"unknown status"


def test_fp8_tile_policy_matches_reference_table(mcb):
    """Restates src/fp8_wgmma.cpp:10-24,61-109 expectations for a set of shapes."""
    lib = mcb.load()
    legal = lib.mcb_fp8_is_legal_shape_v1
    assert legal(64, 8, 32) == 1 and legal(128, 256, 64) == 1
    assert legal(64, 264, 32) == 0 and legal(63, 8, 32) == 0 and legal(64, 8, 31) == 0
    assert legal(0, 8, 32) == 0 and legal(64, 12, 32) == 0
    cfg = lib.mcb_fp8_tile_config_v1
    c = cfg(256, 384, 128)
    assert (c.m_tile, c.n_tile, c.k_tile, c.use_tma) == (128, 128, 32, 0)  # N>256: illegal shape
    c = cfg(128, 256, 64)
    assert (c.m_tile, c.n_tile, c.k_tile, c.use_tma) == (128, 128, 32, 1)
    c = cfg(64, 96, 32)
    assert (c.m_tile, c.n_tile, c.use_tma) == (64, 96, 1)
    c = cfg(64, 100, 32)  # largest legal divisor of 100 that is a multiple of 8: none -> 104
    assert c.n_tile == 104
    c = cfg(64, 40, 32)
    assert c.n_tile == 40
    c = cfg(0, 40, 32)
    assert (c.m_tile, c.n_tile, c.k_tile, c.use_tma) == (64, 128, 32, 0)
    c = cfg(32, 8, 32)  # M not a multiple of 64: tiles chosen, TMA off
    assert (c.m_tile, c.n_tile, c.use_tma) == (64, 8, 0)


def test_invalid_descriptors_rejected_without_gpu(mcb):
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    a = np.zeros((2, 3), np.float32)
    t = _abi.make_tensor(a.ctypes.data, "f32", a.shape, [3, 1], False)
    bad = _abi.make_tensor(a.ctypes.data, "f32", a.shape, [3, 1], False)
    bad.abi_version = 7
    ex = _abi.make_exec()
    assert lib.mcb_strict_gemm_f32_v1(ctypes.byref(t), ctypes.byref(bad), ctypes.byref(t),
                                      ctypes.byref(ex)) == _abi.STATUS_CODE["ABI_MISMATCH"]
    col = _abi.make_tensor(a.ctypes.data, "f32", a.shape, [1, 2], False)  # column-major
    assert lib.mcb_strict_gemm_f32_v1(ctypes.byref(t), ctypes.byref(col), ctypes.byref(t),
                                      ctypes.byref(ex)) == _abi.STATUS_CODE["UNSUPPORTED_LAYOUT"]
    b = np.zeros((4, 2), np.float32)
    tb = _abi.make_tensor(b.ctypes.data, "f32", b.shape, [2, 1], False)
    c = np.zeros((2, 2), np.float32)
    tc = _abi.make_tensor(c.ctypes.data, "f32", c.shape, [2, 1], False)
    assert lib.mcb_strict_gemm_f32_v1(ctypes.byref(tc), ctypes.byref(t), ctypes.byref(tb),
                                      ctypes.byref(ex)) == _abi.STATUS_CODE["SHAPE_MISMATCH"]
    # the output may not overlap an input
    assert lib.mcb_strict_gemm_f32_v1(ctypes.byref(t), ctypes.byref(t), ctypes.byref(tb),
                                      ctypes.byref(ex)) in (_abi.STATUS_CODE["ALIAS_VIOLATION"],
                                                            _abi.STATUS_CODE["SHAPE_MISMATCH"])


def test_compute_without_gpu_fails_loudly(mcb):
    """With no sm_100 device every compute entry point refuses; none computes on the CPU."""
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(mcb.McbError) as e:
        mcb.strict_gemm(np.ones((2, 2), np.float32), np.ones((2, 2), np.float32))
    assert e.value.name == "CANDIDATE_UNAVAILABLE"


def test_stale_buffer_handle_rejected(mcb):
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    h = _abi.Buffer()
    h.ptr, h.size_bytes, h.alloc_id, h.device = 0x1000, 16, 12345, 0
    assert lib.mcb_device_is_valid(h) == 0
    assert lib.mcb_device_free(h) == _abi.STATUS_CODE["STALE_HANDLE"]
    buf = ctypes.create_string_buffer(16)
    assert lib.mcb_device_upload_async(h, buf, 16, None) == _abi.STATUS_CODE["STALE_HANDLE"]
    assert lib.mcb_device_download_async(buf, h, 16, None) == _abi.STATUS_CODE["STALE_HANDLE"]


def test_comm_arguments_checked_without_gpu(mcb):
    """The all-gather entry points validate their arguments before touching
    NCCL or a device."""
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    bad = _abi.STATUS_CODE["INVALID_ARGUMENT"]
    cid = _abi.CommId()
    out = ctypes.c_void_p()
    assert lib.mcb_comm_unique_id_v1(None) == bad
    assert lib.mcb_comm_init_v1(ctypes.byref(cid), 0, 0, 0, ctypes.byref(out)) == bad  # world 0
    assert lib.mcb_comm_init_v1(ctypes.byref(cid), 2, 2, 0, ctypes.byref(out)) == bad  # rank >= world
    assert lib.mcb_comm_init_v1(ctypes.byref(cid), 2, 0, -1, ctypes.byref(out)) == bad  # device
    assert lib.mcb_comm_init_v1(None, 2, 0, 0, ctypes.byref(out)) == bad
    assert lib.mcb_allgather_v1(None, 0x1000, 0x2000, 16, None) == bad
    assert lib.mcb_reduce_scatter_v1(None, 0x1000, 0x2000, 16, _abi.DTYPE["bf16"], None) == bad
    assert lib.mcb_comm_destroy_v1(None) == 0


def test_peer_exchange_arguments_checked_without_gpu(mcb):
    """The two-GPU exchange entry points validate their arguments first."""
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    bad = _abi.STATUS_CODE["INVALID_ARGUMENT"]
    out = ctypes.c_void_p()
    h = _abi.IpcHandle()
    assert lib.mcb_peer_exchange_create_v1(-1, 16, ctypes.byref(out), ctypes.byref(h)) == bad
    assert lib.mcb_peer_exchange_create_v1(0, 0, ctypes.byref(out), ctypes.byref(h)) == bad
    assert lib.mcb_peer_exchange_create_v1(0, 16, None, ctypes.byref(h)) == bad
    assert lib.mcb_peer_exchange_connect_v1(None, ctypes.byref(h)) == bad
    assert lib.mcb_peer_exchange_destroy_v1(None) == 0
    a = np.zeros((1, 2, 8), np.uint16)
    t = _abi.make_tensor(a.ctypes.data, "bf16", a.shape, [16, 8, 1], False)
    w = np.zeros((8, 8), np.uint16)
    tw = _abi.make_tensor(w.ctypes.data, "bf16", w.shape, [8, 1], False)
    y = np.zeros((1, 8), np.uint16)
    ty = _abi.make_tensor(y.ctypes.data, "bf16", y.shape, [8, 1], False)
    ex = _abi.make_exec()
    assert lib.mcb_attn_block_heads_pair_v1(ctypes.byref(ty), ctypes.byref(t), ctypes.byref(tw),
                                            ctypes.byref(tw), ctypes.byref(tw), ctypes.byref(tw),
                                            1, 1e-6, 0, None, ctypes.byref(ex)) == bad


def test_attn_heads_arguments_checked_without_gpu(mcb):
    """The head-sharded block and residual + RMSNorm reject bad shapes and
    arguments before touching a device."""
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    b, s, d, dh = 1, 8, 16, 8
    x = np.zeros((b, s, d), np.uint16)
    w = np.zeros((d, dh), np.uint16)
    wo = np.zeros((dh, d), np.uint16)
    p = np.zeros((b, s, d), np.uint16)
    t = lambda a, st: _abi.make_tensor(a.ctypes.data, "bf16", a.shape, st, False)  # noqa: E731
    tx, tw, two, tp = t(x, [s * d, d, 1]), t(w, [dh, 1]), t(wo, [d, 1]), t(p, [s * d, d, 1])
    ex = _abi.make_exec()
    call = lambda heads, wq=tw, wout=two: lib.mcb_attn_block_heads_v1(  # noqa: E731
        ctypes.byref(tp), ctypes.byref(tx), ctypes.byref(wq), ctypes.byref(tw), ctypes.byref(tw),
        ctypes.byref(wout), heads, ctypes.byref(ex))
    assert call(3) == _abi.STATUS_CODE["INVALID_ARGUMENT"]      # Dh % heads != 0
    assert call(0) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    assert call(2, wout=tw) == _abi.STATUS_CODE["SHAPE_MISMATCH"]  # Wo not [Dh, D]
    assert lib.mcb_attn_block_heads_workspace_bytes_v1(1, 8, 8) == 4 * 256
    y = np.zeros((b, s, d), np.uint16)
    ty = t(y, [s * d, d, 1])
    assert lib.mcb_residual_rmsnorm_v1(ctypes.byref(ty), ctypes.byref(tx), ctypes.byref(tp),
                                       -1.0, ctypes.byref(ex)) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    assert lib.mcb_residual_rmsnorm_v1(ctypes.byref(ty), ctypes.byref(tx), ctypes.byref(tw),
                                       1e-6, ctypes.byref(ex)) in (
        _abi.STATUS_CODE["SHAPE_MISMATCH"], _abi.STATUS_CODE["INVALID_SHAPE"])
    assert lib.mcb_residual_rmsnorm_v1(ctypes.byref(tx), ctypes.byref(tx), ctypes.byref(tp),
                                       1e-6, ctypes.byref(ex)) == _abi.STATUS_CODE["ALIAS_VIOLATION"]


def test_epilogue_chain_encoding(mcb):
    """Host side of mcb_gemm_epilogue_chain_v1: op codes, value side, one
    boundary slot per distinct tensor, and the argument limits (no GPU)."""
    from matcoredsl_b200 import _abi
    from matcoredsl_b200.api import _epilogue_chain
    b0, b1 = np.zeros((4, 4), np.float32), np.ones((4, 4), np.float32)
    ops, bnds = _epilogue_chain(["relu", ("mul", b0), ("sub", b1, "right"), ("max", b0), "rsqrt"])
    assert [o.kind for o in ops] == [1, 34, 33, 37, 10]
    assert [o.value_pos for o in ops] == [0, 0, 1, 0, 0]
    assert [o.boundary for o in ops[1:4]] == [0, 1, 0]
    assert len(bnds) == 2 and bnds[0] is b0 and bnds[1] is b1
    assert ctypes.sizeof(_abi.EpilogueOp) == 16
    with pytest.raises(ValueError):
        _epilogue_chain([])
    with pytest.raises(ValueError):
        _epilogue_chain(["relu"] * (_abi.EPILOGUE_MAX_OPS + 1))
    with pytest.raises(ValueError):
        _epilogue_chain([("add", None)])
    with pytest.raises(ValueError):
        _epilogue_chain([("add", np.zeros(1)) for _ in range(5)])
    with pytest.raises(KeyError):
        _epilogue_chain(["softmax"])


def test_plan_descriptor_base_size_and_chain_extension(mcb):
    """A descriptor built with the first layout (struct_size up to `reserved`)
    is still accepted; the chain op needs the extension and 1..8 ops. No GPU
    here, so accepted descriptors end at CANDIDATE_UNAVAILABLE."""
    from matcoredsl_b200 import _abi
    lib = mcb.load()
    base = _abi.PlanDesc.num_ops.offset

    def desc(op, size, n_tensors, num_ops=0, num_bnd=0):
        d = _abi.PlanDesc()
        d.abi_version, d.struct_size, d.op = _abi.ABI_VERSION, size, op
        d.num_tensors, d.num_ops, d.num_boundaries = n_tensors, num_ops, num_bnd
        for i in range(n_tensors):
            d.tensors[i].abi_version = _abi.ABI_VERSION
            d.tensors[i].struct_size = ctypes.sizeof(_abi.Tensor)
            d.tensors[i].dtype = 1
        return d

    h = ctypes.c_void_p()
    code = lambda d: lib.mcb_plan_create_v1(ctypes.byref(d), ctypes.byref(h))  # noqa: E731
    unavailable = _abi.STATUS_CODE["CANDIDATE_UNAVAILABLE"]
    full = ctypes.sizeof(_abi.PlanDesc)
    assert code(desc(_abi.PLAN_OPS["strict_gemm"], base, 3)) == unavailable
    assert code(desc(_abi.PLAN_OPS["strict_gemm"], base - 8, 3)) == _abi.STATUS_CODE["ABI_MISMATCH"]
    chain = _abi.PLAN_OPS["gemm_epilogue_chain"]
    assert code(desc(chain, base, 5, 2, 2)) == _abi.STATUS_CODE["ABI_MISMATCH"]
    assert code(desc(chain, full, 5, 0, 2)) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    assert code(desc(chain, full, 5, 9, 2)) == _abi.STATUS_CODE["INVALID_ARGUMENT"]
    assert code(desc(chain, full, 4, 2, 2)) == _abi.STATUS_CODE["INVALID_ARGUMENT"]  # 3 + 2 slots
    assert code(desc(chain, full, 5, 2, 2)) == unavailable
