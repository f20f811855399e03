"""ctypes mirror of include/mcb.h (the library's C ABI).

This module only loads ``libmcb.so`` and declares its entry points; it has no
compute of its own and no fallback: if the library is missing or does not
export a declared symbol, loading fails loudly.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmcb.so")
ABI_VERSION = 1
MAX_RANK = 4

# status codes (include/mcb.h)
STATUS = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "ABI_MISMATCH", 3: "UNSUPPORTED_DTYPE",
    4: "UNSUPPORTED_RANK", 5: "INVALID_SHAPE", 6: "UNSUPPORTED_LAYOUT",
    7: "UNSUPPORTED_MEMORY_SPACE", 8: "MIXED_MEMORY_SPACES", 9: "OUTPUT_NOT_MUTABLE",
    11: "SHAPE_MISMATCH", 12: "ALIAS_VIOLATION", 15: "ARITHMETIC_OVERFLOW",
    16: "INVALID_ALIGNMENT", 17: "INSUFFICIENT_WORKSPACE", 18: "UNAVAILABLE_VARIANT",
    40: "ALLOCATION_FAILURE", 41: "CANDIDATE_FAILURE", 42: "CANDIDATE_UNAVAILABLE",
    43: "DEVICE_TIMEOUT", 44: "STALE_HANDLE",
}
STATUS_CODE = {v: k for k, v in STATUS.items()}

DTYPE = {"f32": 1, "f64": 2, "bf16": 3, "i8": 4, "i32": 5, "f16": 6, "e4m3": 7, "e5m2": 8}
MEM_HOST, MEM_DEVICE = 1, 2
EXEC_SYNC, EXEC_TIME = 1, 2
BIAS_MODE = {"none": 0, "row": 1, "full": 2}
BIAS_OP = {"add": 0, "rsub": 1}
ACT = {"none": 0, "relu": 1, "gelu_tanh": 2, "exp": 3, "sigmoid": 4, "tanh": 5}
GEMM_W_TRANSPOSED = 1


class Tensor(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("struct_size", ctypes.c_uint32),
        ("data", ctypes.c_void_p), ("dtype", ctypes.c_uint32), ("rank", ctypes.c_uint32),
        ("dims", ctypes.c_int64 * MAX_RANK), ("strides", ctypes.c_int64 * MAX_RANK),
        ("memory_space", ctypes.c_uint32), ("reserved0", ctypes.c_uint32),
        ("reserved", ctypes.c_uint64 * 2),
    ]


class Report(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("struct_size", ctypes.c_uint32),
        ("route", ctypes.c_char * 48), ("kernel_launches", ctypes.c_int32),
        ("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32), ("tile_k", ctypes.c_int32),
        ("stages", ctypes.c_int32), ("ctas", ctypes.c_int32),
        ("kernel_ms", ctypes.c_float), ("h2d_ms", ctypes.c_float), ("d2h_ms", ctypes.c_float),
        ("h2d_bytes", ctypes.c_uint64), ("d2h_bytes", ctypes.c_uint64),
        ("device_status", ctypes.c_uint32), ("route_flags", ctypes.c_uint32),
    ]


class Exec(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("struct_size", ctypes.c_uint32),
        ("device", ctypes.c_int32), ("flags", ctypes.c_uint32),
        ("stream", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64), ("report", ctypes.POINTER(Report)),
        ("reserved", ctypes.c_uint64 * 2),
    ]


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("struct_size", ctypes.c_uint32),
        ("bias_mode", ctypes.c_uint32), ("bias_op", ctypes.c_uint32),
        ("activation", ctypes.c_uint32), ("reserved0", ctypes.c_uint32),
        ("reserved", ctypes.c_uint64 * 2),
    ]


class Buffer(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_uint64), ("size_bytes", ctypes.c_uint64), ("alloc_id", ctypes.c_uint64),
        ("device", ctypes.c_int32), ("reserved0", ctypes.c_uint32),
    ]


class Shard(ctypes.Structure):
    _fields_ = [("begin", ctypes.c_int64), ("count", ctypes.c_int64),
                ("kv_begin", ctypes.c_int64), ("kv_count", ctypes.c_int64)]


SHARD_ROWS, SHARD_UNITS, SHARD_TOKENS = 0, 1, 2


class Fp8TileConfig(ctypes.Structure):
    _fields_ = [("m_tile", ctypes.c_int32), ("n_tile", ctypes.c_int32),
                ("k_tile", ctypes.c_int32), ("use_tma", ctypes.c_int32)]


PLAN_MAX_TENSORS = 8
PLAN_OPS = {"strict_pair": 1, "strict_gemm": 2, "gemm_epilogue": 3, "gemm_chain": 4, "msm": 5,
            "fp8_gemm": 6, "attn_block": 7, "gemm_i8_i32": 8, "gemm_epilogue_chain": 9}


class EpilogueOp(ctypes.Structure):
    """mcb_epilogue_op: one link of a Family A epilogue chain."""
    _fields_ = [("kind", ctypes.c_uint32), ("value_pos", ctypes.c_uint32),
                ("boundary", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class PlanDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32), ("struct_size", ctypes.c_uint32),
        ("op", ctypes.c_uint32), ("graph_mode", ctypes.c_uint32), ("device", ctypes.c_int32),
        ("num_tensors", ctypes.c_uint32), ("tensors", Tensor * PLAN_MAX_TENSORS),
        ("epilogue", Epilogue), ("gemm_flags", ctypes.c_uint32), ("reserved0", ctypes.c_uint32),
        ("scale", ctypes.c_double), ("block", ctypes.c_int64), ("heads", ctypes.c_int64),
        ("eps", ctypes.c_float), ("reserved1", ctypes.c_uint32),
        ("a_zero_point", ctypes.c_int32), ("b_zero_point", ctypes.c_int32),
        ("reserved", ctypes.c_uint64),
        # chain extension (MCB_PLAN_GEMM_EPILOGUE_CHAIN)
        ("num_ops", ctypes.c_uint32), ("num_boundaries", ctypes.c_uint32),
        ("ops", EpilogueOp * 8),
    ]


# MCB_EW_* codes (unary < 32, binary >= 32).
EW = {"relu": 1, "exp": 2, "log": 3, "tanh": 4, "sqrt": 5, "neg": 6, "abs": 7, "sin": 8,
      "cos": 9, "rsqrt": 10, "sigmoid": 11, "gelu_tanh": 12, "gelu": 12,
      "add": 32, "sub": 33, "mul": 34, "div": 35, "min": 36, "max": 37}
EPILOGUE_MAX_OPS = 8
EPILOGUE_MAX_BOUNDARIES = 4

_P = ctypes.POINTER
_T = _P(Tensor)
_E = _P(Exec)
# name -> (restype, argtypes); every function include/mcb.h declares.
class CommId(ctypes.Structure):
    """mcb_comm_id: an NCCL unique id (128 opaque bytes)."""
    _fields_ = [("internal", ctypes.c_uint8 * 128)]  # raw bytes (c_char would stop at NUL)


class IpcHandle(ctypes.Structure):
    """mcb_ipc_handle: a CUDA IPC memory handle (64 opaque bytes)."""
    _fields_ = [("internal", ctypes.c_uint8 * 64)]


SIGNATURES = {
    "mcb_abi_version": (ctypes.c_uint32, []),
    "mcb_status_message": (ctypes.c_char_p, [ctypes.c_int32]),
    "mcb_device_status": (ctypes.c_int32, [ctypes.c_int32, _P(ctypes.c_uint32), ctypes.c_int32]),
    "mcb_device_timeout_selftest_v1": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_uint64]),
    "mcb_device_peer_timeout_selftest_v1": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_uint64]),
    # test support (host-side fault injection); exercised from C in tests/adapter/
    "mcb_test_set_runtime_hooks_v1": (ctypes.c_int32, [ctypes.c_void_p]),
    "mcb_candidate_available": (ctypes.c_int32, [ctypes.c_int32]),
    "mcb_strict_gemm_f32_v1": (ctypes.c_int32, [_T, _T, _T, _E]),
    "mcb_strict_fused_pair_f32_v1": (ctypes.c_int32, [_T, _T, _T, _T, _E]),
    "mcb_strict_fused_pair_f32_noalloc_v1": (ctypes.c_int32, [_T, _T, _T, _T, _E]),
    "mcb_gemm_epilogue_v1": (ctypes.c_int32, [_T, _T, _T, _T, _P(Epilogue), ctypes.c_uint32, _E]),
    "mcb_gemm_epilogue_chain_v1": (ctypes.c_int32, [_T, _T, _T, _T, ctypes.c_uint32,
                                                    _P(EpilogueOp), ctypes.c_uint32,
                                                    ctypes.c_uint32, _E]),
    "mcb_gemm_chain_v1": (ctypes.c_int32, [_T, _T, _T, _T, _P(Epilogue), _T, _E]),
    "mcb_gemm_i8_i32_v1": (ctypes.c_int32, [_T, _T, _T, _E]),
    "mcb_gemm_i8_i32_zp_v1": (ctypes.c_int32, [_T, _T, _T, ctypes.c_int32, ctypes.c_int32, _E]),
    "mcb_gemm_bf16_f32_fma_v1": (ctypes.c_int32, [_T, _T, _T, _E]),
    "mcb_msm_v1": (ctypes.c_int32, [_T, _T, _T, _T, ctypes.c_double, _E]),
    "mcb_fp8_quantize_blockwise_v1": (ctypes.c_int32, [_T, _T, _T, ctypes.c_int64, _E]),
    "mcb_gemm_fp8_blockscaled_v1": (ctypes.c_int32, [_T, _T, _T, _T, _T, ctypes.c_int64, _E]),
    "mcb_fp8_is_legal_shape_v1": (ctypes.c_int32, [ctypes.c_int64] * 3),
    "mcb_fp8_tile_config_v1": (Fp8TileConfig, [ctypes.c_int64] * 3),
    "mcb_block_attn_res_v1": (ctypes.c_int32, [_T, _T, _T, _T, ctypes.c_int64, ctypes.c_int32,
                                               ctypes.c_float, _E]),
    "mcb_attn_block_workspace_bytes_v1": (ctypes.c_uint64, [ctypes.c_int64] * 3),
    "mcb_attn_block_region_v1": (ctypes.c_int32, [_T, _T, _T, _T, _T, _T, ctypes.c_int64,
                                                  ctypes.c_float, _E]),
    "mcb_attn_block_heads_workspace_bytes_v1": (ctypes.c_uint64, [ctypes.c_int64] * 3),
    "mcb_attn_block_heads_v1": (ctypes.c_int32, [_T, _T, _T, _T, _T, _T, ctypes.c_int64, _E]),
    "mcb_residual_rmsnorm_v1": (ctypes.c_int32, [_T, _T, _T, ctypes.c_float, _E]),
    "mcb_peer_exchange_create_v1": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_uint64,
                                                     _P(ctypes.c_void_p), _P(IpcHandle)]),
    "mcb_peer_exchange_connect_v1": (ctypes.c_int32, [ctypes.c_void_p, _P(IpcHandle)]),
    "mcb_peer_exchange_destroy_v1": (ctypes.c_int32, [ctypes.c_void_p]),
    "mcb_attn_block_heads_pair_v1": (ctypes.c_int32, [_T, _T, _T, _T, _T, _T, ctypes.c_int64,
                                                      ctypes.c_float, ctypes.c_int32,
                                                      ctypes.c_void_p, _E]),
    "mcb_plan_create_v1": (ctypes.c_int32, [_P(PlanDesc), _P(ctypes.c_void_p)]),
    "mcb_plan_execute_v1": (ctypes.c_int32, [ctypes.c_void_p, _T, ctypes.c_uint32,
                                             ctypes.c_void_p]),
    "mcb_plan_generation_v1": (ctypes.c_uint64, [ctypes.c_void_p]),
    "mcb_plan_destroy_v1": (ctypes.c_int32, [ctypes.c_void_p]),
    "mcb_shard_plan_v1": (ctypes.c_int32, [ctypes.c_uint32, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           _P(Shard)]),
    "mcb_device_alloc": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_uint64, _P(Buffer)]),
    "mcb_device_free": (ctypes.c_int32, [Buffer]),
    "mcb_device_is_valid": (ctypes.c_int32, [Buffer]),
    "mcb_device_upload": (ctypes.c_int32, [Buffer, ctypes.c_void_p, ctypes.c_uint64]),
    "mcb_device_download": (ctypes.c_int32, [ctypes.c_void_p, Buffer, ctypes.c_uint64]),
    "mcb_device_upload_async": (ctypes.c_int32, [Buffer, ctypes.c_void_p, ctypes.c_uint64,
                                                 ctypes.c_void_p]),
    "mcb_device_download_async": (ctypes.c_int32, [ctypes.c_void_p, Buffer, ctypes.c_uint64,
                                                   ctypes.c_void_p]),
    "mcb_comm_unique_id_v1": (ctypes.c_int32, [_P(CommId)]),
    "mcb_comm_init_v1": (ctypes.c_int32, [_P(CommId), ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, _P(ctypes.c_void_p)]),
    "mcb_allgather_v1": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_uint64, ctypes.c_void_p]),
    "mcb_reduce_scatter_v1": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_uint64, ctypes.c_int32, ctypes.c_void_p]),
    "mcb_comm_destroy_v1": (ctypes.c_int32, [ctypes.c_void_p]),
    "mcb_device_zero": (ctypes.c_int32, [Buffer]),
    "mcb_device_zero_raw_on_stream": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_uint64,
                                                       ctypes.c_void_p]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load libmcb.so and declare every entry point; raises if anything is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m matcoredsl_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is not exported
        fn.restype = res
        fn.argtypes = args
    if lib.mcb_abi_version() != ABI_VERSION:
        raise ImportError("libmcb ABI version mismatch")
    _lib = lib
    return lib


_TENSOR_SIZE = ctypes.sizeof(Tensor)


def make_tensor(ptr: int, dtype: str, shape, strides, device: bool) -> Tensor:
    t = Tensor()
    t.abi_version = ABI_VERSION
    t.struct_size = _TENSOR_SIZE
    t.data = ptr
    t.dtype = DTYPE[dtype]
    r = len(shape)
    t.rank = r
    t.dims[:r] = [int(d) for d in shape]
    t.strides[:r] = [int(s) for s in strides]
    t.memory_space = MEM_DEVICE if device else MEM_HOST
    return t


def make_exec(device: int = -1, stream: int = 0, flags: int = 0, report: Report | None = None,
              workspace: int = 0, workspace_bytes: int = 0) -> Exec:
    e = Exec()
    e.abi_version = ABI_VERSION
    e.struct_size = ctypes.sizeof(Exec)
    e.device = device
    e.flags = flags
    e.stream = stream
    e.workspace = workspace
    e.workspace_bytes = workspace_bytes
    if report is not None:
        e.report = ctypes.pointer(report)
    return e


def make_report() -> Report:
    r = Report()
    r.abi_version = ABI_VERSION
    r.struct_size = ctypes.sizeof(Report)
    return r


def make_epilogue(bias_mode="none", bias_op="add", act="none") -> Epilogue:
    ep = Epilogue()
    ep.abi_version = ABI_VERSION
    ep.struct_size = ctypes.sizeof(Epilogue)
    ep.bias_mode = BIAS_MODE[bias_mode]
    ep.bias_op = BIAS_OP[bias_op]
    ep.activation = ACT[act]
    return ep


class McbError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        self.name = STATUS.get(code, str(code))
        msg = load().mcb_status_message(code).decode()
        super().__init__(f"{what}: {self.name} ({msg})" if what else f"{self.name} ({msg})")


def check(code: int, what: str = "") -> None:
    if code != 0:
        raise McbError(code, what)
