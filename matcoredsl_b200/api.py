"""Host-side mirror of MatcoreDSL's hot-path operators, over the C ABI.

Each function takes numpy arrays (host memory: the library stages them on the
GPU and returns when the result is back) or torch CUDA tensors (device
memory: the call is queued on torch's current stream), builds the C
descriptors of include/mcb.h and calls libmcb. There is no CPU compute here
and no fallback: a missing library or a non-sm_100 device raises.

Operator meanings follow the reference:
  strict_gemm / strict_fused_pair  Session::gemm / Session::gemmStrictFusedPair
                                   (compiler/lib/runtime/closed_host_v1.cpp)
  gemm_epilogue                    @mc.fused Family A, act(A @ B (+|-) bias)
                                   (src/fusion_emitter_family_a.cpp)
  msm                              @mc.fused Family C, softmax(Q @ K.T) @ V
                                   (src/fusion_emitter_family_c.cpp)
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _abi

try:  # bf16 / fp8 numpy dtypes (optional for host-memory callers)
    import ml_dtypes as _mld
except ImportError:  # pragma: no cover
    _mld = None

_NP_DTYPE = {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64",
             np.dtype(np.float16): "f16", np.dtype(np.int8): "i8", np.dtype(np.int32): "i32"}
if _mld is not None:
    _NP_DTYPE[np.dtype(_mld.bfloat16)] = "bf16"
    _NP_DTYPE[np.dtype(_mld.float8_e4m3fn)] = "e4m3"
    _NP_DTYPE[np.dtype(_mld.float8_e5m2)] = "e5m2"


def _torch():
    import torch
    return torch


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


_TORCH_DTYPE = None  # torch dtype -> ABI dtype name, built on first use


def _torch_dtype_names():
    global _TORCH_DTYPE
    if _TORCH_DTYPE is None:
        torch = _torch()
        _TORCH_DTYPE = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16",
                        torch.int8: "i8", torch.int32: "i32", torch.float64: "f64",
                        torch.float8_e4m3fn: "e4m3", torch.float8_e5m2: "e5m2"}
    return _TORCH_DTYPE


def _desc(x, what: str):
    """(Tensor descriptor, is_device) for a numpy array or a torch tensor."""
    if _is_torch(x):
        name = _torch_dtype_names().get(x.dtype)
        if name is None:
            raise TypeError(f"{what}: unsupported torch dtype {x.dtype}")
        dev = x.is_cuda
        return _abi.make_tensor(x.data_ptr(), name, x.shape, x.stride(), dev), dev
    if isinstance(x, np.ndarray):
        dt = _NP_DTYPE.get(x.dtype)
        if dt is None:
            raise TypeError(f"{what}: unsupported numpy dtype {x.dtype}")
        strides = [s // x.itemsize for s in x.strides]
        return _abi.make_tensor(x.ctypes.data, dt, x.shape, strides, False), False
    raise TypeError(f"{what}: expected a numpy array or torch tensor, got {type(x)}")


def _workspace(ws):
    """(pointer, bytes) of an optional caller workspace: a device tensor
    whose storage the library may use as scratch for the call."""
    if ws is None:
        return 0, 0
    if not (_is_torch(ws) and ws.is_cuda):
        raise TypeError("workspace: expected a CUDA tensor")
    return ws.data_ptr(), ws.numel() * ws.element_size()


def _exec(device_call: bool, device: int, flags: int, report, workspace=None):
    stream = 0
    if device_call:
        torch = _torch()
        if device < 0:
            device = torch.cuda.current_device()
        # The raw handle of torch's current stream; building a Stream object
        # (torch.cuda.current_stream()) costs several microseconds per call.
        raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
        stream = raw(device) if raw is not None else torch.cuda.current_stream(device).cuda_stream
    ws_ptr, ws_bytes = _workspace(workspace)
    return _abi.make_exec(device=device, stream=stream, flags=flags, report=report,
                          workspace=ws_ptr, workspace_bytes=ws_bytes)


def _empty_like_out(ref, shape, dtype_name):
    if _is_torch(ref):
        torch = _torch()
        td = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dtype_name]
        return torch.empty(shape, dtype=td, device=ref.device)
    nd = {"f32": np.float32, "f16": np.float16,
          "bf16": (_mld.bfloat16 if _mld else None)}[dtype_name]
    return np.empty(shape, dtype=nd)


class Result:
    """Route/launch report of the last call (mirrors get_compilation_stats)."""

    def __init__(self, rep: _abi.Report):
        self.route = rep.route.decode()
        self.kernel_launches = rep.kernel_launches
        self.tile = (rep.tile_m, rep.tile_n, rep.tile_k)
        self.stages = rep.stages
        self.ctas = rep.ctas
        self.kernel_ms = rep.kernel_ms
        self.h2d_ms, self.d2h_ms = rep.h2d_ms, rep.d2h_ms
        self.h2d_bytes, self.d2h_bytes = rep.h2d_bytes, rep.d2h_bytes
        self.device_status = rep.device_status
        self.stream_k = bool(rep.route_flags & 1)  # MCB_ROUTE_STREAM_K


last_result: Result | None = None


def _call(fn_name, tensors, extra_args, device=-1, flags=0, workspace=None):
    global last_result
    lib = _abi.load()
    descs, spaces = [], set()
    for name, t in tensors:
        if t is None:
            descs.append(None)
            continue
        d, dev = _desc(t, name)
        descs.append(d)
        spaces.add(dev)
    device_call = True in spaces
    rep = _abi.make_report()
    ex = _exec(device_call, device, flags, rep, workspace)
    ptrs = [ctypes.byref(d) if d is not None else None for d in descs]
    # Every entry point is fn(tensor..., extra..., exec).
    code = getattr(lib, fn_name)(*ptrs, *extra_args, ctypes.byref(ex))
    last_result = Result(rep)
    _abi.check(code, fn_name)
    return last_result


def strict_gemm(a, b, out=None, *, device=-1, flags=0):
    """C = A @ B with the reference's strict f32 arithmetic (bit-exact)."""
    if out is None:
        out = _empty_like_out(a, (a.shape[0], b.shape[1]), "f32")
    _call("mcb_strict_gemm_f32_v1", [("c", out), ("a", a), ("b", b)], [], device, flags)
    return out


def gemm_i8_i32(a, b, out=None, *, a_zero_point=0, b_zero_point=0, device=-1, flags=0,
                workspace=None):
    """C = (A - a_zero_point) @ (B - b_zero_point) for int8 operands, int32
    result modulo 2^32 (bit-exact); zero points 0 give the plain int8 GEMM,
    non-zero ones the legacy quantized matmul (mcb_gemm_i8_i32_zp_v1).
    `workspace` (optional CUDA tensor) holds the B^T copy that B rows which
    are not 16-byte aligned need, and the zero points' row/column sums."""
    if out is None:
        if _is_torch(a):
            torch = _torch()
            out = torch.empty(a.shape[0], b.shape[1], dtype=torch.int32, device=a.device)
        else:
            out = np.empty((a.shape[0], b.shape[1]), np.int32)
    za, zb = _zero_point(a_zero_point), _zero_point(b_zero_point)
    if za or zb:
        _call("mcb_gemm_i8_i32_zp_v1", [("c", out), ("a", a), ("b", b)],
              [ctypes.c_int32(za), ctypes.c_int32(zb)], device, flags, workspace)
    else:
        _call("mcb_gemm_i8_i32_v1", [("c", out), ("a", a), ("b", b)], [], device, flags,
              workspace)
    return out


def _zero_point(z) -> int:
    """An int32 zero point (the reference stores them as std::int32_t)."""
    z = int(z)
    if not -2 ** 31 <= z < 2 ** 31:
        raise ValueError(f"zero point {z} does not fit in int32")
    return z


def gemm_bf16_f32_fma(a, b, out=None, *, device=-1, flags=0):
    """C = A @ B for bf16 operands with one f32 fma per k in order (bit-exact)."""
    if out is None:
        out = _empty_like_out(a, (a.shape[0], b.shape[1]), "f32")
    _call("mcb_gemm_bf16_f32_fma_v1", [("c", out), ("a", a), ("b", b)], [], device, flags)
    return out


def strict_fused_pair(a, b, d, out=None, *, device=-1, flags=0, workspace=None):
    """E = (A @ B) @ D, strict f32, intermediate rounded to f32 (bit-exact).
    `workspace` (optional CUDA tensor) holds the intermediate C when it is
    large enough; otherwise the library allocates stream-ordered scratch."""
    if out is None:
        out = _empty_like_out(a, (a.shape[0], d.shape[1]), "f32")
    _call("mcb_strict_fused_pair_f32_v1", [("e", out), ("a", a), ("b", b), ("d", d)], [],
          device, flags, workspace)
    return out


def gemm_epilogue(x, w, bias=None, *, bias_mode=None, bias_op="add", act="none", out=None,
                  out_dtype=None, w_transposed=False, device=-1, flags=0, chain=None):
    """Y = act(X @ W (+|r-) bias) (Family A). bias [N] broadcasts over rows;
    bias [M,N] is the reference's exact-shape boundary. X and W both bf16,
    both f16 or both f32; Y (default: the inputs' type) f32 or that type."""
    if bias_mode is None:
        bias_mode = "none" if bias is None else ("full" if len(bias.shape) == 2 else "row")
    n = w.shape[0] if w_transposed else w.shape[1]
    if chain is not None and (bias is not None or act != "none"):
        raise ValueError("chain replaces bias/act: give the bias as a chain op")
    if out is None:
        if out_dtype is None:
            xd = str(getattr(x, "dtype", ""))
            out_dtype = ("bf16" if xd.endswith("bfloat16") else
                         "f16" if xd.endswith("float16") else "f32")
        out = _empty_like_out(x, (x.shape[0], n), out_dtype)
    gflags = _abi.GEMM_W_TRANSPOSED if w_transposed else 0
    if chain is not None:
        ops, bnd_list = _epilogue_chain(chain)
        bnds = (_abi.Tensor * max(1, len(bnd_list)))()
        for i, t in enumerate(bnd_list):
            bnds[i] = _desc(t, f"boundary{i}")[0]
        _call("mcb_gemm_epilogue_chain_v1", [("y", out), ("x", x), ("w", w)],
              [bnds, len(bnd_list), ops, len(ops), gflags], device, flags)
        return out
    ep = _abi.make_epilogue(bias_mode, bias_op, act)
    _call("mcb_gemm_epilogue_v1", [("y", out), ("x", x), ("w", w), ("bias", bias)],
          [ctypes.byref(ep), gflags], device, flags)
    return out


def _epilogue_chain(chain):
    """ctypes ops array and boundary list for a Family A epilogue chain. Each
    item is a unary kind ("relu", "sin", ...) or (binary kind, boundary[, side])
    with side "left" (default: value op boundary) or "right" (boundary op
    value); the same boundary object is passed once."""
    if not 0 < len(chain) <= _abi.EPILOGUE_MAX_OPS:
        raise ValueError(f"an epilogue chain has 1..{_abi.EPILOGUE_MAX_OPS} ops")
    ops = (_abi.EpilogueOp * len(chain))()
    bnd_list = []
    for i, item in enumerate(chain):
        if isinstance(item, str):
            kind, bnd, side = item, None, "left"
        else:
            kind, bnd, side = (tuple(item) + ("left",))[:3]
        code = _abi.EW[kind]
        ops[i].kind = code
        if code >= 32:
            if bnd is None:
                raise ValueError(f"binary op {kind!r} needs a boundary tensor")
            idx = next((j for j, t in enumerate(bnd_list) if t is bnd), None)
            if idx is None:
                bnd_list.append(bnd)
                idx = len(bnd_list) - 1
            ops[i].boundary = idx
            ops[i].value_pos = {"left": 0, "right": 1}[side]
    if len(bnd_list) > _abi.EPILOGUE_MAX_BOUNDARIES:
        raise ValueError(f"at most {_abi.EPILOGUE_MAX_BOUNDARIES} boundary tensors")
    return ops, bnd_list


def gemm_chain(a, b, w, boundary=None, *, bias_mode=None, bias_op="add", act="none", out=None,
               out_dtype=None, device=-1, flags=0, workspace=None):
    """E = glue(A @ B) @ W (Family B); glue = act(. (+|r-) boundary)."""
    if bias_mode is None:
        bias_mode = "none" if boundary is None else (
            "full" if len(boundary.shape) == 2 else "row")
    if out is None:
        if out_dtype is None:
            out_dtype = "bf16" if str(getattr(a, "dtype", "")).endswith("bfloat16") else "f32"
        out = _empty_like_out(a, (a.shape[0], w.shape[1]), out_dtype)
    ep = _abi.make_epilogue(bias_mode, bias_op, act)
    lib = _abi.load()
    global last_result
    descs = []
    device_call = False
    for name, t in (("e", out), ("a", a), ("b", b), ("boundary", boundary), ("w", w)):
        if t is None:
            descs.append(None)
            continue
        d, dev = _desc(t, name)
        descs.append(d)
        device_call = device_call or dev
    rep = _abi.make_report()
    ex = _exec(device_call, device, flags, rep, workspace)
    ptr = lambda d: ctypes.byref(d) if d is not None else None  # noqa: E731
    code = lib.mcb_gemm_chain_v1(ptr(descs[0]), ptr(descs[1]), ptr(descs[2]), ptr(descs[3]),
                                 ctypes.byref(ep), ptr(descs[4]), ctypes.byref(ex))
    last_result = Result(rep)
    _abi.check(code, "mcb_gemm_chain_v1")
    return out


def msm(q, k, v, scale=1.0, out=None, *, device=-1, flags=0):
    """O = softmax(scale * Q @ K^T) @ V over the last two dims (Family C)."""
    if out is None:
        shape = tuple(q.shape[:-1]) + (v.shape[-1],)
        dt = "bf16" if str(q.dtype).endswith("bfloat16") else "f32"
        out = _empty_like_out(q, shape, dt)
    _call("mcb_msm_v1", [("o", out), ("q", q), ("k", k), ("v", v)], [float(scale)], device, flags)
    return out


def fp8_quantize_blockwise(x, block=128, fmt="e4m3", *, device=-1, flags=0):
    """(q, scales): per-(block x block) absmax scaling s = absmax/fmt_max,
    q = sat_RNE(x / s) as e4m3 or e5m2 codes."""
    rows, cols = x.shape
    sshape = ((rows + block - 1) // block, (cols + block - 1) // block)
    if _is_torch(x):
        torch = _torch()
        qd = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
        q = torch.empty(rows, cols, dtype=qd, device=x.device)
        s = torch.empty(sshape, dtype=torch.float32, device=x.device)
    else:
        qd = _mld.float8_e4m3fn if fmt == "e4m3" else _mld.float8_e5m2
        q = np.empty((rows, cols), dtype=qd)
        s = np.empty(sshape, dtype=np.float32)
    _call("mcb_fp8_quantize_blockwise_v1", [("q", q), ("scales", s), ("x", x)], [int(block)],
          device, flags)
    return q, s


def gemm_fp8_blockscaled(a, sa, bt, sbt, *, block=128, out=None, out_dtype="bf16", device=-1,
                         flags=0):
    """C = (sa.A) (sbt.Bt)^T with fp8 A [M,K], Bt [N,K] and per-block f32 scales."""
    if out is None:
        out = _empty_like_out(a, (a.shape[0], bt.shape[0]), out_dtype)
    _call("mcb_gemm_fp8_blockscaled_v1",
          [("c", out), ("a", a), ("sa", sa), ("bt", bt), ("sbt", sbt)], [int(block)],
          device, flags)
    return out


def block_attn_res(blocks, partial, query, *, block_count, has_partial=True, eps=1e-6, out=None,
                   device=-1, flags=0):
    """The reference's mc.block_attn_res region op (depth attention, f32)."""
    if out is None:
        out = _empty_like_out(partial, tuple(partial.shape), "f32")
    _call("mcb_block_attn_res_v1",
          [("out", out), ("blocks", blocks), ("partial", partial), ("query", query)],
          [int(block_count), 1 if has_partial else 0, float(eps)], device, flags)
    return out


def attn_block(x, wq, wk, wv, wo, heads, eps=1e-6, out=None, *, device=-1, flags=0,
               workspace=None):
    """Y = RMSNorm(X + MSM(X Wq, X Wk, X Wv) Wo), unit gain, softmax scale
    (D/heads)^-0.5; X [B, S, D] bf16, W* [D, D] bf16. `workspace` (optional
    CUDA tensor of at least mcb_attn_block_workspace_bytes_v1 bytes) holds
    the intermediates."""
    if out is None:
        out = _empty_like_out(x, tuple(x.shape), "bf16")
    _call("mcb_attn_block_region_v1",
          [("y", out), ("x", x), ("wq", wq), ("wk", wk), ("wv", wv), ("wo", wo)],
          [int(heads), float(eps)], device, flags, workspace)
    return out


def attn_block_heads(x, wq, wk, wv, wo, heads, out=None, *, device=-1, flags=0, workspace=None):
    """One head group's share of the attention block's output projection,
    P = MSM(X Wq_g, X Wk_g, X Wv_g) Wo_g: X [B, S, D] bf16, Wq_g/Wk_g/Wv_g
    [D, Dh] (the group's columns of Wq/Wk/Wv), Wo_g [Dh, D] (the matching rows
    of Wo), `heads` heads of Dh/heads. Summing P over all head groups and
    calling residual_rmsnorm(x, sum) gives attn_block(x, ...)."""
    if out is None:
        out = _empty_like_out(x, tuple(x.shape), "bf16")
    _call("mcb_attn_block_heads_v1",
          [("p", out), ("x", x), ("wq", wq), ("wk", wk), ("wv", wv), ("wo", wo)],
          [int(heads)], device, flags, workspace)
    return out


class PeerExchange:
    """This GPU's side of a two-GPU head-sharded attention block
    (mcb_peer_exchange_*_v1): create it on each GPU with the bytes of the
    rows it receives, pass `handle` (64 bytes) to the other process out of
    band, then `connect(other_handle)`. Close it only after both GPUs have
    finished their calls."""

    def __init__(self, device: int, recv_bytes: int):
        self._h = ctypes.c_void_p()
        h = _abi.IpcHandle()
        _abi.check(_abi.load().mcb_peer_exchange_create_v1(device, recv_bytes,
                                                           ctypes.byref(self._h), ctypes.byref(h)),
                   "mcb_peer_exchange_create_v1")
        self.device = device
        self.handle = ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h))

    def connect(self, other: bytes):
        h = _abi.IpcHandle()
        if len(other) != ctypes.sizeof(h):
            raise ValueError("PeerExchange.connect: the handle must be 64 bytes")
        ctypes.memmove(ctypes.addressof(h), other, ctypes.sizeof(h))
        _abi.check(_abi.load().mcb_peer_exchange_connect_v1(self._h, ctypes.byref(h)),
                   "mcb_peer_exchange_connect_v1")

    def close(self):
        if self._h:
            _abi.check(_abi.load().mcb_peer_exchange_destroy_v1(self._h),
                       "mcb_peer_exchange_destroy_v1")
            self._h = ctypes.c_void_p()


def attn_block_heads_pair(x, wq, wk, wv, wo, heads, eps, group, exchange, out=None, *, device=-1,
                          flags=0, workspace=None):
    """GPU `group` (0 or 1) of a two-GPU head-sharded attention block: its
    head group's partial output projection, the other GPU's rows sent into
    that GPU's receive buffer by the GEMM itself, and Y = RMSNorm(X + sum of
    both partials) for this GPU's half of the rows (returned, [B*S/2, D])."""
    if out is None:
        rows = x.shape[0] * x.shape[1] // 2
        out = _empty_like_out(x, (rows, x.shape[2]), "bf16")
    _call("mcb_attn_block_heads_pair_v1",
          [("y", out), ("x", x), ("wq", wq), ("wk", wk), ("wv", wv), ("wo", wo)],
          [int(heads), float(eps), int(group), exchange._h], device, flags, workspace)
    return out


def residual_rmsnorm(x, p, eps=1e-6, out=None, *, device=-1, flags=0):
    """Y = RMSNorm(X + P) over the last dimension (unit gain); X, P, Y dense
    bf16 of one shape (rank 2 or 3)."""
    if out is None:
        out = _empty_like_out(x, tuple(x.shape), "bf16")
    _call("mcb_residual_rmsnorm_v1", [("y", out), ("x", x), ("p", p)], [float(eps)], device,
          flags)
    return out


class Plan:
    """Shape-locked operator call with optional CUDA-graph replay (the
    reference's create_plan / execute_plan). Tensors are passed in the entry
    point's argument order (outputs first); None marks an absent optional
    bias/boundary slot.

    op "gemm_epilogue_chain": templates are (y, x, w) and `chain` is the op
    list of gemm_epilogue(chain=...), whose binary items name boundary
    template tensors; the boundaries become slots 3.. in order of first use,
    and execute takes (y, x, w, *boundaries) in that order."""

    def __init__(self, op, *templates, graph=False, device=-1, bias_mode="none", bias_op="add",
                 act="none", w_transposed=False, scale=1.0, block=128, heads=0, eps=1e-6,
                 a_zero_point=0, b_zero_point=0, chain=None):
        lib = _abi.load()
        chain_ops = None
        if op == "gemm_epilogue_chain":
            if chain is None or len(templates) != 3:
                raise ValueError("gemm_epilogue_chain plans take (y, x, w) and chain=[...]")
            chain_ops, bnd_list = _epilogue_chain(chain)
            templates = tuple(templates) + tuple(bnd_list)
        d = _abi.PlanDesc()
        d.abi_version = _abi.ABI_VERSION
        d.struct_size = ctypes.sizeof(_abi.PlanDesc)
        d.op = _abi.PLAN_OPS[op]
        d.graph_mode = 1 if graph else 0
        on_device = any(t is not None and _is_torch(t) and t.is_cuda for t in templates)
        if device < 0 and on_device:
            device = _torch().cuda.current_device()
        d.device = device
        d.num_tensors = len(templates)
        for i, t in enumerate(templates):
            if t is not None:
                d.tensors[i] = _desc(t, f"slot{i}")[0]
            else:
                d.tensors[i].abi_version = _abi.ABI_VERSION
                d.tensors[i].struct_size = ctypes.sizeof(_abi.Tensor)
        d.epilogue = _abi.make_epilogue(bias_mode, bias_op, act)
        d.gemm_flags = _abi.GEMM_W_TRANSPOSED if w_transposed else 0
        d.scale, d.block, d.heads, d.eps = float(scale), int(block), int(heads), float(eps)
        d.a_zero_point, d.b_zero_point = _zero_point(a_zero_point), _zero_point(b_zero_point)
        if chain_ops is not None:
            d.num_ops = len(chain_ops)
            d.num_boundaries = len(templates) - 3
            for i, o in enumerate(chain_ops):
                d.ops[i] = o
        self._zero_points = (d.a_zero_point, d.b_zero_point)
        self._handle = ctypes.c_void_p()
        _abi.check(lib.mcb_plan_create_v1(ctypes.byref(d), ctypes.byref(self._handle)),
                   "mcb_plan_create_v1")
        self._n = len(templates)
        self._device_call = on_device

    @property
    def generation(self) -> int:
        return int(_abi.load().mcb_plan_generation_v1(self._handle))

    def execute(self, *tensors, a_zero_point=None, b_zero_point=None):
        """Runs the plan. Zero points given here must equal the plan's (the
        reference's execute_plan rejects tensors whose quantization metadata
        differs from the plan's)."""
        for given, frozen, name in ((a_zero_point, self._zero_points[0], "a"),
                                    (b_zero_point, self._zero_points[1], "b")):
            if given is not None and _zero_point(given) != frozen:
                raise RuntimeError(f"quantization mismatch: {name}_zero_point {given} "
                                   f"differs from the plan's {frozen}")
        arr = (_abi.Tensor * self._n)()
        for i, t in enumerate(tensors):
            if t is not None:
                arr[i] = _desc(t, f"slot{i}")[0]
            else:
                arr[i].abi_version = _abi.ABI_VERSION
                arr[i].struct_size = ctypes.sizeof(_abi.Tensor)
        stream = _torch().cuda.current_stream().cuda_stream if self._device_call else None
        _abi.check(_abi.load().mcb_plan_execute_v1(self._handle, arr, len(tensors), stream),
                   "mcb_plan_execute_v1")

    def close(self):
        if self._handle:
            _abi.load().mcb_plan_destroy_v1(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_plan(kind, total, world, rank, *, group=0, align=1):
    """This rank's (begin, count, kv_begin, kv_count) under mcb_shard_plan_v1.
    kind: "rows" (GEMM M rows), "units" ((batch, head) MSM units) or "tokens"
    (attention block tokens; group = sequence length)."""
    k = {"rows": _abi.SHARD_ROWS, "units": _abi.SHARD_UNITS, "tokens": _abi.SHARD_TOKENS}[kind]
    s = _abi.Shard()
    _abi.check(_abi.load().mcb_shard_plan_v1(k, int(total), int(group), int(align), int(world),
                                             int(rank), ctypes.byref(s)), "mcb_shard_plan_v1")
    return s.begin, s.count, s.kv_begin, s.kv_count


class Comm:
    """NCCL communicator for the optional all-gather of output shards and
    the reduce-scatter of the head-sharded attention block (mcb_comm_*_v1). Rank 0 calls Comm.unique_id() and passes the bytes to the
    other ranks out of band; every rank then constructs Comm(uid, world, rank,
    device) (collective)."""

    @staticmethod
    def unique_id() -> bytes:
        cid = _abi.CommId()
        _abi.check(_abi.load().mcb_comm_unique_id_v1(ctypes.byref(cid)), "mcb_comm_unique_id_v1")
        return ctypes.string_at(ctypes.addressof(cid), ctypes.sizeof(cid))

    def __init__(self, uid: bytes, world: int, rank: int, device: int):
        cid = _abi.CommId()
        if len(uid) != ctypes.sizeof(cid):
            raise ValueError("Comm: the id must be the 128 bytes of Comm.unique_id()")
        ctypes.memmove(ctypes.addressof(cid), uid, ctypes.sizeof(cid))
        self._h = ctypes.c_void_p()
        self.world, self.rank, self.device = world, rank, device
        _abi.check(_abi.load().mcb_comm_init_v1(ctypes.byref(cid), world, rank, device,
                                                ctypes.byref(self._h)), "mcb_comm_init_v1")

    def allgather(self, send, recv):
        """Gathers every rank's `send` (a CUDA tensor) into `recv` (world x its
        bytes, rank order) on torch's current stream."""
        nbytes = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() != nbytes * self.world:
            raise ValueError("allgather: recv must hold world x send bytes")
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("allgather: send and recv must be contiguous")
        stream = _exec(True, self.device, 0, None).stream
        _abi.check(_abi.load().mcb_allgather_v1(self._h, send.data_ptr(), recv.data_ptr(), nbytes,
                                                stream), "mcb_allgather_v1")
        return recv

    def reduce_scatter(self, send, recv):
        """Sums `send` (a CUDA tensor of world x recv's elements, f32 or bf16)
        over all ranks and leaves this rank's slot of the sum in `recv`, on
        torch's current stream."""
        names = _torch_dtype_names()
        dt = names.get(send.dtype)
        if dt not in ("f32", "bf16") or recv.dtype != send.dtype:
            raise TypeError("reduce_scatter: send and recv must both be f32 or both bf16")
        if send.numel() != recv.numel() * self.world:
            raise ValueError("reduce_scatter: send must hold world x recv elements")
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("reduce_scatter: send and recv must be contiguous")
        stream = _exec(True, self.device, 0, None).stream
        _abi.check(_abi.load().mcb_reduce_scatter_v1(self._h, send.data_ptr(), recv.data_ptr(),
                                                     recv.numel(), _abi.DTYPE[dt], stream),
                   "mcb_reduce_scatter_v1")
        return recv

    def close(self):
        if self._h:
            _abi.check(_abi.load().mcb_comm_destroy_v1(self._h), "mcb_comm_destroy_v1")
            self._h = ctypes.c_void_p()


def device_status(device=0, clear=False) -> int:
    w = ctypes.c_uint32(0)
    _abi.check(_abi.load().mcb_device_status(device, ctypes.byref(w), 1 if clear else 0),
               "mcb_device_status")
    return int(w.value)
