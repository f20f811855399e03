"""CPU oracle for the MatcoreDSL hot path -- TEST INFRASTRUCTURE ONLY.

This package is the checker the CUDA path is compared against. It is loaded
only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py``; the product library (``matcoredsl_b200``) never imports it.

The arithmetic lives in C++ (``oracle/*.cpp``, built by ``oracle/Makefile``
into ``oracle/_build/liboracle.so``); this module is a thin ctypes wrapper
over it plus numpy helpers for seeded synthetic inputs. Each C++ function
cites the MatcoreDSL source it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_REF_PATH = os.path.join(_HERE, "_ref", "libmcref.so")
_lib = None
_ref = None

ACT = {"none": 0, "relu": 1, "gelu_tanh": 2, "exp": 3, "sigmoid": 4, "tanh": 5}
BIAS_MODE = {"none": 0, "row": 1, "full": 2}
BIAS_OP = {"add": 0, "rsub": 1}
FP8 = {"e4m3": 0, "e5m2": 1}
FP8_MAX = {"e4m3": 448.0, "e5m2": 57344.0}

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64


def build(ref: bool = False) -> None:
    """Compile the oracle (and, when asked, the reference's numeric file)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", _HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "orc_strict_gemm_f32": [_f32p, _f32p, _f32p, _i64, _i64, _i64],
            "orc_strict_fused_pair_f32": [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64],
            "orc_strict_fused_pair_f32_mt": [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, ctypes.c_int],
            "orc_bf16_from_f32": [_f32p, _u16p, _i64],
            "orc_bf16_to_f32": [_u16p, _f32p, _i64],
            "orc_gemm_bf16_f32_fma": [_u16p, _u16p, _f32p, _i64, _i64, _i64],
            "orc_gemm_i8_i32": [_i8p, _i8p, _i32p, _i64, _i64, _i64],
            "orc_gemm_i8_i32_zp": [_i8p, _i8p, _i32p, _i64, _i64, _i64, ctypes.c_int32,
                                   ctypes.c_int32],
            "orc_gemm_epilogue_f64": [_f32p, _f32p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _f64p, _i64, _i64, _i64, ctypes.c_void_p, _i64],
            "orc_msm_f64": [_f32p, _f32p, _f32p, _f64p, _i64, _i64, _i64, _i64, ctypes.c_double],
            "orc_fp8_encode": [_f32p, _u8p, _i64, ctypes.c_int],
            "orc_fp8_decode": [_u8p, _f32p, _i64, ctypes.c_int],
            "orc_fp8_quantize_blockwise": [_f32p, _i64, _i64, _i64, ctypes.c_int, _u8p, _f32p],
            "orc_gemm_fp8_blockscaled_f64": [_u8p, ctypes.c_int, _f32p, _u8p, ctypes.c_int, _f32p,
                                             _f64p, _i64, _i64, _i64, _i64, ctypes.c_void_p, _i64],
            "orc_baseline_gemm_bias_gelu_f32_full": [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64,
                                                     ctypes.c_int],
        }
        for name, argtypes in sig.items():
            fn = getattr(L, name)
            fn.argtypes = argtypes
            fn.restype = None
        L.orc_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own cpu_numeric_reference.cpp, when it was compiled here."""
    global _ref
    if _ref is None and os.path.exists(_REF_PATH):
        R = ctypes.CDLL(_REF_PATH)
        R.ref_bf16_from_f32.argtypes = [_f32p, _u16p, _i64]
        R.ref_bf16_to_f32.argtypes = [_u16p, _f32p, _i64]
        R.ref_gemm_bf16_f32.argtypes = [_u16p, _u16p, _f32p, _i64, _i64, _i64]
        R.ref_gemm_bf16_f32.restype = ctypes.c_int
        R.ref_gemm_i8_i32.argtypes = [_i8p, _i8p, _i32p, _i64, _i64, _i64]
        R.ref_gemm_i8_i32.restype = ctypes.c_int
        _ref = R
    return _ref


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---- strict f32 -----------------------------------------------------------
def strict_gemm(a, b):
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().orc_strict_gemm_f32(a, b, c, m, k, n)
    return c


def strict_fused_pair(a, b, d, threads: int = 1):
    a, b, d = _c(a, np.float32), _c(b, np.float32), _c(d, np.float32)
    m, k = a.shape
    n, p = d.shape
    e = np.empty((m, p), np.float32)
    if threads > 1:
        lib().orc_strict_fused_pair_f32_mt(a.reshape(-1) if a.size else np.zeros(1, np.float32),
                                           b.reshape(-1) if b.size else np.zeros(1, np.float32),
                                           d.reshape(-1) if d.size else np.zeros(1, np.float32),
                                           e.reshape(-1) if e.size else np.zeros(1, np.float32),
                                           m, k, n, p, threads)
    else:
        lib().orc_strict_fused_pair_f32(a.reshape(-1) if a.size else np.zeros(1, np.float32),
                                        b.reshape(-1) if b.size else np.zeros(1, np.float32),
                                        d.reshape(-1) if d.size else np.zeros(1, np.float32),
                                        e.reshape(-1) if e.size else np.zeros(1, np.float32),
                                        m, k, n, p)
    return e


# ---- bf16 ------------------------------------------------------------------
def bf16_from_f32(x):
    x = _c(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_bf16_from_f32(x.reshape(-1), y.reshape(-1), x.size)
    return y


def bf16_to_f32(h):
    h = _c(h, np.uint16)
    y = np.empty(h.shape, np.float32)
    lib().orc_bf16_to_f32(h.reshape(-1), y.reshape(-1), h.size)
    return y


def gemm_bf16_f32_fma(a, b):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().orc_gemm_bf16_f32_fma(a, b, c, m, k, n)
    return c


def gemm_i8_i32(a, b):
    a, b = _c(a, np.int8), _c(b, np.int8)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.int32)
    lib().orc_gemm_i8_i32(a, b, c, m, k, n)
    return c


def gemm_i8_i32_zp(a, b, a_zero_point, b_zero_point):
    """sum_k (A - za)(B - zb) in wrapping int32 (the legacy quantized_i8 matmul)."""
    a, b = _c(a, np.int8), _c(b, np.int8)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.int32)
    lib().orc_gemm_i8_i32_zp(a, b, c, m, k, n, int(a_zero_point), int(b_zero_point))
    return c


# ---- Family A / C (fp64) -----------------------------------------------------
def gemm_epilogue(x, w, bias=None, bias_mode="none", bias_op="add", act="none", rows=None):
    """fp64 y = act(x w (+|r-) bias) for `rows` (all rows when None)."""
    x, w = _c(x, np.float32), _c(w, np.float32)
    m, k = x.shape
    n = w.shape[1]
    bptr = None
    if bias_mode != "none":
        bias = _c(bias, np.float32)
        bptr = bias.ctypes.data
    if rows is None:
        y = np.empty((m, n), np.float64)
        rptr, nr = None, m
    else:
        rows = _c(rows, np.int64)
        y = np.empty((rows.size, n), np.float64)
        rptr, nr = rows.ctypes.data, rows.size
    lib().orc_gemm_epilogue_f64(x, w, bptr, BIAS_MODE[bias_mode], BIAS_OP[bias_op], ACT[act],
                                y, m, k, n, rptr, nr)
    return y



def gemm_epilogue_chain(x, w, chain):
    """fp64 Family A epilogue chain, op by op as the reference emits them
    (src/fusion_emitter_common.cpp:38-160; chain rules
    src/fusion_emitter_family_a.cpp:149-220). `chain` items: a unary kind, or
    (binary kind, boundary[, "left"|"right"]); "right" puts the running value
    on the right of the operator."""
    v = gemm_epilogue(x, w)
    c0, c1 = 0.7978845608, 0.044715
    unary = {
        "relu": lambda a: np.maximum(a, 0.0), "exp": np.exp, "log": np.log, "tanh": np.tanh,
        "sqrt": np.sqrt, "neg": np.negative, "abs": np.abs, "sin": np.sin, "cos": np.cos,
        "rsqrt": lambda a: 1.0 / np.sqrt(a), "sigmoid": lambda a: 1.0 / (1.0 + np.exp(-a)),
        "gelu_tanh": lambda a: 0.5 * a * (1.0 + np.tanh(c0 * (a + c1 * a * a * a))),
    }
    unary["gelu"] = unary["gelu_tanh"]
    binary = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide,
              "min": np.minimum, "max": np.maximum}
    with np.errstate(all="ignore"):
        for item in chain:
            if isinstance(item, str):
                v = unary[item](v)
                continue
            kind, bnd, side = (tuple(item) + ("left",))[:3]
            b = np.asarray(bnd, np.float64)
            v = binary[kind](v, b) if side == "left" else binary[kind](b, v)
    return v

def msm(q, k, v, scale=1.0):
    """fp64 softmax(scale * q k^T) v for rank-2 q [m,d], k [n,d], v [n,dv]."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    m, dqk = q.shape
    n, dv = v.shape
    o = np.empty((m, dv), np.float64)
    lib().orc_msm_f64(q, k, v, o, m, n, dqk, dv, float(scale))
    return o


# ---- FP8 -------------------------------------------------------------------
def fp8_encode(x, fmt="e4m3"):
    x = _c(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    lib().orc_fp8_encode(x.reshape(-1), q.reshape(-1), x.size, FP8[fmt])
    return q


def fp8_decode(q, fmt="e4m3"):
    q = _c(q, np.uint8)
    x = np.empty(q.shape, np.float32)
    lib().orc_fp8_decode(q.reshape(-1), x.reshape(-1), q.size, FP8[fmt])
    return x


def fp8_quantize_blockwise(x, block=128, fmt="e4m3"):
    x = _c(x, np.float32)
    r, c = x.shape
    q = np.empty((r, c), np.uint8)
    s = np.empty(((r + block - 1) // block, (c + block - 1) // block), np.float32)
    lib().orc_fp8_quantize_blockwise(x, r, c, block, FP8[fmt], q, s)
    return q, s


def gemm_fp8_blockscaled(a, sa, bt, sbt, a_fmt="e4m3", b_fmt="e4m3", block=128, rows=None):
    a, bt = _c(a, np.uint8), _c(bt, np.uint8)
    sa, sbt = _c(sa, np.float32), _c(sbt, np.float32)
    m, k = a.shape
    n = bt.shape[0]
    if rows is None:
        c = np.empty((m, n), np.float64)
        rptr, nr = None, m
    else:
        rows = _c(rows, np.int64)
        c = np.empty((rows.size, n), np.float64)
        rptr, nr = rows.ctypes.data, rows.size
    lib().orc_gemm_fp8_blockscaled_f64(a, FP8[a_fmt], sa, bt, FP8[b_fmt], sbt, c, m, k, n,
                                       block, rptr, nr)
    return c


# ---- block_attn_res (depth attention over packed block history, fp64) -----------
def block_attn_res(blocks, partial, query, block_count, has_partial=True, eps=1e-6):
    """The reference's region op (tests/test_block_attn_res.py:16-39): sources
    = blocks[:block_count] (+ partial), each RMS-normalised over D and dotted
    with `query`; softmax over sources; output = weighted sum of the raw
    sources. No sources -> zeros. fp64 throughout, returned as float64."""
    blocks = np.asarray(blocks, np.float64)
    partial = np.asarray(partial, np.float64)
    query = np.asarray(query, np.float64)
    sources = []
    if block_count:
        sources.append(blocks[:block_count])
    if has_partial:
        sources.append(partial[None, ...])
    if not sources:
        return np.zeros_like(partial)
    packed = np.concatenate(sources, axis=0)
    inv_rms = 1.0 / np.sqrt(np.mean(packed * packed, axis=-1, keepdims=True) + eps)
    scores = np.sum((packed * inv_rms) * query.reshape(1, 1, 1, -1), axis=-1)
    scores = scores - np.max(scores, axis=0, keepdims=True)
    w = np.exp(scores)
    w = w / np.sum(w, axis=0, keepdims=True)
    return np.sum(w[..., None] * packed, axis=0)


# ---- attention-residual block (fp64, numpy) -------------------------------------
def attn_block(x, wq, wk, wv, wo, heads, eps=1e-6, batch=0, tokens=None):
    """fp64 Y[b, t] = RMSNorm(X + MSM(X Wq, X Wk, X Wv) Wo) for batch element
    `batch` and the listed tokens (all when None), unit gain, scale hd^-0.5.

    The block is not a reference operator (the reference's region op is the
    depth-attention block_attn_res); this restates BASELINE config 5 from its
    definition, composing the Family A/C semantics above. parity unpinned
    against the reference. K and V are needed for every token of the batch
    element; Q, attention, projection and norm only for the sampled tokens.
    """
    xb = np.asarray(x[batch], np.float64)
    s, d = xb.shape
    hd = d // heads
    t = np.arange(s) if tokens is None else np.asarray(tokens)
    wq, wk, wv, wo = (np.asarray(w, np.float64) for w in (wq, wk, wv, wo))
    q = xb[t] @ wq
    k = xb @ wk
    v = xb @ wv
    attn = np.empty((t.size, d))
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        sc = (q[:, sl] @ k[:, sl].T) * (hd ** -0.5)
        sc -= sc.max(axis=1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=1, keepdims=True)
        attn[:, sl] = p @ v[:, sl]
    r = xb[t] + attn @ wo
    return r / np.sqrt(np.mean(r * r, axis=1, keepdims=True) + eps)


# ---- CPU baseline -------------------------------------------------------------
def baseline_gemm_bias_gelu(x32, w32, b32, threads=None):
    x32, w32, b32 = _c(x32, np.float32), _c(w32, np.float32), _c(b32, np.float32)
    m, k = x32.shape
    n = w32.shape[1]
    y = np.empty((m, n), np.float32)
    lib().orc_baseline_gemm_bias_gelu_f32_full(x32, w32, b32, y, m, k, n,
                                               int(threads or max_threads()))
    return y


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ---- seeded synthetic inputs ----------------------------------------------------
def rel_frobenius(x, ref) -> float:
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))
