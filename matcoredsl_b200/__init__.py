"""B200-native (sm_100a) implementation of MatcoreDSL's data-parallel hot path.

The product is ``libmcb.so`` (hand-written CUDA kernels + C ABI, declared in
``include/mcb.h``); this package builds it (``build.py``), mirrors its ABI in
ctypes (``_abi.py``) and offers the reference's operator shapes on top
(``api.py``). Importing the package loads the library and fails loudly when it
is missing -- there is no CPU fallback.
"""
from . import _abi
from ._abi import McbError, load
from .api import (Comm, PeerExchange, Plan, attn_block, attn_block_heads, attn_block_heads_pair,
                  block_attn_res, device_status,
                  fp8_quantize_blockwise, gemm_bf16_f32_fma,
                  gemm_chain, gemm_epilogue, gemm_fp8_blockscaled, gemm_i8_i32, msm,
                  residual_rmsnorm, shard_plan, strict_fused_pair, strict_gemm)

__all__ = ["McbError", "load", "strict_gemm", "strict_fused_pair", "gemm_epilogue", "gemm_chain",
           "msm",
           "fp8_quantize_blockwise", "gemm_fp8_blockscaled", "attn_block", "attn_block_heads",
           "attn_block_heads_pair", "PeerExchange", "residual_rmsnorm", "shard_plan",
           "device_status", "Comm"]

load()
