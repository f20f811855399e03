"""Helpers shared by the GPU parity tests: seeded inputs, bf16 transfers."""
from __future__ import annotations

import numpy as np

import oracle


def bf16_pair(x32: np.ndarray):
    """(bf16 bits as uint16, their exact f32 widening) using the reference RNE rule."""
    h = oracle.bf16_from_f32(np.ascontiguousarray(x32, np.float32))
    return h, oracle.bf16_to_f32(h)


def to_dev_bf16(bits_u16: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits_u16)).view(torch.bfloat16).cuda()


def to_dev_f32(x: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def from_dev(t) -> np.ndarray:
    """Device tensor -> numpy f32 (bf16 widened exactly)."""
    import torch
    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        return oracle.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))
    return t.float().cpu().numpy()


def sample_rows(m: int, tile: int = 128, seed: int = 0) -> np.ndarray:
    """At least one row per `tile`-row block, plus the first and last rows."""
    rng = np.random.default_rng(seed)
    rows = [min(m - 1, t + int(rng.integers(0, tile))) for t in range(0, m, tile)]
    return np.unique(np.array(rows + [0, m - 1], np.int64))
