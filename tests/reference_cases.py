"""The reference's strict-pair test cases, regenerated bit-for-bit in numpy.

MatcoreDSL's strict tests draw their inputs from ``std::mt19937``; numpy's
legacy ``RandomState(seed)`` uses the same seeding and its raw 32-bit draws
(``randint(0, 2**32, dtype=uint32)``) are the same sequence, so the case lists
below reproduce the reference's inputs exactly, in the same draw order.

  execution_cases()  compiler/tests/generated_cpu_fused_pair/execution_test.cpp:97-135
  physical_cases()   compiler/tests/generated_gpu_fused_pair/physical_test.cpp:297-338
  known_answers()    the discriminator cases whose expected E the reference
                     states outright (execution_test.cpp:118-135,
                     compiler/examples/experimental/two_gemm.mdsl:24-43)
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
EPS = F32(2.0 ** -23)


class _Mt:
    """Sequential raw uint32 draws of std::mt19937(seed)."""

    def __init__(self, seed: int):
        self._rs = np.random.RandomState(seed)

    def __call__(self) -> int:
        return int(self._rs.randint(0, 2 ** 32, dtype=np.uint32))

    def draws(self, n: int) -> np.ndarray:
        if n == 0:
            return np.zeros(0, np.int64)
        return self._rs.randint(0, 2 ** 32, size=n, dtype=np.uint32).astype(np.int64)


def _mat(values, rows, cols):
    return np.asarray(values, F32).reshape(rows, cols)


def execution_cases(include_sweep: bool = True):
    """(name, a, b, d) from the CPU strict-pair execution test."""
    rng = _Mt(0x4128)

    def data(size):  # ldexp(float(int(rng() % 8193) - 4096), -10)
        return ((rng.draws(size) % 8193) - 4096).astype(F32) * F32(2.0 ** -10)

    cases = []
    if include_sweep:
        for m in range(10):
            for k in range(7):
                for n in range(8):
                    for p in range(6):
                        a, b, d = data(m * k), data(k * n), data(n * p)
                        cases.append((f"geometry {m}x{k}x{n}x{p}", _mat(a, m, k), _mat(b, k, n),
                                      _mat(d, n, p)))
    else:  # keep the draw order identical even when the sweep is skipped
        for m in range(10):
            for k in range(7):
                for n in range(8):
                    for p in range(6):
                        rng.draws(m * k + k * n + n * p)
    for m, k, n, p in [(8, 13, 11, 7), (65, 63, 97, 31), (257, 64, 96, 73), (3, 128, 256, 64)]:
        a, b, d = data(m * k), data(k * n), data(n * p)
        cases.append((f"representative {m}x{k}x{n}x{p}", _mat(a, m, k), _mat(b, k, n),
                      _mat(d, n, p)))
    for size in (1, 3, 4, 5, 9):
        a = data(size * size + 1)
        x = _mat(a[:size * size], size, size)
        cases.append((f"alias {size}", x, x, x))
        y = _mat(a[1:size * size + 1], size, size)
        cases.append((f"partial alias {size}", x, y, x))
    return cases


def physical_cases():
    """(name, a, b, d) from the GPU strict-pair physical test."""
    rng = _Mt(0x684197)

    def vals(n):  # (int(rng() % 129) - 64) * 0.03125f
        return ((rng.draws(n) % 129) - 64).astype(F32) * F32(0.03125)

    cases = []
    for m in range(10):
        for k in (0, 1, 3, 5):
            for n in (0, 1, 2, 5):
                for p in (0, 1, 3):
                    a, b, d = vals(m * k), vals(k * n), vals(n * p)
                    cases.append((f"tiny/tail {m}x{k}x{n}x{p}", _mat(a, m, k), _mat(b, k, n),
                                  _mat(d, n, p)))
    for _ in range(32):
        m = 1 + rng() % 33
        k = rng() % 36
        n = 1 + rng() % 37
        p = 1 + rng() % 31
        a, b, d = vals(m * k), vals(k * n), vals(n * p)
        cases.append((f"seeded-mixed {m}x{k}x{n}x{p}", _mat(a, m, k), _mat(b, k, n),
                      _mat(d, n, p)))
    for m, k, n, p in [(8, 128, 128, 128), (64, 32, 64, 32), (65, 31, 64, 32), (1, 65535, 1, 1),
                       (1, 0, 65535, 1), (65535, 1, 1, 1), (1, 0, 1, 65535)]:
        a, b, d = vals(m * k), vals(k * n), vals(n * p)
        cases.append((f"work-cap {m}x{k}x{n}x{p}", _mat(a, m, k), _mat(b, k, n), _mat(d, n, p)))
    inf, nan = F32(np.inf), F32(np.nan)
    denorm = np.frombuffer(np.uint32(1).tobytes(), F32)[0]
    for v in (inf, -inf, nan, F32(0.0), F32(-0.0), denorm, -denorm):
        cases.append(("K0 nonempty consumer", np.zeros((5, 0), F32), np.zeros((0, 1), F32),
                      _mat([v], 1, 1)))
        cases.append(("IEEE first", _mat([v] * 5, 5, 1), _mat([1], 1, 1), _mat([1], 1, 1)))
        cases.append(("IEEE second", _mat([1] * 5, 5, 1), _mat([1], 1, 1), _mat([v], 1, 1)))
    t24 = F32(2.0 ** 24)
    cases += [
        ("producer-FMA", _mat([-1, 1 + EPS], 1, 2), _mat([1, 1 - EPS], 2, 1), _mat([1], 1, 1)),
        ("consumer-FMA", _mat([1], 1, 1), _mat([-1, 1 + EPS], 1, 2), _mat([1, 1 - EPS], 2, 1)),
        ("producer-order", _mat([t24, 1, -t24], 1, 3), _mat([1, 1, 1], 3, 1), _mat([1], 1, 1)),
        ("consumer-order", _mat([1], 1, 1), _mat([t24, 1, -t24], 1, 3), _mat([1, 1, 1], 3, 1)),
        ("producer-rounded-C-boundary", _mat([1 + EPS, 1], 1, 2), _mat([1 - EPS, 0, 0, 1], 2, 2),
         _mat([1, -1], 2, 1)),
    ]
    min_normal = np.frombuffer(np.uint32(0x00800000).tobytes(), F32)[0]
    cases += [
        ("producer-gradual-underflow", _mat([min_normal], 1, 1), _mat([0.5], 1, 1), _mat([1], 1, 1)),
        ("consumer-gradual-underflow", _mat([min_normal], 1, 1), _mat([1], 1, 1), _mat([0.5], 1, 1)),
        ("subnormal-input-not-DAZ", _mat([denorm], 1, 1), _mat([1], 1, 1), _mat([2], 1, 1)),
    ]
    same = _mat(vals(9), 3, 3)
    cases.append(("A-B-D-MAY-alias", same, same, same))
    return cases


def known_answers():
    """(name, a, b, d, expected E) whose result the reference states."""
    one = _mat([1], 1, 1)
    t24 = F32(2.0 ** 24)
    fmax = F32(np.finfo(F32).max)
    out = [
        # FMA discriminator: (1+eps)(1-eps) rounds to 1 before the add -> exactly 0.
        ("separate f32 multiply and add", _mat([-1, 1 + EPS], 1, 2), _mat([1, 1 - EPS], 2, 1),
         one, _mat([0.0], 1, 1)),
        # ((0 + 2^24) + 1) - 2^24 = 0 in increasing K order.
        ("increasing K", _mat([1, 1, 1], 1, 3), _mat([t24, 1, -t24], 3, 1), one, _mat([0.0], 1, 1)),
        ("increasing N", one, _mat([t24, 1, -t24], 1, 3), _mat([1, 1, 1], 3, 1), _mat([0.0], 1, 1)),
        # C is rounded to f32 before the consumer: E = 1 - (1+eps) = -eps.
        ("intermediate f32 boundary", _mat([1 + EPS], 1, 1), _mat([1 - EPS, 1], 1, 2),
         _mat([1, -1], 2, 1), _mat([-EPS], 1, 1)),
        # max*max = inf, inf*0 = NaN: no algebraic reassociation across the pair.
        ("no reassociation", _mat([fmax], 1, 1), _mat([fmax], 1, 1), _mat([0.0], 1, 1),
         _mat([np.nan], 1, 1)),
        # N = 0: the consumer reduction is empty and E is +0.
        ("zero N", np.zeros((1, 0), F32), np.zeros((0, 0), F32), np.zeros((0, 2), F32),
         _mat([0.0, 0.0], 1, 2)),
    ]
    for v in (F32(0.0), F32(-0.0), F32(np.inf), F32(-np.inf), F32(np.nan)):
        exp = F32(np.nan) if not np.isfinite(v) else F32(0.0)
        out.append((f"zero K with D={v}", np.zeros((1, 0), F32), np.zeros((0, 1), F32),
                    _mat([v], 1, 1), _mat([exp], 1, 1)))
    return out


def two_gemm_example():
    """compiler/examples/experimental/two_gemm.mdsl:24-43: C = A B, E = D C."""
    a = _mat([1, 2, 3, 4, 5, 6], 2, 3)
    b = _mat([1, 2, 3, 4, 5, 6], 3, 2)
    d = _mat([1, 2, 0, 1], 2, 2)
    return a, b, d, _mat([22, 28, 49, 64], 2, 2), _mat([120, 156, 49, 64], 2, 2)


def same_bits(x, y) -> bool:
    """Bitwise equality with every NaN treated as equal (the reference's `same`)."""
    x = np.asarray(x, F32)
    y = np.asarray(y, F32)
    if x.shape != y.shape:
        return False
    xn, yn = np.isnan(x), np.isnan(y)
    if not np.array_equal(xn, yn):
        return False
    return bool(np.array_equal(x.view(np.uint32)[~xn], y.view(np.uint32)[~yn]))
