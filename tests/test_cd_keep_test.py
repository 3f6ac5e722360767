"""The division-free keep-code test of the coordinate-descent sweep (common.cuh `cd_keeps_code`).

The repair's sweep (src/engine.rs:624-633) evaluates every column of a selected sub-block as
target = cur + g / h, q = clamp(round(target / s) + z, 0, maxq) and moves the weight iff q differs from its code.
The CUDA sweep first applies a sufficient condition that needs no division and skips the exact evaluation when it
holds.  This file restates that condition and the exact step in numpy float32 (IEEE round-to-nearest, like the
device) and checks, on millions of steps concentrated at the decision boundary, that the condition never holds
for a step that moves - the property that keeps the GPU bit-identical to the oracle.
"""
import numpy as np

F32 = np.float32


def keeps_code(g, h, cur, s, m):
    """cd_keeps_code, element-wise: lim = (0.4998 * h) * s, res = fma(s, m, -cur), both rounded to f32."""
    with np.errstate(all="ignore"):
        lim = (F32(0.4998) * h) * s
        # fma: s * m is exact in f64 (24-bit s times an integer of at most 9 bits) and so is the difference with
        # cur (it lies within a few ulps of s * m), so one rounding to f32 reproduces the device's FMA
        res = (s.astype(np.float64) * m.astype(np.float64) - cur.astype(np.float64)).astype(F32)
        return ((h > 0) & (lim < np.inf) & (np.abs(g) < lim) & (np.abs(res) <= np.abs(cur) * F32(1.1920929e-7))
                & (m == np.rint(m)))


def exact_moves(g, h, cur, s, z, maxq, code):
    """src/engine.rs:624-633 in f32: True where the step changes the code."""
    with np.errstate(all="ignore"):
        target = cur + g / h
        t2 = (target / s).astype(np.float64)
        r = np.where(t2 >= 0, np.floor(t2 + 0.5), -np.floor(-t2 + 0.5)).astype(F32)  # f32::round (half away)
        q = r + z
        q = np.where(q < 0, F32(0), q)
        q = np.where(q > maxq, maxq, q)
        qc = np.where(np.isnan(q), 0, np.nan_to_num(q)).astype(np.int64)
    return qc != code


def _sample(rng, count, bits):
    maxq = F32((1 << bits) - 1)
    # f16-representable scales from the smallest normal up
    s = np.float16(np.exp2(rng.uniform(-14, 4, count))).astype(F32)
    s = np.maximum(s, F32(6.1035156e-5))
    z = rng.integers(0, int(maxq) + 1, count).astype(F32)
    code = rng.integers(0, int(maxq) + 1, count)
    m = (code.astype(F32) - z).astype(F32)
    cur = (s * m).astype(F32)
    h = np.exp2(rng.uniform(-20, 20, count)).astype(F32)
    # gradients at the boundary |g| = 0.5 h s, a few ulps to a few percent either side, and far from it
    rel = np.concatenate([
        F32(0.5) + rng.uniform(-2e-4, 2e-4, count // 2).astype(F32),
        rng.uniform(0.0, 1.5, count - count // 2).astype(F32),
    ])
    sign = np.where(rng.random(count) < 0.5, F32(-1), F32(1))
    g = (sign * rel * h * s).astype(F32)
    return g, h, cur, s, z, maxq, code, m


def test_keep_test_never_holds_for_a_moving_step():
    rng = np.random.default_rng(20261202)
    held = 0
    for bits in (2, 3, 4, 8):
        for _ in range(4):
            g, h, cur, s, z, maxq, code, m = _sample(rng, 500_000, bits)
            keep = keeps_code(g, h, cur, s, m)
            moves = exact_moves(g, h, cur, s, z, maxq, code)
            assert not np.any(keep & moves), "keep-code test held for a step that moves"
            held += int(keep.sum())
    # the test is not vacuous: it settles most steps away from the boundary
    assert held > 1_000_000


def test_keep_test_with_w_hat_off_the_grid():
    """W_hat values that are not s * m (a few ulps to half a step away) must not let the test hold for a move."""
    rng = np.random.default_rng(7)
    for bits in (3, 8):
        g, h, cur, s, z, maxq, code, m = _sample(rng, 500_000, bits)
        off = np.concatenate([rng.integers(-4, 5, 250_000) * np.float32(2.0 ** -22),
                              rng.uniform(-0.5, 0.5, 250_000)]).astype(F32)
        cur = (s * (m + off * np.maximum(np.abs(m), 1))).astype(F32)
        keep = keeps_code(g, h, cur, s, m)
        moves = exact_moves(g, h, cur, s, z, maxq, code)
        assert not np.any(keep & moves)


def test_keep_test_edge_cases():
    one = F32(1.0)
    s = np.array([one, one, one, one, one, one], dtype=F32)
    m = np.array([1, 1, 1, 1, 0, 1], dtype=F32)
    cur = np.array([1, 1, 1, 1, 0, 1.5], dtype=F32)  # last: cur is not s * m
    g = np.array([0.1, np.nan, np.inf, 0.1, 0.0, 0.0], dtype=F32)
    h = np.array([0.0, 1.0, 1.0, np.inf, 1.0, 1.0], dtype=F32)
    keep = keeps_code(g, h, cur, s, m)
    # h = 0, NaN / infinite gradient, infinite h and a W_hat value off the grid all go to the exact evaluation
    assert keep.tolist() == [False, False, False, False, True, False]
    # a half-integer zero point is refused as well
    assert not keeps_code(np.array([0.0], F32), np.array([1.0], F32), np.array([0.5], F32),
                          np.array([1.0], F32), np.array([0.5], F32))[0]
