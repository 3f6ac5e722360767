"""The reference's own unit tests, re-asserted on the CPU oracle (test infrastructure check).

Each test cites the reference test it restates; tolerances are the reference's.  These pin the oracle's
restatement to the reference's documented invariants before it is trusted as the GPU parity checker.
"""
import numpy as np
import pytest

import oracle as orc
from cdclq.abi import Config


def cfg_small(**kw):
    """src/engine.rs:883-885"""
    c = Config(bits=3, group=32, block=64, sub_block=16, act_order=False, row_chunk=8)
    return c.replace(**kw)


def rand_spd(n, seed):
    """src/linalg.rs:426-443: M M^T + I with M n x (n+8) standard normal (f32 draws widened)."""
    m = orc.rng_normal(seed, n * (n + 8)).astype(np.float64).reshape(n, n + 8)
    h = np.zeros((n, n))
    for i in range(n):
        for j in range(n):
            s = 0.0
            for k in range(n + 8):
                s += m[i, k] * m[j, k]
            h[i, j] = s
    h[np.arange(n), np.arange(n)] += 1.0
    return h


@pytest.fixture(scope="module")
def spd150():
    return rand_spd(150, 1)


def test_pack_roundtrip_mixed_bits():
    """src/quant.rs:262-274"""
    g = 32
    n = 32 * 5 + 7
    gbits = np.array([8, 3, 3, 4, 2, 3], np.uint8)
    r = orc.lib()
    rng = np.random.default_rng(9)
    codes = np.array([rng.integers(0, 1 << int(gbits[j // g])) for j in range(n)], np.uint8)
    packed, rb = orc.pack(codes.reshape(1, n), 1, n, g, gbits)
    assert rb == orc.row_bytes(n, g, gbits)
    back = orc.unpack(packed, 1, n, g, gbits)
    assert np.array_equal(back[0], codes)


def test_grid_reproduces_zero_and_is_f16_exact():
    """src/quant.rs:280-286"""
    v = ((np.arange(64, dtype=np.float32) - 20.0) * np.float32(0.013)).astype(np.float32)
    s, z = orc.find_params(v, 3, False)
    assert s[0] == orc.round_f16(s)[0]
    c = np.zeros(1, np.uint8)
    import ctypes

    dq = ctypes.c_float(0)
    cc = ctypes.c_uint8(0)
    orc.lib().oracle_quant_code.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                            ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_float)]
    orc.lib().oracle_quant_code(0.0, float(s[0]), float(z[0]), 7.0, ctypes.byref(cc), ctypes.byref(dq))
    assert abs(dq.value) < 1e-6
    del c


def test_round_f16_matches_ieee_rne():
    """half 2.4.1 f16::from_f32 (src/quant.rs:25) is IEEE round-to-nearest-even: compare with numpy."""
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(3.0),
        (rng.standard_normal(50000) * 1e-5).astype(np.float32),   # subnormal f16 range
        (rng.standard_normal(20000) * 7e4).astype(np.float32),    # overflow range
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, -65520.0, 6.1035156e-5, 5.96e-8, 2.98e-8, 1e-9,
                  np.inf, -np.inf], np.float32),
    ])
    # exact halfway cases between adjacent f16 values
    h = rng.integers(0, 0x7bff, 5000).astype(np.uint16).view(np.float16).astype(np.float32)
    h2 = (h.view(np.uint32) + (1 << 12)).view(np.float32)
    x = np.concatenate([x, h, h2])
    ours = orc.round_f16(x)
    ref = x.astype(np.float16).astype(np.float32)
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))


def test_cholesky_matches_definition(spd150):
    """src/linalg.rs:448-464 (n = 150 crosses the NB = 96 block boundary)"""
    n = 150
    h = spd150
    l = np.array(h, copy=True)
    orc.cholesky_lower(l, n)
    L = np.tril(l)
    err = np.max(np.abs(np.tril(L @ L.T) - np.tril(h)) / np.maximum(np.abs(np.tril(h)), 1.0))
    assert err < 1e-10


def test_upper_factor_of_inverse():
    """src/linalg.rs:471-504"""
    n = 200
    h = rand_spd(n, 2)
    u = orc.upper_chol_of_inverse(h, n).astype(np.float64)
    utu = u.T @ u
    err = np.max(np.abs(utu @ h - np.eye(n)))
    assert err < 5e-4
    assert np.all(np.tril(u, -1) == 0.0)
    assert np.all(np.diag(u) > 0.0)


def test_gemm_order_is_thread_independent():
    """src/linalg.rs:511-541 checks parallel vs serial GEMM; the oracle's fixed order makes them identical."""
    import ctypes

    rng = np.random.default_rng(3)
    for (m, k, n) in [(97, 130, 111), (20, 300, 400)]:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        outs = []
        for t in (1, 4):
            orc.set_threads(t)
            c = np.zeros((m, n), np.float32)
            f = orc.lib().oracle_sgemm
            f.restype = None
            f.argtypes = [ctypes.c_size_t] * 3 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_ssize_t, ctypes.c_ssize_t,
                                                 ctypes.c_void_p, ctypes.c_ssize_t, ctypes.c_ssize_t, ctypes.c_float,
                                                 ctypes.c_void_p, ctypes.c_ssize_t, ctypes.c_ssize_t]
            f(m, k, n, 1.0, a.ctypes.data, k, 1, b.ctypes.data, n, 1, 0.0, c.ctypes.data, n, 1)
            outs.append(c)
        orc.set_threads(0)
        assert np.array_equal(outs[0], outs[1])
        # and the fixed order is a sequential-k FMA chain per element
        ref = np.zeros((m, n), np.float32)
        acc = np.zeros((m, n), np.float32)
        for t in range(k):
            acc = (acc.astype(np.float64) + a[:, t:t + 1].astype(np.float64) * b[t:t + 1, :].astype(np.float64)).astype(
                np.float32)  # fma: product exact in f64, one rounding
        ref[:] = acc
        assert np.array_equal(outs[0], ref)


def test_gptq_loss_decomposition_is_exact():
    """src/engine.rs:891-902"""
    d_out, n = 24, 96
    w, h = orc.problem(d_out, n, 400, 11)
    cfg = cfg_small(method="gptq")
    ql, st = orc.quantize_layer(w, d_out, n, h, None, "t", cfg)
    hd = orc.damped(h, n, cfg.damp)
    direct = orc.proxy_loss(w, ql.dequantize(), d_out, n, hd)
    rel = abs(direct - st.loss_gptq) / direct
    assert rel < 2e-3


def test_repair_is_monotone_and_bookkeeping_exact():
    """src/engine.rs:908-932"""
    d_out, n = 24, 96
    w, h = orc.problem(d_out, n, 400, 12)
    cfg = cfg_small(method="gptq")
    hd = orc.damped(h, n, cfg.damp)
    q0, s0 = orc.quantize_layer(w, d_out, n, h, None, "t", cfg)
    l0 = orc.proxy_loss(w, q0.dequantize(), d_out, n, hd)
    for frac in (0.25, 1.0):
        c2 = cfg.replace(method="cdcl", refine_frac=frac, passes=2)
        q1, s1 = orc.quantize_layer(w, d_out, n, h, None, "t", c2)
        l1 = orc.proxy_loss(w, q1.dequantize(), d_out, n, hd)
        assert abs(s1.loss_gptq - s0.loss_gptq) / s0.loss_gptq < 1e-6
        assert l1 <= l0 * (1.0 + 1e-6)
        assert s1.loss_final <= s1.loss_gptq
        assert abs(l1 - s1.loss_final) / l1 < 5e-3
        assert l1 < l0


def test_skeleton_and_act_order_permutation():
    """src/engine.rs:938-970"""
    d_out, n = 16, 128
    w, h = orc.problem(d_out, n, 300, 13)
    cfg = cfg_small(act_order=True, skeleton_pct=25.0)
    ql, st = orc.quantize_layer(w, d_out, n, h, None, "t", cfg)
    assert sorted(ql.perm.tolist()) == list(range(n))
    assert st.skeleton_groups == 1
    assert ql.gbits[0] == 8
    assert np.all(ql.gbits[1:] == 3)
    wd = ql.dequantize()
    first = set(int(p) for p in ql.perm[:32])
    e = (w - wd).astype(np.float64) ** 2
    mask = np.array([j in first for j in range(n)])
    e8 = e[:, mask].sum()
    e3 = e[:, ~mask].sum()
    assert e8 / 32.0 < e3 / (n - 32.0) * 0.2


def test_asymmetric_target_reduces_to_symmetric_when_m_equals_h():
    """src/engine.rs:976-988"""
    d_out, n = 16, 64
    w, h = orc.problem(d_out, n, 300, 14)
    cfg = cfg_small(method="gptq")
    a, sa = orc.quantize_layer(w, d_out, n, h, None, "t", cfg)
    b, sb = orc.quantize_layer(w, d_out, n, h, h, "t", cfg)
    same = np.mean(a.codes == b.codes)
    assert same > 0.97
    assert abs(sa.loss_gptq - sb.loss_gptq) / sa.loss_gptq < 0.05


def test_validate_messages():
    """src/engine.rs:240-258 texts"""
    cases = [
        (Config(bits=9), "bits and skeleton_bits must be in 2..=8"),
        (Config(block=0), "block and sub_block must be > 0"),
        (Config(group=48, block=128), "group size 48 must divide the block size 128 (or be a multiple of it)"),
        (Config(group=0, skeleton_pct=5.0), "the skeleton needs a finite group size"),
        (Config(refine_frac=1.5), "refine_frac must be in [0, 1]"),
    ]
    for c, msg in cases:
        with pytest.raises(orc.OracleError) as ei:
            orc.validate(c, 256)
        assert str(ei.value) == msg


def test_non_pd_message():
    """src/linalg.rs:215-219"""
    n = 8
    a = np.eye(n)
    a[3, 3] = -1.0
    with pytest.raises(orc.OracleError) as ei:
        orc.cholesky_lower(a, n)
    assert "matrix is not positive definite (pivot 3 =" in str(ei.value)
    assert "increase --damp or check the Hessian" in str(ei.value)
