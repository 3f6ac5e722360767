"""GPU kernels of linalg.rs / quant.rs vs the CPU oracle (bit-exact where the oracle's order is the kernel's)."""
import numpy as np
import pytest

import oracle as orc
from cdclq.abi import Config

pytestmark = pytest.mark.gpu


def spd(n, seed):
    rng = np.random.default_rng(seed)
    m = rng.standard_normal((n, n + 8))
    return m @ m.T + np.eye(n)


@pytest.mark.parametrize("n", [1, 7, 96, 97, 150, 300, 700])
def test_cholesky_bit_exact(gpu, n):
    from cdclq import linalg

    h = spd(n, n)
    a = h.copy()
    b = h.copy()
    linalg.cholesky_lower(a, n)
    orc.cholesky_lower(b, n)
    assert np.array_equal(np.tril(a), np.tril(b))


@pytest.mark.parametrize("n", [5, 96, 200, 385, 700])
def test_tri_inverse_bit_exact(gpu, n):
    from cdclq import linalg

    l = np.tril(spd(n, n + 1))
    l[np.arange(n), np.arange(n)] = np.abs(l[np.arange(n), np.arange(n)]) + n
    y1 = linalg.tri_inverse_lower(l, n)
    y2 = orc.tri_inverse_lower(l, n)
    assert np.array_equal(y1, y2)


@pytest.mark.parametrize("n", [10, 200, 333, 700])
def test_upper_chol_of_inverse_bit_exact_and_contract(gpu, n):
    """src/linalg.rs:471-504 contract plus bit-exactness against the oracle."""
    from cdclq import linalg

    h = spd(n, 2 * n)
    u1 = linalg.upper_chol_of_inverse(h, n)
    u2 = orc.upper_chol_of_inverse(h, n)
    assert np.array_equal(u1, u2)
    u = u1.astype(np.float64)
    assert np.max(np.abs(u.T @ u @ h - np.eye(n))) < 5e-4
    assert np.all(np.tril(u1, -1) == 0.0)
    assert np.all(np.diag(u1) > 0.0)


def test_not_positive_definite_message(gpu):
    import cdclq
    from cdclq import linalg

    n = 100
    a = np.eye(n)
    a[40, 40] = -2.5e-7
    with pytest.raises(cdclq.CdclqError) as ei:
        linalg.cholesky_lower(a, n)
    assert str(ei.value) == ("matrix is not positive definite (pivot 40 = -2.5e-7); increase --damp or check the "
                             "Hessian")
    assert ei.value.code == -2


def test_non_pd_layer_with_zero_damp(gpu):
    """A rank-deficient Hessian with damp = 0 fails in the factorisation with the reference's message."""
    import cdclq

    n, d_out = 64, 8
    x = np.random.default_rng(3).standard_normal((16, n)).astype(np.float32)
    h = (x.T @ x).astype(np.float32)
    w = np.random.default_rng(4).standard_normal((d_out, n)).astype(np.float32)
    with pytest.raises(cdclq.CdclqError) as ei:
        cdclq.quantize_layer(w, d_out, n, h, None, "t", Config(group=32, block=32, damp=0.0))
    assert "matrix is not positive definite" in str(ei.value)
    with pytest.raises(orc.OracleError):
        orc.quantize_layer(w, d_out, n, h, None, "t", Config(group=32, block=32, damp=0.0))


@pytest.mark.parametrize("t,n", [(1, 8), (300, 64), (2048, 130), (5000, 200)])
def test_gram_accumulate_bit_exact(gpu, t, n):
    from cdclq import linalg

    rng = np.random.default_rng(t + n)
    x = (rng.standard_normal((t, n)) * np.exp(rng.standard_normal(n))).astype(np.float32)
    h1 = np.full((n, n), 0.25)
    h2 = h1.copy()
    linalg.gram_accumulate(x, x, t, n, h1)
    orc.gram_accumulate(x, x, t, n, h2)
    assert np.array_equal(h1, h2)
    y = rng.standard_normal((t, n)).astype(np.float32)
    h1 = np.zeros((n, n))
    h2 = np.zeros((n, n))
    linalg.gram_accumulate(x, y, t, n, h1)
    orc.gram_accumulate(x, y, t, n, h2)
    assert np.array_equal(h1, h2)


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("mse", [False, True])
def test_find_params_bit_exact(gpu, bits, mse):
    import cdclq

    rng = np.random.default_rng(bits * 10 + mse)
    v = (rng.standard_normal((500, 37)) * np.exp(rng.standard_normal((500, 1)))).astype(np.float32)
    v[0] = 0.0
    v[1] = np.abs(v[1])
    v[2] = -np.abs(v[2])
    v[3, :5] = 1e-9
    s1, z1 = cdclq.find_params(v, bits, mse)
    s2, z2 = orc.find_params(v, bits, mse)
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    assert np.array_equal(z1.view(np.uint32), z2.view(np.uint32))


def test_rtn_layer_bit_exact(gpu):
    import cdclq

    w, _ = orc.problem(40, 300, 10, 5)
    for cfg in (Config(group=128), Config(group=64, mse_grid=True, bits=2), Config(group=0, bits=4)):
        a = cdclq.rtn_layer(w, 40, 300, cfg)
        b = orc.rtn_layer(w, 40, 300, cfg)
        assert np.array_equal(a, b)


def test_pack_roundtrip_mixed_bits_gpu(gpu):
    """src/quant.rs:262-274 through the GPU packer, byte-identical to the oracle's pack_row."""
    from cdclq.quant import QLayer

    g = 32
    n = 32 * 5 + 7
    gbits = np.array([8, 3, 3, 4, 2, 3], np.uint8)
    rng = np.random.default_rng(9)
    d_out = 37
    codes = np.stack([np.array([rng.integers(0, 1 << int(gbits[j // g])) for j in range(n)], np.uint8)
                      for _ in range(d_out)])
    perm = rng.permutation(n).astype(np.uint32)
    scales = rng.random((d_out, 6)).astype(np.float32)
    zeros = rng.integers(0, 8, (d_out, 6)).astype(np.float32)
    ql = QLayer(d_out, n, g, perm, gbits, codes, scales, zeros)
    packed, rb = ql.pack()
    ref, rb2 = orc.pack(codes, d_out, n, g, gbits)
    assert rb == rb2 and np.array_equal(packed, ref)
    back = QLayer.from_packed(d_out, n, g, perm, gbits, packed, scales, zeros)
    assert np.array_equal(back.codes, codes)
    oq = orc.OQLayer(d_out, n, g, perm, gbits, codes, scales, zeros)
    assert np.array_equal(ql.dequantize(), oq.dequantize())


def test_proxy_loss_close(gpu):
    import cdclq

    d_out, n = 24, 96
    w, h = orc.problem(d_out, n, 400, 11)
    wq = cdclq.rtn_layer(w, d_out, n, Config(group=32))
    a = cdclq.proxy_loss(w, wq, d_out, n, h)
    b = orc.proxy_loss(w, wq, d_out, n, h)
    assert abs(a - b) <= 1e-9 * abs(b)


def test_launch_counter_moves(gpu):
    import cdclq

    before = cdclq.lib().cdclq_launch_count()
    w, h = orc.problem(16, 64, 200, 1)
    cdclq.quantize_layer(w, 16, 64, h, None, "t", Config(group=32, block=32, sub_block=16))
    assert cdclq.lib().cdclq_launch_count() > before
