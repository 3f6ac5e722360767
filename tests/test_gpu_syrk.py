"""The bf16 tensor-core Gram accumulation (cdclq_gram_accumulate_bf16_device, tcgen05) against an exact f64
Gram of the same bf16 activations and against the bit-exact f32 path.

Tolerance: the reference sums each 2048-token chunk of f32 products in f32 (src/linalg.rs:392-416); the
tensor core sums the same exact bf16 x bf16 products in f32 in its own order.  Both differ from the exact sum
by f32 accumulation error, bounded per chunk by 2048 * 2^-24 * sum|x_p x_q|; the tests assert every element
within that bound of the exact Gram, and a Frobenius error within 3x of the f32 path's own."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16_tokens(torch, t, n, seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    scale = torch.exp(torch.randn(n, generator=g))
    x = (torch.randn(t, n, generator=g) * scale).to(torch.bfloat16)
    return x


def exact_gram(x):
    xf = x.to(dtype=x.dtype).float().numpy().astype(np.float64)
    return xf.T @ xf, np.abs(xf).T @ np.abs(xf)


# small n: fewer output tiles than SMs, tokens split into segments; n = 3080: a wave of tiles or more (no split),
# ragged p and q tiles (3080 = 24 * 128 + 8) and a partial second chunk
@pytest.mark.parametrize("t,n", [(5000, 192), (4096, 256), (2048, 136), (300, 64), (6000, 520), (2100, 3080)])
def test_bf16_gram_matches_exact_within_f32_chunk_error(gpu, t, n):
    import torch

    from cdclq import linalg

    x = bf16_tokens(torch, t, n, 1234 + n)
    ex, ab = exact_gram(x)
    h0 = np.random.default_rng(5).standard_normal((n, n))
    h0 = h0 + h0.T  # a symmetric starting value: the call adds to it
    h = torch.tensor(h0, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_bf16_device(x.cuda(), h)
    torch.cuda.synchronize()
    got = h.cpu().numpy() - h0
    chunks = (t + 2047) // 2048
    bound = chunks * 2048 * 2.0 ** -24 * ab + 1e-12
    err = np.abs(got - ex)
    assert np.all(err <= bound), float((err / bound).max())
    # of the order of the reference's own arithmetic (sequential f32 per chunk, the bit-exact f32 path): the
    # tensor core's internal f32 additions truncate, so its error is biased and up to ~2x the sequential one
    xf = x.float().numpy()
    h_f32 = np.zeros((n, n), np.float64)
    linalg.gram_accumulate(xf, xf, t, n, h_f32)
    assert np.linalg.norm(got - ex) <= 3.0 * np.linalg.norm(h_f32 - ex) + 1e-9 * np.linalg.norm(ex)
    hv = h.cpu().numpy()
    assert np.array_equal(hv, hv.T)  # the upper triangle mirrors the lower one exactly


def test_bf16_gram_lower_only_and_repeat(gpu):
    import torch

    from cdclq import linalg

    t, n = 3000, 320
    x = bf16_tokens(torch, t, n, 77).cuda()
    h = torch.full((n, n), 7.0, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_bf16_device(x, h, lower_only=True)
    linalg.gram_accumulate_bf16_device(x, h, lower_only=True)  # accumulates
    torch.cuda.synchronize()
    hv = h.cpu().numpy()
    iu = np.triu_indices(n, 1)
    assert np.all(hv[iu] == 7.0)  # upper triangle untouched
    ex, ab = exact_gram(x.cpu())
    il = np.tril_indices(n)
    got = (hv - 7.0)[il]
    bound = 2 * 2 * 2048 * 2.0 ** -24 * ab[il] + 1e-12
    assert np.all(np.abs(got - 2 * ex[il]) <= bound)


def test_bf16_gram_agrees_with_the_f32_path(gpu):
    """Same activations widened to f32 through the bit-exact f32 Gram (the reference's arithmetic): both are
    within f32 chunk-accumulation error of each other."""
    import torch

    from cdclq import linalg

    t, n = 4100, 256
    x = bf16_tokens(torch, t, n, 99)
    h_tc = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_bf16_device(x.cuda(), h_tc)
    torch.cuda.synchronize()
    xf = x.float().numpy()
    h_f32 = np.zeros((n, n), np.float64)
    linalg.gram_accumulate(xf, xf, t, n, h_f32)
    _, ab = exact_gram(x)
    bound = 2 * 3 * 2048 * 2.0 ** -24 * ab + 1e-12
    assert np.all(np.abs(h_tc.cpu().numpy() - h_f32) <= bound)


def test_bf16_gram_downstream_codes(gpu):
    """A layer quantized with the tensor-core Hessian against the same layer quantized with the f32-path Hessian
    (the reference's arithmetic): the fraction of identical codes is reported and bounded from below."""
    import torch

    import cdclq
    from cdclq import linalg
    from cdclq.abi import Config

    t, n, d_out = 16384, 512, 256
    x = bf16_tokens(torch, t, n, 4242)
    h_tc = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_bf16_device(x.cuda(), h_tc)
    torch.cuda.synchronize()
    xf = x.float().numpy()
    h_f32 = np.zeros((n, n), np.float64)
    linalg.gram_accumulate(xf, xf, t, n, h_f32)
    w = (np.random.default_rng(3).standard_normal((d_out, n)) * 0.02).astype(np.float32)
    cfg = Config(bits=3, group=128, row_chunk=128, passes=4)
    qa, _ = cdclq.quantize_layer(w, d_out, n, h_tc.cpu().numpy().astype(np.float32), None, "a", cfg)
    qb, _ = cdclq.quantize_layer(w, d_out, n, h_f32.astype(np.float32), None, "b", cfg)
    same = float(np.mean(qa.codes == qb.codes)) if np.array_equal(qa.perm, qb.perm) else 0.0
    print("identical codes with the tensor-core Hessian: %.5f" % same)
    assert same >= 0.99


def test_f16_gram_matches_exact_within_f32_chunk_error(gpu):
    """f16 activations (what a half-precision model's forward pass produces) through the same tensor-core SYRK:
    f16 x f16 products are exact in f32 too."""
    import torch

    from cdclq import linalg

    t, n = 4500, 328
    x = (bf16_tokens(torch, t, n, 4711).float() * 0.5).to(torch.float16)
    xf = x.float().numpy().astype(np.float64)
    ex, ab = xf.T @ xf, np.abs(xf).T @ np.abs(xf)
    h = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_half_device(x.cuda(), h)
    torch.cuda.synchronize()
    got = h.cpu().numpy()
    bound = ((t + 2047) // 2048) * 2048 * 2.0 ** -24 * ab + 1e-12
    assert np.all(np.abs(got - ex) <= bound)
    assert np.array_equal(got, got.T)


# the widths of configs[3]'s inputs (4096: q/k/v/o and gate/up; 11008: down_proj), whose SYRK outputs feed the
# quantizer inside the north-star run: a wave or more of output tiles, ragged tiles at 11008 = 43 * 256, a partial
# last token chunk at t = 5100
@pytest.mark.parametrize("t,n", [(5100, 4096), (4096, 11008)])
def test_bf16_gram_wide_matches_exact_within_f32_chunk_error(gpu, t, n):
    import torch

    from cdclq import linalg

    g = torch.Generator(device="cuda")
    g.manual_seed(31 + n)
    scale = torch.exp(torch.randn(n, generator=g, device="cuda"))
    x = (torch.randn(t, n, generator=g, device="cuda") * scale).to(torch.bfloat16)
    xd = x.double()
    ex = xd.T @ xd  # bf16 x bf16 products are exact in f64; f64 sums err by ~t * 2^-53, far inside the bound
    ab = xd.abs().T @ xd.abs()
    del xd
    h = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_bf16_device(x, h)
    torch.cuda.synchronize()
    chunks = (t + 2047) // 2048
    bound = ab.mul_(chunks * 2048 * 2.0 ** -24).add_(1e-12)
    err = (h - ex).abs_()
    ratio = float((err / bound).max())
    assert ratio <= 1.0, ratio
    del err, bound
    h32 = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_device(x.float().contiguous(), h32)  # the reference's arithmetic (bit-exact f32 path)
    torch.cuda.synchronize()
    e_tc = float(torch.linalg.norm(h - ex))
    e_f32 = float(torch.linalg.norm(h32 - ex))
    assert e_tc <= 3.0 * e_f32 + 1e-9 * float(torch.linalg.norm(ex)), (e_tc, e_f32)
    assert torch.equal(h, h.T)  # the upper triangle mirrors the lower one exactly
