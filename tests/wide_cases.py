"""Parity cases at the widths and settings of the named configurations (BASELINE.json configs[1]-[4]).

Each case is a row slice of one layer of a named model shape, quantized with that configuration's settings
and the row chunk pinned to 128: the same row chunks the model-level run quantizes, at full width.  The
inputs are reproducible bit for bit on any x86 host and on the GPU:

  * weights: the oracle's splitmix64/Box-Muller normals (the restatement of src/rng.rs), scaled in f32, the
    configuration's outlier columns x10 (numpy PCG64 permutation), rounded to bf16 by integer arithmetic
    (round to nearest even) where the model's checkpoint dtype is bf16;
  * activations X (tokens x n): normals of the same generator times a per-channel scale exp(N(0,1)) (libm
    exp in f64, then f32), 0.5 % of the channels x20 and 1 % dead (zero), Gaussian or Student-t(3)
    (z / sqrt(chi2_3 / 3), IEEE-exact f32 operations), rounded to bf16;
  * H = X^T X by the f32 Gram of src/linalg.rs:388-418 (2048-token chunks in f32, widened into f64, then
    narrowed to f32): the oracle's gram_accumulate here, the library's bit-exact cdclq_gram_accumulate_device
    on the GPU - the fixture records H's digest so that a test can tell an input difference from a
    quantization difference.

The oracle's results for every case are committed as digests (tests/golden/wide_cases.json, written by
tests/golden/make_wide_golden.py); the GPU tests compare the library's outputs with them.  TEST
INFRASTRUCTURE ONLY.
"""
import hashlib
import math

import numpy as np

TOKENS = 4096  # rank <= 4096 at the widest inputs: the relative damping (0.01 x mean diag) keeps H positive definite


def _cfg(**kw):
    from cdclq.abi import Config

    base = dict(row_chunk=128)
    base.update(kw)
    return Config(**base)


# name: (n, rows, weight kind, weight std, outlier fraction, token kind, settings, seed)
# weight kind "bf16" = bf16-valued weights (configs[1]-[3]), "f32" = f32 weights.
CASES = {
    # configs[1] (TinyLlama-shaped): q_proj (2048 wide) and down_proj (5632 wide); 3-bit g128 --mse-grid,
    # other settings the reference defaults (block 128, sub-block 64, act-order, passes 10, tol 1e-3)
    "c1_q2048": (2048, 256, "bf16", 0.02, 0.0, "gauss", dict(bits=3, group=128, mse_grid=True), 101),
    "c1_down5632": (5632, 256, "bf16", 0.02, 0.0, "gauss", dict(bits=3, group=128, mse_grid=True), 102),
    # configs[3] (Llama-2-7B-shaped, the north star): 4096 (q/k/v/o, gate/up) and 11008 (down) wide; group 64,
    # --mse-grid, refine-frac 0.25, 4-bit and 2-bit; 0.1 % outlier input columns x10
    "c3_4096_b4": (4096, 256, "bf16", 0.02, 0.001, "gauss",
                   dict(bits=4, group=64, mse_grid=True, refine_frac=0.25), 103),
    "c3_4096_b2": (4096, 256, "bf16", 0.02, 0.001, "gauss",
                   dict(bits=2, group=64, mse_grid=True, refine_frac=0.25), 103),
    "c3_11008_b4": (11008, 256, "bf16", 0.02, 0.001, "gauss",
                    dict(bits=4, group=64, mse_grid=True, refine_frac=0.25), 104),
    "c3_11008_b2": (11008, 256, "bf16", 0.02, 0.001, "gauss",
                    dict(bits=2, group=64, mse_grid=True, refine_frac=0.25), 104),
    # configs[2] (Gemma-2B-shaped): 2048 wide (q/k/v/o, gate/up) and 16384 wide (down); 4-bit g128,
    # skeleton-pct 2 (skeleton groups at 8 bits), Student-t(3) tokens
    "c2_2048_skel": (2048, 256, "bf16", 0.02, 0.0, "student3", dict(bits=4, group=128, skeleton_pct=2.0), 105),
    "c2_16384_skel": (16384, 256, "bf16", 0.02, 0.0, "student3", dict(bits=4, group=128, skeleton_pct=2.0), 106),
    # configs[4] (Llama-3-70B stress layers): q_proj 8192 wide and down_proj 28672 wide, f32 weights
    # N(0, 0.015^2); 3-bit g128, block 256, passes 8
    "c4_q8192": (8192, 256, "f32", 0.015, 0.0, "student3", dict(bits=3, group=128, block=256, passes=8), 107),
    "c4_down28672": (28672, 128, "f32", 0.015, 0.0, "student3", dict(bits=3, group=128, block=256, passes=8), 108),
}


def config(name):
    return _cfg(**CASES[name][6])


def bf16_round(x):
    """f32 -> nearest bf16 value (ties to even), as f32; integer arithmetic only."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def channel_scale(n, seed):
    """Per-channel scale: exp(N(0,1)) in f64 (libm), as f32; 0.5 % of channels x20, 1 % zero (dead)."""
    import oracle as orc

    z = orc.rng_normal(seed, n, 1.0)
    s = np.array([math.exp(float(v)) for v in z], dtype=np.float32)
    p = np.random.default_rng(seed).permutation(n)
    n_out, n_dead = max(1, round(0.005 * n)), max(1, round(0.01 * n))
    s[p[:n_out]] *= np.float32(20.0)
    s[p[n_out:n_out + n_dead]] = 0.0
    return s


def tokens(name, t=TOKENS):
    """X (t x n f32, bf16-valued) of a case."""
    import oracle as orc

    n, _, _, _, _, kind, _, seed = CASES[name]
    z = orc.rng_normal(7000 + seed, t * n, 1.0).reshape(t, n)
    if kind == "student3":
        chi = np.zeros((t, n), np.float32)
        for k in range(3):
            a = orc.rng_normal(7100 + 10 * seed + k, t * n, 1.0).reshape(t, n)
            chi += a * a
        z = z / np.sqrt(chi / np.float32(3.0))
    return bf16_round(z * channel_scale(n, 7200 + seed)[None, :])


def weights(name):
    """W rows (rows x n f32) of a case."""
    import oracle as orc

    n, rows, wkind, std, outl, _, _, seed = CASES[name]
    w = orc.rng_normal(8000 + seed, rows * n, std).reshape(rows, n)
    if outl > 0.0:
        cols = np.random.default_rng(8100 + seed).permutation(n)[:max(1, int(round(n * outl)))]
        w[:, cols] *= np.float32(10.0)
    return bf16_round(w) if wkind == "bf16" else np.ascontiguousarray(w)


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def hessian_cpu(name):
    """H (n x n f32) by the oracle's f32 Gram (src/linalg.rs:388-418)."""
    import oracle as orc

    x = tokens(name)
    n = x.shape[1]
    h = np.zeros((n, n), np.float64)
    orc.gram_accumulate(x, x, x.shape[0], n, h)
    return h.astype(np.float32)


def hessian_gpu(name):
    """H (n x n f32, host) by the library's bit-exact f32 Gram on the GPU."""
    import torch

    from cdclq import linalg

    x = torch.from_numpy(tokens(name)).cuda()
    n = x.shape[1]
    h = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    linalg.gram_accumulate_device(x, h, stream=torch.cuda.current_stream().cuda_stream)
    del x
    out = h.float().cpu().numpy()
    del h
    torch.cuda.empty_cache()
    return out


def outputs_digest(ql, stats, passes):
    """The fixture record of one quantized layer: digests of the outputs and the statistics."""
    return {
        "perm": digest(np.asarray(ql.perm, np.uint32)), "gbits": digest(np.asarray(ql.gbits, np.uint8)),
        "codes": digest(np.asarray(ql.codes, np.uint8)), "scales": digest(np.asarray(ql.scales, np.float32)),
        "zeros": digest(np.asarray(ql.zeros, np.float32)),
        "loss_gptq": float(stats.loss_gptq), "loss_final": float(stats.loss_final),
        "code_updates": int(stats.code_updates), "subblocks_refined": int(stats.subblocks_refined),
        "subblocks_total": int(stats.subblocks_total), "skeleton_groups": int(stats.skeleton_groups),
        "passes": [int(p) for p in passes],
    }
