"""GPU (sm_100a) vs CPU oracle: bit-exact parity of the per-layer path through the C ABI.

Bar (stricter than BASELINE.json's north star): permutation, gbits, every integer code, every f16 scale and
zero point identical; loss_gptq identical; loss_final within 1e-9 relative (the repair's f64 loss deltas are
summed per row then per slice on the GPU, per move on the CPU); passes executed per row chunk and the number
of accepted moves identical.  Edge cases follow the reference's tests: ragged last group (172 = 5*32+12),
group == d_in, group > block and block > group, tiny layers (8/16 wide), dead input channels, skeleton groups,
MSE grids, partial repair, the asymmetric target, prep-cache reuse.
"""
import os

import numpy as np
import pytest

import oracle as orc
from cdclq.abi import Config
from conftest import GOLDEN, assert_layers_identical

pytestmark = pytest.mark.gpu


def run_both(w, h, cfg, d_out, n, m=None):
    import cdclq

    qa, sa, pa = cdclq.quantize_layer(w, d_out, n, h, m, "t", cfg, return_chunk_passes=True)
    qb, sb, pb = orc.quantize_layer(w, d_out, n, h, m, "t", cfg, return_chunk_passes=True)
    return (qa, sa, pa), (qb, sb, pb)


def check_parity(w, h, cfg, d_out, n, m=None, what=""):
    (qa, sa, pa), (qb, sb, pb) = run_both(w, h, cfg, d_out, n, m)
    assert_layers_identical(qa, qb, what)
    assert sa.loss_gptq == sb.loss_gptq, (sa.loss_gptq, sb.loss_gptq)
    assert abs(sa.loss_final - sb.loss_final) <= 1e-9 * abs(sb.loss_final), (sa.loss_final, sb.loss_final)
    assert np.array_equal(pa, pb), (pa, pb)
    assert sa.code_updates == sb.code_updates
    assert sa.subblocks_total == sb.subblocks_total
    assert sa.subblocks_refined == sb.subblocks_refined
    assert sa.skeleton_groups == sb.skeleton_groups
    assert sa.bits_codes == sb.bits_codes and sa.bits_total == sb.bits_total
    assert sa.loss_final <= sa.loss_gptq
    return sa


def small(**kw):
    return Config(bits=3, group=32, block=64, sub_block=16, act_order=False, row_chunk=8).replace(**kw)


CASES = [
    ("gptq_small", 24, 96, 400, 11, small(method="gptq")),
    ("cdcl_small", 24, 96, 400, 12, small(passes=2)),
    ("cdcl_frac025", 24, 96, 400, 12, small(passes=2, refine_frac=0.25)),
    ("skeleton_actorder", 16, 128, 300, 13, small(act_order=True, skeleton_pct=25.0)),
    ("defaults_rows300", 300, 256, 1200, 21, Config(row_chunk=128)),
    ("mse_grid", 96, 256, 1000, 22, Config(mse_grid=True, row_chunk=32, passes=4)),
    ("g_gt_b", 40, 256, 900, 23, Config(group=64, block=32, sub_block=32, row_chunk=16)),
    # group starts, U-window ends and block ends that cut the GPTQ pass's 8-column micro-blocks short
    ("group_20_block_40", 40, 200, 900, 46, Config(group=20, block=40, sub_block=10, row_chunk=16)),
    ("group_12_block_36_mse", 40, 216, 900, 47, Config(bits=4, group=12, block=36, sub_block=12, mse_grid=True,
                                                       row_chunk=16)),
    ("group_13_block_26_actorder", 36, 130, 700, 48, Config(bits=3, group=13, block=26, sub_block=7, act_order=True,
                                                            row_chunk=12)),
    ("g_eq_n", 40, 192, 900, 24, Config(group=0, block=64, sub_block=48, row_chunk=40)),
    ("b_gt_g_4bit", 72, 256, 900, 25, Config(bits=4, group=16, block=128, sub_block=32, row_chunk=24)),
    ("2bit_g64_mse", 64, 256, 900, 26, Config(bits=2, group=64, block=64, mse_grid=True, refine_frac=0.25,
                                               row_chunk=32)),
    ("sweeps2_tol0", 32, 128, 600, 27, Config(group=32, block=32, sub_block=16, cd_sweeps=2, tol=0.0, passes=3,
                                               row_chunk=16)),
    ("no_refit", 32, 128, 600, 28, Config(group=32, block=32, sub_block=16, refit_scales=False, row_chunk=16)),
    ("refit_only", 32, 128, 600, 29, Config(group=32, block=32, sub_block=16, refine_frac=0.0, passes=3,
                                             row_chunk=16)),
    ("passes0", 32, 128, 600, 30, Config(group=32, block=32, sub_block=16, passes=0, row_chunk=16)),
    ("tiny_8", 12, 8, 64, 31, Config(bits=3, group=8, block=8, sub_block=4, row_chunk=32)),
    ("tiny_16_4bit", 16, 16, 64, 32, Config(bits=4, group=16, block=16, sub_block=8, row_chunk=32)),
    ("ragged_n_150", 50, 150, 700, 33, Config(group=32, block=32, sub_block=16, row_chunk=20)),
    ("skeleton_8bit_4", 48, 256, 900, 34, Config(bits=4, group=32, block=32, skeleton_pct=10.0, row_chunk=16)),
    ("large_sub_block", 64, 512, 2000, 35, Config(group=128, block=128, sub_block=128, row_chunk=64, passes=3)),
    ("block_256", 64, 512, 2000, 36, Config(group=128, block=256, row_chunk=64, passes=3)),
    ("group_512_refit", 32, 1024, 2500, 37, Config(group=512, block=128, sub_block=64, row_chunk=32, passes=2)),
    # >= 2 x SM-count row chunks: the persistent repair kernel (all passes of a chunk in one CTA)
    ("persistent_many_chunks", 2400, 96, 500, 38, Config(group=32, block=32, sub_block=16, row_chunk=8, passes=4)),
    # 301 chunks of up to 100 rows: one CTA per chunk on 128-row tiles
    ("persistent_rc100_ragged", 30100, 64, 400, 39, Config(group=32, block=64, sub_block=32, row_chunk=100,
                                                           passes=3)),
    # 200-row chunks = two 128-row tiles: a 2-CTA cluster per chunk
    ("cluster_rc200_2tiles", 30000, 48, 300, 40, Config(group=16, block=16, sub_block=16, row_chunk=200, passes=3)),
    # 150 chunks of 128 rows on 296 CTA slots: each chunk's rows split over a 2-CTA cluster of 64-row tiles
    ("cluster_pairs_few_chunks", 19200, 64, 400, 44, Config(group=32, block=64, sub_block=32, row_chunk=128,
                                                            passes=3)),
    # 1200-row chunks = ten 128-row tiles (ragged last tile) split over a cluster
    ("cluster_rc1200_10tiles", 180000, 16, 200, 45, Config(group=8, block=8, sub_block=8, row_chunk=1200,
                                                           passes=2)),
]


@pytest.mark.parametrize("name,d_out,n,tokens,seed,cfg", CASES, ids=[c[0] for c in CASES])
def test_parity_problem(gpu, name, d_out, n, tokens, seed, cfg):
    w, h = orc.problem(d_out, n, tokens, seed)
    check_parity(w, h, cfg, d_out, n, what=name)


def test_parity_dead_columns(gpu):
    d_out, n = 40, 128
    w, h = orc.problem(d_out, n, 600, 41)
    dead = [3, 17, 64, 127]
    h[dead, :] = 0.0
    h[:, dead] = 0.0
    check_parity(w, h, Config(group=32, block=32, sub_block=16, row_chunk=16), d_out, n, what="dead")


def test_parity_asymmetric_target(gpu):
    d_out, n = 32, 128
    w, h = orc.problem(d_out, n, 600, 42)
    _, m = orc.problem(1, n, 600, 43)
    m = (0.5 * h + 0.5 * m).astype(np.float32)
    check_parity(w, h, Config(group=32, block=64, sub_block=32, row_chunk=16, method="gptq"), d_out, n, m=m,
                 what="asym gptq")
    check_parity(w, h, Config(group=32, block=64, sub_block=32, row_chunk=16, passes=2), d_out, n, m=m,
                 what="asym cdcl")


def test_parity_fixture_hessians(gpu):
    """The reference's test-fixture Hessians (tests/fixtures/*/hess.safetensors) with seeded weights, under
    the per-model settings of tests/toy_models.rs:48-58."""
    z = np.load(os.path.join(GOLDEN, "fixture_hessians.npz"))
    settings = {16: Config(bits=4, group=16, block=16, sub_block=8, row_chunk=32),
                64: Config(bits=3, group=32, block=32, sub_block=16, row_chunk=32),
                172: Config(bits=3, group=32, block=32, sub_block=16, row_chunk=32),
                256: Config(bits=3, group=32, block=32, sub_block=16, row_chunk=32)}
    for i, k in enumerate(z.files):
        h = z[k]
        n = h.shape[0]
        for d_out in (8, 96):
            w = orc.rng_normal(1000 + i * 7 + d_out, d_out * n, 0.02).reshape(d_out, n)
            check_parity(w, h, settings[n], d_out, n, what=k)


def test_prep_cache_reuse_matches(gpu):
    """q/k/v share one factorisation through the cache (src/engine.rs:718-722): results equal uncached."""
    import cdclq

    n = 192
    _, h = orc.problem(1, n, 800, 51)
    cache = cdclq.PrepCache()
    cfg = Config(group=64, block=64, sub_block=32, row_chunk=32, passes=2)
    for i, d_out in enumerate((64, 32, 32)):
        w = orc.rng_normal(60 + i, d_out * n, 0.05).reshape(d_out, n)
        qa, sa = cdclq.quantize_layer(w, d_out, n, h, None, "qkv", cfg, cache)
        qb, sb = orc.quantize_layer(w, d_out, n, h, None, "qkv", cfg)
        assert_layers_identical(qa, qb, "cache %d" % i)
        assert sa.loss_gptq == sb.loss_gptq


def test_batch_equals_single_layer_calls(gpu):
    """cdclq_quantize_batch (all layers in flight) == per-layer calls, bit for bit."""
    import ctypes

    import cdclq
    from cdclq.abi import CBatchInput, CBatchLayer, CLayerStats

    cfg = Config(group=32, block=64, sub_block=32, row_chunk=32, passes=3)
    ns = [128, 128, 192]
    hs = [orc.problem(1, n, 700, 70 + i)[1] for i, n in enumerate(ns)]
    specs = [(0, 64), (0, 32), (1, 100), (2, 48), (2, 96)]
    ws = [orc.rng_normal(80 + i, d * ns[inp], 0.04).reshape(d, ns[inp]) for i, (inp, d) in enumerate(specs)]
    ins = (CBatchInput * len(ns))()
    keep = []
    for i, h in enumerate(hs):
        hh = np.ascontiguousarray(h, np.float32)
        keep.append(hh)
        ins[i].h = hh.ctypes.data
        ins[i].n = ns[i]
    lys = (CBatchLayer * len(specs))()
    outs = []
    stats = [CLayerStats() for _ in specs]
    for i, (inp, d) in enumerate(specs):
        n = ns[inp]
        ng = (n + 31) // 32
        o = dict(perm=np.zeros(n, np.uint32), gbits=np.zeros(ng, np.uint8), codes=np.zeros((d, n), np.uint8),
                 scales=np.zeros((d, ng), np.float32), zeros=np.zeros((d, ng), np.float32))
        outs.append(o)
        ww = np.ascontiguousarray(ws[i], np.float32)
        keep.append(ww)
        lys[i].w = ww.ctypes.data
        lys[i].d_out = d
        lys[i].input = inp
        for k in ("perm", "gbits", "codes", "scales", "zeros"):
            setattr(lys[i], k, o[k].ctypes.data)
        lys[i].stats = ctypes.pointer(stats[i])
    c = cfg.to_c()
    cdclq._lib.check(cdclq.lib().cdclq_quantize_batch(ins, len(ns), lys, len(specs), ctypes.byref(c), 0, None))
    for i, (inp, d) in enumerate(specs):
        qb, sb = orc.quantize_layer(ws[i], d, ns[inp], hs[inp], None, "x", cfg)
        o = outs[i]
        assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)
        assert np.array_equal(o["zeros"], qb.zeros) and np.array_equal(o["perm"], qb.perm)
        assert stats[i].loss_gptq == sb.loss_gptq
        assert abs(stats[i].loss_final - sb.loss_final) <= 1e-9 * sb.loss_final


def test_numpy_reference_fixtures_on_gpu(gpu):
    """The GPU reproduces the golden dumps checked against the reference's numpy GPTQ."""
    import glob

    import cdclq

    for path in sorted(glob.glob(os.path.join(GOLDEN, "numpy_gptq_*.npz"))):
        z = np.load(path)
        rows, cols = int(z["rows"]), int(z["cols"])
        cfg = Config(bits=int(z["bits"]), group=int(z["group"]), block=int(z["block"]), damp=float(z["damp"]),
                     method="gptq", act_order=False, row_chunk=int(z["row_chunk"]))
        ql, st = cdclq.quantize_layer(z["w"], rows, cols, z["h"], None, "dump", cfg)
        assert np.array_equal(ql.codes, z["oracle_codes"])
        assert np.array_equal(ql.scales, z["oracle_scales"])
        assert np.array_equal(ql.zeros, z["oracle_zeros"])
        assert st.loss_gptq == float(z["oracle_loss"])
        assert float(np.mean(ql.codes == z["ref_codes"])) >= 0.995


def test_batch_split_heavy_and_light_chunks(gpu):
    """Eight heavy chunks (d_in 512) beside 300 light ones (d_in 64) in one batch: the heavy chunks run as 2-CTA
    clusters that own their SMs, concurrently with a persistent launch of the light chunks.  Same results as the
    oracle per layer."""
    import ctypes

    import cdclq
    from cdclq.abi import CBatchInput, CBatchLayer, CLayerStats

    cfg = Config(group=32, block=64, sub_block=32, row_chunk=128, passes=3)
    ns = [512, 64]
    hs = [orc.problem(1, n, 1500, 90 + i)[1] for i, n in enumerate(ns)]
    specs = [(0, 1024), (1, 38400)]
    ws = [orc.rng_normal(95 + i, d * ns[inp], 0.04).reshape(d, ns[inp]) for i, (inp, d) in enumerate(specs)]
    ins = (CBatchInput * len(ns))()
    keep = []
    for i, h in enumerate(hs):
        hh = np.ascontiguousarray(h, np.float32)
        keep.append(hh)
        ins[i].h = hh.ctypes.data
        ins[i].n = ns[i]
    lys = (CBatchLayer * len(specs))()
    outs, stats = [], [CLayerStats() for _ in specs]
    for i, (inp, d) in enumerate(specs):
        n = ns[inp]
        ng = (n + 31) // 32
        o = dict(perm=np.zeros(n, np.uint32), gbits=np.zeros(ng, np.uint8), codes=np.zeros((d, n), np.uint8),
                 scales=np.zeros((d, ng), np.float32), zeros=np.zeros((d, ng), np.float32))
        outs.append(o)
        ww = np.ascontiguousarray(ws[i], np.float32)
        keep.append(ww)
        lys[i].w = ww.ctypes.data
        lys[i].d_out = d
        lys[i].input = inp
        for k in ("perm", "gbits", "codes", "scales", "zeros"):
            setattr(lys[i], k, o[k].ctypes.data)
        lys[i].stats = ctypes.pointer(stats[i])
    c = cfg.to_c()
    cdclq._lib.check(cdclq.lib().cdclq_quantize_batch(ins, len(ns), lys, len(specs), ctypes.byref(c), 0, None))
    for i, (inp, d) in enumerate(specs):
        qb, sb = orc.quantize_layer(ws[i], d, ns[inp], hs[inp], None, "x", cfg)
        o = outs[i]
        assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)
        assert np.array_equal(o["zeros"], qb.zeros) and np.array_equal(o["perm"], qb.perm)
        assert stats[i].loss_gptq == sb.loss_gptq
        assert abs(stats[i].loss_final - sb.loss_final) <= 1e-9 * sb.loss_final
        assert stats[i].code_updates == sb.code_updates


def configs0_problem(seed=2024):
    """configs[0] of the north star, seeded: W 2048 x 2048 f32 N(0, 0.02^2) with 1 % of input columns x8; X 16384
    tokens x 2048 channels, Gaussian with log-normal channel scales (sigma 1), 0.5 % of channels x20 and 1 % dead;
    H = X^T X accumulated in f64, handed over as f32."""
    n, t = 2048, 16384
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, n)) * 0.02).astype(np.float32)
    w[:, rng.permutation(n)[:n // 100]] *= 8.0
    scale = np.exp(rng.standard_normal(n))
    p = rng.permutation(n)
    scale[p[:round(0.005 * n)]] *= 20.0
    scale[p[round(0.005 * n):round(0.005 * n) + round(0.01 * n)]] = 0.0
    h = np.zeros((n, n))
    for t0 in range(0, t, 4096):
        x = rng.standard_normal((4096, n)) * scale
        h += x.T @ x
    return w, h.astype(np.float32)


def test_parity_configs0_single_layer(gpu):
    """configs[0] at full size (the reference's CPU-runnable case): 3-bit g128, block 128, sub-block 32, damp
    0.01, act-order, passes 4, tol 1e-6, refine-frac 1, one sweep, refit on; row chunk pinned to 128."""
    w, h = configs0_problem()
    cfg = Config(bits=3, group=128, block=128, sub_block=32, damp=0.01, act_order=True, passes=4, tol=1e-6,
                 refine_frac=1.0, cd_sweeps=1, row_chunk=128)
    st = check_parity(w, h, cfg, 2048, 2048, what="configs[0]")
    assert st.skeleton_groups == 0 and st.loss_final < st.loss_gptq
