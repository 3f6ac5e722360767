"""GPU vs CPU oracle at the widths and settings of the named configurations (BASELINE.json configs[1]-[4]).

Every case of tests/wide_cases.py is a full-width row slice of one layer of a named model shape (2048 to 28672
input columns), quantized with its configuration's settings and the row chunk pinned to 128.  The oracle's
results are committed as digests (tests/golden/wide_cases.json, tests/golden/make_wide_golden.py): the oracle
needs minutes per wide case, the GPU seconds.  The bar is the one of tests/test_gpu_parity.py: permutation,
gbits, every code, scale and zero point identical; loss_gptq identical; loss_final within 1e-9 relative; the
passes every row chunk executed and the accepted moves identical.

Each case runs under every repair launch layout the engine can choose for a model (CDCLQ_REPAIR_LAYOUT): one
launch per pass over 64-row slices (what a single layer gets), the persistent kernel with one 128-row CTA per
chunk (what configs[1] gets on one GPU), 2-CTA clusters of 64-row tiles (what a rank's shard gets on several
GPUs), and 4-CTA clusters that also split every GEMM's columns between two CTAs (the heaviest chunks of a shard
on several GPUs); the batch test below adds the heavy/light split in both cluster forms.  The wide widths exercise what the small
cases cannot: the repair's K loops over 5632 to 28672 columns, act-order and skeleton permutations of wide
Hessians, the factorisation of 11008- to 28672-wide inputs.
"""
import ctypes
import json
import os

import numpy as np
import pytest

import oracle as orc
import wide_cases as wc
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

with open(os.path.join(GOLDEN, "wide_cases.json")) as _f:
    FIXTURE = json.load(_f)
NAMES = sorted(FIXTURE, key=lambda k: (FIXTURE[k]["n"], k))
LAYOUTS = ("passes", "single", "pairs", "quads")
_H = {}


def hessian(name):
    """H of a case, rebuilt on the GPU; one kept at a time (the widest is 3.3 GB)."""
    seed = wc.CASES[name][7]
    if seed not in _H:
        _H.clear()
        _H[seed] = wc.hessian_gpu(name)
    return _H[seed]


def compare(name, got, want, layout):
    what = "%s [%s]" % (name, layout)
    diffs = [k for k in ("perm", "gbits", "codes", "scales", "zeros") if got[k] != want[k]]
    assert not diffs, "%s: %s differ from the oracle's" % (what, ", ".join(diffs))
    assert got["loss_gptq"] == want["loss_gptq"], (what, got["loss_gptq"], want["loss_gptq"])
    assert abs(got["loss_final"] - want["loss_final"]) <= 1e-9 * abs(want["loss_final"]), \
        (what, got["loss_final"], want["loss_final"])
    for k in ("passes", "code_updates", "subblocks_refined", "subblocks_total", "skeleton_groups"):
        assert got[k] == want[k], (what, k, got[k], want[k])
    assert got["loss_final"] <= got["loss_gptq"]


def diagnose(name, h, w, cfg, ql):
    """On a mismatch (widths the oracle finishes in minutes): where the GPU and the oracle part."""
    n, rows = wc.CASES[name][0], w.shape[0]
    if n > 11008:
        return "oracle not re-run at n = %d" % n
    qb, sb = orc.quantize_layer(w, rows, n, h, None, name, cfg)
    bad = np.argwhere(ql.codes != qb.codes)
    return "%d codes differ (first at %s); scales differ at %d places" % (
        len(bad), bad[:3].tolist(), int(np.count_nonzero(ql.scales != qb.scales)))


@pytest.mark.parametrize("name", NAMES)
def test_wide_parity(gpu, name, monkeypatch):
    import cdclq

    want = FIXTURE[name]
    n, rows = want["n"], want["rows"]
    h = hessian(name)
    assert wc.digest(h) == want["h"], "%s: the GPU Gram rebuilt a different H than the oracle's" % name
    w = wc.weights(name)
    assert wc.digest(w) == want["w"]
    cfg = wc.config(name)
    cache = cdclq.PrepCache()  # one factorisation per case, reused by every layout
    for layout in LAYOUTS:
        monkeypatch.setenv("CDCLQ_REPAIR_LAYOUT", layout)
        ql, st, passes = cdclq.quantize_layer(w, rows, n, h, None, name, cfg, cache, return_chunk_passes=True)
        got = wc.outputs_digest(ql, st, passes)
        if any(got[k] != want[k] for k in ("codes", "scales", "zeros")):
            pytest.fail("%s [%s]: %s" % (name, layout, diagnose(name, h, w, cfg, ql)))
        compare(name, got, want, layout)
    cache.close()


def _batch(ins_np, specs, cfg):
    """cdclq_quantize_batch over host buffers; returns per layer (outputs dict, stats)."""
    import cdclq
    from cdclq.abi import CBatchInput, CBatchLayer, CLayerStats, num_groups

    ins = (CBatchInput * len(ins_np))()
    for i, h in enumerate(ins_np):
        ins[i].h = h.ctypes.data
        ins[i].n = h.shape[0]
    lys = (CBatchLayer * len(specs))()
    outs, stats = [], [CLayerStats() for _ in specs]
    for i, (inp, w) in enumerate(specs):
        d, n = w.shape
        ng = num_groups(cfg, n)
        o = dict(perm=np.zeros(n, np.uint32), gbits=np.zeros(ng, np.uint8), codes=np.zeros((d, n), np.uint8),
                 scales=np.zeros((d, ng), np.float32), zeros=np.zeros((d, ng), np.float32))
        outs.append(o)
        L = lys[i]
        L.w = w.ctypes.data
        L.d_out = d
        L.input = inp
        for k in ("perm", "gbits", "codes", "scales", "zeros"):
            setattr(L, k, o[k].ctypes.data)
        L.stats = ctypes.pointer(stats[i])
    c = cfg.to_c()
    cdclq._lib.check(cdclq.lib().cdclq_quantize_batch(ins, len(ins_np), lys, len(specs), ctypes.byref(c), 0, None))
    return outs, stats


def test_wide_batch_heavy_split(gpu, monkeypatch):
    """configs[1]'s 5632-wide down_proj rows as the heavy chunks of a batch beside 300 light 256-wide chunks: the
    engine runs the heavy chunks as SM-owning 2-CTA clusters concurrently with a persistent launch of the light
    ones (the layout a rank's shard gets on several GPUs).  The heavy layer must reproduce the oracle's
    committed results, the light one the oracle's live results."""
    from cdclq.abi import LayerStats

    name = "c1_down5632"
    want = FIXTURE[name]
    h_heavy = np.ascontiguousarray(hessian(name), np.float32)
    w_heavy = wc.weights(name)
    cfg = wc.config(name)
    _, h_light = orc.problem(1, 256, 600, 501)  # 256 wide: the same effective group (128) as the heavy layer
    w_light = orc.rng_normal(502, 38400 * 256, 0.02).reshape(38400, 256)
    qb, sb = orc.quantize_layer(w_light, 38400, 256, h_light, None, "light", cfg)
    for layout in ("", "split", "quads"):
        monkeypatch.setenv("CDCLQ_REPAIR_LAYOUT", layout)
        outs, stats = _batch([h_heavy, np.ascontiguousarray(h_light)], [(0, w_heavy), (1, w_light)], cfg)
        o = outs[0]
        s = LayerStats.from_c(stats[0])
        got = {"perm": wc.digest(o["perm"]), "gbits": wc.digest(o["gbits"]), "codes": wc.digest(o["codes"]),
               "scales": wc.digest(o["scales"]), "zeros": wc.digest(o["zeros"]), "loss_gptq": s.loss_gptq,
               "loss_final": s.loss_final, "code_updates": s.code_updates, "subblocks_refined": s.subblocks_refined,
               "subblocks_total": s.subblocks_total, "skeleton_groups": s.skeleton_groups,
               "passes": want["passes"]}  # per-chunk passes are not reported by the batch call
        compare(name, got, want, layout or "auto")
        o = outs[1]
        assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)
        assert np.array_equal(o["zeros"], qb.zeros) and np.array_equal(o["perm"], qb.perm)
        assert stats[1].loss_gptq == sb.loss_gptq
        assert abs(stats[1].loss_final - sb.loss_final) <= 1e-9 * sb.loss_final


def test_factorisation_sub_batches(gpu, monkeypatch):
    """Three same-width inputs factorised in memory-bounded sub-batches (the path a full model takes when its
    factorisations do not fit in free memory at once) give the oracle's results."""
    import cdclq

    n = 2048
    hs = [np.ascontiguousarray(orc.problem(1, n, 2600, 600 + i)[1]) for i in range(3)]
    ws = [orc.rng_normal(610 + i, 128 * n, 0.02).reshape(128, n) for i in range(3)]
    cfg = wc._cfg(bits=3, group=128, mse_grid=True)
    item = 2 * 8 * n * n + 97 * 8 * n + 256  # one input's f64 work matrices (the engine's per-item estimate)
    monkeypatch.setenv("CDCLQ_FACTOR_BUDGET_BYTES", str(int(1.5 * item)))  # one input per sub-batch
    outs, stats = _batch(hs, [(i, ws[i]) for i in range(3)], cfg)
    prof = cdclq._lib.last_run_profile()
    assert prof["factor_batches"] >= 3, prof["factor_batches"]
    for i in range(3):
        qb, sb = orc.quantize_layer(ws[i], 128, n, hs[i], None, "x", cfg)
        o = outs[i]
        assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)
        assert np.array_equal(o["zeros"], qb.zeros) and np.array_equal(o["perm"], qb.perm)
        assert stats[i].loss_gptq == sb.loss_gptq


def test_factorisation_sub_batches_two_widths(gpu, monkeypatch):
    """Two width groups under a factorisation budget smaller than their need: each group works through its inputs
    in sub-batches of its share of the budget on its own stream, one sub-batch of each group in flight at a time;
    the results are the oracle's."""
    import cdclq

    widths = (2048, 2048, 1024, 1024)
    hs = [np.ascontiguousarray(orc.problem(1, n, 2600, 700 + i)[1]) for i, n in enumerate(widths)]
    ws = [orc.rng_normal(710 + i, 128 * n, 0.02).reshape(128, n) for i, n in enumerate(widths)]
    cfg = wc._cfg(bits=3, group=128, mse_grid=True)
    item = 2 * 8 * 2048 * 2048 + 97 * 8 * 2048 + 256  # the engine's per-item estimate at n = 2048
    monkeypatch.setenv("CDCLQ_FACTOR_BUDGET_BYTES", str(int(1.5 * item)))  # one input of each width at a time
    outs, stats = _batch(hs, [(i, ws[i]) for i in range(len(widths))], cfg)
    prof = cdclq._lib.last_run_profile()
    assert prof["factor_batches"] >= 4, prof["factor_batches"]
    for i, n in enumerate(widths):
        qb, sb = orc.quantize_layer(ws[i], 128, n, hs[i], None, "x", cfg)
        o = outs[i]
        assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)
        assert np.array_equal(o["zeros"], qb.zeros) and np.array_equal(o["perm"], qb.perm)
        assert stats[i].loss_gptq == sb.loss_gptq
        assert abs(stats[i].loss_final - sb.loss_final) <= 1e-9 * sb.loss_final
