"""Multi-GPU building blocks on one GPU: caller-supplied factors (cdclq_prepare_factors ->
cdclq_quantize_batch_prepared) and row shards give the single-call result bit for bit, through the C ABI."""
import ctypes

import numpy as np
import pytest

import oracle as orc
from cdclq.abi import Config

pytestmark = pytest.mark.gpu

NS = [128, 192, 128]
SPECS = [(0, 64), (0, 96), (1, 100), (2, 48), (2, 130)]  # (input, d_out)
CFG = Config(group=32, block=64, sub_block=32, row_chunk=32, passes=3)


def model(torch, device):
    hs = [torch.tensor(orc.problem(1, n, 700, 170 + i)[1], dtype=torch.float32) for i, n in enumerate(NS)]
    ws = [torch.tensor(orc.rng_normal(180 + i, d * NS[inp], 0.04).reshape(d, NS[inp]), dtype=torch.float32)
          for i, (inp, d) in enumerate(SPECS)]
    if device == "cuda":
        hs = [h.cuda() for h in hs]
        ws = [w.cuda() for w in ws]
    else:
        hs = [h.pin_memory() for h in hs]
        ws = [w.pin_memory() for w in ws]
    layers = [("l%d" % i, d, NS[inp], inp) for i, (inp, d) in enumerate(SPECS)]
    inputs = [("in%d" % i, n) for i, n in enumerate(NS)]
    return layers, inputs, hs, ws


def outputs(mb):
    return [{k: (v.cpu().numpy() if hasattr(v, "cpu") else v).copy() for k, v in o.items()} for o in mb.outs]


def assert_same(a, b):
    for x, y in zip(a, b):
        for k in ("perm", "gbits", "codes", "scales", "zeros"):
            assert np.array_equal(x[k], y[k]), k


@pytest.mark.parametrize("on_device", [True, False])
def test_prepared_factors_give_the_batch_result(gpu, on_device):
    import torch

    import cdclq
    from cdclq.pipeline import ModelBatch

    layers, inputs, hs, ws = model(torch, "cuda" if on_device else "cpu")
    ref = ModelBatch(torch, layers, inputs, hs, ws, CFG, on_device=on_device)
    ref.run(0)
    torch.cuda.synchronize()
    mb = ModelBatch(torch, layers, inputs, hs, ws, CFG, on_device=on_device)
    us = [torch.full((n, n), float("nan"), dtype=torch.float32, device="cuda") for n in NS]
    mine = [0, 2]  # input 1 is factorised inside the batch call
    which = (ctypes.c_size_t * 2)(*mine)
    u_out = (ctypes.c_void_p * 2)(*[us[i].data_ptr() for i in mine])
    c = CFG.to_c()
    L = cdclq.lib()
    cdclq._lib.check(L.cdclq_prepare_factors(mb.ins, len(NS), ctypes.cast(which, ctypes.c_void_p), 2, ctypes.byref(c),
                                             ctypes.cast(u_out, ctypes.c_void_p), 1 if on_device else 0, None))
    torch.cuda.synchronize()
    for i in mine:  # strictly lower part exactly 0, positive diagonal (src/linalg.rs:498-503)
        u = us[i].cpu().numpy()
        assert np.all(np.tril(u, -1) == 0.0) and np.all(np.diag(u) > 0.0)
    u_in = (ctypes.c_void_p * 3)(us[0].data_ptr(), None, us[2].data_ptr())
    cdclq._lib.check(L.cdclq_quantize_batch_prepared(mb.ins, len(NS), ctypes.cast(u_in, ctypes.c_void_p), mb.lys,
                                                     len(mb.lys), ctypes.byref(c), 1 if on_device else 0, None))
    torch.cuda.synchronize()
    assert_same(outputs(mb), outputs(ref))
    for s, r in zip(mb.stats, ref.stats):
        assert s.loss_gptq == r.loss_gptq and s.loss_final == r.loss_final and s.code_updates == r.code_updates
    # and the oracle agrees on one layer fed by a caller-supplied factor
    qb, sb = orc.quantize_layer(ws[4].cpu().numpy(), SPECS[4][1], NS[2], hs[2].cpu().numpy(), None, "x", CFG)
    o = outputs(mb)[4]
    assert np.array_equal(o["codes"], qb.codes) and np.array_equal(o["scales"], qb.scales)


def test_row_shards_concatenate_to_the_full_result(gpu):
    import torch

    from cdclq.pipeline import ModelBatch

    layers, inputs, hs, ws = model(torch, "cuda")
    full = ModelBatch(torch, layers, inputs, hs, ws, CFG)
    full.run(0)
    torch.cuda.synchronize()
    ref = outputs(full)
    for world in (2, 3):
        parts = []
        for rank in range(world):
            mb = ModelBatch(torch, layers, inputs, hs, ws, CFG, rank=rank, world=world, distribute_factors=False)
            mb.run(0)
            torch.cuda.synchronize()
            parts.append(dict(zip(mb.names, zip(mb.shards, outputs(mb)))))
        for li, (name, d_out, _, _) in enumerate(layers):
            rows = sorted((p[name] for p in parts if name in p), key=lambda x: x[0][0])  # ranks rotate per layer
            assert rows[0][0][0] == 0 and rows[-1][0][1] == d_out
            for k in ("codes", "scales", "zeros"):
                assert np.array_equal(np.concatenate([o[k] for _, o in rows]), ref[li][k]), (name, world, k)
            for _, o in rows:
                assert np.array_equal(o["perm"], ref[li]["perm"])


def test_rank_local_weight_shards_give_the_same_rows(gpu):
    """w_sharded=True: each rank passes only its own rows of W (the multi-GPU bench generates them per rank)."""
    import torch

    from cdclq.pipeline import ModelBatch, shard_rows

    layers, inputs, hs, ws = model(torch, "cuda")
    world = 2
    for rank in range(world):
        a = ModelBatch(torch, layers, inputs, hs, ws, CFG, rank=rank, world=world, distribute_factors=False)
        a.run(0)
        wl = []
        for li, (_, d_out, _, _) in enumerate(layers):
            r0, r1 = shard_rows(d_out, CFG.row_chunk, rank, world, rotate=li)
            wl.append(ws[li][r0:r1].clone() if r1 > r0 else None)
        b = ModelBatch(torch, layers, inputs, hs, wl, CFG, rank=rank, world=world, distribute_factors=False,
                       w_sharded=True)
        b.run(0)
        torch.cuda.synchronize()
        assert a.names == b.names and a.shards == b.shards
        assert_same(outputs(a), outputs(b))
    with pytest.raises(ValueError):
        ModelBatch(torch, layers, inputs, hs, ws, CFG, rank=0, world=2, distribute_factors=False, w_sharded=True)


def test_skeleton_row_shards_use_the_full_matrix_ranking(gpu):
    """A skeleton ranks columns by H_jj ||W_:j||^2 over all rows: row shards take the column scores of the full
    W (cdclq_column_scores_device) and concatenate to the single-GPU result; the ranking from a shard's own rows
    would differ."""
    import torch

    from cdclq.pipeline import ModelBatch

    cfg = Config(group=32, block=64, sub_block=32, row_chunk=32, passes=3, skeleton_pct=30.0)
    layers, inputs, hs, ws = model(torch, "cuda")
    full = ModelBatch(torch, layers, inputs, hs, ws, cfg)
    full.run(0)
    torch.cuda.synchronize()
    ref = outputs(full)
    assert any(int(o["gbits"][0]) == cfg.skeleton_bits for o in ref)  # the skeleton is in use
    world = 2
    parts = []
    for rank in range(world):
        mb = ModelBatch(torch, layers, inputs, hs, ws, cfg, rank=rank, world=world, distribute_factors=False)
        mb.run(0)
        torch.cuda.synchronize()
        parts.append(dict(zip(mb.names, zip(mb.shards, outputs(mb)))))
    for li, (name, d_out, _, _) in enumerate(layers):
        rows = sorted((p[name] for p in parts if name in p), key=lambda x: x[0][0])
        for k in ("codes", "scales", "zeros"):
            assert np.array_equal(np.concatenate([o[k] for _, o in rows]), ref[li][k]), (name, k)
        for _, o in rows:
            assert np.array_equal(o["perm"], ref[li]["perm"]) and np.array_equal(o["gbits"], ref[li]["gbits"])


def test_layer_factors_give_the_batch_result(gpu):
    """Skeleton permutations are per layer: cdclq_prepare_layer_factors computes a layer's factor for its own
    permutation, and a batch given those factors (descriptor field `u`) returns the single-call result bit for
    bit; one layer is left to factorise inside the call."""
    import torch

    import cdclq
    from cdclq.pipeline import ModelBatch

    cfg = Config(group=32, block=64, sub_block=32, row_chunk=32, passes=3, skeleton_pct=30.0)
    layers, inputs, hs, ws = model(torch, "cuda")
    ref = ModelBatch(torch, layers, inputs, hs, ws, cfg)
    ref.run(0)
    torch.cuda.synchronize()
    mb = ModelBatch(torch, layers, inputs, hs, ws, cfg)
    us = [torch.full((NS[inp], NS[inp]), float("nan"), dtype=torch.float32, device="cuda") for (inp, _) in SPECS]
    mine = [0, 1, 3, 4]  # layer 2 is factorised inside the batch call
    which = (ctypes.c_size_t * len(mine))(*mine)
    u_out = (ctypes.c_void_p * len(mine))(*[us[i].data_ptr() for i in mine])
    c = cfg.to_c()
    L = cdclq.lib()
    cdclq._lib.check(L.cdclq_prepare_layer_factors(mb.ins, len(NS), mb.lys, len(mb.lys),
                                                   ctypes.cast(which, ctypes.c_void_p), len(mine), ctypes.byref(c),
                                                   ctypes.cast(u_out, ctypes.c_void_p), 1, None))
    torch.cuda.synchronize()
    for i in mine:  # strictly lower part exactly 0, positive diagonal (src/linalg.rs:498-503)
        u = us[i].cpu().numpy()
        assert np.all(np.tril(u, -1) == 0.0) and np.all(np.diag(u) > 0.0)
    # layers 0 and 1 share an input but not a permutation: their factors differ
    assert not torch.equal(us[0], us[1])
    for i in mine:
        mb.lys[i].u = us[i].data_ptr()
    cdclq._lib.check(L.cdclq_quantize_batch(mb.ins, len(NS), mb.lys, len(mb.lys), ctypes.byref(c), 1, None))
    torch.cuda.synchronize()
    assert_same(outputs(mb), outputs(ref))
    for s, r in zip(mb.stats, ref.stats):
        assert s.loss_gptq == r.loss_gptq and s.loss_final == r.loss_final and s.code_updates == r.code_updates
