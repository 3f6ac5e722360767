"""Host logic of the multi-GPU path (cdclq.pipeline) without a GPU: row shards, the factorisation owners,
the factor exchange over a world-size-2 gloo process group, and the prepared-factor entry points' argument
checks."""
import ctypes
import os
import socket

import pytest
from conftest import ROOT

TINYLLAMA_INPUTS = [2048, 2048, 2048, 5632] * 22


def test_shard_rows_cover_every_row_in_whole_chunks():
    from cdclq.pipeline import shard_rows

    for d_out in (1, 64, 127, 128, 129, 256, 1000, 2048, 5632):
        for rc in (16, 100, 128):
            for world in (1, 2, 3, 4, 8):
                for rotate in (0, 1, 5):
                    spans = sorted(shard_rows(d_out, rc, r, world, rotate) for r in range(world))
                    assert spans[0][0] == 0 and spans[-1][1] == d_out
                    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                        assert a1 == b0  # the ranks' ranges tile the rows without overlap
                    for r0, r1 in spans:
                        assert r0 <= r1
                        assert r0 % rc == 0  # a shard starts on a row-chunk boundary
                        assert r1 % rc == 0 or r1 == d_out


def test_rotated_shards_balance_a_model():
    """TinyLlama-shaped layers: with the per-layer rotation no rank holds more than one row chunk per layer
    group above the mean."""
    from cdclq.pipeline import shard_rows

    block = [(2048, 2048), (256, 2048), (256, 2048), (2048, 2048), (5632, 2048), (5632, 2048), (2048, 5632)]
    layers = block * 22
    for world in (2, 4, 8):
        load = [0] * world
        for li, (d_out, d_in) in enumerate(layers):
            for r in range(world):
                r0, r1 = shard_rows(d_out, 128, r, world, rotate=li)
                load[r] += (r1 - r0) * d_in * d_in
        assert max(load) <= 1.06 * (sum(load) / world), (world, max(load) / (sum(load) / world))


def test_factorisation_owners_balance_n_cubed():
    from cdclq.pipeline import assign_factorisations

    ns = TINYLLAMA_INPUTS
    for world in (1, 2, 4, 8):
        owner = assign_factorisations(ns, world)
        assert owner == assign_factorisations(ns, world)  # deterministic: every rank derives the same table
        assert set(owner) == set(range(world))
        load = [sum(float(n) ** 3 for n, o in zip(ns, owner) if o == r) for r in range(world)]
        # LPT bound: no rank above the mean by more than the largest single job
        assert max(load) <= sum(load) / world + 5632.0 ** 3 + 1.0
    # the 22 widest inputs (the down projections) are spread first, one per rank in turn
    owner = assign_factorisations(ns, 8)
    down = [owner[i] for i in range(3, len(ns), 4)]
    assert sorted(down[:8]) == list(range(8))


def test_hessian_owners_balance_n_squared():
    """Hessian accumulations (cost n^2 at a fixed token count) of the Llama-2-7B-shaped model: 96 inputs of
    4096 and 32 of 11008 channels spread by LPT on n^2 within one job of the mean."""
    from cdclq.pipeline import assign_factorisations

    ns = [4096, 4096, 4096, 11008] * 32
    for world in (2, 4, 8):
        owner = assign_factorisations(ns, world, power=2)
        load = [sum(float(n) ** 2 for n, o in zip(ns, owner) if o == r) for r in range(world)]
        assert max(load) <= sum(load) / world + 11008.0 ** 2 + 1.0
        assert set(owner) == set(range(world))


def test_prepared_entry_points_reject_a_weight_dependent_permutation():
    import cdclq
    from cdclq.abi import CBatchInput, Config

    L = cdclq.lib()
    c = Config(skeleton_pct=2.0).to_c()
    ins = (CBatchInput * 1)()
    ins[0].n = 64
    u = (ctypes.c_void_p * 1)(None)
    which = (ctypes.c_size_t * 1)(0)
    rc = L.cdclq_prepare_factors(ins, 1, ctypes.cast(which, ctypes.c_void_p), 1, ctypes.byref(c),
                                 ctypes.cast(u, ctypes.c_void_p), 1, None)
    assert rc == -1  # CDCLQ_ERR_CONFIG
    assert L.cdclq_last_error().decode() == "prepared factors need a W-independent permutation (skeleton_pct = 0)"
    rc = L.cdclq_quantize_batch_prepared(ins, 1, ctypes.cast(u, ctypes.c_void_p), None, 0, ctypes.byref(c), 1, None)
    assert rc == -1
    rc = L.cdclq_quantize_batch_prepared(ins, 1, None, None, 0, ctypes.byref(Config().to_c()), 1, None)
    assert rc == -3 and L.cdclq_last_error().decode() == "null argument"  # CDCLQ_ERR_ARG


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_worker(rank, world, port, q):
    import sys

    sys.path.insert(0, os.path.join(ROOT, "cdcl-gptq_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from cdclq.pipeline import assign_factorisations, exchange_factors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ns = [8, 16, 8, 24, 16]
        owner = assign_factorisations(ns, world)
        # each rank fills only the factors it owns; the others hold garbage before the exchange
        fac = []
        for i, n in enumerate(ns):
            t = torch.full((n, n), -1.0)
            if owner[i] == rank:
                t = torch.arange(n * n, dtype=torch.float32).reshape(n, n) + 1000.0 * i
            fac.append(t)
        exchange_factors(fac, owner)
        ok = all(torch.equal(t, torch.arange(n * n, dtype=torch.float32).reshape(n, n) + 1000.0 * i)
                 for i, (t, n) in enumerate(zip(fac, ns)))
        q.put((rank, ok, owner))
    finally:
        dist.destroy_process_group()


def test_factor_exchange_two_ranks_gloo():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert all(ok for _, ok, _ in res)
    assert res[0][2] == res[1][2]  # both ranks derived the same owners


def test_skeleton_shards_need_the_full_weights():
    """Row shards with a skeleton: the column ranking needs the whole W, so rank-local weight shards are refused
    before anything is allocated."""
    import torch

    from cdclq.abi import Config
    from cdclq.pipeline import ModelBatch

    cfg = Config(group=32, row_chunk=32, skeleton_pct=30.0)
    with pytest.raises(ValueError, match="whole weight matrix"):
        ModelBatch(torch, [("l0", 64, 128, 0)], [("in0", 128)], [None], [None], cfg, rank=0, world=2, w_sharded=True)
