"""Host logic of the multi-GPU runtime, without a GPU: the row sharding and the factorisation owners the library
uses (cdclq_shard_rows, cdclq_assign_owners) against the Python pipeline's, and the unique-id exchange over a
world-size-2 gloo process group (the N > 1 path's plumbing on CPU)."""
import os

import pytest
import torch.multiprocessing as mp


def test_shard_rows_match_the_python_pipeline():
    from cdclq.pipeline import shard_rows as py_shard
    from cdclq.runtime import shard_rows

    for d_out in (1, 37, 100, 128, 129, 1000, 5632):
        for rc in (1, 32, 64, 128, 256):
            for world in (1, 2, 3, 4, 8):
                for rot in (0, 1, 5):
                    spans = [shard_rows(d_out, rc, r, world, rot) for r in range(world)]
                    assert spans == [py_shard(d_out, rc, r, world, rotate=rot) for r in range(world)]
                    covered = sorted(spans)
                    assert covered[0][0] == 0 and covered[-1][1] == d_out
                    for (a0, a1), (b0, b1) in zip(covered, covered[1:]):
                        assert a1 == b0  # contiguous, disjoint
                    for a0, a1 in spans:
                        assert a0 % rc == 0 and (a1 % rc == 0 or a1 == d_out)  # whole row chunks


def test_owners_match_the_python_pipeline():
    from cdclq.pipeline import assign_factorisations
    from cdclq.runtime import assign_owners

    ns = [2048, 2048, 2048, 5632] * 22
    for world in (1, 2, 4, 8):
        for power in (2, 3):
            assert assign_owners(ns, world, power) == assign_factorisations(ns, world, power=power)
    assert assign_owners([11008, 4096, 4096, 4096], 2) == [0, 1, 1, 1]


def _uid_rank(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from cdclq.runtime import shared_unique_id

    q.put((rank, shared_unique_id()))
    dist.destroy_process_group()


def test_unique_id_exchange_over_gloo():
    from cdclq.runtime import UNIQUE_ID_BYTES

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_uid_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(got[0]) == UNIQUE_ID_BYTES and got[0] == got[1]


def test_model_requires_an_output():
    import cdclq
    from cdclq.runtime import QuantOpts, quantize_model

    with pytest.raises(cdclq.CdclqError) as ei:
        quantize_model(QuantOpts(["m.safetensors"], ["h.safetensors"], "/tmp/none", emit_packed=False,
                                 emit_dequant=False))
    assert str(ei.value) == "nothing to write: both --no-packed and --no-dequant are set"


def test_runtime_first_then_torch_shares_one_nccl():
    """A process that opens the runtime's NCCL before importing torch (a Rust or C caller embedding Python, a
    worker that builds its runtime first) must still be able to import torch: the library opens the NCCL copy
    torch will use, not the first libnccl.so.2 on the loader's path."""
    import subprocess
    import sys

    from conftest import ROOT

    code = ("import sys; sys.path.insert(0, %r); import cdclq.runtime as r; assert len(r.unique_id()) == 128; "
            "import torch; print('ok')") % os.path.join(ROOT, "cdcl-gptq_b200")
    env = {k: v for k, v in os.environ.items() if k != "CDCLQ_NCCL_LIBRARY"}
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]
