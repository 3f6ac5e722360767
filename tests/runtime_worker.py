"""One rank of the multi-GPU runtime tests (tests/test_gpu_runtime.py), run as its own process.

    python tests/runtime_worker.py <case> <rank> <world> <workdir>

Rank 0 makes the NCCL unique id and writes it to <workdir>/uid; the other ranks wait for it (bounded).  Cases:
  batch / skeleton / auto_chunk   Runtime.quantize_batch of tests' synthetic batch (host buffers, gathered on
                                  rank 0); outputs and statistics saved to <workdir>/r<rank>.npz
  model                           cdclq_quantize_model of the toy checkpoint over the ranks into <workdir>/out
  bad_arg                         rank 1 passes an invalid configuration: every rank must fail, rank 0 with
                                  "rank 1 failed: ..." (host-side failure, no GPU fault)
  leave                           rank 1 leaves after joining, between steps; rank 0's next call must end with an
                                  error within its (short) timeout
TEST INFRASTRUCTURE ONLY.
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "cdcl-gptq_b200")):
    sys.path.insert(0, p)


def synthetic_batch(case):
    """(Hessians, [(input, W)], cfg): widths 64 / 128 / 96, layers of 1000 (ragged chunks), 100 (one chunk: some
    ranks hold none of its rows), 300 and 37 rows."""
    import oracle as orc
    from cdclq.abi import Config

    ns = [64, 128, 96]
    hs = [orc.problem(1, n, 4 * n, 300 + i)[1] for i, n in enumerate(ns)]
    specs = [(0, 1000), (0, 100), (1, 300), (2, 37), (1, 256), (0, 129)]
    ws = [orc.rng_normal(400 + k, d * ns[i], 0.04).reshape(d, ns[i]) for k, (i, d) in enumerate(specs)]
    if case == "skeleton":
        cfg = Config(bits=3, group=16, block=32, sub_block=16, skeleton_pct=25.0, row_chunk=64, passes=3)
    elif case == "auto_chunk":
        cfg = Config(bits=4, group=32, block=32, sub_block=16, row_chunk=0, threads=8, passes=2)
    else:
        cfg = Config(bits=3, group=32, block=32, sub_block=16, row_chunk=64, passes=3, mse_grid=True)
    return hs, [(i, w) for (i, _), w in zip(specs, ws)], cfg


def save_batch(path, outs, stats):
    d = {}
    for k, (o, s) in enumerate(zip(outs, stats)):
        for key, v in o.items():
            d["%s_%d" % (key, k)] = v
        d["stats_%d" % k] = np.array([s.loss_gptq, s.loss_final, s.code_updates, s.subblocks_total,
                                      s.subblocks_refined, s.skeleton_groups, s.bits_total, s.passes_max], np.float64)
    np.savez(path, **d)


def main():
    case, rank, world, work = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    from cdclq import CdclqError
    from cdclq.runtime import QuantOpts, Runtime, batch_tables, quantize_model, unique_id

    uid_path = os.path.join(work, "uid")
    if rank == 0:
        with open(uid_path + ".tmp", "wb") as f:
            f.write(unique_id())
        os.rename(uid_path + ".tmp", uid_path)
    t0 = time.time()
    while not os.path.exists(uid_path):
        if time.time() - t0 > 60:
            raise SystemExit("no unique id from rank 0")
        time.sleep(0.05)
    with open(uid_path, "rb") as f:
        uid = f.read()
    timeout = 20.0 if case == "leave" else 180.0
    rt = Runtime(device=rank, nranks=world, rank=rank, uid=uid, timeout_s=timeout)
    if case in ("batch", "skeleton", "auto_chunk"):
        hs, layers, cfg = synthetic_batch(case)
        ins, lys, outs, stats, keep = batch_tables(hs, layers, cfg)
        rt.quantize_batch(ins, lys, cfg, on_device=False, gather=True)
        save_batch(os.path.join(work, "r%d.npz" % rank), outs, stats)
    elif case == "model":
        import toy_model
        from cdclq.abi import Config

        model, hess, _, _ = toy_model.write(os.path.join(work, "in%d" % rank), "bf16")
        cfg = Config(bits=3, group=32, block=32, sub_block=16, row_chunk=32, passes=3)
        quantize_model(QuantOpts([model], [hess], os.path.join(work, "out"), cfg), runtime=rt)
    elif case == "bad_arg":
        hs, layers, cfg = synthetic_batch("batch")
        if rank == 1:
            cfg = cfg.replace(refine_frac=2.0)  # only this rank's configuration is invalid
        ins, lys, outs, stats, keep = batch_tables(hs, layers, cfg)
        try:
            rt.quantize_batch(ins, lys, cfg, on_device=False, gather=True)
            msg = "no error"
        except CdclqError as e:
            msg = "%d|%s" % (e.code, e)
        with open(os.path.join(work, "msg%d" % rank), "w") as f:
            f.write(msg)
    elif case == "leave":
        if rank != 0:
            rt.close()  # leaves between steps: nothing of it is in flight
            return
        hs, layers, cfg = synthetic_batch("batch")
        ins, lys, outs, stats, keep = batch_tables(hs, layers, cfg)
        t1 = time.time()
        try:
            rt.quantize_batch(ins, lys, cfg, on_device=False, gather=True)
            msg = "no error"
        except CdclqError as e:
            msg = "%d|%s" % (e.code, e)
        with open(os.path.join(work, "msg0"), "w") as f:
            f.write("%.1f|%s" % (time.time() - t1, msg))
        return  # the runtime is broken; the process exits without using it again
    rt.close()


if __name__ == "__main__":
    main()
