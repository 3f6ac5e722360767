"""The multi-GPU runtime (cdclq_runtime_*) against one GPU: one process per rank (tests/runtime_worker.py).

Every rank-sharded result must equal the single-GPU batch bit for bit (codes, scales, zero points, permutation,
group widths; accepted moves and sub-block counts), with the f64 loss sums within 1e-12 relative (the ranks'
partial sums are added by an all-reduce, one GPU adds its row chunks in order).  Cases: act-order with the MSE
grid, a skeleton (its column scores summed rank by rank in row order), the automatic row chunk, and the model
pipeline (output files identical to one GPU's).  Failure detection without any GPU fault: a rank whose own
configuration is invalid makes every rank fail with its message; a rank that leaves between steps makes the
others' next call end with an error within their short timeout.  NVLS is off in these runs.  Needs >= 2 GPUs.
"""
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
WORKER = os.path.join(ROOT, "tests", "runtime_worker.py")


def gpu_count():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


need2 = pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")


def run_ranks(case, world, work, timeout=420):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONUNBUFFERED="1")
    procs = [subprocess.Popen([sys.executable, WORKER, case, str(r), str(world), str(work)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(world)]
    t0, outs = time.time(), []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=max(1.0, timeout - (time.time() - t0)))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise AssertionError("%s: a rank did not finish in %d s" % (case, timeout))
        outs.append((p.returncode, out))
    return outs


def single_gpu_batch(case):
    import ctypes

    import cdclq
    from cdclq.runtime import batch_tables
    from runtime_worker import synthetic_batch

    hs, layers, cfg = synthetic_batch(case)
    ins, lys, outs, stats, keep = batch_tables(hs, layers, cfg)
    c = cfg.to_c()
    cdclq._lib.check(cdclq.lib().cdclq_quantize_batch(ins, len(hs), lys, len(layers), ctypes.byref(c), 0, None))
    return outs, stats


@need2
@pytest.mark.parametrize("case", ["batch", "skeleton", "auto_chunk"])
def test_runtime_batch_equals_one_gpu(gpu, tmp_path, case):
    world = 2
    res = run_ranks(case, world, tmp_path)
    for rc, out in res:
        assert rc == 0, out[-3000:]
    outs, stats = single_gpu_batch(case)
    for r in range(world):
        z = np.load(str(tmp_path / ("r%d.npz" % r)))
        for k, (o, s) in enumerate(zip(outs, stats)):
            for key in ("perm", "gbits"):
                assert np.array_equal(z["%s_%d" % (key, k)], o[key]), (r, k, key)
            st = z["stats_%d" % k]
            assert abs(st[0] - s.loss_gptq) <= 1e-12 * s.loss_gptq and abs(st[1] - s.loss_final) <= 1e-12 * s.loss_final
            assert (st[2], st[3], st[4], st[5]) == (s.code_updates, s.subblocks_total, s.subblocks_refined,
                                                    s.skeleton_groups), (r, k)
            assert st[6] == s.bits_total and st[7] == s.passes_max
            if r == 0:  # gathered: every row
                for key in ("codes", "scales", "zeros"):
                    assert np.array_equal(z["%s_%d" % (key, k)], o[key]), (case, k, key)


@need2
def test_runtime_model_equals_one_gpu(gpu, tmp_path):
    import json

    import toy_model
    from cdclq.abi import Config
    from cdclq.runtime import QuantOpts, quantize_model

    res = run_ranks("model", 2, tmp_path)
    for rc, out in res:
        assert rc == 0, out[-3000:]
    model, hess, _, _ = toy_model.write(str(tmp_path / "in_single"), "bf16")
    cfg = Config(bits=3, group=32, block=32, sub_block=16, row_chunk=32, passes=3)
    single = str(tmp_path / "single")
    quantize_model(QuantOpts([model], [hess], single, cfg))
    for sub in ("dequant", "packed"):
        a = open(os.path.join(single, sub, "model.safetensors"), "rb").read()
        b = open(str(tmp_path / "out" / sub / "model.safetensors"), "rb").read()
        assert a == b, sub
    ra = json.load(open(os.path.join(single, "report.json")))
    rb = json.load(open(str(tmp_path / "out" / "report.json")))
    for la, lb in zip(ra["layers"], rb["layers"]):
        assert la["name"] == lb["name"] and la["code_updates"] == lb["code_updates"]
        assert abs(la["loss_final"] - lb["loss_final"]) <= 1e-12 * la["loss_final"]


@need2
def test_runtime_one_rank_fails_all_fail(gpu, tmp_path):
    res = run_ranks("bad_arg", 2, tmp_path)
    for rc, out in res:
        assert rc == 0, out[-3000:]
    m0 = open(str(tmp_path / "msg0")).read()
    m1 = open(str(tmp_path / "msg1")).read()
    assert m1 == "-1|refine_frac must be in [0, 1]"
    assert m0 == "-1|rank 1 failed: refine_frac must be in [0, 1]"


@need2
def test_runtime_rank_leaving_ends_the_others_call(gpu, tmp_path):
    res = run_ranks("leave", 2, tmp_path, timeout=180)
    for rc, out in res:
        assert rc == 0, out[-3000:]
    secs, code, msg = open(str(tmp_path / "msg0")).read().split("|", 2)
    assert code == "-4" and float(secs) < 20.0 + 30.0, (secs, msg)
