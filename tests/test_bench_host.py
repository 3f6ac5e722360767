"""The bench's workloads match the configurations they are quoted on (BASELINE.json configs[1]-[3]), without a
GPU: layer shapes, distinct inputs, weight counts and quantizer settings."""
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)


def test_configs1_tinyllama_shape_and_settings():
    import bench

    layers, inputs = bench.model_layers()
    assert len(layers) == 154 and len(inputs) == 88
    assert sum(l[1] * l[2] for l in layers) == 968_884_224  # 9.69e8 weights
    cfg = bench.bench_config()
    assert (cfg.bits, cfg.group, bool(cfg.mse_grid), cfg.row_chunk) == (3, 128, True, 128)
    assert bench.TOKENS == 128 * 2048


def test_configs3_llama2_7b_shape_and_settings():
    import argparse

    import bench

    layers, inputs = bench.spec_layers(bench.MODEL_SPECS["llama2-7b"])
    assert len(layers) == 224 and len(inputs) == 128
    assert sum(l[1] * l[2] for l in layers) == 6_476_005_376  # 6.48e9 weights
    assert sorted({n for _, n in inputs}) == [4096, 11008]
    for bits in (4, 2):
        cfg = bench.model_config("llama2-7b", argparse.Namespace(bits=bits, group=0))
        assert (cfg.bits, cfg.group, bool(cfg.mse_grid), cfg.refine_frac, cfg.row_chunk) == (bits, 64, True, 0.25, 128)
    # the north star's literal 4-bit / g128 setting
    assert bench.model_config("llama2-7b", argparse.Namespace(bits=4, group=128)).group == 128


def test_configs2_gemma2b_shape_and_settings():
    import argparse

    import bench

    spec = bench.MODEL_SPECS["gemma2b"]
    layers, inputs = bench.spec_layers(spec)
    assert len(layers) == 126 and len(inputs) == 72
    assert sum(l[1] * l[2] for l in layers) == 1_981_808_640  # 1.98e9 weights
    kv = [l for l in layers if l[0].endswith(("k_proj", "v_proj"))]
    assert all(l[1] == 256 for l in kv)  # one KV head of dim 256
    cfg = bench.model_config("gemma2b", argparse.Namespace(bits=4, group=0))
    assert (cfg.bits, cfg.group, cfg.skeleton_pct, cfg.skeleton_bits) == (4, 128, 2.0, 8)
    assert spec["tokens"] == "student3" and not spec["hessians_timed"]


def test_reference_arm_job_order_and_prep_reuse():
    """The CPU reference arm steps through the decoder layer in the reference's job order (sorted by Hessian owner,
    then name: src/pipeline.rs:109-112), one linear layer per step, with the prep cache shared within an owner."""
    import torch

    import bench
    from cdclq.abi import Config

    layers = [("m.0.q_proj", 32, 64, 0), ("m.0.k_proj", 16, 64, 0), ("m.0.v_proj", 16, 64, 0), ("m.0.o_proj", 32, 64, 1),
              ("m.0.gate_proj", 48, 64, 2), ("m.0.up_proj", 48, 64, 2), ("m.0.down_proj", 64, 48, 3)]
    order = bench.reference_jobs(layers)
    assert [layers[i][0] for i in order] == ["m.0.down_proj", "m.0.gate_proj", "m.0.up_proj", "m.0.o_proj",
                                             "m.0.k_proj", "m.0.q_proj", "m.0.v_proj"]
    inputs = [("m.0.attn", 64), ("m.0.o", 64), ("m.0.mlp", 64), ("m.0.down", 48)]
    H = [bench.make_hessian(n, 10 + i, 256, torch, "cpu") for i, (_, n) in enumerate(inputs)]
    W = [bench.make_weight(d, n, 20 + i, torch, "cpu") for i, (_, d, n, _) in enumerate(layers)]
    cfg = Config(bits=3, group=32, block=32, sub_block=16, row_chunk=16, passes=2)
    ref = bench.CpuReference(layers, inputs, H, W, cfg, 2)
    seen = [ref.step()[0] for _ in range(7)]
    assert seen == order and sorted(ref.results) == list(range(7))
    assert ref.decoder_layer_seconds({li: [0.5] for li in range(7)}) == 3.5


def test_reference_arm_uses_every_host_core_under_torchrun():
    """torchrun sets OMP_NUM_THREADS=1 for every rank; the reference arm pins the oracle's threads to the process's
    CPU affinity regardless."""
    import os
    import subprocess

    import bench

    code = ("import sys; sys.path[:0] = [%r, %r, %r]; import bench, torch; from cdclq.abi import Config; "
            "ref = bench.CpuReference([], [], [], [], Config(), bench.host_cores()); "
            "print(ref.orc.max_threads())") % (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "cdcl-gptq_b200"))
    out = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, OMP_NUM_THREADS="1"), capture_output=True,
                         text=True, check=True).stdout.split()[-1]
    assert int(out) == bench.host_cores()
