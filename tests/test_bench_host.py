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
