"""Hessian capture host logic without a GPU: pass planning (scripts/capture_hessians.py:73-99), output names,
and the shared-input probe on a tiny random Llama (:187-213)."""
import pytest


def tiny_llama(torch, dtype=None):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256)
    torch.manual_seed(0)
    m = LlamaForCausalLM(cfg).eval()
    return m.to(dtype) if dtype is not None else m


def test_plan_bins_first_fit_decreasing():
    from cdclq.capture import accumulator_bytes, plan_bins

    fam = {"a.q": 100, "b.down": 200, "c.q": 100, "d.o": 50}
    bins = plan_bins(fam, accumulator_bytes(200) + accumulator_bytes(100))
    assert [b["owners"] for b in bins] == [["b.down", "a.q"], ["c.q", "d.o"]]  # largest first, ties by name
    assert bins[1]["bytes"] == accumulator_bytes(100) + accumulator_bytes(50)
    assert len(plan_bins(fam, 10 ** 12)) == 1


def test_plan_bins_refuses_a_layer_above_the_budget():
    from cdclq.capture import accumulator_bytes, plan_bins

    with pytest.raises(ValueError, match="b.down: a single Hessian at d_in=200"):
        plan_bins({"b.down": 200}, accumulator_bytes(200) - 1)


def test_out_path_for():
    from cdclq.capture import out_path_for

    assert out_path_for("d/h.safetensors", 1, 1) == "d/h.safetensors"
    assert out_path_for("d/h.safetensors", 2, 3) == "d/h.2of3.safetensors"


def test_probe_finds_shared_inputs():
    import torch

    from cdclq.capture import linear_targets, probe_aliases

    m = tiny_llama(torch)
    t = linear_targets(m)
    assert len(t) == 14 and not any("lm_head" in n for n, _ in t)
    al = probe_aliases(m, t, torch.randint(0, 256, (1, 16)))
    for b in range(2):
        p = "model.layers.%d." % b
        assert al[p + "self_attn.k_proj"] == p + "self_attn.q_proj"
        assert al[p + "self_attn.v_proj"] == p + "self_attn.q_proj"
        assert al[p + "mlp.up_proj"] == p + "mlp.gate_proj"
    assert len(al) == 6
    assert [n for n, _ in linear_targets(m, only=("mlp",))][:3] == ["model.layers.0.mlp.gate_proj",
                                                                     "model.layers.0.mlp.up_proj",
                                                                     "model.layers.0.mlp.down_proj"]


def test_capture_needs_a_gpu_model():
    import torch

    from cdclq.capture import capture

    with pytest.raises(RuntimeError, match="CUDA"):
        capture(tiny_llama(torch), [torch.randint(0, 256, (2, 8))])
