"""A small Llama-shaped checkpoint and its Hessian file, for the model-level pipeline tests.

Mirrors the reference's end-to-end fixtures (tests/toy_models.rs, tests/fixtures/*/hess.safetensors): two decoder
layers of q/k/v/o, gate/up and down projections plus embeddings, lm_head and norm gains that have no Hessian and
must be copied through; one `.H` per distinct input (k_proj for the attention input, o_proj, gate_proj, down_proj)
and an `aliases` metadata entry for the layers that share one (q/v -> k, up -> gate), like the reference's capture.
The Hessians are seeded Grams (the oracle's problem generator); one down_proj Hessian is the reference's own
fixture (tests/golden/fixture_hessians.npz, 172 wide).  Weights are seeded normals, stored as bf16 or f32.
TEST INFRASTRUCTURE ONLY.
"""
import json
import os

import numpy as np

HIDDEN, INTER, KV, VOCAB = 64, 172, 32, 96


def layer_shapes(n_layers=2):
    """[(tensor name, d_out, d_in, hessian owner layer)]"""
    out = []
    for b in range(n_layers):
        p = "model.layers.%d." % b
        k = p + "self_attn.k_proj"
        out += [(p + "self_attn.q_proj.weight", HIDDEN, HIDDEN, k), (k + ".weight", KV, HIDDEN, k),
                (p + "self_attn.v_proj.weight", KV, HIDDEN, k),
                (p + "self_attn.o_proj.weight", HIDDEN, HIDDEN, p + "self_attn.o_proj"),
                (p + "mlp.gate_proj.weight", INTER, HIDDEN, p + "mlp.gate_proj"),
                (p + "mlp.up_proj.weight", INTER, HIDDEN, p + "mlp.gate_proj"),
                (p + "mlp.down_proj.weight", HIDDEN, INTER, p + "mlp.down_proj")]
    return out


def bf16_round(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def write(dirpath, dtype="bf16", n_layers=2, seed=0, fixture_hessians=None):
    """Writes <dir>/model.safetensors and <dir>/hess.safetensors; returns (model path, hessian path, tensors, H)
    with `tensors` the f32 values of every weight (as stored) and `H` {owner: n x n f32}."""
    import oracle as orc
    import torch
    from safetensors.torch import save_file

    os.makedirs(dirpath, exist_ok=True)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    tensors, H = {}, {}
    for i, (name, d_out, d_in, owner) in enumerate(layer_shapes(n_layers)):
        w = orc.rng_normal(1000 * seed + 10 + i, d_out * d_in, 0.05).reshape(d_out, d_in)
        tensors[name] = bf16_round(w) if dtype == "bf16" else w
        if owner not in H:
            if fixture_hessians is not None and d_in == 172 and "fixture" not in H:
                H[owner] = np.asarray(fixture_hessians, np.float32)
                H["fixture"] = None
            else:
                H[owner] = orc.problem(1, d_in, 4 * d_in, 1000 * seed + 500 + len(H))[1]
    H.pop("fixture", None)
    extra = {"model.embed_tokens.weight": (VOCAB, HIDDEN), "lm_head.weight": (VOCAB, HIDDEN), "model.norm.weight": (HIDDEN,)}
    for b in range(n_layers):
        extra["model.layers.%d.input_layernorm.weight" % b] = (HIDDEN,)
    for j, (name, shape) in enumerate(sorted(extra.items())):
        v = orc.rng_normal(1000 * seed + 900 + j, int(np.prod(shape)), 0.1).reshape(shape)
        tensors[name] = bf16_round(v) if dtype == "bf16" else v
    model = os.path.join(dirpath, "model.safetensors")
    save_file({k: torch.from_numpy(np.ascontiguousarray(v)).to(tdt) for k, v in tensors.items()}, model,
              metadata={"format": "pt"})
    aliases = {}
    for b in range(n_layers):
        p = "model.layers.%d." % b
        aliases[p + "self_attn.q_proj"] = p + "self_attn.k_proj"
        aliases[p + "self_attn.v_proj"] = p + "self_attn.k_proj"
        aliases[p + "mlp.up_proj"] = p + "mlp.gate_proj"
    hess = os.path.join(dirpath, "hess.safetensors")
    save_file({k + ".H": torch.from_numpy(np.ascontiguousarray(v)) for k, v in H.items()}, hess,
              metadata={"format": "cdclq-hessians", "aliases": json.dumps(aliases)})
    return model, hess, tensors, H
