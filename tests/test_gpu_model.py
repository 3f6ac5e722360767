"""The model-level pipeline through the C ABI (cdclq_quantize_model, cdclq_dequantize_packed) on one GPU.

Mirrors the reference's end-to-end test of a checkpoint (tests/toy_models.rs:247-442) on a small Llama-shaped
checkpoint with a Hessian file using aliases (tests/toy_model.py): the fake-quant output is a drop-in replacement
(same tensors, shapes, dtypes); every reported layer has its six packed tensors, which unpack to exactly the
fake-quant values; every code fits its group's width; the loss rebuilt from the packed file alone matches the
tracked loss_final (5e-3) and the repair never raised it; every tensor without a Hessian is copied byte for
byte; the packed header carries quantization=cdclq-v1 and orig_dtype; the packed file expanded by
cdclq_dequantize_packed equals the fake-quant file; and the packed codes are much smaller than the weights.
On top of the reference's checks, every layer is compared bit for bit with the CPU oracle run on the same
weights and Hessian (codes, f16 scales, zero points, permutation, loss_gptq; loss_final within 1e-9).
"""
import json
import os

import numpy as np
import pytest

import oracle as orc
import toy_model
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def load(path):
    """{name: (dtype string, shape, raw bytes, f32 values or None)} plus the metadata of a safetensors file."""
    with open(path, "rb") as f:
        data = f.read()
    hl = int.from_bytes(data[:8], "little")
    hdr = json.loads(data[8:8 + hl])
    meta = hdr.pop("__metadata__", {})
    base = 8 + hl
    out = {}
    for name, e in hdr.items():
        a, b = e["data_offsets"]
        raw = data[base + a:base + b]
        dt = e["dtype"]
        if dt == "F32":
            v = np.frombuffer(raw, np.float32)
        elif dt == "BF16":
            v = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
        elif dt == "F16":
            v = np.frombuffer(raw, np.float16).astype(np.float32)
        else:
            v = None
        out[name] = (dt, tuple(e["shape"]), raw, None if v is None else v.reshape(e["shape"]))
    return out, meta


def rounded_bytes(x, dt):
    x = np.ascontiguousarray(x, np.float32)
    if dt == "F32":
        return x.tobytes()
    if dt == "F16":
        return x.astype(np.float16).tobytes()
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)).tobytes()


def fixture_down():
    return np.load(os.path.join(GOLDEN, "fixture_hessians.npz"))["tiny-random-llama2/model.layers.0.mlp.down_proj.H"]


CFG = dict(bits=3, group=32, block=32, sub_block=16, row_chunk=32, passes=3)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_model_quantize_and_roundtrip(gpu, tmp_path, dtype):
    from cdclq.abi import Config
    from cdclq.io import read_packed_layer
    from cdclq.runtime import QuantOpts, dequantize_packed, quantize_model

    model, hess, tensors, H = toy_model.write(str(tmp_path / "in"), dtype, fixture_hessians=fixture_down())
    out = str(tmp_path / "out")
    cfg = Config(**CFG)
    rep = quantize_model(QuantOpts([model], [hess], out, cfg, verbose=True))
    layers = rep["layers"]
    assert len(layers) == 14 and rep["_totals"]["layers"] == 14
    assert rep["config"].startswith("Config { bits: 3, group: 32, block: 32, damp: 0.01, act_order: true")
    orig, _ = load(model)
    deq, _ = load(os.path.join(out, "dequant", "model.safetensors"))
    pk, pmeta = load(os.path.join(out, "packed", "model.safetensors"))

    # (1) drop-in replacement: same tensors, shapes, dtypes
    assert set(orig) == set(deq)
    for k in orig:
        assert orig[k][:2] == deq[k][:2], k
    owners = {n[:-len(".weight")]: o for (n, _, _, o) in toy_model.layer_shapes()}
    quantized = set()
    for L in layers:
        name = L["name"]
        quantized.add(name + ".weight")
        # (2) the six packed tensors, unpacking to exactly the fake-quant values
        tens = {}
        for suf in ("qweight", "scales", "qzeros", "perm", "gbits", "gsize"):
            dt, sh, raw, v = pk[name + "." + suf]
            np_dt = {"U8": np.uint8, "F16": np.float16, "I32": np.int32}[dt]
            tens[name + "." + suf] = np.frombuffer(raw, np_dt).reshape(sh)
        ql = read_packed_layer(tens, name)
        assert (ql.d_out, ql.d_in) == (L["d_out"], L["d_in"])
        via_reader = ql.dequantize()
        dt = deq[name + ".weight"][0]
        assert rounded_bytes(via_reader, dt) == deq[name + ".weight"][2], name
        # (3) codes fit their group's width
        maxc = (1 << ql.gbits.astype(np.int64)[np.arange(ql.d_in) // ql.group]) - 1
        assert np.all(ql.codes <= maxc[None, :]), name
        # bit-exact against the CPU oracle on the same weights and Hessian
        w = tensors[name + ".weight"]
        h = H[owners[name]]
        qb, sb = orc.quantize_layer(w, L["d_out"], L["d_in"], h, None, owners[name], cfg)
        assert np.array_equal(ql.perm, qb.perm) and np.array_equal(ql.codes, qb.codes), name
        assert np.array_equal(ql.scales, qb.scales) and np.array_equal(ql.zeros, qb.zeros), name
        assert L["loss_gptq"] == sb.loss_gptq, name
        assert abs(L["loss_final"] - sb.loss_final) <= 1e-9 * sb.loss_final, name
        assert L["code_updates"] == sb.code_updates and L["subblocks_refined"] == sb.subblocks_refined
        assert L["bits_total"] == sb.bits_total
        # (4) the loss rebuilt from the packed file alone
        # the damped permuted Hessian rebuilt independently (src/engine.rs:320-342)
        hdiag = np.diag(h)
        w0 = np.where(hdiag[None, :] == 0.0, 0.0, w)
        p = ql.perm.astype(np.int64)
        hp = h.astype(np.float64)[np.ix_(p, p)]
        d = hp.diagonal().copy()
        d[d == 0.0] = 1.0
        hp[np.diag_indices(len(p))] = d + cfg.damp * (np.cumsum(d)[-1] / len(p))
        g = ql.group
        s = np.repeat(ql.scales, g, axis=1)[:, :ql.d_in]
        z = np.repeat(ql.zeros, g, axis=1)[:, :ql.d_in]
        e = (w0[:, p] - (s * (ql.codes.astype(np.float32) - z)).astype(np.float32)).astype(np.float64)
        loss = float(np.sum((e @ hp) * e))
        assert abs(loss - L["loss_final"]) / loss <= 5e-3, (name, loss, L["loss_final"])
        assert L["loss_final"] <= L["loss_gptq"] * (1 + 1e-9)
    # (5) pass-through is exact
    untouched = [k for k in orig if k not in quantized]
    for k in untouched:
        assert orig[k][2] == deq[k][2] and orig[k][2] == pk[k][2], k
    assert len(untouched) >= 2 and "lm_head.weight" in untouched and "model.embed_tokens.weight" in untouched
    # (6) the packed header
    assert pmeta.get("quantization") == "cdclq-v1" and pmeta.get("orig_dtype") == {"bf16": "BF16", "f32": "F32"}[dtype]
    assert pmeta.get("bits") == "3" and pmeta.get("format") == "pt"
    # (7) cdclq dequant reproduces dequant/
    rt = os.path.join(out, "roundtrip", "model.safetensors")
    assert dequantize_packed(os.path.join(out, "packed", "model.safetensors"), rt) == len(layers)
    rts, _ = load(rt)
    assert set(rts) == set(orig)
    for k in orig:
        assert rts[k][:2] == orig[k][:2] and rts[k][2] == deq[k][2], k
    # (8) packed codes are much smaller than the weights they replace
    orig_bytes = sum(len(orig[k][2]) for k in quantized)
    qw_bytes = sum(len(v[2]) for k, v in pk.items() if k.endswith(".qweight"))
    assert qw_bytes * 2 < orig_bytes
    # the report on disk
    with open(os.path.join(out, "report.json")) as f:
        disk = json.load(f)
    assert abs(disk["total_loss_final"] - sum(L["loss_final"] for L in layers)) <= 1e-9 * disk["total_loss_final"]
    assert disk["total_gain_pct"] > 0.0


def test_model_filters_aliases_and_errors(gpu, tmp_path):
    """--only / --skip by substring, layers without a Hessian left untouched, and the reference's messages for a
    width mismatch, a non-finite Hessian and an empty run."""
    import torch
    from safetensors.torch import load_file, save_file

    import cdclq
    from cdclq.abi import Config
    from cdclq.runtime import QuantOpts, dequantize_packed, quantize_model

    model, hess, _, H = toy_model.write(str(tmp_path / "in"), "bf16")
    cfg = Config(**CFG)
    rep = quantize_model(QuantOpts([model], [hess], str(tmp_path / "o1"), cfg, only=["mlp"], skip=["down"]))
    assert sorted(L["name"] for L in rep["layers"]) == sorted(
        "model.layers.%d.mlp.%s" % (b, k) for b in (0, 1) for k in ("gate_proj", "up_proj"))
    rep = quantize_model(QuantOpts([model], [hess], str(tmp_path / "o2"), cfg, emit_packed=False))
    assert not os.path.exists(tmp_path / "o2" / "packed") and len(rep["layers"]) == 14
    # a later Hessian file overrides an earlier one: a wrong width for layer 1's down_proj
    bad = {"model.layers.1.mlp.down_proj.H": torch.ones(64, 64) + torch.eye(64)}
    save_file(bad, str(tmp_path / "bad.safetensors"))
    with pytest.raises(cdclq.CdclqError) as ei:
        quantize_model(QuantOpts([model], [hess, str(tmp_path / "bad.safetensors")], str(tmp_path / "o3"), cfg))
    assert str(ei.value) == "model.layers.1.mlp.down_proj: Hessian is 64x64 but the weight has 172 input columns"
    # a non-finite entry is refused at load time, named by tensor and position
    hs = load_file(hess)
    h = hs["model.layers.0.self_attn.o_proj.H"].clone()
    h[3, 5] = float("nan")
    save_file({"model.layers.0.self_attn.o_proj.H": h}, str(tmp_path / "nan.safetensors"))
    with pytest.raises(cdclq.CdclqError) as ei:
        quantize_model(QuantOpts([model], [hess, str(tmp_path / "nan.safetensors")], str(tmp_path / "o4"), cfg))
    assert str(ei.value) == ("model.layers.0.self_attn.o_proj.H: 64 x 64 matrix has a non-finite entry (NaN) at "
                             "[ 3, 5 ]; the calibration data or the captured forward is corrupt, refusing to quantize")
    # no Hessian matches: nothing quantized, everything copied
    save_file({"unrelated.H": torch.eye(8)}, str(tmp_path / "none.safetensors"))
    rep = quantize_model(QuantOpts([model], [str(tmp_path / "none.safetensors")], str(tmp_path / "o5"), cfg))
    assert rep["layers"] == [] and rep["total_loss_gptq"] == 0.0
    with pytest.raises(cdclq.CdclqError) as ei:
        quantize_model(QuantOpts([model], [hess], str(tmp_path / "o6"), cfg, emit_packed=False, emit_dequant=False))
    assert str(ei.value) == "nothing to write: both --no-packed and --no-dequant are set"
    with pytest.raises(cdclq.CdclqError) as ei:
        dequantize_packed(str(tmp_path / "o1" / "packed" / "model.safetensors"), str(tmp_path / "x.safetensors"),
                          "int4")
    assert str(ei.value) == "unknown dtype int4"
    # explicit output dtype
    n = dequantize_packed(str(tmp_path / "o1" / "packed" / "model.safetensors"), str(tmp_path / "f32.safetensors"),
                          "float32")
    assert n == 4
    f32, _ = load(str(tmp_path / "f32.safetensors"))
    assert f32["model.layers.0.mlp.gate_proj.weight"][0] == "F32" and f32["lm_head.weight"][0] == "BF16"


def test_model_asymmetric_target_layers(gpu, tmp_path):
    """An owner with a cross-covariance `.M` (asymmetric calibration, src/engine.rs:737-755): its layers take the
    single-layer path; the others stay batched.  Every layer equals the oracle."""
    import torch
    from safetensors.torch import load_file, save_file

    from cdclq.abi import Config
    from cdclq.io import read_packed_layer
    from cdclq.runtime import QuantOpts, quantize_model

    model, hess, tensors, H = toy_model.write(str(tmp_path / "in"), "f32", n_layers=1)
    owner = "model.layers.0.mlp.gate_proj"
    _, m = orc.problem(1, 64, 600, 77)
    m = (0.5 * H[owner] + 0.5 * m).astype(np.float32)
    hs = dict(load_file(hess))
    hs[owner + ".M"] = torch.from_numpy(m)
    import json as _json

    from safetensors import safe_open

    with safe_open(hess, "pt") as f:
        meta = f.metadata()
    save_file(hs, str(tmp_path / "hm.safetensors"), metadata=meta)
    cfg = Config(**CFG)
    out = str(tmp_path / "out")
    rep = quantize_model(QuantOpts([model], [str(tmp_path / "hm.safetensors")], out, cfg))
    pk, _ = load(os.path.join(out, "packed", "model.safetensors"))
    owners = {n[:-len(".weight")]: o for (n, _, _, o) in toy_model.layer_shapes(1)}
    for L in rep["layers"]:
        name = L["name"]
        tens = {}
        for suf in ("qweight", "scales", "qzeros", "perm", "gbits", "gsize"):
            dt, sh, raw, _ = pk[name + "." + suf]
            tens[name + "." + suf] = np.frombuffer(raw, {"U8": np.uint8, "F16": np.float16, "I32": np.int32}[dt]).reshape(sh)
        ql = read_packed_layer(tens, name)
        mm = m if owners[name] == owner else None
        qb, sb = orc.quantize_layer(tensors[name + ".weight"], L["d_out"], L["d_in"], H[owners[name]], mm, owners[name],
                                    cfg)
        assert np.array_equal(ql.codes, qb.codes) and np.array_equal(ql.scales, qb.scales), name
        assert L["loss_gptq"] == sb.loss_gptq, name
    assert _json.dumps(rep["layers"][0]["name"])
