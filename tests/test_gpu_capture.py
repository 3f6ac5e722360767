"""Hessian capture on the device (cdclq.capture, after scripts/capture_hessians.py): each captured H against the
f64 Gram of the very activations the hooks saw, divided by the token count.

Tolerance: the SYRK (f16/bf16 models) and the f32 path sum at most 2048 exact products per chunk in f32, each
chunk widened into f64; the final division is in f64 and rounded once to f32.  So every element is within
2048 * 2^-24 * sum|x_p x_q| / N (chunk sums) + 2^-24 |H| (the final rounding) of the exact value."""
import numpy as np
import pytest

from test_capture_host import tiny_llama

pytestmark = pytest.mark.gpu


def record(model, targets):
    """Pre-hooks keeping every hooked input (f64, CPU) per module, batch shape (2, S) only (the probe's single
    sample is left out)."""
    seen = {}

    def make(name):
        def hook(module, inputs):
            x = inputs[0]
            if x.shape[0] == 2:
                seen.setdefault(name, []).append(x.reshape(-1, x.shape[-1]).double().cpu())

        return hook

    return seen, [mod.register_forward_pre_hook(make(name)) for name, mod in targets]


def check_against_f64(cap, seen, weights=None):
    import torch

    for name, h in cap.h.items():
        x = torch.cat(seen[name])
        xw = x if weights is None else x * weights.double().sqrt().unsqueeze(1)
        ref = (xw.t() @ xw) / x.shape[0]
        ab = (xw.abs().t() @ xw.abs()) / x.shape[0]
        got = h.double().cpu()
        bound = 2048 * 2.0 ** -24 * ab + 2.0 ** -24 * ref.abs() + 1e-30
        assert torch.all((got - ref).abs() <= bound), (name, float(((got - ref).abs() / bound).max()))
        assert torch.equal(got, got.t()), name  # exactly symmetric
        assert cap.count[name] == x.shape[0]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_capture_matches_the_f64_gram_of_the_hooked_activations(gpu, dtype):
    import torch

    from cdclq.capture import capture, linear_targets

    m = tiny_llama(torch, getattr(torch, dtype)).cuda()
    g = torch.Generator().manual_seed(7)
    batches = [torch.randint(0, 256, (2, 96), generator=g) for _ in range(3)]
    seen, handles = record(m, linear_targets(m))
    caps = capture(m, batches)
    for hd in handles:
        hd.remove()
    assert len(caps) == 1
    cap = caps[0]
    assert len(cap.h) == 8 and len(cap.aliases) == 6  # q, o, gate, down per block; k/v -> q, up -> gate
    assert cap.resolve("model.layers.1.mlp.up_proj") == "model.layers.1.mlp.gate_proj"
    check_against_f64(cap, seen)
    md = cap.metadata()
    assert md["format"] == "hessian_v1" and md["calib_tokens"] == str(576) and "calib_tokens_min" not in md


def test_weighted_tokens_use_the_f32_path(gpu):
    import torch

    from cdclq.capture import capture, linear_targets

    m = tiny_llama(torch, torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(11)
    batches = [torch.randint(0, 256, (2, 64), generator=g) for _ in range(2)]
    tw = torch.ones(256, device="cuda")
    tw[::7] = 3.0  # every 7th vocabulary id is "structural"
    targets = linear_targets(m, only=("mlp",))
    seen, handles = record(m, targets)
    cap = capture(m, batches, only=("mlp",), token_weight=tw)[0]
    for hd in handles:
        hd.remove()
    w = torch.cat([tw[b.cuda()].reshape(-1).cpu() for b in batches])
    assert set(cap.h) == {"model.layers.0.mlp.gate_proj", "model.layers.0.mlp.down_proj",
                          "model.layers.1.mlp.gate_proj", "model.layers.1.mlp.down_proj"}
    check_against_f64(cap, seen, w)


def test_split_passes_equal_one_pass_and_the_files_load(gpu, tmp_path):
    import torch

    from cdclq.capture import accumulator_bytes, capture, out_path_for
    from cdclq.io import HessianStore

    m = tiny_llama(torch, torch.float16).cuda()
    g = torch.Generator().manual_seed(3)
    batches = [torch.randint(0, 256, (2, 80), generator=g) for _ in range(2)]
    one = capture(m, batches)[0]
    parts = capture(m, batches, max_bytes=accumulator_bytes(128) + accumulator_bytes(64))
    assert len(parts) == 3  # first fit decreasing: [down0, gate0], [down1, o0], [q0, gate1, o1, q1]
    merged = {}
    for p in parts:
        merged.update(p.h)
    assert set(merged) == set(one.h)
    for k in one.h:
        assert torch.equal(merged[k], one.h[k]), k  # the same batches in the same order: bit for bit
    paths = [str(tmp_path / out_path_for("h.safetensors", i + 1, len(parts))) for i in range(len(parts))]
    for p, c in zip(paths, parts):
        c.save(p)
    store = HessianStore(paths)
    for layer in ("model.layers.0.self_attn.v_proj", "model.layers.1.mlp.down_proj"):
        owner = store.resolve(layer)
        assert owner == one.resolve(layer)
        h, n = store.get_h(owner)
        assert torch.equal(h, one.hessian(layer)) and n == h.shape[0]


def test_captured_hessian_quantizes(gpu):
    import torch

    import cdclq
    from cdclq.abi import Config
    from cdclq.capture import capture

    m = tiny_llama(torch, torch.bfloat16).cuda()
    g = torch.Generator().manual_seed(5)
    cap = capture(m, [torch.randint(0, 256, (2, 128), generator=g) for _ in range(4)])[0]
    name = "model.layers.0.mlp.down_proj"
    w = m.get_submodule(name).weight.detach().float().cpu().numpy()
    h = cap.hessian(name).cpu().numpy()
    q, st = cdclq.quantize_layer(w, w.shape[0], w.shape[1], h, None, name, Config(bits=3, group=32, row_chunk=32))
    assert st.loss_final <= st.loss_gptq and np.all(q.codes <= 7)


def model_dir(torch, path):
    """A tiny random Llama with a word-level tokenizer saved as a Hugging Face directory (built offline)."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {"<unk>": 0}
    for i in range(255):
        vocab["w%d" % i] = i + 1
    tk = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="<unk>").save_pretrained(str(path))
    tiny_llama(torch).save_pretrained(str(path))
    return str(path)


def test_command_line_writes_the_reference_files(gpu, tmp_path):
    """`python -m cdclq.capture` (the reference script's arguments): one file, or one per pass under a small
    --max-hessian-mem, each readable by HessianStore and equal to the library call on the same batches; with
    --struct-chars the Hessians change."""
    import torch
    from transformers import AutoModelForCausalLM, AutoTokenizer

    from cdclq import capture as cap
    from cdclq.io import HessianStore

    d = model_dir(torch, tmp_path / "model")
    rng = np.random.default_rng(1)
    text = tmp_path / "calib.txt"
    text.write_text(" ".join("w%d" % v for v in rng.integers(0, 255, 600)))
    args = ["--model", d, "--text", str(text), "--nsamples", "4", "--seqlen", "64", "--batch", "2", "--dtype",
            "bfloat16"]
    out = str(tmp_path / "h.safetensors")
    cap.main(args + ["--out", out])
    store = HessianStore([out])
    assert set(store.index) == {"model.layers.%d.%s" % (b, m) for b in range(2)
                                for m in ("self_attn.q_proj", "self_attn.o_proj", "mlp.gate_proj", "mlp.down_proj")}
    assert store.resolve("model.layers.0.self_attn.k_proj") == "model.layers.0.self_attn.q_proj"
    # the same capture through the library
    tok = AutoTokenizer.from_pretrained(d)
    m = AutoModelForCausalLM.from_pretrained(d, dtype=torch.bfloat16).cuda().eval()
    ids = tok(text.read_text(), return_tensors="pt").input_ids[0][:4 * 64].view(4, 64)
    lib = cap.capture(m, [ids[0:2], ids[2:4]])[0]
    for owner in store.index:
        h, _ = store.get_h(owner)
        assert torch.equal(h, lib.h[owner]), owner
    # several passes, several files
    split = str(tmp_path / "s.safetensors")
    cap.main(args + ["--out", split, "--max-hessian-mem", str(2.5 * 128 * 128 * 8 / 2 ** 30)])
    files = sorted(str(p) for p in tmp_path.glob("s.*of*.safetensors"))
    assert len(files) >= 2
    multi = HessianStore(files)
    for owner in store.index:
        assert torch.equal(multi.get_h(owner)[0], store.get_h(owner)[0]), owner
    # structural tokens weighted
    wout = str(tmp_path / "w.safetensors")
    cap.main(args + ["--out", wout, "--struct-chars", "7", "--struct-weight", "3.0"])
    hw, _ = HessianStore([wout]).get_h("model.layers.0.mlp.gate_proj")
    assert not torch.equal(hw, store.get_h("model.layers.0.mlp.gate_proj")[0])
