"""`scripts/capture_hessians.py` on the device: calibration Hessians from a model's forward pass.

For every matched nn.Linear the layer input x_t of each calibration token is hooked and accumulated into
H = (1/N) sum_t w_t x_t x_t^T, as the reference's capture script does (scripts/capture_hessians.py:233-269),
with these differences of placement, not of meaning:

  * the accumulation runs where the activations already are: f16/bf16 activations go straight into the
    tcgen05 SYRK (cdclq_gram_accumulate_half_device: products exact in f32, token chunks of 2048 summed in
    f32 and widened into an f64 accumulator); f32 activations, and any capture with per-token weights (whose
    sqrt(w_t) x_t rows are formed in f32), take the bit-exact f32 Gram path;
  * the accumulators are f64 and divided by N before the final rounding to f32 (the reference sums in f32 and
    divides in f32);
  * the Hessians stay on the GPU (`Captured.hessian`) so the quantizer reads them without a file round trip,
    and `Captured.save` writes the reference's file format: `<module>.H` f32 tensors with the `format`,
    `generator`, `calib_tokens` (`calib_tokens_min`) and `aliases` metadata that cdclq.io.HessianStore reads.

The layer inputs shared by several modules (q/k/v, gate/up) are found as the reference finds them: a probe
forward pass on one sample compares the identity of consecutive hooked input tensors (:187-213); an aliased
module stores nothing.  A memory budget packs the distinct inputs into passes, first-fit decreasing
(:73-99), one output file per pass; every pass walks the same batches in the same order, so a split capture
equals a single-pass one bit for bit.
"""
import json
import os

from . import linalg

GIB = 1 << 30


def accumulator_bytes(d_in):
    """Size of one f64 d_in x d_in accumulator: what the memory budget bounds."""
    return d_in * d_in * 8


def plan_bins(families, budget):
    """Pack the distinct layer inputs {owner name: d_in} into bins of at most `budget` bytes of accumulators,
    largest first (ties by name), each into the first bin with room (scripts/capture_hessians.py:73-99)."""
    bins = []
    for owner, d_in in sorted(families.items(), key=lambda kv: (-accumulator_bytes(kv[1]), kv[0])):
        need = accumulator_bytes(d_in)
        if need > budget:
            raise ValueError("%s: a single Hessian at d_in=%d needs %d bytes, above the budget of %d bytes; raise "
                             "the budget, or capture this layer on its own" % (owner, d_in, need, budget))
        for b in bins:
            if b["bytes"] + need <= budget:
                b["bytes"] += need
                b["owners"].append(owner)
                break
        else:
            bins.append({"bytes": need, "owners": [owner]})
    return bins


def out_path_for(out, i, n):
    """`out` itself for a single pass, `<stem>.<i>of<n><ext>` for pass i of n."""
    if n == 1:
        return out
    stem, ext = os.path.splitext(out)
    return "%s.%dof%d%s" % (stem, i, n, ext)


def linear_targets(model, only=(), skip=("lm_head",)):
    """(name, module) of the nn.Linear modules to hook, in named_modules order (the order hooks fire in)."""
    import torch.nn as nn

    out = []
    for name, mod in model.named_modules():
        if not isinstance(mod, nn.Linear):
            continue
        if only and not any(s in name for s in only):
            continue
        if any(s in name for s in skip):
            continue
        out.append((name, mod))
    return out


def probe_aliases(model, targets, sample):
    """{module: owner} for the modules whose input is the very tensor object the previously hooked module
    received (one forward pass that accumulates nothing)."""
    import torch

    aliases = {}
    last = {"x": None, "owner": None}

    def make(name):
        def hook(module, inputs):
            x = inputs[0]
            if x is last["x"]:
                aliases[name] = last["owner"]
                return
            last["x"], last["owner"] = x, name

        return hook

    handles = [mod.register_forward_pre_hook(make(name)) for name, mod in targets]
    try:
        with torch.no_grad():
            model(input_ids=sample, use_cache=False)
    finally:
        for h in handles:
            h.remove()
    return aliases


class Captured:
    """The Hessians of one capture pass, on the device: `h[name]` (f32 d_in x d_in, H = sum w x x^T / N),
    `count[name]` = N, `aliases` {module: owner} for the owners of this pass."""

    def __init__(self, h, count, aliases):
        self.h, self.count, self.aliases = h, count, aliases

    def resolve(self, layer):
        """The owner whose Hessian serves `layer` (itself or its alias target), or None."""
        if layer in self.h:
            return layer
        o = self.aliases.get(layer)
        return o if o in self.h else None

    def hessian(self, layer):
        o = self.resolve(layer)
        if o is None:
            raise KeyError("no Hessian for %s" % layer)
        return self.h[o]

    def metadata(self):
        seen = set(self.count.values())
        md = {"format": "hessian_v1", "generator": "cdclq-capture", "calib_tokens": str(max(seen) if seen else 0),
              "aliases": json.dumps(self.aliases)}
        if len(seen) > 1:
            md["calib_tokens_min"] = str(min(seen))
        return md

    def save(self, path):
        from safetensors.torch import save_file

        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        save_file({"%s.H" % n: t.detach().cpu().contiguous() for n, t in self.h.items()}, path,
                  metadata=self.metadata())


def capture(model, batches, only=(), skip=("lm_head",), token_weight=None, max_bytes=None, stream=0):
    """Capture the calibration Hessians of `model` (on a CUDA device) over `batches` (an iterable, walked once
    per pass, of (batch, seq) input-id tensors).  token_weight: optional per-vocabulary-id weights (a tensor
    indexed by the input ids, as --struct-chars/--struct-weight build it).  max_bytes: budget of f64
    accumulators held at once (None: everything in one pass).  Returns one Captured per pass."""
    import torch

    batches = list(batches)
    if not batches:
        raise ValueError("no calibration batches")
    dev = next(model.parameters()).device
    if dev.type != "cuda":
        raise RuntimeError("the capture accumulates on the GPU: move the model to a CUDA device")
    targets = linear_targets(model, only, skip)
    if not targets:
        raise ValueError("no Linear module matched only/skip")
    aliases = probe_aliases(model, targets, batches[0][0:1].to(dev))
    families = {name: mod.in_features for name, mod in targets if name not in aliases}
    budget = max_bytes if max_bytes is not None else sum(accumulator_bytes(d) for d in families.values())
    bins = plan_bins(families, budget)
    out = []
    for b in bins:
        owners = set(b["owners"])
        acc, count, kind = {}, {}, {}
        state = {"w": None}

        def make(name):
            def hook(module, inputs):
                x = inputs[0]
                x2 = x.reshape(-1, x.shape[-1])
                t, n = int(x2.shape[0]), int(x2.shape[1])
                if name not in acc:
                    acc[name] = torch.zeros(n, n, dtype=torch.float64, device=x.device)
                    count[name] = 0
                    half = x.dtype in (torch.float16, torch.bfloat16) and n % 8 == 0 and state["w"] is None
                    kind[name] = "half" if half else "f32"
                if kind[name] == "half":
                    linalg.gram_accumulate_half_device(x2.contiguous(), acc[name], lower_only=True, stream=stream)
                else:
                    xf = x2.float()
                    if state["w"] is not None:
                        xf = xf * state["w"].sqrt().unsqueeze(1)
                    linalg.gram_accumulate_device(xf.contiguous(), acc[name], stream=stream)
                count[name] += t

            return hook

        handles = [mod.register_forward_pre_hook(make(name)) for name, mod in targets if name in owners]
        try:
            with torch.no_grad():
                for ids in batches:
                    ids = ids.to(dev)
                    state["w"] = token_weight[ids].reshape(-1).to(torch.float32) if token_weight is not None else None
                    model(input_ids=ids, use_cache=False)
        finally:
            for h in handles:
                h.remove()
        hs = {}
        for name, a in acc.items():
            if kind[name] == "half":  # the SYRK wrote the lower triangle: the upper one is its mirror
                a = torch.tril(a) + torch.tril(a, -1).t()
            hs[name] = (a / count[name]).to(torch.float32).contiguous()
        del acc
        out.append(Captured(hs, count, {d: o for d, o in aliases.items() if o in owners}))
        torch.cuda.empty_cache()
    return out


def main(argv=None):
    """Command line of the reference's capture script (scripts/capture_hessians.py:102-135), on a CUDA device."""
    import argparse
    import sys

    import torch
    from transformers import AutoModelForCausalLM, AutoTokenizer

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", required=True, help="Hugging Face model directory")
    ap.add_argument("--text", required=True, help="UTF-8 text file used as calibration data")
    ap.add_argument("--out", required=True, help="output .safetensors with the Hessians")
    ap.add_argument("--nsamples", type=int, default=128)
    ap.add_argument("--seqlen", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--dtype", default="float16", choices=["float16", "bfloat16", "float32"])
    ap.add_argument("--only", default="", help="comma separated substrings: only hook matching modules")
    ap.add_argument("--skip", default="lm_head", help="comma separated substrings of modules to skip")
    ap.add_argument("--struct-chars", default="", help="characters marking structural tokens")
    ap.add_argument("--struct-weight", type=float, default=1.0)
    ap.add_argument("--max-hessian-mem", type=float, default=64.0, metavar="GIB",
                    help="GiB of f64 accumulators held at once; more is captured in several passes, one file each")
    args = ap.parse_args(argv)
    if args.max_hessian_mem <= 0:
        sys.exit("--max-hessian-mem must be a positive number of GiB")
    tok = AutoTokenizer.from_pretrained(args.model)
    model = AutoModelForCausalLM.from_pretrained(args.model, dtype=getattr(torch, args.dtype))
    model = model.to("cuda").eval()
    with open(args.text, encoding="utf-8") as f:
        ids = tok(f.read(), return_tensors="pt").input_ids[0]
    need = args.nsamples * args.seqlen
    if ids.numel() < need:
        sys.exit("calibration text has %d tokens, need %d: use a bigger file or lower --nsamples/--seqlen"
                 % (ids.numel(), need))
    samples = ids[:need].view(args.nsamples, args.seqlen)
    token_w = None
    if args.struct_chars and args.struct_weight != 1.0:
        token_w = torch.ones(len(tok))
        for t in range(len(tok)):
            if any(c in tok.decode([t]) for c in args.struct_chars):
                token_w[t] = args.struct_weight
        token_w = token_w.to("cuda")
    batches = [samples[s:s + args.batch] for s in range(0, args.nsamples, args.batch)]
    parts = capture(model, batches, [s for s in args.only.split(",") if s], [s for s in args.skip.split(",") if s],
                    token_w, int(args.max_hessian_mem * GIB))
    written = []
    for i, c in enumerate(parts, 1):
        p = out_path_for(args.out, i, len(parts))
        c.save(p)
        written.append(p)
        print("saved %d Hessians (%d aliased) -> %s" % (len(c.h), len(c.aliases), p), file=sys.stderr)
    if len(written) > 1:
        print("  " + " ".join("--hessians %s" % p for p in written), file=sys.stderr)


if __name__ == "__main__":
    main()
