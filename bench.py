#!/usr/bin/env python
"""bench.py - cdclq-b200 benchmark under the driver's contract.

Workload: a TinyLlama-1.1B-shaped model, 22 decoder layers x 7 linear layers
(q 2048x2048, k/v 256x2048, o 2048x2048, gate/up 5632x2048, down 2048x5632) = 9.69e8 weights, random-init
bf16 weights ~ N(0, 0.02^2) (widened to f32 as the reference does for bf16 checkpoints, src/io.rs:37-44),
and per distinct layer input (q/k/v, o, gate/up, down: 88 Hessians) a synthetic Hessian H = X^T X from
128 x 2048 = 262144 seeded tokens distributed as configs[0] (per-channel log-normal scale sigma = 1,
0.5 % channels x20, 1 % dead channels).  Settings: 3-bit, group 128, --mse-grid, reference defaults otherwise
(block 128, sub-block 64, damp 0.01, act-order, CDCL, 10 passes, tol 1e-3), row chunk pinned to 128 rows.

One step = quantizing the whole model from resident inputs: 88 factorisations (the q/k/v and gate/up layers
share theirs), the GPTQ pass and the CDCL repair of all 154 layers.  The Hessians are inputs, as they are for
the reference's `cdclq quantize` (captured by a separate script).

Legs:
  value     device-resident inputs (W, H in HBM; 7.7 GB, larger than L2), CUDA events on the stream
  e2e       the public C ABI with pinned HOST buffers (cdclq_quantize_batch, on_device = 0): H2D of W and H and
            D2H of codes/scales/zeros inside the timed region
  cpu_baseline  the CPU oracle (C++ restatement of the reference's rayon path) on a bounded sample, rank 0,
            N = 1 only
  --impl reference  the oracle port on the host cores (the Rust reference cannot be built here), same sample

N > 1: one process per GPU (torchrun), cdclq.pipeline.ModelBatch: every layer's rows are split across ranks in
whole row chunks (rows are independent and row chunks are the reference's unit of conflict selection and
stopping); the 88 factorisations are spread over the ranks (longest-processing-time on n^3) and each factor U
is broadcast from its owner over NCCL; the result is identical to N = 1; the per-layer losses are all-reduced
over NCCL.  Weak/strong: strong (the model is fixed).
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cdcl-gptq_b200"))

METRIC = "seconds per model quantized (incl. CDCL repair) at 1/2/4/8 B200; weights/sec"
HIDDEN, INTER, N_LAYERS, KV_OUT = 2048, 5632, 22, 256
TOKENS = 128 * 2048
ROW_CHUNK = 128

# (name, d_out, d_in, input kind)
BLOCK = [("q_proj", HIDDEN, HIDDEN, "attn"), ("k_proj", KV_OUT, HIDDEN, "attn"), ("v_proj", KV_OUT, HIDDEN, "attn"),
         ("o_proj", HIDDEN, HIDDEN, "o"), ("gate_proj", INTER, HIDDEN, "mlp"), ("up_proj", INTER, HIDDEN, "mlp"),
         ("down_proj", HIDDEN, INTER, "down")]
INPUT_DIM = {"attn": HIDDEN, "o": HIDDEN, "mlp": HIDDEN, "down": INTER}


def bench_config():
    from cdclq.abi import Config

    return Config(bits=3, group=128, mse_grid=True, row_chunk=ROW_CHUNK)


# ------------------------------------------------------------------------------------------------------------
# seeded synthetic inputs (torch is plumbing here: RNG and the TF32 GEMM that builds H from bf16 tokens)
def channel_profile(n, seed, torch, device):
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    s = torch.exp(torch.randn(n, generator=g, dtype=torch.float64))
    perm = torch.randperm(n, generator=g)
    n_out = max(1, round(0.005 * n))
    n_dead = max(1, round(0.01 * n))
    s[perm[:n_out]] *= 20.0
    s[perm[n_out:n_out + n_dead]] = 0.0
    return s.to(device=device, dtype=torch.float32)


def make_hessian(n, seed, tokens, torch, device):
    """H = X^T X over `tokens` seeded tokens; X is bf16-representable so the TF32 GEMM products are exact."""
    scale = channel_profile(n, seed, torch, device)
    g = torch.Generator(device=device)
    g.manual_seed(seed + 1)
    h = torch.zeros(n, n, dtype=torch.float64, device=device)
    chunk = 8192
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for t0 in range(0, tokens, chunk):
            tc = min(chunk, tokens - t0)
            x = (torch.randn(tc, n, generator=g, device=device) * scale).to(torch.bfloat16).float()
            h += (x.t() @ x).double()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
    return h.float().contiguous()


def make_weight(d_out, n, seed, torch, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = (torch.randn(d_out, n, generator=g, device=device) * 0.02).to(torch.bfloat16).float()
    return w.contiguous()


def model_layers(n_layers=N_LAYERS):
    """[(layer name, d_out, d_in, input index)], inputs [(name, n)]."""
    layers, inputs = [], []
    for b in range(n_layers):
        idx = {}
        for kind in ("attn", "o", "mlp", "down"):
            idx[kind] = len(inputs)
            inputs.append(("model.layers.%d.%s" % (b, kind), INPUT_DIM[kind]))
        for name, d_out, d_in, kind in BLOCK:
            layers.append(("model.layers.%d.%s" % (b, name), d_out, d_in, idx[kind]))
    return layers, inputs


def generate(torch, device, n_layers=N_LAYERS, tokens=TOKENS):
    layers, inputs = model_layers(n_layers)
    H = [make_hessian(n, 1000 + i, tokens, torch, device) for i, (_, n) in enumerate(inputs)]
    W = [make_weight(d_out, d_in, 50000 + i, torch, device) for i, (_, d_out, d_in, _) in enumerate(layers)]
    return layers, inputs, H, W


# ------------------------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = float(p[2])
                power.append(float(p[3]))
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def fp32_simt_peak_tflops(torch):
    """Measured FP32 CUDA-core peak: cuBLAS SGEMM with TF32 disabled (FFMA), best of 5."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n = 8192
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        for _ in range(2):
            a @ b
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            a @ b
            e1.record()
            e1.synchronize()
            best = max(best, 2.0 * n ** 3 / (e0.elapsed_time(e1) * 1e-3) / 1e12)
        return best
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


# ------------------------------------------------------------------------------------------------------------
class RuntimeBatch:
    """Descriptor tables of the model for cdclq_runtime_quantize_batch: FULL layers on every rank (each rank
    quantizes its rows), inputs and outputs on the device (on_device=True) or in pinned host memory.

    h2d_bytes / d2h_bytes count what this rank copies per step in the host mode: the Hessians it owns (the
    runtime uploads each Hessian once, on its owner, and broadcasts it), its rows of every W, and its rows of
    codes, scales and zero points back (rank 0: every row, gathered over NVLink)."""

    def __init__(self, torch, rt, layers, inputs, H, W, cfg, on_device):
        from cdclq.abi import CBatchInput, CBatchLayer, CLayerStats, num_groups
        from cdclq.runtime import assign_owners, shard_rows

        self.rt, self.cfg, self.on_device = rt, cfg, on_device
        self.keep = list(H) + list(W)
        self.ins = (CBatchInput * len(inputs))()
        for i, (_, n) in enumerate(inputs):
            self.ins[i].h = H[i].data_ptr()
            self.ins[i].n = n
        self.lys = (CBatchLayer * len(layers))()
        self.stats = [CLayerStats() for _ in layers]
        self.outs = []
        self.layer_index = list(range(len(layers)))
        dev = "cuda" if on_device else "cpu"
        owner = assign_owners([n for (_, n) in inputs], rt.nranks, 3)
        self.h2d_bytes = sum(n * n * 4 for i, (_, n) in enumerate(inputs) if owner[i] == rt.rank)
        self.d2h_bytes = 0
        for li, (name, d_out, d_in, inp) in enumerate(layers):
            ng = num_groups(cfg, d_in)
            o = dict(perm=np.zeros(d_in, np.uint32), gbits=np.zeros(ng, np.uint8),
                     codes=torch.empty(d_out, d_in, dtype=torch.uint8, device=dev, pin_memory=not on_device),
                     scales=torch.empty(d_out, ng, dtype=torch.float32, device=dev, pin_memory=not on_device),
                     zeros=torch.empty(d_out, ng, dtype=torch.float32, device=dev, pin_memory=not on_device))
            self.outs.append(o)
            L = self.lys[li]
            L.w = W[li].data_ptr()
            L.d_out = d_out
            L.input = inp
            L.perm = o["perm"].ctypes.data
            L.gbits = o["gbits"].ctypes.data
            L.codes = o["codes"].data_ptr()
            L.scales = o["scales"].data_ptr()
            L.zeros = o["zeros"].data_ptr()
            L.stats = ctypes.pointer(self.stats[li])
            r0, r1 = shard_rows(d_out, cfg.row_chunk, rt.rank, rt.nranks, li)
            self.h2d_bytes += (r1 - r0) * d_in * 4
            rows = d_out if rt.rank == 0 else r1 - r0
            self.d2h_bytes += rows * d_in + 2 * rows * ng * 4

    def run(self, gather):
        self.rt.quantize_batch(self.ins, self.lys, self.cfg, self.on_device, gather)


def host_cores():
    """Host CPU threads this process may run on (the affinity mask, not OMP_NUM_THREADS: torchrun sets that
    to 1 for every rank)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_jobs(layers):
    """The decoder layer's linear layers in the reference's job order (src/pipeline.rs:109-112: sorted by the
    Hessian owner, then by layer name), so that the single-entry prep cache hits for q/k/v and gate/up."""
    first = {}
    for (name, _, _, inp) in layers:
        first.setdefault(inp, name)  # the owner of an input is its first layer (q_proj, gate_proj)
    return sorted(range(len(layers)), key=lambda i: (first[layers[i][3]], layers[i][0]))


class CpuReference:
    """The reference's CPU path (the oracle, oracle/: the C++ restatement, OpenMP over row chunks like the
    reference's rayon) on one decoder layer of the model, one linear layer per step.

    Step k quantizes job k mod 7 of the decoder layer in the reference's order, through the oracle's
    quantize_layer with a single-entry prep cache keyed by the Hessian owner - exactly the reference's
    sequential per-layer loop (src/pipeline.rs:121-175): the factorisation runs when the owner changes, q/k/v
    and gate/up reuse it.  Seven consecutive steps are one whole decoder layer; the model time is 22 times the
    decoder layer (the 22 layers are identical in shape), which is an extrapolation and is labelled as one."""

    def __init__(self, layers, inputs, H, W, cfg, cores):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as orc

        self.orc = orc
        orc.set_threads(cores)
        self.cores = cores
        self.cfg = cfg
        self.layers, self.inputs = layers, inputs
        self.H = [h.float().cpu().numpy() for h in H]
        self.W = [w.float().cpu().numpy() for w in W]
        self.order = reference_jobs(layers)
        self.cache = orc.PrepCache()
        self.k = 0
        self.results = {}

    def step(self):
        """One linear layer; returns (layer index, seconds, weights)."""
        li = self.order[self.k % len(self.order)]
        self.k += 1
        name, d_out, d_in, inp = self.layers[li]
        t0 = time.perf_counter()
        ql, st = self.orc.quantize_layer(self.W[li], d_out, d_in, self.H[inp], None, self.inputs[inp][0], self.cfg,
                                         self.cache)
        dt = time.perf_counter() - t0
        self.results[li] = (ql, st)
        return li, dt, d_out * d_in

    def decoder_layer_seconds(self, per_layer):
        """Seconds of one decoder layer from per-layer timings {layer index: [seconds...]} (mean per layer)."""
        return sum(statistics.mean(per_layer[li]) for li in self.order)


def cpu_baseline_sample(layers, inputs, H, W, cfg):
    """cpu_baseline (rank 0, N = 1): the CPU reference path over one whole decoder layer (7 steps of
    CpuReference), timed; the model time is 22 decoder layers (stated as an extrapolation).  Also returns the
    oracle's outputs for the parity check against the GPU's rows of the same layers."""
    ref = CpuReference(layers, inputs, H, W, cfg, host_cores())
    per, t0 = {}, time.perf_counter()
    for _ in range(len(layers)):
        li, dt, _ = ref.step()
        per.setdefault(li, []).append(dt)
    wall = time.perf_counter() - t0
    layer_s = ref.decoder_layer_seconds(per)
    model_s = N_LAYERS * layer_s
    weights = N_LAYERS * sum(l[1] * l[2] for l in layers)
    return {
        "value": weights / model_s, "unit": "weights/s", "cores": ref.cores, "kind": "port",
        "seconds_per_model": model_s, "seconds_per_decoder_layer": layer_s, "sample_wall_s": wall,
        "sample": ("one whole decoder layer (7 linear layers, 4 factorisations, all row chunks) through the CPU "
                   "oracle (C++ restatement of the reference's rayon path, OpenMP over row chunks, %d threads), "
                   "timed; model = 22 x the decoder layer (extrapolation: identical layer shapes)" % ref.cores),
    }, ref.results


def parity_report(ref_results, batch, layers):
    """The GPU's outputs for the decoder layer the CPU reference quantized (rows the persistent repair kernel
    produced inside the timed model run) against the oracle's: fractions of identical codes, scales and zero
    points, identical permutations, and the largest relative loss difference over the layers."""
    n_codes = same_codes = n_groups = same_scales = same_zeros = 0
    perms_identical = True
    lg = lf = 0.0
    for li, (ql, st) in sorted(ref_results.items()):
        bi = batch.layer_index.index(li)
        o = batch.outs[bi]
        codes = o["codes"].cpu().numpy()
        scales = o["scales"].cpu().numpy()
        zeros = o["zeros"].cpu().numpy()
        perms_identical &= bool(np.array_equal(o["perm"], ql.perm))
        n_codes += codes.size
        same_codes += int(np.count_nonzero(codes == ql.codes))
        n_groups += scales.size
        same_scales += int(np.count_nonzero(scales == ql.scales))
        same_zeros += int(np.count_nonzero(zeros == ql.zeros))
        s = batch.stats[bi]
        lg = max(lg, abs(s.loss_gptq - st.loss_gptq) / st.loss_gptq)
        lf = max(lf, abs(s.loss_final - st.loss_final) / st.loss_final)
    return {"layers": [layers[li][0] for li in sorted(ref_results)], "weights": n_codes,
            "codes_identical_frac": same_codes / n_codes, "scales_identical_frac": same_scales / n_groups,
            "zeros_identical_frac": same_zeros / n_groups, "perms_identical": perms_identical,
            "loss_gptq_rel_max": lg, "loss_final_rel_max": lf,
            "bar": "north star: codes >= 99.99 % identical, ties only; losses within 1e-6 relative"}


def run_reference_arm(args, torch, rank, world):
    """`--impl reference`: the reference's CPU path (the oracle port: no Rust toolchain on this image) on the
    host cores, rank 0 only.  A step is one linear layer of configs[1]'s decoder layer in the reference's job
    order (CpuReference): 7 consecutive steps are one decoder layer, each step timed as it runs.  value = model
    weights / (22 x the decoder layer's time composed from the per-layer means of the timed steps); with fewer
    than 7 timed steps, weights / seconds of the steps that ran."""
    if rank != 0:
        return
    cfg = bench_config()
    device = "cuda" if torch.cuda.is_available() else "cpu"
    layers, inputs = model_layers(1)
    H = [make_hessian(n, 1000 + i, TOKENS, torch, device) for i, (_, n) in enumerate(inputs)]
    W = [make_weight(d_out, d_in, 50000 + i, torch, device) for i, (_, d_out, d_in, _) in enumerate(layers)]
    ref = CpuReference(layers, inputs, H, W, cfg, host_cores())
    for _ in range(args.warmup):
        ref.step()
    per, secs, wts = {}, [], 0
    for _ in range(args.steps):
        li, dt, nw = ref.step()
        per.setdefault(li, []).append(dt)
        secs.append(dt)
        wts += nw
    ms_per_step = 1e3 * sum(secs) / len(secs)
    full_layers, _ = model_layers(N_LAYERS)
    model_weights = sum(l[1] * l[2] for l in full_layers)
    if len(per) == len(layers):
        layer_s = ref.decoder_layer_seconds(per)
        model_s = N_LAYERS * layer_s
        value = model_weights / model_s
        how = ("per-layer mean times of the timed steps summed over the decoder layer's 7 linear layers, x22 "
               "decoder layers (extrapolation: identical shapes)")
    else:
        value = wts / sum(secs)
        model_s = model_weights / value
        how = "weights / seconds of the timed steps (fewer than 7: not every layer of the decoder layer timed)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "weights/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "seconds_per_model": model_s,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg),
        "step": "one linear layer of the decoder layer, in the reference's job order (7 steps = 1 decoder layer)",
        "model_time": how,
        "cpu_baseline": {"value": value, "unit": "weights/s", "cores": ref.cores, "kind": "port",
                         "sample": "%d timed steps of one linear layer each (CPU oracle, %d threads)" % (
                             args.steps, ref.cores)},
        "e2e": {"value": value, "unit": "weights/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is a Rust crate and no Rust toolchain exists on this image; the timed CPU path is "
                "the C++ restatement of it (oracle/), run with all host threads (sched_getaffinity), like the "
                "reference's rayon pool",
    }
    print(json.dumps(line), flush=True)


def repair_traffic_bytes(weights):
    """DRAM bytes of one repair launch for `weights` weights, from the committed ncu summary of the repair kernel
    on the 2-layer case (dram__bytes_read.sum + dram__bytes_write.sum of the launch, per weight); None when the
    summary is absent."""
    path = os.path.join(ROOT, "profiles", "repair_persistent_kernel_tinyllama_2layers.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_weight:"):
                return float(line.split(":", 1)[1]) * weights
    except OSError:
        pass
    return None


def run_syrk_bench(args, torch):
    """H (f64) += X^T X for 262144 seeded bf16 tokens per width (the Hessian accumulation of configs[3]; the
    configs[1] bench takes its Hessians as inputs).  Algorithmic work T*n*(n+1) flops (the lower triangle and
    the diagonal), against the measured dense bf16 tensor peak.  X (>= 1 GB) exceeds the L2."""
    import cdclq
    from cdclq import linalg

    cdclq.lib()
    peaks = load_peaks()
    peak = peaks.get("bf16_tflops") or 1590.0
    t = args.syrk_tokens
    for n in [int(v) for v in args.syrk_widths.split(",")]:
        g = torch.Generator(device="cuda")
        g.manual_seed(7000 + n)
        x = torch.randn(t, n, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
        h = torch.zeros(n, n, dtype=torch.float64, device="cuda")
        st = torch.cuda.current_stream()
        for _ in range(max(3, args.warmup)):
            linalg.gram_accumulate_bf16_device(x, h, lower_only=True, stream=st.cuda_stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(args.steps):
            linalg.gram_accumulate_bf16_device(x, h, lower_only=True, stream=st.cuda_stream)
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        flops = float(t) * n * (n + 1)
        tf = flops / (ms * 1e-3) / 1e12
        print(json.dumps({"metric": "bf16 Gram accumulation H += X^T X (lower triangle)", "kernel": "syrk_bf16_kernel",
                          "n": n, "tokens": t, "ms": ms, "value": tf, "unit": "TFLOP/s",
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                                       "frac": tf / peak, "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst)"},
                          "steps": args.steps}), flush=True)
        del x, h
        torch.cuda.empty_cache()


# ---- model-level configurations beyond configs[1]: configs[2] (Gemma-2B-shaped, skeleton), configs[3]
# (Llama-2-7B-shaped, the north star, Hessians accumulated on the GPU) and configs[4] (Llama-3-70B stress layers)

MODEL_SPECS = {
    # hidden, intermediate, q/o width, k/v rows, decoder layers, blocks per single-GPU batch
    "llama2-7b": dict(config=3, hidden=4096, inter=11008, q_out=4096, kv=4096, layers=32, per_batch=16,
                      tokens="gauss", hessians_timed=True, outliers=0.001, label="Llama-2-7B-shaped"),
    "gemma2b": dict(config=2, hidden=2048, inter=16384, q_out=2048, kv=256, layers=18, per_batch=18,
                    tokens="student3", hessians_timed=False, outliers=0.0, label="Gemma-2B-shaped"),
}


def model_config(name, args):
    from cdclq.abi import Config

    if name == "llama2-7b":  # configs[3]: 4-bit and 2-bit, group 64, --mse-grid, refine-frac 0.25
        return Config(bits=args.bits, group=args.group or 64, mse_grid=True, refine_frac=0.25, row_chunk=ROW_CHUNK)
    # 4-bit, group 128, skeleton-pct 2 (skeleton groups at 8 bits)
    return Config(bits=4, group=128, skeleton_pct=2.0, row_chunk=ROW_CHUNK)


def spec_layers(spec):
    """(layers, inputs) of a decoder stack: q, k, v, o, gate, up, down per block; distinct inputs attn (q/k/v),
    o, mlp (gate/up) and down."""
    h, it, qo, kv = spec["hidden"], spec["inter"], spec["q_out"], spec["kv"]
    block = [("q_proj", qo, h, "attn"), ("k_proj", kv, h, "attn"), ("v_proj", kv, h, "attn"), ("o_proj", h, qo, "o"),
             ("gate_proj", it, h, "mlp"), ("up_proj", it, h, "mlp"), ("down_proj", h, it, "down")]
    dims = {"attn": h, "o": qo, "mlp": h, "down": it}
    layers, inputs = [], []
    for b in range(spec["layers"]):
        idx = {}
        for kind in ("attn", "o", "mlp", "down"):
            idx[kind] = len(inputs)
            inputs.append(("model.layers.%d.%s" % (b, kind), dims[kind]))
        for name, d_out, d_in, kind in block:
            layers.append(("model.layers.%d.%s" % (b, name), d_out, d_in, idx[kind]))
    return layers, inputs


def synth_weight(torch, i, d_out, n, std, outliers, bf16, rows=None, seed0=90000):
    """Seeded N(0, std^2) weights, `outliers` of the input columns x10, bf16-valued unless bf16=False; `rows`
    keeps a row range only (generated whole, so every rank sees the same matrix)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed0 + i)
    w = torch.randn(d_out, n, generator=g, device="cuda") * std
    if outliers > 0.0:
        gc = torch.Generator(device="cpu")
        gc.manual_seed(seed0 + 1000 + i)
        w[:, torch.randperm(n, generator=gc)[:max(1, int(round(n * outliers)))].to("cuda")] *= 10.0
    if rows is not None:
        w = w[rows[0]:rows[1]]
    return (w.to(torch.bfloat16).float() if bf16 else w).contiguous()


def synth_tokens(torch, scale, seed, t, kind):
    """t seeded bf16 activations over len(scale) channels scaled per channel; kind "gauss" or "student3"
    (heavy-tailed: N(0,1) / sqrt(chi2_3 / 3), Student-t with 3 degrees of freedom)."""
    n = scale.numel()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(t, n, generator=g, device="cuda")
    if kind == "student3":
        chi = torch.randn(t, n, 3, generator=g, device="cuda").pow_(2).sum(-1)
        x.div_(chi.div_(3.0).sqrt_())
        del chi
    return (x * scale).to(torch.bfloat16).contiguous()


def gpu_hessian(torch, i, n, t, kind, stream, chunk=32768):
    """Untimed input Hessian: H = X^T X (f32, accumulated in f64) of synthetic tokens with the configs[0] channel
    profile, by the tensor-core SYRK in token chunks of `chunk` (a multiple of the reference's 2048, so the
    result is that of one call) to keep wide inputs small on the device."""
    from cdclq import linalg

    scale = channel_profile(n, 3000 + i, torch, "cuda")
    h64 = torch.zeros(n, n, dtype=torch.float64, device="cuda")
    for t0 in range(0, t, chunk):
        x = synth_tokens(torch, scale, 4000 + 7919 * i + t0 // chunk, min(chunk, t - t0), kind)
        linalg.gram_accumulate_bf16_device(x, h64, lower_only=t0 + chunk < t, stream=stream)
        del x
    return h64.float()


class PhaseClock:
    """Device time of timed steps on one stream (CUDA events around each step, synchronised), per phase."""

    def __init__(self, torch, stream, phases):
        self.torch, self.st = torch, stream
        self.ms = {p: 0.0 for p in phases}

    def __call__(self, fn, phase):
        e0, e1 = self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True)
        e0.record(self.st)
        out = fn()
        e1.record(self.st)
        self.torch.cuda.synchronize()
        self.ms[phase] += e0.elapsed_time(e1)
        return out

    def total(self):
        return sum(self.ms.values())


def max_over_ranks(torch, values, world, op="max"):
    if world == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX if op == "max" else torch.distributed.ReduceOp.SUM)
    return [float(v) for v in t]


def run_model(args, torch, rank, world):
    """configs[3] (`--model llama2-7b`, the north star) and configs[2] (`--model gemma2b`) end to end.

    32 Llama-2-7B-shaped blocks, 6.48e9 bf16-valued weights N(0, 0.02^2) with 0.1 % of input columns
    x10; every distinct input's Hessian accumulated on the GPU by the tensor-core SYRK from 262144 seeded bf16
    activations (configs[0] channel profile) INSIDE the timed region; then `--bits` (4 or 2), group 64 (or
    `--group`), --mse-grid, refine-frac 0.25.  N > 1: Hessian owners by longest processing time on n^2, each
    broadcast (f32, NCCL); quantization by cdclq.pipeline.ModelBatch on rank-local row shards.
    18 Gemma-2B-shaped blocks (k/v 256 rows, intermediate 16384), 1.98e9 weights; Hessians from
    262144 Student-t(3) tokens are inputs (built by the SYRK, not timed); 4-bit, group 128, skeleton-pct 2.
    N > 1: every rank holds the full W for the skeleton's column scores.
    Timed: CUDA events, max over ranks.  Not timed: synthetic activations and weights."""
    import cdclq
    from cdclq import linalg
    from cdclq.pipeline import ModelBatch, assign_factorisations, shard_rows

    cdclq.lib()
    spec = MODEL_SPECS[args.model]
    cfg = model_config(args.model, args)
    st = torch.cuda.current_stream()
    layers, inputs = spec_layers(spec)
    total_weights = sum(l[1] * l[2] for l in layers)
    skel = cfg.skeleton_pct > 0.0
    clock = PhaseClock(torch, st, ("hessians", "hessian_broadcast", "quantization"))

    # ---- Hessians
    H = [None] * len(inputs)
    if spec["hessians_timed"]:
        owner = assign_factorisations([n for (_, n) in inputs], world, power=2) if world > 1 else [0] * len(inputs)
        if world > 1:
            torch.distributed.barrier()
        for i, (_, n) in enumerate(inputs):
            if owner[i] != rank:
                H[i] = torch.empty(n, n, dtype=torch.float32, device="cuda")
                continue
            x = synth_tokens(torch, channel_profile(n, 3000 + i, torch, "cuda"), 4000 + i, TOKENS, spec["tokens"])
            h64 = torch.zeros(n, n, dtype=torch.float64, device="cuda")
            clock(lambda: linalg.gram_accumulate_bf16_device(x, h64, lower_only=False, stream=st.cuda_stream),
                  "hessians")
            H[i] = clock(lambda: h64.float(), "hessians")
            del x, h64
        if world > 1:
            def bcast():
                for i, h in enumerate(H):
                    torch.distributed.broadcast(h, src=owner[i])
            clock(bcast, "hessian_broadcast")
    else:
        for i, (_, n) in enumerate(inputs):
            H[i] = gpu_hessian(torch, i, n, TOKENS, spec["tokens"], st.cuda_stream)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    # ---- quantization
    stats = []
    eng = {k: 0.0 for k in ("ms_prepare", "ms_phase1", "ms_stats", "ms_repair", "ms_final")}

    def quantize(part, W, **kw):
        b = ModelBatch(torch, part, inputs, H, W, cfg, on_device=True, **kw)
        if world > 1:
            torch.distributed.barrier()
        clock(lambda: b.run(st.cuda_stream), "quantization")
        prof = cdclq._lib.last_run_profile()
        for k in eng:
            eng[k] += prof[k]
        stats.extend(b.stats)

    wstd, outl = 0.02, spec["outliers"]
    if world > 1:
        W = []
        for i, (_, d_out, n, _) in enumerate(layers):
            if skel:  # the skeleton's column scores need every row
                W.append(synth_weight(torch, i, d_out, n, wstd, outl, True))
            else:
                r = shard_rows(d_out, ROW_CHUNK, rank, world, rotate=i)
                W.append(synth_weight(torch, i, d_out, n, wstd, outl, True, r) if r[1] > r[0] else None)
        quantize(layers, W, rank=rank, world=world, w_sharded=not skel)
        del W
    else:
        per = spec["per_batch"] * 7
        for l0 in range(0, len(layers), per):
            part = layers[l0:l0 + per]
            W = [synth_weight(torch, l0 + j, d_out, n, wstd, outl, True) for j, (_, d_out, n, _) in enumerate(part)]
            quantize(part, W)
            del W
            torch.cuda.empty_cache()
    loss = max_over_ranks(torch, [sum(s.loss_gptq for s in stats), sum(s.loss_final for s in stats)], world, "sum")
    names = ("hessians", "hessian_broadcast", "quantization")
    t = max_over_ranks(torch, [clock.total()] + [clock.ms[k] for k in names], world)
    if rank == 0:
        c3 = spec["config"] == 3
        print(json.dumps({
            "metric": "seconds per model quantized incl. %sCDCL repair" % ("Hessian accumulation and " if c3 else ""),
            "value": t[0] * 1e-3, "unit": "s", "higher_is_better": False, "n_gpus": world,
            "weights_per_s": total_weights / (t[0] * 1e-3),
            "target_s": 60.0 if c3 else None, "target_gpus": 8 if c3 else None,
            "config": {"workload": "%s model (configs[%d]): %d layers, %d linear layers, %.3g weights, %d Hessians "
                                   "from %d %s bf16 tokens each%s" % (
                                       spec["label"], spec["config"], spec["layers"], len(layers), total_weights,
                                       len(inputs), TOKENS, "Student-t(3)" if spec["tokens"] == "student3" else "Gaussian",
                                       " accumulated on the GPU inside the timed region" if c3 else " (inputs)"),
                       "bits": cfg.bits, "group": cfg.group, "mse_grid": bool(cfg.mse_grid),
                       "refine_frac": cfg.refine_frac, "skeleton_pct": cfg.skeleton_pct, "row_chunk": ROW_CHUNK},
            "timed": ("tensor-core Hessian accumulation + quantization" if c3 else "quantization") +
                     " (synthetic activation and weight generation excluded)",
            "engine_phases_ms_rank0": eng,
            "phases_s_max_over_ranks": {k: v * 1e-3 for k, v in zip(names, t[1:])},
            "loss_gptq": loss[0], "loss_final": loss[1], "data": "synthetic (seeded)",
        }), flush=True)


def north_star(torch, rank, world, rt, bits=4, group=64):
    """configs[3], the north star, once: 32 Llama-2-7B-shaped blocks (6.48e9 bf16-valued weights N(0, 0.02^2), 0.1 %
    of input columns x10); each of the 128 distinct inputs' Hessian accumulated on the GPU by the tcgen05 SYRK from
    262144 seeded bf16 activations (configs[0] channel profile) on its owner rank (longest processing time on n^2)
    INSIDE the timed region, broadcast over NCCL, then every layer quantized through the library's runtime
    (cdclq_runtime_quantize_batch: row shards in whole 128-row chunks, factors computed by their owner and
    broadcast in one NCCL group, statistics all-reduced) with `bits`, group 64, --mse-grid, refine-frac 0.25.  One
    GPU quantizes the model in two halves (HBM); several GPUs in one batch.  Timed with CUDA events on the runtime's
    stream, max over ranks; not timed: generating the activations and the weights."""
    from cdclq import linalg
    from cdclq.abi import Config
    from cdclq.runtime import assign_owners

    spec = MODEL_SPECS["llama2-7b"]
    cfg = Config(bits=bits, group=group, mse_grid=True, refine_frac=0.25, row_chunk=ROW_CHUNK)
    layers, inputs = spec_layers(spec)
    total_weights = sum(l[1] * l[2] for l in layers)
    st = torch.cuda.ExternalStream(rt.stream_handle)
    names = ("hessians", "hessian_broadcast", "quantization")
    clock = PhaseClock(torch, st, names)
    eng = {k: 0.0 for k in ("ms_prepare", "ms_phase1", "ms_stats", "ms_repair", "ms_final")}
    factor_batches, free_gb = 0, []
    stats = []
    with torch.cuda.stream(st):
        owner = assign_owners([n for (_, n) in inputs], world, 2)
        if world > 1:
            torch.distributed.barrier()
        H = [None] * len(inputs)
        for i, (_, n) in enumerate(inputs):
            if owner[i] != rank:
                H[i] = torch.empty(n, n, dtype=torch.float32, device="cuda")
                continue
            x = synth_tokens(torch, channel_profile(n, 3000 + i, torch, "cuda"), 4000 + i, TOKENS, spec["tokens"])
            h64 = torch.zeros(n, n, dtype=torch.float64, device="cuda")
            torch.cuda.synchronize()
            clock(lambda: linalg.gram_accumulate_bf16_device(x, h64, lower_only=False, stream=st.cuda_stream),
                  "hessians")
            H[i] = clock(lambda: h64.float(), "hessians")
            del x, h64
        if world > 1:
            def bcast():
                for i, h in enumerate(H):
                    torch.distributed.broadcast(h, src=owner[i])
            clock(bcast, "hessian_broadcast")
        torch.cuda.empty_cache()
        per = (16 if world == 1 else spec["layers"]) * 7
        for l0 in range(0, len(layers), per):
            part = layers[l0:l0 + per]
            used = sorted({inp for (_, _, _, inp) in part})
            remap = {inp: k for k, inp in enumerate(used)}
            part_l = [(nm, d, n, remap[inp]) for (nm, d, n, inp) in part]
            part_in = [inputs[i] for i in used]
            W = [synth_weight(torch, l0 + j, d_out, n, 0.02, spec["outliers"], True)
                 for j, (_, d_out, n, _) in enumerate(part)]
            b = RuntimeBatch(torch, rt, part_l, part_in, [H[i] for i in used], W, cfg, on_device=True)
            torch.cuda.synchronize()
            free_gb.append(round(torch.cuda.mem_get_info()[0] / 2 ** 30, 1))
            if world > 1:
                torch.distributed.barrier()
            clock(lambda: b.run(gather=False), "quantization")
            prof = __import__("cdclq")._lib.last_run_profile()
            for k in eng:
                eng[k] += prof[k]
            factor_batches += int(prof.get("factor_batches", 0))
            stats.extend(b.stats)
            del W, b
            torch.cuda.empty_cache()
        del H
        torch.cuda.empty_cache()
    t = max_over_ranks(torch, [clock.total()] + [clock.ms[k] for k in names], world)
    return {
        "workload": "Llama-2-7B-shaped model (configs[3]): 32 layers, 224 linear layers, %.3g weights, 128 Hessians "
                    "accumulated on the GPU from 262144 seeded bf16 tokens each, inside the timed region" % total_weights,
        "seconds_per_model": t[0] * 1e-3, "weights_per_s": total_weights / (t[0] * 1e-3), "n_gpus": world,
        "target_s": 60.0, "target_gpus": 8, "bits": cfg.bits, "group": cfg.group, "mse_grid": True,
        "refine_frac": cfg.refine_frac, "row_chunk": ROW_CHUNK,
        "phases_s_max_over_ranks": {k: v * 1e-3 for k, v in zip(names, t[1:])},
        "engine_phases_ms_rank0": eng,
        "factor_batches_rank0": factor_batches, "free_gib_before_each_batch_rank0": free_gb,
        "loss_gptq": sum(s.loss_gptq for s in stats), "loss_final": sum(s.loss_final for s in stats),
        "timed": "tensor-core Hessian accumulation + Hessian broadcast + quantization through the runtime "
                 "(synthetic activation and weight generation excluded)",
    }


def fp64_gemm_peak_tflops(torch):
    """cuBLAS DGEMM (8192^3, f64) measured in this run: the FP64 roofline of the factorisation kernels (FP64
    CUDA-core and DMMA peaks are the same on B200; the driver's peaks file has no FP64 figure)."""
    a = torch.randn(8192, 8192, dtype=torch.float64, device="cuda")
    b = torch.randn(8192, 8192, dtype=torch.float64, device="cuda")
    for _ in range(2):
        torch.matmul(a, b)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        torch.matmul(a, b)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 5
    del a, b
    return 2.0 * 8192 ** 3 / (ms * 1e-3) / 1e12


def run_stress70b(args, torch, rank, world):
    """Llama-3-70B-shaped stress layers, down_proj 8192 x 28672 and q_proj 8192 x 8192, f32 weights
    N(0, 0.015^2), Hessians from 262144 Student-t(3) tokens (inputs, built by the SYRK, not timed); 3-bit,
    group 128, block 256, passes 8.  Timed separately (rank 0): the damped f64 Cholesky + triangular inverse of
    the 28672-wide Hessian (cdclq_prepare_factors on that input alone), against a cuBLAS DGEMM measured in the
    same run.  Then the quantization of both layers (which factorises again inside), max over ranks."""
    import ctypes

    import cdclq
    from cdclq.abi import CBatchInput, Config
    from cdclq.pipeline import ModelBatch, shard_rows

    cdclq.lib()
    cfg = Config(bits=3, group=128, block=256, passes=8, row_chunk=ROW_CHUNK)
    st = torch.cuda.current_stream()
    inputs = [("model.layers.0.mlp.down_proj", 28672), ("model.layers.0.self_attn.q_proj", 8192)]
    layers = [("model.layers.0.mlp.down_proj", 8192, 28672, 0), ("model.layers.0.self_attn.q_proj", 8192, 8192, 1)]
    total_weights = sum(l[1] * l[2] for l in layers)
    H = [gpu_hessian(torch, 200 + i, n, TOKENS, "student3", st.cuda_stream, chunk=8192) for i, (_, n) in
         enumerate(inputs)]
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    clock = PhaseClock(torch, st, ("factorisation", "quantization"))
    fact = None
    if rank == 0:
        peak64 = fp64_gemm_peak_tflops(torch)
        ins = (CBatchInput * len(inputs))()
        for i, (_, ni) in enumerate(inputs):
            ins[i].h = H[i].data_ptr()
            ins[i].n = ni
        n = inputs[0][1]
        u = torch.empty(n, n, dtype=torch.float32, device="cuda")
        which = (ctypes.c_size_t * 1)(0)
        u_out = (ctypes.c_void_p * 1)(u.data_ptr())
        c = cfg.to_c()

        def factorise():
            cdclq._lib.check(cdclq.lib().cdclq_prepare_factors(
                ins, len(inputs), ctypes.cast(which, ctypes.c_void_p), 1, ctypes.byref(c),
                ctypes.cast(u_out, ctypes.c_void_p), 1, ctypes.c_void_p(st.cuda_stream)))
        factorise()  # warm-up (allocator pool, first-launch costs)
        clock.ms["factorisation"] = 0.0
        clock(factorise, "factorisation")
        flops = 2.0 * n ** 3 / 3.0  # Cholesky n^3/3 + triangular inverse n^3/3
        ms = clock.ms["factorisation"]
        fact = {"n": n, "s": ms * 1e-3, "flops": flops, "tflops": flops / (ms * 1e-3) / 1e12,
                "fp64_peak_tflops": peak64, "frac": flops / (ms * 1e-3) / 1e12 / peak64,
                "peak_source": "cuBLAS DGEMM 8192^3 measured in this run"}
        del u
        torch.cuda.empty_cache()
    W = []
    for i, (_, d_out, n, _) in enumerate(layers):
        r = shard_rows(d_out, ROW_CHUNK, rank, world, rotate=i) if world > 1 else (0, d_out)
        W.append(synth_weight(torch, i, d_out, n, 0.015, 0.0, False, r, seed0=95000) if r[1] > r[0] else None)
    b = ModelBatch(torch, layers, inputs, H, W, cfg, rank=rank, world=world, on_device=True, w_sharded=True)
    if world > 1:
        torch.distributed.barrier()
    clock(lambda: b.run(st.cuda_stream), "quantization")
    prof = cdclq._lib.last_run_profile()
    loss = max_over_ranks(torch, [sum(s.loss_gptq for s in b.stats), sum(s.loss_final for s in b.stats)], world, "sum")
    t = max_over_ranks(torch, [clock.ms["quantization"]], world)[0]
    if rank == 0:
        print(json.dumps({
            "metric": "seconds to quantize the configs[4] stress layers (incl. CDCL repair)", "value": t * 1e-3,
            "unit": "s", "higher_is_better": False, "n_gpus": world, "weights_per_s": total_weights / (t * 1e-3),
            "config": {"workload": "Llama-3-70B-shaped stress layers (configs[4]): down_proj 8192x28672 + q_proj "
                                   "8192x8192, f32 weights, Hessians from 262144 Student-t(3) tokens (inputs)",
                       "bits": 3, "group": 128, "block": 256, "passes": 8, "row_chunk": ROW_CHUNK},
            "factorisation_n28672_rank0": fact,
            "engine_phases_ms_rank0": {k: prof[k] for k in ("ms_prepare", "ms_phase1", "ms_stats", "ms_repair",
                                                             "ms_final")},
            "loss_gptq": loss[0], "loss_final": loss[1], "data": "synthetic (seeded)",
        }), flush=True)


def workload_config(cfg):
    return {"workload": "TinyLlama-1.1B-shaped model (configs[1]): 22 decoder layers, 154 linear layers, "
                        "9.69e8 bf16-valued weights, 88 Hessians from 262144 seeded tokens",
            "bits": cfg.bits, "group": cfg.group, "mse_grid": cfg.mse_grid, "method": cfg.method,
            "block": cfg.block, "sub_block": cfg.sub_block, "passes": cfg.passes, "tol": cfg.tol,
            "row_chunk": cfg.row_chunk, "l2": "inputs (W 3.9 GB + H 3.8 GB f32) larger than the 126 MB L2"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="decoder layers (22 = the configs[1] model)")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-north-star", action="store_true",
                    help="skip the one-shot configs[3] (Llama-2-7B-shaped, the north star) measurement of the line")
    ap.add_argument("--kernel", default="model", choices=["model", "syrk"],
                    help="syrk: time the bf16 tensor-core Hessian accumulation alone (one JSON line per width)")
    ap.add_argument("--syrk-widths", default="2048,4096,5632,11008", help="--kernel syrk: channel counts n")
    ap.add_argument("--model", default="tinyllama", choices=["tinyllama", "llama2-7b", "gemma2b", "llama3-70b-layers"],
                    help="tinyllama: configs[1] (the driver's line); llama2-7b: configs[3], the north star, Hessians "
                         "accumulated on the GPU inside the timed region; gemma2b: configs[2]; llama3-70b-layers: "
                         "configs[4].  The last three print their own JSON line.")
    ap.add_argument("--bits", type=int, default=4, help="--model llama2-7b: code width (4 or 2)")
    ap.add_argument("--group", type=int, default=0, help="--model llama2-7b: group width (default 64, configs[3])")
    ap.add_argument("--syrk-tokens", type=int, default=TOKENS, help="--kernel syrk: tokens per Hessian")
    args = ap.parse_args()

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)

    if args.impl == "reference":
        run_reference_arm(args, torch, rank, world)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if args.kernel == "syrk":
        if rank == 0:
            run_syrk_bench(args, torch)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if args.model == "llama2-7b":  # the north star alone, through the library's runtime
        import cdclq
        from cdclq.runtime import Runtime

        cdclq.lib()
        rt = Runtime.from_process_group(device=local) if world > 1 else Runtime(device=0)
        res = north_star(torch, rank, world, rt, bits=args.bits, group=args.group or 64)
        if rank == 0:
            print(json.dumps(dict(metric="seconds per model quantized incl. Hessian accumulation and CDCL repair",
                                  value=res["seconds_per_model"], unit="s", higher_is_better=False, **res)),
                  flush=True)
        rt.close()
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if args.model in ("gemma2b", "llama3-70b-layers"):
        (run_stress70b if args.model == "llama3-70b-layers" else run_model)(args, torch, rank, world)
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    import cdclq
    from cdclq.runtime import Runtime

    cdclq.lib()
    cfg = bench_config()
    device = "cuda"
    layers, inputs, H, W = generate(torch, device, args.layers)
    total_weights = sum(l[1] * l[2] for l in layers)
    # the library's runtime on every N: one rank per GPU, its own NCCL communicator (factor broadcasts grouped)
    rt = Runtime.from_process_group(device=local) if world > 1 else Runtime(device=0)
    batch = RuntimeBatch(torch, rt, layers, inputs, H, W, cfg, on_device=True)
    stream = torch.cuda.ExternalStream(rt.stream_handle)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        batch.run(gather=False)
    torch.cuda.synchronize()
    barrier()
    launches0 = cdclq.lib().cdclq_launch_count()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    e0.record(stream)
    profiles = []
    for _ in range(args.steps):
        batch.run(gather=False)
        profiles.append(cdclq._lib.last_run_profile())
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    launches = cdclq.lib().cdclq_launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    # the runtime all-reduces every layer's statistics: every rank holds the model totals
    loss_gptq = sum(s.loss_gptq for s in batch.stats)
    loss_final = sum(s.loss_final for s in batch.stats)

    # ---- e2e through the public C ABI with pinned host buffers: each Hessian uploaded by its owner rank and
    # broadcast over NVLink, each rank uploading its rows of W, outputs gathered on rank 0 and copied to the host
    Hh = [h.cpu().pin_memory() for h in H]
    Wh = [w.cpu().pin_memory() for w in W]
    hb = RuntimeBatch(torch, rt, layers, inputs, Hh, Wh, cfg, on_device=False)
    hb.run(gather=True)  # warm the host path once
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        hb.run(gather=True)
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / args.e2e_steps
    e2e_prof = cdclq._lib.last_run_profile()
    e2e_bytes = (hb.h2d_bytes, hb.d2h_bytes)
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_s = float(t.item())

    # ---- the north star once, in the same run: seconds per Llama-2-7B-shaped model
    ns = None
    if not args.no_north_star:
        # the configs[1] inputs are released (the first decoder layer's stay for the CPU baseline, and every
        # layer's outputs for the parity report); the library keeps its memory pool for the next call
        del hb, Hh, Wh
        batch.keep = []
        H = H[:4] + [None] * (len(H) - 4)
        W = W[:7] + [None] * (len(W) - 7)
        torch.cuda.empty_cache()
        try:
            ns = north_star(torch, rank, world, rt)
        except Exception as ex:  # reported, never at the cost of the main line
            ns = {"error": "%s: %s" % (type(ex).__name__, ex)}
            torch.cuda.empty_cache()

    if rank == 0:
        prof = profiles[-1]
        peaks = load_peaks()
        fp32_peak = fp32_simt_peak_tflops(torch)
        rep_ms = prof["ms_repair"] + prof["ms_final"]  # the persistent repair launch includes the final refit
        rep_flops = prof["flops_repair"] + prof["flops_final"]
        rep_tflops = rep_flops / (rep_ms * 1e-3) / 1e12 if rep_ms > 0 else 0.0
        p1_tflops = prof["flops_phase1"] / (prof["ms_phase1"] * 1e-3) / 1e12 if prof["ms_phase1"] > 0 else 0.0
        line = {
            "metric": METRIC, "value": total_weights / (ms * 1e-3), "unit": "weights/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "seconds_per_model": ms * 1e-3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded bf16-valued weights and tokens; no checkpoints or datasets offline)",
            "config": workload_config(cfg),
            "e2e": {"value": total_weights / e2e_s, "unit": "weights/s", "seconds_per_model": e2e_s,
                    "h2d_bytes_per_step": e2e_bytes[0], "d2h_bytes_per_step": e2e_bytes[1],
                    "bytes_scope": "rank 0: the Hessians it owns (each uploaded once, then broadcast over NVLink) and "
                                   "its rows of W in; every row's codes, scales and zero points out (gathered)",
                    "phases_ms": {k: e2e_prof[k] for k in ("ms_prepare", "ms_phase1", "ms_stats", "ms_repair",
                                                           "ms_final")}},
            "gpu_launches": int(launches),
            "roofline": {
                "kernel": "repair_persistent_kernel (CDCL repair: block gradients on the FP32 SIMT GEMM core, "
                          "per-row refit and coordinate descent)",
                "bound": "fp32", "achieved": rep_tflops, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": rep_tflops / fp32_peak if fp32_peak else None,
                "traffic": repair_traffic_bytes(prof["weights"]),
                "traffic_source": "profiles/repair_persistent_kernel_tinyllama_2layers.md (ncu DRAM bytes of the 2-layer "
                                  "launch per weight, times this launch's weights)",
                "peak_source": "measured in this run: cuBLAS SGEMM 8192^3 with TF32 off (FFMA); MEASURED_PEAKS.json "
                               "has no FP32 CUDA-core figure",
            },
            "phases_ms": {k: prof[k] for k in ("ms_prepare", "ms_phase1", "ms_stats", "ms_repair", "ms_final")},
            "phase1_tflops": p1_tflops,
            "factorisations": prof["factorisations"], "repair_pass_launches": prof["repair_launches"],
            "repair_layout": prof["repair_layout"],
            "loss_gptq": loss_gptq, "loss_final": loss_final,
            "clocks": clk,
            "peaks_file": {k: peaks.get(k) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")},
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"], ref_results = cpu_baseline_sample(layers[:7], inputs[:4], H[:4], W[:7], cfg)
            line["parity"] = parity_report(ref_results, batch, layers)
        if ns is not None:
            line["north_star"] = ns
        print(json.dumps(line), flush=True)
    rt.close()  # every rank: the library's communicator is released before the process group
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
