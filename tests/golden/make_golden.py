"""Generate the golden fixtures under tests/golden/ (run in a container where the reference is mounted).

    python tests/golden/make_golden.py /path/to/reference

1. `numpy_gptq_<case>.npz`: the reference's own independent float64 numpy GPTQ (scripts/ref_gptq_check.py)
   executed on a dump in the format of `cdclq bench --dump` (src/bench.rs:345-366).  The dump's inputs W/H
   are seeded synthetic problems; its codes/scales/zeros/loss come from the CPU oracle in GPTQ mode with
   act-order off (the script works in natural column order).  The fixture stores the inputs, the oracle's
   outputs and the numpy reference's own codes/scales/zeros/loss, plus the script's verdict.  The script's
   pass rule (codes >= 99.5 % identical, direct loss within 5e-3) is the reference's own cross-check
   threshold (scripts/ref_gptq_check.py:82).
2. `fixture_hessians.npz`: a few calibration Hessians of the reference's test fixtures
   (tests/fixtures/*/hess.safetensors, synthetic by scripts/gen_toy_hessians.py), used as real `H` inputs of
   the parity tests, with the widths the reference's end-to-end suite exercises (16, 64, 172, 256).

Nothing here is read from the reference at test time; only the committed .npz files are.
"""
import contextlib
import io
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "cdcl-gptq_b200"))

import oracle as orc  # noqa: E402
from cdclq.abi import Config  # noqa: E402

CASES = [
    # name, rows, cols, tokens, seed, bits, group, block
    ("r64_c256_g64_b3", 64, 256, 1024, 101, 3, 64, 128),
    ("r48_c192_g32_b4", 48, 192, 800, 202, 4, 32, 64),
    ("r32_c128_g128_b2", 32, 128, 512, 303, 2, 128, 32),
]


def run_reference_check(ref_root, dump_dir):
    """Execute scripts/ref_gptq_check.py on `dump_dir`; return (globals, exit_code, stdout)."""
    script = os.path.join(ref_root, "scripts", "ref_gptq_check.py")
    src = open(script).read()
    g = {"__name__": "__main__", "__file__": script}
    argv = sys.argv
    sys.argv = [script, dump_dir]
    buf = io.StringIO()
    code = 0
    try:
        with contextlib.redirect_stdout(buf):
            exec(compile(src, script, "exec"), g)
    except SystemExit as e:
        code = int(e.code or 0)
    finally:
        sys.argv = argv
    return g, code, buf.getvalue()


def make_numpy_cases(ref_root):
    for name, rows, cols, tokens, seed, bits, group, block in CASES:
        w, h = orc.problem(rows, cols, tokens, seed)
        cfg = Config(bits=bits, group=group, block=block, method="gptq", act_order=False, row_chunk=16)
        ql, st = orc.quantize_layer(w, rows, cols, h, None, "dump", cfg)
        with tempfile.TemporaryDirectory() as d:
            w.astype("<f4").tofile(os.path.join(d, "W.f32"))
            h.astype("<f4").tofile(os.path.join(d, "H.f32"))
            ql.codes.astype(np.uint8).tofile(os.path.join(d, "codes.u8"))
            ql.scales.astype("<f4").tofile(os.path.join(d, "scales.f32"))
            ql.zeros.astype("<f4").tofile(os.path.join(d, "zeros.f32"))
            with open(os.path.join(d, "meta.json"), "w") as f:
                f.write(json.dumps({"rows": rows, "cols": cols, "bits": bits, "group": group, "damp": cfg.damp,
                                    "block": block, "loss": st.loss_gptq}))
            g, code, out = run_reference_check(ref_root, d)
        np.savez_compressed(
            os.path.join(HERE, "numpy_gptq_%s.npz" % name),
            w=w, h=h, rows=rows, cols=cols, bits=bits, group=group, block=block, damp=cfg.damp, row_chunk=16,
            oracle_codes=ql.codes, oracle_scales=ql.scales, oracle_zeros=ql.zeros, oracle_loss=st.loss_gptq,
            ref_codes=g["codes"], ref_scales=g["scales"].astype(np.float32), ref_zeros=g["zeros"].astype(np.float32),
            ref_loss_tracked=float(g["loss"]), ref_exit=code, ref_stdout=np.array(out),
        )
        print(name, "reference check exit", code)
        print(out)


def make_fixture_hessians(ref_root):
    from safetensors import safe_open

    picks = [
        ("tiny-random-Llama-3", "model.layers.0.mlp.gate_proj.H"),   # 16 wide
        ("tiny-random-Llama-3", "model.layers.0.mlp.down_proj.H"),   # 64 wide
        ("tiny-random-llama2", "model.layers.0.mlp.down_proj.H"),    # 172 wide (ragged groups)
        ("tiny-random-llama2", "model.layers.1.self_attn.k_proj.H"), # 256 wide
    ]
    out = {}
    for model, key in picks:
        p = os.path.join(ref_root, "tests", "fixtures", model, "hess.safetensors")
        with safe_open(p, "np") as f:
            out["%s/%s" % (model, key)] = f.get_tensor(key).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "fixture_hessians.npz"), **out)
    print("fixture hessians:", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CDCLQ_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py /path/to/reference")
    make_numpy_cases(ref)
    make_fixture_hessians(ref)
