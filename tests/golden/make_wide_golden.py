#!/usr/bin/env python
"""Generate tests/golden/wide_cases.json: the CPU oracle's results on the wide parity cases of tests/wide_cases.py.

    python tests/golden/make_wide_golden.py [case ...]

For each case (a row slice of a configs[1]-[4] layer at full width, with that configuration's settings) the
script builds the inputs, runs the oracle (oracle/, the C++ restatement of the reference's CPU path) and
records digests of H, W and of every output (permutation, gbits, codes, scales, zero points), the losses,
the accepted moves and the passes each row chunk executed.  The wide inputs are too large to commit; their
digests let the GPU test check that it rebuilt the same inputs before it compares the outputs.

The oracle needs minutes per wide case (the 28672-wide factorisation alone is ~2.5e13 f64 flops), which is
why its results are committed rather than recomputed on the GPU host.  Results are written after every case,
so an interrupted run keeps what it finished.  TEST INFRASTRUCTURE ONLY.
"""
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "cdcl-gptq_b200"))

import oracle as orc  # noqa: E402
import wide_cases as wc  # noqa: E402

OUT = os.path.join(HERE, "wide_cases.json")


def main():
    names = sys.argv[1:] or sorted(wc.CASES, key=lambda k: (wc.CASES[k][0], k))
    try:
        with open(OUT) as f:
            done = json.load(f)
    except (OSError, ValueError):
        done = {}
    cache = {}
    for name in names:
        n, rows, _, _, _, _, settings, seed = wc.CASES[name]
        t0 = time.time()
        if seed not in cache:
            cache.clear()
            cache[seed] = wc.hessian_cpu(name)
        h = cache[seed]
        t_h = time.time() - t0
        w = wc.weights(name)
        cfg = wc.config(name)
        t1 = time.time()
        ql, st, passes = orc.quantize_layer(w, rows, n, h, None, name, cfg, return_chunk_passes=True)
        rec = wc.outputs_digest(ql, st, passes)
        rec.update({"n": n, "rows": rows, "settings": settings, "tokens": wc.TOKENS, "h": wc.digest(h),
                    "w": wc.digest(w), "oracle_threads": orc.max_threads(),
                    "oracle_seconds": {"hessian": round(t_h, 1), "prepare": round(st.secs_prepare, 1),
                                       "quantize": round(st.secs_quant, 1), "wall": round(time.time() - t1, 1)}})
        done[name] = rec
        with open(OUT, "w") as f:
            json.dump(done, f, indent=1, sort_keys=True)
        print("%-15s n=%5d rows=%d loss %.6e -> %.6e passes %s (%.0f s)" % (
            name, n, rows, rec["loss_gptq"], rec["loss_final"], rec["passes"], time.time() - t0), flush=True)


if __name__ == "__main__":
    main()
