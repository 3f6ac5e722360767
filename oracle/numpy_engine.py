"""An independent numpy restatement of the reference's per-layer path, for cross-checking the C++ oracle.

TEST INFRASTRUCTURE ONLY: imported by tests/ (tests/test_numpy_restatement.py), never by the product package.

The C++ oracle (oracle/oracle.cpp) is the bit-exact checker of the GPU library.  This module is a second
restatement written separately, straight from the reference crate, in the style of the reference's own
cross-check script (scripts/ref_gptq_check.py, which restates phase 1 in float64 numpy): vectorised over the
rows of a row chunk, with the reference's f32 / f64 types, but with every GEMM done by numpy (BLAS, whose
summation order differs from the oracle's fixed one) and no code shared with the oracle.  It restates:

  find_params / quant_code / round_f16     src/quant.rs:20-95
  compute_perm                             src/engine.rs:271-304
  build_prepared (damp, dead columns)      src/engine.rs:320-342 (the factor U through numpy's Cholesky of
                                           H^-1, the same unique upper factor as src/linalg.rs:362-375)
  process_chunk phase 1 (blocked GPTQ)     src/engine.rs:366-479
  process_chunk phase 2 (CDCL repair)      src/engine.rs:480-671: conflict selection, the closed-form scale
                                           refit, coordinate descent with the rank-1 gradient updates, the
                                           per-chunk stop rule and the final refit
  quantize_layer (chunking, statistics)    src/engine.rs:690-799

The reference loops over rows inside phase 2; rows are independent there (each row's refit, sweep and
early-exit depend on that row only), so the loops run over columns with all rows of the chunk at once, and a
row leaves a sub-block's sweeps when it made no move (src/engine.rs:651-653).  Sequential f32 sums of the
reference (the MSE error sums, the refit's numerator and denominator) stay sequential here.
"""
import numpy as np

F16_MIN_NORMAL = np.float32(6.1035156e-5)
F32 = np.float32

# The product used for the repair's block gradients (G = E H[:, cols], u H_CC).  None: numpy's BLAS in f32.  A
# caller may set another f32 product here to study how a different arithmetic for those GEMMs (a tensor-core
# emulation, say) changes the repair's decisions; tests/test_numpy_restatement.py does.
REPAIR_MATMUL = None


def _repair_mm(a, b):
    return (REPAIR_MATMUL(a, b) if REPAIR_MATMUL is not None else a @ b).astype(np.float32)


def round_f16(x):
    """src/quant.rs:24-26: nearest f16 (ties to even), widened back to f32."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def round_away(x):
    """f32::round: half away from zero (exact for every f32)."""
    x = np.asarray(x, np.float32)
    t = np.trunc(x)
    frac = np.abs(x - t)  # exact: x and trunc(x) share the exponent range
    return (t + np.sign(x) * (frac >= F32(0.5)).astype(np.float32)).astype(np.float32)


def quant_code(x, scale, zero, maxq):
    """src/quant.rs:90-93 (elementwise)."""
    q = np.clip(round_away(x / scale) + zero, F32(0.0), maxq).astype(np.float32)
    return q, (scale * (q - zero)).astype(np.float32)


def find_params(vals, bits, mse):
    """src/quant.rs:40-83 for every row of `vals` (rows x len) at once."""
    vals = np.asarray(vals, np.float32)
    maxq = F32((1 << bits) - 1)
    xmin = np.minimum(vals.min(axis=1), F32(0.0))
    xmax = np.maximum(vals.max(axis=1), F32(0.0))
    flat = (xmin == 0.0) & (xmax == 0.0)
    xmin = np.where(flat, F32(-1.0), xmin).astype(np.float32)
    xmax = np.where(flat, F32(1.0), xmax).astype(np.float32)

    def mk(lo, hi):
        s = round_f16((hi - lo) / maxq)
        s = np.where(s < F16_MIN_NORMAL, F16_MIN_NORMAL, s).astype(np.float32)
        z = np.clip(round_away(-lo / s), F32(0.0), maxq).astype(np.float32)
        return s, z

    if not mse:
        return mk(xmin, xmax)
    best_s, best_z = mk(xmin, xmax)
    best_err = np.full(vals.shape[0], np.inf, np.float32)
    for i in range(24):
        p = F32(1.0) - F32(0.02) * F32(i)
        s, z = mk(p * xmin, p * xmax)
        err = np.zeros(vals.shape[0], np.float32)
        for k in range(vals.shape[1]):  # sequential f32 sum, as the reference's loop
            _, d = quant_code(vals[:, k], s, z, maxq)
            e = d - vals[:, k]
            err = (err + e * e).astype(np.float32)
        better = err < best_err
        best_err = np.where(better, err, best_err)
        best_s = np.where(better, s, best_s)
        best_z = np.where(better, z, best_z)
    return best_s.astype(np.float32), best_z.astype(np.float32)


def effective_group(group, n):
    """src/engine.rs:227-233."""
    return n if group == 0 or group >= n else group


def compute_perm(hdiag, w, n, g, cfg):
    """src/engine.rs:271-304: (perm, nskel)."""
    nskel = 0
    perm = []
    in_skel = np.zeros(n, bool)
    if cfg.skeleton_pct > 0.0 and g < n:
        nskel = min(int(round_half_away(cfg.skeleton_pct / 100.0 * n / g)), max(n // g - 1, 0))
        if nskel > 0:
            w64 = np.asarray(w, np.float64)
            colsq = np.zeros(n)
            for r in range(w64.shape[0]):  # row-ordered f64 sums
                colsq += w64[r] * w64[r]
            crit = hdiag * colsq
            idx = sorted(range(n), key=lambda j: (-crit[j], j))
            for j in idx[:nskel * g]:
                in_skel[j] = True
                perm.append(j)
    rest = [j for j in range(n) if not in_skel[j]]
    if cfg.act_order:
        rest.sort(key=lambda j: (-hdiag[j], j))
    return np.array(perm + rest, np.uint32), nskel


def round_half_away(x):
    return np.floor(x + 0.5) if x >= 0 else -np.floor(-x + 0.5)


def build_prepared(h, n, perm, damp):
    """src/engine.rs:320-342: (U f32, damped permuted H as f32, damp_val)."""
    hp = np.asarray(h, np.float32).reshape(n, n).astype(np.float64)[np.ix_(perm, perm)]
    d = np.diagonal(hp).copy()
    d[d == 0.0] = 1.0
    mean = np.cumsum(d)[-1] / n  # sequential sum
    damp_val = damp * mean
    hp[np.diag_indices(n)] = d + damp_val
    h32 = hp.astype(np.float32)
    u = np.linalg.cholesky(np.linalg.inv(hp)).T  # the unique upper U with H^-1 = U^T U, positive diagonal
    return np.triu(u).astype(np.float32), h32, damp_val


def process_chunk(wt, u, h, gbits, g, cfg):
    """src/engine.rs:366-671 on one row chunk.  Returns (codes, scales, zeros, stats dict)."""
    rows, n = wt.shape
    ng = (n + g - 1) // g
    bsz = cfg.block
    w = wt.astype(np.float32).copy()
    wq = np.zeros((rows, n), np.float32)
    codes = np.zeros((rows, n), np.float32)  # integer-valued
    scales = np.zeros((rows, ng), np.float32)
    zeros = np.zeros((rows, ng), np.float32)
    colloss = np.zeros(n)

    # ---- phase 1: blocked GPTQ with lazy updates (src/engine.rs:398-466)
    i1 = 0
    while i1 < n:
        i2 = min(i1 + bsz, n)
        cnt = i2 - i1
        w1 = w[:, i1:i2].copy()
        err1 = np.zeros((rows, cnt), np.float32)
        for i in range(cnt):
            j = i1 + i
            if j % g == 0:
                gi = j // g
                gend = min(j + g, n)
                cols = [w1[:, c - i1] if c < i2 else w[:, c] for c in range(j, gend)]
                s, z = find_params(np.stack(cols, axis=1), int(gbits[gi]), cfg.mse_grid)
                scales[:, gi], zeros[:, gi] = s, z
            gi = j // g
            maxq = F32((1 << int(gbits[gi])) - 1)
            inv_d = F32(1.0) / u[j, j]
            q, dq = quant_code(w1[:, i], scales[:, gi], zeros[:, gi], maxq)
            codes[:, j] = q
            wq[:, j] = dq
            e = ((w1[:, i] - dq) * inv_d).astype(np.float32)
            colloss[j] = float(np.cumsum((e * e).astype(np.float64))[-1])  # rows in order
            err1[:, i] = e
            if i + 1 < cnt:
                w1[:, i + 1:] = (w1[:, i + 1:] - e[:, None] * u[j, j + 1:i2][None, :]).astype(np.float32)
        if i2 < n:
            w[:, i2:] = (w[:, i2:] - err1 @ u[i1:i2, i2:]).astype(np.float32)
        i1 = i2
    loss_gptq = float(np.cumsum(colloss)[-1])

    # ---- phase 2: conflict selection and repair (src/engine.rs:480-671)
    sbw = cfg.sub_block
    n_sb = (n + sbw - 1) // sbw
    loss_delta, refined, updates, passes_done = 0.0, 0, 0, 0
    do_cd = cfg.refine_frac > 0.0 and cfg.cd_sweeps > 0 and cfg.passes > 0
    do_refit = bool(cfg.refit_scales) and g <= 1024
    if cfg.method == "cdcl" and (do_cd or do_refit):
        sel = []
        if do_cd:
            sbl = [(float(np.cumsum(colloss[s * sbw:min((s + 1) * sbw, n)])[-1]), s) for s in range(n_sb)]
            sbl.sort(key=lambda x: (-x[0], x[1]))
            k = min(max(int(np.ceil(cfg.refine_frac * n_sb)), 1), n_sb)
            sel = sorted(s for _, s in sbl[:k])
            refined = len(sel)
        e = (wt - wq).astype(np.float32)

        def refit_all():
            nonlocal loss_delta
            changed = 0
            for gi in range(ng):
                c0, c1 = gi * g, min(gi * g + g, n)
                gs = _repair_mm(e, h[:, c0:c1])
                hcc = h[c0:c1, c0:c1]
                uu = (codes[:, c0:c1] - zeros[:, gi][:, None]).astype(np.float32)
                hu = _repair_mm(uu, hcc)
                num = np.zeros(rows, np.float32)
                den = np.zeros(rows, np.float32)
                for k in range(c1 - c0):  # sequential f32 sums, as the reference's iterator sums
                    num = (num + uu[:, k] * gs[:, k]).astype(np.float32)
                    den = (den + uu[:, k] * hu[:, k]).astype(np.float32)
                ok = den > F32(1e-30)
                s_old = scales[:, gi]
                with np.errstate(divide="ignore", invalid="ignore"):
                    s_new = round_f16(s_old + num / den)
                s_new = np.where(s_new < F16_MIN_NORMAL, F16_MIN_NORMAL, s_new).astype(np.float32)
                d = (s_new - s_old).astype(np.float32)
                dl = (F32(-2.0) * d * num + d * d * den).astype(np.float32).astype(np.float64)
                acc = ok & (dl < 0.0)
                for r in np.nonzero(acc)[0]:  # rows in order
                    loss_delta += float(dl[r])
                if acc.any():
                    ndq = (s_new[:, None] * uu).astype(np.float32)
                    blk_e = (e[:, c0:c1] + (wq[:, c0:c1] - ndq)).astype(np.float32)
                    e[:, c0:c1] = np.where(acc[:, None], blk_e, e[:, c0:c1])
                    wq[:, c0:c1] = np.where(acc[:, None], ndq, wq[:, c0:c1])
                    scales[:, gi] = np.where(acc, s_new, s_old)
                    changed += int(acc.sum())
            return changed

        prev_delta = 0.0
        for _ in range(max(cfg.passes, 1)):
            passes_done += 1
            pass_updates = 0
            if do_refit:
                pass_updates += refit_all()
            if do_cd:
                for s in sel:
                    c0, c1 = s * sbw, min((s + 1) * sbw, n)
                    wd = c1 - c0
                    gs = _repair_mm(e, h[:, c0:c1])
                    hss = h[c0:c1, c0:c1]
                    active = np.ones(rows, bool)
                    deltas = np.zeros(rows)  # per-row running sums, added in row order below
                    for _sw in range(cfg.cd_sweeps):
                        changed = np.zeros(rows, bool)
                        for jj in range(wd):
                            j = c0 + jj
                            gi = j // g
                            maxq = F32((1 << int(gbits[gi])) - 1)
                            sc, z = scales[:, gi], zeros[:, gi]
                            hjj = hss[jj, jj]
                            cur = wq[:, j]
                            target = (cur + gs[:, jj] / hjj).astype(np.float32)
                            q, newdq = quant_code(target, sc, z, maxq)
                            mv = active & (q != codes[:, j])
                            if not mv.any():
                                continue
                            de = (cur - newdq).astype(np.float32)
                            dlt = (F32(2.0) * de * gs[:, jj] + de * de * hjj).astype(np.float32).astype(np.float64)
                            deltas = np.where(mv, deltas + dlt, deltas)
                            gs = np.where(mv[:, None], (gs + de[:, None] * hss[jj][None, :]).astype(np.float32), gs)
                            wq[:, j] = np.where(mv, newdq, cur)
                            codes[:, j] = np.where(mv, q, codes[:, j])
                            e[:, j] = np.where(mv, (e[:, j] + de).astype(np.float32), e[:, j])
                            pass_updates += int(mv.sum())
                            changed |= mv
                        active &= changed  # a row's sweeps stop once a sweep moved nothing
                        if not active.any():
                            break
                    for r in range(rows):
                        loss_delta += float(deltas[r])
            updates += pass_updates
            gain = prev_delta - loss_delta
            prev_delta = loss_delta
            if pass_updates == 0 or gain < cfg.tol * (loss_gptq + loss_delta):
                break
        if do_refit:
            updates += refit_all()
    stats = dict(loss_gptq=loss_gptq, loss_final=loss_gptq + loss_delta, sb_total=n_sb, sb_refined=refined,
                 updates=updates, passes=passes_done)
    return codes.astype(np.uint8), scales, zeros, stats


def quantize_layer(w, h, cfg, prepared=None):
    """src/engine.rs:690-799 (symmetric target).  `prepared` = (perm, U, h32) to start from given factors (to
    compare phases 1-2 alone); None restates the preparation here.  Returns a dict of the outputs and the
    summed statistics, plus the passes each row chunk executed."""
    w = np.asarray(w, np.float32)
    d_out, n = w.shape
    h = np.asarray(h, np.float32).reshape(n, n)
    g = effective_group(cfg.group, n)
    ng = (n + g - 1) // g
    hdiag = np.diagonal(h).astype(np.float64)
    w0 = w.copy()
    w0[:, hdiag == 0.0] = 0.0  # dead columns (src/engine.rs:708-716)
    if prepared is None:
        perm, nskel = compute_perm(hdiag, w0, n, g, cfg)
        u, h32, _ = build_prepared(h, n, perm, cfg.damp)
    else:
        perm, u, h32 = prepared
        perm = np.asarray(perm, np.uint32)
        _, nskel = compute_perm(hdiag, w0, n, g, cfg)
    wt = w0[:, perm]
    gbits = np.array([cfg.skeleton_bits if gi < nskel else cfg.bits for gi in range(ng)], np.uint8)
    rc = cfg.row_chunk
    codes = np.zeros((d_out, n), np.uint8)
    scales = np.zeros((d_out, ng), np.float32)
    zeros = np.zeros((d_out, ng), np.float32)
    tot = dict(loss_gptq=0.0, loss_final=0.0, sb_total=0, sb_refined=0, updates=0)
    passes = []
    for r0 in range(0, d_out, rc):
        r1 = min(r0 + rc, d_out)
        c, s, z, st = process_chunk(wt[r0:r1], u, h32, gbits, g, cfg)
        codes[r0:r1], scales[r0:r1], zeros[r0:r1] = c, s, z
        for k in tot:
            tot[k] += st[k]
        passes.append(st["passes"])
    return dict(perm=perm, gbits=gbits, codes=codes, scales=scales, zeros=zeros, stats=tot,
                passes=np.array(passes), skeleton_groups=nskel)
