// oracle.cpp - CPU restatement of the reference's per-layer quantization path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA library is compared against; it is
// loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU-baseline / `--impl reference` legs, and
// by nothing else.  The product library (cdcl-gptq_b200/) never links or calls it.
//
// What it restates (all citations are paths inside the reference crate tailot/CDCL-GPTQ):
//   src/rng.rs:22-57         splitmix64 + Box-Muller generator            -> Rng
//   src/quant.rs:20-95        f16 rounding, find_params, quant_code         -> round_f16, find_params, quant_code
//   src/quant.rs:98-151       row_bits/row_bytes, pack_row/unpack_row      -> row_bytes, pack_row, unpack_row
//   src/quant.rs:189-202      QLayer::dequantize                           -> oracle_dequantize
//   src/linalg.rs:56-184      strided GEMM wrappers                        -> gemm<T>
//   src/linalg.rs:200-276     blocked right-looking Cholesky (NB=96,TB=64) -> cholesky_lower
//   src/linalg.rs:284-347     blocked lower-triangular inverse (NB=96)     -> tri_inverse_lower
//   src/linalg.rs:362-375     flip-trick upper factor of H^-1              -> upper_chol_of_inverse
//   src/linalg.rs:388-418     Gram accumulation, 2048-token chunks         -> gram_accumulate
//   src/engine.rs:227-342     effective_group, validate, compute_perm, build_prepared
//   src/engine.rs:366-674     process_chunk (phase 1 GPTQ, phase 2 CDCL repair)
//   src/engine.rs:690-799     quantize_layer (chunking, stats summation)
//   src/engine.rs:808-838     proxy_loss, rtn_layer
//
// The one place where the reference's arithmetic is not in the reference itself: every GEMM goes through the
// third-party crate `matrixmultiply` =0.3.8 (Cargo.lock), which is not vendored.  Its summation order is
// therefore unpinned, and this restatement fixes one: for every output element, the products are accumulated
// in increasing k with a fused multiply-add starting from +0, and the result is combined as
//     beta == 0 : c = alpha * acc
//     beta != 0 : c = alpha * acc + beta * c      (two roundings for the products, one for the sum)
// (see gemm<T> below).  The CUDA kernels follow this order element by element, which is what makes the
// comparison bit-exact.  Everything else (scalar loops in linalg.rs and engine.rs) follows the reference's
// own operation order, with no FMA contraction (compile with -ffp-contract=off), as Rust never contracts.
//
// Parallelism mirrors the reference's rayon use (row chunks in parallel, Cholesky panel rows in parallel)
// via OpenMP; no result depends on the thread count except through the automatic row chunk, exactly as in
// the reference.

#include "cdclq.h"

#include <omp.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace orc {

static thread_local std::string g_err;

static int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

// ---------------------------------------------------------------------------------------------------------
// src/rng.rs:22-57  splitmix64 + Box-Muller (spare cached)
struct Rng {
    uint64_t s;
    bool has_spare = false;
    float spare = 0.f;
    explicit Rng(uint64_t seed) : s(seed + 0x9E3779B97F4A7C15ull) {}
    uint64_t next_u64() {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t z = s;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    float uniform() { return ((float)(next_u64() >> 40) + 0.5f) / (float)(1ull << 24); }
    float normal() {
        if (has_spare) {
            has_spare = false;
            return spare;
        }
        float u1 = uniform();
        float u2 = uniform();
        float r = std::sqrt(-2.0f * std::log(u1));
        float th = 2.0f * 3.14159274101257324219f * u2;  // std::f32::consts::PI
        spare = r * std::sin(th);
        has_spare = true;
        return r * std::cos(th);
    }
};

// ---------------------------------------------------------------------------------------------------------
// src/quant.rs:20-26  F16_MIN_NORMAL and round_f16 (half 2.4.1 f16::from_f32 is IEEE round-to-nearest-even)
static const float F16_MIN_NORMAL = 6.1035156e-5f;

static inline float bits_f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
static inline uint32_t f_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}

// f32 -> f16 (round to nearest, ties to even) -> f32, written from the IEEE-754 binary16 definition.
static inline float round_f16(float x) {
    uint32_t u = f_bits(x);
    uint32_t sign = u & 0x80000000u;
    uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) return x;                       // inf / nan unchanged (nan stays nan)
    if (a >= 0x477ff000u) return bits_f(sign | 0x7f800000u);  // >= 65520 rounds to infinity
    if (a < 0x38800000u) {                                // below 2^-14: f16 subnormal grid of step 2^-24
        float ax = bits_f(a);
        float k = std::nearbyint(ax * 16777216.0f);       // exact scaling; nearbyint = ties to even
        return bits_f(sign | f_bits(k * 5.9604644775390625e-8f));
    }
    uint32_t lsb = (a >> 13) & 1u;
    a += 0x0fffu + lsb;
    a &= 0xffffe000u;
    return bits_f(sign | a);
}

// src/quant.rs:92-95  quant_code.  Rust's clamp lets NaN through and `as u8` maps NaN to 0.
static inline void quant_code(float x, float scale, float zero, float maxq, uint8_t* c, float* dq) {
    float q = std::round(x / scale) + zero;  // f32::round = half away from zero = std::round
    if (q < 0.0f) q = 0.0f;
    if (q > maxq) q = maxq;
    *c = (q == q) ? (uint8_t)q : (uint8_t)0;
    *dq = scale * (q - zero);
}

// src/quant.rs:54-61  the `mk` closure of find_params
static inline void grid_mk(float lo, float hi, float maxq, float* s, float* z) {
    float scale = round_f16((hi - lo) / maxq);
    if (scale < F16_MIN_NORMAL) scale = F16_MIN_NORMAL;
    float zero = std::round(-lo / scale);
    if (zero < 0.0f) zero = 0.0f;
    if (zero > maxq) zero = maxq;
    *s = scale;
    *z = zero;
}

// src/quant.rs:40-83  find_params over `len` values read with stride `stride`.
// Range seeded with 0 (so the grid contains 0); min/max by strict comparison (Rust leaves the sign of a zero
// result unspecified; the compare-select form is the IEEE minNum restatement both implementations share).
static inline void find_params(const float* v, size_t len, size_t stride, uint32_t bits, bool mse, float* s_out,
                               float* z_out) {
    float maxq = (float)((1u << bits) - 1u);
    float xmin = 0.0f, xmax = 0.0f;
    for (size_t i = 0; i < len; i++) {
        float x = v[i * stride];
        if (x < xmin) xmin = x;
        if (x > xmax) xmax = x;
    }
    if (xmin == 0.0f && xmax == 0.0f) {
        xmin = -1.0f;
        xmax = 1.0f;
    }
    float bs, bz;
    grid_mk(xmin, xmax, maxq, &bs, &bz);
    if (!mse) {
        *s_out = bs;
        *z_out = bz;
        return;
    }
    float best_err = INFINITY;
    for (int i = 0; i < 24; i++) {
        float p = 1.0f - 0.02f * (float)i;
        float s, z;
        grid_mk(p * xmin, p * xmax, maxq, &s, &z);
        float err = 0.0f;
        for (size_t t = 0; t < len; t++) {
            float x = v[t * stride];
            uint8_t c;
            float d;
            quant_code(x, s, z, maxq, &c, &d);
            float e = d - x;
            err += e * e;
        }
        if (err < best_err) {
            best_err = err;
            bs = s;
            bz = z;
        }
    }
    *s_out = bs;
    *z_out = bz;
}

// ---------------------------------------------------------------------------------------------------------
// src/linalg.rs:56-99  C = alpha * A * B + beta * C with explicit strides, in the fixed order documented at
// the top of this file.  Vectorised over output columns; the per-element order is sequential in k.
template <typename T>
static void gemm(size_t m, size_t k, size_t n, T alpha, const T* a, ptrdiff_t rsa, ptrdiff_t csa, const T* b,
                 ptrdiff_t rsb, ptrdiff_t csb, T beta, T* c, ptrdiff_t rsc, ptrdiff_t csc, bool parallel) {
    if (m == 0 || n == 0) return;
    if (k == 0) {  // src/linalg.rs:82-91
        if (beta != (T)1) {
            for (size_t i = 0; i < m; i++)
                for (size_t j = 0; j < n; j++) {
                    T* p = c + (ptrdiff_t)i * rsc + (ptrdiff_t)j * csc;
                    *p = (beta == (T)0) ? (T)0 : *p * beta;
                }
        }
        return;
    }
    // B with unit column stride is read in place; otherwise a row-major copy is taken (exact).
    std::vector<T> bcopy;
    const T* bb = b;
    ptrdiff_t ldb = rsb;
    if (csb != 1) {
        bcopy.resize(k * n);
        for (size_t t = 0; t < k; t++)
            for (size_t j = 0; j < n; j++) bcopy[t * n + j] = b[(ptrdiff_t)t * rsb + (ptrdiff_t)j * csb];
        bb = bcopy.data();
        ldb = (ptrdiff_t)n;
    }
    const size_t JT = 512;
    auto row_block = [&](size_t i0, size_t i1) {
        std::vector<T> acc(4 * JT);
        for (size_t j0 = 0; j0 < n; j0 += JT) {
            size_t jn = std::min(JT, n - j0);
            for (size_t i = i0; i < i1; i += 4) {
                size_t ni = std::min<size_t>(4, i1 - i);
                std::fill(acc.begin(), acc.end(), (T)0);
                for (size_t t = 0; t < k; t++) {
                    const T* brow = bb + (ptrdiff_t)t * ldb + (ptrdiff_t)j0;
                    for (size_t r = 0; r < ni; r++) {
                        T av = a[(ptrdiff_t)(i + r) * rsa + (ptrdiff_t)t * csa];
                        T* ac = acc.data() + r * JT;
                        for (size_t j = 0; j < jn; j++) ac[j] = std::fma(av, brow[j], ac[j]);
                    }
                }
                for (size_t r = 0; r < ni; r++) {
                    const T* ac = acc.data() + r * JT;
                    for (size_t j = 0; j < jn; j++) {
                        T* p = c + (ptrdiff_t)(i + r) * rsc + (ptrdiff_t)(j0 + j) * csc;
                        if (beta == (T)0)
                            *p = alpha * ac[j];
                        else
                            *p = alpha * ac[j] + beta * *p;
                    }
                }
            }
        }
    };
    if (parallel && m >= 8 && (double)m * (double)n * (double)k >= (double)(1u << 21)) {
        size_t nb = (m + 3) / 4;
#pragma omp parallel for schedule(dynamic, 1)
        for (size_t bi = 0; bi < nb; bi++) row_block(bi * 4, std::min(m, bi * 4 + 4));
    } else {
        row_block(0, m);
    }
}

// ---------------------------------------------------------------------------------------------------------
// src/linalg.rs:200-276  blocked right-looking Cholesky, NB = 96 diagonal blocks, TB = 64 trailing row chunks.
static int cholesky_lower(double* a, size_t n) {
    const size_t NB = 96, TB = 64;
    size_t k = 0;
    while (k < n) {
        size_t kb = std::min(NB, n - k);
        size_t kend = k + kb;
        // 1. unblocked factorisation of the diagonal block (src/linalg.rs:209-229)
        for (size_t j = k; j < kend; j++) {
            double d = a[j * n + j];
            for (size_t t = k; t < j; t++) {
                double v = a[j * n + t];
                d -= v * v;
            }
            if (!(d > 0.0) || !std::isfinite(d)) {
                char buf[256];
                std::snprintf(buf, sizeof buf,
                              "matrix is not positive definite (pivot %zu = %e); increase --damp or check the Hessian",
                              j, d);
                return fail(CDCLQ_ERR_NOT_PD, buf);
            }
            d = std::sqrt(d);
            a[j * n + j] = d;
            for (size_t i = j + 1; i < kend; i++) {
                double s = a[i * n + j];
                for (size_t t = k; t < j; t++) s -= a[i * n + t] * a[j * n + t];
                a[i * n + j] = s / d;
            }
        }
        if (kend < n) {
            // 2. panel solve X L_kk^T = A_panel (src/linalg.rs:232-241)
#pragma omp parallel for schedule(static)
            for (size_t i = kend; i < n; i++) {
                double* row = a + i * n;
                for (size_t j = k; j < kend; j++) {
                    double s = row[j];
                    for (size_t t = k; t < j; t++) s -= row[t] * a[j * n + t];
                    row[j] = s / a[j * n + j];
                }
            }
            // 3. trailing lower update with a copy of the panel (src/linalg.rs:242-271)
            size_t rows_below = n - kend;
            std::vector<double> panel(rows_below * kb);
            for (size_t i = 0; i < rows_below; i++)
                std::memcpy(&panel[i * kb], a + (kend + i) * n + k, kb * sizeof(double));
            size_t nchunks = (rows_below + TB - 1) / TB;
#pragma omp parallel for schedule(dynamic, 1)
            for (size_t ci = 0; ci < nchunks; ci++) {
                size_t i0 = ci * TB;
                size_t mrows = std::min(TB, rows_below - i0);
                size_t cols = i0 + mrows;
                gemm<double>(mrows, kb, cols, -1.0, panel.data() + i0 * kb, (ptrdiff_t)kb, 1, panel.data(), 1,
                             (ptrdiff_t)kb, 1.0, a + (kend + i0) * n + kend, (ptrdiff_t)n, 1, false);
            }
        }
        k = kend;
    }
    return CDCLQ_OK;
}

// src/linalg.rs:284-347  blocked inverse of a lower-triangular matrix (lower triangle of l read only).
static void tri_inverse_lower(const double* l, size_t n, double* y) {
    const size_t NB = 96;
    std::fill(y, y + n * n, 0.0);
    size_t s = 0;
    while (s < n) {
        size_t e = std::min(s + NB, n);
        size_t w = e - s;
        std::vector<double> yii(w * w, 0.0);
        for (size_t c = 0; c < w; c++) {
            yii[c * w + c] = 1.0 / l[(s + c) * n + (s + c)];
            for (size_t i = c + 1; i < w; i++) {
                double acc = 0.0;
                for (size_t t = c; t < i; t++) acc += l[(s + i) * n + (s + t)] * yii[t * w + c];
                yii[i * w + c] = -acc / l[(s + i) * n + (s + i)];
            }
        }
        for (size_t i = 0; i < w; i++)
            for (size_t j = 0; j <= i; j++) y[(s + i) * n + (s + j)] = yii[i * w + j];
        if (s > 0) {
            std::vector<double> t(w * s);
            gemm<double>(w, s, s, 1.0, l + s * n, (ptrdiff_t)n, 1, y, (ptrdiff_t)n, 1, 0.0, t.data(), (ptrdiff_t)s,
                         1, true);
            gemm<double>(w, w, s, -1.0, yii.data(), (ptrdiff_t)w, 1, t.data(), (ptrdiff_t)s, 1, 0.0, y + s * n,
                         (ptrdiff_t)n, 1, true);
        }
        s = e;
    }
}

// src/linalg.rs:362-375  U (upper, f32) with H^-1 = U^T U via the flip trick.  `h` is consumed.
static int upper_chol_of_inverse(std::vector<double>& h, size_t n, float* u) {
    std::reverse(h.begin(), h.end());  // conjugate by J on both axes
    int rc = cholesky_lower(h.data(), n);
    if (rc != CDCLQ_OK) return rc;
    std::vector<double> y(n * n);
    tri_inverse_lower(h.data(), n, y.data());
    std::vector<double>().swap(h);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++)
        for (size_t j = 0; j < n; j++)
            u[i * n + j] = (j >= i) ? (float)y[(n - 1 - i) * n + (n - 1 - j)] : 0.0f;
    return CDCLQ_OK;
}

// src/linalg.rs:388-418  H += X^T Y in 2048-token chunks (f32 GEMM into a scratch, widened into f64).
static void gram_accumulate(const float* x, const float* y, size_t t, size_t n, double* h) {
    const size_t TC = 2048;
    std::vector<float> tmp(n * n);
    for (size_t t0 = 0; t0 < t; t0 += TC) {
        size_t tc = std::min(TC, t - t0);
        gemm<float>(n, tc, n, 1.0f, x + t0 * n, 1, (ptrdiff_t)n, y + t0 * n, (ptrdiff_t)n, 1, 0.0f, tmp.data(),
                    (ptrdiff_t)n, 1, true);
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < n * n; i++) h[i] += (double)tmp[i];
    }
}

// ---------------------------------------------------------------------------------------------------------
// src/engine.rs:227-258
static size_t effective_group(const cdclq_config* cfg, size_t n) {
    return (cfg->group == 0 || cfg->group >= n) ? n : (size_t)cfg->group;
}

static int validate(const cdclq_config* cfg, size_t n) {
    if (cfg->bits < 2 || cfg->bits > 8 || cfg->skeleton_bits < 2 || cfg->skeleton_bits > 8)
        return fail(CDCLQ_ERR_CONFIG, "bits and skeleton_bits must be in 2..=8");
    if (cfg->block == 0 || cfg->sub_block == 0) return fail(CDCLQ_ERR_CONFIG, "block and sub_block must be > 0");
    size_t g = effective_group(cfg, n);
    if (g < n && cfg->block % g != 0 && g % cfg->block != 0)
        return fail(CDCLQ_ERR_CONFIG, "group size " + std::to_string(g) + " must divide the block size " +
                                          std::to_string(cfg->block) + " (or be a multiple of it)");
    if (cfg->skeleton_pct > 0.0 && g >= n) return fail(CDCLQ_ERR_CONFIG, "the skeleton needs a finite group size");
    if (!(cfg->refine_frac >= 0.0 && cfg->refine_frac <= 1.0))
        return fail(CDCLQ_ERR_CONFIG, "refine_frac must be in [0, 1]");
    return CDCLQ_OK;
}

// src/engine.rs:271-304
static void compute_perm(const std::vector<double>& hdiag, const float* w, size_t d_out, size_t n, size_t g,
                         const cdclq_config* cfg, std::vector<uint32_t>& perm, size_t* nskel_out) {
    size_t nskel = 0;
    perm.clear();
    std::vector<char> in_skel(n, 0);
    if (cfg->skeleton_pct > 0.0 && g < n) {
        size_t full_groups = n / g;
        double r = std::round(cfg->skeleton_pct / 100.0 * (double)n / (double)g);
        size_t want = r > 0.0 ? (size_t)r : 0;  // `as usize` saturates at 0
        nskel = std::min(want, full_groups > 0 ? full_groups - 1 : 0);
        if (nskel > 0) {
            std::vector<double> colsq(n, 0.0);
            for (size_t rr = 0; rr < d_out; rr++)
                for (size_t j = 0; j < n; j++) colsq[j] += (double)w[rr * n + j] * (double)w[rr * n + j];
            std::vector<size_t> idx(n);
            for (size_t j = 0; j < n; j++) idx[j] = j;
            std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
                double ca = hdiag[a] * colsq[a], cb = hdiag[b] * colsq[b];
                if (cb < ca) return true;   // descending
                if (ca < cb) return false;
                return a < b;               // ties (and NaN) by ascending index
            });
            for (size_t t = 0; t < nskel * g; t++) {
                in_skel[idx[t]] = 1;
                perm.push_back((uint32_t)idx[t]);
            }
        }
    }
    std::vector<size_t> rest;
    for (size_t j = 0; j < n; j++)
        if (!in_skel[j]) rest.push_back(j);
    if (cfg->act_order) {
        std::sort(rest.begin(), rest.end(), [&](size_t a, size_t b) {
            if (hdiag[b] < hdiag[a]) return true;
            if (hdiag[a] < hdiag[b]) return false;
            return a < b;
        });
    }
    for (size_t j : rest) perm.push_back((uint32_t)j);
    *nskel_out = nskel;
}

// src/engine.rs:201-218 Prepared
struct Prepared {
    std::vector<uint32_t> perm;
    std::vector<float> h32;
    std::vector<float> u;
    double damp_val = 0.0;
};

// src/engine.rs:320-342
static int build_prepared(const float* h, size_t n, const std::vector<uint32_t>& perm, const cdclq_config* cfg,
                          Prepared& out) {
    std::vector<double> hp(n * n);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        size_t pi = perm[i];
        for (size_t j = 0; j < n; j++) hp[i * n + j] = (double)h[pi * n + perm[j]];
    }
    for (size_t i = 0; i < n; i++)
        if (hp[i * n + i] == 0.0) hp[i * n + i] = 1.0;
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) sum += hp[i * n + i];
    double mean_diag = sum / (double)n;
    double damp_val = cfg->damp * mean_diag;
    for (size_t i = 0; i < n; i++) hp[i * n + i] += damp_val;
    out.h32.resize(n * n);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n * n; i++) out.h32[i] = (float)hp[i];
    out.u.assign(n * n, 0.0f);
    int rc = upper_chol_of_inverse(hp, n, out.u.data());
    if (rc != CDCLQ_OK) return rc;
    out.perm = perm;
    out.damp_val = damp_val;
    return CDCLQ_OK;
}

struct ChunkStats {
    double loss_gptq = 0, loss_final = 0;
    size_t sb_total = 0, sb_refined = 0, updates = 0, passes = 0;
};

// src/engine.rs:366-674  phase 1 (blocked GPTQ, lazy updates) + phase 2 (conflict repair) on one row chunk.
static ChunkStats process_chunk(const float* wt, size_t rows, size_t n, size_t ng, size_t g, const float* u,
                                const float* h, const uint8_t* gbits, const cdclq_config* cfg, uint8_t* codes,
                                float* scales, float* zeros) {
    const size_t bsz = cfg->block;
    std::vector<float> w(wt, wt + rows * n);
    std::vector<float> wq(rows * n, 0.0f);
    std::vector<double> colloss(n, 0.0);
    const size_t bw = std::min(bsz, n);
    std::vector<float> w1(rows * bw, 0.0f), err1(rows * bw, 0.0f);
    std::vector<float> tmp(std::min(g, n), 0.0f);

    // ---- Phase 1 (src/engine.rs:397-473)
    size_t i1 = 0;
    while (i1 < n) {
        size_t i2 = std::min(i1 + bsz, n);
        size_t cnt = i2 - i1;
        for (size_t r = 0; r < rows; r++) std::memcpy(&w1[r * cnt], &w[r * n + i1], cnt * sizeof(float));
        for (size_t i = 0; i < cnt; i++) {
            size_t j = i1 + i;
            if (j % g == 0) {
                size_t gi = j / g;
                uint32_t bits = gbits[gi];
                size_t gend = std::min(j + g, n);
                for (size_t r = 0; r < rows; r++) {
                    for (size_t col = j, kk = 0; col < gend; col++, kk++)
                        tmp[kk] = (col < i2) ? w1[r * cnt + (col - i1)] : w[r * n + col];
                    float s, z;
                    find_params(tmp.data(), gend - j, 1, bits, cfg->mse_grid != 0, &s, &z);
                    scales[r * ng + gi] = s;
                    zeros[r * ng + gi] = z;
                }
            }
            size_t gi = j / g;
            float maxq = (float)((1u << gbits[gi]) - 1u);
            float inv_d = 1.0f / u[j * n + j];
            const float* urow = u + j * n + j + 1;
            size_t ulen = i2 - (j + 1);
            double cl = 0.0;
            for (size_t r = 0; r < rows; r++) {
                float wv = w1[r * cnt + i];
                uint8_t c;
                float dq;
                quant_code(wv, scales[r * ng + gi], zeros[r * ng + gi], maxq, &c, &dq);
                codes[r * n + j] = c;
                wq[r * n + j] = dq;
                float e = (wv - dq) * inv_d;
                cl += (double)(e * e);
                err1[r * cnt + i] = e;
                float* row = &w1[r * cnt + i + 1];
                for (size_t t = 0; t < ulen; t++) row[t] -= e * urow[t];
            }
            colloss[j] = cl;
        }
        if (i2 < n)
            gemm<float>(rows, cnt, n - i2, -1.0f, err1.data(), (ptrdiff_t)cnt, 1, u + i1 * n + i2, (ptrdiff_t)n, 1,
                        1.0f, w.data() + i2, (ptrdiff_t)n, 1, false);
        i1 = i2;
    }
    std::vector<float>().swap(w1);
    std::vector<float>().swap(err1);
    std::vector<float>().swap(w);

    ChunkStats st;
    double loss_gptq = 0.0;
    for (size_t j = 0; j < n; j++) loss_gptq += colloss[j];
    const size_t sbw = cfg->sub_block;
    const size_t n_sb = (n + sbw - 1) / sbw;
    double loss_delta = 0.0;
    size_t refined = 0, updates = 0, passes_done = 0;

    // ---- Phase 2 (src/engine.rs:488-671)
    const bool do_cd = cfg->refine_frac > 0.0 && cfg->cd_sweeps > 0 && cfg->passes > 0;
    const bool do_refit = cfg->refit_scales && g <= 1024;
    if (cfg->method == CDCLQ_METHOD_CDCL && (do_cd || do_refit)) {
        std::vector<size_t> sel;
        if (do_cd) {
            std::vector<std::pair<double, size_t>> sbl(n_sb);
            for (size_t s = 0; s < n_sb; s++) {
                size_t c0 = s * sbw, c1 = std::min((s + 1) * sbw, n);
                double acc = 0.0;
                for (size_t j = c0; j < c1; j++) acc += colloss[j];
                sbl[s] = {acc, s};
            }
            std::sort(sbl.begin(), sbl.end(), [](const std::pair<double, size_t>& a, const std::pair<double, size_t>& b) {
                if (b.first < a.first) return true;
                if (a.first < b.first) return false;
                return a.second < b.second;
            });
            double kf = std::ceil(cfg->refine_frac * (double)n_sb);
            size_t k = kf > 0.0 ? (size_t)kf : 0;
            k = std::max<size_t>(1, std::min(k, n_sb));
            for (size_t t = 0; t < k; t++) sel.push_back(sbl[t].second);
            std::sort(sel.begin(), sel.end());
            refined = sel.size();
        }
        std::vector<float> e(rows * n);
        for (size_t i = 0; i < rows * n; i++) e[i] = wt[i] - wq[i];
        const size_t gcap = std::min<size_t>(g, 1024);
        std::vector<float> gs(rows * std::max(sbw, gcap));
        std::vector<float> hss(sbw * sbw);
        std::vector<float> uu(do_refit ? rows * gcap : 0), hu(do_refit ? rows * gcap : 0),
            hcc(do_refit ? gcap * gcap : 0);

        // src/engine.rs:534-589
        auto refit_all = [&]() -> size_t {
            size_t changed = 0;
            for (size_t gi = 0; gi < ng; gi++) {
                size_t c0 = gi * g, c1 = std::min(c0 + g, n), wd = c1 - c0;
                gemm<float>(rows, n, wd, 1.0f, e.data(), (ptrdiff_t)n, 1, h + c0, (ptrdiff_t)n, 1, 0.0f, gs.data(),
                            (ptrdiff_t)wd, 1, false);
                for (size_t a = 0; a < wd; a++) std::memcpy(&hcc[a * wd], h + (c0 + a) * n + c0, wd * sizeof(float));
                for (size_t r = 0; r < rows; r++) {
                    float z = zeros[r * ng + gi];
                    for (size_t kk = 0; kk < wd; kk++) uu[r * wd + kk] = (float)codes[r * n + c0 + kk] - z;
                }
                gemm<float>(rows, wd, wd, 1.0f, uu.data(), (ptrdiff_t)wd, 1, hcc.data(), (ptrdiff_t)wd, 1, 0.0f,
                            hu.data(), (ptrdiff_t)wd, 1, false);
                for (size_t r = 0; r < rows; r++) {
                    const float* ur = &uu[r * wd];
                    float num = 0.0f, den = 0.0f;
                    for (size_t kk = 0; kk < wd; kk++) num += ur[kk] * gs[r * wd + kk];
                    for (size_t kk = 0; kk < wd; kk++) den += ur[kk] * hu[r * wd + kk];
                    if (!(den > 1e-30f)) continue;
                    float s_old = scales[r * ng + gi];
                    // f32::max(x, MIN) returns MIN for x < MIN and for NaN
                    float s_new = round_f16(s_old + num / den);
                    if (!(s_new >= F16_MIN_NORMAL)) s_new = F16_MIN_NORMAL;
                    float d = s_new - s_old;
                    double dl = (double)(-2.0f * d * num + d * d * den);
                    if (dl < 0.0) {
                        scales[r * ng + gi] = s_new;
                        for (size_t kk = 0; kk < wd; kk++) {
                            size_t j = c0 + kk;
                            float ndq = s_new * ur[kk];
                            e[r * n + j] += wq[r * n + j] - ndq;
                            wq[r * n + j] = ndq;
                        }
                        loss_delta += dl;
                        changed++;
                    }
                }
            }
            return changed;
        };

        double prev_delta = 0.0;
        size_t max_passes = std::max<size_t>(cfg->passes, 1);
        for (size_t pass = 0; pass < max_passes; pass++) {
            size_t pass_updates = 0;
            passes_done++;
            if (do_refit) pass_updates += refit_all();
            if (do_cd) {
                for (size_t s : sel) {
                    size_t c0 = s * sbw, c1 = std::min((s + 1) * sbw, n), wd = c1 - c0;
                    gemm<float>(rows, n, wd, 1.0f, e.data(), (ptrdiff_t)n, 1, h + c0, (ptrdiff_t)n, 1, 0.0f,
                                gs.data(), (ptrdiff_t)wd, 1, false);
                    for (size_t a = 0; a < wd; a++) std::memcpy(&hss[a * wd], h + (c0 + a) * n + c0, wd * sizeof(float));
                    for (size_t r = 0; r < rows; r++) {
                        float* gsr = &gs[r * wd];
                        for (size_t sw = 0; sw < cfg->cd_sweeps; sw++) {
                            bool changed = false;
                            for (size_t jj = 0; jj < wd; jj++) {
                                size_t j = c0 + jj;
                                size_t gi = j / g;
                                float maxq = (float)((1u << gbits[gi]) - 1u);
                                float sc = scales[r * ng + gi];
                                float z = zeros[r * ng + gi];
                                float hjj = hss[jj * wd + jj];
                                float cur = wq[r * n + j];
                                float target = cur + gsr[jj] / hjj;
                                float q = std::round(target / sc) + z;
                                if (q < 0.0f) q = 0.0f;
                                if (q > maxq) q = maxq;
                                float newdq = sc * (q - z);
                                uint8_t qc = (q == q) ? (uint8_t)q : (uint8_t)0;
                                if (qc != codes[r * n + j]) {
                                    float de = cur - newdq;
                                    loss_delta += (double)(2.0f * de * gsr[jj] + de * de * hjj);
                                    const float* hrow = &hss[jj * wd];
                                    for (size_t kk = 0; kk < wd; kk++) gsr[kk] += de * hrow[kk];
                                    wq[r * n + j] = newdq;
                                    codes[r * n + j] = qc;
                                    e[r * n + j] += de;
                                    pass_updates++;
                                    changed = true;
                                }
                            }
                            if (!changed) break;
                        }
                    }
                }
            }
            updates += pass_updates;
            double gain = prev_delta - loss_delta;
            prev_delta = loss_delta;
            if (pass_updates == 0 || gain < cfg->tol * (loss_gptq + loss_delta)) break;
        }
        if (do_refit) updates += refit_all();
    }
    st.loss_gptq = loss_gptq;
    st.loss_final = loss_gptq + loss_delta;
    st.sb_total = n_sb;
    st.sb_refined = refined;
    st.updates = updates;
    st.passes = passes_done;
    return st;
}

static size_t row_chunk(const cdclq_config* cfg, size_t d_out) {
    size_t rc;
    if (cfg->row_chunk > 0) {
        rc = cfg->row_chunk;
    } else {
        size_t nt = cfg->threads > 0 ? (size_t)cfg->threads : (size_t)omp_get_num_procs();
        rc = std::min<size_t>(std::max<size_t>((d_out + nt - 1) / nt, 32), 256);
    }
    rc = std::max<size_t>(std::min(rc, d_out), 1);
    return rc;
}

}  // namespace orc

// =========================================================================================================
// extern "C" surface (same argument meaning as include/cdclq.h, prefixed oracle_)
struct oracle_prep_cache {
    bool valid = false;
    std::string key;
    orc::Prepared prep;
};

extern "C" {

const char* oracle_last_error(void) { return orc::g_err.c_str(); }

void oracle_set_threads(int t) {
    if (t > 0) omp_set_num_threads(t);
}

int oracle_max_threads(void) { return omp_get_max_threads(); }

oracle_prep_cache* oracle_prep_cache_new(void) { return new oracle_prep_cache(); }
void oracle_prep_cache_free(oracle_prep_cache* c) { delete c; }

size_t oracle_effective_group(const cdclq_config* cfg, size_t n) { return orc::effective_group(cfg, n); }
int oracle_validate(const cdclq_config* cfg, size_t n) { return orc::validate(cfg, n); }
size_t oracle_row_chunk(const cdclq_config* cfg, size_t d_out) { return orc::row_chunk(cfg, d_out); }

float oracle_round_f16(float x) { return orc::round_f16(x); }

void oracle_round_f16_array(const float* x, size_t n, float* out) {
    for (size_t i = 0; i < n; i++) out[i] = orc::round_f16(x[i]);
}

void oracle_quant_code(float x, float scale, float zero, float maxq, uint8_t* c, float* dq) {
    orc::quant_code(x, scale, zero, maxq, c, dq);
}

void oracle_find_params(const float* vals, size_t rows, size_t len, uint32_t bits, int mse, float* s, float* z) {
    for (size_t r = 0; r < rows; r++) orc::find_params(vals + r * len, len, 1, bits, mse != 0, &s[r], &z[r]);
}

int oracle_cholesky_lower(double* a, size_t n) { return orc::cholesky_lower(a, n); }
void oracle_tri_inverse_lower(const double* l, size_t n, double* y) { orc::tri_inverse_lower(l, n, y); }
int oracle_upper_chol_of_inverse(const double* h, size_t n, float* u) {
    std::vector<double> hh(h, h + n * n);
    return orc::upper_chol_of_inverse(hh, n, u);
}
void oracle_gram_accumulate(const float* x, const float* y, size_t t, size_t n, double* h) {
    orc::gram_accumulate(x, y, t, n, h);
}
void oracle_sgemm(size_t m, size_t k, size_t n, float alpha, const float* a, ptrdiff_t rsa, ptrdiff_t csa,
                  const float* b, ptrdiff_t rsb, ptrdiff_t csb, float beta, float* c, ptrdiff_t rsc, ptrdiff_t csc) {
    orc::gemm<float>(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, true);
}
void oracle_dgemm(size_t m, size_t k, size_t n, double alpha, const double* a, ptrdiff_t rsa, ptrdiff_t csa,
                  const double* b, ptrdiff_t rsb, ptrdiff_t csb, double beta, double* c, ptrdiff_t rsc,
                  ptrdiff_t csc) {
    orc::gemm<double>(m, k, n, alpha, a, rsa, csa, b, rsb, csb, beta, c, rsc, csc, true);
}

// src/engine.rs:271-304 (exposed for the permutation tests)
int oracle_compute_perm(const float* h, const float* w, size_t d_out, size_t n, const cdclq_config* cfg,
                        uint32_t* perm_out, size_t* nskel_out) {
    int rc = orc::validate(cfg, n);
    if (rc) return rc;
    size_t g = orc::effective_group(cfg, n);
    std::vector<double> hdiag(n);
    for (size_t j = 0; j < n; j++) hdiag[j] = (double)h[j * n + j];
    std::vector<float> w0(w, w + d_out * n);
    for (size_t j = 0; j < n; j++)
        if (hdiag[j] == 0.0)
            for (size_t r = 0; r < d_out; r++) w0[r * n + j] = 0.0f;
    std::vector<uint32_t> perm;
    orc::compute_perm(hdiag, w0.data(), d_out, n, g, cfg, perm, nskel_out);
    std::memcpy(perm_out, perm.data(), n * sizeof(uint32_t));
    return CDCLQ_OK;
}

// src/engine.rs:320-342 (exposed so tests can compare U and h32 directly)
int oracle_build_prepared(const float* h, size_t n, const uint32_t* perm, const cdclq_config* cfg, float* u_out,
                          float* h32_out, double* damp_out) {
    orc::Prepared p;
    std::vector<uint32_t> pv(perm, perm + n);
    int rc = orc::build_prepared(h, n, pv, cfg, p);
    if (rc) return rc;
    std::memcpy(u_out, p.u.data(), n * n * sizeof(float));
    std::memcpy(h32_out, p.h32.data(), n * n * sizeof(float));
    *damp_out = p.damp_val;
    return CDCLQ_OK;
}

// src/engine.rs:690-799
int oracle_quantize_layer_ex(const float* w, size_t d_out, size_t d_in, const float* h, const float* m,
                             const char* hkey, const cdclq_config* cfg, oracle_prep_cache* cache, uint32_t* perm_out,
                             uint8_t* gbits_out, uint8_t* codes_out, float* scales_out, float* zeros_out,
                             cdclq_layer_stats* stats_out, uint32_t* chunk_passes_out) {
    using namespace orc;
    if (!w || !h || !cfg || !perm_out || !gbits_out || !codes_out || !scales_out || !zeros_out || !stats_out)
        return fail(CDCLQ_ERR_ARG, "null argument");
    const size_t n = d_in;
    if (n == 0 || d_out == 0) return fail(CDCLQ_ERR_ARG, "empty layer");
    int rc = validate(cfg, n);
    if (rc) return rc;
    const size_t g = effective_group(cfg, n);
    const size_t ng = (n + g - 1) / g;
    auto t0 = std::chrono::steady_clock::now();

    std::vector<double> hdiag(n);
    for (size_t j = 0; j < n; j++) hdiag[j] = (double)h[j * n + j];
    std::vector<float> w0(w, w + d_out * n);
    for (size_t j = 0; j < n; j++)
        if (hdiag[j] == 0.0)
            for (size_t r = 0; r < d_out; r++) w0[r * n + j] = 0.0f;
    std::vector<uint32_t> perm;
    size_t nskel = 0;
    compute_perm(hdiag, w0.data(), d_out, n, g, cfg, perm, &nskel);

    oracle_prep_cache local;
    oracle_prep_cache* pc = cache ? cache : &local;
    std::string key = hkey ? hkey : "";
    bool reuse = pc->valid && pc->key == key && pc->prep.perm == perm;
    if (!reuse) {
        pc->valid = false;
        pc->prep = Prepared();
        rc = build_prepared(h, n, perm, cfg, pc->prep);
        if (rc) return rc;
        pc->key = key;
        pc->valid = true;
    }
    const Prepared& prep = pc->prep;

    std::vector<float> wp(d_out * n);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < d_out; r++)
        for (size_t j = 0; j < n; j++) wp[r * n + j] = w0[r * n + prep.perm[j]];
    std::vector<float>().swap(w0);

    if (m) {  // asymmetric target, src/engine.rs:737-755
        std::vector<float> mp(n * n);
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < n; i++) {
            size_t pi = prep.perm[i];
            for (size_t j = 0; j < n; j++) mp[i * n + j] = m[pi * n + prep.perm[j]];
            mp[i * n + i] += (float)prep.damp_val;
        }
        std::vector<float> t1(d_out * n), t2(d_out * n);
        gemm<float>(d_out, n, n, 1.0f, wp.data(), (ptrdiff_t)n, 1, mp.data(), (ptrdiff_t)n, 1, 0.0f, t1.data(),
                    (ptrdiff_t)n, 1, true);
        gemm<float>(d_out, n, n, 1.0f, t1.data(), (ptrdiff_t)n, 1, prep.u.data(), 1, (ptrdiff_t)n, 0.0f, t2.data(),
                    (ptrdiff_t)n, 1, true);
        gemm<float>(d_out, n, n, 1.0f, t2.data(), (ptrdiff_t)n, 1, prep.u.data(), (ptrdiff_t)n, 1, 0.0f, wp.data(),
                    (ptrdiff_t)n, 1, true);
    }
    double secs_prepare = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

    std::vector<uint8_t> gbits(ng);
    for (size_t gi = 0; gi < ng; gi++) gbits[gi] = (uint8_t)(gi < nskel ? cfg->skeleton_bits : cfg->bits);

    const size_t rc_rows = row_chunk(cfg, d_out);
    const size_t nchunks = (d_out + rc_rows - 1) / rc_rows;
    std::vector<ChunkStats> stats(nchunks);
    auto t1 = std::chrono::steady_clock::now();
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t ci = 0; ci < nchunks; ci++) {
        size_t r0 = ci * rc_rows;
        size_t rows = std::min(rc_rows, d_out - r0);
        stats[ci] = process_chunk(wp.data() + r0 * n, rows, n, ng, g, prep.u.data(), prep.h32.data(), gbits.data(), cfg,
                                  codes_out + r0 * n, scales_out + r0 * ng, zeros_out + r0 * ng);
    }
    double secs_quant = std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count();

    std::memcpy(perm_out, prep.perm.data(), n * sizeof(uint32_t));
    std::memcpy(gbits_out, gbits.data(), ng);
    cdclq_layer_stats st;
    std::memset(&st, 0, sizeof st);
    for (size_t ci = 0; ci < nchunks; ci++) {
        st.loss_gptq += stats[ci].loss_gptq;
        st.loss_final += stats[ci].loss_final;
        st.subblocks_total += stats[ci].sb_total;
        st.subblocks_refined += stats[ci].sb_refined;
        st.code_updates += stats[ci].updates;
        st.passes_max = std::max<uint64_t>(st.passes_max, stats[ci].passes);
        if (chunk_passes_out) chunk_passes_out[ci] = (uint32_t)stats[ci].passes;
    }
    st.skeleton_groups = nskel;
    // QLayer::bits_codes / bits_total (src/quant.rs:239-250)
    size_t rb = 0;
    for (size_t j = 0; j < n; j++) rb += gbits[j / g];
    st.bits_codes = (double)rb / (double)n;
    st.bits_total = st.bits_codes + 24.0 / (double)g;
    st.secs_prepare = secs_prepare;
    st.secs_quant = secs_quant;
    *stats_out = st;
    return CDCLQ_OK;
}

int oracle_quantize_layer(const float* w, size_t d_out, size_t d_in, const float* h, const float* m, const char* hkey,
                          const cdclq_config* cfg, oracle_prep_cache* cache, uint32_t* perm_out, uint8_t* gbits_out,
                          uint8_t* codes_out, float* scales_out, float* zeros_out, cdclq_layer_stats* stats_out) {
    return oracle_quantize_layer_ex(w, d_out, d_in, h, m, hkey, cfg, cache, perm_out, gbits_out, codes_out,
                                    scales_out, zeros_out, stats_out, nullptr);
}

// src/engine.rs:808-815
double oracle_proxy_loss(const float* w_t, const float* w_hat, size_t rows, size_t n, const float* h) {
    std::vector<float> e(rows * n), eh(rows * n);
    for (size_t i = 0; i < rows * n; i++) e[i] = w_t[i] - w_hat[i];
    orc::gemm<float>(rows, n, n, 1.0f, e.data(), (ptrdiff_t)n, 1, h, (ptrdiff_t)n, 1, 0.0f, eh.data(), (ptrdiff_t)n, 1,
                     true);
    double s = 0.0;
    for (size_t i = 0; i < rows * n; i++) s += (double)e[i] * (double)eh[i];
    return s;
}

// src/engine.rs:822-838
void oracle_rtn_layer(const float* w, size_t d_out, size_t n, const cdclq_config* cfg, float* out) {
    size_t g = orc::effective_group(cfg, n);
    float maxq = (float)((1u << cfg->bits) - 1u);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < d_out; r++) {
        const float* src = w + r * n;
        size_t j = 0;
        while (j < n) {
            size_t e = std::min(j + g, n);
            float s, z;
            orc::find_params(src + j, e - j, 1, cfg->bits, cfg->mse_grid != 0, &s, &z);
            for (size_t k = j; k < e; k++) {
                uint8_t c;
                orc::quant_code(src[k], s, z, maxq, &c, &out[r * n + k]);
            }
            j = e;
        }
    }
}

// src/quant.rs:98-151
size_t oracle_row_bytes(size_t n, size_t g, const uint8_t* gbits) {
    size_t bits = 0;
    for (size_t j = 0; j < n; j++) bits += gbits[j / g];
    return (bits + 7) / 8;
}

void oracle_pack_row(const uint8_t* codes, size_t n, size_t g, const uint8_t* gbits, uint8_t* out) {
    uint64_t acc = 0;
    uint32_t nacc = 0;
    size_t o = 0;
    for (size_t j = 0; j < n; j++) {
        uint32_t b = gbits[j / g];
        acc |= (uint64_t)codes[j] << nacc;
        nacc += b;
        while (nacc >= 8) {
            out[o++] = (uint8_t)(acc & 0xff);
            acc >>= 8;
            nacc -= 8;
        }
    }
    if (nacc > 0) out[o] = (uint8_t)(acc & 0xff);
}

void oracle_unpack_row(const uint8_t* data, size_t n, size_t g, const uint8_t* gbits, uint8_t* codes) {
    uint64_t acc = 0;
    uint32_t nacc = 0;
    size_t o = 0;
    for (size_t j = 0; j < n; j++) {
        uint32_t b = gbits[j / g];
        while (nacc < b) {
            acc |= (uint64_t)data[o++] << nacc;
            nacc += 8;
        }
        codes[j] = (uint8_t)(acc & ((1ull << b) - 1));
        acc >>= b;
        nacc -= b;
    }
}

// src/quant.rs:189-202
void oracle_dequantize(size_t d_out, size_t n, size_t g, const uint32_t* perm, const uint8_t* codes,
                       const float* scales, const float* zeros, float* out) {
    size_t ng = (n + g - 1) / g;
    for (size_t r = 0; r < d_out; r++)
        for (size_t j = 0; j < n; j++) {
            size_t gi = j / g;
            out[r * n + perm[j]] = scales[r * ng + gi] * ((float)codes[r * n + j] - zeros[r * ng + gi]);
        }
}

// src/rng.rs (for seeded synthetic inputs)
void oracle_rng_normal(uint64_t seed, size_t count, float scale, float* out) {
    orc::Rng r(seed);
    for (size_t i = 0; i < count; i++) out[i] = r.normal() * scale;
}

// src/engine.rs:850-869 `problem()`: correlated activations (rank n/4), log-normal channel scales, noise 0.3,
// W ~ 0.05 N(0,1); H = gram_accumulate(X, X) narrowed to f32.
void oracle_problem(size_t d_out, size_t n, size_t tokens, uint64_t seed, float* w_out, float* h_out) {
    orc::Rng r(seed);
    size_t rank = n / 4;
    std::vector<float> a(rank * n), z(tokens * rank), x(tokens * n);
    float sq = std::sqrt((float)rank);
    for (auto& v : a) v = r.normal() / sq;
    for (auto& v : z) v = r.normal();
    orc::gemm<float>(tokens, rank, n, 1.0f, z.data(), (ptrdiff_t)rank, 1, a.data(), (ptrdiff_t)n, 1, 0.0f, x.data(),
                     (ptrdiff_t)n, 1, false);
    std::vector<float> s(n);
    for (auto& v : s) v = std::exp(0.5f * r.normal());
    for (size_t t = 0; t < tokens; t++)
        for (size_t j = 0; j < n; j++) x[t * n + j] = (x[t * n + j] + 0.3f * r.normal()) * s[j];
    for (size_t i = 0; i < d_out * n; i++) w_out[i] = r.normal() * 0.05f;
    std::vector<double> h(n * n, 0.0);
    orc::gram_accumulate(x.data(), x.data(), tokens, n, h.data());
    for (size_t i = 0; i < n * n; i++) h_out[i] = (float)h[i];
}

}  // extern "C"
