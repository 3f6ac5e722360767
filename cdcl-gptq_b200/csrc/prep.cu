// prep.cu - Hessian preparation and the f64 factorisation H^-1 = U^T U (src/engine.rs:320-342,
// src/linalg.rs:200-375), batched over the distinct layer inputs of one width.
//
// Every element goes through exactly the reference's sequence of roundings:
//   * permute + dead-diagonal patch + relative damping in f64, the mean of the diagonal summed in order;
//   * the flip (h.reverse()) is folded into the write of the permuted matrix (hr[n-1-i][n-1-j] = hp[i][j]);
//   * blocked right-looking Cholesky with NB = 96: the diagonal block and the panel solve are scalar code in
//     the reference (mul then sub, no FMA) and stay so here; the left-looking dot products of the reference
//     are applied in the same per-element order (t ascending) as right-looking updates, which exposes the
//     parallelism without changing a single rounding;
//   * the trailing update is a GEMM (the unpinned `matrixmultiply` call) in the fixed order: acc = sum_t
//     fma(.), then a -= acc;
//   * the triangular inverse: explicit 96-wide diagonal-block inverses (scalar, `acc += l*y`), then
//     T = L[s:e, :s] Y[:s, :s] and Y[s:e, :s] = -Yii T, both GEMMs in the fixed order.  Terms that multiply
//     an exact zero of a triangular operand are skipped: the accumulator is never -0, so a zero product is
//     an exact no-op;
//   * U[i][j] = (f32) Y[n-1-i][n-1-j] for j >= i.
// FP64 runs on the SIMT DFMA pipe: on B200 its peak equals the FP64 tensor-core (DMMA) peak, and DMMA would
// not reproduce the fixed summation order.
#include <cmath>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace cdclq {

constexpr int NB = 96;  // src/linalg.rs:202 and :285

// ---------------------------------------------------------------------------------------------------------
// src/engine.rs:321-338: patched diagonal, its mean in order, the damping value
__global__ void prep_diag_kernel(const PrepItem* __restrict__ items, int n) {
    const PrepItem it = items[blockIdx.y];
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t p = it.perm[i];
    double v = (double)it.h[(int64_t)p * n + p];
    it.dg[i] = (v == 0.0) ? 1.0 : v;
}

__global__ void prep_mean_kernel(const PrepItem* __restrict__ items, int n, double damp) {
    const PrepItem it = items[blockIdx.x];
    if (threadIdx.x != 0) return;
    double s = 0.0;
    for (int i = 0; i < n; i++) s = __dadd_rn(s, it.dg[i]);
    double mean = __ddiv_rn(s, (double)n);
    *it.damp_val = __dmul_rn(damp, mean);
    it.status->err = 0;
    it.status->pivot = -1;
    it.status->value = 0.0;
}

// hp[a][b] = (f64) h[perm a][perm b], diagonal patched and damped; h32 = (f32) hp; hr = flip(hp).  Either
// output may be absent (null): h32 alone when the factor U comes from elsewhere, hr alone when only U is wanted.
__global__ void prep_fill_kernel(const PrepItem* __restrict__ items, int n) {
    const PrepItem it = items[blockIdx.z];
    int a = blockIdx.y;
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n) return;
    double v;
    if (a == b)
        v = __dadd_rn(it.dg[a], *it.damp_val);
    else
        v = (double)it.h[(int64_t)it.perm[a] * n + it.perm[b]];
    if (it.h32) it.h32[(int64_t)a * n + b] = (float)v;
    if (it.hr) it.hr[(int64_t)(n - 1 - a) * n + (n - 1 - b)] = v;
}

int launch_prepare(const PrepItem* items_dev, int nitems, int n, double damp, cudaStream_t st) {
    if (nitems == 0) return 0;
    dim3 g1((n + 255) / 256, nitems);
    CDCLQ_LAUNCH(prep_diag_kernel, g1, 256, 0, st, items_dev, n);
    CDCLQ_LAUNCH(prep_mean_kernel, nitems, 32, 0, st, items_dev, n, damp);
    dim3 g2((n + 255) / 256, n, nitems);
    CDCLQ_LAUNCH(prep_fill_kernel, g2, 256, 0, st, items_dev, n);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "prepare kernels launch");
}

// ---------------------------------------------------------------------------------------------------------
// Cholesky step 1 (src/linalg.rs:209-229): the kb x kb diagonal block, one CTA per matrix.
// Right-looking form of the reference's left-looking loops: after column t is final, every later element
// (i, c) of the block, c <= i, receives its `- a[i][t]*a[c][t]` term - the same terms in the same order.
struct CholArgs {
    double* a;
    FactorStatus* status;
};

// The block lives in shared memory (row stride NB + 1: the column reads of a warp fall in distinct banks); per
// column j one thread takes the square root of the diagonal (after every earlier term was subtracted) and
// checks the pivot, the rows below divide their column-j entry, then a 16 x 16 thread grid applies the
// column's `- a[i][j]*a[c][j]` term to every (i, c) with j < c <= i (mul then sub, as the reference's scalar
// code).  Three barriers per column and no work outside the triangle.
constexpr int CHOL_LD = NB + 1;
constexpr size_t CHOL_DIAG_SMEM = (size_t)NB * CHOL_LD * sizeof(double);

__global__ void __launch_bounds__(256) chol_diag_kernel(const CholArgs* __restrict__ args, int n, int k, int kb) {
    extern __shared__ double blk[];  // [NB][CHOL_LD], lower triangle of the diagonal block
    __shared__ int bad;
    const CholArgs ar = args[blockIdx.x];
    if (ar.status->err) return;
    double* A = ar.a;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    for (int idx = tid; idx < kb * kb; idx += blockDim.x) {
        const int i = idx / kb, c = idx - i * kb;
        if (c <= i) blk[i * CHOL_LD + c] = A[(int64_t)(k + i) * n + (k + c)];
    }
    if (tid == 0) bad = 0;
    __syncthreads();
    for (int j = 0; j < kb; j++) {
        if (tid == 0) {
            const double d = blk[j * CHOL_LD + j];
            if (!(d > 0.0) || !isfinite(d)) {
                bad = 1;
                ar.status->err = 1;
                ar.status->pivot = k + j;
                ar.status->value = d;
            } else {
                blk[j * CHOL_LD + j] = __dsqrt_rn(d);
            }
        }
        __syncthreads();
        if (bad) return;
        const double dj = blk[j * CHOL_LD + j];
        for (int i = j + 1 + tid; i < kb; i += blockDim.x) blk[i * CHOL_LD + j] = __ddiv_rn(blk[i * CHOL_LD + j], dj);
        __syncthreads();
        for (int i = j + 1 + ty; i < kb; i += 16) {
            const double aij = blk[i * CHOL_LD + j];
            for (int c = j + 1 + tx; c <= i; c += 16)
                blk[i * CHOL_LD + c] = __dsub_rn(blk[i * CHOL_LD + c], __dmul_rn(aij, blk[c * CHOL_LD + j]));
        }
        __syncthreads();
    }
    for (int idx = tid; idx < kb * kb; idx += blockDim.x) {
        const int i = idx / kb, c = idx - i * kb;
        if (c <= i) A[(int64_t)(k + i) * n + (k + c)] = blk[i * CHOL_LD + c];
    }
}

// Cholesky step 2 (src/linalg.rs:232-241): panel rows i >= kend solve X L_kk^T = A_panel, one thread per row
// with the row in registers: row[j] = (row[j] - sum_t row[t] L[j][t]) / L[j][j], the terms subtracted in
// increasing t as soon as row[t] is final (the reference's per-element order).  The diagonal block is read
// transposed from shared memory (every thread reads the same element: broadcasts); columns past kb are
// identity padding.
__global__ void __launch_bounds__(128) chol_panel_kernel(const CholArgs* __restrict__ args, int n, int k, int kb) {
    extern __shared__ double lt[];  // [NB][NB]: lt[j][c] = L[k+c][k+j] for j <= c < kb
    const CholArgs ar = args[blockIdx.y];
    if (ar.status->err) return;
    double* A = ar.a;
    const int kend = k + kb;
    for (int idx = threadIdx.x; idx < NB * NB; idx += blockDim.x) {
        int j = idx / NB, c = idx - j * NB;
        double v;
        if (c < kb && j < kb)
            v = (j <= c) ? A[(int64_t)(k + c) * n + (k + j)] : 0.0;
        else
            v = (c == j) ? 1.0 : 0.0;
        lt[idx] = v;
    }
    __syncthreads();
    const int i = kend + blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    double* row = A + (int64_t)i * n + k;
    double x[NB];
#pragma unroll
    for (int c = 0; c < NB; c++) x[c] = (c < kb) ? row[c] : 0.0;
#pragma unroll
    for (int j = 0; j < NB; j++) {
        x[j] = __ddiv_rn(x[j], lt[j * NB + j]);
#pragma unroll
        for (int c = 0; c < NB; c++)  // constant trip count: unrolls into registers once j is known
            if (c > j) x[c] = __dsub_rn(x[c], __dmul_rn(x[j], lt[j * NB + c]));
    }
#pragma unroll
    for (int c = 0; c < NB; c++)
        if (c < kb) row[c] = x[c];
}

// ---------------------------------------------------------------------------------------------------------
// f64 GEMM tile core: CTA tile (16*TM) x 64 outputs, 256 threads; thread (ty, tx) owns rows ty + 16*i and
// columns tx + 16*j (strided, so shared-memory reads are broadcasts (A) or consecutive doubles (B)).  K is
// staged 16 at a time with a register prefetch of the next stage.  Operands come through callables
// fa(r, k) / fb(k, c) (bounds handled there); B_ALONG_K says which index of B is contiguous in memory so the
// fetch is coalesced.  Each accumulator receives its products in increasing k (the fixed order).
constexpr int DKT = 16;
constexpr int DBLD = 65;  // odd strides: conflict-free transposed stores
template <int TM>
struct DTile {
    static constexpr int ROWS = 16 * TM;
    static constexpr int ALD = ROWS + 1;
    static constexpr int APER = ROWS * DKT / 256;  // A elements fetched per thread per stage
    static constexpr int BPER = 64 * DKT / 256;    // 4
    static constexpr int SMEM_DOUBLES = 2 * DKT * ALD + 2 * DKT * DBLD;
};

template <int TM, bool B_ALONG_K, class FA, class FB>
__device__ __forceinline__ void dgemm_tile(double (&acc)[TM][4], FA fa, FB fb, int kbeg, int kend, double* smem) {
    using T = DTile<TM>;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    // stage buffers: A at smem + buf * DKT*ALD, B after both A buffers (no pointer arrays: they would live in
    // local memory when indexed by the runtime buffer number)
    double* const As0 = smem;
    double* const Bs0 = smem + 2 * DKT * T::ALD;
    double ra[T::APER], rb[T::BPER];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int m = 0; m < T::APER; m++) {
            int idx = tid + 256 * m, r = idx / DKT, k = k0 + (idx % DKT);
            ra[m] = (k < kend) ? fa(r, k) : 0.0;
        }
#pragma unroll
        for (int m = 0; m < T::BPER; m++) {
            int idx = tid + 256 * m, c, k;
            if (B_ALONG_K) {
                c = idx / DKT;
                k = k0 + (idx % DKT);
            } else {
                k = k0 + idx / 64;
                c = idx % 64;
            }
            rb[m] = (k < kend) ? fb(k, c) : 0.0;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int m = 0; m < T::APER; m++) {
            int idx = tid + 256 * m, r = idx / DKT, kk = idx % DKT;
            As0[buf * DKT * T::ALD + kk * T::ALD + r] = ra[m];
        }
#pragma unroll
        for (int m = 0; m < T::BPER; m++) {
            int idx = tid + 256 * m, c, kk;
            if (B_ALONG_K) {
                c = idx / DKT;
                kk = idx % DKT;
            } else {
                kk = idx / 64;
                c = idx % 64;
            }
            Bs0[buf * DKT * DBLD + kk * DBLD + c] = rb[m];
        }
    };
    if (kbeg >= kend) return;
    fetch(kbeg);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += DKT) {
        const bool more = k0 + DKT < kend;
        if (more) fetch(k0 + DKT);
        const double* A = As0 + buf * DKT * T::ALD;
        const double* Bq = Bs0 + buf * DKT * DBLD;
#pragma unroll
        for (int kk = 0; kk < DKT; kk++) {
            double av[TM], bv[4];
#pragma unroll
            for (int i = 0; i < TM; i++) av[i] = A[kk * T::ALD + ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; j++) bv[j] = Bq[kk * DBLD + tx + 16 * j];
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fma_rn(av[i], bv[j], acc[i][j]);
        }
        if (more) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
}

// f64 GEMM tile core with paired fragments: CTA tile (32*RP) x 64 outputs, 256 threads as 16 (ty) x 16 (tx);
// thread (ty, tx) owns the row pairs 2ty + 32i + {0, 1} (i < RP) and the column pairs 2tx + 32j + {0, 1}
// (j < 2), so each k-step reads its fragments with 16-byte shared-memory loads: RP + 2 loads (RP + 4
// wavefronts) per 8 RP DFMA, half the shared-memory traffic per DFMA of dgemm_tile, whose 4-row fragments
// need a load per value.  Staging as in dgemm_tile (register prefetch of the next K stage, 16 at a time);
// each accumulator receives its products in increasing k (the fixed order).  Dynamic shared memory:
// DTile2<RP>::SMEM_BYTES.
template <int RP>
struct DTile2 {
    static constexpr int ROWS = 32 * RP;
    static constexpr int ALD = ROWS + 2;  // even: 16-byte aligned pairs
    static constexpr int BLD = 64 + 2;
    static constexpr int APER = ROWS * DKT / 256;
    static constexpr int BPER = 64 * DKT / 256;
    static constexpr int STAGE = DKT * ALD + DKT * BLD;  // doubles
    static constexpr size_t SMEM_BYTES = 2 * (size_t)STAGE * sizeof(double);
    static __device__ __forceinline__ int row(int ty, int i) { return 2 * ty + 32 * (i >> 1) + (i & 1); }
    static __device__ __forceinline__ int col(int tx, int j) { return 2 * tx + 32 * (j >> 1) + (j & 1); }
};

template <int RP, bool B_ALONG_K, class FA, class FB>
__device__ __forceinline__ void dgemm_tile2(double (&acc)[2 * RP][4], FA fa, FB fb, int kbeg, int kend,
                                            double* smem) {
    using T = DTile2<RP>;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    double ra[T::APER], rb[T::BPER];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int m = 0; m < T::APER; m++) {
            int idx = tid + 256 * m, r = idx / DKT, k = k0 + (idx % DKT);
            ra[m] = (k < kend) ? fa(r, k) : 0.0;
        }
#pragma unroll
        for (int m = 0; m < T::BPER; m++) {
            int idx = tid + 256 * m, c, k;
            if (B_ALONG_K) {
                c = idx / DKT;
                k = k0 + (idx % DKT);
            } else {
                k = k0 + idx / 64;
                c = idx % 64;
            }
            rb[m] = (k < kend) ? fb(k, c) : 0.0;
        }
    };
    auto store = [&](int buf) {
        double* As = smem + buf * T::STAGE;
        double* Bs = As + DKT * T::ALD;
#pragma unroll
        for (int m = 0; m < T::APER; m++) {
            int idx = tid + 256 * m, r = idx / DKT, kk = idx % DKT;
            As[kk * T::ALD + r] = ra[m];
        }
#pragma unroll
        for (int m = 0; m < T::BPER; m++) {
            int idx = tid + 256 * m, c, kk;
            if (B_ALONG_K) {
                c = idx / DKT;
                kk = idx % DKT;
            } else {
                kk = idx / 64;
                c = idx % 64;
            }
            Bs[kk * T::BLD + c] = rb[m];
        }
    };
    if (kbeg >= kend) return;
    fetch(kbeg);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += DKT) {
        const bool more = k0 + DKT < kend;
        if (more) fetch(k0 + DKT);
        const double* A = smem + buf * T::STAGE;
        const double* Bq = A + DKT * T::ALD;
#pragma unroll
        for (int kk = 0; kk < DKT; kk++) {
            double av[2 * RP], bv[4];
#pragma unroll
            for (int i = 0; i < RP; i++) {
                const double2 a = *reinterpret_cast<const double2*>(A + kk * T::ALD + 2 * ty + 32 * i);
                av[2 * i] = a.x;
                av[2 * i + 1] = a.y;
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const double2 b = *reinterpret_cast<const double2*>(Bq + kk * T::BLD + 2 * tx + 32 * j);
                bv[2 * j] = b.x;
                bv[2 * j + 1] = b.y;
            }
#pragma unroll
            for (int i = 0; i < 2 * RP; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fma_rn(av[i], bv[j], acc[i][j]);
        }
        if (more) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
}

// Cholesky step 3 (src/linalg.rs:242-271): A22[i][c] -= sum_t P[i][t] P[c][t] for kend <= c <= i < n, in
// tiles of 128 rows x 64 columns holding some c <= i (the reference also updates some upper-triangle garbage
// that is never read).  Zero-padded k beyond kb contributes exact zeros; each accumulator runs t = 0..kb-1 in
// order.  Tile index -> (row block ti, column tile tc): row block ti has min(T64, 2 ti + 2) column tiles.
__host__ __device__ inline long long chol_trail_tiles(int rows) {
    const long long t64 = (rows + 63) / 64, t128 = (rows + 127) / 128, b = t64 / 2;
    return b * (b + 1) + (t128 - b) * t64;
}

__global__ void __launch_bounds__(256, 2) chol_trail_kernel(const CholArgs* __restrict__ args, int n, int k, int kb) {
    extern __shared__ __align__(16) double dsm[];
    const CholArgs ar = args[blockIdx.y];
    if (ar.status->err) return;
    double* A = ar.a;
    const int kend = k + kb;
    const int t64 = (n - kend + 63) / 64, b = t64 / 2;
    const long long x = blockIdx.x, cb = (long long)b * (b + 1);
    int ti, tc;
    if (x < cb) {  // row blocks ti < b: 2 ti + 2 column tiles each, ti (ti + 1) tiles before ti
        ti = (int)((sqrt(4.0 * (double)x + 1.0) - 1.0) * 0.5);
        while ((long long)(ti + 1) * (ti + 2) <= x) ti++;
        while ((long long)ti * (ti + 1) > x) ti--;
        tc = (int)(x - (long long)ti * (ti + 1));
    } else {
        ti = b + (int)((x - cb) / t64);
        tc = (int)((x - cb) % t64);
    }
    const int r0 = kend + ti * 128, c0 = kend + tc * 64;
    using T = DTile2<4>;
    double acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
    auto fa = [&](int r, int t) -> double {
        int i = r0 + r;
        return (i < n) ? A[(int64_t)i * n + k + t] : 0.0;
    };
    auto fb = [&](int t, int c) -> double {
        int cc = c0 + c;
        return (cc < n) ? A[(int64_t)cc * n + k + t] : 0.0;
    };
    dgemm_tile2<4, true>(acc, fa, fb, 0, kb, dsm);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
#pragma unroll
    for (int a = 0; a < 8; a++) {
        int i = r0 + T::row(ty, a);
        if (i >= n) continue;
#pragma unroll
        for (int bb = 0; bb < 4; bb++) {
            int c = c0 + T::col(tx, bb);
            if (c <= i) {
                double* p = A + (int64_t)i * n + c;
                *p = __dsub_rn(*p, acc[a][bb]);
            }
        }
    }
}

static int run_cholesky(const CholArgs* args_dev, int nitems, int n, cudaStream_t st) {
    cudaFuncSetAttribute(chol_trail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DTile2<4>::SMEM_BYTES);
    cudaFuncSetAttribute(chol_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CHOL_DIAG_SMEM);
    for (int k = 0; k < n; k += NB) {
        int kb = min(NB, n - k);
        int kend = k + kb;
        CDCLQ_LAUNCH(chol_diag_kernel, nitems, 256, CHOL_DIAG_SMEM, st, args_dev, n, k, kb);
        if (kend < n) {
            int rows_below = n - kend;
            size_t smem2 = (size_t)NB * NB * sizeof(double);
            cudaFuncSetAttribute(chol_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
            dim3 gp((rows_below + 127) / 128, nitems);
            CDCLQ_LAUNCH(chol_panel_kernel, gp, 128, smem2, st, args_dev, n, k, kb);
            dim3 gt((unsigned)chol_trail_tiles(rows_below), nitems);
            CDCLQ_LAUNCH(chol_trail_kernel, gt, 256, DTile2<4>::SMEM_BYTES, st, args_dev, n, k, kb);
        }
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "cholesky kernels launch");
}

// ---------------------------------------------------------------------------------------------------------
// Triangular inverse step 1 (src/linalg.rs:292-306): explicit inverse of the w x w diagonal block.
// Thread c computes column c by forward substitution: y_c = 1/l_cc; y_t = -acc_t / l_tt with
// acc_t = sum_{t'=c}^{t-1} l[t][t'] y_t' accumulated as `acc += l*y` from 0.0 in increasing t'.
struct TriArgs {
    const double* l;
    double* y;
    double* t;
    FactorStatus* status;
};

__global__ void __launch_bounds__(128) tri_diag_kernel(const TriArgs* __restrict__ args, int n, int s, int w) {
    extern __shared__ double Ls[];  // [NB][NB] lower block, identity past w
    const TriArgs ar = args[blockIdx.x];
    if (ar.status->err) return;
    for (int idx = threadIdx.x; idx < NB * NB; idx += blockDim.x) {
        int i = idx / NB, c = idx - i * NB;
        double v;
        if (i < w && c < w)
            v = (c <= i) ? ar.l[(int64_t)(s + i) * n + (s + c)] : 0.0;
        else
            v = (i == c) ? 1.0 : 0.0;
        Ls[idx] = v;
    }
    __syncthreads();
    const int c = threadIdx.x;  // column of the block inverse owned by this thread
    if (c >= w) return;
    double acc[NB];
#pragma unroll
    for (int i = 0; i < NB; i++) acc[i] = 0.0;
#pragma unroll
    for (int t = 0; t < NB; t++) {
        if (t >= c) {
            const double yt = (t == c) ? __ddiv_rn(1.0, Ls[t * NB + t]) : __ddiv_rn(-acc[t], Ls[t * NB + t]);
            if (t < w) ar.y[(int64_t)(s + t) * n + (s + c)] = yt;
#pragma unroll
            for (int i = 0; i < NB; i++)  // constant trip count: unrolls into registers once t is known
                if (i > t) acc[i] = __dadd_rn(acc[i], __dmul_rn(Ls[i * NB + t], yt));
        }
    }
}

// Triangular inverse step 2 (src/linalg.rs:307-325): T[i][j] = sum_k L[s+i][k] Y[k][j], k in [0, s).
// Y is lower triangular: for the column tile starting at j0 every k < j0 multiplies an exact zero, so the
// accumulation starts at k = j0.  One CTA covers all w <= 96 rows of the block and 64 columns (the j0 = 0
// tile's chain of s terms sets a step's duration when one matrix is factorised alone; splitting the rows over
// three 32-row CTAs measured slower, the smaller tile costing more than the shorter chain saved).
__global__ void __launch_bounds__(256, 2) tri_gemm1_kernel(const TriArgs* __restrict__ args, int n, int s, int w) {
    extern __shared__ __align__(16) double dsm[];
    const TriArgs ar = args[blockIdx.y];
    if (ar.status->err) return;
    const int j0 = blockIdx.x * 64;
    double acc[6][4];
#pragma unroll
    for (int i = 0; i < 6; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
    const double* L = ar.l;
    const double* Y = ar.y;
    auto fa = [&](int r, int k) -> double { return (r < w) ? L[(int64_t)(s + r) * n + k] : 0.0; };
    auto fb = [&](int k, int c) -> double {
        int j = j0 + c;
        return (j < s) ? Y[(int64_t)k * n + j] : 0.0;
    };
    dgemm_tile2<3, false>(acc, fa, fb, j0, s, dsm);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
#pragma unroll
    for (int a = 0; a < 6; a++) {
        int i = DTile2<3>::row(ty, a);
        if (i >= w) continue;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            int j = j0 + DTile2<3>::col(tx, b);
            if (j < s) ar.t[(int64_t)i * n + j] = acc[a][b];
        }
    }
}

// Triangular inverse step 3 (src/linalg.rs:326-341): Y[s+i][j] = -sum_k Yii[i][k] T[k][j], k in [0, w);
// Yii is lower triangular, so the k > i terms are exact zeros.
__global__ void __launch_bounds__(256) tri_gemm2_kernel(const TriArgs* __restrict__ args, int n, int s, int w) {
    __shared__ __align__(16) double smem[DTile<6>::SMEM_DOUBLES];
    const TriArgs ar = args[blockIdx.y];
    if (ar.status->err) return;
    const int j0 = blockIdx.x * 64;
    double acc[6][4];
#pragma unroll
    for (int i = 0; i < 6; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;
    double* Y = ar.y;
    const double* T = ar.t;
    auto fa = [&](int r, int k) -> double {
        return (r < w && k <= r) ? Y[(int64_t)(s + r) * n + (s + k)] : 0.0;
    };
    auto fb = [&](int k, int c) -> double {
        int j = j0 + c;
        return (j < s) ? T[(int64_t)k * n + j] : 0.0;
    };
    dgemm_tile<6, false>(acc, fa, fb, 0, w, smem);
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
#pragma unroll
    for (int a = 0; a < 6; a++) {
        int i = ty + 16 * a;
        if (i >= w) continue;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            int j = j0 + tx + 16 * b;
            if (j < s) Y[(int64_t)(s + i) * n + j] = -acc[a][b];
        }
    }
}

static int run_tri_inverse(const TriArgs* args_dev, int nitems, int n, cudaStream_t st) {
    for (int s = 0; s < n; s += NB) {
        int w = min(NB, n - s);
        size_t smem = (size_t)NB * NB * sizeof(double);
        cudaFuncSetAttribute(tri_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        CDCLQ_LAUNCH(tri_diag_kernel, nitems, 128, smem, st, args_dev, n, s, w);
        if (s > 0) {
            dim3 g((s + 63) / 64, nitems);
            CDCLQ_LAUNCH(tri_gemm1_kernel, g, 256, DTile2<3>::SMEM_BYTES, st, args_dev, n, s, w);
            CDCLQ_LAUNCH(tri_gemm2_kernel, g, 256, 0, st, args_dev, n, s, w);
        }
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "triangular inverse kernels launch");
}

// ---------------------------------------------------------------------------------------------------------
// src/linalg.rs:368-373: U[i][j] = (f32) Y[n-1-i][n-1-j] for j >= i, else 0
__global__ void u_scatter_kernel(const PrepItem* __restrict__ items, int n) {
    const PrepItem it = items[blockIdx.z];
    if (it.status->err) return;
    int i = blockIdx.y;
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    it.u[(int64_t)i * n + j] = (j >= i) ? (float)it.y[(int64_t)(n - 1 - i) * n + (n - 1 - j)] : 0.0f;
}

// The batched launchers build per-item argument tables in device memory carved from the items' own
// scratch: the host passes PrepItem tables, the factorisation kernels need (a, status) and (l, y, t, status).
__global__ void make_chol_args_kernel(const PrepItem* items, CholArgs* chol, TriArgs* tri, int nitems) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nitems) return;
    chol[i].a = items[i].hr;
    chol[i].status = items[i].status;
    tri[i].l = items[i].hr;
    tri[i].y = items[i].y;
    tri[i].t = items[i].tbuf;
    tri[i].status = items[i].status;
}

struct ArgTables {
    CholArgs* chol = nullptr;
    TriArgs* tri = nullptr;
};

static int make_tables(const PrepItem* items_dev, int nitems, cudaStream_t st, ArgTables& t) {
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&t.chol, sizeof(CholArgs) * nitems, st));
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&t.tri, sizeof(TriArgs) * nitems, st));
    CDCLQ_LAUNCH(make_chol_args_kernel, (nitems + 127) / 128, 128, 0, st, items_dev, t.chol, t.tri, nitems);
    return 0;
}

static void free_tables(ArgTables& t, cudaStream_t st) {
    if (t.chol) cudaFreeAsync(t.chol, st);
    if (t.tri) cudaFreeAsync(t.tri, st);
    t.chol = nullptr;
    t.tri = nullptr;
}

// Cholesky and triangular inverse of a batch, pipelined over two streams.  Step s of the inverse reads only
// the block row s of L (columns < s + 96), which is final once the Cholesky's diagonal kernel of step s has run:
// later panel solves and trailing updates write rows >= s + 96 only.  So the inverse runs on a second stream,
// each step waiting for an event recorded after that diagonal kernel, and its latency-bound steps (diagonal
// inverses, the early narrow products) overlap the Cholesky's trailing updates.  Same kernels, same operands,
// same results as running the two one after the other.
int launch_factor(const PrepItem* items_dev, int nitems, int n, cudaStream_t st) {
    ArgTables t;
    int rc = make_tables(items_dev, nitems, st, t);
    if (rc) return rc;
    const int steps = (n + NB - 1) / NB;
    std::vector<cudaEvent_t> ev(steps + 1, nullptr);
    cudaStream_t st2 = nullptr;
    int prio = 0;
    cudaStreamGetPriority(st, &prio);  // the inverse runs at its Cholesky's priority
    cudaError_t e = cudaStreamCreateWithPriority(&st2, cudaStreamNonBlocking, prio);
    for (int i = 0; i <= steps && e == cudaSuccess; i++) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev[steps], st);  // the argument tables and the prepared matrices
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st2, ev[steps], 0);
    if (e != cudaSuccess) rc = cuda_error(e, "factorisation streams");
    cudaFuncSetAttribute(chol_trail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DTile2<4>::SMEM_BYTES);
    cudaFuncSetAttribute(chol_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)CHOL_DIAG_SMEM);
    const size_t smem_nb = (size_t)NB * NB * sizeof(double);
    cudaFuncSetAttribute(chol_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_nb);
    cudaFuncSetAttribute(tri_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_nb);
    for (int i = 0; i < steps && !rc; i++) {
        const int k = i * NB, kb = min(NB, n - k), kend = k + kb;
        CDCLQ_LAUNCH(chol_diag_kernel, nitems, 256, CHOL_DIAG_SMEM, st, t.chol, n, k, kb);
        e = cudaEventRecord(ev[i], st);
        if (e != cudaSuccess) {
            rc = cuda_error(e, "factorisation event");
            break;
        }
        if (kend < n) {
            const int rows_below = n - kend;
            dim3 gp((rows_below + 127) / 128, nitems);
            CDCLQ_LAUNCH(chol_panel_kernel, gp, 128, smem_nb, st, t.chol, n, k, kb);
            dim3 gt((unsigned)chol_trail_tiles(rows_below), nitems);
            CDCLQ_LAUNCH(chol_trail_kernel, gt, 256, DTile2<4>::SMEM_BYTES, st, t.chol, n, k, kb);
        }
        // inverse step i on the second stream, after block row i of L is final
        e = cudaStreamWaitEvent(st2, ev[i], 0);
        if (e != cudaSuccess) {
            rc = cuda_error(e, "factorisation event wait");
            break;
        }
        CDCLQ_LAUNCH(tri_diag_kernel, nitems, 128, smem_nb, st2, t.tri, n, k, kb);
        if (k > 0) {
            dim3 g((k + 63) / 64, nitems);
            CDCLQ_LAUNCH(tri_gemm1_kernel, g, 256, DTile2<3>::SMEM_BYTES, st2, t.tri, n, k, kb);
            CDCLQ_LAUNCH(tri_gemm2_kernel, g, 256, 0, st2, t.tri, n, k, kb);
        }
    }
    if (!rc && (e = cudaGetLastError()) != cudaSuccess) rc = cuda_error(e, "factorisation kernels launch");
    // join: the caller's stream continues after both chains (also on an error, so nothing is left in flight
    // on the second stream when the tables are released)
    if (st2 && ev[steps]) {
        cudaEventRecord(ev[steps], st2);
        cudaStreamWaitEvent(st, ev[steps], 0);
    }
    for (auto x : ev)
        if (x) cudaEventDestroy(x);
    if (st2) cudaStreamDestroy(st2);
    free_tables(t, st);
    return rc;
}

int launch_u_scatter(const PrepItem* items_dev, int nitems, int n, cudaStream_t st) {
    dim3 g((n + 255) / 256, n, nitems);
    CDCLQ_LAUNCH(u_scatter_kernel, g, 256, 0, st, items_dev, n);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "u_scatter_kernel launch");
}

// Single-matrix entry points for the C ABI (cholesky_lower / tri_inverse_lower on their own).
int device_cholesky(double* a, int n, FactorStatus* status, cudaStream_t st) {
    CholArgs* args = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&args, sizeof(CholArgs), st));
    CholArgs h{a, status};
    cudaError_t e = cudaMemcpyAsync(args, &h, sizeof h, cudaMemcpyHostToDevice, st);
    int rc = (e == cudaSuccess) ? 0 : cuda_error(e, "cholesky args");
    if (!rc) rc = run_cholesky(args, 1, n, st);
    cudaStreamSynchronize(st);
    cudaFreeAsync(args, st);
    return rc;
}

int device_tri_inverse(const double* l, double* y, double* tbuf, int n, cudaStream_t st) {
    TriArgs* args = nullptr;
    FactorStatus* status = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&args, sizeof(TriArgs), st));
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&status, sizeof(FactorStatus), st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(FactorStatus), st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(y, 0, sizeof(double) * (size_t)n * n, st));
    TriArgs h{l, y, tbuf, status};
    cudaError_t e = cudaMemcpyAsync(args, &h, sizeof h, cudaMemcpyHostToDevice, st);
    int rc = (e == cudaSuccess) ? 0 : cuda_error(e, "tri args");
    if (!rc) rc = run_tri_inverse(args, 1, n, st);
    cudaStreamSynchronize(st);
    cudaFreeAsync(args, st);
    cudaFreeAsync(status, st);
    return rc;
}

// ---------------------------------------------------------------------------------------------------------
// Weight-side preparation
__global__ void hdiag_kernel(const float* h, int n, double* hdiag) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) hdiag[j] = (double)h[(int64_t)j * n + j];
}

int launch_hdiag(const float* h, int n, double* hdiag, cudaStream_t st) {
    CDCLQ_LAUNCH(hdiag_kernel, (n + 255) / 256, 256, 0, st, h, n, hdiag);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "hdiag_kernel launch");
}

// src/engine.rs:279-285 over the dead-zeroed weights: rows summed in order, (w as f64) * (w as f64), starting
// from init[j] (the running sums of the rows before these, held by another rank) or from 0 when init is null
__global__ void colsq_kernel(const float* w, const double* hdiag, int d_out, int n, const double* init, double* colsq) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    bool dead = hdiag[j] == 0.0;
    double s = init ? init[j] : 0.0;
    for (int r = 0; r < d_out; r++) {
        double v = dead ? 0.0 : (double)w[(int64_t)r * n + j];
        s = __dadd_rn(s, __dmul_rn(v, v));
    }
    colsq[j] = s;
}

int launch_colsq(const float* w, const double* hdiag, int d_out, int n, double* colsq, cudaStream_t st) {
    return launch_colsq_from(w, hdiag, d_out, n, nullptr, colsq, st);
}

int launch_colsq_from(const float* w, const double* hdiag, int d_out, int n, const double* init, double* colsq,
                      cudaStream_t st) {
    CDCLQ_LAUNCH(colsq_kernel, (n + 255) / 256, 256, 0, st, w, hdiag, d_out, n, init, colsq);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "colsq_kernel launch");
}

__global__ void permute_w_kernel(const float* w, const double* hdiag, const uint32_t* perm, int d_out, int n,
                                 float* wt) {
    int r = blockIdx.y;
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n || r >= d_out) return;
    uint32_t p = perm[j];
    wt[(int64_t)r * n + j] = (hdiag[p] == 0.0) ? 0.0f : w[(int64_t)r * n + p];
}

int launch_permute_w(const float* w, const double* hdiag, const uint32_t* perm, int d_out, int n, float* wt,
                     cudaStream_t st) {
    for (int r0 = 0; r0 < d_out; r0 += 65535) {
        int rows = min(65535, d_out - r0);
        dim3 g((n + 255) / 256, rows);
        CDCLQ_LAUNCH(permute_w_kernel, g, 256, 0, st, w + (int64_t)r0 * n, hdiag, perm, rows, n, wt + (int64_t)r0 * n);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "permute_w_kernel launch");
}

}  // namespace cdclq
