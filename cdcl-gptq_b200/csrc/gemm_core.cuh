// gemm_core.cuh - the register-tiled SIMT FP32 GEMM core shared by the GPTQ lazy update (phase 1) and the
// repair gradients (phase 2).
//
// Why SIMT FFMA and not tcgen05: the reference's GEMMs are f32 `matrixmultiply` calls whose results feed
// rounding decisions (code choice, scale acceptance).  A tensor-core f32 emulation (3xTF32 / bf16x9) rounds
// differently and would turn exact parity into tie-level agreement.  This core keeps, for every output
// element, one f32 accumulator that receives the products in increasing k through __fmaf_rn, starting from
// +0 - the fixed order of the oracle - so results are bit-identical to it.
//
// CTA tile: 64 rows x (16*TN) columns, 256 threads laid out 16 (ty) x 16 (tx).  Thread (ty, tx) owns rows
// ty*4 .. ty*4+3 and columns
//     TN == 8 : tx*4 .. tx*4+3  and  64 + tx*4 .. 64 + tx*4+3
//     TN == 4 : tx*4 .. tx*4+3
//     TN == 2 : tx*2 .. tx*2+1
// K is consumed in stages of KT = 16: the A stage is held k-major in shared memory ([KT][A_LD]) so that one
// 16-byte load yields a thread's four rows, the B stage is row-major ([KT][16*TN]).  The next stage is
// fetched into registers while the current one is multiplied (register double buffering).
#pragma once

#include <cstdint>

namespace cdclq {

constexpr int GEMM_KT = 16;
constexpr int GEMM_RT = 64;      // rows per CTA tile
constexpr int GEMM_ALD = 68;     // k-major A row stride (64 rows + 4 pad, keeps 16-byte alignment)
constexpr int GEMM_THREADS = 256;

// Thread coordinates inside the 16 x 16 thread grid of a CTA tile.  Each warp covers 8 (ty) x 4 (tx)
// threads, so per k-step its A fragments are 32 consecutive rows (one 128-byte shared-memory wavefront) and its
// B fragments 4 x 4 consecutive columns (one 64-byte broadcast wavefront per 16-byte load): 3 wavefronts per
// warp and k at TN = 8 instead of 5 with a 2 x 16 warp shape.
__device__ __forceinline__ void gemm_coords(int tid, int& ty, int& tx) {
    const int lane = tid & 31, warp = tid >> 5;
    ty = ((warp >> 2) << 3) | (lane >> 2);
    tx = ((warp & 3) << 2) | (lane & 3);
}

template <int TN>
struct ColMap {
    // column (within the CTA tile) of the thread's j-th accumulator
    static __device__ __forceinline__ int col(int tx, int j) {
        if constexpr (TN == 8) return (j < 4) ? (tx * 4 + j) : (64 + tx * 4 + (j - 4));
        else if constexpr (TN == 4) return tx * 4 + j;
        else return tx * 2 + j;
    }
};

// Shared-memory footprint of the staging buffers, in floats.
template <int TN>
__host__ __device__ constexpr int gemm_stage_floats() {
    return 2 * GEMM_KT * GEMM_ALD + 2 * GEMM_KT * 16 * TN;
}

// Multiply-accumulate one KT stage held in shared memory.
template <int TN>
__device__ __forceinline__ void gemm_stage_mac(float (&acc)[4][TN], const float* __restrict__ As,
                                               const float* __restrict__ Bs, int ty, int tx) {
#pragma unroll
    for (int kk = 0; kk < GEMM_KT; kk++) {
        float4 a = *reinterpret_cast<const float4*>(As + kk * GEMM_ALD + ty * 4);
        float av[4] = {a.x, a.y, a.z, a.w};
        float bv[TN];
        const float* brow = Bs + kk * (16 * TN);
        if constexpr (TN == 8) {
            float4 b0 = *reinterpret_cast<const float4*>(brow + tx * 4);
            float4 b1 = *reinterpret_cast<const float4*>(brow + 64 + tx * 4);
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
            bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
        } else if constexpr (TN == 4) {
            float4 b0 = *reinterpret_cast<const float4*>(brow + tx * 4);
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
        } else {
            float2 b0 = *reinterpret_cast<const float2*>(brow + tx * 2);
            bv[0] = b0.x; bv[1] = b0.y;
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < TN; j++) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
    }
}

// A operand read from global memory: rows [0, rows_valid) of a row-major matrix with leading dimension lda,
// columns (the K index) [k0, K).  Out-of-range elements read as 0 (an exact no-op in the accumulation: the
// accumulator is never -0, so adding a zero product leaves it unchanged).  Plain (coherent) loads: the
// repair kernels rewrite the error matrix between two GEMMs of the same launch.
struct AGlobal {
    const float* a;
    int64_t lda;
    int rows_valid;
    int K;
    bool vec;  // 16-byte aligned rows and K % 4 == 0
    // Each thread fetches 4 consecutive k of one row: thread t -> row t%64, k-quad t/64.  A warp then covers
    // 32 consecutive rows, which makes the transposed shared-memory stores below conflict-free.
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[4]) const {
        int row = tid & 63, q = tid >> 6;
        int k = k0 + q * 4;
        if (row < rows_valid) {
            const float* p = a + (int64_t)row * lda + k;
            if (vec && k + 3 < K) {
                float4 v = *reinterpret_cast<const float4*>(p);
                r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) r[i] = (k + i < K) ? p[i] : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) r[i] = 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* As, int tid, const float (&r)[4]) const {
        int row = tid & 63, q = tid >> 6;
#pragma unroll
        for (int i = 0; i < 4; i++) As[(q * 4 + i) * GEMM_ALD + row] = r[i];
    }
};

// B operand: B[k][col0 + c] of a row-major matrix (leading dimension ldb), c in [0, wd), k in [k0, K).
template <int TN>
struct BGlobal {
    const float* __restrict__ b;
    int64_t ldb;
    int64_t col0;
    int wd;
    int K;
    bool vec;  // (b + col0) 16-byte aligned and ldb % 4 == 0
    static constexpr int WT = 16 * TN;
    static constexpr int PER = GEMM_KT * WT / GEMM_THREADS;  // floats per thread per stage (1, 2, 4 or 8)
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[PER > 0 ? PER : 1]) const {
        // thread covers PER consecutive columns of one k row
        constexpr int TPR = WT / PER;  // threads per k row
        int kr = tid / TPR, c = (tid % TPR) * PER;
        int k = k0 + kr;
        const float* p = b + (int64_t)k * ldb + col0 + c;
        if (k < K) {
            if (PER >= 4 && vec && c + PER <= wd) {
#pragma unroll
                for (int v = 0; v < PER / 4; v++) {
                    float4 x = __ldg(reinterpret_cast<const float4*>(p) + v);
                    r[v * 4 + 0] = x.x; r[v * 4 + 1] = x.y; r[v * 4 + 2] = x.z; r[v * 4 + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < PER; i++) r[i] = (c + i < wd) ? __ldg(p + i) : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < PER; i++) r[i] = 0.0f;
        }
    }
    // Vector stores: a warp writes 32 x PER consecutive floats of one or two k rows (no bank conflicts).
    __device__ __forceinline__ void store(float* Bs, int tid, const float (&r)[PER > 0 ? PER : 1]) const {
        constexpr int TPR = WT / PER;
        int kr = tid / TPR, c = (tid % TPR) * PER;
        float* dst = Bs + kr * WT + c;
        if constexpr (PER % 4 == 0) {
#pragma unroll
            for (int v = 0; v < PER / 4; v++)
                reinterpret_cast<float4*>(dst)[v] = make_float4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
        } else if constexpr (PER == 2) {
            *reinterpret_cast<float2*>(dst) = make_float2(r[0], r[1]);
        } else {
#pragma unroll
            for (int i = 0; i < PER; i++) dst[i] = r[i];
        }
    }
};

// acc[i][j] (+)= sum_k A[row_i][k] * B[k][col_j] over k in [0, K), A from global memory.
// `stage` points at gemm_stage_floats<TN>() floats of shared memory.  Ends with a __syncthreads().
template <int TN>
__device__ void gemm_global_a(float (&acc)[4][TN], const AGlobal& A, const BGlobal<TN>& B, int K, float* stage) {
    const int tid = threadIdx.x;
    int ty, tx;
    gemm_coords(tid, ty, tx);
    float* const As0 = stage;                            // As[buf] = As0 + buf * KT*ALD
    float* const Bs0 = stage + 2 * GEMM_KT * GEMM_ALD;   // Bs[buf] = Bs0 + buf * KT*16*TN
    constexpr int PER = BGlobal<TN>::PER;
    float ra[4], rb[PER];
    A.fetch(0, tid, ra);
    B.fetch(0, tid, rb);
    A.store(As0, tid, ra);
    B.store(Bs0, tid, rb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += GEMM_KT) {
        bool more = k0 + GEMM_KT < K;
        if (more) {
            A.fetch(k0 + GEMM_KT, tid, ra);
            B.fetch(k0 + GEMM_KT, tid, rb);
        }
        gemm_stage_mac<TN>(acc, As0 + buf * GEMM_KT * GEMM_ALD, Bs0 + buf * GEMM_KT * 16 * TN, ty, tx);
        if (more) {
            A.store(As0 + (buf ^ 1) * GEMM_KT * GEMM_ALD, tid, ra);
            B.store(Bs0 + (buf ^ 1) * GEMM_KT * 16 * TN, tid, rb);
        }
        __syncthreads();
        buf ^= 1;
    }
}

// Same with A already resident in shared memory, k-major with row stride GEMM_ALD (A_s[k][row]); only the
// B operand is staged.  K rows of A_s must exist; rows beyond the valid rows must hold zeros or be ignored
// by the caller.  Ends with a __syncthreads().
template <int TN>
__device__ void gemm_smem_a(float (&acc)[4][TN], const float* As_full, const BGlobal<TN>& B, int K, float* stage) {
    const int tid = threadIdx.x;
    int ty, tx;
    gemm_coords(tid, ty, tx);
    float* const Bs0 = stage + 2 * GEMM_KT * GEMM_ALD;   // Bs[buf] = Bs0 + buf * KT*16*TN
    constexpr int PER = BGlobal<TN>::PER;
    float rb[PER];
    B.fetch(0, tid, rb);
    B.store(Bs0, tid, rb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += GEMM_KT) {
        bool more = k0 + GEMM_KT < K;
        if (more) B.fetch(k0 + GEMM_KT, tid, rb);
        int kn = K - k0 < GEMM_KT ? K - k0 : GEMM_KT;
        const float* As = As_full + (int64_t)k0 * GEMM_ALD;
        const float* Bb = Bs0 + buf * GEMM_KT * 16 * TN;
        if (kn == GEMM_KT) {
            gemm_stage_mac<TN>(acc, As, Bb, ty, tx);
        } else {
            for (int kk = 0; kk < kn; kk++) {
                float4 a = *reinterpret_cast<const float4*>(As + kk * GEMM_ALD + ty * 4);
                float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < TN; j++)
                        acc[i][j] = __fmaf_rn(av[i], Bb[kk * (16 * TN) + ColMap<TN>::col(tx, j)], acc[i][j]);
            }
        }
        if (more) B.store(Bs0 + (buf ^ 1) * GEMM_KT * 16 * TN, tid, rb);
        __syncthreads();
        buf ^= 1;
    }
}

// A operand stored transposed in global memory: A(i, k) = a[k * lda + i] (e.g. X^T of a token matrix).
// Contiguous along i, so a stage is fetched as 16 k rows x 64 i and stored k-major without a transpose.
struct AGlobalT {
    const float* a;
    int64_t lda;
    int64_t row0;     // first i of the CTA tile
    int rows_valid;   // i < rows_valid (relative to row0)
    int K;
    bool vec;         // (a + row0) 16-byte aligned and lda % 4 == 0
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[4]) const {
        int kr = tid >> 4, q = (tid & 15) * 4;
        int k = k0 + kr;
        if (k < K) {
            const float* p = a + (int64_t)k * lda + row0 + q;
            if (vec && q + 3 < rows_valid) {
                float4 v = *reinterpret_cast<const float4*>(p);
                r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) r[i] = (q + i < rows_valid) ? p[i] : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) r[i] = 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* As, int tid, const float (&r)[4]) const {
        int kr = tid >> 4, q = (tid & 15) * 4;
        *reinterpret_cast<float4*>(As + kr * GEMM_ALD + q) = make_float4(r[0], r[1], r[2], r[3]);
    }
};

// Staged GEMM with an arbitrary A loader (AGlobal, AGlobalT, or a shared-memory source).  Ends with a
// __syncthreads().
template <int TN, class AL>
__device__ void gemm_loader_a(float (&acc)[4][TN], const AL& A, const BGlobal<TN>& B, int K, float* stage) {
    const int tid = threadIdx.x;
    int ty, tx;
    gemm_coords(tid, ty, tx);
    float* const As0 = stage;                            // As[buf] = As0 + buf * KT*ALD
    float* const Bs0 = stage + 2 * GEMM_KT * GEMM_ALD;   // Bs[buf] = Bs0 + buf * KT*16*TN
    constexpr int PER = BGlobal<TN>::PER;
    float ra[4], rb[PER];
    A.fetch(0, tid, ra);
    B.fetch(0, tid, rb);
    A.store(As0, tid, ra);
    B.store(Bs0, tid, rb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += GEMM_KT) {
        bool more = k0 + GEMM_KT < K;
        if (more) {
            A.fetch(k0 + GEMM_KT, tid, ra);
            B.fetch(k0 + GEMM_KT, tid, rb);
        }
        gemm_stage_mac<TN>(acc, As0 + buf * GEMM_KT * GEMM_ALD, Bs0 + buf * GEMM_KT * 16 * TN, ty, tx);
        if (more) {
            A.store(As0 + (buf ^ 1) * GEMM_KT * GEMM_ALD, tid, ra);
            B.store(Bs0 + (buf ^ 1) * GEMM_KT * 16 * TN, tid, rb);
        }
        __syncthreads();
        buf ^= 1;
    }
}

}  // namespace cdclq
