// gemm_core.cuh - the register-tiled SIMT FP32 GEMM core shared by the GPTQ lazy update (phase 1), the
// repair gradients (phase 2) and the stand-alone GEMMs.
//
// Why SIMT FFMA and not tcgen05: the reference's GEMMs are f32 `matrixmultiply` calls whose results feed
// rounding decisions (code choice, scale acceptance).  A tensor-core f32 emulation (3xTF32 / bf16x9) rounds
// differently and would turn exact parity into tie-level agreement.  This core keeps, for every output
// element, one f32 accumulator that receives the products in increasing k through __fmaf_rn, starting from
// +0 - the fixed order of the oracle - so results are bit-identical to it.  The products are issued as packed
// f32x2 FMAs (`fma.rn.f32x2`, two lanes of the accumulator tile per instruction): each lane is an independent
// IEEE round-to-nearest FMA, so packing changes the instruction count, not a single rounding.
//
// CTA tile BM x BN (BM in {64, 128} rows, BN in {32, 64, 128} columns), 256 threads in a 16 x 16 grid, so a
// thread owns TM = BM/16 rows x TN = BN/16 columns: rows ty*TM .. ty*TM+TM-1 and columns in TN/4 groups of 4,
// the groups spaced BN/(TN/4) apart (TN = 2: two adjacent columns).  Each warp covers 8 (tx) x 4 (ty) threads,
// so a k-step's fragment loads are single 128-byte shared-memory wavefronts.  K is consumed in stages of KT:
// the A stage is held k-major in shared memory ([KT][BM+4], one 16-byte load = 4 rows of a thread), the B stage
// row-major ([KT][BN]); the next stage is fetched into registers while the current one is multiplied, and
// within a stage the fragments of the next k-step are read while the current k-step's products issue.
#pragma once

#include <cstdint>

namespace cdclq {

constexpr int GEMM_THREADS = 256;

template <int BM_, int BN_, int KT_>
struct Tile {
    static constexpr int BM = BM_, BN = BN_, KT = KT_;
    static constexpr int TM = BM / 16, TN = BN / 16;
    static constexpr int ALD = BM + 4;                  // k-major A row stride (16-byte aligned rows)
    static constexpr int AP = BM * KT / GEMM_THREADS;   // A floats fetched per thread per stage
    static constexpr int BP = BN * KT / GEMM_THREADS;   // B floats fetched per thread per stage
    static constexpr int B_STAGE_FLOATS = 2 * KT * BN;  // B double buffer alone (A resident in shared memory)
    static constexpr int STAGE_FLOATS = 2 * KT * ALD + B_STAGE_FLOATS;
    // Staged A: the row index is XOR-swizzled per k so that the QPR threads sharing a row in AGlobal::store
    // (rows tid / QPR) write to distinct banks; the XOR keeps every aligned 4-row group contiguous.
    static constexpr int QPR = KT / AP;
    static constexpr int SWZ = (QPR == 2 && (4 * AP) % 32 == 0) ? 16 : (QPR == 4 && (4 * AP) % 32 == 16) ? 8 : 0;
    static __host__ __device__ constexpr int a_swz(int k) {
        return SWZ == 16 ? ((k / AP) & 1) * 16 : SWZ == 8 ? (((k / AP) >> 1) & 1) * 8 : 0;
    }
    static_assert(TM == 4 || TM == 8, "BM must be 64 or 128");
    static_assert(TN == 2 || TN == 4 || TN == 8, "BN must be 32, 64 or 128");
    static_assert(AP >= 2 && BP >= 1, "stage too small");
};

// Thread coordinates in the 16 x 16 thread grid: a warp is 8 (tx) x 4 (ty) threads; warps tile the grid 2 x 4.
__device__ __forceinline__ void gemm_coords(int tid, int& ty, int& tx) {
    const int lane = tid & 31, warp = tid >> 5;
    tx = ((warp & 1) << 3) | (lane & 7);
    ty = ((warp >> 1) << 2) | (lane >> 3);
}

template <class S>
struct TileMap {
    // row (within the CTA tile) of the thread's i-th accumulator row, column of its j-th accumulator column
    static __device__ __forceinline__ int row(int ty, int i) { return ty * S::TM + i; }
    static __device__ __forceinline__ int col(int tx, int j) {
        if constexpr (S::TN == 2) return tx * 2 + j;
        else return (j >> 2) * (S::BN / (S::TN / 4)) + tx * 4 + (j & 3);
    }
};

// Multiply-accumulate one KT stage held in shared memory (the first kn k-steps of it); the fragments of k-step
// kk+1 are loaded before the products of kk are issued.
template <class S, bool SWZ>
__device__ __forceinline__ void frag_load(float (&av)[S::TM], float (&bv)[S::TN], const float* __restrict__ As,
                                          const float* __restrict__ Bs, int kk, int ty, int tx) {
#pragma unroll
    for (int v = 0; v < S::TM / 4; v++) {
        const int row = SWZ ? ((ty * S::TM + 4 * v) ^ S::a_swz(kk)) : ty * S::TM + 4 * v;
        float4 a = *reinterpret_cast<const float4*>(As + kk * S::ALD + row);
        av[4 * v] = a.x; av[4 * v + 1] = a.y; av[4 * v + 2] = a.z; av[4 * v + 3] = a.w;
    }
    const float* brow = Bs + kk * S::BN;
    if constexpr (S::TN == 2) {
        float2 b = *reinterpret_cast<const float2*>(brow + tx * 2);
        bv[0] = b.x; bv[1] = b.y;
    } else {
#pragma unroll
        for (int v = 0; v < S::TN / 4; v++) {
            float4 b = *reinterpret_cast<const float4*>(brow + v * (S::BN / (S::TN / 4)) + tx * 4);
            bv[4 * v] = b.x; bv[4 * v + 1] = b.y; bv[4 * v + 2] = b.z; bv[4 * v + 3] = b.w;
        }
    }
}

// (c0, c1) += (a0 * b0, a1 * b1) as one packed f32x2 FMA: two independent IEEE round-to-nearest FMAs, each the
// same result as __fmaf_rn on its lane, so the per-element accumulation order is unchanged.
__device__ __forceinline__ void ffma2(float& c0, float& c1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ta, tb, tc;\n\t"
        "mov.b64 ta, {%2, %3};\n\t"
        "mov.b64 tb, {%4, %5};\n\t"
        "mov.b64 tc, {%0, %1};\n\t"
        "fma.rn.f32x2 tc, ta, tb, tc;\n\t"
        "mov.b64 {%0, %1}, tc;\n\t}"
        : "+f"(c0), "+f"(c1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// SWZ: the A stage was written with the k-dependent row swizzle (staged operands); resident A is not swizzled.
template <class S, bool SWZ>
__device__ __forceinline__ void gemm_stage_mac(float (&acc)[S::TM][S::TN], const float* __restrict__ As,
                                               const float* __restrict__ Bs, int ty, int tx, int kn = S::KT) {
    float av[2][S::TM], bv[2][S::TN];
    frag_load<S, SWZ>(av[0], bv[0], As, Bs, 0, ty, tx);
#pragma unroll
    for (int kk = 0; kk < S::KT; kk++) {
        if (kk + 1 < S::KT && kk + 1 < kn)
            frag_load<S, SWZ>(av[(kk + 1) & 1], bv[(kk + 1) & 1], As, Bs, kk + 1, ty, tx);
        if (kk < kn) {
            // Packed f32x2 FMAs (sm_100): half the FMA instructions of a scalar loop, same per-element order.
            // Lanes pair along the longer side of the thread's tile, so the operand that must be duplicated
            // into both lanes is the shorter fragment.
            if constexpr (S::TM > S::TN) {
#pragma unroll
                for (int j = 0; j < S::TN; j++)
#pragma unroll
                    for (int i = 0; i < S::TM; i += 2)
                        ffma2(acc[i][j], acc[i + 1][j], av[kk & 1][i], av[kk & 1][i + 1], bv[kk & 1][j],
                              bv[kk & 1][j]);
            } else {
#pragma unroll
                for (int i = 0; i < S::TM; i++)
#pragma unroll
                    for (int j = 0; j < S::TN; j += 2)
                        ffma2(acc[i][j], acc[i][j + 1], av[kk & 1][i], av[kk & 1][i], bv[kk & 1][j],
                              bv[kk & 1][j + 1]);
            }
        }
    }
}

// ---- A operand loaders ------------------------------------------------------------------------------------
// Out-of-range elements read as 0: an exact no-op in the accumulation (the accumulator is never -0, so adding a
// zero product leaves it unchanged).

// Row-major A from global memory: rows [0, rows_valid) with leading dimension lda, K index in [0, K).  Each
// thread fetches AP consecutive k of one row (coalesced).  Plain (coherent) loads: the repair kernels rewrite
// the error matrix between two GEMMs of the same launch.
template <class S>
struct AGlobal {
    const float* a;
    int64_t lda;
    int rows_valid;
    int K;
    bool vec;  // 16-byte aligned rows and K % 4 == 0
    static constexpr int QPR = S::KT / S::AP;  // threads per row
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[S::AP]) const {
        const int row = tid / QPR, k = k0 + (tid % QPR) * S::AP;
        if (row < rows_valid) {
            const float* p = a + (int64_t)row * lda + k;
            if (S::AP % 4 == 0 && vec && k + S::AP <= K) {
#pragma unroll
                for (int v = 0; v < S::AP / 4; v++) {
                    float4 x = *reinterpret_cast<const float4*>(p + 4 * v);
                    r[4 * v] = x.x; r[4 * v + 1] = x.y; r[4 * v + 2] = x.z; r[4 * v + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < S::AP; i++) r[i] = (k + i < K) ? p[i] : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < S::AP; i++) r[i] = 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* As, int tid, const float (&r)[S::AP]) const {
        const int row = tid / QPR, q = tid % QPR;
#pragma unroll
        for (int i = 0; i < S::AP; i++) As[(q * S::AP + i) * S::ALD + (row ^ S::a_swz(q * S::AP + i))] = r[i];
    }
};

// A stored transposed in global memory: A(i, k) = a[k * lda + i] (e.g. X^T of a token matrix), i relative to
// row0.  Contiguous along i, so a stage is fetched as KT k rows x BM i and stored without a transpose.
template <class S>
struct AGlobalT {
    const float* a;
    int64_t lda;
    int64_t row0;
    int rows_valid;
    int K;
    bool vec;  // (a + row0) 16-byte aligned and lda % 4 == 0
    static constexpr int TPR = S::BM / S::AP;  // threads per k row
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[S::AP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::AP, k = k0 + kr;
        if (k < K) {
            const float* p = a + (int64_t)k * lda + row0 + c;
            if (S::AP % 4 == 0 && vec && c + S::AP <= rows_valid) {
#pragma unroll
                for (int v = 0; v < S::AP / 4; v++) {
                    float4 x = *reinterpret_cast<const float4*>(p + 4 * v);
                    r[4 * v] = x.x; r[4 * v + 1] = x.y; r[4 * v + 2] = x.z; r[4 * v + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < S::AP; i++) r[i] = (c + i < rows_valid) ? p[i] : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < S::AP; i++) r[i] = 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* As, int tid, const float (&r)[S::AP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::AP;
#pragma unroll
        for (int i = 0; i < S::AP; i++) As[kr * S::ALD + ((c + i) ^ S::a_swz(kr))] = r[i];
    }
};

// ---- B operand: B[k][col0 + c] of a row-major matrix (leading dimension ldb), c in [0, wd), k in [k0, K) ----
template <class S>
struct BGlobal {
    const float* __restrict__ b;
    int64_t ldb;
    int64_t col0;
    int wd;
    int K;
    bool vec;  // (b + col0) 16-byte aligned and ldb % 4 == 0
    static constexpr int TPR = S::BN / S::BP;  // threads per k row
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[S::BP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::BP, k = k0 + kr;
        if (k < K) {
            const float* p = b + (int64_t)k * ldb + col0 + c;
            if (S::BP % 4 == 0 && vec && c + S::BP <= wd) {
#pragma unroll
                for (int v = 0; v < S::BP / 4; v++) {
                    float4 x = __ldg(reinterpret_cast<const float4*>(p) + v);
                    r[4 * v] = x.x; r[4 * v + 1] = x.y; r[4 * v + 2] = x.z; r[4 * v + 3] = x.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < S::BP; i++) r[i] = (c + i < wd) ? __ldg(p + i) : 0.0f;
            }
        } else {
#pragma unroll
            for (int i = 0; i < S::BP; i++) r[i] = 0.0f;
        }
    }
    // Vector stores: a warp writes consecutive floats of one or two k rows (no bank conflicts).
    __device__ __forceinline__ void store(float* Bs, int tid, const float (&r)[S::BP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::BP;
        float* dst = Bs + kr * S::BN + c;
        if constexpr (S::BP % 4 == 0) {
#pragma unroll
            for (int v = 0; v < S::BP / 4; v++)
                reinterpret_cast<float4*>(dst)[v] = make_float4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
        } else if constexpr (S::BP == 2) {
            *reinterpret_cast<float2*>(dst) = make_float2(r[0], r[1]);
        } else {
            *dst = r[0];
        }
    }
};

// acc (+)= A B over k in [0, K) with A from a loader.  `stage` points at S::STAGE_FLOATS floats of shared
// memory.  Ends with a __syncthreads().
template <class S, class AL>
__device__ void gemm_loader_a(float (&acc)[S::TM][S::TN], const AL& A, const BGlobal<S>& B, int K, float* stage) {
    const int tid = threadIdx.x;
    int ty, tx;
    gemm_coords(tid, ty, tx);
    float* const As0 = stage;                       // As[buf] = As0 + buf * KT*ALD
    float* const Bs0 = stage + 2 * S::KT * S::ALD;  // Bs[buf] = Bs0 + buf * KT*BN
    float ra[S::AP], rb[S::BP];
    A.fetch(0, tid, ra);
    B.fetch(0, tid, rb);
    A.store(As0, tid, ra);
    B.store(Bs0, tid, rb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += S::KT) {
        const bool more = k0 + S::KT < K;
        if (more) {
            A.fetch(k0 + S::KT, tid, ra);
            B.fetch(k0 + S::KT, tid, rb);
        }
        gemm_stage_mac<S, true>(acc, As0 + buf * S::KT * S::ALD, Bs0 + buf * S::KT * S::BN, ty, tx);
        if (more) {
            A.store(As0 + (buf ^ 1) * S::KT * S::ALD, tid, ra);
            B.store(Bs0 + (buf ^ 1) * S::KT * S::BN, tid, rb);
        }
        __syncthreads();
        buf ^= 1;
    }
}

// Same with A already resident in shared memory, k-major with row stride S::ALD (As[k][row]); only B is
// staged, in `bstage` (S::B_STAGE_FLOATS floats).  K rows of As must exist.  Ends with a __syncthreads().
template <class S>
__device__ void gemm_smem_a(float (&acc)[S::TM][S::TN], const float* As_full, const BGlobal<S>& B, int K,
                            float* bstage) {
    const int tid = threadIdx.x;
    int ty, tx;
    gemm_coords(tid, ty, tx);
    float* const Bs0 = bstage;
    float rb[S::BP];
    B.fetch(0, tid, rb);
    B.store(Bs0, tid, rb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += S::KT) {
        const bool more = k0 + S::KT < K;
        if (more) B.fetch(k0 + S::KT, tid, rb);
        const int kn = K - k0 < S::KT ? K - k0 : S::KT;
        gemm_stage_mac<S, false>(acc, As_full + (int64_t)k0 * S::ALD, Bs0 + buf * S::KT * S::BN, ty, tx, kn);
        if (more) B.store(Bs0 + (buf ^ 1) * S::KT * S::BN, tid, rb);
        __syncthreads();
        buf ^= 1;
    }
}

}  // namespace cdclq
