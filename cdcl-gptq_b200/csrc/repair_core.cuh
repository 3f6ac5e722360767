// repair_core.cuh - the tile-level building blocks and the persistent kernels of phase 2 (the CDCL repair,
// src/engine.rs:478-671), templated on the row-tile height BM (64 or 128).  Each BM is instantiated in its own
// translation unit (repair_bm64.cu, repair_bm128.cu); repair.cu holds the statistics, mode A and dispatch.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "gemm_core.cuh"
#include "kernels.h"

namespace cdclq {

static __host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~(size_t)15; }

// ---------------------------------------------------------------------------------------------------------
// GEMM tiles of the repair: result widths 128 (group refit), 64 and 32 (sub-blocks), K stages of 16.  The
// staging buffers of a GEMM share shared memory with the tile that receives its result (the result is only
// written after the last stage has been consumed), which keeps two 128-row CTAs on one SM.
template <int BM>
struct RepairTiles {
    using W128 = Tile<BM, 128, 16>;
    using W64 = Tile<BM, 64, 16>;
    using W32 = Tile<BM, 32, 16>;
    static constexpr int LD = BM + 4;    // [col][row] GEMM result tiles (16-byte aligned rows)
    static constexpr int CSLD = BM + 4;  // [col][row] code tiles, bytes: consecutive columns start in distinct banks
    static constexpr int LDW = BM + 1;   // [col][row] W_hat tile: consecutive columns start in distinct banks
    // Coordinate descent: P = 256 / BM threads share a row, thread h updating gradient columns h, h + P, ...;
    // the gradient tile's column stride LDG = BM + BM/8 (= 32/P mod 32) puts the P threads of a row in
    // distinct banks.
    static constexpr int P = GEMM_THREADS / BM;
    static constexpr int LDG = BM + BM / 8;
    static_assert(LDG % 4 == 0 && (LDG % 32) * P == 32, "gradient stride");
    static constexpr int STAGE_FLOATS = W128::STAGE_FLOATS > W64::STAGE_FLOATS
                                            ? (W128::STAGE_FLOATS > W32::STAGE_FLOATS ? W128::STAGE_FLOATS
                                                                                      : W32::STAGE_FLOATS)
                                            : (W64::STAGE_FLOATS > W32::STAGE_FLOATS ? W64::STAGE_FLOATS
                                                                                     : W32::STAGE_FLOATS);
    static_assert(W128::ALD == LD && W64::ALD == LD && W32::ALD == LD, "result tiles share the A stride");
};

// A operand of the u H_CC product: A[k][row] = codes[k][row] - z[row] (src/engine.rs:553-558), staged from the
// shared-memory code tile.  The code tile is k-major ([K][BM] bytes) like the A stage, so a thread converts
// AP consecutive rows of one k and stores them with one vector store.
template <class S>
struct ACodes {
    const uint8_t* cs;  // [K][BM + 4]
    const float* zr;    // [BM], 16-byte aligned
    int rows_valid;
    int K;
    static constexpr int TPR = S::BM / S::AP;  // threads per k row
    static constexpr int LDC = S::BM + 4;
    static_assert(S::AP % 4 == 0, "code rows are converted four at a time");
    __device__ __forceinline__ void fetch(int k0, int tid, float (&r)[S::AP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::AP, k = k0 + kr;
#pragma unroll
        for (int v = 0; v < S::AP / 4; v++) {
            uchar4 q = make_uchar4(0, 0, 0, 0);
            if (k < K) q = *reinterpret_cast<const uchar4*>(cs + k * LDC + c + 4 * v);
            const int b = c + 4 * v;
            const float4 z = *reinterpret_cast<const float4*>(zr + b);
            r[4 * v] = (k < K && b < rows_valid) ? __fsub_rn((float)q.x, z.x) : 0.0f;
            r[4 * v + 1] = (k < K && b + 1 < rows_valid) ? __fsub_rn((float)q.y, z.y) : 0.0f;
            r[4 * v + 2] = (k < K && b + 2 < rows_valid) ? __fsub_rn((float)q.z, z.z) : 0.0f;
            r[4 * v + 3] = (k < K && b + 3 < rows_valid) ? __fsub_rn((float)q.w, z.w) : 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* As, int tid, const float (&r)[S::AP]) const {
        const int kr = tid / TPR, c = (tid % TPR) * S::AP;
#pragma unroll
        for (int v = 0; v < S::AP / 4; v++)
            *reinterpret_cast<float4*>(As + kr * S::ALD + ((c + 4 * v) ^ S::a_swz(kr))) =
                make_float4(r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3]);
    }
};

// The A operand of a repair GEMM: the error rows E (global) or the centred codes (shared memory).
struct AFromE {
    const float* e;
    int64_t lde;
    int rows_valid;
    int K;
    bool vec;
    template <class S>
    __device__ __forceinline__ AGlobal<S> make() const { return AGlobal<S>{e, lde, rows_valid, K, vec}; }
};
struct AFromCodes {
    const uint8_t* cs;
    const float* zr;
    int rows_valid;
    int K;
    template <class S>
    __device__ __forceinline__ ACodes<S> make() const { return ACodes<S>{cs, zr, rows_valid, K}; }
};

template <class S, class AM>
__device__ __forceinline__ void gemm_to_tile_s(const AM& am, const float* b, int64_t ldb, int64_t col0, int wd,
                                               int K, float* out, int ldo, float* stage) {
    int ty, tx;
    gemm_coords(threadIdx.x, ty, tx);
    float acc[S::TM][S::TN];
#pragma unroll
    for (int i = 0; i < S::TM; i++)
#pragma unroll
        for (int j = 0; j < S::TN; j++) acc[i][j] = 0.0f;
    const auto A = am.template make<S>();
    BGlobal<S> Bop{b, ldb, col0, wd, K, (ldb % 4 == 0) && (col0 % 4 == 0)};
    gemm_loader_a<S>(acc, A, Bop, K, stage);
#pragma unroll
    for (int j = 0; j < S::TN; j++) {
        const int cc = TileMap<S>::col(tx, j);
        if (cc < wd) {
#pragma unroll
            for (int v = 0; v < S::TM / 4; v++)
                *reinterpret_cast<float4*>(out + cc * ldo + TileMap<S>::row(ty, 4 * v)) =
                    make_float4(acc[4 * v][j], acc[4 * v + 1][j], acc[4 * v + 2][j], acc[4 * v + 3][j]);
        }
    }
}

// out[c * ldo + row] = (A B)[row][c] for c < wd (wd <= 128), B = b[k][col0 + c], via the narrowest fitting
// tile; ldo is a multiple of 4.  Ends synchronised.
template <int BM, class AM>
__device__ void gemm_to_tile(const AM& am, const float* b, int64_t ldb, int64_t col0, int wd, int K, float* out,
                             int ldo, float* stage) {
    using RT = RepairTiles<BM>;
    if (wd > 64)
        gemm_to_tile_s<typename RT::W128>(am, b, ldb, col0, wd, K, out, ldo, stage);
    else if (wd > 32)
        gemm_to_tile_s<typename RT::W64>(am, b, ldb, col0, wd, K, out, ldo, stage);
    else
        gemm_to_tile_s<typename RT::W32>(am, b, ldb, col0, wd, K, out, ldo, stage);
    __syncthreads();
}

// Column split of the repair GEMMs between the two CTAs of a row tile in a 4-CTA cluster (cluster ranks 2 t + ch,
// t the row tile, ch the column half): CTA ch computes half of a result tile's columns and writes them into its
// partner's copy of the tile through distributed shared memory, so both hold the whole result; everything after
// the GEMMs (the per-row refit, the coordinate sweeps) runs identically in both CTAs, but only ch = 0 writes
// global memory (E, W_hat, codes, scales), and cluster barriers order those writes before the partner's next
// reads.  Each element of a result keeps its single accumulation order, so results are those of one CTA.
struct ColSplit {
    int ch;       // -1: no split (the whole tile in this CTA); 0 / 1: the column half this CTA computes
    int partner;  // cluster rank of the CTA holding the other half
    __device__ __forceinline__ bool writes() const { return ch == 0; }
};

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// gemm_to_tile, split by columns between the CTAs of a ColSplit pair (ends with the whole tile in both).
template <int BM, bool SPLIT, class AM>
__device__ void gemm_to_tile_cs(const AM& am, const float* b, int64_t ldb, int64_t col0, int wd, int K, float* out,
                                int ldo, float* stage, const ColSplit& cs) {
    if constexpr (!SPLIT) {
        gemm_to_tile<BM>(am, b, ldb, col0, wd, K, out, ldo, stage);
        return;
    }
    namespace cg = cooperative_groups;
    const int h0 = min(wd, ((wd + 1) / 2 + 3) & ~3);  // columns of half 0
    const int c_begin = cs.ch == 0 ? 0 : h0, c_count = cs.ch == 0 ? h0 : wd - h0;
    cluster_sync_all();  // the partner's global writes before this GEMM (E rows) are visible
    if (c_count > 0) gemm_to_tile<BM>(am, b, ldb, col0 + c_begin, c_count, K, out + (size_t)c_begin * ldo, ldo, stage);
    cluster_sync_all();  // both halves computed; neither CTA still reads its staging area (inside `out`)
    float* peer = cg::this_cluster().map_shared_rank(out, cs.partner);
    constexpr int Q = BM / 4;
    for (int idx = threadIdx.x; idx < c_count * Q; idx += blockDim.x) {
        const int c = idx / Q, r4 = (idx - c * Q) * 4;
        const size_t o = (size_t)(c_begin + c) * ldo + r4;
        *reinterpret_cast<float4*>(peer + o) = *reinterpret_cast<const float4*>(out + o);
    }
    cluster_sync_all();  // the partner's half has arrived
}

// Tile staging between the row-major global matrices and the [col][row] shared-memory tiles.  A thread moves
// one column of four consecutive rows: its global accesses are coalesced across the warp (consecutive
// columns), and its shared-memory word lands in a distinct bank per column (strides CSLD / LDW).  Each thread
// takes STAGE_U such items at a time and issues all their global loads before its shared-memory stores, so
// the loads of a pass are in flight together.
constexpr int STAGE_U = 4;

template <int BM>
__device__ __forceinline__ void stage_codes(uint8_t* cs, const uint8_t* codes, int64_t n, int c0, int rs, int wd) {
    constexpr int CSLD = RepairTiles<BM>::CSLD;
    const int total = ((rs + 3) >> 2) * wd;
    for (int base = threadIdx.x; base < total; base += STAGE_U * blockDim.x) {
        uint32_t word[STAGE_U];
#pragma unroll
        for (int u = 0; u < STAGE_U; u++) {
            const int idx = base + u * blockDim.x;
            word[u] = 0;
            if (idx < total) {
                const int q = idx / wd, k = idx - q * wd, r = 4 * q;
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (r + i < rs) word[u] |= (uint32_t)codes[(int64_t)(r + i) * n + c0 + k] << (8 * i);
            }
        }
#pragma unroll
        for (int u = 0; u < STAGE_U; u++) {
            const int idx = base + u * blockDim.x;
            if (idx < total) {
                const int q = idx / wd, k = idx - q * wd;
                *reinterpret_cast<uint32_t*>(cs + k * CSLD + 4 * q) = word[u];
            }
        }
    }
}

template <int BM>
__device__ __forceinline__ void stage_cd_tiles(uint8_t* cs, float* wqs, const uint8_t* codes, const float* wq,
                                               int64_t n, int c0, int rs, int wd) {
    constexpr int CSLD = RepairTiles<BM>::CSLD, LDW = RepairTiles<BM>::LDW;
    const int total = ((rs + 3) >> 2) * wd;
    for (int base = threadIdx.x; base < total; base += STAGE_U * blockDim.x) {
        uint32_t word[STAGE_U];
        float v[STAGE_U][4];
#pragma unroll
        for (int u = 0; u < STAGE_U; u++) {
            const int idx = base + u * blockDim.x;
            word[u] = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) v[u][i] = 0.0f;
            if (idx < total) {
                const int q = idx / wd, k = idx - q * wd, r = 4 * q;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (r + i < rs) {
                        const int64_t off = (int64_t)(r + i) * n + c0 + k;
                        word[u] |= (uint32_t)codes[off] << (8 * i);
                        v[u][i] = wq[off];
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < STAGE_U; u++) {
            const int idx = base + u * blockDim.x;
            if (idx < total) {
                const int q = idx / wd, k = idx - q * wd, r = 4 * q;
#pragma unroll
                for (int i = 0; i < 4; i++)
                    if (r + i < rs) wqs[k * LDW + r + i] = v[u][i];
                *reinterpret_cast<uint32_t*>(cs + k * CSLD + r) = word[u];
            }
        }
    }
}

template <int BM>
__device__ __forceinline__ void unstage_cd_tiles(const uint8_t* cs, const float* wqs, uint8_t* codes, float* wq,
                                                 int64_t n, int c0, int rs, int wd) {
    constexpr int CSLD = RepairTiles<BM>::CSLD, LDW = RepairTiles<BM>::LDW;
    const int quads = (rs + 3) >> 2;
    for (int idx = threadIdx.x; idx < quads * wd; idx += blockDim.x) {
        const int q = idx / wd, k = idx - q * wd, r = 4 * q;
        const uint32_t word = *reinterpret_cast<const uint32_t*>(cs + k * CSLD + r);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (r + i < rs) {
                const int64_t off = (int64_t)(r + i) * n + c0 + k;
                codes[off] = (uint8_t)(word >> (8 * i));
                wq[off] = wqs[k * LDW + r + i];
            }
        }
    }
}

// Shared-memory layout of the repair kernels: a body shared by the refit (group code tile + one 128-column
// result tile, which also holds the GEMM staging buffers) and the coordinate descent (sub-block code tile,
// gradient tile - holding the staging buffers too when the sub-block is one GEMM tile wide -, W_hat tile and
// the sub-block Hessian), then per-row scalars.
constexpr int HSS_MAX_BYTES = 16384;  // sub-blocks up to 64 columns keep their whole Hessian block on chip

struct RepairLayout {
    size_t refit_tile, cd_gt, cd_stage, cd_wqs, cd_hss;  // body offsets
    size_t body, zrow, snew, accept, rowdelta, upd, total;
};

static __host__ __device__ inline size_t cd_hss_bytes(int sbw) {
    size_t full = (size_t)sbw * sbw * 4;
    return full <= (size_t)HSS_MAX_BYTES ? al16(full) : al16((size_t)sbw * 4);
}

template <int BM>
static __host__ __device__ inline RepairLayout repair_layout(int g, int sbw) {
    constexpr int LD = RepairTiles<BM>::LD, CSLD = RepairTiles<BM>::CSLD, LDW = RepairTiles<BM>::LDW;
    constexpr size_t STAGE = (size_t)RepairTiles<BM>::STAGE_FLOATS * 4;
    static_assert((size_t)128 * LD * 4 >= STAGE, "the refit result tile holds the staging buffers");
    RepairLayout L;
    size_t gcap = (size_t)(g < 1024 ? g : 1024);
    L.refit_tile = al16(gcap * CSLD);
    size_t refit = L.refit_tile + al16((size_t)128 * LD * 4);
    L.cd_gt = al16((size_t)sbw * CSLD);
    size_t gt_bytes = al16((size_t)sbw * RepairTiles<BM>::LDG * 4);
    if (sbw <= 128) {  // one GEMM tile: staging inside the gradient tile
        L.cd_stage = L.cd_gt;
        L.cd_wqs = L.cd_gt + (gt_bytes > STAGE ? gt_bytes : al16(STAGE));
    } else {  // several GEMM tiles fill the gradient tile one after the other: separate staging
        L.cd_stage = L.cd_gt + gt_bytes;
        L.cd_wqs = L.cd_stage + al16(STAGE);
    }
    L.cd_hss = L.cd_wqs + al16((size_t)sbw * LDW * 4);
    size_t cd = L.cd_hss + cd_hss_bytes(sbw);
    L.body = refit > cd ? refit : cd;
    L.zrow = L.body;
    L.snew = L.zrow + BM * 4;
    L.accept = L.snew + BM * 4;
    L.rowdelta = L.accept + BM * 4;
    L.upd = L.rowdelta + BM * 8;
    L.total = L.upd + BM * 8;
    return L;
}


struct TileSmem {
    unsigned char* body;
    float* refit_tile;  // [128][LD] (+ staging)
    float* cd_gt;       // [sbw][LD]
    float* cd_stage;
    float* cd_wqs;      // [sbw][LDW]
    float* cd_hss;
    float* zrow;
    float* snew;
    int* accept;
    double* rowdelta;
    unsigned long long* rowupd;
};

template <int BM>
__device__ __forceinline__ TileSmem tile_smem(unsigned char* raw, int g, int sbw) {
    const RepairLayout L = repair_layout<BM>(g, sbw);
    TileSmem t;
    t.body = raw;
    t.refit_tile = reinterpret_cast<float*>(raw + L.refit_tile);
    t.cd_gt = reinterpret_cast<float*>(raw + L.cd_gt);
    t.cd_stage = reinterpret_cast<float*>(raw + L.cd_stage);
    t.cd_wqs = reinterpret_cast<float*>(raw + L.cd_wqs);
    t.cd_hss = reinterpret_cast<float*>(raw + L.cd_hss);
    t.zrow = reinterpret_cast<float*>(raw + L.zrow);
    t.snew = reinterpret_cast<float*>(raw + L.snew);
    t.accept = reinterpret_cast<int*>(raw + L.accept);
    t.rowdelta = reinterpret_cast<double*>(raw + L.rowdelta);
    t.rowupd = reinterpret_cast<unsigned long long*>(raw + L.upd);
    return t;
}

// ---------------------------------------------------------------------------------------------------------
// Closed-form scale refit of every (row, group) of the rows [r0, r0 + rs) of a chunk, groups in order
// (src/engine.rs:534-589).  Thread r < rs accumulates its row's accepted loss deltas and refits.
template <int BM, bool SPLIT = false>
__device__ void refit_tile(const ChunkInfo& ci, int r0, int rs, const TileSmem& sm, double& my_delta,
                           unsigned long long& my_upd, const ColSplit& split) {
    const bool writer = !SPLIT || split.writes();  // the CTA that writes global memory
    constexpr int LD = RepairTiles<BM>::LD, CSLD = RepairTiles<BM>::CSLD;
    const int tid = threadIdx.x, n = ci.n, g = ci.g, ng = ci.ng;
    float* E = ci.e + (int64_t)r0 * n;
    float* WQ = ci.wq + (int64_t)r0 * n;
    const uint8_t* CODES = ci.codes + (int64_t)r0 * n;
    float* SC = ci.scales + (int64_t)r0 * ng;
    const float* ZR = ci.zeros + (int64_t)r0 * ng;
    const float* H = ci.h;
    uint8_t* cs = sm.body;        // [gcap][CSLD] codes of the group
    float* tile = sm.refit_tile;  // [128][LD] G, then u H_CC; also the GEMM staging buffers
    for (int gi = 0; gi < ng; gi++) {
        const int c0 = gi * g, wd = min(g, n - c0);
        stage_codes<BM>(cs, CODES, n, c0, rs, wd);
        if (tid < BM) sm.zrow[tid] = (tid < rs) ? ZR[(int64_t)tid * ng + gi] : 0.0f;
        // the group's current scale, read before the GEMMs: with a column split the partner CTA writes the new
        // scale once both have passed the GEMMs' cluster barriers
        const float s_old = (tid < rs) ? SC[(int64_t)tid * ng + gi] : 0.0f;
        __syncthreads();
        // num = sum_k u_k * G_k with G = E H[:, c0:c1]
        float num = 0.0f, den = 0.0f;
        for (int t0 = 0; t0 < wd; t0 += 128) {
            int wt = min(128, wd - t0);
            gemm_to_tile_cs<BM, SPLIT>(AFromE{E, (int64_t)n, rs, n, (n % 4 == 0)}, H, (int64_t)n, (int64_t)(c0 + t0), wt, n,
                                tile, LD, tile, split);
            if (tid < rs) {
                const float zr = sm.zrow[tid];
                for (int k = 0; k < wt; k++) {
                    float u = __fsub_rn((float)cs[(t0 + k) * CSLD + tid], zr);
                    num = __fadd_rn(num, __fmul_rn(u, tile[k * LD + tid]));
                }
            }
            __syncthreads();
        }
        // den = sum_k u_k * (u H_CC)_k
        for (int t0 = 0; t0 < wd; t0 += 128) {
            int wt = min(128, wd - t0);
            gemm_to_tile_cs<BM, SPLIT>(AFromCodes{cs, sm.zrow, rs, wd}, H + (int64_t)c0 * n, (int64_t)n, (int64_t)(c0 + t0),
                                wt, wd, tile, LD, tile, split);
            if (tid < rs) {
                const float zr = sm.zrow[tid];
                for (int k = 0; k < wt; k++) {
                    float u = __fsub_rn((float)cs[(t0 + k) * CSLD + tid], zr);
                    den = __fadd_rn(den, __fmul_rn(u, tile[k * LD + tid]));
                }
            }
            __syncthreads();
        }
        if (tid < BM) sm.accept[tid] = 0;
        if (tid < rs && den > 1e-30f) {
            float s_new = round_f16(__fadd_rn(s_old, __fdiv_rn(num, den)));
            if (!(s_new >= kF16MinNormal)) s_new = kF16MinNormal;  // f32::max(x, MIN)
            const float d = __fsub_rn(s_new, s_old);
            const float dlf = __fadd_rn(__fmul_rn(__fmul_rn(-2.0f, d), num), __fmul_rn(__fmul_rn(d, d), den));
            const double dl = (double)dlf;
            if (dl < 0.0) {
                if (writer) SC[(int64_t)tid * ng + gi] = s_new;
                sm.snew[tid] = s_new;
                sm.accept[tid] = 1;
                my_delta = __dadd_rn(my_delta, dl);
                my_upd++;
            }
        }
        __syncthreads();
        // accepted rows: W_hat = s_new * u and E += W_hat_old - W_hat_new over the group (loads batched)
        const int total = writer ? rs * wd : 0;
        for (int base = tid; base < total; base += STAGE_U * blockDim.x) {
            float ev[STAGE_U], wv[STAGE_U];
#pragma unroll
            for (int u = 0; u < STAGE_U; u++) {
                const int idx = base + u * blockDim.x;
                ev[u] = 0.0f;
                wv[u] = 0.0f;
                if (idx < total) {
                    const int rr = idx / wd, k = idx - rr * wd;
                    if (sm.accept[rr]) {
                        const int64_t off = (int64_t)rr * n + c0 + k;
                        ev[u] = E[off];
                        wv[u] = WQ[off];
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < STAGE_U; u++) {
                const int idx = base + u * blockDim.x;
                if (idx < total) {
                    const int rr = idx / wd, k = idx - rr * wd;
                    if (sm.accept[rr]) {
                        const float uc = __fsub_rn((float)cs[k * CSLD + rr], sm.zrow[rr]);
                        const float ndq = __fmul_rn(sm.snew[rr], uc);
                        const int64_t off = (int64_t)rr * n + c0 + k;
                        E[off] = __fadd_rn(ev[u], __fsub_rn(wv[u], ndq));
                        WQ[off] = ndq;
                    }
                }
            }
        }
        __syncthreads();
    }
}

// The rank-1 gradient update of one move, g[kk] += de * h(kk) for the columns kk = h0, h0 + P, ... < wd of one
// row (the thread's share): eight columns at a time, all loads issued before the stores, so a move costs a few
// shared-memory round trips instead of one per column.  Each element still receives one f32 multiply and add.
template <int P, int LD, class HF>
__device__ __forceinline__ void rank1_update(float* gt, int r, int h0, int wd, float de, HF hval) {
    constexpr int U = 8;
    for (int base = h0; base < wd; base += U * P) {
        float hv[U], gv[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int kk = base + u * P;
            hv[u] = kk < wd ? hval(kk) : 0.0f;
            gv[u] = kk < wd ? gt[kk * LD + r] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int kk = base + u * P;
            if (kk < wd) gt[kk * LD + r] = __fadd_rn(gv[u], __fmul_rn(de, hv[u]));
        }
    }
}

// Coordinate descent over the selected sub-blocks for rows [r0, r0 + rs) (src/engine.rs:600-658).
template <int BM, bool SPLIT = false>
__device__ void cd_tile(const ChunkInfo& ci, int r0, int rs, int cd_sweeps, const TileSmem& sm, double& my_delta,
                        unsigned long long& my_upd, const ColSplit& split) {
    const bool writer = !SPLIT || split.writes();  // the CTA that writes global memory
    constexpr int LD = RepairTiles<BM>::LDG, CSLD = RepairTiles<BM>::CSLD, LDW = RepairTiles<BM>::LDW;
    constexpr int P = RepairTiles<BM>::P;
    const int tid = threadIdx.x, n = ci.n, g = ci.g, ng = ci.ng, sbw = ci.sbw;
    float* E = ci.e + (int64_t)r0 * n;
    float* WQ = ci.wq + (int64_t)r0 * n;
    uint8_t* CODES = ci.codes + (int64_t)r0 * n;
    // sweep layout: P consecutive lanes share row r; lane h of the group owns gradient columns h, h+P, ...
    const int lane = tid & 31;
    const int r = (tid >> 5) * (32 / P) + lane / P, h = lane % P;
    const unsigned pmask = ((1u << P) - 1u) << (lane & ~(P - 1));
    // the row's loss bookkeeping moves to shared memory while the sweep threads own the rows
    __syncthreads();
    if (tid < BM) {
        sm.rowdelta[tid] = my_delta;
        sm.rowupd[tid] = my_upd;
    }
    const float* SC = ci.scales + (int64_t)r0 * ng;
    const float* ZR = ci.zeros + (int64_t)r0 * ng;
    const float* H = ci.h;
    const int n_sel = ci.st->n_sel;
    uint8_t* cs = sm.body;     // [sbw][CSLD]
    float* gt = sm.cd_gt;      // [sbw][LDG] block gradient
    float* wqs = sm.cd_wqs;    // [sbw][LDW] W_hat
    float* hss = sm.cd_hss;    // [sbw][sbw] or its diagonal
    const bool hss_full = (size_t)sbw * sbw * 4 <= (size_t)HSS_MAX_BYTES;
    for (int si = 0; si < n_sel; si++) {
        const int s = ci.sel[si];
        const int c0 = s * sbw, wd = min(sbw, n - c0);
        if (SPLIT) cluster_sync_all();  // the partner's codes / W_hat / E / scale writes are visible
        stage_cd_tiles<BM>(cs, wqs, CODES, WQ, n, c0, rs, wd);
        if (hss_full) {
            for (int base = tid; base < wd * wd; base += STAGE_U * blockDim.x) {
                float hv[STAGE_U];
#pragma unroll
                for (int u = 0; u < STAGE_U; u++) {
                    const int idx = base + u * blockDim.x, a = idx / wd, b = idx - a * wd;
                    hv[u] = idx < wd * wd ? __ldg(H + (int64_t)(c0 + a) * n + c0 + b) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < STAGE_U; u++)
                    if (base + u * blockDim.x < wd * wd) hss[base + u * blockDim.x] = hv[u];
            }
        } else {
            for (int a = tid; a < wd; a += blockDim.x) hss[a] = __ldg(H + (int64_t)(c0 + a) * n + c0 + a);
        }
        for (int t0 = 0; t0 < wd; t0 += 128) {
            int wt = min(128, wd - t0);
            gemm_to_tile_cs<BM, SPLIT>(AFromE{E, (int64_t)n, rs, n, (n % 4 == 0)}, H, (int64_t)n, (int64_t)(c0 + t0), wt, n,
                                gt + (size_t)t0 * LD, LD, sm.cd_stage, split);
        }
        if (r < rs) {
            // The P threads of a row take every decision together (identical inputs, identical results) and
            // split each rank-1 gradient update; thread h = 0 writes the row's state and keeps its bookkeeping.
            double row_delta = h == 0 ? sm.rowdelta[r] : 0.0;
            unsigned long long row_upd = 0ull;
            for (int sw = 0; sw < cd_sweeps; sw++) {
                bool changed = false;
                int cur_gi = -1;
                float sc = 1.0f, z = 0.0f, maxq = 1.0f;
                for (int jj = 0; jj < wd; jj++) {
                    const int j = c0 + jj;
                    const int gi = j / g;
                    if (gi != cur_gi) {
                        cur_gi = gi;
                        maxq = (float)((1u << ci.gbits[gi]) - 1u);
                        sc = SC[(int64_t)r * ng + gi];
                        z = ZR[(int64_t)r * ng + gi];
                    }
                    const float hjj = hss_full ? hss[jj * wd + jj] : hss[jj];
                    const float cur = wqs[jj * LDW + r];
                    const float gj = gt[jj * LD + r];
                    // most steps keep their code: prove it without the two divisions (identical inputs in the
                    // row's P threads, so they skip together; nothing shared changes, so no warp sync)
                    if (cd_keeps_code(gj, hjj, cur, sc, __fsub_rn((float)cs[jj * CSLD + r], z))) continue;
                    const float target = __fadd_rn(cur, __fdiv_rn(gj, hjj));
                    float q = __fadd_rn(roundf(__fdiv_rn(target, sc)), z);
                    if (q < 0.0f) q = 0.0f;
                    if (q > maxq) q = maxq;
                    const float newdq = __fmul_rn(sc, __fsub_rn(q, z));
                    const uint8_t qc = (q == q) ? (uint8_t)q : (uint8_t)0;
                    if (qc != cs[jj * CSLD + r]) {
                        // closed-form loss change, then the rank-1 gradient update (src/engine.rs:634-650)
                        const float de = __fsub_rn(cur, newdq);
                        if (h == 0) {
                            const float t1 = __fmul_rn(__fmul_rn(2.0f, de), gj);
                            const float t2 = __fmul_rn(__fmul_rn(de, de), hjj);
                            row_delta = __dadd_rn(row_delta, (double)__fadd_rn(t1, t2));
                        }
                        if (hss_full)
                            rank1_update<P, LD>(gt, r, h, wd, de, [&](int kk) { return hss[jj * wd + kk]; });
                        else
                            rank1_update<P, LD>(gt, r, h, wd, de,
                                                [&](int kk) { return __ldg(H + (int64_t)j * n + c0 + kk); });
                        // every thread of the row has read column jj's code and W_hat before they change
                        __syncwarp(pmask);
                        if (h == 0) {
                            wqs[jj * LDW + r] = newdq;
                            cs[jj * CSLD + r] = qc;
                            if (writer) {
                                float* ep = &E[(int64_t)r * n + j];
                                *ep = __fadd_rn(*ep, de);
                            }
                            row_upd++;
                        }
                        changed = true;
                    }
                    __syncwarp(pmask);  // this column's updates are visible to the row's next decision
                }
                if (!changed) break;
            }
            if (h == 0) {
                sm.rowdelta[r] = row_delta;
                sm.rowupd[r] += row_upd;
            }
        }
        __syncthreads();
        if (writer) unstage_cd_tiles<BM>(cs, wqs, CODES, WQ, n, c0, rs, wd);
        __syncthreads();
    }
    if (tid < BM) {
        my_delta = sm.rowdelta[tid];
        my_upd = sm.rowupd[tid];
    }
}

// Sum of the tile's per-row results, rows in order; valid in thread 0.  Ends synchronised.
template <int BM>
__device__ __forceinline__ void tile_reduce(int rs, const TileSmem& sm, double my_delta, unsigned long long my_upd,
                                            double& d, unsigned long long& u) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid < BM) {
        sm.rowdelta[tid] = (tid < rs) ? my_delta : 0.0;
        sm.rowupd[tid] = (tid < rs) ? my_upd : 0ull;
    }
    __syncthreads();
    d = 0.0;
    u = 0ull;
    if (tid == 0) {
        for (int r = 0; r < rs; r++) {
            d = __dadd_rn(d, sm.rowdelta[r]);
            u += sm.rowupd[r];
        }
    }
    __syncthreads();
}

// One tile of one pass (refit then coordinate descent, or the final refit alone); the tile's delta and
// update count are valid in thread 0.
template <int BM, bool SPLIT = false>
__device__ __forceinline__ void run_tile(const ChunkInfo& ci, int r0, int rs, const RepairParams& rp, bool final_refit,
                                         const TileSmem& sm, double& d, unsigned long long& u,
                                         const ColSplit& split = ColSplit{-1, 0}) {
    double my_delta = 0.0;
    unsigned long long my_upd = 0ull;
    if (rp.do_refit) refit_tile<BM, SPLIT>(ci, r0, rs, sm, my_delta, my_upd, split);
    if (rp.do_cd && !final_refit) cd_tile<BM, SPLIT>(ci, r0, rs, rp.cd_sweeps, sm, my_delta, my_upd, split);
    tile_reduce<BM>(rs, sm, my_delta, my_upd, d, u);
}

// The reference's stop rule after a pass (src/engine.rs:660-665), in thread 0 / one thread.
__device__ __forceinline__ void apply_pass(ChunkState* st, double pass_delta, unsigned long long pass_upd, double tol) {
    st->loss_delta = __dadd_rn(st->loss_delta, pass_delta);
    st->updates += pass_upd;
    st->passes += 1;
    const double gain = __dsub_rn(st->prev_delta, st->loss_delta);
    st->prev_delta = st->loss_delta;
    if (pass_upd == 0ull || gain < tol * __dadd_rn(st->loss_gptq, st->loss_delta)) st->done = 1;
}


template <int BM>
__global__ void __launch_bounds__(256, 2) repair_persistent_kernel(const ChunkInfo* __restrict__ chunks, int nchunks,
                                                                   RepairParams rp, int* __restrict__ counter) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int s_chunk, s_done;
    __shared__ ChunkInfo ci;  // chunk descriptor kept on chip (not in registers across the tile loops)
    const int tid = threadIdx.x;
    for (;;) {
        if (tid == 0) {
            s_chunk = atomicAdd(counter, 1);
            if (s_chunk < nchunks) ci = chunks[s_chunk];
        }
        __syncthreads();
        const int c = s_chunk;
        if (c >= nchunks) return;
        ChunkState* st = ci.st;
        const TileSmem sm = tile_smem<BM>(smem_raw, ci.g, ci.sbw);
        if (tid == 0) s_done = st->done;
        __syncthreads();
        for (int pass = 0; pass < rp.max_passes && !s_done; pass++) {
            double pd = 0.0;
            unsigned long long pu = 0ull;
            for (int r0 = 0; r0 < ci.rows; r0 += BM) {
                double d;
                unsigned long long u;
                run_tile<BM>(ci, r0, min(BM, ci.rows - r0), rp, false, sm, d, u);
                if (tid == 0) {
                    pd = __dadd_rn(pd, d);
                    pu += u;
                }
            }
            if (tid == 0) {
                apply_pass(st, pd, pu, rp.tol);
                s_done = st->done;
            }
            __syncthreads();
        }
        if (rp.do_refit) {  // final refit (src/engine.rs:668-670)
            double fd = 0.0;
            unsigned long long fu = 0ull;
            for (int r0 = 0; r0 < ci.rows; r0 += BM) {
                double d;
                unsigned long long u;
                run_tile<BM>(ci, r0, min(BM, ci.rows - r0), rp, true, sm, d, u);
                if (tid == 0) {
                    fd = __dadd_rn(fd, d);
                    fu += u;
                }
            }
            if (tid == 0) {
                st->loss_delta = __dadd_rn(st->loss_delta, fd);
                st->updates += fu;
            }
        }
        __syncthreads();
    }
}

// Mode C - persistent clusters: a cluster of 2 CTAs takes a whole row chunk of several tiles (heaviest first);
// CTA rank r handles the chunk's tiles r, r+2, ...  A row chunk's passes are the latency-critical unit, and
// splitting its rows over two SMs halves that critical path.  At the end of each pass the tiles' partial sums
// are written into rank 0's shared memory (distributed shared memory), rank 0 adds them in tile order - the
// order of mode B - applies the stop rule and writes the decision back into rank 1; hardware cluster barriers
// order these steps.

constexpr int RP_MAX_TILES = RP_MAX_TILES_PER_CHUNK;

template <int BM>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 2)
    repair_cluster_kernel(const ChunkInfo* __restrict__ chunks, int nchunks, RepairParams rp, int* __restrict__ counter) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int s_chunk, s_done;
    __shared__ ChunkInfo ci;
    __shared__ double s_tile_delta[RP_MAX_TILES];
    __shared__ unsigned long long s_tile_upd[RP_MAX_TILES];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int tid = threadIdx.x;
    int* chunk0 = cluster.map_shared_rank(&s_chunk, 0);
    int* done1 = cluster.map_shared_rank(&s_done, 1);
    double* tdelta0 = cluster.map_shared_rank(&s_tile_delta[0], 0);
    unsigned long long* tupd0 = cluster.map_shared_rank(&s_tile_upd[0], 0);
    for (;;) {
        if (rank == 0 && tid == 0) s_chunk = atomicAdd(counter, 1);
        cluster.sync();
        const int c = *chunk0;
        if (tid == 0 && c < nchunks) ci = chunks[c];
        cluster.sync();  // every rank has read rank 0's s_chunk before anyone may leave or overwrite it
        if (c >= nchunks) return;
        ChunkState* st = ci.st;
        const TileSmem sm = tile_smem<BM>(smem_raw, ci.g, ci.sbw);
        const int ntiles = (ci.rows + BM - 1) / BM;
        if (tid == 0) s_done = st->done;
        __syncthreads();
        for (int pass = 0; pass < rp.max_passes && !s_done; pass++) {
            for (int t = rank; t < ntiles; t += 2) {
                const int r0 = t * BM;
                double d;
                unsigned long long u;
                run_tile<BM>(ci, r0, min(BM, ci.rows - r0), rp, false, sm, d, u);
                if (tid == 0) {
                    tdelta0[t] = d;
                    tupd0[t] = u;
                }
            }
            cluster.sync();  // all tile partials are in rank 0
            if (rank == 0 && tid == 0) {
                double pd = 0.0;
                unsigned long long pu = 0ull;
                for (int t = 0; t < ntiles; t++) {
                    pd = __dadd_rn(pd, s_tile_delta[t]);
                    pu += s_tile_upd[t];
                }
                apply_pass(st, pd, pu, rp.tol);
                s_done = st->done;
                *done1 = st->done;
            }
            cluster.sync();  // the decision is visible in both ranks
        }
        if (rp.do_refit) {  // final refit (src/engine.rs:668-670)
            for (int t = rank; t < ntiles; t += 2) {
                const int r0 = t * BM;
                double d;
                unsigned long long u;
                run_tile<BM>(ci, r0, min(BM, ci.rows - r0), rp, true, sm, d, u);
                if (tid == 0) {
                    tdelta0[t] = d;
                    tupd0[t] = u;
                }
            }
            cluster.sync();
            if (rank == 0 && tid == 0) {
                double fd = 0.0;
                unsigned long long fu = 0ull;
                for (int t = 0; t < ntiles; t++) {
                    fd = __dadd_rn(fd, s_tile_delta[t]);
                    fu += s_tile_upd[t];
                }
                st->loss_delta = __dadd_rn(st->loss_delta, fd);
                st->updates += fu;
            }
        }
        __syncthreads();
    }
}


// Mode Q - persistent 4-CTA clusters for chunks of exactly two row tiles: cluster rank 2 t + ch runs row tile t with
// column half ch of every repair GEMM (ColSplit); the ch = 0 CTAs report their tile's partial sums to rank 0, which
// applies the stop rule in tile order and writes the decision into the other three ranks.  The heaviest chunks
// (the widest layers' rows, whose passes are the longest sequential chains of a rank's repair) get four SMs.
template <int BM>
__global__ void __cluster_dims__(4, 1, 1) __launch_bounds__(256, 1)
    repair_quad_kernel(const ChunkInfo* __restrict__ chunks, int nchunks, RepairParams rp, int* __restrict__ counter) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ int s_chunk, s_done;
    __shared__ ChunkInfo ci;
    __shared__ double s_tile_delta[2];
    __shared__ unsigned long long s_tile_upd[2];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int t = rank >> 1;  // row tile
    const ColSplit split{rank & 1, rank ^ 1};
    const int tid = threadIdx.x;
    int* chunk0 = cluster.map_shared_rank(&s_chunk, 0);
    double* tdelta0 = cluster.map_shared_rank(&s_tile_delta[0], 0);
    unsigned long long* tupd0 = cluster.map_shared_rank(&s_tile_upd[0], 0);
    for (;;) {
        if (rank == 0 && tid == 0) s_chunk = atomicAdd(counter, 1);
        cluster.sync();
        const int c = *chunk0;
        if (tid == 0 && c < nchunks) ci = chunks[c];
        cluster.sync();  // every rank has read rank 0's s_chunk before anyone may leave or overwrite it
        if (c >= nchunks) return;
        ChunkState* st = ci.st;
        const TileSmem sm = tile_smem<BM>(smem_raw, ci.g, ci.sbw);
        if (tid == 0) s_done = st->done;
        __syncthreads();
        const int r0 = t * BM, rs = min(BM, ci.rows - r0);  // the host gives this kernel two-tile chunks only
        for (int pass = 0; pass < rp.max_passes && !s_done; pass++) {
            double d;
            unsigned long long u;
            run_tile<BM, true>(ci, r0, rs, rp, false, sm, d, u, split);
            if (tid == 0 && split.ch == 0) {
                tdelta0[t] = d;
                tupd0[t] = u;
            }
            cluster.sync();  // both tiles' partials are in rank 0; every global write of the pass is visible
            if (rank == 0 && tid == 0) {
                apply_pass(st, __dadd_rn(__dadd_rn(0.0, s_tile_delta[0]), s_tile_delta[1]), s_tile_upd[0] + s_tile_upd[1],
                           rp.tol);
                for (int q = 0; q < 4; q++) *cluster.map_shared_rank(&s_done, q) = st->done;
            }
            cluster.sync();  // the decision is visible in every rank
        }
        if (rp.do_refit) {  // final refit (src/engine.rs:668-670)
            double d;
            unsigned long long u;
            run_tile<BM, true>(ci, r0, rs, rp, true, sm, d, u, split);
            if (tid == 0 && split.ch == 0) {
                tdelta0[t] = d;
                tupd0[t] = u;
            }
            cluster.sync();
            if (rank == 0 && tid == 0) {
                st->loss_delta = __dadd_rn(st->loss_delta, __dadd_rn(__dadd_rn(0.0, s_tile_delta[0]), s_tile_delta[1]));
                st->updates += s_tile_upd[0] + s_tile_upd[1];
            }
        }
        cluster.sync();  // the chunk's last global writes and rank 0's bookkeeping precede the next chunk
    }
}

static inline int set_repair_smem(const void* fn, size_t smem) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return e == cudaSuccess ? 0 : cuda_error(e, "repair smem attribute");
}

static inline int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

// max_ctas > 0 caps the grid (the launch then shares the GPU with another one).
template <int BM>
static int launch_cluster_bm(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                             int* counter_dev, cudaStream_t st, int max_ctas = 0) {
    int rc = set_repair_smem((const void*)repair_cluster_kernel<BM>, smem);
    if (rc) return rc;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, repair_cluster_kernel<BM>, 256, smem);
    if (per_sm < 1) per_sm = 1;
    int clusters = sm_count() * per_sm / 2;
    if (max_ctas > 0 && clusters > max_ctas / 2) clusters = max_ctas / 2;
    if (clusters > nchunks) clusters = nchunks;
    if (clusters < 1) clusters = 1;
    CDCLQ_CUDA_TRY(cudaMemsetAsync(counter_dev, 0, sizeof(int), st));
    CDCLQ_LAUNCH(repair_cluster_kernel<BM>, 2 * clusters, 256, smem, st, chunks_dev, nchunks, rp, counter_dev);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "repair_cluster_kernel launch");
}

template <int BM>
static int launch_quad_bm(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                          int* counter_dev, cudaStream_t st, int max_ctas) {
    int rc = set_repair_smem((const void*)repair_quad_kernel<BM>, smem);
    if (rc) return rc;
    int quads = max_ctas / 4;
    if (quads > nchunks) quads = nchunks;
    if (quads < 1) quads = 1;
    CDCLQ_CUDA_TRY(cudaMemsetAsync(counter_dev, 0, sizeof(int), st));
    CDCLQ_LAUNCH(repair_quad_kernel<BM>, 4 * quads, 256, smem, st, chunks_dev, nchunks, rp, counter_dev);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "repair_quad_kernel launch");
}

template <int BM>
static int launch_persistent_bm(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                int* counter_dev, cudaStream_t st, int max_ctas = 0) {
    int rc = set_repair_smem((const void*)repair_persistent_kernel<BM>, smem);
    if (rc) return rc;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, repair_persistent_kernel<BM>, 256, smem);
    if (per_sm < 1) per_sm = 1;
    int grid = sm_count() * per_sm;
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    if (grid > nchunks) grid = nchunks;
    CDCLQ_CUDA_TRY(cudaMemsetAsync(counter_dev, 0, sizeof(int), st));
    CDCLQ_LAUNCH(repair_persistent_kernel<BM>, grid, 256, smem, st, chunks_dev, nchunks, rp, counter_dev);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "repair_persistent_kernel launch");
}

// CTAs of the persistent kernel that fit on one SM with `smem` bytes of dynamic shared memory (0 on error).
template <int BM>
static int persistent_ctas_per_sm(size_t smem) {
    if (set_repair_smem((const void*)repair_persistent_kernel<BM>, smem)) {
        cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, repair_persistent_kernel<BM>, 256, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm;
}

// Per-BM entry points (repair_bm64.cu, repair_bm128.cu); max_ctas > 0 caps the grid.
int launch_repair_persistent_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                  int* counter_dev, cudaStream_t st, int max_ctas);
int launch_repair_cluster_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                               int* counter_dev, cudaStream_t st, int max_ctas);
int launch_repair_quad_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                            int* counter_dev, cudaStream_t st, int max_ctas);
int launch_repair_persistent_bm128(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                   int* counter_dev, cudaStream_t st, int max_ctas);
int launch_repair_cluster_bm128(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                int* counter_dev, cudaStream_t st, int max_ctas);
int repair_persistent_ctas_per_sm_bm128(size_t smem);

}  // namespace cdclq
