// kernels.h - work-item descriptors and launchers shared between the kernels and the host engine.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "cdclq.h"
#include "common.cuh"

namespace cdclq {

// ---------------------------------------------------------------------------------------------------------
// Hessian preparation and factorisation (prep.cu).  One item per distinct (input, permutation); all items of
// one launch share n.
struct PrepItem {
    const float* h;         // n x n f32, original column order
    const uint32_t* perm;   // n, permuted position -> original column
    double* hr;             // n x n f64: flipped damped permuted Hessian, then L in its lower triangle (or null)
    double* y;              // n x n f64: L^-1 (lower)
    double* tbuf;           // 96 x n f64 scratch of the triangular inverse
    float* h32;             // n x n f32 damped permuted Hessian (phase 2 metric, or null)
    float* u;               // n x n f32 upper factor, H^-1 = U^T U (phase 1)
    double* dg;             // n f64 scratch: patched diagonal
    double* damp_val;       // 1 f64 out
    FactorStatus* status;   // 1
};

int launch_prepare(const PrepItem* items_dev, int nitems, int n, double damp, cudaStream_t st);
// damped f64 Cholesky then triangular inverse of every item (src/linalg.rs:200-347), pipelined over two streams
int launch_factor(const PrepItem* items_dev, int nitems, int n, cudaStream_t st);
int launch_u_scatter(const PrepItem* items_dev, int nitems, int n, cudaStream_t st);

// Stand-alone linalg entry points (single matrix, device pointers); used by the C ABI wrappers.
int device_cholesky(double* a, int n, FactorStatus* status, cudaStream_t st);
int device_tri_inverse(const double* l, double* y, double* tbuf, int n, cudaStream_t st);

// ---------------------------------------------------------------------------------------------------------
// Weight-side preparation (prep.cu)
// colsq[j] = sum_r w[r][j]^2 in f64, rows in order, dead columns read as 0 (src/engine.rs:279-285)
int launch_colsq(const float* w, const double* hdiag, int d_out, int n, double* colsq, cudaStream_t st);
// the same sums continued from init[j] (in place when init == colsq): a row shard after the rows before it
int launch_colsq_from(const float* w, const double* hdiag, int d_out, int n, const double* init, double* colsq,
                      cudaStream_t st);
// wt[r][j] = dead(perm[j]) ? 0 : w[r][perm[j]]  (src/engine.rs:708-731)
int launch_permute_w(const float* w, const double* hdiag, const uint32_t* perm, int d_out, int n, float* wt,
                     cudaStream_t st);
// hdiag[j] = (double) h[j][j]
int launch_hdiag(const float* h, int n, double* hdiag, cudaStream_t st);

// ---------------------------------------------------------------------------------------------------------
// Phase 1: blocked GPTQ (gptq.cu).  One item = up to 64 rows of one layer.
struct P1Item {
    float* w;               // layer working copy (d_out x n), updated in place by the lazy GEMM
    float* wq;              // layer dequantized weights
    float* eps2;            // layer eps_j^2 per element (aliases the repair error buffer)
    uint8_t* codes;         // layer codes
    float* scales;          // layer scales d_out x ng
    float* zeros;           // layer zeros d_out x ng
    const float* u;         // n x n
    const uint8_t* gbits;   // ng
    int n, g, ng, row0, rows;
};

int launch_phase1(const P1Item* items_dev, int nitems, int block, int mse, cudaStream_t st);
size_t phase1_smem_bytes(int block);

// ---------------------------------------------------------------------------------------------------------
// Phase 2: conflict selection + repair (repair.cu)
struct ChunkState {
    double loss_gptq;
    double loss_delta;
    double prev_delta;
    unsigned long long updates;
    int n_sel;
    int passes;
    int done;
    int pad;
};

struct ChunkInfo {
    const float* wt;      // chunk base: rows x n permuted target
    float* wq;            // chunk base
    float* e;             // chunk base: holds eps^2 after phase 1, then E = W - W_hat
    uint8_t* codes;       // chunk base
    float* scales;        // chunk base rows x ng
    float* zeros;         // chunk base rows x ng
    const float* h;       // n x n damped permuted Hessian (f32)
    const uint8_t* gbits; // ng
    double* colloss;      // n scratch
    double* sbsum;        // n_sb scratch
    int32_t* sel;         // n_sb capacity
    ChunkState* st;
    int n, rows, g, ng, sbw, n_sb, k_sel, pad;
};

struct SliceItem {
    int chunk;
    int r0;
    int rs;
    int pad;
};

struct SliceAcc {
    double delta;
    unsigned long long updates;
};

struct RepairParams {
    int do_refit;
    int do_cd;
    int cd_sweeps;
    int method_cdcl;
    int final_refit;  // 1: this launch is the final refit (runs on every chunk)
    int max_passes;   // max(passes, 1) (src/engine.rs:595)
    double tol;
};

int launch_chunk_stats(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, cudaStream_t st);
int launch_repair_pass(const ChunkInfo* chunks_dev, const SliceItem* slices_dev, int nslices, SliceAcc* acc_dev,
                       const RepairParams& rp, int g, int sbw, cudaStream_t st);
int launch_pass_end(const ChunkInfo* chunks_dev, int nchunks, const int* slice_begin_dev, const SliceAcc* acc_dev,
                    const RepairParams& rp, cudaStream_t st);
// Dynamic shared memory of a repair CTA working on tiles of bm (64 or 128) rows.
size_t repair_smem_bytes(int g, int sbw, int bm);
// Row-tile height of the persistent repair kernels for chunks of at most max_rows rows: 128 when a chunk has
// more than 64 rows and two 128-row CTAs fit on one SM, else 64.
int repair_tile_rows(int g, int sbw, int max_rows);
constexpr int RP_MAX_TILES_PER_CHUNK = 32;  // mode C keeps at most this many tile partials per chunk
// All passes + final refit of every chunk in one launch (chunks taken from *counter_dev, in array order).
// max_ctas > 0 caps the grid (the launch shares the GPU with another one).
int launch_repair_persistent(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw, int bm,
                             int* counter_dev, cudaStream_t st, int max_ctas = 0);
// Same with a 2-CTA cluster per chunk (chunks of more than one and at most RP_MAX_TILES_PER_CHUNK tiles).
// smem_floor > 0 reserves that much shared memory per CTA so that no other CTA shares its SM.
int launch_repair_cluster(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw, int bm,
                          int* counter_dev, cudaStream_t st, int max_ctas = 0, size_t smem_floor = 0);
// A 4-CTA cluster per chunk of exactly two 64-row tiles: row tile x column half of every repair GEMM, one CTA per SM
// (smem_floor reserves the SM).  max_ctas = the SMs given to the launch.
int launch_repair_quad(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw,
                       int* counter_dev, cudaStream_t st, int max_ctas, size_t smem_floor);

// ---------------------------------------------------------------------------------------------------------
// Generic f32 GEMM with the fixed order: C = alpha*A*B (+ beta*C), A row-major or transposed (gemm.cu)
int launch_sgemm(int m, int n, int k, float alpha, const float* a, int64_t lda, bool a_trans, const float* b,
                 int64_t ldb, bool b_trans, float beta, float* c, int64_t ldc, cudaStream_t st);
// Gram accumulation h += x^T y (f32 products, chunks of 2048 tokens widened into f64)
int launch_gram_f32(const float* x, const float* y, int64_t t, int n, double* h, float* tmp, cudaStream_t st);
// bf16 (bf16 = true) or f16 activations; both kinds are exact products in f32.
int launch_gram_half_tc(const void* x, bool bf16, int64_t t, int n, double* h, int lower_only, cudaStream_t st);

// Elementwise helpers (gemm.cu)
int launch_sub(const float* a, const float* b, int64_t count, float* out, cudaStream_t st);
int launch_permute_m(const float* m, const uint32_t* perm, int n, float damp, float* mp, cudaStream_t st);
int launch_transpose(const float* a, int rows, int cols, float* out, cudaStream_t st);
int launch_proxy_loss(const float* e, const float* eh, int64_t count, double* out, cudaStream_t st);

// Packing (pack.cu)
int launch_pack(const uint8_t* codes, int d_out, int n, int g, const uint8_t* gbits, const uint32_t* bitoff,
                int row_bytes, uint8_t* out, cudaStream_t st);
int launch_unpack_dequant(const uint8_t* packed, int d_out, int n, int g, const uint8_t* gbits,
                          const uint32_t* bitoff, int row_bytes, const uint32_t* perm, const float* scales,
                          const float* zeros, float* out, cudaStream_t st);
int launch_find_params(const float* vals, int rows, int len, int bits, int mse, float* s, float* z,
                       cudaStream_t st);
int launch_rtn(const float* w, int d_out, int n, int g, int bits, int mse, float* out, cudaStream_t st);

}  // namespace cdclq
