// gptq.cu - phase 1: the blocked GPTQ pass with lazy batch updates (src/engine.rs:388-479).
//
// One CTA owns up to 64 rows of one layer for the whole pass (rows are independent under the objective,
// src/engine.rs:9-15).  Per block of B columns:
//   1. the block w1 = w[:, i1:i2] is staged in shared memory, k-major ([B][72]) so that each row is a column;
//   2. columns are processed in order.  Four threads share a row: they compute the group grid together at a
//      group start (min/max split four ways, the 24 MSE clip candidates split four ways), quantize the
//      column redundantly, and split the rank-1 in-block compensation w1[:, j+1:i2] -= eps * U[j, j+1:i2]
//      four ways.  The four lanes sit in one warp, so a __syncwarp orders consecutive columns.  Columns go in
//      micro-blocks of up to 8: a column's compensation of the rest of its micro-block is on the sequential
//      chain, its compensation of the later columns is applied once per micro-block, every element taking
//      the micro-block's terms in column order (the reference's sequence of roundings, fewer round trips).
//      The rows of U the compensation reads come from a shared-memory window of P1_UWIN rows, double-buffered
//      with cp.async (the next window is in flight while the current one is used), so no global load sits
//      inside the column-to-column dependency chain;
//   3. the deferred compensation w[:, i2:] -= err1 * U[i1:i2, i2:] runs on the FP32 GEMM core
//      (A = err1 from shared memory, B = U tiles), one subtraction per element per block as in the reference.
// Outputs per element: code, dequantized value, and eps^2 (consumed by the per-chunk conflict statistics).
// Every rounding follows src/engine.rs:404-449 and src/quant.rs:40-95 (see common.cuh).
#include "common.cuh"
#include "gemm_core.cuh"
#include "kernels.h"

namespace cdclq {

constexpr int P1_ROWS = 64;
using P1Tile = Tile<P1_ROWS, 128, 16>;  // lazy-update GEMM: 64 rows x 128 columns per step
// w1 stride: 72 = 8 (mod 32), so the 4 columns x 8 rows a warp touches in one column step fall in 32
// distinct banks
constexpr int P1_W1LD = 72;
constexpr int P1_ELD = P1Tile::ALD;  // err1 stride (16-byte aligned k-major A operand)

static __host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

// U window: up to P1_UWIN rows of U[j, i1:i1+B] per buffer, two buffers in the lazy GEMM's B staging area
// (unused during the column loop): 2 * 16 * 128 floats = the Tile's B_STAGE_FLOATS; wider blocks get fewer rows.
constexpr int P1_UWIN = 16;
constexpr int P1_MB = 8;  // micro-block width of the column loop
static_assert(2 * P1_UWIN * 128 <= P1Tile::B_STAGE_FLOATS, "the U window must fit the staging buffer");
__host__ __device__ inline int p1_uwin(int B) {
    int w = (P1Tile::B_STAGE_FLOATS / 2) / B;
    return w < 1 ? 1 : (w > P1_UWIN ? P1_UWIN : w);
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Rows j0 .. j0+rows-1 of U, columns i1 .. i1+cnt-1, into win[(j - j0) * B + k].  16-byte copies when every row
// segment is 16-byte aligned (n and i1 multiples of 4; the block width B is), plain loads otherwise.
__device__ __forceinline__ void load_u_window(float* win, const float* U, int n, int i1, int j0, int rows, int cnt,
                                              int B, bool vec, int tid) {
    if (vec) {
        const int q = (cnt + 3) >> 2;  // 16-byte segments per row (cnt % 4 == 0 here)
        for (int idx = tid; idx < rows * q; idx += GEMM_THREADS) {
            const int rr = idx / q, c4 = (idx - rr * q) << 2;
            cp_async16(win + rr * B + c4, U + (int64_t)(j0 + rr) * n + i1 + c4);
        }
        cp_async_commit();
    } else {
        for (int idx = tid; idx < rows * cnt; idx += GEMM_THREADS) {
            const int rr = idx / cnt, k = idx - rr * cnt;
            win[rr * B + k] = __ldg(U + (int64_t)(j0 + rr) * n + i1 + k);
        }
    }
}

size_t phase1_smem_bytes(int block) {
    size_t b = (size_t)block;
    return align16(b * P1_W1LD * 4) + align16(b * P1_ELD * 4) + align16(b * P1_ROWS) +
           (size_t)P1Tile::B_STAGE_FLOATS * 4 + align16(b * 4);
}

__global__ void __launch_bounds__(256, 2) gptq_phase1_kernel(const P1Item* __restrict__ items, int B, int mse) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const P1Item it = items[blockIdx.x];
    const int n = it.n, g = it.g, ng = it.ng, rows = it.rows;
    const int tid = threadIdx.x;
    const int r = tid >> 2, sub = tid & 3;
    const bool rvalid = r < rows;

    float* w1 = reinterpret_cast<float*>(smem_raw);
    float* err1 = reinterpret_cast<float*>(smem_raw + align16((size_t)B * P1_W1LD * 4));
    uint8_t* cbuf = smem_raw + align16((size_t)B * P1_W1LD * 4) + align16((size_t)B * P1_ELD * 4);
    float* stage = reinterpret_cast<float*>(cbuf + align16((size_t)B * P1_ROWS));
    float* invd = stage + P1Tile::B_STAGE_FLOATS;  // [B] 1 / U_jj of the block's columns

    float* w = it.w + (int64_t)it.row0 * n;  // tile rows: w[rr * n + c]
    const float* U = it.u;

    float s = 1.0f, z = 0.0f, maxq = 1.0f;  // current group grid of this thread's row
    for (int i1 = 0; i1 < n; i1 += B) {
        const int i2 = min(i1 + B, n), cnt = i2 - i1;
        for (int idx = tid; idx < P1_ROWS * cnt; idx += blockDim.x) {
            int rr = idx / cnt, k = idx - rr * cnt;
            w1[k * P1_W1LD + rr] = (rr < rows) ? w[(int64_t)rr * n + i1 + k] : 0.0f;
        }
        for (int idx = tid; idx < P1_ELD * cnt; idx += blockDim.x) err1[idx] = 0.0f;
        for (int k = tid; k < cnt; k += blockDim.x) invd[k] = __fdiv_rn(1.0f, __ldg(U + (int64_t)(i1 + k) * n + i1 + k));
        const bool uvec = (n % 4 == 0) && (i1 % 4 == 0) && (cnt % 4 == 0);
        const int uw = p1_uwin(B);
        load_u_window(stage, U, n, i1, i1, min(uw, cnt), cnt, B, uvec, tid);

        // Micro-blocks of up to P1_MB columns inside one U window and one quantization group: the per-column
        // chain quantizes a column and compensates only the rest of its micro-block; the columns past the
        // micro-block then receive the micro-block's compensations in one pass, each element still taking
        // them one at a time in column order (w -= e_i * U[i][k], i ascending): the reference's roundings.
        for (int i0 = 0; i0 < cnt;) {
            const int j0 = i1 + i0;
            if (i0 % uw == 0) {
                // window i0 / uw has landed; every warp is done with the previous one, whose buffer now receives
                // the next window
                if (uvec) cp_async_wait_all();
                __syncthreads();
                const int nw = i0 + uw;
                if (nw < cnt)
                    load_u_window(stage + ((nw / uw) & 1) * uw * B, U, n, i1, i1 + nw, min(uw, cnt - nw), cnt, B, uvec,
                                  tid);
            }
            // micro-block [i0, ie): ends at P1_MB columns, the window's end, the block's end or the next group
            const int ie = min(min(i0 + P1_MB, cnt), min((i0 / uw + 1) * uw, g - j0 % g + i0));
            float emb[P1_MB];
#pragma unroll
            for (int m = 0; m < P1_MB; m++) {
                const int i = i0 + m;
                if (i >= ie) break;
                const int j = i1 + i;
                if (j % g == 0) {
                    // ---- group grid from the weights current at its first column (src/engine.rs:410-423)
                    const int gi = j / g, gend = min(j + g, n);
                    const uint32_t bits = it.gbits[gi];
                    maxq = (float)((1u << bits) - 1u);
                    float xmin = 0.0f, xmax = 0.0f;
                    for (int col = j + sub; col < gend; col += 4) {
                        float v = (col < i2) ? w1[(col - i1) * P1_W1LD + r] : (rvalid ? w[(int64_t)r * n + col] : 0.0f);
                        xmin = min_sel(xmin, v);
                        xmax = max_sel(xmax, v);
                    }
#pragma unroll
                    for (int o = 1; o < 4; o <<= 1) {
                        xmin = min_sel(xmin, __shfl_xor_sync(0xffffffffu, xmin, o));
                        xmax = max_sel(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
                    }
                    if (xmin == 0.0f && xmax == 0.0f) {
                        xmin = -1.0f;
                        xmax = 1.0f;
                    }
                    grid_mk(xmin, xmax, maxq, s, z);
                    if (mse) {
                        // this thread's 6 of the 24 clip candidates (ci = sub + 4m), each error summed over the
                        // group's columns in order; one read of each value feeds all six
                        constexpr int NC = 24 / 4;
                        float cs[NC], cz[NC], cerr[NC];
#pragma unroll
                        for (int m = 0; m < NC; m++) {
                            const float p = clip_ratio(sub + 4 * m);
                            grid_mk(__fmul_rn(p, xmin), __fmul_rn(p, xmax), maxq, cs[m], cz[m]);
                            cerr[m] = 0.0f;
                        }
                        for (int col = j; col < gend; col++) {
                            const float v = (col < i2) ? w1[(col - i1) * P1_W1LD + r]
                                                       : (rvalid ? w[(int64_t)r * n + col] : 0.0f);
#pragma unroll
                            for (int m = 0; m < NC; m++) {
                                uint8_t c;
                                float d;
                                quant_code(v, cs[m], cz[m], maxq, c, d);
                                const float e = __fsub_rn(d, v);
                                cerr[m] = __fadd_rn(cerr[m], __fmul_rn(e, e));
                            }
                        }
                        float best_err = INFINITY;
                        int best_i = 24;
#pragma unroll
                        for (int m = 0; m < NC; m++) {
                            if (cerr[m] < best_err) {
                                best_err = cerr[m];
                                best_i = sub + 4 * m;
                            }
                        }
                        // first index of the strict minimum == min error, ties to the smaller index
#pragma unroll
                        for (int o = 1; o < 4; o <<= 1) {
                            float oe = __shfl_xor_sync(0xffffffffu, best_err, o);
                            int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
                            if (oe < best_err || (oe == best_err && oi < best_i)) {
                                best_err = oe;
                                best_i = oi;
                            }
                        }
                        if (best_i < 24) {
                            float p = clip_ratio(best_i);
                            grid_mk(__fmul_rn(p, xmin), __fmul_rn(p, xmax), maxq, s, z);
                        }
                    }
                    if (sub == 0 && rvalid) {
                        int64_t so = (int64_t)(it.row0 + r) * ng + gi;
                        it.scales[so] = s;
                        it.zeros[so] = z;
                    }
                }
                // ---- quantize column j and compensate the rest of the micro-block (src/engine.rs:424-448)
                const float wv = w1[i * P1_W1LD + r];
                uint8_t c;
                float dq;
                quant_code(wv, s, z, maxq, c, dq);
                const float e = __fmul_rn(__fsub_rn(wv, dq), invd[i]);
                emb[m] = e;
                __syncwarp();
                if (sub == 0) {
                    err1[i * P1_ELD + r] = e;
                    cbuf[i * P1_ROWS + r] = c;
                    w1[i * P1_W1LD + r] = dq;  // column i is final: keep its dequantized value
                }
                const float* urow = stage + ((i / uw) & 1) * uw * B + (i % uw) * B;  // U[j, i1:i2]
                for (int k = i + 1 + sub; k < ie; k += 4) {
                    float* x = &w1[k * P1_W1LD + r];
                    *x = __fsub_rn(*x, __fmul_rn(e, urow[k]));
                }
                __syncwarp();
            }
            // ---- the micro-block's compensations of the block's later columns, in column order per element
            const int mb = ie - i0;
            const float* ubase = stage + ((i0 / uw) & 1) * uw * B + (i0 % uw) * B;  // U[j0 + m, i1:i2] at m * B
            for (int k = ie + sub; k < cnt; k += 4) {
                float x = w1[k * P1_W1LD + r];
#pragma unroll
                for (int m = 0; m < P1_MB; m++)
                    if (m < mb) x = __fsub_rn(x, __fmul_rn(emb[m], ubase[m * B + k]));
                w1[k * P1_W1LD + r] = x;
            }
            __syncwarp();
            i0 = ie;
        }
        __syncthreads();

        // ---- block outputs: codes, dequantized weights, eps^2
        for (int idx = tid; idx < rows * cnt; idx += blockDim.x) {
            int rr = idx / cnt, k = idx - rr * cnt;
            int64_t off = (int64_t)(it.row0 + rr) * n + i1 + k;
            it.codes[off] = cbuf[k * P1_ROWS + rr];
            it.wq[off] = w1[k * P1_W1LD + rr];
            float ev = err1[k * P1_ELD + rr];
            it.eps2[off] = __fmul_rn(ev, ev);
        }

        // ---- lazy update of the columns past the block (src/engine.rs:452-471): w -= err1 * U[i1:i2, i2:]
        if (i2 < n) {
            using S = P1Tile;
            int ty, tx;
            gemm_coords(tid, ty, tx);
            const bool vec = (n % 4 == 0) && (i2 % 4 == 0);
            for (int c0 = i2; c0 < n; c0 += S::BN) {
                float acc[S::TM][S::TN];
#pragma unroll
                for (int a = 0; a < S::TM; a++)
#pragma unroll
                    for (int b = 0; b < S::TN; b++) acc[a][b] = 0.0f;
                BGlobal<S> Bop{U + (int64_t)i1 * n, (int64_t)n, (int64_t)c0, min(S::BN, n - c0), cnt, vec};
                gemm_smem_a<S>(acc, err1, Bop, cnt, stage);
#pragma unroll
                for (int a = 0; a < S::TM; a++) {
                    const int rr = TileMap<S>::row(ty, a);
                    if (rr >= rows) continue;
                    float* wrow = w + (int64_t)rr * n;
#pragma unroll
                    for (int v = 0; v < S::TN / 4; v++) {
                        const int cc = c0 + TileMap<S>::col(tx, 4 * v);  // columns cc .. cc+3
                        if (vec && cc + 3 < n) {
                            float4 o = *reinterpret_cast<float4*>(wrow + cc);
                            o.x = __fsub_rn(o.x, acc[a][4 * v]);
                            o.y = __fsub_rn(o.y, acc[a][4 * v + 1]);
                            o.z = __fsub_rn(o.z, acc[a][4 * v + 2]);
                            o.w = __fsub_rn(o.w, acc[a][4 * v + 3]);
                            *reinterpret_cast<float4*>(wrow + cc) = o;
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; q++)
                                if (cc + q < n) wrow[cc + q] = __fsub_rn(wrow[cc + q], acc[a][4 * v + q]);
                        }
                    }
                }
            }
        }
        __syncthreads();
    }
}

int launch_phase1(const P1Item* items_dev, int nitems, int block, int mse, cudaStream_t st) {
    if (nitems == 0) return 0;
    size_t smem = phase1_smem_bytes(block);
    cudaError_t e = cudaFuncSetAttribute(gptq_phase1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_error(e, "phase1 smem attribute");
    CDCLQ_LAUNCH(gptq_phase1_kernel, nitems, 256, smem, st, items_dev, block, mse);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "gptq_phase1_kernel launch");
    return 0;
}

}  // namespace cdclq
