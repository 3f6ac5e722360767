// gemm.cu - stand-alone f32 GEMM in the fixed order (asymmetric target, proxy loss), Gram accumulation with
// f32 activations, and small elementwise helpers.
//
//   src/engine.rs:737-755  W* = ((W M) U^T) U      -> launch_sgemm x3
//   src/engine.rs:808-815  proxy_loss              -> launch_sgemm + launch_proxy_loss
//   src/linalg.rs:388-418  gram_accumulate         -> launch_gram_f32 (token chunks of 2048, f32 products
//                                                     accumulated per chunk, widened into the f64 sum)
#include "common.cuh"
#include "gemm_core.cuh"
#include "kernels.h"

namespace cdclq {

// C[i][j] = alpha * acc (beta == 0) or alpha * acc + beta * C[i][j]; CTA tile 128 x 128.
using SgemmTile = Tile<128, 128, 8>;

__device__ __forceinline__ float sgemm_out(float alpha, float beta, float acc, float old) {
    const float v = __fmul_rn(alpha, acc);
    return (beta == 0.0f) ? v : __fadd_rn(v, __fmul_rn(beta, old));
}

template <bool AT>
__global__ void __launch_bounds__(256) sgemm_kernel(int m, int n, int k, float alpha, const float* a, int64_t lda,
                                                    const float* b, int64_t ldb, float beta, float* c, int64_t ldc,
                                                    int lower_only) {
    using S = SgemmTile;
    __shared__ __align__(16) float stage[S::STAGE_FLOATS];
    const int r0 = blockIdx.y * S::BM, c0 = blockIdx.x * S::BN;
    if (lower_only && c0 > r0 + S::BM - 1) return;  // tile entirely above the diagonal
    float acc[S::TM][S::TN];
#pragma unroll
    for (int i = 0; i < S::TM; i++)
#pragma unroll
        for (int j = 0; j < S::TN; j++) acc[i][j] = 0.0f;
    BGlobal<S> B{b, ldb, (int64_t)c0, min(S::BN, n - c0), k,
                 (ldb % 4 == 0) && (c0 % 4 == 0) && (((uintptr_t)b & 15) == 0)};
    if (AT) {
        AGlobalT<S> A{a, lda, (int64_t)r0, min(S::BM, m - r0), k,
                      (lda % 4 == 0) && (r0 % 4 == 0) && (((uintptr_t)a & 15) == 0)};
        gemm_loader_a<S>(acc, A, B, k, stage);
    } else {
        AGlobal<S> A{a + (int64_t)r0 * lda, lda, min(S::BM, m - r0), k, (lda % 4 == 0) && (((uintptr_t)a & 15) == 0)};
        gemm_loader_a<S>(acc, A, B, k, stage);
    }
    int ty, tx;
    gemm_coords(threadIdx.x, ty, tx);
    const bool vec = (ldc % 4 == 0) && (((uintptr_t)c & 15) == 0);
#pragma unroll
    for (int i = 0; i < S::TM; i++) {
        const int r = r0 + TileMap<S>::row(ty, i);
        if (r >= m) continue;
        float* crow = c + (int64_t)r * ldc;
#pragma unroll
        for (int v = 0; v < S::TN / 4; v++) {
            const int cc = c0 + TileMap<S>::col(tx, 4 * v);  // four consecutive columns cc .. cc+3
            if (vec && cc + 3 < n) {
                float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (beta != 0.0f) o = *reinterpret_cast<const float4*>(crow + cc);
                o.x = sgemm_out(alpha, beta, acc[i][4 * v], o.x);
                o.y = sgemm_out(alpha, beta, acc[i][4 * v + 1], o.y);
                o.z = sgemm_out(alpha, beta, acc[i][4 * v + 2], o.z);
                o.w = sgemm_out(alpha, beta, acc[i][4 * v + 3], o.w);
                *reinterpret_cast<float4*>(crow + cc) = o;
            } else {
#pragma unroll
                for (int q = 0; q < 4; q++)
                    if (cc + q < n)
                        crow[cc + q] = sgemm_out(alpha, beta, acc[i][4 * v + q], beta == 0.0f ? 0.0f : crow[cc + q]);
            }
        }
    }
}

__global__ void transpose_kernel(const float* a, int rows, int cols, float* out) {
    __shared__ float t[32][33];
    int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int y = threadIdx.y; y < 32; y += 8) {
        int r = by + y, c = bx + threadIdx.x;
        if (r < rows && c < cols) t[y][threadIdx.x] = a[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += 8) {
        int r = bx + y, c = by + threadIdx.x;  // out is cols x rows
        if (r < cols && c < rows) out[(int64_t)r * rows + c] = t[threadIdx.x][y];
    }
}

int launch_transpose(const float* a, int rows, int cols, float* out, cudaStream_t st) {
    dim3 g((cols + 31) / 32, (rows + 31) / 32), b(32, 8);
    CDCLQ_LAUNCH(transpose_kernel, g, b, 0, st, a, rows, cols, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "transpose_kernel launch");
}

int launch_sgemm(int m, int n, int k, float alpha, const float* a, int64_t lda, bool a_trans, const float* b,
                 int64_t ldb, bool b_trans, float beta, float* c, int64_t ldc, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    const float* bb = b;
    float* bt = nullptr;
    if (b_trans) {  // B(k, j) = b[j * ldb + k]: take an exact row-major copy first
        if (ldb != k) return set_error(CDCLQ_ERR_ARG, "launch_sgemm: transposed B must be dense");
        CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&bt, sizeof(float) * (size_t)k * n, st));
        int rc = launch_transpose(b, n, k, bt, st);
        if (rc) return rc;
        bb = bt;
        ldb = n;
    }
    dim3 g((n + SgemmTile::BN - 1) / SgemmTile::BN, (m + SgemmTile::BM - 1) / SgemmTile::BM);
    if (a_trans)
        CDCLQ_LAUNCH(sgemm_kernel<true>, g, 256, 0, st, m, n, k, alpha, a, lda, bb, ldb, beta, c, ldc, 0);
    else
        CDCLQ_LAUNCH(sgemm_kernel<false>, g, 256, 0, st, m, n, k, alpha, a, lda, bb, ldb, beta, c, ldc, 0);
    cudaError_t e = cudaGetLastError();
    if (bt) cudaFreeAsync(bt, st);
    return e == cudaSuccess ? 0 : cuda_error(e, "sgemm_kernel launch");
}

// h[i][j] += (double) tmp[i][j]; with `sym` the lower triangle of tmp is mirrored (X^T X is exactly symmetric:
// tmp[i][j] and tmp[j][i] accumulate identical products in identical order).
__global__ void widen_add_kernel(const float* tmp, int n, double* h, int sym) {
    int i = blockIdx.y;
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float v = (sym && j > i) ? tmp[(int64_t)j * n + i] : tmp[(int64_t)i * n + j];
    h[(int64_t)i * n + j] = __dadd_rn(h[(int64_t)i * n + j], (double)v);
}

int launch_gram_f32(const float* x, const float* y, int64_t t, int n, double* h, float* tmp, cudaStream_t st) {
    const int64_t TC = 2048;  // src/linalg.rs:392
    const bool sym = (x == y);
    for (int64_t t0 = 0; t0 < t; t0 += TC) {
        int tc = (int)((t - t0) < TC ? (t - t0) : TC);
        dim3 g((n + SgemmTile::BN - 1) / SgemmTile::BN, (n + SgemmTile::BM - 1) / SgemmTile::BM);
        CDCLQ_LAUNCH(sgemm_kernel<true>, g, 256, 0, st, n, n, tc, 1.0f, x + t0 * n, (int64_t)n, y + t0 * n, (int64_t)n,
                     0.0f, tmp, (int64_t)n, sym ? 1 : 0);
        dim3 g2((n + 255) / 256, n);  // n <= 65535 (checked by the caller)
        CDCLQ_LAUNCH(widen_add_kernel, g2, 256, 0, st, tmp, n, h, sym ? 1 : 0);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "gram kernels launch");
}

__global__ void sub_kernel(const float* a, const float* b, int64_t count, float* out) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    for (; i < count; i += (int64_t)gridDim.x * blockDim.x) out[i] = __fsub_rn(a[i], b[i]);
}

int launch_sub(const float* a, const float* b, int64_t count, float* out, cudaStream_t st) {
    int blocks = (int)((count + 255) / 256);
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    CDCLQ_LAUNCH(sub_kernel, blocks, 256, 0, st, a, b, count, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "sub_kernel launch");
}

// src/engine.rs:740-746: mp[i][j] = M[perm i][perm j], plus (damp_val as f32) on the diagonal
__global__ void permute_m_kernel(const float* m, const uint32_t* perm, int n, float damp, float* mp) {
    int i = blockIdx.y;
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float v = m[(int64_t)perm[i] * n + perm[j]];
    if (i == j) v = __fadd_rn(v, damp);
    mp[(int64_t)i * n + j] = v;
}

int launch_permute_m(const float* m, const uint32_t* perm, int n, float damp, float* mp, cudaStream_t st) {
    dim3 g((n + 255) / 256, n);
    CDCLQ_LAUNCH(permute_m_kernel, g, 256, 0, st, m, perm, n, damp, mp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "permute_m_kernel launch");
}

// sum_i (f64) e[i] * (f64) eh[i]: per-block partial sums, then one block reduces the partials in order.
__global__ void dot_partial_kernel(const float* e, const float* eh, int64_t count, double* part) {
    __shared__ double s[256];
    double acc = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        acc = __fma_rn((double)e[i], (double)eh[i], acc);
    s[threadIdx.x] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
        if (threadIdx.x < o) s[threadIdx.x] = __dadd_rn(s[threadIdx.x], s[threadIdx.x + o]);
        __syncthreads();
    }
    if (threadIdx.x == 0) part[blockIdx.x] = s[0];
}

__global__ void sum_partials_kernel(const double* part, int np, double* out) {
    if (threadIdx.x != 0) return;
    double s = 0.0;
    for (int i = 0; i < np; i++) s = __dadd_rn(s, part[i]);
    *out = s;
}

int launch_proxy_loss(const float* e, const float* eh, int64_t count, double* out, cudaStream_t st) {
    const int np = 148 * 4;
    double* part = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&part, sizeof(double) * np, st));
    CDCLQ_LAUNCH(dot_partial_kernel, np, 256, 0, st, e, eh, count, part);
    CDCLQ_LAUNCH(sum_partials_kernel, 1, 32, 0, st, part, np, out);
    cudaFreeAsync(part, st);
    cudaError_t e2 = cudaGetLastError();
    return e2 == cudaSuccess ? 0 : cuda_error(e2, "proxy loss kernels launch");
}

}  // namespace cdclq
