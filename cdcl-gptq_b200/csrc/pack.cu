// pack.cu - the packed container and the grid helpers on the GPU.
//
//   src/quant.rs:106-131  pack_row: LSB-first bit stream, per-group widths      -> pack_kernel (one thread per
//                                                                                 output byte: the byte is the
//                                                                                 OR of the <= 4 codes whose
//                                                                                 bits it holds)
//   src/quant.rs:133-151  unpack_row + src/quant.rs:189-202 dequantize          -> unpack_dequant_kernel
//   src/quant.rs:40-83    find_params                                           -> find_params_kernel
//   src/engine.rs:822-838 rtn_layer                                             -> rtn_kernel
// bitoff[j] = sum of the widths of columns 0..j-1 (same for every row), bitoff[n] = bits per row.
#include "common.cuh"
#include "kernels.h"

namespace cdclq {

__global__ void pack_kernel(const uint8_t* codes, int d_out, int n, const uint32_t* bitoff, int row_bytes,
                            const uint8_t* widths_per_col_unused, uint8_t* out) {
    int r = blockIdx.y;
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= row_bytes || r >= d_out) return;
    const uint32_t lo = (uint32_t)b * 8u, hi = lo + 8u;
    // first column whose bits end after `lo`
    int a = 0, z = n;
    while (a < z) {
        int mid = (a + z) >> 1;
        if (bitoff[mid + 1] <= lo) a = mid + 1; else z = mid;
    }
    uint32_t byte = 0;
    for (int j = a; j < n && bitoff[j] < hi; j++) {
        uint32_t c = codes[(int64_t)r * n + j];
        uint32_t off = bitoff[j];
        if (off >= lo) byte |= c << (off - lo);
        else byte |= c >> (lo - off);
    }
    out[(int64_t)r * row_bytes + b] = (uint8_t)(byte & 0xffu);
}

int launch_pack(const uint8_t* codes, int d_out, int n, int g, const uint8_t* gbits, const uint32_t* bitoff,
                int row_bytes, uint8_t* out, cudaStream_t st) {
    (void)g;
    (void)gbits;
    for (int r0 = 0; r0 < d_out; r0 += 65535) {
        int rows = d_out - r0 < 65535 ? d_out - r0 : 65535;
        dim3 grid((row_bytes + 127) / 128, rows);
        CDCLQ_LAUNCH(pack_kernel, grid, 128, 0, st, codes + (int64_t)r0 * n, rows, n, bitoff, row_bytes, nullptr,
                     out + (int64_t)r0 * row_bytes);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "pack_kernel launch");
}

__global__ void unpack_dequant_kernel(const uint8_t* packed, int d_out, int n, int g, int ng, const uint8_t* gbits,
                                      const uint32_t* bitoff, int row_bytes, const uint32_t* perm, const float* scales,
                                      const float* zeros, float* out) {
    int r = blockIdx.y;
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n || r >= d_out) return;
    const uint8_t* row = packed + (int64_t)r * row_bytes;
    uint32_t off = bitoff[j];
    uint32_t w = gbits[j / g];
    uint32_t byte = off >> 3, sh = off & 7u;
    uint32_t v = row[byte];
    if (sh + w > 8u) v |= (uint32_t)row[byte + 1] << 8;
    uint32_t code = (v >> sh) & ((1u << w) - 1u);
    int gi = j / g;
    float s = scales[(int64_t)r * ng + gi];
    float z = zeros[(int64_t)r * ng + gi];
    out[(int64_t)r * n + perm[j]] = __fmul_rn(s, __fsub_rn((float)code, z));
}

int launch_unpack_dequant(const uint8_t* packed, int d_out, int n, int g, const uint8_t* gbits,
                          const uint32_t* bitoff, int row_bytes, const uint32_t* perm, const float* scales,
                          const float* zeros, float* out, cudaStream_t st) {
    int ng = (n + g - 1) / g;
    for (int r0 = 0; r0 < d_out; r0 += 65535) {
        int rows = d_out - r0 < 65535 ? d_out - r0 : 65535;
        dim3 grid((n + 255) / 256, rows);
        CDCLQ_LAUNCH(unpack_dequant_kernel, grid, 256, 0, st, packed + (int64_t)r0 * row_bytes, rows, n, g, ng, gbits,
                     bitoff, row_bytes, perm, scales + (int64_t)r0 * ng, zeros + (int64_t)r0 * ng,
                     out + (int64_t)r0 * n);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "unpack_dequant_kernel launch");
}

// find_params over one group (sequential, as the reference's scalar loop)
__device__ void find_params_seq(const float* v, int len, float maxq, int mse, float& s, float& z) {
    float xmin = 0.0f, xmax = 0.0f;
    for (int i = 0; i < len; i++) {
        xmin = min_sel(xmin, v[i]);
        xmax = max_sel(xmax, v[i]);
    }
    if (xmin == 0.0f && xmax == 0.0f) {
        xmin = -1.0f;
        xmax = 1.0f;
    }
    grid_mk(xmin, xmax, maxq, s, z);
    if (!mse) return;
    float best_err = INFINITY;
    for (int ci = 0; ci < 24; ci++) {
        float p = clip_ratio(ci), cs, cz;
        grid_mk(__fmul_rn(p, xmin), __fmul_rn(p, xmax), maxq, cs, cz);
        float err = 0.0f;
        for (int i = 0; i < len; i++) {
            uint8_t c;
            float d;
            quant_code(v[i], cs, cz, maxq, c, d);
            float e = __fsub_rn(d, v[i]);
            err = __fadd_rn(err, __fmul_rn(e, e));
        }
        if (err < best_err) {
            best_err = err;
            s = cs;
            z = cz;
        }
    }
}

__global__ void find_params_kernel(const float* vals, int rows, int len, float maxq, int mse, float* s, float* z) {
    int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float ss, zz;
    find_params_seq(vals + (int64_t)r * len, len, maxq, mse, ss, zz);
    s[r] = ss;
    z[r] = zz;
}

int launch_find_params(const float* vals, int rows, int len, int bits, int mse, float* s, float* z,
                       cudaStream_t st) {
    float maxq = (float)((1u << bits) - 1u);
    CDCLQ_LAUNCH(find_params_kernel, (rows + 127) / 128, 128, 0, st, vals, rows, len, maxq, mse, s, z);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "find_params_kernel launch");
}

// src/engine.rs:822-838: one thread per (row, group)
__global__ void rtn_kernel(const float* w, int d_out, int n, int g, int ng, float maxq, int mse, float* out) {
    int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (t >= (int64_t)d_out * ng) return;
    int r = (int)(t / ng), gi = (int)(t % ng);
    int j0 = gi * g, len = min(g, n - j0);
    const float* src = w + (int64_t)r * n + j0;
    float s, z;
    find_params_seq(src, len, maxq, mse, s, z);
    for (int i = 0; i < len; i++) {
        uint8_t c;
        float d;
        quant_code(src[i], s, z, maxq, c, d);
        out[(int64_t)r * n + j0 + i] = d;
    }
}

int launch_rtn(const float* w, int d_out, int n, int g, int bits, int mse, float* out, cudaStream_t st) {
    int ng = (n + g - 1) / g;
    int64_t total = (int64_t)d_out * ng;
    float maxq = (float)((1u << bits) - 1u);
    CDCLQ_LAUNCH(rtn_kernel, (unsigned)((total + 127) / 128), 128, 0, st, w, d_out, n, g, ng, maxq, mse, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "rtn_kernel launch");
}

}  // namespace cdclq
