// io.cu - the device side of the reference's safetensors ingest and packed writer (src/io.rs):
//   tensor_to_f32        (src/io.rs:37-45)   bf16/f16 -> f32 widening (lossless), on the device after the raw copy
//   first_non_finite     (src/io.rs:120-122) index of the first NaN/inf, a parallel min-index scan
//   HessianStore::tensor (src/io.rs:195-213) the load-time refusal of a non-finite matrix, same message
//   packed_tensors       (src/io.rs:244-270) scales as f16 bits and zero points as u8 (the codes' bit stream is
//                                            cdclq_pack's kernel)
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace cdclq {

__global__ void widen_f16_kernel(const __half* __restrict__ src, int64_t count, float* __restrict__ dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half2float(src[i]);
}

__global__ void widen_bf16_kernel(const uint16_t* __restrict__ src, int64_t count, float* __restrict__ dst) {
    // bf16 is the upper half of an f32: exact
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

__global__ void first_non_finite_kernel(const float* __restrict__ x, int64_t count, unsigned long long* first) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        if ((unsigned long long)i > *(volatile unsigned long long*)first) return;  // an earlier one is known
        if (!isfinite(x[i])) {
            atomicMin(first, (unsigned long long)i);
            return;
        }
    }
}

__global__ void encode_groups_kernel(const float* __restrict__ scales, const float* __restrict__ zeros, int64_t count,
                                     uint16_t* __restrict__ scales_f16, uint8_t* __restrict__ qzeros) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        scales_f16[i] = __half_as_ushort(__float2half_rn(scales[i]));  // exact: scales are f16 values
        qzeros[i] = (uint8_t)zeros[i];                                 // 0..=maxq <= 255
    }
}

static int grid_for(int64_t count) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t b = (count + 255) / 256;
    const int64_t cap = (int64_t)sms * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// Rust's `{}` rendering of an f32 that is not finite
static std::string rust_non_finite(float v) {
    if (v != v) return "NaN";
    return v > 0 ? "inf" : "-inf";
}

}  // namespace cdclq

using namespace cdclq;

extern "C" {

int cdclq_widen_to_f32_device(const void* src, int dtype, size_t count, float* dst, void* stream) {
    if ((!src || !dst) && count) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (count == 0) return CDCLQ_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t c = (int64_t)count;
    if (dtype == CDCLQ_DTYPE_F32) {
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyDeviceToDevice, st));
        return CDCLQ_OK;
    }
    if (dtype == CDCLQ_DTYPE_F16)
        CDCLQ_LAUNCH(widen_f16_kernel, grid_for(c), 256, 0, st, (const __half*)src, c, dst);
    else if (dtype == CDCLQ_DTYPE_BF16)
        CDCLQ_LAUNCH(widen_bf16_kernel, grid_for(c), 256, 0, st, (const uint16_t*)src, c, dst);
    else
        return set_error(CDCLQ_ERR_ARG, "unsupported weight dtype (need F32/F16/BF16)");
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CDCLQ_OK : cuda_error(e, "widen kernel launch");
}

int cdclq_first_non_finite_device(const float* x, size_t count, int64_t* index_out, void* stream) {
    if (!index_out || (!x && count)) return set_error(CDCLQ_ERR_ARG, "null argument");
    *index_out = -1;
    if (count == 0) return CDCLQ_OK;
    cudaStream_t st = (cudaStream_t)stream;
    unsigned long long* first = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&first, sizeof(unsigned long long), st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(first, 0xff, sizeof(unsigned long long), st));
    CDCLQ_LAUNCH(first_non_finite_kernel, grid_for((int64_t)count), 256, 0, st, x, (int64_t)count, first);
    unsigned long long h = ULLONG_MAX;
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, first, sizeof h, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFreeAsync(first, st);
    if (e != cudaSuccess) return cuda_error(e, "first_non_finite_kernel");
    *index_out = (h == ULLONG_MAX) ? -1 : (int64_t)h;
    return CDCLQ_OK;
}

int cdclq_check_matrix_device(const float* h, size_t n, const char* key, void* stream) {
    int64_t i = -1;
    int rc = cdclq_first_non_finite_device(h, n * n, &i, stream);
    if (rc) return rc;
    if (i < 0) return CDCLQ_OK;
    float v = 0.0f;
    CDCLQ_CUDA_TRY(cudaMemcpy(&v, h + i, sizeof v, cudaMemcpyDeviceToHost));
    const std::string d = std::to_string(n);
    return set_error(CDCLQ_ERR_NONFINITE, std::string(key ? key : "") + ": " + d + " x " + d +
                                              " matrix has a non-finite entry (" + rust_non_finite(v) + ") at [ " +
                                              std::to_string((size_t)i / n) + ", " + std::to_string((size_t)i % n) +
                                              " ]; the calibration data or the captured forward is corrupt, "
                                              "refusing to quantize");
}

int cdclq_encode_groups_device(const float* scales, const float* zeros, size_t count, uint16_t* scales_f16,
                               uint8_t* qzeros, void* stream) {
    if ((!scales || !zeros || !scales_f16 || !qzeros) && count) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (count == 0) return CDCLQ_OK;
    cudaStream_t st = (cudaStream_t)stream;
    CDCLQ_LAUNCH(encode_groups_kernel, grid_for((int64_t)count), 256, 0, st, scales, zeros, (int64_t)count, scales_f16,
                 qzeros);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CDCLQ_OK : cuda_error(e, "encode_groups_kernel launch");
}

}  // extern "C"
