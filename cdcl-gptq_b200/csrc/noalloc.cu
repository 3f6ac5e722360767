// noalloc.cu - Gram accumulation that performs no device allocation.
//
// cdclq_gram_accumulate_device needs an n x n f32 scratch for each 2048-token chunk (the f32 GEMM result
// that is widened into the f64 Hessian, src/linalg.rs:392-416) and obtains it with cudaMallocAsync.  Some
// callers cannot allocate device memory at the point where they accumulate a Hessian: a calibration hook
// running inside a framework whose allocator already owns the device memory (an extra cudaMalloc there can
// fail or fragment the framework's pool), or a runtime that reserves all of its memory at start-up and
// forbids allocation afterwards.  This file gives them a variant whose scratch is a file-scope
// `__device__` array of fixed size, kept by every GPU that uses it until the process exits.
//
// When the array's device memory is reserved: with CUDA's lazy module loading (the default since CUDA 12.2,
// CUDA_MODULE_LOADING=LAZY) this file's module is loaded into a device's context - and the 4 MiB array
// reserved there - only when something of the module is first needed on that device, here the
// cudaGetSymbolAddress of the first call.  That first call per device can therefore itself take device
// memory (the module and the array); a caller that forbids allocation after start-up makes that first call at
// start-up (a call with t = 0 resolves the scratch and launches nothing), before any stream capture.  With
// CUDA_MODULE_LOADING=EAGER the module, array included, is loaded with the context.
//
// The caller still owns and passes the inputs (x, y) and the output (h); only the scratch is internal.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace cdclq {

// Largest Hessian width the allocation-free variant accepts: the scratch holds one n x n f32 chunk result.
constexpr size_t kNoAllocGramMaxN = 1024;

// The scratch: 1024 * 1024 f32 = 4 MiB in every device's global memory.  Host code must not take this
// symbol's address directly: in host code the name refers to a host-side stand-in, so its device address
// is obtained with cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) float g_noalloc_gram_scratch[kNoAllocGramMaxN * kNoAllocGramMaxN];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch on the current device, looked up on the first call per device.
static int noalloc_scratch(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return set_error(CDCLQ_ERR_CUDA, "device index out of range for the scratch table");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_gram_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_gram_scratch)");
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}

}  // namespace cdclq

extern "C" int cdclq_gram_accumulate_device_noalloc(const float* x, const float* y, size_t t, size_t n, double* h,
                                                    void* stream) {
    using namespace cdclq;
    if (!x || !y || !h || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (n > kNoAllocGramMaxN)
        return set_error(CDCLQ_ERR_ARG, "n = " + std::to_string(n) +
                                            " exceeds the allocation-free scratch of cdclq_gram_accumulate_device_noalloc "
                                            "(at most " + std::to_string(kNoAllocGramMaxN) + " columns); use "
                                            "cdclq_gram_accumulate_device");
    float* tmp = nullptr;
    int rc = noalloc_scratch(&tmp);  // first call on a device: loads the module, reserves the array
    if (rc) return rc;
    if (t == 0) return 0;  // nothing to add: a start-up call that only resolves the scratch
    // Every element of the scratch that a chunk reads is written by the same chunk's GEMM first (beta = 0;
    // for x == y the widening reads only the lower triangle, which the GEMM always writes), so the previous
    // call's contents never leak into a result and nothing needs clearing.
    return launch_gram_f32(x, y, (int64_t)t, (int)n, h, tmp, (cudaStream_t)stream);
}
