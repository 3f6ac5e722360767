// common.cuh - shared device numerics, launch accounting and error helpers for the cdclq CUDA library.
//
// Numerics contract.  Every kernel that decides a code, a scale or a loss term reproduces the reference's
// scalar f32/f64 operation order exactly (Rust never contracts a*b+c into an FMA), so this library is built
// with -fmad=false and the parity-critical arithmetic below spells each rounding out with __f*_rn intrinsics.
// The only fused multiply-adds are the explicit __fmaf_rn/__fma_rn of the GEMM accumulations, whose order
// (per output element: k ascending, acc starting at +0, then alpha*acc [+ beta*c]) is the fixed order of the
// oracle's restatement of `matrixmultiply` (the reference's unvendored GEMM crate).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <string>

namespace cdclq {

extern std::atomic<uint64_t> g_launches;

// Every kernel launch of the library goes through this macro so cdclq_launch_count() is exact.
#define CDCLQ_LAUNCH(kernel, grid, block, smem, stream, ...)                      \
    do {                                                                           \
        ::cdclq::g_launches.fetch_add(1, std::memory_order_relaxed);              \
        kernel<<<(grid), (block), (smem), (stream)>>>(__VA_ARGS__);               \
    } while (0)

// ---- reference constants ------------------------------------------------------------------------------
// src/quant.rs:20  F16_MIN_NORMAL = 6.103_515_6e-5 (exactly 2^-14 in f32)
constexpr float kF16MinNormal = 6.1035156e-5f;

// src/quant.rs:24-26  round_f16: f32 -> f16 (IEEE round to nearest even) -> f32
__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// src/quant.rs:92-95  quant_code.  q = clamp(round(x / scale) + zero, 0, maxq); Rust's f32::round rounds half
// away from zero, as CUDA's roundf does; `q as u8` maps NaN to 0.
__device__ __forceinline__ void quant_code(float x, float scale, float zero, float maxq, uint8_t& code, float& dq) {
    float q = __fadd_rn(roundf(__fdiv_rn(x, scale)), zero);
    if (q < 0.0f) q = 0.0f;
    if (q > maxq) q = maxq;
    code = (q == q) ? (uint8_t)q : (uint8_t)0;
    dq = __fmul_rn(scale, __fsub_rn(q, zero));
}

// src/quant.rs:54-61  the `mk` closure of find_params
__device__ __forceinline__ void grid_mk(float lo, float hi, float maxq, float& s, float& z) {
    float scale = round_f16(__fdiv_rn(__fsub_rn(hi, lo), maxq));
    if (scale < kF16MinNormal) scale = kF16MinNormal;
    float zero = roundf(__fdiv_rn(-lo, scale));
    if (zero < 0.0f) zero = 0.0f;
    if (zero > maxq) zero = maxq;
    s = scale;
    z = zero;
}

// A sufficient, division-free condition for a coordinate-descent step to keep a weight's code
// (src/engine.rs:624-633: target = cur + g / h, q = clamp(round(target / s) + z, 0, maxq), a move iff
// q != code).  Let m = code - z: small integers, so exact (zero points are integers; checked).  When
// cur = RN(s * m) - checked through the FMA residual |s * m - cur| <= 2^-23 |cur| - the exact evaluation
// t2 = RN(RN(cur + RN(g / h)) / s) satisfies |t2 - m| <= |g| / (h s) (1 + 3u) + 4.1u |m|, u = 2^-24, and
// |m| <= 255 (8-bit codes) makes the last term < 6.3e-5.  So |g| < 0.4998 h s (evaluated in f32, two more
// roundings of < 1.2e-7 relative) bounds |t2 - m| below 0.4999 + 6.3e-5 < 0.5: round(t2) = m, q = m + z =
// code, and the step keeps the code.  Infinite or NaN operands and h <= 0 fail the test (the caller then
// evaluates the step exactly).  The test never holds for a step that moves, so skipping the exact evaluation
// when it holds changes no decision.
__device__ __forceinline__ bool cd_keeps_code(float g, float h, float cur, float s, float m) {
    const float lim = __fmul_rn(__fmul_rn(0.4998f, h), s);
    const float res = __fmaf_rn(s, m, -cur);
    return h > 0.0f && lim < INFINITY && fabsf(g) < lim && fabsf(res) <= __fmul_rn(fabsf(cur), 1.1920929e-7f) &&
           m == rintf(m);
}

// The MSE clip ratio p_i = 1 - 0.02 * i (src/quant.rs:68-69), in f32.
__device__ __forceinline__ float clip_ratio(int i) { return __fsub_rn(1.0f, __fmul_rn(0.02f, (float)i)); }

// Min/max by strict comparison from a +0 seed (src/quant.rs:42-47): order-independent for finite values,
// so a tree of partial results equals the sequential scan.
__device__ __forceinline__ float min_sel(float a, float b) { return (b < a) ? b : a; }
__device__ __forceinline__ float max_sel(float a, float b) { return (b > a) ? b : a; }

// ---- status ----------------------------------------------------------------------------------------------
// Device-side failure record of a factorisation (one per batch item): the reference aborts on the first
// non-positive / non-finite Cholesky pivot (src/linalg.rs:215-219); kernels check `err` and become no-ops
// after a failure so the host can report it after one synchronisation.
struct FactorStatus {
    int err;       // 0 ok, 1 not positive definite
    int pivot;     // pivot index j of the failing diagonal element
    double value;  // the non-positive / non-finite value d
};

// Host helpers (defined in engine.cu)
int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
std::string rust_exp(double v);  // Rust's `{:e}` formatting of an f64

#define CDCLQ_CUDA_TRY(expr)                                         \
    do {                                                             \
        cudaError_t _e = (expr);                                     \
        if (_e != cudaSuccess) return ::cdclq::cuda_error(_e, #expr); \
    } while (0)

}  // namespace cdclq
