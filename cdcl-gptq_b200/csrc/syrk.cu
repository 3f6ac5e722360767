// syrk.cu - Hessian accumulation H += X^T X from bf16 activations on the tcgen05 tensor cores.
#include "common.cuh"
#include "kernels.h"

namespace cdclq {

int launch_gram_bf16_tc(const void* x, int64_t t, int n, double* h, int lower_only, cudaStream_t st) {
    (void)x; (void)t; (void)n; (void)h; (void)lower_only; (void)st;
    return set_error(CDCLQ_ERR_CUDA, "the bf16 tensor-core Gram kernel is not part of this build yet");
}

}  // namespace cdclq
