// repair_bm128.cu - the persistent repair kernels (modes B and C) instantiated for 128-row tiles.
#include "repair_core.cuh"

namespace cdclq {

int launch_repair_persistent_bm128(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                  int* counter_dev, cudaStream_t st, int max_ctas) {
    return launch_persistent_bm<128>(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int launch_repair_cluster_bm128(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                               int* counter_dev, cudaStream_t st, int max_ctas) {
    return launch_cluster_bm<128>(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int repair_persistent_ctas_per_sm_bm128(size_t smem) { return persistent_ctas_per_sm<128>(smem); }

}  // namespace cdclq
