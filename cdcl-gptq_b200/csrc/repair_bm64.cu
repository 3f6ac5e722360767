// repair_bm64.cu - the persistent repair kernels (modes B and C) instantiated for 64-row tiles.
#include "repair_core.cuh"

namespace cdclq {

int launch_repair_persistent_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                                  int* counter_dev, cudaStream_t st, int max_ctas) {
    return launch_persistent_bm<64>(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int launch_repair_cluster_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                               int* counter_dev, cudaStream_t st, int max_ctas) {
    return launch_cluster_bm<64>(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int launch_repair_quad_bm64(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, size_t smem,
                            int* counter_dev, cudaStream_t st, int max_ctas) {
    return launch_quad_bm<64>(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

}  // namespace cdclq
