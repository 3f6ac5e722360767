// repair.cu - phase 2: conflict selection and the monotone CDCL repair (src/engine.rs:478-671).
//
// Work decomposition.  The reference runs phase 2 per row chunk (rc rows): conflict selection sums eps^2
// over the chunk's rows and the `tol` stop is decided per chunk (src/engine.rs:499-508, 663).  Inside one pass
// every move (scale refit of a (row, group), code move of a (row, column)) depends only on its own row, so a
// chunk's rows are processed in TILES of BM rows (BM = 64 or 128, a compile-time parameter of the kernels)
// whose per-pass loss deltas are added in tile order.  Three launch modes share the tile code:
//   A  one launch per pass over 64-row slices, a pass-end kernel reducing each chunk's slices in order (few
//      chunks: a chunk's rows spread over several SMs);
//   B  persistent: a CTA takes whole chunks from a counter (heaviest first) and runs all their passes;
//   C  persistent 2-CTA clusters: the tiles of a chunk of several tiles are split over two SMs.
//
// Inside a tile (256 threads):
//   * the block gradients G = E H[:, c0:c1] run on the FP32 GEMM core (fixed k order, bit-exact);
//   * the sequential per-row work (refit numerators/denominators, the coordinate sweep with its rank-1
//     gradient updates) runs one thread per row, in the reference's order, on shared-memory tiles.
#include "repair_core.cuh"

namespace cdclq {

// ---------------------------------------------------------------------------------------------------------
// Per-chunk statistics after phase 1: colloss (rows summed in order), loss_gptq, sub-block sums, conflict
// selection (src/engine.rs:478-511), and E = W - W_hat (src/engine.rs:516-519).
__global__ void __launch_bounds__(256) chunk_stats_kernel(const ChunkInfo* __restrict__ chunks, RepairParams rp) {
    const ChunkInfo ci = chunks[blockIdx.x];
    const int n = ci.n, rows = ci.rows, tid = threadIdx.x, nt = blockDim.x;
    const float* eps2 = ci.e;
    for (int j = tid; j < n; j += nt) {
        double cl = 0.0;
        for (int r = 0; r < rows; r++) cl = __dadd_rn(cl, (double)eps2[(int64_t)r * n + j]);
        ci.colloss[j] = cl;
    }
    __syncthreads();
    if (tid == 0) {
        double lg = 0.0;
        for (int j = 0; j < n; j++) lg = __dadd_rn(lg, ci.colloss[j]);
        ci.st->loss_gptq = lg;
        ci.st->loss_delta = 0.0;
        ci.st->prev_delta = 0.0;
        ci.st->updates = 0ull;
        ci.st->passes = 0;
        ci.st->n_sel = 0;
        // a chunk with nothing to repair never enters a pass
        ci.st->done = (rp.method_cdcl && (rp.do_cd || rp.do_refit)) ? 0 : 1;
    }
    const int sbw = ci.sbw, n_sb = ci.n_sb;
    for (int s = tid; s < n_sb; s += nt) {
        int c0 = s * sbw, c1 = min(c0 + sbw, n);
        double acc = 0.0;
        for (int j = c0; j < c1; j++) acc = __dadd_rn(acc, ci.colloss[j]);
        ci.sbsum[s] = acc;
    }
    __syncthreads();
    if (rp.method_cdcl && rp.do_cd) {
        // rank of each sub-block in (descending loss, ascending index) order; the k best are selected and
        // kept in ascending index order (src/engine.rs:506-509)
        for (int s = tid; s < n_sb; s += nt) {
            double v = ci.sbsum[s];
            int rank = 0;
            for (int s2 = 0; s2 < n_sb; s2++) {
                double v2 = ci.sbsum[s2];
                rank += (v2 > v || (v2 == v && s2 < s)) ? 1 : 0;
            }
            ci.sel[s] = (rank < ci.k_sel) ? 1 : 0;  // flag first, compacted below
        }
        __syncthreads();
        if (tid == 0) {
            int cnt = 0;
            for (int s = 0; s < n_sb; s++)
                if (ci.sel[s]) ci.sel[cnt++] = s;  // in place: cnt <= s
            ci.st->n_sel = cnt;
        }
    }
    __syncthreads();
    if (rp.method_cdcl && (rp.do_cd || rp.do_refit)) {
        int64_t total = (int64_t)rows * n;
        for (int64_t i = tid; i < total; i += nt) ci.e[i] = __fsub_rn(ci.wt[i], ci.wq[i]);
    }
}

int launch_chunk_stats(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, cudaStream_t st) {
    if (nchunks == 0) return 0;
    CDCLQ_LAUNCH(chunk_stats_kernel, nchunks, 256, 0, st, chunks_dev, rp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "chunk_stats_kernel launch");
}


size_t repair_smem_bytes(int g, int sbw, int bm) {
    return bm == 128 ? repair_layout<128>(g, sbw).total : repair_layout<64>(g, sbw).total;
}


// ---------------------------------------------------------------------------------------------------------
// Mode A - one launch per pass over 64-row slices (used when there are few row chunks, so that a chunk's
// rows spread over several SMs); pass_end_kernel then reduces each chunk's slices in order.
__global__ void __launch_bounds__(256, 2) repair_pass_kernel(const ChunkInfo* __restrict__ chunks,
                                                             const SliceItem* __restrict__ slices,
                                                             SliceAcc* __restrict__ acc_out, RepairParams rp) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ ChunkInfo ci;  // chunk descriptor kept on chip (not in registers across the tile loops)
    const SliceItem sl = slices[blockIdx.x];
    if (threadIdx.x == 0) ci = chunks[sl.chunk];
    __syncthreads();
    if (!rp.final_refit && ci.st->done) return;  // this chunk has converged (src/engine.rs:663-665)
    const TileSmem sm = tile_smem<64>(smem_raw, ci.g, ci.sbw);
    double d;
    unsigned long long u;
    run_tile<64>(ci, sl.r0, sl.rs, rp, rp.final_refit != 0, sm, d, u);
    if (threadIdx.x == 0) {
        acc_out[blockIdx.x].delta = d;
        acc_out[blockIdx.x].updates = u;
    }
}

// Mode B - persistent: each CTA takes whole row chunks from a counter (heaviest first) and runs all of a
// chunk's passes, its stop rule and its final refit itself, so no launch-wide barrier separates passes.  The
// arithmetic is that of mode A; the pass delta adds the BM-row tiles' sums in tile order.

int repair_tile_rows(int g, int sbw, int max_rows) {
    if (max_rows <= 64) return 64;
    // 128-row tiles only while two CTAs still fit on one SM
    return repair_persistent_ctas_per_sm_bm128(repair_smem_bytes(g, sbw, 128)) >= 2 ? 128 : 64;
}

int launch_repair_pass(const ChunkInfo* chunks_dev, const SliceItem* slices_dev, int nslices, SliceAcc* acc_dev,
                       const RepairParams& rp, int g, int sbw, cudaStream_t st) {
    if (nslices == 0) return 0;
    size_t smem = repair_smem_bytes(g, sbw, 64);
    int rc = set_repair_smem((const void*)repair_pass_kernel, smem);
    if (rc) return rc;
    CDCLQ_LAUNCH(repair_pass_kernel, nslices, 256, smem, st, chunks_dev, slices_dev, acc_dev, rp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "repair_pass_kernel launch");
}

int launch_repair_cluster(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw, int bm,
                          int* counter_dev, cudaStream_t st, int max_ctas, size_t smem_floor) {
    if (nchunks == 0) return 0;
    size_t smem = repair_smem_bytes(g, sbw, bm);
    if (smem < smem_floor) smem = smem_floor;  // reserved, unused: keeps other CTAs off the SM
    return bm == 128 ? launch_repair_cluster_bm128(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas)
                     : launch_repair_cluster_bm64(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int launch_repair_quad(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw,
                       int* counter_dev, cudaStream_t st, int max_ctas, size_t smem_floor) {
    if (nchunks == 0) return 0;
    size_t smem = repair_smem_bytes(g, sbw, 64);
    if (smem < smem_floor) smem = smem_floor;
    return launch_repair_quad_bm64(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

int launch_repair_persistent(const ChunkInfo* chunks_dev, int nchunks, const RepairParams& rp, int g, int sbw, int bm,
                             int* counter_dev, cudaStream_t st, int max_ctas) {
    if (nchunks == 0) return 0;
    size_t smem = repair_smem_bytes(g, sbw, bm);
    return bm == 128 ? launch_repair_persistent_bm128(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas)
                     : launch_repair_persistent_bm64(chunks_dev, nchunks, rp, smem, counter_dev, st, max_ctas);
}

// ---------------------------------------------------------------------------------------------------------
// Per-chunk end of a pass: add the slices' deltas in order, then the reference's stop rule
// `pass_updates == 0 || gain < tol * (loss_gptq + loss_delta)` (src/engine.rs:660-665).  For the final refit
// only the bookkeeping is updated (src/engine.rs:668-670).
__global__ void pass_end_kernel(const ChunkInfo* __restrict__ chunks, int nchunks, const int* __restrict__ slice_begin,
                                const SliceAcc* __restrict__ acc, RepairParams rp) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= nchunks) return;
    ChunkState* st = chunks[c].st;
    if (!rp.final_refit && st->done) return;
    if (rp.final_refit && !(rp.method_cdcl && rp.do_refit)) return;
    double d = 0.0;
    unsigned long long u = 0ull;
    for (int s = slice_begin[c]; s < slice_begin[c + 1]; s++) {
        d = __dadd_rn(d, acc[s].delta);
        u += acc[s].updates;
    }
    if (rp.final_refit) {
        st->loss_delta = __dadd_rn(st->loss_delta, d);
        st->updates += u;
        return;
    }
    apply_pass(st, d, u, rp.tol);
}

int launch_pass_end(const ChunkInfo* chunks_dev, int nchunks, const int* slice_begin_dev, const SliceAcc* acc_dev,
                    const RepairParams& rp, cudaStream_t st) {
    if (nchunks == 0) return 0;
    int threads = 128, blocks = (nchunks + threads - 1) / threads;
    CDCLQ_LAUNCH(pass_end_kernel, blocks, threads, 0, st, chunks_dev, nchunks, slice_begin_dev, acc_dev, rp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : cuda_error(e, "pass_end_kernel launch");
}

}  // namespace cdclq
