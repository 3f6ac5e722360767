// syrk.cu - Hessian accumulation H += X^T X from bf16 activations on the tcgen05 tensor cores
// (src/linalg.rs:388-418, symmetric use x == y).
//
// The reference multiplies f32 activations in token chunks of 2048 (f32 products summed in f32) and widens each
// chunk's sum into the f64 Hessian.  Here each 2048-token chunk is one f32 tensor-core accumulation in tensor
// memory (bf16 x bf16 products are exact in f32; the summation order inside the tensor core differs from a
// sequential sum, so this path agrees with the f32 path to f32 accumulation error, not bit for bit), then the
// epilogue widens the chunk into the f64 Hessian in global memory, as the reference does.  Only the lower
// triangle is accumulated; when the full matrix is wanted, one pass at the end copies it onto the upper triangle
// (the reference's H is symmetric: both triangles receive the same sums in the same order).
//
// One CTA computes output tiles D[p][q] = sum_t X[t][p] X[t][q] of 128 (p) x 256 (q) channels with q >= p
// somewhere in the tile, tiles taken round-robin by a persistent grid.  Per 64-token K block, TMA brings the
// p block (2 boxes of 64 channels x 64 tokens) and the q block (4 boxes) into a 3-stage shared-memory ring
// (128-byte swizzle, MN-major for the MMA: channels are contiguous in X); one thread issues four
// 128x256x16 bf16 MMAs per block into a tensor-memory accumulator.  Two accumulators (2 x 256 columns) let the
// eight epilogue warps widen chunk c while the MMAs of chunk c+1 run.  D[p][q] is added into H[q][p] for
// q >= p (TMEM lane p = one element of a row of H): off the diagonal by bulk f64 additions at L2 from a
// shared-memory staging buffer, each tile's chunks in order (a chunk's additions complete before the next
// chunk's are issued), so every element receives the same sums in the same order as a sequential widening.
//
// Roles: warps 0-7 epilogue (warp w reads TMEM lanes 32(w%4).. and columns 128(w/4)..), warp 8 TMA producer,
// warp 9 MMA issuer and TMEM owner.  Every wait on an mbarrier is bounded: on timeout the kernel records an error, leaves its loops,
// waits (bounded) for its own copies and MMAs in flight, frees its tensor memory and returns.  No TMA multicast.
#include <cuda.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace cdclq {

namespace syrk {

constexpr int BMP = 128;         // tile rows p (TMEM lanes)
constexpr int BNQ = 256;         // tile columns q
constexpr int KB = 64;           // tokens per K block (one TMA box height)
constexpr int CHUNK = 2048;      // tokens per f32 accumulation (src/linalg.rs:392)
constexpr int NS = 3;            // shared-memory stages
constexpr int BOX_BYTES = 64 * KB * 2;              // 64 channels x 64 tokens bf16 = 8 KB
constexpr int A_BYTES = 2 * BOX_BYTES;              // 128 channels
constexpr int B_BYTES = 4 * BOX_BYTES;              // 256 channels
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;      // 48 KB
constexpr int EPI_WARPS = 8;     // two per TMEM lane quadrant, each taking half of the tile's columns
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr int TMEM_COLS = 2 * BNQ;                  // two accumulators
constexpr int EPI_BUF_BYTES = 16 * 32 * 8;           // 16 rows q x 32 columns p of f64: one epilogue staging buffer
constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF_BYTES;  // two buffers per epilogue warp (64 KB)
constexpr size_t smem_bytes(int ns) {
    return (size_t)ns * STAGE_BYTES + EPI_BYTES + 1024 /* alignment */ + 256 /* barriers */;
}
constexpr int WAIT_LIMIT = 1 << 24;
constexpr int TILE_BAND = 16;    // p blocks per band of the tile order

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(smem_u32(b)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the completion of the phase with the given parity; false (and the error flag set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int* err) {
    for (int it = 0; it < WAIT_LIMIT; it++) {
        if (mbar_try(b, parity)) return true;
        if ((it & 1023) == 1023 && *(volatile int*)err) return false;  // another role gave up
    }
    atomicExch(err, 1);
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Bulk f64 additions from shared memory into global memory, performed at L2 (round to nearest, as __dadd_rn).
__device__ __forceinline__ void bulk_add_f64(double* gdst, uint32_t ssrc, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f64 [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every bulk operation of this thread has completed (its additions are performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// at most the most recent bulk group of this thread still reads its shared-memory source
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor of an MN-major operand with the 128-byte swizzle: 64-element (128-byte) atoms
// along MN, `lbo` bytes apart; 8-token row groups along K, `sbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}

// Instruction descriptor: D f32, A and B both bf16 (BF16) or both f16, both MN-major, M = 128, N = 256.
template <bool BF16>
__host__ __device__ constexpr uint32_t idesc() {
    return (1u << 4) | ((BF16 ? 1u : 0u) << 7) | ((BF16 ? 1u : 0u) << 10) | (1u << 15) | (1u << 16) |
           ((uint32_t)(BNQ >> 3) << 17) | ((uint32_t)(BMP >> 4) << 24);
}

template <bool BF16>
__device__ __forceinline__ void mma_half(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc<BF16>()), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

struct Params {
    double* h;
    int n;
    int64_t t;
    int tiles_p;   // p blocks
    int tiles_q;   // q blocks
    const int2* tiles;  // (p block, q block) of each tile in processing order
    int ntiles;    // tiles with q >= p somewhere
    int lower_only;
    int nseg;        // token segments per tile (split over CTAs when there are few tiles)
    int cps;         // chunks per segment
    double* scratch; // nseg > 1: per (segment, tile) f64 partial sums, [q][p] within a tile
    int* err;
};

// Work item -> (tile, chunk range); items are segment-major so that the CTAs of a wave read the same tokens.
__device__ __forceinline__ void item_range(const Params& P, int item, int nchunks, int& tile, int& c0, int& c1) {
    const int seg = item / P.ntiles;
    tile = item - seg * P.ntiles;
    c0 = seg * P.cps;
    c1 = min(nchunks, c0 + P.cps);
}


__device__ __forceinline__ void tile_coords(const Params& P, int tile, int& pb, int& qb) {
    const int2 t = P.tiles[tile];
    pb = t.x;
    qb = t.y;
}

template <int NSTAGES, bool BF16>
__global__ void __launch_bounds__(THREADS, 1) syrk_bf16_kernel(const __grid_constant__ CUtensorMap tmap, const Params P) {
    constexpr int NS = NSTAGES;  // shared-memory stages
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char* epi_base = base + NS * STAGE_BYTES;  // epilogue staging buffers
    uint64_t* full = reinterpret_cast<uint64_t*>(epi_base + EPI_BYTES);
    uint64_t* empty = full + NS;
    uint64_t* accf = empty + NS;
    uint64_t* acce = accf + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int* err = P.err;

    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], EPI_WARPS * 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == EPI_WARPS + 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"((uint32_t)TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    const int n = P.n;
    const int64_t T = P.t;
    const int nchunks = (int)((T + CHUNK - 1) / CHUNK);

    if (warp == EPI_WARPS) {
        // ---------------- TMA producer
        if (lane == 0) {
            int ctr = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < P.ntiles * P.nseg && ok; item += gridDim.x) {
                int tile, c0, c1, pb, qb;
                item_range(P, item, nchunks, tile, c0, c1);
                tile_coords(P, tile, pb, qb);
                const int p0 = pb * BMP, q0 = qb * BNQ;
                for (int c = c0; c < c1 && ok; c++) {
                    const int64_t tok0 = (int64_t)c * CHUNK;
                    const int nkb = (int)((min((int64_t)CHUNK, T - tok0) + KB - 1) / KB);
                    for (int kb = 0; kb < nkb; kb++, ctr++) {
                        const int s = ctr % NS;
                        if (ctr >= NS && !mbar_wait(&empty[s], ((ctr / NS) - 1) & 1, err)) {
                            ok = false;
                            break;
                        }
                        unsigned char* st = base + s * STAGE_BYTES;
                        mbar_expect_tx(&full[s], STAGE_BYTES);
                        const int y = (int)(tok0 + (int64_t)kb * KB);
                        tma_load_2d(st, &tmap, p0, y, &full[s]);
                        tma_load_2d(st + BOX_BYTES, &tmap, p0 + 64, y, &full[s]);
#pragma unroll
                        for (int h = 0; h < 4; h++)
                            tma_load_2d(st + A_BYTES + h * BOX_BYTES, &tmap, q0 + 64 * h, y, &full[s]);
                    }
                }
            }
            // copies still in flight land before the CTA leaves (bounded)
            for (int k = (ctr > NS ? ctr - NS : 0); k < ctr; k++) mbar_wait(&full[k % NS], (k / NS) & 1, err);
        }
    } else if (warp == EPI_WARPS + 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            int ctr = 0, acc = 0;
            bool ok = true;
            const uint32_t a_base = smem_u32(base);
            for (int item = blockIdx.x; item < P.ntiles * P.nseg && ok; item += gridDim.x) {
                int tile, c0, c1;
                item_range(P, item, nchunks, tile, c0, c1);
                for (int c = c0; c < c1 && ok; c++, acc++) {
                    const int b = acc & 1;
                    if (acc >= 2 && !mbar_wait(&acce[b], ((acc / 2) - 1) & 1, err)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t d = tmem_base + (uint32_t)(b * BNQ);
                    const int64_t tok0 = (int64_t)c * CHUNK;
                    const int nkb = (int)((min((int64_t)CHUNK, T - tok0) + KB - 1) / KB);
                    for (int kb = 0; kb < nkb; kb++, ctr++) {
                        const int s = ctr % NS;
                        if (!mbar_wait(&full[s], (ctr / NS) & 1, err)) {
                            ok = false;
                            mma_commit(&accf[b]);  // tracks the MMAs already issued for this chunk
                            acc++;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t sa = a_base + s * STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                        for (int k = 0; k < KB / 16; k++)
                            mma_half<BF16>(d, smem_desc(sa + k * 2048, BOX_BYTES, 1024), smem_desc(sb + k * 2048, BOX_BYTES, 1024),
                                     (kb | k) != 0 ? 1u : 0u);
                        mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                    }
                    if (!ok) break;
                    mma_commit(&accf[b]);  // accumulator b holds chunk c
                }
            }
            // every issued MMA has completed before the tensor memory is released (bounded)
            if (acc > 0) mbar_wait(&accf[(acc - 1) & 1], ((acc - 1) / 2) & 1, err);
        }
    } else {
        // ---------------- epilogue: warps 0..7; TMEM lanes 32*(warp%4) .., columns 128*(warp/4) ..
        // Each 32 (p) x 32 (q) block of the chunk is widened to f64.  Into H, a block wholly below the diagonal goes
        // through the warp's staging buffers into bulk additions performed at L2 (one 256-byte row segment
        // H[q][p..p+31] per q) - against a read-modify-write from the SM this moved n = 4096 from 650 to 1000
        // TFLOP/s; the diagonal block is added element by element (q >= p only).  With split tokens the item's
        // partial tile in the scratch, [q - q0][p - p0], is written element by element.
        const int quad = warp & 3, half = warp >> 2;
        double* ebuf = reinterpret_cast<double*>(epi_base + (size_t)warp * 2 * EPI_BUF_BYTES);
        const uint32_t ebuf_s = smem_u32(ebuf);
        int bi = 0;  // the staging buffer filled next
        int acc = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < P.ntiles * P.nseg && ok; item += gridDim.x) {
            int tile, c0, c1, pb, qb;
            item_range(P, item, nchunks, tile, c0, c1);
            tile_coords(P, tile, pb, qb);
            const int p0 = pb * BMP, q0 = qb * BNQ;
            const int prow0 = p0 + quad * 32;  // this warp's 32 rows p
            const int p = prow0 + lane;
            const bool split = P.nseg > 1;
            double* dst = split ? P.scratch + (int64_t)item * (BMP * BNQ) : P.h;
            const int64_t ld = split ? BMP : n;
            const int qofs = split ? q0 : 0, pofs = split ? p0 : 0;
            for (int c = c0; c < c1; c++, acc++) {
                const int b = acc & 1;
                if (!mbar_wait(&accf[b], (acc / 2) & 1, err)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                // the previous chunk's additions have been performed: every element receives its chunks in order
                if (lane == 0) bulk_wait_all();
                __syncwarp();
                for (int cb = half * (BNQ / 64); cb < (half + 1) * (BNQ / 64); cb++) {
                    const int qc0 = q0 + cb * 32;
                    float v[32];
                    tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BNQ + cb * 32), v);
                    if (qc0 + 31 < prow0 || prow0 >= n) continue;  // the whole block has q < p, or no row p < n
                    if (split || qc0 == prow0) {
                        // element by element, q >= p: the first chunk of a split partial is stored, every other
                        // chunk added (all loads before any store).  A split partial is private to its CTA and
                        // L2-resident while its segment runs; its bulk additions measured slower than this.
                        if (split && c == c0) {
#pragma unroll
                            for (int i = 0; i < 32; i++) {
                                const int q = qc0 + i;
                                if (p < n && q < n && q >= p) dst[(int64_t)(q - qofs) * ld + (p - pofs)] = (double)v[i];
                            }
                            continue;
                        }
                        double old[32];
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const int q = qc0 + i;
                            old[i] = (p < n && q < n && q >= p) ? dst[(int64_t)(q - qofs) * ld + (p - pofs)] : 0.0;
                        }
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const int q = qc0 + i;
                            if (p < n && q < n && q >= p)
                                dst[(int64_t)(q - qofs) * ld + (p - pofs)] = __dadd_rn(old[i], (double)v[i]);
                        }
                        continue;
                    }
                    const uint32_t bytes = (uint32_t)min(32, n - prow0) * 8u;  // n % 8 == 0: a multiple of 64
#pragma unroll
                    for (int hb = 0; hb < 2; hb++) {
                        if (lane == 0) bulk_wait_read_le1();  // this buffer's previous additions have read it
                        __syncwarp();
                        double* buf = ebuf + bi * (EPI_BUF_BYTES / 8);
#pragma unroll
                        for (int i = 0; i < 16; i++) buf[i * 32 + lane] = (double)v[hb * 16 + i];
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            for (int i = 0; i < 16; i++) {
                                const int q = qc0 + hb * 16 + i;
                                if (q < n)
                                    bulk_add_f64(dst + (int64_t)(q - qofs) * ld + (prow0 - pofs),
                                                 ebuf_s + (uint32_t)(bi * EPI_BUF_BYTES + i * 256), bytes);
                            }
                            bulk_commit();
                        }
                        bi ^= 1;
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                mbar_arrive(&acce[b]);
            }
        }
        if (lane == 0) bulk_wait_all();  // the additions are performed before the CTA leaves
    }

    // teardown: every role is done with the tensor memory
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == EPI_WARPS + 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)TMEM_COLS));
}

}  // namespace syrk

namespace syrk {

// Split tiles: H[q][p] += partial_0 + partial_1 + ... (segments in order), q >= p.
// Block = 128 threads (p within the tile), grid = (tiles, 256 / 32 column groups).
__global__ void __launch_bounds__(128) syrk_reduce_kernel(const Params P) {
    const int tile = blockIdx.x;
    int pb, qb;
    tile_coords(P, tile, pb, qb);
    const int pl = threadIdx.x, p = pb * BMP + pl, n = P.n;
    if (p >= n) return;
    for (int ql = blockIdx.y * 32; ql < blockIdx.y * 32 + 32; ql++) {
        const int q = qb * BNQ + ql;
        if (q >= n || q < p) continue;
        double lo = P.h[(int64_t)q * n + p];
        for (int sg = 0; sg < P.nseg; sg++)
            lo = __dadd_rn(lo, P.scratch[((int64_t)sg * P.ntiles + tile) * (BMP * BNQ) + (int64_t)ql * BMP + pl]);
        P.h[(int64_t)q * n + p] = lo;
    }
}

// Full-matrix result: the upper triangle becomes the lower one's mirror, H[p][q] = H[q][p] for q > p, through
// 32 x 32 shared-memory tiles (reads and writes coalesced).  Grid (T, T) blocks of 32 x 8 threads, T = n / 32
// rounded up; the blocks above the diagonal exit.
__global__ void __launch_bounds__(256) syrk_mirror_kernel(double* h, int n) {
    const int bi = blockIdx.y, bj = blockIdx.x;  // source tile: rows 32 bi.., columns 32 bj.. (lower: bj <= bi)
    if (bj > bi) return;
    __shared__ double t[32][33];
    const int tx = threadIdx.x, ty = threadIdx.y;
    for (int r = ty; r < 32; r += 8) {
        const int row = bi * 32 + r, col = bj * 32 + tx;
        if (row < n && col < n) t[r][tx] = h[(int64_t)row * n + col];
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int row = bj * 32 + r, col = bi * 32 + tx;  // destination H[row][col] = H[col][row], col > row
        if (row < n && col < n && col > row) h[(int64_t)row * n + col] = t[tx][r];
    }
}

}  // namespace syrk

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

int launch_gram_half_tc(const void* x, bool bf16, int64_t t, int n, double* h, int lower_only, cudaStream_t st) {
    using namespace syrk;
    if (t <= 0) return 0;
    if (n % 8 != 0) return set_error(CDCLQ_ERR_ARG, "half Gram: n must be a multiple of 8 (16-byte rows)");
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return set_error(CDCLQ_ERR_ARG, "half Gram: x must be 16-byte aligned");
    if (t > 0x7fffffffLL - CHUNK) return set_error(CDCLQ_ERR_ARG, "half Gram: too many tokens for one call");
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return set_error(CDCLQ_ERR_CUDA, "half Gram: cuTensorMapEncodeTiled is unavailable");
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)t};
    cuuint64_t strides[1] = {(cuuint64_t)n * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)KB};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = enc(&map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(CDCLQ_ERR_CUDA, "half Gram: tensor map encoding failed");
    Params P;
    P.h = h;
    P.n = n;
    P.t = t;
    P.tiles_p = (n + BMP - 1) / BMP;
    P.tiles_q = (n + BNQ - 1) / BNQ;
    P.ntiles = 0;
    // Tiles (p block, q block) holding some q >= p, in bands of TILE_BAND p blocks; within a band q block by
    // q block.  Consecutive tiles share the q block (B operand), and a wave of one tile per SM spans about
    // TILE_BAND p blocks x (SMs / TILE_BAND) q blocks, so each token chunk of X that a wave reads is a small part
    // of the n channels and stays in L2 for every tile of the wave that needs it.
    std::vector<int2> order;
    for (int b0 = 0; b0 < P.tiles_p; b0 += TILE_BAND) {
        const int b1 = std::min(P.tiles_p, b0 + TILE_BAND);
        for (int qb = b0 >> 1; qb < P.tiles_q; qb++)
            for (int pb = b0; pb < b1; pb++)
                if ((pb >> 1) <= qb) order.push_back(make_int2(pb, qb));
    }
    P.ntiles = (int)order.size();
    P.lower_only = lower_only ? 1 : 0;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // fewer tiles than SMs (small n): split each tile's tokens into segments so that every SM gets about four
    // items; with a wave or more of tiles the per-segment partials cost more than the idle tail saves
    const int nchunks = (int)((t + CHUNK - 1) / CHUNK);
    int nseg = P.ntiles >= sms ? 1 : (4 * sms + P.ntiles - 1) / P.ntiles;
    if (nseg > nchunks) nseg = nchunks;
    if (nseg < 1) nseg = 1;
    P.cps = (nchunks + nseg - 1) / nseg;
    P.nseg = (nchunks + P.cps - 1) / P.cps;
    P.scratch = nullptr;
    if (P.nseg > 1) {
        const size_t sb = sizeof(double) * (size_t)P.nseg * P.ntiles * BMP * BNQ;
        CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&P.scratch, sb, st));
    }
    // one allocation: the error flag, then the tile order
    int* err = nullptr;
    const size_t tiles_off = 16;
    CDCLQ_CUDA_TRY(cudaMallocAsync((void**)&err, tiles_off + order.size() * sizeof(int2), st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
    int2* tiles_dev = reinterpret_cast<int2*>(reinterpret_cast<char*>(err) + tiles_off);
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(tiles_dev, order.data(), order.size() * sizeof(int2), cudaMemcpyHostToDevice, st));
    P.err = err;
    P.tiles = tiles_dev;
    auto kern = bf16 ? syrk_bf16_kernel<NS, true> : syrk_bf16_kernel<NS, false>;
    const size_t smem = smem_bytes(NS);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
        cudaFreeAsync(err, st);
        if (P.scratch) cudaFreeAsync(P.scratch, st);
        return cuda_error(e, "bf16 Gram smem attribute");
    }
    const int items = P.ntiles * P.nseg;
    const int grid = items < sms ? items : sms;
    CDCLQ_LAUNCH(kern, grid, THREADS, smem, st, map, P);
    e = cudaGetLastError();
    if (e == cudaSuccess && P.nseg > 1) {
        dim3 rg(P.ntiles, BNQ / 32);
        CDCLQ_LAUNCH(syrk_reduce_kernel, rg, BMP, 0, st, P);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && !P.lower_only) {
        const int tt = (n + 31) / 32;
        CDCLQ_LAUNCH(syrk_mirror_kernel, dim3(tt, tt), dim3(32, 8), 0, st, h, n);
        e = cudaGetLastError();
    }
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaFreeAsync(err, st);
    if (P.scratch) cudaFreeAsync(P.scratch, st);
    if (e != cudaSuccess) return cuda_error(e, "syrk_bf16_kernel");
    if (herr) return set_error(CDCLQ_ERR_CUDA, "half Gram: a pipeline wait timed out (kernel abandoned its tiles)");
    return 0;
}

}  // namespace cdclq
