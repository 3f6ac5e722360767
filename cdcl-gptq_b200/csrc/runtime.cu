// runtime.cu - the multi-GPU runtime of the C ABI (cdclq_runtime*): one process per GPU, an NCCL communicator
// owned by the library, and the model-level batch sharded over the ranks.
//
// The reference runs on one host: pipeline::quantize_model walks the layers sequentially and the engine splits
// each layer's rows over the rayon pool (src/pipeline.rs:121-175, src/engine.rs:768-782).  Over several GPUs the
// same independence structure is used: every layer's rows are split in whole row chunks (rows are independent,
// src/engine.rs:9-15; conflict selection and the tol stop are per row chunk, so chunk boundaries never move), the
// distinct inputs' factorisations are spread over the ranks and each factor U is broadcast from its owner over
// NVLink, and the per-layer statistics are all-reduced.  Results equal a single-GPU run's.
//
// NCCL is resolved at run time (dlopen): a process that already loaded NCCL (torch) shares that copy, a process
// that has not yet loads the copy CDCLQ_NCCL_LIBRARY names (else libnccl.so.2 from the loader's path), and the
// library has no link-time dependency on it.  The communicator is non-blocking, so that every wait
// - communicator creation included - is bounded by the runtime's timeout; on a timeout or an NCCL failure the
// communicator is aborted and every call on the runtime fails from then on.
#include <dlfcn.h>
#include <nccl.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "cdclq.h"
#include "common.cuh"
#include "kernels.h"
#include "runtime.h"

namespace cdclq {

// ---- NCCL, resolved at run time -------------------------------------------------------------------------
namespace {

struct Nccl {
    bool loaded = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;  // optional (NCCL >= 2.14)
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

Nccl& nccl() {
    static Nccl api;
    static std::once_flag once;
    std::call_once(once, [] {
        // an NCCL already in the process first (a framework's: a second copy under the same soname would shadow
        // the one the framework needs), then CDCLQ_NCCL_LIBRARY (a path: the copy the caller's framework will
        // load), then the loader's search path
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        const char* env = getenv("CDCLQ_NCCL_LIBRARY");
        if (!h && env && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.why = std::string("NCCL not found (libnccl.so.2): ") + dlerror();
            return;
        }
        bool ok = true;
        auto sym = [&](const char* name) {
            void* p = dlsym(h, name);
            if (!p) ok = false;
            return p;
        };
        api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
        api.CommInitRankConfig = (decltype(api.CommInitRankConfig))sym("ncclCommInitRankConfig");
        api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
        api.CommFinalize = (decltype(api.CommFinalize))dlsym(h, "ncclCommFinalize");
        api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
        api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
        api.Broadcast = (decltype(api.Broadcast))sym("ncclBroadcast");
        api.AllReduce = (decltype(api.AllReduce))sym("ncclAllReduce");
        api.Send = (decltype(api.Send))sym("ncclSend");
        api.Recv = (decltype(api.Recv))sym("ncclRecv");
        api.GroupStart = (decltype(api.GroupStart))sym("ncclGroupStart");
        api.GroupEnd = (decltype(api.GroupEnd))sym("ncclGroupEnd");
        api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
        if (!ok) {
            api.why = "NCCL library lacks a required symbol (need NCCL >= 2.14)";
            return;
        }
        api.loaded = true;
    });
    return api;
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int nccl_error(Runtime* rt, ncclResult_t r, const char* what) {
    Nccl& N = nccl();
    std::string m = std::string("NCCL error in ") + what + ": " + (N.GetErrorString ? N.GetErrorString(r) : "?");
    if (rt && rt->comm && !rt->broken) {
        N.CommAbort((ncclComm_t)rt->comm);
        rt->comm = nullptr;
        rt->broken = true;
    }
    return set_error(CDCLQ_ERR_CUDA, m);
}

// Non-blocking communicator: wait until the last NCCL call has been issued (or fail / time out).
int nccl_settle(Runtime* rt, ncclResult_t r, const char* what) {
    Nccl& N = nccl();
    if (r != ncclSuccess && r != ncclInProgress) return nccl_error(rt, r, what);
    const double t0 = now_s();
    for (;;) {
        ncclResult_t s = ncclSuccess;
        ncclResult_t q = N.CommGetAsyncError((ncclComm_t)rt->comm, &s);
        if (q != ncclSuccess) return nccl_error(rt, q, what);
        if (s == ncclSuccess) return 0;
        if (s != ncclInProgress) return nccl_error(rt, s, what);
        if (now_s() - t0 > rt->timeout_s) {
            nccl_error(rt, ncclInProgress, what);
            return set_error(CDCLQ_ERR_CUDA, std::string("timed out after ") + std::to_string((int)rt->timeout_s) +
                                                 " s waiting for the other ranks (" + what + ")");
        }
        usleep(200);
    }
}

int check_rt(Runtime* rt) {
    if (!rt) return set_error(CDCLQ_ERR_ARG, "null runtime");
    if (rt->broken) return set_error(CDCLQ_ERR_CUDA, "the runtime's communicator was aborted after an earlier failure");
    cudaError_t e = cudaSetDevice(rt->device);
    if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    return 0;
}

}  // namespace

// ---- sharding and ownership -----------------------------------------------------------------------------
void shard_rows(size_t d_out, size_t row_chunk, int rank, int nranks, size_t rotate, size_t* r0, size_t* r1) {
    const size_t rc = std::max<size_t>(row_chunk, 1);
    const size_t chunks = (d_out + rc - 1) / rc;
    const size_t v = ((size_t)rank + rotate) % (size_t)nranks;
    const size_t c0 = chunks * v / (size_t)nranks, c1 = chunks * (v + 1) / (size_t)nranks;
    *r0 = std::min(c0 * rc, d_out);
    *r1 = std::min(c1 * rc, d_out);
}

int first_range_rank(int nranks, size_t rotate) {
    return (int)(((size_t)nranks - rotate % (size_t)nranks) % (size_t)nranks);
}

std::vector<int> assign_owners(const std::vector<size_t>& ns, int nranks, int power) {
    std::vector<size_t> idx(ns.size());
    for (size_t i = 0; i < idx.size(); i++) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return ns[a] > ns[b]; });
    std::vector<double> load((size_t)nranks, 0.0);
    std::vector<int> owner(ns.size(), 0);
    for (size_t i : idx) {
        int r = 0;
        for (int q = 1; q < nranks; q++)
            if (load[(size_t)q] < load[(size_t)r]) r = q;
        owner[i] = r;
        double c = 1.0;
        for (int p = 0; p < power; p++) c *= (double)ns[i];
        load[(size_t)r] += c;
    }
    return owner;
}

// ---- collectives ------------------------------------------------------------------------------------------
int rt_group_begin(Runtime* rt) {
    if (rt->nranks == 1) return 0;
    ncclResult_t r = nccl().GroupStart();
    return r == ncclSuccess ? 0 : nccl_error(rt, r, "ncclGroupStart");
}

int rt_group_end(Runtime* rt) {
    if (rt->nranks == 1) return 0;
    return nccl_settle(rt, nccl().GroupEnd(), "ncclGroupEnd");
}

int rt_broadcast(Runtime* rt, void* buf, size_t bytes, int root) { return rt_broadcast_on(rt, rt->st, buf, bytes, root); }

int rt_broadcast_on(Runtime* rt, cudaStream_t stream, void* buf, size_t bytes, int root) {
    if (rt->nranks == 1 || bytes == 0) return 0;
    ncclResult_t r = nccl().Broadcast(buf, buf, bytes, ncclUint8, root, (ncclComm_t)rt->comm, stream);
    return r == ncclSuccess || r == ncclInProgress ? 0 : nccl_error(rt, r, "ncclBroadcast");
}

int rt_send(Runtime* rt, const void* buf, size_t bytes, int peer) {
    if (rt->nranks == 1 || bytes == 0) return 0;
    ncclResult_t r = nccl().Send(buf, bytes, ncclUint8, peer, (ncclComm_t)rt->comm, rt->st);
    return r == ncclSuccess || r == ncclInProgress ? 0 : nccl_error(rt, r, "ncclSend");
}

int rt_recv(Runtime* rt, void* buf, size_t bytes, int peer) {
    if (rt->nranks == 1 || bytes == 0) return 0;
    ncclResult_t r = nccl().Recv(buf, bytes, ncclUint8, peer, (ncclComm_t)rt->comm, rt->st);
    return r == ncclSuccess || r == ncclInProgress ? 0 : nccl_error(rt, r, "ncclRecv");
}

static int allreduce(Runtime* rt, void* buf, size_t count, ncclDataType_t t, ncclRedOp_t op, const char* what) {
    if (rt->nranks == 1 || count == 0) return 0;
    return nccl_settle(rt, nccl().AllReduce(buf, buf, count, t, op, (ncclComm_t)rt->comm, rt->st), what);
}

int rt_allreduce_sum_f64(Runtime* rt, double* b, size_t n) { return allreduce(rt, b, n, ncclFloat64, ncclSum, "ncclAllReduce"); }
int rt_allreduce_sum_u64(Runtime* rt, uint64_t* b, size_t n) { return allreduce(rt, b, n, ncclUint64, ncclSum, "ncclAllReduce"); }
int rt_allreduce_max_u64(Runtime* rt, uint64_t* b, size_t n) { return allreduce(rt, b, n, ncclUint64, ncclMax, "ncclAllReduce"); }

int rt_sync(Runtime* rt) {
    const double t0 = now_s();
    for (;;) {
        cudaError_t e = cudaStreamQuery(rt->st);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) return cuda_error(e, "runtime stream");
        if (rt->nranks > 1 && rt->comm) {
            ncclResult_t s = ncclSuccess;
            nccl().CommGetAsyncError((ncclComm_t)rt->comm, &s);
            if (s != ncclSuccess && s != ncclInProgress) return nccl_error(rt, s, "collective");
        }
        if (now_s() - t0 > rt->timeout_s) {
            if (rt->nranks > 1) nccl_error(rt, ncclInProgress, "wait");
            return set_error(CDCLQ_ERR_CUDA, "timed out after " + std::to_string((int)rt->timeout_s) +
                                                 " s waiting for the runtime's stream (another rank stopped?)");
        }
        usleep(100);
    }
}

int rt_agree(Runtime* rt, int rc) {
    if (rt->nranks == 1) return rc;
    if (rt->broken) return rc ? rc : set_error(CDCLQ_ERR_CUDA, "the runtime's communicator was aborted");
    int32_t h[2] = {rc ? 1 : 0, rc ? rt->rank : rt->nranks};
    int32_t first = 0;
    // max of the failure flags, min of the failing ranks: two int32 all-reduces on the runtime's scratch
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(rt->flag_dev, h, sizeof h, cudaMemcpyHostToDevice, rt->st));
    int r = allreduce(rt, rt->flag_dev, 1, ncclInt32, ncclMax, "error consensus");
    if (!r) r = allreduce(rt, rt->flag_dev + 1, 1, ncclInt32, ncclMin, "error consensus");
    if (!r) {
        cudaError_t e = cudaMemcpyAsync(h, rt->flag_dev, sizeof h, cudaMemcpyDeviceToHost, rt->st);
        if (e != cudaSuccess) r = cuda_error(e, "error consensus");
    }
    if (!r) r = rt_sync(rt);
    if (r) return rc ? rc : r;
    if (!h[0]) return 0;
    first = h[1];
    // the first failing rank's status and message
    char msg[512];
    std::memset(msg, 0, sizeof msg);
    if (rt->rank == first) {
        int32_t code = rc;
        std::memcpy(msg, &code, 4);
        std::strncpy(msg + 4, cdclq_last_error(), sizeof msg - 5);
    }
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(rt->msg_dev, msg, sizeof msg, cudaMemcpyHostToDevice, rt->st));
    r = nccl_settle(rt, nccl().Broadcast(rt->msg_dev, rt->msg_dev, sizeof msg, ncclUint8, first, (ncclComm_t)rt->comm,
                                         rt->st),
                    "error message");
    if (!r) {
        cudaError_t e = cudaMemcpyAsync(msg, rt->msg_dev, sizeof msg, cudaMemcpyDeviceToHost, rt->st);
        if (e != cudaSuccess) r = cuda_error(e, "error message");
    }
    if (!r) r = rt_sync(rt);
    if (rc) return rc;
    if (r) return r;
    int32_t code = 0;
    std::memcpy(&code, msg, 4);
    msg[sizeof msg - 1] = 0;
    return set_error(code ? code : CDCLQ_ERR_CUDA, "rank " + std::to_string(first) + " failed: " + (msg + 4));
}

// ---- the sharded batch ----------------------------------------------------------------------------------
namespace {

// Stream-ordered device buffers of one call, released together.
struct Bufs {
    cudaStream_t st;
    std::vector<void*> p;
    explicit Bufs(cudaStream_t s) : st(s) {}
    ~Bufs() {
        for (void* q : p) cudaFreeAsync(q, st);
    }
    template <class T>
    int alloc(T** out, size_t count) {
        void* q = nullptr;
        cudaError_t e = cudaMallocAsync(&q, std::max<size_t>(count, 1) * sizeof(T), st);
        if (e != cudaSuccess) return cuda_error(e, "cudaMallocAsync");
        p.push_back(q);
        *out = (T*)q;
        return 0;
    }
};

size_t num_groups_of(const cdclq_config& cfg, size_t n) { return cdclq_num_groups(&cfg, n); }

}  // namespace

int runtime_quantize_batch(Runtime* rt, const cdclq_batch_input* in, size_t nin, const cdclq_batch_layer* ly,
                           size_t nly, const cdclq_config& cfg, bool on_device, bool gather) {
    int rc = check_rt(rt);
    if (rc) return rc;
    if (rt->nranks == 1) {
        rc = cdclq_quantize_batch(in, nin, ly, nly, &cfg, on_device ? 1 : 0, rt->st);
        if (!rc) CDCLQ_CUDA_TRY(cudaStreamSynchronize(rt->st));
        return rc;
    }
    const int R = rt->nranks, me = rt->rank;
    cudaStream_t st = rt->st;
    Bufs bufs(st);
    std::vector<size_t> ns(nin);
    for (size_t i = 0; i < nin; i++) ns[i] = in[i].n;
    const std::vector<int> owner = assign_owners(ns, R, 3);

    // ---- arguments (checked on every rank; a failure anywhere stops every rank)
    for (size_t i = 0; i < nin && !rc; i++) {
        if (ns[i] == 0) rc = set_error(CDCLQ_ERR_ARG, "input " + std::to_string(i) + " has n = 0");
        else if ((on_device || owner[i] == me) && !in[i].h) rc = set_error(CDCLQ_ERR_ARG, "null Hessian");
        else rc = cdclq_validate(&cfg, ns[i]);
    }
    for (size_t l = 0; l < nly && !rc; l++) {
        const cdclq_batch_layer& L = ly[l];
        if (L.input >= nin) rc = set_error(CDCLQ_ERR_ARG, "layer input index out of range");
        else if (!L.w || !L.perm || !L.gbits || !L.stats || !L.codes || !L.scales || !L.zeros || L.d_out == 0)
            rc = set_error(CDCLQ_ERR_ARG, "null argument");
    }
    if ((rc = rt_agree(rt, rc))) return rc;

    // ---- Hessians on every device: host inputs uploaded by their owner, then broadcast
    std::vector<float*> hdev(nin, nullptr);
    for (size_t i = 0; i < nin && !rc; i++) {
        if (on_device) {
            hdev[i] = const_cast<float*>(in[i].h);
            continue;
        }
        rc = bufs.alloc(&hdev[i], ns[i] * ns[i]);
        if (!rc && owner[i] == me) {
            cudaError_t e = cudaMemcpyAsync(hdev[i], in[i].h, ns[i] * ns[i] * sizeof(float), cudaMemcpyHostToDevice, st);
            if (e != cudaSuccess) rc = cuda_error(e, "Hessian upload");
        }
    }
    if ((rc = rt_agree(rt, rc))) return rc;
    if (!on_device) {
        if ((rc = rt_group_begin(rt))) return rc;
        for (size_t i = 0; i < nin && !rc; i++) rc = rt_broadcast(rt, hdev[i], ns[i] * ns[i] * sizeof(float), owner[i]);
        int r2 = rt_group_end(rt);
        if (rc || r2) return rc ? rc : r2;
    }

    // ---- this rank's rows; weights of host layers uploaded row range by row range
    struct Part {
        size_t r0, r1, rc, n, ng;
        float* w = nullptr;        // device, this rank's rows
        uint8_t* codes = nullptr;  // device, this rank's rows (into the caller's buffer when on_device)
        float* scales = nullptr;
        float* zeros = nullptr;
        double* colsq = nullptr;   // device, full-W column scores (skeleton)
        float* u = nullptr;        // device factor of the layer (skeleton)
    };
    std::vector<Part> part(nly);
    const bool skel = cfg.skeleton_pct > 0.0;
    for (size_t l = 0; l < nly && !rc; l++) {
        Part& P = part[l];
        const cdclq_batch_layer& L = ly[l];
        P.n = ns[L.input];
        P.ng = num_groups_of(cfg, P.n);
        P.rc = cdclq_row_chunk(&cfg, L.d_out);
        shard_rows(L.d_out, P.rc, me, R, l, &P.r0, &P.r1);
        const size_t rows = P.r1 - P.r0;
        if (on_device) {
            P.w = const_cast<float*>(L.w) + P.r0 * P.n;
            P.codes = L.codes + P.r0 * P.n;
            P.scales = L.scales + P.r0 * P.ng;
            P.zeros = L.zeros + P.r0 * P.ng;
            continue;
        }
        if (rows == 0) continue;
        if ((rc = bufs.alloc(&P.w, rows * P.n))) break;
        cudaError_t e = cudaMemcpyAsync(P.w, L.w + P.r0 * P.n, rows * P.n * sizeof(float), cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) {
            rc = cuda_error(e, "weight upload");
            break;
        }
        if ((rc = bufs.alloc(&P.codes, rows * P.n))) break;
        if ((rc = bufs.alloc(&P.scales, rows * P.ng))) break;
        if ((rc = bufs.alloc(&P.zeros, rows * P.ng))) break;
    }
    if ((rc = rt_agree(rt, rc))) return rc;

    // ---- skeleton: the full weight's column scores, summed rank by rank in row order (the rows of range v
    // continue the sums of ranges 0..v-1, exactly the single-GPU order), then known to every rank
    if (skel) {
        std::vector<double*> hdiag(nin, nullptr);
        for (size_t i = 0; i < nin && !rc; i++) {
            rc = bufs.alloc(&hdiag[i], ns[i]);
            if (!rc) rc = launch_hdiag(hdev[i], (int)ns[i], hdiag[i], st);
        }
        for (size_t l = 0; l < nly && !rc; l++) rc = bufs.alloc(&part[l].colsq, part[l].n);
        if ((rc = rt_agree(rt, rc))) return rc;
        for (int v = 0; v < R && !rc; v++) {
            if (v > 0) {  // pass the running sums from range v-1 to range v
                if ((rc = rt_group_begin(rt))) return rc;
                for (size_t l = 0; l < nly && !rc; l++) {
                    const int from = (first_range_rank(R, l) + v - 1) % R, to = (first_range_rank(R, l) + v) % R;
                    if (me == from) rc = rt_send(rt, part[l].colsq, part[l].n * sizeof(double), to);
                    if (me == to && !rc) rc = rt_recv(rt, part[l].colsq, part[l].n * sizeof(double), from);
                }
                int r2 = rt_group_end(rt);
                if (rc || r2) return rc ? rc : r2;
            }
            for (size_t l = 0; l < nly && !rc; l++) {
                if ((first_range_rank(R, l) + v) % R != me) continue;
                Part& P = part[l];
                rc = launch_colsq_from(P.w, hdiag[ly[l].input], (int)(P.r1 - P.r0), (int)P.n, v > 0 ? P.colsq : nullptr,
                                       P.colsq, st);
            }
        }
        if ((rc = rt_agree(rt, rc))) return rc;
        if ((rc = rt_group_begin(rt))) return rc;
        for (size_t l = 0; l < nly && !rc; l++)
            rc = rt_broadcast(rt, part[l].colsq, part[l].n * sizeof(double), (first_range_rank(R, l) + R - 1) % R);
        int r2 = rt_group_end(rt);
        if (rc || r2) return rc ? rc : r2;
    }

    // ---- permutations and group widths of every layer on every rank (rows or not)
    std::vector<std::vector<uint32_t>> perm(nly);
    std::vector<std::vector<uint8_t>> gbits(nly);
    std::vector<size_t> nskel(nly, 0);
    std::vector<long> first_of_input(nin, -1);  // without a skeleton every layer of an input shares its permutation
    for (size_t l = 0; l < nly && !rc; l++) {
        const long f = first_of_input[ly[l].input];
        if (!skel && f >= 0) {
            perm[l] = perm[f];
            gbits[l] = gbits[f];
            nskel[l] = nskel[f];
            continue;
        }
        first_of_input[ly[l].input] = (long)l;
        std::vector<double> cs;
        if (skel) {
            cs.resize(part[l].n);
            cudaError_t e = cudaMemcpyAsync(cs.data(), part[l].colsq, part[l].n * sizeof(double), cudaMemcpyDeviceToHost, st);
            if (e != cudaSuccess) {
                rc = cuda_error(e, "column scores");
                break;
            }
        }
        rc = layer_perm(hdev[ly[l].input], part[l].n, skel ? cs.data() : nullptr, cfg, perm[l], gbits[l], nskel[l], st);
    }
    if ((rc = rt_agree(rt, rc))) return rc;

    // ---- factors: each owner factorises its share, then every factor is broadcast from its owner
    std::vector<float*> u(nin, nullptr);
    std::vector<int> lowner;
    if (!skel) {
        std::vector<size_t> which;
        std::vector<float*> uo;
        for (size_t i = 0; i < nin && !rc; i++) {
            rc = bufs.alloc(&u[i], ns[i] * ns[i]);
            if (owner[i] == me) {
                which.push_back(i);
                uo.push_back(u[i]);
            }
        }
        cdclq_batch_input* ind = nullptr;
        std::vector<cdclq_batch_input> in_dev(nin);
        for (size_t i = 0; i < nin; i++) in_dev[i] = cdclq_batch_input{hdev[i], ns[i]};
        ind = in_dev.data();
        if (!rc && !which.empty())
            rc = cdclq_prepare_factors(ind, nin, which.data(), which.size(), &cfg, uo.data(), 1, st);
    } else {
        std::vector<size_t> lns(nly);
        for (size_t l = 0; l < nly; l++) lns[l] = part[l].n;
        lowner = assign_owners(lns, R, 3);
        std::vector<size_t> which;
        std::vector<float*> uo;
        std::vector<cdclq_batch_layer> full(nly);
        for (size_t l = 0; l < nly && !rc; l++) {
            rc = bufs.alloc(&part[l].u, part[l].n * part[l].n);
            full[l] = cdclq_batch_layer{};
            full[l].d_out = ly[l].d_out;
            full[l].input = ly[l].input;
            full[l].colsq = part[l].colsq;
            if (lowner[l] == me) {
                which.push_back(l);
                uo.push_back(part[l].u);
            }
        }
        std::vector<cdclq_batch_input> in_dev(nin);
        for (size_t i = 0; i < nin; i++) in_dev[i] = cdclq_batch_input{hdev[i], ns[i]};
        if (!rc && !which.empty())
            rc = cdclq_prepare_layer_factors(in_dev.data(), nin, full.data(), nly, which.data(), which.size(), &cfg,
                                             uo.data(), 1, st);
    }
    if ((rc = rt_agree(rt, rc))) return rc;
    // The factors travel on the communication stream, ordered after this rank's factorisations; every layer is
    // then quantized in one batch once they have landed.  (Quantizing the layers whose factor this rank computed
    // first, in a batch of their own, would hide the broadcast - tens of milliseconds over NVLink - but give
    // the repair two launches, each ending on its own tail of wide row chunks: measured slower at N = 2.)
    cudaEvent_t ev_f = nullptr, ev_b = nullptr;
    CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&ev_f, cudaEventDisableTiming));
    CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&ev_b, cudaEventDisableTiming));
    struct Ev {
        cudaEvent_t a, b;
        ~Ev() {
            cudaEventDestroy(a);
            cudaEventDestroy(b);
        }
    } evs{ev_f, ev_b};
    CDCLQ_CUDA_TRY(cudaEventRecord(ev_f, st));
    CDCLQ_CUDA_TRY(cudaStreamWaitEvent(rt->comm_st, ev_f, 0));
    if ((rc = rt_group_begin(rt))) return rc;
    if (!skel) {
        for (size_t i = 0; i < nin && !rc; i++)
            rc = rt_broadcast_on(rt, rt->comm_st, u[i], ns[i] * ns[i] * sizeof(float), owner[i]);
    } else {
        for (size_t l = 0; l < nly && !rc; l++)
            rc = rt_broadcast_on(rt, rt->comm_st, part[l].u, part[l].n * part[l].n * sizeof(float), lowner[l]);
    }
    {
        int r2 = rt_group_end(rt);
        if (rc || r2) return rc ? rc : r2;
    }
    CDCLQ_CUDA_TRY(cudaEventRecord(ev_b, rt->comm_st));

    // ---- this rank's rows, one batch per row chunk (layers whose automatic row chunk differs)
    std::vector<cdclq_layer_stats> lst(nly);
    std::vector<std::vector<uint32_t>> scratch_perm(nly);
    std::vector<std::vector<uint8_t>> scratch_gb(nly);
    std::map<size_t, std::vector<size_t>> by_rc;  // row chunk -> layers
    for (size_t l = 0; l < nly; l++)
        if (part[l].r1 > part[l].r0) by_rc[part[l].rc].push_back(l);
    std::vector<cdclq_batch_input> in_dev(nin);
    for (size_t i = 0; i < nin; i++) in_dev[i] = cdclq_batch_input{hdev[i], ns[i]};
    {
        cudaError_t e = cudaStreamWaitEvent(st, ev_b, 0);
        if (e != cudaSuccess) return cuda_error(e, "factor broadcast wait");
    }
    for (auto& kv : by_rc) {
        if (rc) break;
        cdclq_config c = cfg;
        c.row_chunk = kv.first;
        std::vector<cdclq_batch_layer> d(kv.second.size());
        for (size_t k = 0; k < kv.second.size(); k++) {
            const size_t l = kv.second[k];
            Part& P = part[l];
            scratch_perm[l].resize(P.n);
            scratch_gb[l].resize(P.ng);
            d[k] = cdclq_batch_layer{};
            d[k].w = P.w;
            d[k].d_out = P.r1 - P.r0;
            d[k].input = ly[l].input;
            d[k].perm = scratch_perm[l].data();
            d[k].gbits = scratch_gb[l].data();
            d[k].codes = P.codes;
            d[k].scales = P.scales;
            d[k].zeros = P.zeros;
            d[k].stats = &lst[l];
            if (skel) {
                d[k].colsq = P.colsq;
                d[k].u = P.u;
            }
        }
        rc = skel ? cdclq_quantize_batch(in_dev.data(), nin, d.data(), d.size(), &c, 1, st)
                  : cdclq_quantize_batch_prepared(in_dev.data(), nin, u.data(), d.data(), d.size(), &c, 1, st);
    }
    if ((rc = rt_agree(rt, rc))) return rc;

    // ---- statistics of every layer: sums over the ranks' rows
    {
        std::vector<double> f(2 * nly);
        std::vector<uint64_t> s(3 * nly), m(nly);
        for (size_t l = 0; l < nly; l++) {
            f[2 * l] = lst[l].loss_gptq;
            f[2 * l + 1] = lst[l].loss_final;
            s[3 * l] = lst[l].subblocks_total;
            s[3 * l + 1] = lst[l].subblocks_refined;
            s[3 * l + 2] = lst[l].code_updates;
            m[l] = lst[l].passes_max;
        }
        double* fd = nullptr;
        uint64_t *sd = nullptr, *md = nullptr;
        if ((rc = bufs.alloc(&fd, f.size()))) return rc;
        if ((rc = bufs.alloc(&sd, s.size()))) return rc;
        if ((rc = bufs.alloc(&md, m.size()))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(fd, f.data(), f.size() * 8, cudaMemcpyHostToDevice, st));
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(sd, s.data(), s.size() * 8, cudaMemcpyHostToDevice, st));
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(md, m.data(), m.size() * 8, cudaMemcpyHostToDevice, st));
        if ((rc = rt_allreduce_sum_f64(rt, fd, f.size()))) return rc;
        if ((rc = rt_allreduce_sum_u64(rt, sd, s.size()))) return rc;
        if ((rc = rt_allreduce_max_u64(rt, md, m.size()))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(f.data(), fd, f.size() * 8, cudaMemcpyDeviceToHost, st));
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(s.data(), sd, s.size() * 8, cudaMemcpyDeviceToHost, st));
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(m.data(), md, m.size() * 8, cudaMemcpyDeviceToHost, st));
        if ((rc = rt_sync(rt))) return rc;
        for (size_t l = 0; l < nly; l++) {
            cdclq_layer_stats o = lst[l];
            o.loss_gptq = f[2 * l];
            o.loss_final = f[2 * l + 1];
            o.subblocks_total = s[3 * l];
            o.subblocks_refined = s[3 * l + 1];
            o.code_updates = s[3 * l + 2];
            o.passes_max = m[l];
            o.skeleton_groups = nskel[l];
            const size_t g = cdclq_effective_group(&cfg, part[l].n);
            double bits = 0.0;
            for (size_t j = 0; j < part[l].n; j++) bits += gbits[l][j / g];
            o.bits_codes = bits / (double)part[l].n;
            o.bits_total = o.bits_codes + 24.0 / (double)g;
            *ly[l].stats = o;
            std::memcpy(ly[l].perm, perm[l].data(), part[l].n * sizeof(uint32_t));
            std::memcpy(ly[l].gbits, gbits[l].data(), part[l].ng);
        }
    }

    // ---- outputs: host layers copy their rows back; with `gather`, rank 0 also receives every other rank's rows
    struct Stage {
        size_t l;
        int from;
        size_t r0, r1;
        uint8_t* codes;
        float* scales;
        float* zeros;
    };
    std::vector<Stage> incoming;
    if (gather) {
        if ((rc = rt_group_begin(rt))) return rc;
        for (size_t l = 0; l < nly && !rc; l++) {
            const Part& P = part[l];
            for (int q = 1; q < R && !rc; q++) {
                size_t r0 = 0, r1 = 0;
                shard_rows(ly[l].d_out, P.rc, q, R, l, &r0, &r1);
                if (r1 == r0) continue;
                const size_t rows = r1 - r0;
                if (me == q) {
                    rc = rt_send(rt, P.codes, rows * P.n, 0);
                    if (!rc) rc = rt_send(rt, P.scales, rows * P.ng * sizeof(float), 0);
                    if (!rc) rc = rt_send(rt, P.zeros, rows * P.ng * sizeof(float), 0);
                } else if (me == 0) {
                    Stage s{l, q, r0, r1, nullptr, nullptr, nullptr};
                    if (on_device) {
                        s.codes = ly[l].codes + r0 * P.n;
                        s.scales = ly[l].scales + r0 * P.ng;
                        s.zeros = ly[l].zeros + r0 * P.ng;
                    } else {
                        if ((rc = bufs.alloc(&s.codes, rows * P.n))) break;
                        if ((rc = bufs.alloc(&s.scales, rows * P.ng))) break;
                        if ((rc = bufs.alloc(&s.zeros, rows * P.ng))) break;
                    }
                    rc = rt_recv(rt, s.codes, rows * P.n, q);
                    if (!rc) rc = rt_recv(rt, s.scales, rows * P.ng * sizeof(float), q);
                    if (!rc) rc = rt_recv(rt, s.zeros, rows * P.ng * sizeof(float), q);
                    incoming.push_back(s);
                }
            }
        }
        int r2 = rt_group_end(rt);
        if (rc || r2) return rc ? rc : r2;
    }
    if (!on_device) {
        for (size_t l = 0; l < nly; l++) {
            const Part& P = part[l];
            const size_t rows = P.r1 - P.r0;
            if (!rows) continue;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[l].codes + P.r0 * P.n, P.codes, rows * P.n, cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[l].scales + P.r0 * P.ng, P.scales, rows * P.ng * 4, cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[l].zeros + P.r0 * P.ng, P.zeros, rows * P.ng * 4, cudaMemcpyDeviceToHost, st));
        }
        for (const Stage& s : incoming) {
            const Part& P = part[s.l];
            const size_t rows = s.r1 - s.r0;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[s.l].codes + s.r0 * P.n, s.codes, rows * P.n, cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[s.l].scales + s.r0 * P.ng, s.scales, rows * P.ng * 4, cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ly[s.l].zeros + s.r0 * P.ng, s.zeros, rows * P.ng * 4, cudaMemcpyDeviceToHost, st));
        }
    }
    return rt_sync(rt);
}

}  // namespace cdclq

// =========================================================================================================
// C ABI
using cdclq::Runtime;

struct cdclq_runtime : Runtime {};

extern "C" {

int cdclq_runtime_unique_id(uint8_t* id_out) {
    using namespace cdclq;
    if (!id_out) return set_error(CDCLQ_ERR_ARG, "null argument");
    static_assert(sizeof(ncclUniqueId) == CDCLQ_UNIQUE_ID_BYTES, "ncclUniqueId size");
    Nccl& N = nccl();
    if (!N.loaded) return set_error(CDCLQ_ERR_CUDA, N.why);
    ncclUniqueId id;
    ncclResult_t r = N.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_error(nullptr, r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof id);
    return CDCLQ_OK;
}

int cdclq_runtime_create(int device, int nranks, int rank, const uint8_t* unique_id, double timeout_s,
                         cdclq_runtime** out) {
    using namespace cdclq;
    if (!out || nranks < 1 || rank < 0 || rank >= nranks || (nranks > 1 && !unique_id))
        return set_error(CDCLQ_ERR_ARG, "bad runtime arguments (need 0 <= rank < nranks and, with nranks > 1, the "
                                        "unique id from cdclq_runtime_unique_id)");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return set_error(CDCLQ_ERR_CUDA, std::string("no CUDA device available: ") + cudaGetErrorString(e));
    if (device < 0 || device >= count) return set_error(CDCLQ_ERR_ARG, "device index out of range");
    CDCLQ_CUDA_TRY(cudaSetDevice(device));
    int rc = ensure_device();
    if (rc) return rc;
    cdclq_runtime* rt = new cdclq_runtime();
    rt->device = device;
    rt->nranks = nranks;
    rt->rank = rank;
    rt->timeout_s = timeout_s > 0.0 ? timeout_s : 600.0;
    e = cudaStreamCreateWithFlags(&rt->st, cudaStreamNonBlocking);
    rt->owned_stream = e == cudaSuccess;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&rt->comm_st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&rt->flag_dev, 2 * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&rt->msg_dev, 512);
    if (e != cudaSuccess) rc = cuda_error(e, "runtime set-up");
    if (!rc && nranks > 1) {
        Nccl& N = nccl();
        if (!N.loaded) {
            rc = set_error(CDCLQ_ERR_CUDA, N.why);
        } else {
            ncclUniqueId id;
            std::memcpy(&id, unique_id, sizeof id);
            ncclConfig_t conf = NCCL_CONFIG_INITIALIZER;
            conf.blocking = 0;  // bounded waits: creation is polled against the timeout
            ncclComm_t comm = nullptr;
            ncclResult_t r = N.CommInitRankConfig(&comm, nranks, id, rank, &conf);
            if (r != ncclSuccess && r != ncclInProgress) {
                rc = nccl_error(nullptr, r, "ncclCommInitRankConfig");
            } else {
                rt->comm = comm;
                rc = nccl_settle(rt, r, "ncclCommInitRankConfig");
            }
        }
    }
    if (rc) {
        const std::string keep = cdclq_last_error();
        cdclq_runtime_destroy(rt);
        return set_error(rc, keep);
    }
    *out = rt;
    return CDCLQ_OK;
}

void cdclq_runtime_destroy(cdclq_runtime* rt) {
    using namespace cdclq;
    if (!rt) return;
    cudaSetDevice(rt->device);
    if (rt->comm) {
        // finish (bounded) whatever is queued, flush the communicator (bounded), then release it; abort otherwise
        Nccl& N = nccl();
        int rc = rt_sync(rt);
        if (!rc && rt->comm && N.CommFinalize) rc = nccl_settle(rt, N.CommFinalize((ncclComm_t)rt->comm), "ncclCommFinalize");
        if (rt->comm) {
            if (!rc) N.CommDestroy((ncclComm_t)rt->comm);
            else N.CommAbort((ncclComm_t)rt->comm);
            rt->comm = nullptr;
        }
    }
    if (rt->st) cudaStreamSynchronize(rt->st);
    if (rt->comm_st) cudaStreamSynchronize(rt->comm_st);
    cudaFree(rt->flag_dev);
    cudaFree(rt->msg_dev);
    if (rt->owned_stream && rt->st) cudaStreamDestroy(rt->st);
    if (rt->comm_st) cudaStreamDestroy(rt->comm_st);
    delete rt;
}

void* cdclq_runtime_stream(const cdclq_runtime* rt) { return rt ? (void*)rt->st : nullptr; }

int cdclq_runtime_quantize_batch(cdclq_runtime* rt, const cdclq_batch_input* inputs, size_t n_inputs,
                                 const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config* cfg,
                                 int on_device, int gather) {
    using namespace cdclq;
    if (!cfg || (!inputs && n_inputs) || (!layers && n_layers)) return set_error(CDCLQ_ERR_ARG, "null argument");
    return runtime_quantize_batch(rt, inputs, n_inputs, layers, n_layers, *cfg, on_device != 0, gather != 0);
}

void cdclq_shard_rows(size_t d_out, size_t row_chunk, int rank, int nranks, size_t rotate, size_t* r0, size_t* r1) {
    cdclq::shard_rows(d_out, row_chunk, rank, nranks < 1 ? 1 : nranks, rotate, r0, r1);
}

void cdclq_assign_owners(const size_t* ns, size_t count, int nranks, int power, int* owner_out) {
    std::vector<size_t> v(ns, ns + count);
    std::vector<int> o = cdclq::assign_owners(v, nranks < 1 ? 1 : nranks, power);
    std::copy(o.begin(), o.end(), owner_out);
}

}  // extern "C"
