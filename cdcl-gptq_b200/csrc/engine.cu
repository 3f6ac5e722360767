// engine.cu - host orchestration of the per-layer path and the C ABI (include/cdclq.h).
//
// The reference's engine::quantize_layer (src/engine.rs:690-799) runs, per layer: validate -> dead columns ->
// permutation -> prepared factors (cached per Hessian owner) -> permuted weights -> [asymmetric target] ->
// row chunks through phase 1 + phase 2 -> summed statistics.  Here the same steps run for a whole BATCH of
// layers at once: permutations on the host (they are sorts of n keys), every distinct (input, permutation)
// factorised once in a batched launch sequence per width, then ONE phase-1 launch over all rows of all
// layers, ONE statistics launch over all row chunks, and one launch per repair pass over all row slices.
// Small layers (k/v projections) therefore never leave SMs idle, and q/k/v and gate/up share one
// factorisation exactly as the reference's PrepCache arranges by sorting jobs by Hessian owner
// (src/pipeline.rs:109-112, src/engine.rs:718-722).
#include <sched.h>

#include <algorithm>
#include <chrono>
#include <charconv>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "cdclq.h"
#include "common.cuh"
#include "kernels.h"

namespace cdclq {

std::atomic<uint64_t> g_launches{0};
static thread_local std::string g_last_error;

int set_error(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(CDCLQ_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e) + " (" + what + ")");
}

// Rust's `{:e}` (LowerExp) for f64: shortest round-trip digits, exponent without padding or '+'.
std::string rust_exp(double v) {
    if (std::isnan(v)) return "NaN";
    if (std::isinf(v)) return v > 0 ? "inf" : "-inf";
    char buf[64];
    auto res = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::scientific);
    std::string s(buf, res.ptr);
    size_t e = s.find('e');
    if (e == std::string::npos) return s;
    std::string mant = s.substr(0, e), ex = s.substr(e + 1);
    bool neg = false;
    size_t i = 0;
    if (i < ex.size() && (ex[i] == '+' || ex[i] == '-')) {
        neg = ex[i] == '-';
        i++;
    }
    while (i + 1 < ex.size() && ex[i] == '0') i++;
    return mant + "e" + (neg ? "-" : "") + ex.substr(i);
}

static size_t host_threads() {
    cpu_set_t set;
    CPU_ZERO(&set);
    if (sched_getaffinity(0, sizeof set, &set) == 0) {
        int c = CPU_COUNT(&set);
        if (c > 0) return (size_t)c;
    }
    unsigned h = std::thread::hardware_concurrency();
    return h ? h : 1;
}

static size_t effective_group(const cdclq_config& c, size_t n) { return (c.group == 0 || c.group >= n) ? n : c.group; }

// src/engine.rs:240-258
static int validate(const cdclq_config& c, size_t n) {
    if (c.bits < 2 || c.bits > 8 || c.skeleton_bits < 2 || c.skeleton_bits > 8)
        return set_error(CDCLQ_ERR_CONFIG, "bits and skeleton_bits must be in 2..=8");
    if (c.block == 0 || c.sub_block == 0) return set_error(CDCLQ_ERR_CONFIG, "block and sub_block must be > 0");
    size_t g = effective_group(c, n);
    if (g < n && c.block % g != 0 && g % c.block != 0)
        return set_error(CDCLQ_ERR_CONFIG, "group size " + std::to_string(g) + " must divide the block size " +
                                               std::to_string(c.block) + " (or be a multiple of it)");
    if (c.skeleton_pct > 0.0 && g >= n) return set_error(CDCLQ_ERR_CONFIG, "the skeleton needs a finite group size");
    if (!(c.refine_frac >= 0.0 && c.refine_frac <= 1.0))
        return set_error(CDCLQ_ERR_CONFIG, "refine_frac must be in [0, 1]");
    return CDCLQ_OK;
}

// Limits of this build's shared-memory tiling (the reference has none).
static int check_tiling(const cdclq_config& c, size_t n) {
    int dev = 0, maxsm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    size_t g = effective_group(c, n);
    if (phase1_smem_bytes((int)std::min<size_t>(c.block, n)) > (size_t)maxsm)
        return set_error(CDCLQ_ERR_CONFIG, "block " + std::to_string(c.block) +
                                               " exceeds the GPTQ kernel's shared-memory tile (max 320 columns)");
    if (repair_smem_bytes((int)g, (int)std::min<size_t>(c.sub_block, n), 64) > (size_t)maxsm)
        return set_error(CDCLQ_ERR_CONFIG, "sub_block " + std::to_string(c.sub_block) +
                                               " exceeds the repair kernel's shared-memory tile (max 256 columns)");
    if (n > 65535) return set_error(CDCLQ_ERR_CONFIG, "d_in above 65535 is not supported");
    return CDCLQ_OK;
}

static size_t row_chunk(const cdclq_config& c, size_t d_out) {
    size_t rc;
    if (c.row_chunk > 0) {
        rc = c.row_chunk;
    } else {
        size_t nt = c.threads > 0 ? (size_t)c.threads : host_threads();
        rc = std::min<size_t>(std::max<size_t>((d_out + nt - 1) / nt, 32), 256);
    }
    return std::max<size_t>(std::min(rc, d_out), 1);
}

// src/engine.rs:271-304 on the host (sorting n keys; the O(d_out n) column sums ran on the GPU)
static void compute_perm(const std::vector<double>& hdiag, const std::vector<double>* colsq, size_t n, size_t g,
                         const cdclq_config& c, std::vector<uint32_t>& perm, size_t& nskel) {
    nskel = 0;
    perm.clear();
    perm.reserve(n);
    std::vector<char> in_skel(n, 0);
    if (c.skeleton_pct > 0.0 && g < n) {
        size_t full_groups = n / g;
        double r = std::round(c.skeleton_pct / 100.0 * (double)n / (double)g);
        size_t want = r > 0.0 ? (size_t)r : 0;
        nskel = std::min(want, full_groups > 0 ? full_groups - 1 : 0);
        if (nskel > 0) {
            std::vector<size_t> idx(n);
            for (size_t j = 0; j < n; j++) idx[j] = j;
            std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
                double ca = hdiag[a] * (*colsq)[a], cb = hdiag[b] * (*colsq)[b];
                if (cb < ca) return true;
                if (ca < cb) return false;
                return a < b;
            });
            for (size_t t = 0; t < nskel * g; t++) {
                in_skel[idx[t]] = 1;
                perm.push_back((uint32_t)idx[t]);
            }
        }
    }
    std::vector<size_t> rest;
    rest.reserve(n);
    for (size_t j = 0; j < n; j++)
        if (!in_skel[j]) rest.push_back(j);
    if (c.act_order)
        std::sort(rest.begin(), rest.end(), [&](size_t a, size_t b) {
            if (hdiag[b] < hdiag[a]) return true;
            if (hdiag[a] < hdiag[b]) return false;
            return a < b;
        });
    for (size_t j : rest) perm.push_back((uint32_t)j);
}

// Stream-ordered device allocations released together.
class Arena {
   public:
    explicit Arena(cudaStream_t s) : st_(s) {}
    ~Arena() { release(); }
    template <class T>
    int alloc(T** p, size_t count) {
        void* q = nullptr;
        cudaError_t e = cudaMallocAsync(&q, std::max<size_t>(count, 1) * sizeof(T), st_);
        if (e != cudaSuccess) return cuda_error(e, "cudaMallocAsync");
        ptrs_.push_back(q);
        *p = static_cast<T*>(q);
        return 0;
    }
    void free_one(void* p) {
        auto it = std::find(ptrs_.begin(), ptrs_.end(), p);
        if (it != ptrs_.end()) {
            cudaFreeAsync(p, st_);
            ptrs_.erase(it);
        }
    }
    void release() {
        for (void* p : ptrs_) cudaFreeAsync(p, st_);
        ptrs_.clear();
    }

   private:
    cudaStream_t st_;
    std::vector<void*> ptrs_;
};

// Prepared factors of one (input, permutation): device U, damped permuted Hessian, permutation.
struct PrepEntry {
    size_t n = 0;
    std::vector<uint32_t> perm;
    double damp_val = 0.0;
    float* u = nullptr;
    float* h32 = nullptr;
    uint32_t* perm_dev = nullptr;
    bool owned = false;  // cudaMalloc'd (prep cache) rather than arena
    bool ext_u = false;  // u supplied by the caller (prepared on another rank): only h32 is built here
    void release() {
        if (owned) {
            cudaFree(u);
            cudaFree(h32);
            cudaFree(perm_dev);
        }
        u = h32 = nullptr;
        perm_dev = nullptr;
        owned = false;
        perm.clear();
        n = 0;
    }
};

}  // namespace cdclq

struct cdclq_prep_cache {
    bool valid = false;
    std::string key;
    cdclq::PrepEntry e;
    ~cdclq_prep_cache() { e.release(); }
};

namespace cdclq {

struct InputReq {
    const float* h = nullptr;  // host or device
    size_t n = 0;
};

struct LayerReq {
    const float* w = nullptr;  // host or device
    size_t d_out = 0;
    size_t input = 0;
    const float* m = nullptr;  // optional (host or device), single-layer path only
    uint32_t* perm = nullptr;
    uint8_t* gbits = nullptr;
    uint8_t* codes = nullptr;
    float* scales = nullptr;
    float* zeros = nullptr;
    cdclq_layer_stats* stats = nullptr;
    uint32_t* chunk_passes = nullptr;  // host, optional
    const double* colsq = nullptr;     // optional skeleton column scores over the full matrix (host or device)
    const float* u = nullptr;          // optional caller-supplied factor of this layer's (input, perm) (device)
};

static thread_local cdclq_run_profile g_profile;

// Events at the phase boundaries of one run (recorded on the run's stream).
struct PhaseEvents {
    cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    bool ok = true;
    PhaseEvents() {
        for (auto& e : ev)
            if (cudaEventCreate(&e) != cudaSuccess) ok = false;
    }
    ~PhaseEvents() {
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
    }
    void record(int i, cudaStream_t st) {
        if (ok) cudaEventRecord(ev[i], st);
    }
    double ms(int a, int b) {
        float t = 0.0f;
        if (!ok || cudaEventElapsedTime(&t, ev[a], ev[b]) != cudaSuccess) return 0.0;
        return (double)t;
    }
};

static cudaStream_t lib_stream() {
    static thread_local cudaStream_t s = nullptr;
    if (!s) cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    return s;
}

static cudaStream_t copy_stream() {
    static thread_local cudaStream_t s = nullptr;
    if (!s) cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    return s;
}

static double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

struct LayerPlan {
    size_t d_out = 0, n = 0, g = 0, ng = 0, nskel = 0, rc = 0, nchunks = 0;
    std::vector<uint32_t> perm;
    std::vector<uint8_t> gbits;
    int prep = -1;
    const float* w_dev = nullptr;
    float* wt = nullptr;
    float* w = nullptr;
    float* wq = nullptr;
    float* e = nullptr;
    uint8_t* codes = nullptr;
    float* scales = nullptr;
    float* zeros = nullptr;
    uint8_t* gbits_dev = nullptr;
    double* colloss = nullptr;
    double* sbsum = nullptr;
    int32_t* sel = nullptr;
    size_t chunk0 = 0;
};

// Factorisation of a set of distinct inputs of one width (one batch of launches on its own stream).
struct FactorGroup {
    size_t n = 0;
    std::vector<size_t> inputs;     // input index of each item
    cudaEvent_t ready = nullptr;    // its Hessians are on the device (null: everything issued so far on `st`)
    bool h32_only = false;          // U supplied by the caller: only the damped permuted Hessian is built
    std::vector<const float*> hs;   // device Hessians (original order)
    std::vector<PrepEntry*> es;     // receive damp_val; u/h32/perm_dev already allocated
    size_t b0 = 0, nb = 0;          // current sub-batch
    cudaStream_t st = nullptr;
    std::unique_ptr<Arena> ar;
    FactorStatus* status_dev = nullptr;
    double* damp_dev = nullptr;
    std::vector<FactorStatus> status;
    std::vector<double> damp;
    bool launched = false;          // a sub-batch is in flight: factor_finish reads its status back
};

static size_t factor_item_bytes(size_t n, bool h32_only = false) {
    if (h32_only) return n * sizeof(double) + 256;
    return 2 * n * n * sizeof(double) + 96 * n * sizeof(double) + n * sizeof(double) + 256;
}

// Streams of the factorisation groups.  Stream 0 carries the widest group (groups are ordered widest first),
// whose chain of block steps is the longest, so it gets the device's highest stream priority: its latency-bound
// diagonal and panel kernels then take SMs ahead of the narrower groups' launches.
static cudaStream_t pool_stream(size_t i) {
    static thread_local std::vector<cudaStream_t> pool;
    while (pool.size() <= i) {
        cudaStream_t s = nullptr;
        int least = 0, greatest = 0;
        cudaDeviceGetStreamPriorityRange(&least, &greatest);
        cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, pool.empty() ? greatest : least);
        pool.push_back(s);
    }
    return pool[i];
}

// Enqueue items [g.b0, g.b0 + g.nb) of the group: prepare, Cholesky, triangular inverse, U scatter, and the
// status / damping read-back (src/engine.rs:320-342, src/linalg.rs:362-375).
static int factor_launch(FactorGroup& g, const cdclq_config& cfg) {
    const size_t n = g.n, nb = g.nb;
    g.ar.reset(new Arena(g.st));
    Arena& ar = *g.ar;
    std::vector<PrepItem> items(nb);
    int rc = ar.alloc(&g.damp_dev, nb);
    if (!rc) rc = ar.alloc(&g.status_dev, nb);
    if (rc) return rc;
    for (size_t i = 0; i < nb; i++) {
        PrepEntry* pe = g.es[g.b0 + i];
        PrepItem& it = items[i];
        it = PrepItem{};
        it.h = g.hs[g.b0 + i];
        it.perm = pe->perm_dev;
        if (!g.h32_only) {
            if ((rc = ar.alloc(&it.hr, n * n))) return rc;
            if ((rc = ar.alloc(&it.y, n * n))) return rc;
            if ((rc = ar.alloc(&it.tbuf, 96 * n))) return rc;
            it.u = pe->u;
            CDCLQ_CUDA_TRY(cudaMemsetAsync(it.y, 0, n * n * sizeof(double), g.st));
        }
        if ((rc = ar.alloc(&it.dg, n))) return rc;
        it.h32 = pe->h32;
        it.damp_val = g.damp_dev + i;
        it.status = g.status_dev + i;
    }
    PrepItem* items_dev = nullptr;
    if ((rc = ar.alloc(&items_dev, nb))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(items_dev, items.data(), sizeof(PrepItem) * nb, cudaMemcpyHostToDevice, g.st));
    if ((rc = launch_prepare(items_dev, (int)nb, (int)n, cfg.damp, g.st))) return rc;
    if (!g.h32_only) {
        if ((rc = launch_factor(items_dev, (int)nb, (int)n, g.st))) return rc;
        if ((rc = launch_u_scatter(items_dev, (int)nb, (int)n, g.st))) return rc;
    }
    g.status.assign(nb, FactorStatus{0, -1, 0.0});
    g.damp.assign(nb, 0.0);
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(g.status.data(), g.status_dev, sizeof(FactorStatus) * nb, cudaMemcpyDeviceToHost, g.st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(g.damp.data(), g.damp_dev, sizeof(double) * nb, cudaMemcpyDeviceToHost, g.st));
    g.launched = true;
    return 0;
}

// Waits for the group's sub-batch, releases its work memory and reads its status back (nothing to read when its
// launch failed part-way, or never happened because an earlier group's failed).
static int factor_finish(FactorGroup& g) {
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(g.st));
    g.ar.reset();
    if (!g.launched) return 0;
    g.launched = false;
    for (size_t i = 0; i < g.nb; i++) {
        if (g.status[i].err) {
            return set_error(CDCLQ_ERR_NOT_PD, "matrix is not positive definite (pivot " +
                                                   std::to_string(g.status[i].pivot) + " = " +
                                                   rust_exp(g.status[i].value) +
                                                   "); increase --damp or check the Hessian");
        }
        g.es[g.b0 + i]->damp_val = g.damp[i];
    }
    return 0;
}

// Test and tuning overrides, read at every call from the environment (unset = the automatic choice):
//   CDCLQ_FACTOR_BUDGET_BYTES  caps the device memory the factorisations may use at once, so a batch of
//                              inputs is factorised in memory-bounded sub-batches as on a full device;
//   CDCLQ_REPAIR_LAYOUT        the repair launch layout: "passes" (one launch per pass over 64-row slices),
//                              "single" (persistent, one CTA per chunk), "pairs" (persistent, each chunk over a
//                              2-CTA cluster of 64-row tiles), "split" (the widest layers' chunks as SM-owning
//                              clusters beside a persistent launch of the others), "quads" (the same with the
//                              widest layers' chunks over 4-CTA clusters that also split every GEMM's columns).
// Every layout gives the same codes, scales, zero points and pass counts.
static size_t env_size(const char* name) {
    const char* s = getenv(name);
    if (!s || !*s) return 0;
    return (size_t)strtoull(s, nullptr, 10);
}

enum RepairLayout {
    LAYOUT_AUTO = -1, LAYOUT_PASSES = 0, LAYOUT_SINGLE = 1, LAYOUT_PAIRS = 2, LAYOUT_SPLIT = 3, LAYOUT_QUADS = 4
};

static int repair_layout_override() {
    const char* s = getenv("CDCLQ_REPAIR_LAYOUT");
    if (!s || !*s) return LAYOUT_AUTO;
    if (!strcmp(s, "passes")) return LAYOUT_PASSES;
    if (!strcmp(s, "single")) return LAYOUT_SINGLE;
    if (!strcmp(s, "pairs")) return LAYOUT_PAIRS;
    if (!strcmp(s, "split")) return LAYOUT_SPLIT;
    if (!strcmp(s, "quads")) return LAYOUT_QUADS;
    return LAYOUT_AUTO;
}

// Factorise every group.  Groups of different widths are independent: when their work matrices fit in
// free memory together they run concurrently on separate streams (the latency-bound panel steps of one
// width overlap the other's); otherwise each group runs alone in memory-bounded sub-batches.
static int factorize_groups(std::vector<FactorGroup>& groups, const cdclq_config& cfg, cudaStream_t st,
                            uint64_t* batches = nullptr) {
    if (groups.empty()) return 0;
    size_t freeb = 0, totalb = 0;
    cudaMemGetInfo(&freeb, &totalb);
    {
        // memory the stream-ordered pool keeps cached (released by this library's earlier calls) is free for
        // the pool's next allocations, although the driver counts it as used
        int dev = 0;
        cudaMemPool_t pool;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t reserved = 0, used = 0;
            if (cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &reserved) == cudaSuccess &&
                cudaMemPoolGetAttribute(pool, cudaMemPoolAttrUsedMemCurrent, &used) == cudaSuccess && reserved > used)
                freeb += (size_t)(reserved - used);
        }
    }
    size_t budget = freeb > ((size_t)4 << 30) ? freeb - ((size_t)4 << 30) : freeb / 2;
    if (size_t cap = env_size("CDCLQ_FACTOR_BUDGET_BYTES")) budget = std::min(budget, cap);
    size_t need = 0;
    for (auto& g : groups) need += factor_item_bytes(g.n, g.h32_only) * g.hs.size();
    cudaEvent_t ready = nullptr;
    CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    cudaEventRecord(ready, st);  // inputs uploaded / permutations copied on `st`
    int rc = 0;
    for (size_t k = 0; k < groups.size(); k++) {
        groups[k].st = pool_stream(k);
        cudaStreamWaitEvent(groups[k].st, groups[k].ready ? groups[k].ready : ready, 0);
        if (groups[k].ready) {
            cudaEventDestroy(groups[k].ready);
            groups[k].ready = nullptr;
        }
    }
    cudaEventDestroy(ready);
    if (need <= budget) {
        if (batches) *batches += groups.size();
        for (auto& g : groups) {
            g.b0 = 0;
            g.nb = g.hs.size();
            if ((rc = factor_launch(g, cfg))) break;
        }
        for (auto& g : groups) {
            int r2 = factor_finish(g);
            if (!rc) rc = r2;
        }
        return rc;
    }
    // Not everything fits at once: each width group gets a share of the budget in proportion to its need and
    // works through its inputs in sub-batches of that size on its own stream; one sub-batch of every unfinished
    // group is in flight at a time, so the groups still overlap.
    std::vector<size_t> max_items(groups.size());
    for (size_t k = 0; k < groups.size(); k++) {
        const size_t item = factor_item_bytes(groups[k].n, groups[k].h32_only);
        const double share = (double)budget * (double)(item * groups[k].hs.size()) / (double)need;
        max_items[k] = std::max<size_t>(1, (size_t)(share / (double)item));
        groups[k].b0 = 0;
    }
    for (bool more = true; more && !rc;) {
        more = false;
        std::vector<size_t> live;
        for (size_t k = 0; k < groups.size() && !rc; k++) {
            FactorGroup& g = groups[k];
            if (g.b0 >= g.hs.size()) continue;
            g.nb = std::min(max_items[k], g.hs.size() - g.b0);
            if (batches) *batches += 1;
            if ((rc = factor_launch(g, cfg))) {  // nothing to read back: wait for what was issued, release it
                cudaStreamSynchronize(g.st);
                g.ar.reset();
                break;
            }
            live.push_back(k);
        }
        for (size_t k : live) {
            FactorGroup& g = groups[k];
            const int r2 = factor_finish(g);
            if (!rc) rc = r2;
            g.b0 += g.nb;
            if (g.b0 < g.hs.size()) more = true;
        }
    }
    return rc;
}

// The whole path for a batch of layers.  `cache` (single-layer calls only) is the one-entry memo.
static int run(const std::vector<InputReq>& inputs, const std::vector<LayerReq>& layers, const cdclq_config& cfg,
               bool on_device, cudaStream_t st, cdclq_prep_cache* cache, const std::string& hkey,
               const float* const* u_ext = nullptr) {
    const double t_start = now_s();
    const uint64_t launches0 = g_launches.load();
    PhaseEvents pev;
    pev.record(0, st);
    for (const auto& L : layers) {
        if (L.input >= inputs.size()) return set_error(CDCLQ_ERR_ARG, "layer input index out of range");
        size_t n = inputs[L.input].n;
        if (n == 0 || L.d_out == 0) return set_error(CDCLQ_ERR_ARG, "empty layer");
        if (!L.w || !inputs[L.input].h || !L.perm || !L.gbits || !L.codes || !L.scales || !L.zeros || !L.stats)
            return set_error(CDCLQ_ERR_ARG, "null argument");
        int rc = validate(cfg, n);
        if (rc) return rc;
        if ((rc = check_tiling(cfg, n))) return rc;
    }
    Arena ar(st);
    int rc = 0;
    const size_t nin = inputs.size();

    // ---- Hessian diagonals (raw, unpermuted) for dead columns and act-order
    std::vector<std::vector<double>> hdiag(nin);
    std::vector<double*> hdiag_dev(nin, nullptr);
    std::vector<const float*> h_dev(nin, nullptr);
    std::vector<char> input_used(nin, 0);
    for (const auto& L : layers) input_used[L.input] = 1;
    for (size_t i = 0; i < nin; i++) {
        if (!input_used[i]) continue;
        size_t n = inputs[i].n;
        hdiag[i].resize(n);
        if ((rc = ar.alloc(&hdiag_dev[i], n))) return rc;
        if (on_device) {
            if ((rc = launch_hdiag(inputs[i].h, (int)n, hdiag_dev[i], st))) return rc;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(hdiag[i].data(), hdiag_dev[i], n * sizeof(double), cudaMemcpyDeviceToHost, st));
        } else {
            for (size_t j = 0; j < n; j++) hdiag[i][j] = (double)inputs[i].h[j * n + j];
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(hdiag_dev[i], hdiag[i].data(), n * sizeof(double), cudaMemcpyHostToDevice, st));
        }
    }

    // ---- weights on the device, permutations
    std::vector<LayerPlan> plans(layers.size());
    std::vector<size_t> w_uploads;  // host weights copied behind the Hessians
    std::vector<std::vector<uint32_t>> input_perm(nin);  // cache of the W-independent permutation
    std::vector<char> input_perm_done(nin, 0);
    {
        // The W-independent permutations of all inputs (act-order sorts of n keys each) on host threads.
        std::vector<size_t> todo;
        for (const auto& L : layers) {
            const size_t n = inputs[L.input].n, g = effective_group(cfg, n);
            const bool skel = cfg.skeleton_pct > 0.0 && g < n;
            if (!skel && !input_perm_done[L.input]) {
                input_perm_done[L.input] = 1;
                todo.push_back(L.input);
            }
        }
        if (!todo.empty()) {
            CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));  // the diagonals are on the host
            const size_t nt = std::max<size_t>(1, std::min(todo.size(), host_threads()));
            auto work = [&](size_t t0) {
                for (size_t k = t0; k < todo.size(); k += nt) {
                    const size_t in = todo[k], n = inputs[in].n;
                    size_t ns = 0;
                    compute_perm(hdiag[in], nullptr, n, effective_group(cfg, n), cfg, input_perm[in], ns);
                }
            };
            std::vector<std::thread> pool;
            for (size_t t = 1; t < nt; t++) pool.emplace_back(work, t);
            work(0);
            for (auto& th : pool) th.join();
        }
    }
    for (size_t li = 0; li < layers.size(); li++) {
        const LayerReq& L = layers[li];
        LayerPlan& P = plans[li];
        P.d_out = L.d_out;
        P.n = inputs[L.input].n;
        P.g = effective_group(cfg, P.n);
        P.ng = (P.n + P.g - 1) / P.g;
        const bool skel = cfg.skeleton_pct > 0.0 && P.g < P.n;
        if (on_device) {
            P.w_dev = L.w;
        } else {
            float* wd = nullptr;
            if ((rc = ar.alloc(&wd, P.d_out * P.n))) return rc;
            P.w_dev = wd;
            if (skel)  // the skeleton ranks columns by W: upload now
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(wd, L.w, P.d_out * P.n * sizeof(float), cudaMemcpyHostToDevice, st));
            else  // uploaded on the copy stream while the factorisations run
                w_uploads.push_back(li);
        }
        if (skel) {
            std::vector<double> colsq(P.n);
            if (L.colsq && !on_device) {  // caller-supplied scores of the full matrix (a row shard's caller)
                std::copy(L.colsq, L.colsq + P.n, colsq.begin());
            } else if (L.colsq) {
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(colsq.data(), L.colsq, P.n * sizeof(double), cudaMemcpyDeviceToHost, st));
                CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
            } else {
                double* cs_dev = nullptr;
                if ((rc = ar.alloc(&cs_dev, P.n))) return rc;
                if ((rc = launch_colsq(P.w_dev, hdiag_dev[L.input], (int)P.d_out, (int)P.n, cs_dev, st))) return rc;
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(colsq.data(), cs_dev, P.n * sizeof(double), cudaMemcpyDeviceToHost, st));
                CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
                ar.free_one(cs_dev);
            }
            compute_perm(hdiag[L.input], &colsq, P.n, P.g, cfg, P.perm, P.nskel);
        } else {
            P.perm = input_perm[L.input];
            P.nskel = 0;
        }
        P.gbits.resize(P.ng);
        for (size_t gi = 0; gi < P.ng; gi++) P.gbits[gi] = (uint8_t)(gi < P.nskel ? cfg.skeleton_bits : cfg.bits);
    }

    // ---- distinct (input, permutation) factorisations
    std::vector<PrepEntry> preps;
    std::vector<size_t> prep_input;
    preps.reserve(layers.size());
    PrepEntry* cached = nullptr;
    for (size_t li = 0; li < layers.size(); li++) {
        LayerPlan& P = plans[li];
        if (cache && cache->valid && cache->key == hkey && cache->e.n == P.n && cache->e.perm == P.perm) {
            cached = &cache->e;
            P.prep = -2;  // cache hit (src/engine.rs:718)
            continue;
        }
        int found = -1;
        for (size_t k = 0; k < preps.size(); k++)
            if (prep_input[k] == layers[li].input && preps[k].perm == P.perm) {
                found = (int)k;
                break;
            }
        if (found < 0) {
            PrepEntry pe;
            pe.n = P.n;
            pe.perm = P.perm;
            // a caller-supplied factor: the layer's own (computed for its permutation), or the input's, which
            // stands for the input's W-independent permutation only
            pe.ext_u = layers[li].u != nullptr ||
                       (u_ext && u_ext[layers[li].input] && P.nskel == 0 && !(cfg.skeleton_pct > 0.0 && P.g < P.n));
            if (pe.ext_u) pe.u = const_cast<float*>(layers[li].u ? layers[li].u : u_ext[layers[li].input]);
            preps.push_back(pe);
            prep_input.push_back(layers[li].input);
            found = (int)preps.size() - 1;
        }
        P.prep = found;
    }
    if (cache && !preps.empty()) {  // the previous factorisation is dropped before the next is built
        cache->valid = false;
        cache->e.release();
    }
    // allocate factors and upload Hessians that are needed
    std::map<size_t, std::vector<size_t>> by_n, by_n_h32;
    for (size_t k = 0; k < preps.size(); k++) {
        PrepEntry& pe = preps[k];
        size_t n = pe.n;
        if (pe.ext_u) {  // pe.u is the caller's
            if ((rc = ar.alloc(&pe.h32, n * n))) return rc;
            if ((rc = ar.alloc(&pe.perm_dev, n))) return rc;
        } else if (cache) {
            CDCLQ_CUDA_TRY(cudaMalloc(&pe.u, n * n * sizeof(float)));
            CDCLQ_CUDA_TRY(cudaMalloc(&pe.h32, n * n * sizeof(float)));
            CDCLQ_CUDA_TRY(cudaMalloc(&pe.perm_dev, n * sizeof(uint32_t)));
            pe.owned = true;
        } else {
            if ((rc = ar.alloc(&pe.u, n * n))) return rc;
            if ((rc = ar.alloc(&pe.h32, n * n))) return rc;
            if ((rc = ar.alloc(&pe.perm_dev, n))) return rc;
        }
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(pe.perm_dev, pe.perm.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
        size_t in = prep_input[k];
        if (!h_dev[in]) {
            if (on_device) {
                h_dev[in] = inputs[in].h;
            } else {
                float* hd = nullptr;  // uploaded below, group by group
                if ((rc = ar.alloc(&hd, n * n))) return rc;
                h_dev[in] = hd;
            }
        }
        (pe.ext_u ? by_n_h32 : by_n)[n].push_back(k);
    }
    std::vector<FactorGroup> groups;
    for (int pass = 0; pass < 2; pass++) {
        auto& m = pass == 0 ? by_n : by_n_h32;
        for (auto it = m.rbegin(); it != m.rend(); ++it) {  // widest first: the longest factorisations
            auto& kv = *it;
            FactorGroup g;
            g.n = kv.first;
            g.h32_only = pass == 1;
            for (size_t k : kv.second) {
                g.hs.push_back(h_dev[prep_input[k]]);
                g.es.push_back(&preps[k]);
                g.inputs.push_back(prep_input[k]);
            }
            groups.push_back(std::move(g));
        }
    }
    // Host Hessians: uploaded group by group (widest first) so that each group's factorisation starts as soon
    // as its own inputs have arrived.
    if (!on_device) {
        std::vector<char> sent(nin, 0);
        for (auto& g : groups) {
            for (size_t i = 0; i < g.hs.size(); i++) {
                const size_t in = g.inputs[i];
                if (sent[in]) continue;
                sent[in] = 1;
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(const_cast<float*>(h_dev[in]), inputs[in].h, g.n * g.n * sizeof(float),
                                               cudaMemcpyHostToDevice, st));
            }
            CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&g.ready, cudaEventDisableTiming));
            cudaEventRecord(g.ready, st);
        }
    }
    // Host weights: copied on a second stream after the Hessians (which the factorisations need first), so the
    // transfer overlaps the factorisations; `st` waits for it before the weights are permuted.
    cudaEvent_t w_ready = nullptr;
    if (!w_uploads.empty()) {
        cudaStream_t cs = copy_stream();
        cudaEvent_t h_done = nullptr;
        CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&h_done, cudaEventDisableTiming));
        CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&w_ready, cudaEventDisableTiming));
        cudaEventRecord(h_done, st);
        cudaStreamWaitEvent(cs, h_done, 0);
        cudaEventDestroy(h_done);
        for (size_t li : w_uploads) {
            const LayerPlan& P = plans[li];
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(const_cast<float*>(P.w_dev), layers[li].w, P.d_out * P.n * sizeof(float),
                                           cudaMemcpyHostToDevice, cs));
        }
        cudaEventRecord(w_ready, cs);
    }
    uint64_t factor_batches = 0;
    rc = factorize_groups(groups, cfg, st, &factor_batches);
    if (w_ready) {
        cudaStreamWaitEvent(st, w_ready, 0);
        cudaEventDestroy(w_ready);
    }
    if (rc) {
        if (cache) {
            for (auto& pe : preps) pe.release();
        }
        return rc;
    }
    if (cache && !preps.empty()) {
        cache->e = preps[0];
        cache->key = hkey;
        cache->valid = true;
        preps[0].owned = false;  // ownership moved to the cache
        cached = &cache->e;
        for (auto& P : plans)
            if (P.prep == 0) P.prep = -2;
    }
    auto prep_of = [&](const LayerPlan& P) -> const PrepEntry& { return P.prep == -2 ? *cached : preps[P.prep]; };

    // ---- permuted target weights, asymmetric target, working buffers
    const bool cdcl = cfg.method == CDCLQ_METHOD_CDCL;
    const bool do_cd = cfg.refine_frac > 0.0 && cfg.cd_sweeps > 0 && cfg.passes > 0;
    size_t total_chunks = 0;
    for (size_t li = 0; li < layers.size(); li++) {
        LayerPlan& P = plans[li];
        const LayerReq& L = layers[li];
        const PrepEntry& pe = prep_of(P);
        const size_t cnt = P.d_out * P.n;
        if ((rc = ar.alloc(&P.wt, cnt))) return rc;
        if ((rc = launch_permute_w(P.w_dev, hdiag_dev[L.input], pe.perm_dev, (int)P.d_out, (int)P.n, P.wt, st)))
            return rc;
        if (!on_device) ar.free_one(const_cast<float*>(P.w_dev));
        if (L.m) {  // src/engine.rs:737-755
            const size_t n = P.n;
            const float* m_dev = L.m;
            float* mtmp = nullptr;
            if (!on_device) {
                if ((rc = ar.alloc(&mtmp, n * n))) return rc;
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(mtmp, L.m, n * n * sizeof(float), cudaMemcpyHostToDevice, st));
                m_dev = mtmp;
            }
            float *mp = nullptr, *t1 = nullptr, *t2 = nullptr;
            if ((rc = ar.alloc(&mp, n * n))) return rc;
            if ((rc = ar.alloc(&t1, cnt))) return rc;
            if ((rc = ar.alloc(&t2, cnt))) return rc;
            if ((rc = launch_permute_m(m_dev, pe.perm_dev, (int)n, (float)pe.damp_val, mp, st))) return rc;
            if ((rc = launch_sgemm((int)P.d_out, (int)n, (int)n, 1.0f, P.wt, (int64_t)n, false, mp, (int64_t)n, false,
                                   0.0f, t1, (int64_t)n, st)))
                return rc;
            if ((rc = launch_sgemm((int)P.d_out, (int)n, (int)n, 1.0f, t1, (int64_t)n, false, pe.u, (int64_t)n, true,
                                   0.0f, t2, (int64_t)n, st)))
                return rc;
            if ((rc = launch_sgemm((int)P.d_out, (int)n, (int)n, 1.0f, t2, (int64_t)n, false, pe.u, (int64_t)n, false,
                                   0.0f, P.wt, (int64_t)n, st)))
                return rc;
            ar.free_one(mp);
            ar.free_one(t1);
            ar.free_one(t2);
            if (mtmp) ar.free_one(mtmp);
        }
        if ((rc = ar.alloc(&P.w, cnt))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(P.w, P.wt, cnt * sizeof(float), cudaMemcpyDeviceToDevice, st));
        if ((rc = ar.alloc(&P.wq, cnt))) return rc;
        if ((rc = ar.alloc(&P.e, cnt))) return rc;
        if (on_device) {
            P.codes = L.codes;
            P.scales = L.scales;
            P.zeros = L.zeros;
        } else {
            if ((rc = ar.alloc(&P.codes, cnt))) return rc;
            if ((rc = ar.alloc(&P.scales, P.d_out * P.ng))) return rc;
            if ((rc = ar.alloc(&P.zeros, P.d_out * P.ng))) return rc;
        }
        if ((rc = ar.alloc(&P.gbits_dev, P.ng))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(P.gbits_dev, P.gbits.data(), P.ng, cudaMemcpyHostToDevice, st));
        P.rc = row_chunk(cfg, P.d_out);
        P.nchunks = (P.d_out + P.rc - 1) / P.rc;
        P.chunk0 = total_chunks;
        total_chunks += P.nchunks;
        const size_t sbw = cfg.sub_block, n_sb = (P.n + sbw - 1) / sbw;
        if ((rc = ar.alloc(&P.colloss, P.nchunks * P.n))) return rc;
        if ((rc = ar.alloc(&P.sbsum, P.nchunks * n_sb))) return rc;
        if ((rc = ar.alloc(&P.sel, P.nchunks * n_sb))) return rc;
    }
    pev.record(1, st);
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    const double t_prep = now_s();

    // ---- work lists, heaviest layers first (cost ~ rows * n^2)
    std::vector<size_t> order(layers.size());
    for (size_t i = 0; i < order.size(); i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return plans[a].n > plans[b].n; });
    std::vector<P1Item> p1;
    std::vector<ChunkInfo> chunks(total_chunks);
    std::vector<SliceItem> slices;
    std::vector<int> chunk_order;  // chunk indices in launch order
    ChunkState* states_dev = nullptr;
    if ((rc = ar.alloc(&states_dev, total_chunks))) return rc;
    for (size_t oi : order) {
        LayerPlan& P = plans[oi];
        const PrepEntry& pe = prep_of(P);
        for (size_t r0 = 0; r0 < P.d_out; r0 += 64) {
            P1Item it;
            it.w = P.w;
            it.wq = P.wq;
            it.eps2 = P.e;
            it.codes = P.codes;
            it.scales = P.scales;
            it.zeros = P.zeros;
            it.u = pe.u;
            it.gbits = P.gbits_dev;
            it.n = (int)P.n;
            it.g = (int)P.g;
            it.ng = (int)P.ng;
            it.row0 = (int)r0;
            it.rows = (int)std::min<size_t>(64, P.d_out - r0);
            p1.push_back(it);
        }
        const size_t sbw = cfg.sub_block, n_sb = (P.n + sbw - 1) / sbw;
        double kf = std::ceil(cfg.refine_frac * (double)n_sb);
        size_t ksel = kf > 0.0 ? (size_t)kf : 0;
        ksel = std::max<size_t>(1, std::min(ksel, n_sb));
        for (size_t c = 0; c < P.nchunks; c++) {
            size_t r0 = c * P.rc, rows = std::min(P.rc, P.d_out - r0);
            ChunkInfo ci;
            ci.wt = P.wt + r0 * P.n;
            ci.wq = P.wq + r0 * P.n;
            ci.e = P.e + r0 * P.n;
            ci.codes = P.codes + r0 * P.n;
            ci.scales = P.scales + r0 * P.ng;
            ci.zeros = P.zeros + r0 * P.ng;
            ci.h = pe.h32;
            ci.gbits = P.gbits_dev;
            ci.colloss = P.colloss + c * P.n;
            ci.sbsum = P.sbsum + c * n_sb;
            ci.sel = P.sel + c * n_sb;
            ci.st = states_dev + P.chunk0 + c;
            ci.n = (int)P.n;
            ci.rows = (int)rows;
            ci.g = (int)P.g;
            ci.ng = (int)P.ng;
            ci.sbw = (int)sbw;
            ci.n_sb = (int)n_sb;
            ci.k_sel = (int)ksel;
            ci.pad = 0;
            chunks[P.chunk0 + c] = ci;
            chunk_order.push_back((int)(P.chunk0 + c));
        }
    }
    // chunks in launch order (their states keep the layer-major index)
    std::vector<ChunkInfo> chunks_l(total_chunks);
    std::vector<int> slice_begin(total_chunks + 1, 0);
    for (size_t i = 0; i < total_chunks; i++) {
        chunks_l[i] = chunks[chunk_order[i]];
        slice_begin[i] = (int)slices.size();
        for (int r0 = 0; r0 < chunks_l[i].rows; r0 += 64) {
            SliceItem s;
            s.chunk = (int)i;
            s.r0 = r0;
            s.rs = std::min(64, chunks_l[i].rows - r0);
            s.pad = 0;
            slices.push_back(s);
        }
    }
    slice_begin[total_chunks] = (int)slices.size();
    P1Item* p1_dev = nullptr;
    ChunkInfo* chunks_dev = nullptr;
    SliceItem* slices_dev = nullptr;
    SliceAcc* acc_dev = nullptr;
    int* sb_dev = nullptr;
    if ((rc = ar.alloc(&p1_dev, p1.size()))) return rc;
    if ((rc = ar.alloc(&chunks_dev, total_chunks))) return rc;
    if ((rc = ar.alloc(&slices_dev, slices.size()))) return rc;
    if ((rc = ar.alloc(&acc_dev, slices.size()))) return rc;
    if ((rc = ar.alloc(&sb_dev, total_chunks + 1))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(p1_dev, p1.data(), sizeof(P1Item) * p1.size(), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(chunks_dev, chunks_l.data(), sizeof(ChunkInfo) * total_chunks, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(slices_dev, slices.data(), sizeof(SliceItem) * slices.size(), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(sb_dev, slice_begin.data(), sizeof(int) * (total_chunks + 1), cudaMemcpyHostToDevice, st));

    // ---- phase 1, statistics, phase 2
    const size_t blk = cfg.block;
    size_t maxn = 0;
    for (auto& P : plans) maxn = std::max(maxn, P.n);
    if ((rc = launch_phase1(p1_dev, (int)p1.size(), (int)std::min(blk, maxn), cfg.mse_grid ? 1 : 0, st))) return rc;
    pev.record(2, st);
    RepairParams rp;
    rp.do_refit = (cfg.refit_scales && plans[0].g <= 1024) ? 1 : 0;
    rp.do_cd = do_cd ? 1 : 0;
    rp.cd_sweeps = (int)cfg.cd_sweeps;
    rp.method_cdcl = cdcl ? 1 : 0;
    rp.final_refit = 0;
    rp.tol = cfg.tol;
    // refit is decided per layer in the reference (g <= 1024); all layers of a batch share cfg but g depends
    // on n, so a batch mixing "g <= 1024" and "g > 1024" layers is split by the caller.
    if ((rc = launch_chunk_stats(chunks_dev, (int)total_chunks, rp, st))) return rc;
    pev.record(3, st);
    uint64_t repair_launches = 0;
    rp.max_passes = (int)std::max<size_t>(cfg.passes, 1);
    int sms = 148;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    // Many row chunks: one persistent launch, chunks scheduled heaviest first.  Few row chunks: one launch per
    // pass over 64-row slices, so a chunk's rows spread over several SMs.  All modes give identical codes,
    // scales and pass counts; the f64 loss bookkeeping adds per-tile sums, so its last bits depend on the tile
    // height.
    size_t max_rows = 0;
    for (auto& P : plans) max_rows = std::max(max_rows, std::min(P.rc, P.d_out));
    const int layout = repair_layout_override();
    int layout_used = 5;  // reported in the run profile (cdclq_run_profile.repair_layout)
    const bool persistent = layout == LAYOUT_AUTO ? total_chunks >= (size_t)sms : layout != LAYOUT_PASSES;
    if (cdcl && (rp.do_cd || rp.do_refit) && persistent) {
        int* counter = nullptr;
        if ((rc = ar.alloc(&counter, 1))) return rc;
        const int g0 = (int)plans[0].g, sbw0 = (int)std::min<size_t>(cfg.sub_block, maxn);
        int bm = repair_tile_rows(g0, sbw0, (int)max_rows);
        // chunks of more than one row tile: a 2-CTA cluster per chunk
        bool cluster = max_rows > (size_t)bm && max_rows <= (size_t)bm * RP_MAX_TILES_PER_CHUNK;
        int split = 0, split_sms = 0;  // > 0: the first `split` chunks run apart (see below)
        bool quads = false;            // ... as 4-CTA clusters (else as 2-CTA clusters)
        if (!cluster && bm == 128) {
            // Launch layouts, compared by their estimated makespan (chunk work ~ rows x n^2 per pass):
            //  S  one CTA per 128-row chunk, two CTAs per SM: the efficient GEMM shape, but a chunk's passes run
            //     on one CTA, so the heaviest chunk alone can outlast the average load of a CTA slot (few chunks
            //     per slot, as in one GPU's row shard of a model);
            //  P  every chunk's rows over a 2-CTA cluster of 64-row tiles (GEMMs at ~0.79 of the 128-row rate);
            //  H  the heaviest chunks (the widest layers, first in launch order) as 2-CTA clusters whose CTAs each
            //     own an SM (an 8-warp CTA alone runs ~1.3x faster than when it shares the SM), concurrently with
            //     a persistent launch of the other chunks on the remaining SMs.
            //  Q  as H, the heavy chunks (two 64-row tiles each) over 4-CTA clusters that also split every GEMM's
            //     columns between two CTAs (QS: the measured speed-up of a 5632-wide chunk over its 2-CTA form:
            //     only the GEMMs shrink, the per-row sequential refit and sweeps keep their latency).
            constexpr double E64 = 0.79, ALONE = 1.3, QS = 1.2;
            std::vector<double> cw(total_chunks);
            double total_w = 0.0, max_w = 0.0;
            for (size_t i = 0; i < total_chunks; i++) {
                const ChunkInfo& c = chunks_l[i];
                cw[i] = (double)c.rows * (double)c.n * (double)c.n;
                total_w += cw[i];
                max_w = std::max(max_w, cw[i]);
            }
            const double slots = 2.0 * sms;
            const double t_single = std::max(total_w / slots, max_w);
            const double t_pair = std::max(total_w / (slots * E64), 0.5 * max_w / E64);
            double best = std::min(t_single, t_pair);
            int mode = t_pair < t_single ? 1 : 0;
            // heavy prefix: the chunks of the widest layers
            size_t nh = 0;
            while (nh < total_chunks && chunks_l[nh].n == chunks_l[0].n) nh++;
            bool two_tiles = true;  // the 4-CTA form takes chunks of exactly two 64-row tiles
            for (size_t i = 0; i < nh; i++) two_tiles = two_tiles && chunks_l[i].rows > 64 && chunks_l[i].rows <= 128;
            if (nh < total_chunks && max_w > total_w / slots) {
                double wh = 0.0;
                for (size_t i = 0; i < nh; i++) wh += cw[i];
                const double wl = total_w - wh;
                for (int s_h = 2; s_h < sms; s_h += 2) {
                    if ((size_t)s_h > 4 * nh) break;
                    const double tl = wl / (2.0 * (sms - s_h));
                    if ((size_t)s_h <= 2 * nh) {
                        const double th = std::max(max_w / (2.0 * E64 * ALONE), wh / (s_h * E64 * ALONE));
                        const double t = std::max(th, tl);
                        if (t < best) {
                            best = t;
                            mode = 2;
                            split = (int)nh;
                            split_sms = s_h;
                        }
                    }
                    if (two_tiles && s_h % 4 == 0) {
                        const double th = std::max(max_w / (2.0 * E64 * ALONE * QS), wh / (0.5 * s_h * E64 * ALONE * QS));
                        const double t = std::max(th, tl);
                        if (t < best) {
                            best = t;
                            mode = 3;
                            split = (int)nh;
                            split_sms = s_h;
                        }
                    }
                }
            }
            if (layout == LAYOUT_SINGLE) mode = 0;
            if (layout == LAYOUT_PAIRS) mode = 1;
            if (layout == LAYOUT_SPLIT || (layout == LAYOUT_QUADS && !two_tiles)) {
                if (nh < total_chunks) {  // the widest layers' chunks apart, each cluster CTA on its own SM
                    mode = 2;
                    split = (int)nh;
                    split_sms = (int)std::max<size_t>(2, std::min<size_t>(2 * nh, (size_t)sms / 2)) & ~1;
                } else {
                    mode = 0;  // one width only: nothing to split off
                }
            } else if (layout == LAYOUT_QUADS) {
                mode = 3;  // the widest layers' chunks as quads (all of them when there is one width only)
                split = (int)nh;
                split_sms = (int)std::max<size_t>(4, std::min<size_t>(4 * nh, (size_t)sms / 2)) & ~3;
            }
            if (mode == 1) {
                bm = 64;
                cluster = true;
            }
            if (mode != 2 && mode != 3) split = 0;
            quads = mode == 3;
        }
        layout_used = split > 0 ? (quads ? 4 : 3) : cluster ? 2 : 1;
        if (split > 0) {
            // heavy chunks on `st` (one CTA per SM), the others on a second stream, joined on `st`
            int* counter_l = nullptr;
            if ((rc = ar.alloc(&counter_l, 1))) return rc;
            cudaStream_t ls = pool_stream(0);
            cudaEvent_t fork = nullptr, join = nullptr;
            CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
            CDCLQ_CUDA_TRY(cudaEventCreateWithFlags(&join, cudaEventDisableTiming));
            cudaEventRecord(fork, st);
            cudaStreamWaitEvent(ls, fork, 0);
            size_t maxsm = 0;
            {
                int dev = 0, v = 0;
                cudaGetDevice(&dev);
                cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
                maxsm = (size_t)v;
            }
            rc = quads ? launch_repair_quad(chunks_dev, split, rp, g0, sbw0, counter, st, split_sms, maxsm / 2 + 4096)
                       : launch_repair_cluster(chunks_dev, split, rp, g0, sbw0, 64, counter, st, split_sms,
                                               maxsm / 2 + 4096);
            if (!rc && split < (int)total_chunks)
                rc = launch_repair_persistent(chunks_dev + split, (int)total_chunks - split, rp, g0, sbw0, 128,
                                              counter_l, ls, 2 * (sms - split_sms));
            cudaEventRecord(join, ls);
            cudaStreamWaitEvent(st, join, 0);
            cudaEventDestroy(fork);
            cudaEventDestroy(join);
        } else if (cluster)
            rc = launch_repair_cluster(chunks_dev, (int)total_chunks, rp, g0, sbw0, bm, counter, st);
        else
            rc = launch_repair_persistent(chunks_dev, (int)total_chunks, rp, g0, sbw0, bm, counter, st);
        if (rc) return rc;
        repair_launches = 1;
        pev.record(4, st);
    } else if (cdcl && (rp.do_cd || rp.do_refit)) {
        layout_used = 0;
        size_t max_passes = std::max<size_t>(cfg.passes, 1);
        for (size_t p = 0; p < max_passes; p++) {
            if ((rc = launch_repair_pass(chunks_dev, slices_dev, (int)slices.size(), acc_dev, rp, (int)plans[0].g,
                                         (int)std::min<size_t>(cfg.sub_block, maxn), st)))
                return rc;
            if ((rc = launch_pass_end(chunks_dev, (int)total_chunks, sb_dev, acc_dev, rp, st))) return rc;
            repair_launches++;
        }
        pev.record(4, st);
        if (rp.do_refit) {
            RepairParams fr = rp;
            fr.final_refit = 1;
            if ((rc = launch_repair_pass(chunks_dev, slices_dev, (int)slices.size(), acc_dev, fr, (int)plans[0].g,
                                         (int)std::min<size_t>(cfg.sub_block, maxn), st)))
                return rc;
            if ((rc = launch_pass_end(chunks_dev, (int)total_chunks, sb_dev, acc_dev, fr, st))) return rc;
        }
    }
    if (!(cdcl && (rp.do_cd || rp.do_refit)) || persistent) pev.record(4, st);
    pev.record(5, st);
    std::vector<ChunkState> states(total_chunks);
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(states.data(), states_dev, sizeof(ChunkState) * total_chunks, cudaMemcpyDeviceToHost, st));
    if (!on_device) {
        for (size_t li = 0; li < layers.size(); li++) {
            const LayerPlan& P = plans[li];
            const LayerReq& L = layers[li];
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(L.codes, P.codes, P.d_out * P.n, cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(L.scales, P.scales, P.d_out * P.ng * sizeof(float), cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(L.zeros, P.zeros, P.d_out * P.ng * sizeof(float), cudaMemcpyDeviceToHost, st));
        }
    }
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    const double t_end = now_s();

    // ---- profile: event times and algorithmic work
    {
        cdclq_run_profile& pf = g_profile;
        std::memset(&pf, 0, sizeof pf);
        pf.ms_prepare = pev.ms(0, 1);
        pf.ms_phase1 = pev.ms(1, 2);
        pf.ms_stats = pev.ms(2, 3);
        pf.ms_repair = pev.ms(3, 4);
        pf.ms_final = pev.ms(4, 5);
        pf.repair_launches = repair_launches;
        for (const auto& P : plans) {
            const double rows = (double)P.d_out, n = (double)P.n;
            pf.weights += P.d_out * P.n;
            double f1 = 0.0;
            for (size_t i1 = 0; i1 < P.n; i1 += cfg.block) {
                size_t i2 = std::min(i1 + (size_t)cfg.block, P.n), cnt = i2 - i1;
                f1 += 2.0 * (double)cnt * (double)(P.n - i2) + (double)cnt * (double)(cnt - 1);
            }
            pf.flops_phase1 += rows * f1;
            if (cdcl && (rp.do_cd || rp.do_refit)) {
                for (size_t c = 0; c < P.nchunks; c++) {
                    const ChunkState& cs = states[P.chunk0 + c];
                    const double cr = (double)std::min(P.rc, P.d_out - c * P.rc);
                    double f_refit = rp.do_refit ? 2.0 * cr * n * n + 2.0 * cr * n * (double)P.g : 0.0;
                    double sel_cols = 0.0;
                    if (rp.do_cd) {
                        // selected sub-blocks are full width except possibly the last one
                        const size_t sbw = cfg.sub_block, n_sb = (P.n + sbw - 1) / sbw;
                        const size_t last_w = P.n - (n_sb - 1) * sbw;
                        sel_cols = (double)cs.n_sel * (double)sbw;
                        if ((size_t)cs.n_sel == n_sb) sel_cols = sel_cols - (double)sbw + (double)last_w;
                    }
                    double f_cd = 2.0 * cr * n * sel_cols;
                    pf.flops_repair += (double)cs.passes * (f_refit + f_cd);
                    pf.flops_final += f_refit;
                }
            }
        }
        for (const auto& pe : preps) {
            const double n = (double)pe.n;
            pf.flops_factor += 2.0 * n * n * n / 3.0;
            pf.factorisations++;
        }
        pf.launches = g_launches.load() - launches0;
        pf.factor_batches = factor_batches;
        pf.ms_host = (now_s() - t_start) * 1e3;
        pf.repair_layout = (uint64_t)layout_used;
    }

    // ---- statistics, summed over chunks in order (src/engine.rs:786-797)
    for (size_t li = 0; li < layers.size(); li++) {
        const LayerPlan& P = plans[li];
        const LayerReq& L = layers[li];
        cdclq_layer_stats s;
        std::memset(&s, 0, sizeof s);
        const size_t n_sb = (P.n + cfg.sub_block - 1) / cfg.sub_block;
        for (size_t c = 0; c < P.nchunks; c++) {
            const ChunkState& cs = states[P.chunk0 + c];
            s.loss_gptq += cs.loss_gptq;
            s.loss_final += cs.loss_gptq + cs.loss_delta;
            s.subblocks_total += n_sb;
            s.subblocks_refined += (cdcl && (rp.do_cd || rp.do_refit)) ? (uint64_t)cs.n_sel : 0;
            s.code_updates += cs.updates;
            s.passes_max = std::max<uint64_t>(s.passes_max, (uint64_t)cs.passes);
            if (L.chunk_passes) L.chunk_passes[c] = (uint32_t)cs.passes;
        }
        s.skeleton_groups = P.nskel;
        size_t bits = 0;
        for (size_t j = 0; j < P.n; j++) bits += P.gbits[j / P.g];
        s.bits_codes = (double)bits / (double)P.n;
        s.bits_total = s.bits_codes + 24.0 / (double)P.g;
        s.secs_prepare = t_prep - t_start;
        s.secs_quant = t_end - t_prep;
        *L.stats = s;
        std::memcpy(L.perm, P.perm.data(), P.n * sizeof(uint32_t));
        std::memcpy(L.gbits, P.gbits.data(), P.ng);
    }
    return CDCLQ_OK;
}

// Permutation, group widths and skeleton group count of a layer (src/engine.rs:271-304, 761-763) from its
// Hessian on the device and, with a skeleton, the column scores of its full weight matrix (host, n f64, original
// order; null without a skeleton).  What cdclq_quantize_batch computes for the layer; the multi-GPU runtime
// uses it on every rank, rows or not, so that each rank reports every layer's permutation.
int layer_perm(const float* h_dev, size_t n, const double* colsq, const cdclq_config& cfg, std::vector<uint32_t>& perm,
               std::vector<uint8_t>& gbits, size_t& nskel, cudaStream_t st) {
    double* hd = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync(&hd, n * sizeof(double), st));
    int rc = launch_hdiag(h_dev, (int)n, hd, st);
    std::vector<double> hdiag(n);
    if (!rc) {
        cudaError_t e = cudaMemcpyAsync(hdiag.data(), hd, n * sizeof(double), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_error(e, "hdiag read-back");
    }
    cudaFreeAsync(hd, st);
    if (rc) return rc;
    const size_t g = effective_group(cfg, n);
    std::vector<double> cs;
    if (colsq) cs.assign(colsq, colsq + n);
    compute_perm(hdiag, colsq ? &cs : nullptr, n, g, cfg, perm, nskel);
    const size_t ng = (n + g - 1) / g;
    gbits.resize(ng);
    for (size_t gi = 0; gi < ng; gi++) gbits[gi] = (uint8_t)(gi < nskel ? cfg.skeleton_bits : cfg.bits);
    return 0;
}

int ensure_device() {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return set_error(CDCLQ_ERR_CUDA, std::string("no CUDA device available: ") + cudaGetErrorString(e));
    // The per-call buffers come from the device's default stream-ordered pool.  Keep freed pool memory cached
    // instead of returning it to the driver at every synchronisation (release threshold 0 by default), so a
    // repeated call does not pay for re-mapping tens of GB.
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
        static bool configured[64] = {false};
        if (!configured[dev]) {
            cudaMemPool_t pool;
            if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
                uint64_t threshold = UINT64_MAX;
                cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
            }
            configured[dev] = true;
        }
    }
    return 0;
}

}  // namespace cdclq

// =========================================================================================================
// C ABI
using namespace cdclq;

extern "C" {

const char* cdclq_version(void) { return "cdclq-b200 0.1 (sm_100a)"; }

uint64_t cdclq_launch_count(void) { return g_launches.load(); }

int cdclq_last_run_profile(cdclq_run_profile* out) {
    if (!out) return set_error(CDCLQ_ERR_ARG, "null argument");
    *out = g_profile;
    return CDCLQ_OK;
}

const char* cdclq_last_error(void) { return g_last_error.c_str(); }

void cdclq_config_default(cdclq_config* c) {
    if (!c) return;
    std::memset(c, 0, sizeof *c);
    c->bits = 3;
    c->group = 128;
    c->block = 128;
    c->damp = 0.01;
    c->act_order = 1;
    c->skeleton_pct = 0.0;
    c->skeleton_bits = 8;
    c->mse_grid = 0;
    c->method = CDCLQ_METHOD_CDCL;
    c->refine_frac = 1.0;
    c->sub_block = 64;
    c->cd_sweeps = 1;
    c->passes = 10;
    c->tol = 1e-3;
    c->refit_scales = 1;
    c->row_chunk = 0;
    c->threads = 0;
}

size_t cdclq_effective_group(const cdclq_config* c, size_t n) { return c ? effective_group(*c, n) : n; }

size_t cdclq_num_groups(const cdclq_config* c, size_t n) {
    if (!c || n == 0) return 0;
    size_t g = effective_group(*c, n);
    return (n + g - 1) / g;
}

int cdclq_validate(const cdclq_config* c, size_t n) {
    if (!c) return set_error(CDCLQ_ERR_ARG, "null config");
    return validate(*c, n);
}

size_t cdclq_row_chunk(const cdclq_config* c, size_t d_out) { return c ? row_chunk(*c, d_out) : 0; }

cdclq_prep_cache* cdclq_prep_cache_new(void) { return new cdclq_prep_cache(); }

void cdclq_prep_cache_free(cdclq_prep_cache* c) { delete c; }

int cdclq_quantize_layer_ex(const float* w, size_t d_out, size_t d_in, const float* h, const float* m,
                            const char* hkey, const cdclq_config* cfg, cdclq_prep_cache* cache, uint32_t* perm_out,
                            uint8_t* gbits_out, uint8_t* codes_out, float* scales_out, float* zeros_out,
                            cdclq_layer_stats* stats_out, uint32_t* chunk_passes_out) {
    if (!cfg) return set_error(CDCLQ_ERR_ARG, "null config");
    int rc = ensure_device();
    if (rc) return rc;
    std::vector<InputReq> in(1);
    in[0].h = h;
    in[0].n = d_in;
    std::vector<LayerReq> ly(1);
    ly[0].w = w;
    ly[0].d_out = d_out;
    ly[0].input = 0;
    ly[0].m = m;
    ly[0].perm = perm_out;
    ly[0].gbits = gbits_out;
    ly[0].codes = codes_out;
    ly[0].scales = scales_out;
    ly[0].zeros = zeros_out;
    ly[0].stats = stats_out;
    ly[0].chunk_passes = chunk_passes_out;
    std::string key = hkey ? hkey : "";
    return run(in, ly, *cfg, false, lib_stream(), cache, key);
}

int cdclq_quantize_layer(const float* w, size_t d_out, size_t d_in, const float* h, const float* m, const char* hkey,
                         const cdclq_config* cfg, cdclq_prep_cache* cache, uint32_t* perm_out, uint8_t* gbits_out,
                         uint8_t* codes_out, float* scales_out, float* zeros_out, cdclq_layer_stats* stats_out) {
    return cdclq_quantize_layer_ex(w, d_out, d_in, h, m, hkey, cfg, cache, perm_out, gbits_out, codes_out, scales_out,
                                   zeros_out, stats_out, nullptr);
}

static int quantize_batch_impl(const cdclq_batch_input* inputs, size_t n_inputs, const float* const* u_in,
                               const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config* cfg, int on_device,
                               void* stream) {
    if (!cfg || (!inputs && n_inputs) || (!layers && n_layers)) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    if (n_layers == 0) return CDCLQ_OK;
    std::vector<InputReq> in(n_inputs);
    for (size_t i = 0; i < n_inputs; i++) {
        in[i].h = inputs[i].h;
        in[i].n = inputs[i].n;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : (on_device ? (cudaStream_t)0 : lib_stream());
    // The refit switch depends on the group width (src/engine.rs:492); a batch runs one switch, so layers are
    // grouped by (g <= 1024) and by width-independent settings.
    std::vector<LayerReq> small, large;
    for (size_t i = 0; i < n_layers; i++) {
        LayerReq L;
        L.w = layers[i].w;
        L.d_out = layers[i].d_out;
        L.input = layers[i].input;
        L.perm = layers[i].perm;
        L.gbits = layers[i].gbits;
        L.codes = layers[i].codes;
        L.scales = layers[i].scales;
        L.zeros = layers[i].zeros;
        L.stats = layers[i].stats;
        L.colsq = layers[i].colsq;
        L.u = layers[i].u;
        if (L.input >= n_inputs) return set_error(CDCLQ_ERR_ARG, "layer input index out of range");
        size_t g = effective_group(*cfg, in[L.input].n);
        (g <= 1024 ? small : large).push_back(L);
    }
    // mixed group widths: layers whose g differs get their own launch sequence
    auto run_groups = [&](std::vector<LayerReq>& v) -> int {
        std::map<size_t, std::vector<LayerReq>> by_g;
        for (auto& L : v) by_g[effective_group(*cfg, in[L.input].n)].push_back(L);
        for (auto& kv : by_g) {
            int r = run(in, kv.second, *cfg, on_device != 0, st, nullptr, "", u_in);
            if (r) return r;
        }
        return 0;
    };
    if ((rc = run_groups(small))) return rc;
    return run_groups(large);
}

int cdclq_quantize_batch(const cdclq_batch_input* inputs, size_t n_inputs, const cdclq_batch_layer* layers,
                         size_t n_layers, const cdclq_config* cfg, int on_device, void* stream) {
    return quantize_batch_impl(inputs, n_inputs, nullptr, layers, n_layers, cfg, on_device, stream);
}

int cdclq_quantize_batch_prepared(const cdclq_batch_input* inputs, size_t n_inputs, const float* const* u_in,
                                  const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config* cfg,
                                  int on_device, void* stream) {
    if (!u_in) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (cfg && cfg->skeleton_pct > 0.0)
        return set_error(CDCLQ_ERR_CONFIG, "prepared factors need a W-independent permutation (skeleton_pct = 0)");
    return quantize_batch_impl(inputs, n_inputs, u_in, layers, n_layers, cfg, on_device, stream);
}

int cdclq_prepare_factors(const cdclq_batch_input* inputs, size_t n_inputs, const size_t* which, size_t n_which,
                          const cdclq_config* cfg, float* const* u_out, int on_device, void* stream) {
    if (!cfg || (!inputs && n_inputs) || (!which && n_which) || (!u_out && n_which))
        return set_error(CDCLQ_ERR_ARG, "null argument");
    if (cfg->skeleton_pct > 0.0)
        return set_error(CDCLQ_ERR_CONFIG, "prepared factors need a W-independent permutation (skeleton_pct = 0)");
    int rc = ensure_device();
    if (rc) return rc;
    if (n_which == 0) return CDCLQ_OK;
    cudaStream_t st = stream ? (cudaStream_t)stream : (on_device ? (cudaStream_t)0 : lib_stream());
    Arena ar(st);
    std::vector<PrepEntry> preps(n_which);
    std::vector<const float*> h_dev(n_which, nullptr);
    std::map<size_t, std::vector<size_t>> by_n;
    for (size_t k = 0; k < n_which; k++) {
        const size_t i = which[k];
        if (i >= n_inputs) return set_error(CDCLQ_ERR_ARG, "input index out of range");
        const size_t n = inputs[i].n;
        if (n == 0 || !inputs[i].h || !u_out[k]) return set_error(CDCLQ_ERR_ARG, "null argument");
        if ((rc = validate(*cfg, n))) return rc;
        if ((rc = check_tiling(*cfg, n))) return rc;
        // act-order (or natural) permutation from the raw diagonal (src/engine.rs:271-304, no skeleton)
        std::vector<double> hdiag(n);
        if (on_device) {
            double* dg = nullptr;
            if ((rc = ar.alloc(&dg, n))) return rc;
            if ((rc = launch_hdiag(inputs[i].h, (int)n, dg, st))) return rc;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(hdiag.data(), dg, n * sizeof(double), cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
            ar.free_one(dg);
            h_dev[k] = inputs[i].h;
        } else {
            for (size_t j = 0; j < n; j++) hdiag[j] = (double)inputs[i].h[j * n + j];
            float* hd = nullptr;
            if ((rc = ar.alloc(&hd, n * n))) return rc;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(hd, inputs[i].h, n * n * sizeof(float), cudaMemcpyHostToDevice, st));
            h_dev[k] = hd;
        }
        PrepEntry& pe = preps[k];
        size_t nskel = 0;
        compute_perm(hdiag, nullptr, n, effective_group(*cfg, n), *cfg, pe.perm, nskel);
        pe.n = n;
        pe.u = u_out[k];
        pe.h32 = nullptr;  // only U is wanted: the quantizing ranks rebuild the damped Hessian themselves
        if ((rc = ar.alloc(&pe.perm_dev, n))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(pe.perm_dev, pe.perm.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
        by_n[n].push_back(k);
    }
    std::vector<FactorGroup> groups;
    for (auto it = by_n.rbegin(); it != by_n.rend(); ++it) {  // widest first: the longest factorisations
        FactorGroup g;
        g.n = it->first;
        for (size_t k : it->second) {
            g.hs.push_back(h_dev[k]);
            g.es.push_back(&preps[k]);
        }
        groups.push_back(std::move(g));
    }
    // factorize_groups waits on the host for every factor stream: the factors are complete on return
    rc = factorize_groups(groups, *cfg, st);
    if (!rc) CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return rc;
}

int cdclq_prepare_layer_factors(const cdclq_batch_input* inputs, size_t n_inputs, const cdclq_batch_layer* layers,
                                size_t n_layers, const size_t* which, size_t n_which, const cdclq_config* cfg,
                                float* const* u_out, int on_device, void* stream) {
    if (!cfg || (!inputs && n_inputs) || (!layers && n_layers) || (!which && n_which) || (!u_out && n_which))
        return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    if (n_which == 0) return CDCLQ_OK;
    cudaStream_t st = stream ? (cudaStream_t)stream : (on_device ? (cudaStream_t)0 : lib_stream());
    Arena ar(st);
    // per input: the raw diagonal (host and device) and the Hessian on the device
    std::vector<std::vector<double>> hdiag(n_inputs);
    std::vector<double*> hdiag_dev(n_inputs, nullptr);
    std::vector<const float*> h_dev(n_inputs, nullptr);
    std::vector<PrepEntry> preps(n_which);
    std::map<size_t, std::vector<size_t>> by_n;
    for (size_t k = 0; k < n_which; k++) {
        const size_t li = which[k];
        if (li >= n_layers) return set_error(CDCLQ_ERR_ARG, "layer index out of range");
        const cdclq_batch_layer& L = layers[li];
        const size_t i = L.input;
        if (i >= n_inputs) return set_error(CDCLQ_ERR_ARG, "layer input index out of range");
        const size_t n = inputs[i].n;
        if (n == 0 || !inputs[i].h || !u_out[k]) return set_error(CDCLQ_ERR_ARG, "null argument");
        if ((rc = validate(*cfg, n))) return rc;
        if ((rc = check_tiling(*cfg, n))) return rc;
        if (!h_dev[i]) {
            if (on_device) {
                h_dev[i] = inputs[i].h;
            } else {
                float* hd = nullptr;
                if ((rc = ar.alloc(&hd, n * n))) return rc;
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(hd, inputs[i].h, n * n * sizeof(float), cudaMemcpyHostToDevice, st));
                h_dev[i] = hd;
            }
            hdiag[i].resize(n);
            if ((rc = ar.alloc(&hdiag_dev[i], n))) return rc;
            if ((rc = launch_hdiag(h_dev[i], (int)n, hdiag_dev[i], st))) return rc;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(hdiag[i].data(), hdiag_dev[i], n * sizeof(double), cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
        }
        // the permutation exactly as the batch call builds it (src/engine.rs:271-304)
        const size_t g = effective_group(*cfg, n);
        const bool skel = cfg->skeleton_pct > 0.0 && g < n;
        std::vector<double> colsq;
        if (skel) {
            colsq.resize(n);
            if (L.colsq && !on_device) {
                std::copy(L.colsq, L.colsq + n, colsq.begin());
            } else if (L.colsq) {
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(colsq.data(), L.colsq, n * sizeof(double), cudaMemcpyDeviceToHost, st));
                CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
            } else {
                if (!L.w || L.d_out == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
                const float* wd = L.w;
                float* wtmp = nullptr;
                if (!on_device) {
                    if ((rc = ar.alloc(&wtmp, L.d_out * n))) return rc;
                    CDCLQ_CUDA_TRY(cudaMemcpyAsync(wtmp, L.w, L.d_out * n * sizeof(float), cudaMemcpyHostToDevice, st));
                    wd = wtmp;
                }
                double* cs_dev = nullptr;
                if ((rc = ar.alloc(&cs_dev, n))) return rc;
                if ((rc = launch_colsq(wd, hdiag_dev[i], (int)L.d_out, (int)n, cs_dev, st))) return rc;
                CDCLQ_CUDA_TRY(cudaMemcpyAsync(colsq.data(), cs_dev, n * sizeof(double), cudaMemcpyDeviceToHost, st));
                CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
                ar.free_one(cs_dev);
                if (wtmp) ar.free_one(wtmp);
            }
        }
        PrepEntry& pe = preps[k];
        size_t nskel = 0;
        compute_perm(hdiag[i], skel ? &colsq : nullptr, n, g, *cfg, pe.perm, nskel);
        pe.n = n;
        pe.u = u_out[k];
        pe.h32 = nullptr;  // only U is wanted: the quantizing ranks rebuild the damped Hessian themselves
        if ((rc = ar.alloc(&pe.perm_dev, n))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(pe.perm_dev, pe.perm.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
        by_n[n].push_back(k);
    }
    std::vector<FactorGroup> groups;
    for (auto it = by_n.rbegin(); it != by_n.rend(); ++it) {  // widest first
        FactorGroup g;
        g.n = it->first;
        for (size_t k : it->second) {
            g.hs.push_back(h_dev[layers[which[k]].input]);
            g.es.push_back(&preps[k]);
        }
        groups.push_back(std::move(g));
    }
    rc = factorize_groups(groups, *cfg, st);
    if (!rc) CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return rc;
}

// ---- linalg entry points (host buffers) -------------------------------------------------------------------

int cdclq_cholesky_lower(double* a, size_t n) {
    if (!a || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    double* d = nullptr;
    FactorStatus* s = nullptr;
    if ((rc = ar.alloc(&d, n * n)) || (rc = ar.alloc(&s, 1))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(d, a, n * n * sizeof(double), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(s, 0, sizeof(FactorStatus), st));
    if ((rc = device_cholesky(d, (int)n, s, st))) return rc;
    FactorStatus hs;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(&hs, s, sizeof hs, cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(a, d, n * n * sizeof(double), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    if (hs.err)
        return set_error(CDCLQ_ERR_NOT_PD, "matrix is not positive definite (pivot " + std::to_string(hs.pivot) + " = " +
                                               rust_exp(hs.value) + "); increase --damp or check the Hessian");
    return CDCLQ_OK;
}

int cdclq_tri_inverse_lower(const double* l, size_t n, double* y) {
    if (!l || !y || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    double *ld = nullptr, *yd = nullptr, *tb = nullptr;
    if ((rc = ar.alloc(&ld, n * n)) || (rc = ar.alloc(&yd, n * n)) || (rc = ar.alloc(&tb, 96 * n))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(ld, l, n * n * sizeof(double), cudaMemcpyHostToDevice, st));
    if ((rc = device_tri_inverse(ld, yd, tb, (int)n, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(y, yd, n * n * sizeof(double), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_upper_chol_of_inverse(const double* h, size_t n, float* u_out) {
    if (!h || !u_out || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    double *hr = nullptr, *yd = nullptr, *tb = nullptr;
    float* ud = nullptr;
    FactorStatus* s = nullptr;
    if ((rc = ar.alloc(&hr, n * n)) || (rc = ar.alloc(&yd, n * n)) || (rc = ar.alloc(&tb, 96 * n)) ||
        (rc = ar.alloc(&ud, n * n)) || (rc = ar.alloc(&s, 1)))
        return rc;
    // h.reverse() on the host-side copy (src/linalg.rs:364)
    std::vector<double> flipped(h, h + n * n);
    std::reverse(flipped.begin(), flipped.end());
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(hr, flipped.data(), n * n * sizeof(double), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemsetAsync(s, 0, sizeof(FactorStatus), st));
    if ((rc = device_cholesky(hr, (int)n, s, st))) return rc;
    FactorStatus hs;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(&hs, s, sizeof hs, cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    if (hs.err)
        return set_error(CDCLQ_ERR_NOT_PD, "matrix is not positive definite (pivot " + std::to_string(hs.pivot) + " = " +
                                               rust_exp(hs.value) + "); increase --damp or check the Hessian");
    if ((rc = device_tri_inverse(hr, yd, tb, (int)n, st))) return rc;
    PrepItem it;
    std::memset(&it, 0, sizeof it);
    it.y = yd;
    it.u = ud;
    it.status = s;
    PrepItem* itd = nullptr;
    if ((rc = ar.alloc(&itd, 1))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(itd, &it, sizeof it, cudaMemcpyHostToDevice, st));
    if ((rc = launch_u_scatter(itd, 1, (int)n, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(u_out, ud, n * n * sizeof(float), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_gram_accumulate_device(const float* x, const float* y, size_t t, size_t n, double* h, void* stream) {
    if (!x || !y || !h || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (n > 65535) return set_error(CDCLQ_ERR_ARG, "n above 65535 is not supported");
    cudaStream_t st = (cudaStream_t)stream;
    Arena ar(st);
    float* tmp = nullptr;
    int rc = ar.alloc(&tmp, n * n);
    if (rc) return rc;
    return launch_gram_f32(x, y, (int64_t)t, (int)n, h, tmp, st);
}

int cdclq_gram_accumulate(const float* x, const float* y, size_t t, size_t n, double* h) {
    if (!x || !y || !h || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    float *xd = nullptr, *yd = nullptr;
    double* hd = nullptr;
    if ((rc = ar.alloc(&xd, t * n)) || (rc = ar.alloc(&hd, n * n))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(xd, x, t * n * sizeof(float), cudaMemcpyHostToDevice, st));
    if (y == x) {
        yd = xd;
    } else {
        if ((rc = ar.alloc(&yd, t * n))) return rc;
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(yd, y, t * n * sizeof(float), cudaMemcpyHostToDevice, st));
    }
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(hd, h, n * n * sizeof(double), cudaMemcpyHostToDevice, st));
    if ((rc = cdclq_gram_accumulate_device(xd, yd, t, n, hd, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(h, hd, n * n * sizeof(double), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_column_scores_device(const float* w, size_t d_out, size_t n, const float* h, double* colsq_out,
                               void* stream) {
    if (!w || !h || !colsq_out || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (n > 0x7fffffff || d_out > 0x7fffffff) return set_error(CDCLQ_ERR_ARG, "matrix too large");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    Arena ar(st);
    double* hdiag = nullptr;
    if ((rc = ar.alloc(&hdiag, n))) return rc;
    if ((rc = launch_hdiag(h, (int)n, hdiag, st))) return rc;
    if ((rc = launch_colsq(w, hdiag, (int)d_out, (int)n, colsq_out, st))) return rc;
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_gram_accumulate_bf16_device(const void* x_bf16, size_t t, size_t n, double* h, int lower_only,
                                      void* stream) {
    if (!x_bf16 || !h || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();  // the split-token partials come from the (caching) stream-ordered pool
    if (rc) return rc;
    return launch_gram_half_tc(x_bf16, true, (int64_t)t, (int)n, h, lower_only, (cudaStream_t)stream);
}

int cdclq_gram_accumulate_half_device(const void* x, int dtype, size_t t, size_t n, double* h, int lower_only,
                                      void* stream) {
    if (!x || !h || n == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (dtype != CDCLQ_DTYPE_BF16 && dtype != CDCLQ_DTYPE_F16)
        return set_error(CDCLQ_ERR_ARG, "half Gram: dtype must be CDCLQ_DTYPE_BF16 or CDCLQ_DTYPE_F16");
    int rc = ensure_device();
    if (rc) return rc;
    return launch_gram_half_tc(x, dtype == CDCLQ_DTYPE_BF16, (int64_t)t, (int)n, h, lower_only, (cudaStream_t)stream);
}

int cdclq_proxy_loss(const float* w_t, const float* w_hat, size_t rows, size_t n, const float* h, double* out) {
    if (!w_t || !w_hat || !h || !out) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    float *a = nullptr, *b = nullptr, *hd = nullptr, *e = nullptr, *eh = nullptr;
    double* od = nullptr;
    if ((rc = ar.alloc(&a, rows * n)) || (rc = ar.alloc(&b, rows * n)) || (rc = ar.alloc(&hd, n * n)) ||
        (rc = ar.alloc(&e, rows * n)) || (rc = ar.alloc(&eh, rows * n)) || (rc = ar.alloc(&od, 1)))
        return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(a, w_t, rows * n * sizeof(float), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(b, w_hat, rows * n * sizeof(float), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(hd, h, n * n * sizeof(float), cudaMemcpyHostToDevice, st));
    if ((rc = launch_sub(a, b, (int64_t)(rows * n), e, st))) return rc;
    if ((rc = launch_sgemm((int)rows, (int)n, (int)n, 1.0f, e, (int64_t)n, false, hd, (int64_t)n, false, 0.0f, eh,
                           (int64_t)n, st)))
        return rc;
    if ((rc = launch_proxy_loss(e, eh, (int64_t)(rows * n), od, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(out, od, sizeof(double), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_rtn_layer(const float* w, size_t d_out, size_t n, const cdclq_config* cfg, float* out) {
    if (!w || !cfg || !out) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    float *wd = nullptr, *od = nullptr;
    if ((rc = ar.alloc(&wd, d_out * n)) || (rc = ar.alloc(&od, d_out * n))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(wd, w, d_out * n * sizeof(float), cudaMemcpyHostToDevice, st));
    if ((rc = launch_rtn(wd, (int)d_out, (int)n, (int)effective_group(*cfg, n), (int)cfg->bits, cfg->mse_grid ? 1 : 0,
                         od, st)))
        return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(out, od, d_out * n * sizeof(float), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_find_params(const float* vals, size_t rows, size_t len, uint32_t bits, int mse, float* scales, float* zeros) {
    if (!vals || !scales || !zeros) return set_error(CDCLQ_ERR_ARG, "null argument");
    if (bits < 2 || bits > 8) return set_error(CDCLQ_ERR_CONFIG, "bits and skeleton_bits must be in 2..=8");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    float *vd = nullptr, *sd = nullptr, *zd = nullptr;
    if ((rc = ar.alloc(&vd, rows * len)) || (rc = ar.alloc(&sd, rows)) || (rc = ar.alloc(&zd, rows))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(vd, vals, rows * len * sizeof(float), cudaMemcpyHostToDevice, st));
    if ((rc = launch_find_params(vd, (int)rows, (int)len, (int)bits, mse, sd, zd, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(scales, sd, rows * sizeof(float), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(zeros, zd, rows * sizeof(float), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

size_t cdclq_row_bytes(size_t n, size_t g, const uint8_t* gbits) {
    if (!gbits || g == 0) return 0;
    size_t bits = 0;
    for (size_t j = 0; j < n; j++) bits += gbits[j / g];
    return (bits + 7) / 8;
}

static std::vector<uint32_t> bit_offsets(size_t n, size_t g, const uint8_t* gbits) {
    std::vector<uint32_t> off(n + 1);
    uint32_t acc = 0;
    for (size_t j = 0; j < n; j++) {
        off[j] = acc;
        acc += gbits[j / g];
    }
    off[n] = acc;
    return off;
}

int cdclq_pack(const uint8_t* codes, size_t d_out, size_t n, size_t g, const uint8_t* gbits, uint8_t* out) {
    if (!codes || !gbits || !out || g == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    size_t ng = (n + g - 1) / g, rb = cdclq_row_bytes(n, g, gbits);
    std::vector<uint32_t> off = bit_offsets(n, g, gbits);
    uint8_t *cd = nullptr, *gd = nullptr, *od = nullptr;
    uint32_t* offd = nullptr;
    if ((rc = ar.alloc(&cd, d_out * n)) || (rc = ar.alloc(&gd, ng)) || (rc = ar.alloc(&od, d_out * rb)) ||
        (rc = ar.alloc(&offd, n + 1)))
        return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(cd, codes, d_out * n, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(gd, gbits, ng, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(offd, off.data(), (n + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    if ((rc = launch_pack(cd, (int)d_out, (int)n, (int)g, gd, offd, (int)rb, od, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(out, od, d_out * rb, cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

int cdclq_pack_device(const uint8_t* codes, size_t d_out, size_t n, size_t g, const uint8_t* gbits, uint8_t* out,
                      void* stream) {
    if (!codes || !gbits || !out || g == 0) return set_error(CDCLQ_ERR_ARG, "null argument");
    cudaStream_t st = (cudaStream_t)stream;
    Arena ar(st);
    size_t ng = (n + g - 1) / g, rb = cdclq_row_bytes(n, g, gbits);
    std::vector<uint32_t> off = bit_offsets(n, g, gbits);
    uint8_t* gd = nullptr;
    uint32_t* offd = nullptr;
    int rc = 0;
    if ((rc = ar.alloc(&gd, ng)) || (rc = ar.alloc(&offd, n + 1))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(gd, gbits, ng, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(offd, off.data(), (n + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    if ((rc = launch_pack(codes, (int)d_out, (int)n, (int)g, gd, offd, (int)rb, out, st))) return rc;
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));  // the staged offsets outlive the kernel
    return CDCLQ_OK;
}

int cdclq_unpack_dequant(const uint8_t* packed, size_t d_out, size_t n, size_t g, const uint8_t* gbits,
                         const uint32_t* perm, const float* scales, const float* zeros, float* out) {
    if (!packed || !gbits || !perm || !scales || !zeros || !out || g == 0)
        return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    cudaStream_t st = lib_stream();
    Arena ar(st);
    size_t ng = (n + g - 1) / g, rb = cdclq_row_bytes(n, g, gbits);
    std::vector<uint32_t> off = bit_offsets(n, g, gbits);
    uint8_t *pd = nullptr, *gd = nullptr;
    uint32_t *offd = nullptr, *permd = nullptr;
    float *sd = nullptr, *zd = nullptr, *od = nullptr;
    if ((rc = ar.alloc(&pd, d_out * rb)) || (rc = ar.alloc(&gd, ng)) || (rc = ar.alloc(&offd, n + 1)) ||
        (rc = ar.alloc(&permd, n)) || (rc = ar.alloc(&sd, d_out * ng)) || (rc = ar.alloc(&zd, d_out * ng)) ||
        (rc = ar.alloc(&od, d_out * n)))
        return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(pd, packed, d_out * rb, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(gd, gbits, ng, cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(offd, off.data(), (n + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(permd, perm, n * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(sd, scales, d_out * ng * sizeof(float), cudaMemcpyHostToDevice, st));
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(zd, zeros, d_out * ng * sizeof(float), cudaMemcpyHostToDevice, st));
    if ((rc = launch_unpack_dequant(pd, (int)d_out, (int)n, (int)g, gd, offd, (int)rb, permd, sd, zd, od, st))) return rc;
    CDCLQ_CUDA_TRY(cudaMemcpyAsync(out, od, d_out * n * sizeof(float), cudaMemcpyDeviceToHost, st));
    CDCLQ_CUDA_TRY(cudaStreamSynchronize(st));
    return CDCLQ_OK;
}

}  // extern "C"
