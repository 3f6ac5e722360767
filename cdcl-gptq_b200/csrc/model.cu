// model.cu - the model-level pipeline of the C ABI: safetensors shards in, packed and dequantized safetensors and
// report.json out (the reference's pipeline::quantize_model and pipeline::dequantize_packed, src/pipeline.rs).
//
// Per weight shard the reference walks its eligible layers one by one (src/pipeline.rs:121-175).  Here all
// eligible layers of a shard go through one batched quantization (every layer's rows in flight at once, one
// factorisation per distinct Hessian owner - what the reference's owner-sorted job order achieves with its
// single-entry PrepCache), over the runtime's GPUs when it has several; the outputs are then built on the
// device (dequantized values in the checkpoint's dtype, bit-packed codes, f16 scales, u8 zero points) and written
// by rank 0.  Policy, names, metadata and error messages follow the reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <sys/stat.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "cdclq.h"
#include "common.cuh"
#include "kernels.h"
#include "model_io.h"
#include "runtime.h"

namespace cdclq {

// ---- device kernels ------------------------------------------------------------------------------------
// QLayer::dequantize (src/quant.rs:189-200): row[perm[j]] = s * (code - z), original column order, f32.
__global__ void dequant_codes_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                     const float* __restrict__ zeros, const uint32_t* __restrict__ perm, int n, int g,
                                     int ng, float* __restrict__ out) {
    const int64_t r = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const int gi = j / g;
    const float s = scales[r * ng + gi], z = zeros[r * ng + gi];
    out[r * n + perm[j]] = __fmul_rn(s, __fsub_rn((float)codes[r * n + j], z));
}

// f32_to_bytes (src/io.rs:50-57): round once, to nearest even, from the exact f32 value.
__global__ void narrow_kernel(const float* __restrict__ x, int64_t count, int dtype, void* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        if (dtype == CDCLQ_DTYPE_F16) ((__half*)out)[i] = __float2half_rn(x[i]);
        else ((__nv_bfloat16*)out)[i] = __float2bfloat16_rn(x[i]);
    }
}

namespace {

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

int dtype_code(const std::string& d) {
    if (d == "F32") return CDCLQ_DTYPE_F32;
    if (d == "F16") return CDCLQ_DTYPE_F16;
    if (d == "BF16") return CDCLQ_DTYPE_BF16;
    return -1;
}

// dtype_from_name (src/io.rs:70-78)
std::string dtype_from_name(const std::string& s) {
    std::string u;
    for (char c : s) u += (char)toupper((unsigned char)c);
    if (u == "F32" || u == "FLOAT32") return "F32";
    if (u == "F16" || u == "FLOAT16" || u == "HALF") return "F16";
    if (u == "BF16" || u == "BFLOAT16") return "BF16";
    return "";
}

// Device f32 (count values) -> little-endian bytes of `dtype` on the host.
int to_dtype_bytes(const float* x_dev, size_t count, const std::string& dtype, std::vector<uint8_t>& out,
                   cudaStream_t st) {
    const int code = dtype_code(dtype);
    if (code < 0) return set_error(CDCLQ_ERR_ARG, "unsupported output dtype " + dtype);
    out.resize(count * (code == CDCLQ_DTYPE_F32 ? 4 : 2));
    if (count == 0) return 0;
    if (code == CDCLQ_DTYPE_F32) {
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(out.data(), x_dev, count * 4, cudaMemcpyDeviceToHost, st));
        return 0;
    }
    void* tmp = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync(&tmp, count * 2, st));
    const int grid = (int)std::min<int64_t>(((int64_t)count + 255) / 256, 148 * 16);
    CDCLQ_LAUNCH(narrow_kernel, grid, 256, 0, st, x_dev, (int64_t)count, code, tmp);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(out.data(), tmp, count * 2, cudaMemcpyDeviceToHost, st);
    cudaFreeAsync(tmp, st);
    return e == cudaSuccess ? 0 : cuda_error(e, "narrow_kernel");
}

bool contains_any(const std::string& s, const std::vector<std::string>& subs) {
    for (auto& x : subs)
        if (s.find(x) != std::string::npos) return true;
    return false;
}

std::string basename_of(const std::string& p) {
    size_t k = p.rfind('/');
    return k == std::string::npos ? p : p.substr(k + 1);
}

// Shortest decimal form that reads back as v.
std::string shortest(double v) {
    char b[40];
    for (int p = 1; p <= 17; p++) {
        snprintf(b, sizeof b, "%.*e", p - 1, v);
        if (strtod(b, nullptr) == v) break;
    }
    return b;  // d.ddde[+-]XX
}

// An f64 as serde_json prints it (ryu, shortest round-trip; integral values keep ".0"); null when not finite.
std::string json_f64(double v) {
    if (!std::isfinite(v)) return "null";
    if (v == 0.0) return std::signbit(v) ? "-0.0" : "0.0";
    std::string s = shortest(v);
    size_t e = s.find('e');
    std::string mant = s.substr(0, e);
    int exp = atoi(s.c_str() + e + 1);
    bool neg = mant[0] == '-';
    if (neg) mant = mant.substr(1);
    std::string digits;
    for (char c : mant)
        if (c != '.') digits += c;
    while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
    std::string o;
    const int nd = (int)digits.size();
    if (exp >= -5 && exp < 16) {
        if (exp >= 0) {
            if (nd <= exp + 1) o = digits + std::string(exp + 1 - nd, '0') + ".0";
            else o = digits.substr(0, exp + 1) + "." + digits.substr(exp + 1);
        } else {
            o = "0." + std::string(-exp - 1, '0') + digits;
        }
    } else {
        o = digits.substr(0, 1) + (nd > 1 ? "." + digits.substr(1) : "") + "e" + std::to_string(exp);
    }
    return (neg ? "-" : "") + o;
}

// Rust's `{:?}` of an f64 (the Debug form of Config's fields): fixed notation between 1e-5 and 1e16, with ".0"
// when integral; scientific ("1e-6") outside.
std::string rust_f64(double v) {
    std::string s = json_f64(v);
    return s == "null" ? (std::isnan(v) ? "NaN" : (v > 0 ? "inf" : "-inf")) : s;
}

// format!("{:?}", cfg): the report's self-description of the run (src/pipeline.rs:215).
std::string config_debug(const cdclq_config& c) {
    return "Config { bits: " + std::to_string(c.bits) + ", group: " + std::to_string(c.group) + ", block: " +
           std::to_string(c.block) + ", damp: " + rust_f64(c.damp) + ", act_order: " + (c.act_order ? "true" : "false") +
           ", skeleton_pct: " + rust_f64(c.skeleton_pct) + ", skeleton_bits: " + std::to_string(c.skeleton_bits) +
           ", mse_grid: " + (c.mse_grid ? "true" : "false") + ", method: " +
           (c.method == CDCLQ_METHOD_GPTQ ? "Gptq" : "Cdcl") + ", refine_frac: " + rust_f64(c.refine_frac) +
           ", sub_block: " + std::to_string(c.sub_block) + ", cd_sweeps: " + std::to_string(c.cd_sweeps) +
           ", passes: " + std::to_string(c.passes) + ", tol: " + rust_f64(c.tol) + ", refit_scales: " +
           (c.refit_scales ? "true" : "false") + ", row_chunk: " + std::to_string(c.row_chunk) + " }";
}

// Rust's `{:.4e}`: one digit, '.', four digits, 'e', the exponent without '+' or leading zeros.
std::string rust_e4(double v) {
    char b[40];
    snprintf(b, sizeof b, "%.4e", v);
    std::string s = b;
    size_t e = s.find('e');
    if (e == std::string::npos) return s;
    return s.substr(0, e + 1) + std::to_string(atoi(s.c_str() + e + 1));
}

struct LayerReport {
    std::string name;
    size_t d_out, d_in;
    cdclq_layer_stats s;
    double gain;
};

struct Job {
    std::string name, layer, owner;
    const io::TensorView* w;
    size_t d_out, d_in;
};

// Little-endian bytes of plain values.
template <class T>
std::vector<uint8_t> le_bytes(const T* v, size_t n) {
    std::vector<uint8_t> b(n * sizeof(T));
    std::memcpy(b.data(), v, b.size());  // x86-64 and the GPU are little-endian
    return b;
}

int write_report(const std::string& out_dir, const cdclq_config& cfg, const std::vector<LayerReport>& L,
                 double tg, double tf, double gain, double secs) {
    std::string j = "{\n  \"config\": " + io::json_quote(config_debug(cfg)) + ",\n  \"layers\": [";
    for (size_t k = 0; k < L.size(); k++) {
        const LayerReport& r = L[k];
        j += (k ? ",\n" : "\n");
        j += "    {\n      \"name\": " + io::json_quote(r.name) + ",\n      \"d_out\": " + std::to_string(r.d_out) +
             ",\n      \"d_in\": " + std::to_string(r.d_in) + ",\n      \"loss_gptq\": " + json_f64(r.s.loss_gptq) +
             ",\n      \"loss_final\": " + json_f64(r.s.loss_final) + ",\n      \"gain_pct\": " + json_f64(r.gain) +
             ",\n      \"subblocks_refined\": " + std::to_string(r.s.subblocks_refined) +
             ",\n      \"subblocks_total\": " + std::to_string(r.s.subblocks_total) +
             ",\n      \"code_updates\": " + std::to_string(r.s.code_updates) +
             ",\n      \"skeleton_groups\": " + std::to_string(r.s.skeleton_groups) +
             ",\n      \"bits_codes\": " + json_f64(r.s.bits_codes) + ",\n      \"bits_total\": " +
             json_f64(r.s.bits_total) + ",\n      \"secs_prepare\": " + json_f64(r.s.secs_prepare) +
             ",\n      \"secs_quant\": " + json_f64(r.s.secs_quant) + "\n    }";
    }
    j += (L.empty() ? "],\n" : "\n  ],\n");
    j += "  \"total_loss_gptq\": " + json_f64(tg) + ",\n  \"total_loss_final\": " + json_f64(tf) +
         ",\n  \"total_gain_pct\": " + json_f64(gain) + ",\n  \"total_secs\": " + json_f64(secs) + "\n}";
    std::string path = out_dir + "/report.json";
    std::string dir = out_dir;
    {  // create_dir_all(out_dir)
        std::string cur;
        size_t p = 0;
        while (p != std::string::npos) {
            p = dir.find('/', p + 1);
            cur = dir.substr(0, p);
            if (!cur.empty()) mkdir(cur.c_str(), 0755);
        }
    }
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return set_error(CDCLQ_ERR_ARG, "cannot write " + path);
    bool ok = fwrite(j.data(), 1, j.size(), f) == j.size();
    if (fclose(f) != 0 || !ok) return set_error(CDCLQ_ERR_ARG, "writing " + path + " failed");
    return 0;
}

// Upload a tensor's raw bytes and widen them to f32 on the device (tensor_to_f32, src/io.rs:37-45).
int upload_f32(const io::TensorView* t, size_t elem0, size_t count, float* dst, cudaStream_t st) {
    const int code = dtype_code(t->dtype);
    const size_t es = io::dtype_size(t->dtype);
    if (count == 0) return 0;
    if (code == CDCLQ_DTYPE_F32) {
        CDCLQ_CUDA_TRY(cudaMemcpyAsync(dst, t->data + elem0 * 4, count * 4, cudaMemcpyHostToDevice, st));
        return 0;
    }
    void* raw = nullptr;
    CDCLQ_CUDA_TRY(cudaMallocAsync(&raw, count * es, st));
    cudaError_t e = cudaMemcpyAsync(raw, t->data + elem0 * es, count * es, cudaMemcpyHostToDevice, st);
    int rc = e == cudaSuccess ? cdclq_widen_to_f32_device(raw, code, count, dst, st) : cuda_error(e, "upload");
    cudaFreeAsync(raw, st);
    return rc;
}

}  // namespace

// One shard's layers through the runtime, outputs written by rank 0.
static int quantize_shard(Runtime* rt, const cdclq_model_opts& o, const io::HessianStore& store,
                          const std::string& shard, std::vector<LayerReport>& reports) {
    cudaStream_t st = rt->st;
    io::SafeTensorsFile f;
    int rc = rt_agree(rt, f.open(shard));
    if (rc) return rc;
    std::vector<std::string> only, skip;
    for (size_t k = 0; k < o.n_only; k++) only.push_back(o.only[k]);
    for (size_t k = 0; k < o.n_skip; k++) skip.push_back(o.skip[k]);
    const std::vector<std::string> names = f.names();

    // jobs: 2-D `.weight` tensors with a Hessian, sorted by owner then layer (src/pipeline.rs:92-112)
    std::vector<Job> jobs;
    for (auto& name : names) {
        if (name.size() < 7 || name.compare(name.size() - 7, 7, ".weight") != 0) continue;
        const std::string layer = name.substr(0, name.size() - 7);
        const io::TensorView* t = f.tensor(name);
        if (t->shape.size() != 2) continue;
        if (!only.empty() && !contains_any(layer, only)) continue;
        if (contains_any(layer, skip)) continue;
        std::string owner = store.resolve(layer);
        if (owner.empty()) continue;
        jobs.push_back(Job{name, layer, owner, t, t->shape[0], t->shape[1]});
    }
    std::stable_sort(jobs.begin(), jobs.end(), [](const Job& a, const Job& b) {
        return a.owner != b.owner ? a.owner < b.owner : a.layer < b.layer;
    });

    // per job, in order: the weight's dtype, the Hessian (present, square, f32/f16/bf16), the width check
    // (src/pipeline.rs:122-127), the optional M (src/io.rs:222-224)
    std::map<std::string, size_t> owner_index;
    std::vector<const io::TensorView*> hview, mview;
    std::vector<size_t> hn;
    std::vector<size_t> job_input(jobs.size());
    for (size_t k = 0; k < jobs.size() && !rc; k++) {
        const Job& J = jobs[k];
        if (dtype_code(J.w->dtype) < 0) {
            rc = set_error(CDCLQ_ERR_ARG, "unsupported weight dtype " + J.w->dtype + " (need F32/F16/BF16)");
            break;
        }
        auto it = owner_index.find(J.owner);
        if (it == owner_index.end()) {
            bool missing = false;
            size_t n = 0;
            const io::TensorView* h = store.tensor(J.owner, "H", &n, &missing);
            if (!h) {
                rc = missing ? set_error(CDCLQ_ERR_ARG, "missing " + J.owner + ".H") : CDCLQ_ERR_ARG;
                break;
            }
            const io::TensorView* m = store.tensor(J.owner, "M", &n, &missing);
            if (!m && !missing) {
                rc = CDCLQ_ERR_ARG;
                break;
            }
            n = h->shape[0];
            it = owner_index.emplace(J.owner, hview.size()).first;
            hview.push_back(h);
            mview.push_back(m);
            hn.push_back(n);
        }
        job_input[k] = it->second;
        if (hn[it->second] != J.d_in) {
            const std::string s = std::to_string(hn[it->second]);
            rc = set_error(CDCLQ_ERR_ARG, J.layer + ": Hessian is " + s + "x" + s + " but the weight has " +
                                              std::to_string(J.d_in) + " input columns");
            break;
        }
        if (mview[it->second] && mview[it->second]->shape[0] != J.d_in) {
            rc = set_error(CDCLQ_ERR_ARG, J.owner + ".M: expected " + std::to_string(J.d_in) + " x " +
                                              std::to_string(J.d_in));
            break;
        }
    }
    if ((rc = rt_agree(rt, rc))) return rc;
    const size_t nin = hview.size();
    const int R = rt->nranks, me = rt->rank;

    // Hessians on the device: each uploaded, widened and scanned by its owner rank (src/io.rs:204-211), then
    // broadcast over NVLink
    std::vector<size_t> nsz(nin);
    for (size_t i = 0; i < nin; i++) nsz[i] = hn[i];
    const std::vector<int> owner = assign_owners(nsz, R, 3);
    std::vector<float*> hdev(nin, nullptr), mdev(nin, nullptr);
    struct Free {
        std::vector<void*> p;
        cudaStream_t st;
        ~Free() {
            for (void* q : p) cudaFreeAsync(q, st);
            cudaStreamSynchronize(st);
        }
    } fr{{}, st};
    auto dalloc = [&](void** p, size_t bytes) -> int {
        cudaError_t e = cudaMallocAsync(p, std::max<size_t>(bytes, 1), st);
        if (e != cudaSuccess) return cuda_error(e, "cudaMallocAsync");
        fr.p.push_back(*p);
        return 0;
    };
    std::vector<std::string> owner_name(nin);
    for (auto& kv : owner_index) owner_name[kv.second] = kv.first;
    for (size_t i = 0; i < nin && !rc; i++) {
        const size_t n = hn[i];
        rc = dalloc((void**)&hdev[i], n * n * 4);
        if (!rc && mview[i]) rc = dalloc((void**)&mdev[i], n * n * 4);
        if (rc || owner[i] != me) continue;
        rc = upload_f32(hview[i], 0, n * n, hdev[i], st);
        if (!rc) rc = cdclq_check_matrix_device(hdev[i], n, (owner_name[i] + ".H").c_str(), st);
        if (!rc && mview[i]) {
            rc = upload_f32(mview[i], 0, n * n, mdev[i], st);
            if (!rc) rc = cdclq_check_matrix_device(mdev[i], n, (owner_name[i] + ".M").c_str(), st);
        }
    }
    if ((rc = rt_agree(rt, rc))) return rc;
    if (R > 1) {
        if ((rc = rt_group_begin(rt))) return rc;
        for (size_t i = 0; i < nin && !rc; i++) {
            rc = rt_broadcast(rt, hdev[i], hn[i] * hn[i] * 4, owner[i]);
            if (!rc && mdev[i]) rc = rt_broadcast(rt, mdev[i], hn[i] * hn[i] * 4, owner[i]);
        }
        int r2 = rt_group_end(rt);
        if (rc || r2) return rc ? rc : r2;
    }

    // weights: full-size f32 buffers, each rank fills its own rows (the runtime quantizes exactly those)
    const cdclq_config& cfg = o.cfg;
    std::vector<size_t> batch_jobs, m_jobs;
    for (size_t k = 0; k < jobs.size(); k++) (mdev[job_input[k]] ? m_jobs : batch_jobs).push_back(k);
    const size_t nb = batch_jobs.size();
    std::vector<float*> wdev(jobs.size(), nullptr);
    std::vector<uint8_t*> codes(jobs.size(), nullptr);
    std::vector<float*> scales(jobs.size(), nullptr), zeros(jobs.size(), nullptr);
    std::vector<size_t> ngs(jobs.size());
    std::vector<std::vector<uint32_t>> perm(jobs.size());
    std::vector<std::vector<uint8_t>> gbits(jobs.size());
    std::vector<cdclq_layer_stats> stats(jobs.size());
    for (size_t k = 0; k < jobs.size() && !rc; k++) {
        const Job& J = jobs[k];
        ngs[k] = cdclq_num_groups(&cfg, J.d_in);
        perm[k].resize(J.d_in);
        gbits[k].resize(ngs[k]);
        if ((rc = dalloc((void**)&wdev[k], J.d_out * J.d_in * 4))) break;
        if ((rc = dalloc((void**)&codes[k], J.d_out * J.d_in))) break;
        if ((rc = dalloc((void**)&scales[k], J.d_out * ngs[k] * 4))) break;
        if ((rc = dalloc((void**)&zeros[k], J.d_out * ngs[k] * 4))) break;
    }
    for (size_t b = 0; b < nb && !rc; b++) {
        const size_t k = batch_jobs[b];
        const Job& J = jobs[k];
        size_t r0 = 0, r1 = J.d_out;
        if (R > 1) shard_rows(J.d_out, cdclq_row_chunk(&cfg, J.d_out), me, R, b, &r0, &r1);
        rc = upload_f32(J.w, r0 * J.d_in, (r1 - r0) * J.d_in, wdev[k] + r0 * J.d_in, st);
    }
    for (size_t k : m_jobs)
        if (!rc) rc = upload_f32(jobs[k].w, 0, jobs[k].d_out * jobs[k].d_in, wdev[k], st);
    if ((rc = rt_agree(rt, rc))) return rc;

    // quantize: the batch over the ranks (gathered on rank 0); layers with an asymmetric target one by one
    if (nb) {
        std::vector<cdclq_batch_input> ins(nin);
        for (size_t i = 0; i < nin; i++) ins[i] = cdclq_batch_input{hdev[i], hn[i]};
        std::vector<cdclq_batch_layer> lys(nb);
        for (size_t b = 0; b < nb; b++) {
            const size_t k = batch_jobs[b];
            lys[b] = cdclq_batch_layer{};
            lys[b].w = wdev[k];
            lys[b].d_out = jobs[k].d_out;
            lys[b].input = job_input[k];
            lys[b].perm = perm[k].data();
            lys[b].gbits = gbits[k].data();
            lys[b].codes = codes[k];
            lys[b].scales = scales[k];
            lys[b].zeros = zeros[k];
            lys[b].stats = &stats[k];
        }
        rc = runtime_quantize_batch(rt, ins.data(), nin, lys.data(), nb, cfg, true, true);
        if (rc) return rc;  // already agreed inside
    }
    for (size_t k : m_jobs) {  // every rank runs these (one GPU each), so every rank holds the same statistics
        const Job& J = jobs[k];
        const size_t n = J.d_in, i = job_input[k];
        std::vector<float> w(J.d_out * n), h(n * n), m(n * n);
        std::vector<uint8_t> c(J.d_out * n);
        std::vector<float> s(J.d_out * ngs[k]), z(J.d_out * ngs[k]);
        cudaError_t e = cudaMemcpyAsync(w.data(), wdev[k], w.size() * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(h.data(), hdev[i], h.size() * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(m.data(), mdev[i], m.size() * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        rc = e == cudaSuccess ? 0 : cuda_error(e, "asymmetric layer read-back");
        if (!rc)
            rc = cdclq_quantize_layer(w.data(), J.d_out, n, h.data(), m.data(), J.owner.c_str(), &cfg, nullptr,
                                      perm[k].data(), gbits[k].data(), c.data(), s.data(), z.data(), &stats[k]);
        if (!rc) {
            e = cudaMemcpyAsync(codes[k], c.data(), c.size(), cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = cudaMemcpyAsync(scales[k], s.data(), s.size() * 4, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = cudaMemcpyAsync(zeros[k], z.data(), z.size() * 4, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            if (e != cudaSuccess) rc = cuda_error(e, "asymmetric layer upload");
        }
        if (rc) break;
    }
    if ((rc = rt_agree(rt, rc))) return rc;

    // per-layer records and progress lines (src/pipeline.rs:131-161)
    for (size_t k = 0; k < jobs.size(); k++) {
        const Job& J = jobs[k];
        const cdclq_layer_stats& s = stats[k];
        const double gain = s.loss_gptq > 0.0 ? 100.0 * (s.loss_gptq - s.loss_final) / s.loss_gptq : 0.0;
        reports.push_back(LayerReport{J.layer, J.d_out, J.d_in, s, gain});
        if (o.verbose && me == 0) {
            char pct[32], bpw[32], sp[32], sq[32];
            snprintf(pct, sizeof pct, "%+.1f", -gain);
            snprintf(bpw, sizeof bpw, "%.2f", s.bits_total);
            snprintf(sp, sizeof sp, "%.1f", s.secs_prepare);
            snprintf(sq, sizeof sq, "%.1f", s.secs_quant);
            fprintf(stderr, "[%3zu/%-3zu] %s [%zux%zu] loss %s -> %s (%s%%) | %s bpw | prep %ss quant %ss\n", k + 1,
                    jobs.size(), J.layer.c_str(), J.d_out, J.d_in, rust_e4(s.loss_gptq).c_str(),
                    rust_e4(s.loss_final).c_str(), pct, bpw, sp, sq);
        }
    }
    if (me != 0) return 0;

    // outputs (rank 0): dequantized tensors in the checkpoint's dtype, packed tensors, pass-through
    std::vector<io::OutTensor> deq, pk;
    std::set<std::string> done;
    std::string orig_dtype;
    for (size_t k = 0; k < jobs.size() && !rc; k++) {
        const Job& J = jobs[k];
        const size_t n = J.d_in, ng = ngs[k], g = cdclq_effective_group(&cfg, n);
        if (orig_dtype.empty()) orig_dtype = J.w->dtype;
        if (o.emit_dequant) {
            float* fd = nullptr;
            uint32_t* pd = nullptr;
            if ((rc = dalloc((void**)&fd, J.d_out * n * 4)) || (rc = dalloc((void**)&pd, n * 4))) break;
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(pd, perm[k].data(), n * 4, cudaMemcpyHostToDevice, st));
            dim3 grid((unsigned)((n + 255) / 256), (unsigned)J.d_out);
            for (size_t r0 = 0; r0 < J.d_out; r0 += 65535) {
                const size_t rows = std::min<size_t>(65535, J.d_out - r0);
                grid.y = (unsigned)rows;
                CDCLQ_LAUNCH(dequant_codes_kernel, grid, 256, 0, st, codes[k] + r0 * n, scales[k] + r0 * ng,
                             zeros[k] + r0 * ng, pd, (int)n, (int)g, (int)ng, fd + r0 * n);
            }
            CDCLQ_CUDA_TRY(cudaGetLastError());
            io::OutTensor t{J.name, J.w->dtype, {J.d_out, n}, {}};
            if ((rc = to_dtype_bytes(fd, J.d_out * n, J.w->dtype, t.bytes, st))) break;
            deq.push_back(std::move(t));
        }
        if (o.emit_packed) {
            // packed_tensors (src/io.rs:244-270)
            const size_t rb = cdclq_row_bytes(n, g, gbits[k].data());
            uint8_t *qw = nullptr, *qz = nullptr;
            uint16_t* s16 = nullptr;
            if ((rc = dalloc((void**)&qw, J.d_out * rb)) || (rc = dalloc((void**)&qz, J.d_out * ng)) ||
                (rc = dalloc((void**)&s16, J.d_out * ng * 2)))
                break;
            if ((rc = cdclq_pack_device(codes[k], J.d_out, n, g, gbits[k].data(), qw, st))) break;
            if ((rc = cdclq_encode_groups_device(scales[k], zeros[k], J.d_out * ng, s16, qz, st))) break;
            io::OutTensor tq{J.layer + ".qweight", "U8", {J.d_out, rb}, std::vector<uint8_t>(J.d_out * rb)};
            io::OutTensor ts{J.layer + ".scales", "F16", {J.d_out, ng}, std::vector<uint8_t>(J.d_out * ng * 2)};
            io::OutTensor tz{J.layer + ".qzeros", "U8", {J.d_out, ng}, std::vector<uint8_t>(J.d_out * ng)};
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(tq.bytes.data(), qw, tq.bytes.size(), cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(ts.bytes.data(), s16, ts.bytes.size(), cudaMemcpyDeviceToHost, st));
            CDCLQ_CUDA_TRY(cudaMemcpyAsync(tz.bytes.data(), qz, tz.bytes.size(), cudaMemcpyDeviceToHost, st));
            std::vector<int32_t> p32(perm[k].begin(), perm[k].end());
            const int32_t gs = (int32_t)g;
            pk.push_back(std::move(tq));
            pk.push_back(std::move(ts));
            pk.push_back(std::move(tz));
            pk.push_back(io::OutTensor{J.layer + ".perm", "I32", {n}, le_bytes(p32.data(), n)});
            pk.push_back(io::OutTensor{J.layer + ".gbits", "U8", {ng}, gbits[k]});
            pk.push_back(io::OutTensor{J.layer + ".gsize", "I32", {1}, le_bytes(&gs, 1)});
        }
        done.insert(J.name);
    }
    if (!rc) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_error(e, "output build");
    }
    if (rc) return rc;
    // pass-through (src/pipeline.rs:180-192)
    for (auto& name : names) {
        if (done.count(name)) continue;
        const io::TensorView* t = f.tensor(name);
        io::OutTensor x{name, t->dtype, t->shape, std::vector<uint8_t>(t->data, t->data + t->nbytes)};
        if (o.emit_dequant) deq.push_back(x);
        if (o.emit_packed) pk.push_back(std::move(x));
    }
    const std::string fname = basename_of(shard);
    std::map<std::string, std::string> meta{{"format", "pt"}};
    if (o.emit_dequant && !deq.empty())
        if ((rc = io::write_tensors(std::string(o.out_dir) + "/dequant/" + fname, deq, meta))) return rc;
    if (o.emit_packed && !pk.empty()) {
        meta["quantization"] = "cdclq-v1";
        meta["orig_dtype"] = orig_dtype.empty() ? "F16" : orig_dtype;
        meta["bits"] = std::to_string(cfg.bits);
        if ((rc = io::write_tensors(std::string(o.out_dir) + "/packed/" + fname, pk, meta))) return rc;
    }
    return 0;
}

}  // namespace cdclq

using namespace cdclq;

extern "C" int cdclq_quantize_model(cdclq_runtime* rt_in, const cdclq_model_opts* o, cdclq_model_report* rep) {
    if (!o || !o->out_dir || (!o->weights && o->n_weights) || (!o->hessians && o->n_hessians) ||
        (!o->only && o->n_only) || (!o->skip && o->n_skip))
        return set_error(CDCLQ_ERR_ARG, "null argument");
    if (!o->emit_packed && !o->emit_dequant)
        return set_error(CDCLQ_ERR_ARG, "nothing to write: both --no-packed and --no-dequant are set");
    const double t_all = now_s();
    cdclq_runtime* local = nullptr;
    Runtime* rt = (Runtime*)rt_in;
    if (!rt) {
        int dev = 0;
        cudaGetDevice(&dev);
        int rc = cdclq_runtime_create(dev, 1, 0, nullptr, 0.0, &local);
        if (rc) return rc;
        rt = (Runtime*)local;
    } else {
        cudaError_t e = cudaSetDevice(rt->device);
        if (e != cudaSuccess) return cuda_error(e, "cudaSetDevice");
    }
    int rc = 0;
    std::vector<std::string> hp;
    for (size_t k = 0; k < o->n_hessians; k++) hp.push_back(o->hessians[k]);
    io::HessianStore store;
    rc = rt_agree(rt, store.open(hp));
    std::vector<LayerReport> reports;
    for (size_t k = 0; k < o->n_weights && !rc; k++) rc = quantize_shard(rt, *o, store, o->weights[k], reports);
    if (!rc) {
        double tg = 0.0, tf = 0.0;
        for (auto& r : reports) {
            tg += r.s.loss_gptq;
            tf += r.s.loss_final;
        }
        const double gain = tg > 0.0 ? 100.0 * (tg - tf) / tg : 0.0;
        const double secs = now_s() - t_all;
        if (rt->rank == 0) rc = write_report(o->out_dir, o->cfg, reports, tg, tf, gain, secs);
        rc = rt_agree(rt, rc);
        if (!rc && rep) {
            rep->layers = reports.size();
            rep->total_loss_gptq = tg;
            rep->total_loss_final = tf;
            rep->total_gain_pct = gain;
            rep->total_secs = secs;
        }
    }
    if (local) {
        std::string keep = rc ? cdclq_last_error() : "";
        cdclq_runtime_destroy(local);
        if (rc) set_error(rc, keep);
    }
    return rc;
}

extern "C" int cdclq_dequantize_packed(const char* input, const char* output, const char* dtype, uint64_t* layers_out) {
    if (!input || !output) return set_error(CDCLQ_ERR_ARG, "null argument");
    int rc = ensure_device();
    if (rc) return rc;
    io::SafeTensorsFile f;
    if ((rc = f.open(input))) return rc;
    std::string dt;
    if (dtype) {
        dt = dtype_from_name(dtype);
        if (dt.empty()) return set_error(CDCLQ_ERR_ARG, std::string("unknown dtype ") + dtype);
    } else {
        auto it = f.metadata().find("orig_dtype");
        if (it != f.metadata().end()) dt = dtype_from_name(it->second);
        if (dt.empty()) dt = "F16";
    }
    const std::vector<std::string> names = f.names();
    std::vector<std::string> layers;
    for (auto& n : names)
        if (n.size() > 8 && n.compare(n.size() - 8, 8, ".qweight") == 0) layers.push_back(n.substr(0, n.size() - 8));
    cudaStream_t st = nullptr;
    CDCLQ_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    std::vector<io::OutTensor> out;
    std::set<std::string> drop;
    for (size_t k = 0; k < layers.size() && !rc; k++) {
        const std::string& l = layers[k];
        auto get = [&](const char* suf) -> const io::TensorView* {
            const io::TensorView* t = f.tensor(l + "." + suf);
            if (!t) set_error(CDCLQ_ERR_ARG, l + "." + suf + ": tensor not found");
            return t;
        };
        const io::TensorView *qw = get("qweight"), *sc = qw ? get("scales") : nullptr, *qz = sc ? get("qzeros") : nullptr,
                             *pm = qz ? get("perm") : nullptr, *gb = pm ? get("gbits") : nullptr,
                             *gs = gb ? get("gsize") : nullptr;
        if (!gs) {
            rc = CDCLQ_ERR_ARG;
            break;
        }
        // read_packed_layer (src/io.rs:276-296)
        const size_t d_out = qw->shape[0], d_in = pm->shape[0];
        int32_t g32 = 0;
        std::memcpy(&g32, gs->data, 4);
        const size_t g = (size_t)g32, ng = gb->numel();
        if (g == 0 || sc->numel() != d_out * ng || qz->numel() != d_out * ng || pm->dtype != "I32" || sc->dtype != "F16") {
            rc = set_error(CDCLQ_ERR_ARG, l + ": inconsistent packed tensors");
            break;
        }
        std::vector<uint32_t> perm(d_in);
        for (size_t j = 0; j < d_in; j++) {
            int32_t v = 0;
            std::memcpy(&v, pm->data + 4 * j, 4);
            perm[j] = (uint32_t)v;
        }
        std::vector<float> scales(d_out * ng), zeros(d_out * ng), w(d_out * d_in);
        for (size_t i = 0; i < d_out * ng; i++) {
            __half_raw hr;
            std::memcpy(&hr.x, sc->data + 2 * i, 2);
            scales[i] = __half2float(__half(hr));
            zeros[i] = (float)qz->data[i];
        }
        if ((rc = cdclq_unpack_dequant(qw->data, d_out, d_in, g, gb->data, perm.data(), scales.data(), zeros.data(),
                                       w.data())))
            break;
        io::OutTensor t{l + ".weight", dt, {d_out, d_in}, {}};
        if (dt == "F32") {
            t.bytes = le_bytes(w.data(), w.size());
        } else {
            float* wd = nullptr;
            cudaError_t e = cudaMallocAsync((void**)&wd, w.size() * 4, st);
            if (e == cudaSuccess) e = cudaMemcpyAsync(wd, w.data(), w.size() * 4, cudaMemcpyHostToDevice, st);
            rc = e == cudaSuccess ? to_dtype_bytes(wd, w.size(), dt, t.bytes, st) : cuda_error(e, "dequant upload");
            if (wd) cudaFreeAsync(wd, st);
            if (!rc) {
                e = cudaStreamSynchronize(st);
                if (e != cudaSuccess) rc = cuda_error(e, "dequant");
            }
            if (rc) break;
        }
        out.push_back(std::move(t));
        for (const char* suf : {"qweight", "scales", "qzeros", "perm", "gbits", "gsize"}) drop.insert(l + "." + suf);
    }
    cudaStreamDestroy(st);
    if (rc) return rc;
    for (auto& n : names) {
        if (drop.count(n)) continue;
        const io::TensorView* t = f.tensor(n);
        out.push_back(io::OutTensor{n, t->dtype, t->shape, std::vector<uint8_t>(t->data, t->data + t->nbytes)});
    }
    if ((rc = io::write_tensors(output, out, {{"format", "pt"}}))) return rc;
    if (layers_out) *layers_out = layers.size();
    return CDCLQ_OK;
}
