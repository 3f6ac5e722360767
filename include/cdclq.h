/*
 * cdclq.h - C ABI of the B200 (sm_100a) CDCL-GPTQ per-layer quantization path.
 *
 * The reference (tailot/CDCL-GPTQ, a Rust crate) has no C ABI: its drop-in unit is the Rust function
 *     engine::quantize_layer(w, d_out, d_in, h, m, hkey, cfg, cache) -> Result<(QLayer, LayerStats)>
 * (src/engine.rs:690-699), built on linalg.rs (Cholesky, triangular inverse, U factor, Gram accumulation)
 * and quant.rs (grid, code).  Every entry point below replaces one of those functions; the comment on each
 * cites the reference function it stands in for.  A Rust caller binds them with an `extern "C"` block;
 * Python binds them with ctypes (cdcl-gptq_b200/cdclq/_lib.py).
 *
 * Conventions shared by all entry points
 *  - Plain pointers and sizes only.  Matrices are row-major.  Functions without a `_device` suffix take HOST
 *    pointers and do their own host<->device copies; `_device` functions take device pointers and a CUDA
 *    stream (passed as `void*`, NULL = the legacy default stream).
 *  - Return value: CDCLQ_OK (0) or a negative CDCLQ_ERR_* status.  cdclq_last_error() then returns the
 *    message of the last failure on the calling thread; configuration and factorisation messages keep the
 *    reference's wording (src/engine.rs:242-255, src/linalg.rs:216-218).
 *  - All quantized outputs are in the PERMUTED column order, exactly as `QLayer` (src/quant.rs:153-175).
 *  - Calls are synchronous from the caller's view.  The library is not re-entrant on one prep cache.
 */
#ifndef CDCLQ_H_
#define CDCLQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CDCLQ_OK 0
#define CDCLQ_ERR_CONFIG (-1)    /* engine::validate rejected the configuration (src/engine.rs:240-258) */
#define CDCLQ_ERR_NOT_PD (-2)    /* non-positive / non-finite Cholesky pivot (src/linalg.rs:215-219) */
#define CDCLQ_ERR_ARG (-3)       /* null pointer or size mismatch (the reference asserts: src/engine.rs:701-702) */
#define CDCLQ_ERR_CUDA (-4)      /* CUDA runtime failure, or no usable device */
#define CDCLQ_ERR_NONFINITE (-5) /* non-finite Hessian entry (src/io.rs:205-212) */

#define CDCLQ_METHOD_GPTQ 0 /* engine::Method::Gptq (src/engine.rs:85) */
#define CDCLQ_METHOD_CDCL 1 /* engine::Method::Cdcl (src/engine.rs:87) */

/* Mirrors engine::Config (src/engine.rs:93-144) field by field.  `threads` is the CLI's global --threads
 * (src/main.rs:22); it only matters when row_chunk == 0, where the reference derives the row chunk from the
 * worker count (src/engine.rs:768-770).  threads == 0 means "number of host CPUs", like rayon's default. */
typedef struct cdclq_config {
    uint64_t group;     /* 0 = one group per row */
    uint64_t block;     /* lazy-update block of the GPTQ pass */
    uint64_t sub_block; /* repair sub-block width */
    uint64_t cd_sweeps;
    uint64_t passes;
    uint64_t row_chunk; /* 0 = automatic */
    uint64_t threads;
    double damp;
    double skeleton_pct;
    double refine_frac;
    double tol;
    uint32_t bits;
    uint32_t skeleton_bits;
    int32_t act_order;
    int32_t mse_grid;
    int32_t method; /* CDCLQ_METHOD_* */
    int32_t refit_scales;
} cdclq_config;

/* Mirrors engine::LayerStats (src/engine.rs:173-199).  `passes_max` is an addition: the largest number of
 * repair passes any row chunk of the layer executed (the reference does not report it). */
typedef struct cdclq_layer_stats {
    double loss_gptq;
    double loss_final;
    uint64_t subblocks_total;
    uint64_t subblocks_refined;
    uint64_t code_updates;
    uint64_t skeleton_groups;
    double bits_codes;
    double bits_total;
    double secs_prepare;
    double secs_quant;
    uint64_t passes_max;
} cdclq_layer_stats;

/* Opaque single-entry memo of the prepared factors, replacing engine::PrepCache (src/engine.rs:207-223):
 * keyed by (hessian key, permutation); owns the device copies of U, the damped permuted Hessian and perm. */
typedef struct cdclq_prep_cache cdclq_prep_cache;

/* ---- configuration helpers ------------------------------------------------------------------------- */

/* Config::default (src/engine.rs:146-167). */
void cdclq_config_default(cdclq_config* cfg);
/* effective_group (src/engine.rs:227-233). */
size_t cdclq_effective_group(const cdclq_config* cfg, size_t n);
/* ceil(n / effective_group): the `ng` of src/engine.rs:705, i.e. the length of gbits and of one row of
 * scales/zeros. */
size_t cdclq_num_groups(const cdclq_config* cfg, size_t n);
/* validate (src/engine.rs:240-258).  CDCLQ_ERR_CONFIG with the reference's message on failure. */
int cdclq_validate(const cdclq_config* cfg, size_t n);
/* Message of the last failed call on this thread ("" if none). */
const char* cdclq_last_error(void);

/* ---- per-layer engine ------------------------------------------------------------------------------ */

cdclq_prep_cache* cdclq_prep_cache_new(void);
void cdclq_prep_cache_free(cdclq_prep_cache* cache);

/* engine::quantize_layer (src/engine.rs:690-799).  Host buffers:
 *   w      d_out x d_in f32, original column order
 *   h      d_in x d_in f32 calibration Hessian (any positive scale)
 *   m      optional d_in x d_in cross-covariance (NULL = symmetric calibration)
 *   hkey   Hessian identity for the prep cache (NUL-terminated; may be NULL when cache is NULL)
 *   cache  may be NULL (no reuse)
 * Outputs (caller-allocated, permuted order):
 *   perm_out d_in, gbits_out ng, codes_out d_out*d_in, scales_out / zeros_out d_out*ng, stats_out 1. */
int cdclq_quantize_layer(const float* w, size_t d_out, size_t d_in, const float* h, const float* m,
                         const char* hkey, const cdclq_config* cfg, cdclq_prep_cache* cache,
                         uint32_t* perm_out, uint8_t* gbits_out, uint8_t* codes_out, float* scales_out,
                         float* zeros_out, cdclq_layer_stats* stats_out);

/* Same as cdclq_quantize_layer, plus the number of repair passes each row chunk executed
 * (chunk_passes_out: ceil(d_out / row_chunk) entries, may be NULL). */
int cdclq_quantize_layer_ex(const float* w, size_t d_out, size_t d_in, const float* h, const float* m,
                            const char* hkey, const cdclq_config* cfg, cdclq_prep_cache* cache,
                            uint32_t* perm_out, uint8_t* gbits_out, uint8_t* codes_out, float* scales_out,
                            float* zeros_out, cdclq_layer_stats* stats_out, uint32_t* chunk_passes_out);

/* Row chunk actually used for a layer with d_out rows (src/engine.rs:768-770). */
size_t cdclq_row_chunk(const cdclq_config* cfg, size_t d_out);

/* ---- model-level batch (pipeline::quantize_model's per-layer loop, src/pipeline.rs:121-175) ----------- */

/* One distinct layer input (a Hessian owner in pipeline terms).  All layers pointing at the same
 * `input` share one factorisation when their permutations agree, like the PrepCache hits the reference gets
 * from its owner-sorted job order (src/pipeline.rs:109-112). */
typedef struct cdclq_batch_input {
    const float* h; /* n x n f32 */
    size_t n;
} cdclq_batch_input;

typedef struct cdclq_batch_layer {
    const float* w; /* d_out x n f32, original order */
    size_t d_out;
    size_t input; /* index into the inputs array */
    /* outputs (permuted order), caller-allocated */
    uint32_t* perm;   /* n */
    uint8_t* gbits;   /* ng */
    uint8_t* codes;   /* d_out * n */
    float* scales;    /* d_out * ng */
    float* zeros;     /* d_out * ng */
    cdclq_layer_stats* stats;
    /* optional input, NULL = computed from this call's rows: the skeleton's column scores (n f64, original
     * column order) over the layer's FULL weight matrix, as cdclq_column_scores_device returns them.  A caller
     * that passes only a shard of the rows (several GPUs) and configures a skeleton must supply them, or the
     * ranking of src/engine.rs:271-304 would see only its rows. */
    const double* colsq;
    /* optional input, NULL = factorised in the call: the factor U (n x n f32, device) of this layer's (input,
     * permutation) pair, as cdclq_prepare_layer_factors returns it (computed once on another rank). */
    const float* u;
} cdclq_batch_layer;

/* Quantize many layers in one batched pass: every layer's rows are in flight at once, so small layers
 * (k/v projections) no longer leave the GPU idle.  Results are identical to calling
 * cdclq_quantize_layer on each layer.  `on_device` = 0: all pointers are host pointers (copies inside);
 * 1: all are device pointers (stats stays a host pointer), `stream` is used for all work. */
int cdclq_quantize_batch(const cdclq_batch_input* inputs, size_t n_inputs, const cdclq_batch_layer* layers,
                         size_t n_layers, const cdclq_config* cfg, int on_device, void* stream);

/* Per-layer factors for weight-dependent permutations (skeleton_pct > 0; also valid without a skeleton): for
 * each k, the factor U of layers[which[k]]'s (input, permutation) pair into u_out[k] (n x n f32, device), the
 * permutation computed exactly as cdclq_quantize_batch computes it - from the descriptor's colsq when given,
 * else from its rows (w, d_out; device pointers when on_device).  Only w, d_out, input and colsq of the
 * descriptors are read.  A rank factorises its share; the factors are exchanged and handed back to
 * cdclq_quantize_batch in the descriptors' `u` field. */
int cdclq_prepare_layer_factors(const cdclq_batch_input* inputs, size_t n_inputs, const cdclq_batch_layer* layers,
                                size_t n_layers, const size_t* which, size_t n_which, const cdclq_config* cfg,
                                float* const* u_out, int on_device, void* stream);

/* The skeleton ranking's column scores (src/engine.rs:271-304, the ||W_:j||^2 of compute_perm): colsq[j] =
 * sum over rows r = 0 .. d_out-1, in order, of (f64) w[r][j] squared (f64 multiply, then add); 0 where the raw
 * H_jj == 0 (dead column).  w: d_out x n f32 original order, h: n x n f32, colsq_out: n f64; device pointers. */
int cdclq_column_scores_device(const float* w, size_t d_out, size_t n, const float* h, double* colsq_out,
                               void* stream);

/* ---- ingest and packed output on the device (src/io.rs) ------------------------------------------------- */

#define CDCLQ_DTYPE_F32 0
#define CDCLQ_DTYPE_F16 1
#define CDCLQ_DTYPE_BF16 2
/* tensor_to_f32 (src/io.rs:37-45) on the device: dst[i] = (f32) src[i] for a tensor copied raw from a safetensors
 * file (dtype CDCLQ_DTYPE_*); the widening is lossless.  Device pointers. */
int cdclq_widen_to_f32_device(const void* src, int dtype, size_t count, float* dst, void* stream);
/* first_non_finite (src/io.rs:120-122) on the device: index of the first NaN/inf of x (device), -1 if none. */
int cdclq_first_non_finite_device(const float* x, size_t count, int64_t* index_out, void* stream);
/* The load-time check of HessianStore::tensor (src/io.rs:204-211): CDCLQ_ERR_NONFINITE with the reference's
 * message ("<key>: <n> x <n> matrix has a non-finite entry (<v>) at [ <r>, <c> ]; ...") when the device matrix
 * h (n x n) holds a NaN or an infinity. */
int cdclq_check_matrix_device(const float* h, size_t n, const char* key, void* stream);
/* QLayer::pack (src/quant.rs:113-151) with device codes and output (out: d_out x row_bytes). gbits is host. */
int cdclq_pack_device(const uint8_t* codes, size_t d_out, size_t n, size_t g, const uint8_t* gbits, uint8_t* out,
                      void* stream);
/* The group encodings of packed_tensors (src/io.rs:248-251): scales as f16 bits, zero points as u8 (device). */
int cdclq_encode_groups_device(const float* scales, const float* zeros, size_t count, uint16_t* scales_f16,
                               uint8_t* qzeros, void* stream);

/* ---- multi-GPU: factorisations spread over ranks (the "compute once on the owning GPU, then broadcast"
 * option for Prepared's U, src/engine.rs:320-342; the reference itself runs on one host) ----------------- */

/* Upper factor U (H^-1 = U^T U of the damped Hessian, permuted order, src/linalg.rs:362-375) of the inputs
 * listed in `which`, written to the caller's DEVICE buffers u_out[k] (n x n f32 each).  The permutation is
 * the W-independent one (act-order or natural), so skeleton_pct must be 0.  `on_device` says where the
 * Hessians live.  A rank factorises its share, then the factors are broadcast (NCCL) to every rank. */
int cdclq_prepare_factors(const cdclq_batch_input* inputs, size_t n_inputs, const size_t* which, size_t n_which,
                          const cdclq_config* cfg, float* const* u_out, int on_device, void* stream);

/* cdclq_quantize_batch with the factorisation replaced by caller-supplied factors: u_in[i] is a DEVICE
 * n x n f32 buffer produced by cdclq_prepare_factors for input i (on any rank, same configuration), or NULL
 * to factorise that input here.  Only the damped permuted Hessian is rebuilt locally.  Results are identical
 * to cdclq_quantize_batch.  skeleton_pct must be 0. */
int cdclq_quantize_batch_prepared(const cdclq_batch_input* inputs, size_t n_inputs, const float* const* u_in,
                                  const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config* cfg,
                                  int on_device, void* stream);

/* ---- runtime: one process per GPU, the NCCL communicator owned by the library ---------------------------
 * The reference runs on one host (pipeline::quantize_model over the rayon pool, src/pipeline.rs:79-227,
 * src/main.rs:199-203).  A runtime is one rank of a multi-GPU job: its device, its stream and, with more than one
 * rank, its NCCL communicator (NCCL is loaded at run time; a process that already loaded it shares that copy).
 * Every wait - the communicator's creation included - is bounded by timeout_s; after a timeout or an NCCL
 * failure the communicator is aborted and later calls on the runtime fail.  Calls are collective: every rank
 * makes the same calls in the same order.  Not re-entrant. */
typedef struct cdclq_runtime cdclq_runtime;

#define CDCLQ_UNIQUE_ID_BYTES 128
/* ncclGetUniqueId: rank 0 calls it and hands the bytes to every rank over any channel of the caller's. */
int cdclq_runtime_unique_id(uint8_t* id_out);
/* One rank: binds `device`, creates its stream and, with nranks > 1, joins the communicator of `unique_id`.
 * timeout_s <= 0 means 600 s. */
int cdclq_runtime_create(int device, int nranks, int rank, const uint8_t* unique_id, double timeout_s,
                         cdclq_runtime** out);
void cdclq_runtime_destroy(cdclq_runtime* rt);
/* The runtime's CUDA stream (cudaStream_t as void*): every kernel and collective of its calls runs on it, so a
 * caller times them with events recorded there. */
void* cdclq_runtime_stream(const cdclq_runtime* rt);

/* cdclq_quantize_batch over the runtime's ranks, with results identical to one GPU's.  The descriptors describe
 * FULL layers on every rank (w and the outputs point at row 0; a rank reads and writes only its rows): every
 * layer's rows are split in whole row chunks (the chunk each layer gets on one GPU), contiguous per rank, the
 * ranks' ranges rotating from layer to layer; each distinct input is factorised by one owner rank and its U
 * broadcast (per layer with a skeleton, whose column scores are summed over the ranks' rows in row order);
 * statistics are all-reduced and perm / gbits / stats are filled on every rank.  on_device = 0: host buffers
 * (an input's Hessian is only read on its owner rank - see cdclq_assign_owners with power 3 - and broadcast);
 * 1: device buffers on every rank.  gather != 0: rank 0 also receives every other rank's rows of codes, scales
 * and zero points.  The descriptors' colsq and u fields are not read. */
int cdclq_runtime_quantize_batch(cdclq_runtime* rt, const cdclq_batch_input* inputs, size_t n_inputs,
                                 const cdclq_batch_layer* layers, size_t n_layers, const cdclq_config* cfg,
                                 int on_device, int gather);
/* The row range [r0, r1) of `rank` for a layer of d_out rows: whole row chunks, contiguous, the range index
 * rotated by `rotate` (the layer's index in the batch). */
void cdclq_shard_rows(size_t d_out, size_t row_chunk, int rank, int nranks, size_t rotate, size_t* r0, size_t* r1);
/* Owner rank of each of `count` items of size ns[i]: longest processing time on ns[i]^power (3: a factorisation),
 * largest first, ties by index, to the least-loaded rank (ties to the lowest rank). */
void cdclq_assign_owners(const size_t* ns, size_t count, int nranks, int power, int* owner_out);

/* ---- model level: safetensors in, packed / dequantized safetensors and report.json out -----------------
 * pipeline::quantize_model (src/pipeline.rs:79-227).  Per weight shard: every 2-D `<layer>.weight` tensor that
 * passes the only / skip substring filters and has a Hessian (`<layer>.H`, or an alias of one) is quantized;
 * all such layers of the shard are quantized as one batch (over the runtime's ranks), then rank 0 writes
 * <out_dir>/dequant/<shard> (same names, shapes and dtypes, values on the grid) and <out_dir>/packed/<shard>
 * (six tensors per layer: .qweight .scales .qzeros .perm .gbits .gsize; header quantization=cdclq-v1,
 * orig_dtype, bits), every other tensor copied byte for byte, and <out_dir>/report.json.  Error messages are the
 * reference's.  rt = NULL: one GPU (the current device). */
typedef struct cdclq_model_opts {
    const char* const* weights; /* safetensors shard paths */
    size_t n_weights;
    const char* const* hessians; /* Hessian files (later files override earlier ones) */
    size_t n_hessians;
    const char* out_dir;
    const char* const* only; /* substrings; empty = every layer */
    size_t n_only;
    const char* const* skip;
    size_t n_skip;
    int32_t emit_packed;
    int32_t emit_dequant;
    int32_t verbose; /* per-layer progress lines on stderr, as the reference prints them */
    int32_t pad;
    cdclq_config cfg;
} cdclq_model_opts;

/* The Report's totals (src/pipeline.rs:69-76); the per-layer records are in report.json. */
typedef struct cdclq_model_report {
    uint64_t layers;
    double total_loss_gptq;
    double total_loss_final;
    double total_gain_pct;
    double total_secs;
} cdclq_model_report;

int cdclq_quantize_model(cdclq_runtime* rt, const cdclq_model_opts* opts, cdclq_model_report* report_out);

/* pipeline::dequantize_packed (src/pipeline.rs:239-275): expands every `<layer>.qweight` of a packed shard into
 * `<layer>.weight` (dtype: `dtype` if not NULL - F32 / F16 / BF16, HF spellings accepted - else the file's
 * orig_dtype, else F16), drops the companion tensors, copies everything else.  *layers_out = layers expanded. */
int cdclq_dequantize_packed(const char* input, const char* output, const char* dtype, uint64_t* layers_out);

/* ---- linear-algebra kernels (linalg.rs) ------------------------------------------------------------ */

/* cholesky_lower (src/linalg.rs:200-276): in place on a host n x n f64 matrix; lower triangle = L. */
int cdclq_cholesky_lower(double* a, size_t n);
/* tri_inverse_lower (src/linalg.rs:284-347): y = L^-1 (reads the lower triangle of l only). */
int cdclq_tri_inverse_lower(const double* l, size_t n, double* y);
/* upper_chol_of_inverse (src/linalg.rs:362-375): U upper, H^-1 = U^T U, stored as f32. */
int cdclq_upper_chol_of_inverse(const double* h, size_t n, float* u_out);
/* gram_accumulate (src/linalg.rs:388-418): h (n x n f64) += x^T y over t tokens (x, y: t x n f32). */
int cdclq_gram_accumulate(const float* x, const float* y, size_t t, size_t n, double* h);
/* Device variant of gram_accumulate for bf16 activations on the tcgen05 tensor cores: h (f64, device)
 * += x^T x over t tokens of x (t x n bf16, device), token chunks of 2048 accumulated in f32 then widened,
 * as src/linalg.rs:392-416 does.  Only the lower triangle of h is written when lower_only != 0. */
int cdclq_gram_accumulate_bf16_device(const void* x_bf16, size_t t, size_t n, double* h, int lower_only,
                                      void* stream);
/* The same for f16 or bf16 activations (dtype CDCLQ_DTYPE_F16 / CDCLQ_DTYPE_BF16; f16 x f16 products are exact
 * in f32 as well): what a half-precision model's forward pass hands to the Hessian capture. */
int cdclq_gram_accumulate_half_device(const void* x, int dtype, size_t t, size_t n, double* h, int lower_only,
                                      void* stream);
/* Device variant of gram_accumulate for f32 activations (bit-exact with the f32 path above). */
int cdclq_gram_accumulate_device(const float* x, const float* y, size_t t, size_t n, double* h, void* stream);
/* No counterpart in the reference.  Same computation and result as cdclq_gram_accumulate_device, but the
 * library allocates no device memory for it: the per-chunk f32 scratch is a fixed array inside the library
 * (CDCLQ_NOALLOC_GRAM_MAX_N^2 floats = 4 MiB, held on every GPU that loads the library until the process
 * exits).  For callers that cannot call cudaMalloc where they accumulate a Hessian - a hook inside a
 * framework whose allocator owns the device memory, or a runtime that forbids allocation after start-up.
 * The caller passes device pointers for x, y and h.  n above CDCLQ_NOALLOC_GRAM_MAX_N returns CDCLQ_ERR_ARG.
 * The first call on each device looks up the scratch's device address (cudaGetSymbolAddress); under CUDA's
 * default lazy module loading that first call is also when the library's module and the 4 MiB array are
 * loaded into the device's memory, so it can itself take device memory: make it at start-up (t = 0 only
 * resolves the scratch and computes nothing) and before any stream capture.  All calls share the one
 * scratch: calls that overlap on the GPU (other streams, other host threads) race and must be serialised
 * by the caller. */
#define CDCLQ_NOALLOC_GRAM_MAX_N 1024
int cdclq_gram_accumulate_device_noalloc(const float* x, const float* y, size_t t, size_t n, double* h,
                                         void* stream);

/* proxy_loss (src/engine.rs:808-815): sum_r e_r (E H)_r with E = w_t - w_hat. */
int cdclq_proxy_loss(const float* w_t, const float* w_hat, size_t rows, size_t n, const float* h,
                     double* out);
/* rtn_layer (src/engine.rs:822-838): round-to-nearest dequantized weights. */
int cdclq_rtn_layer(const float* w, size_t d_out, size_t n, const cdclq_config* cfg, float* out);
/* find_params (src/quant.rs:40-83) over `rows` independent groups of `len` values each. */
int cdclq_find_params(const float* vals, size_t rows, size_t len, uint32_t bits, int mse, float* scales,
                      float* zeros);

/* ---- packed format (quant.rs / io.rs) -------------------------------------------------------------- */

/* row_bytes (src/quant.rs:102-104). */
size_t cdclq_row_bytes(size_t n, size_t g, const uint8_t* gbits);
/* QLayer::pack (src/quant.rs:207-214) on the GPU: LSB-first mixed-width bit stream, d_out x row_bytes. */
int cdclq_pack(const uint8_t* codes, size_t d_out, size_t n, size_t g, const uint8_t* gbits, uint8_t* out);
/* QLayer::from_packed + dequantize (src/quant.rs:189-235) on the GPU: original column order, f32. */
int cdclq_unpack_dequant(const uint8_t* packed, size_t d_out, size_t n, size_t g, const uint8_t* gbits,
                         const uint32_t* perm, const float* scales, const float* zeros, float* out);

/* ---- runtime ---------------------------------------------------------------------------------------- */

/* Device-side profile of the last quantize call made on this thread: elapsed times between CUDA events
 * recorded on the call's stream at the phase boundaries, and the algorithmic work of each phase
 * (flops as 2 per multiply-add; repair counts only the passes each row chunk actually executed). */
typedef struct cdclq_run_profile {
    double ms_prepare;      /* permutations, factorisations, permuted weights */
    double ms_phase1;       /* blocked GPTQ: one launch over all rows */
    double ms_stats;        /* per-chunk conflict statistics: one launch */
    double ms_repair;       /* all repair pass launches and their pass-end reductions */
    double ms_final;        /* final scale refit */
    double flops_phase1;    /* f32: lazy GEMMs + in-block rank-1 updates */
    double flops_repair;    /* f32: refit and coordinate-descent gradient GEMMs of executed passes */
    double flops_final;     /* f32: final refit GEMMs */
    double flops_factor;    /* f64: n^3/3 Cholesky + n^3/3 triangular inverse per factorisation */
    uint64_t repair_launches;
    uint64_t factorisations;
    uint64_t weights;
    uint64_t launches;      /* kernel launches issued by the call */
    uint64_t factor_batches; /* factorisation launch batches: one per width when all fit in free memory */
    double ms_host;         /* host wall time of the call */
    uint64_t repair_layout; /* 0 one launch per pass, 1 persistent CTAs, 2 persistent 2-CTA clusters, 3 heavy chunks
                               as SM-owning 2-CTA clusters beside a persistent launch, 4 the same as 4-CTA clusters
                               with column-split GEMMs, 5 none (GPTQ only) */
} cdclq_run_profile;

int cdclq_last_run_profile(cdclq_run_profile* out);

/* Number of CUDA kernel launches this library has issued so far in this process. */
uint64_t cdclq_launch_count(void);
/* Library version string. */
const char* cdclq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CDCLQ_H_ */
