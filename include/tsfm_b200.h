/*
 * tsfm_b200.h — C ABI of the B200 forecast backend.
 *
 * One shared library (libtsfm_b200.so) replaces the forward pass of tsfm-zig's three model
 * families with sm_100a CUDA kernels. Every entry point takes plain pointers and sizes, returns a
 * tsfm_status (0 = success) and never throws; the message of the last failure on the calling
 * thread is tsfm_last_error(). There is no CPU fallback: an unusable device is an error.
 *
 * Two seams of the reference are replaced:
 *
 *  1. The family seam. Each family's `forecaster.forecast` becomes one call:
 *       chronos2/forecaster.zig:14-22      -> tsfm_forecast_chronos2
 *       chronos_bolt/forecaster.zig:22     -> tsfm_forecast_bolt
 *       timestral/forecaster.zig:57-69     -> tsfm_forecast_timestral
 *     The weights come from the caller's safetensors mapping (core/safetensors.zig:59-97) through
 *     a table of named tensors; the tensor names and element counts are those the reference's
 *     `Model.load` functions ask for (chronos2/model.zig:77-125, chronos_bolt/model.zig:101-172,
 *     timestral/model.zig:136-200), and a missing tensor, a wrong element count or an unsupported
 *     dtype is reported like `Weights.get` reports it.
 *
 *  2. The GEMM offload seam of the CUDA backend (platform/cuda/gemm.c:232-330): the four
 *     functions cuda_weight_register / cuda_weight_release / cuda_sgemm_nt / cuda_sgemm_nn keep
 *     their signatures and meaning as tsfm_weight_register ... tsfm_sgemm_nn.
 *
 * Layouts are row-major. Host-pointer entry points copy inputs to the device and results back and
 * return when the results are written; *_device entry points take device pointers and a CUDA
 * stream (cudaStream_t passed as void*) and return after enqueueing.
 */
#ifndef TSFM_B200_H
#define TSFM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------------------------------------
 * Status codes. The reference returns Zig error unions; each code below names the error it
 * stands for (e.g. error.MissingTensor in core/safetensors.zig:62).
 */
typedef enum tsfm_status {
    TSFM_OK = 0,
    TSFM_ERR_INVALID_ARGUMENT = 1,   /* null pointer, zero size, bad option */
    TSFM_ERR_INVALID_CONFIG = 2,     /* error.InvalidConfig (config.zig validate) */
    TSFM_ERR_MISSING_TENSOR = 3,     /* error.MissingTensor */
    TSFM_ERR_SHAPE_MISMATCH = 4,     /* error.ShapeMismatch */
    TSFM_ERR_UNSUPPORTED_DTYPE = 5,  /* error.UnsupportedDtype */
    TSFM_ERR_CUDA = 6,               /* a CUDA runtime or driver call failed */
    TSFM_ERR_OUT_OF_MEMORY = 7,      /* device or host allocation failed */
    TSFM_ERR_DEVICE_TIMEOUT = 8,     /* a kernel's bounded wait gave up (see tsfm_last_error) */
    TSFM_ERR_EMPTY_INPUT = 9,        /* error.EmptyInput */
    TSFM_ERR_HORIZON_TOO_LONG = 10,  /* error.HorizonTooLong */
    TSFM_ERR_UNSUPPORTED = 11,       /* a configuration the backend does not implement */
    TSFM_ERR_DEGENERATE_INPUT = 12,  /* error.DegenerateInput (timestral/forecaster.zig:419) */
    TSFM_ERR_ASYMMETRIC_QUANTILES = 13, /* error.AsymmetricQuantiles (timestral/forecaster.zig:110) */
    TSFM_ERR_COVARIATES_UNSUPPORTED = 14, /* error.CovariatesUnsupported / KnownCovariatesUnsupported */
    TSFM_ERR_NO_DEVICE = 15,         /* no CUDA device, or the device ordinal is out of range */
    TSFM_ERR_BUFFER_TOO_SMALL = 16,  /* an output buffer is shorter than the result (the needed size is returned) */
    TSFM_ERR_IO = 17,                /* writing to a file descriptor failed */
    TSFM_ERR_RAGGED_INPUT = 18,      /* error.RaggedInput (core/series.zig:58) */
    TSFM_ERR_RAGGED_BLOCKS = 19      /* error.RaggedBlocks (core/series.zig:39, 64) */
} tsfm_status;

typedef enum tsfm_family {
    TSFM_CHRONOS2 = 1,
    TSFM_CHRONOS_BOLT = 2,
    TSFM_TIMESTRAL = 3
} tsfm_family;

/* Checkpoint dtypes accepted by the weight table (core/safetensors.zig:66: F32, F16, BF16). */
typedef enum tsfm_dtype {
    TSFM_DTYPE_F32 = 0,
    TSFM_DTYPE_F16 = 1,
    TSFM_DTYPE_BF16 = 2
} tsfm_dtype;

/* Operand type of the tensor-core contractions; accumulation and the residual stream are always
 * FP32. F16 and BF16 run at the same tensor-core rate; F16 keeps 3 more mantissa bits (the
 * precision of TF32), BF16 the FP32 exponent range. TF32 is reserved.
 * F16C ("FP16, corrected") adds to every FP16 product the two first-order rounding terms
 * x_hi * (W - f16(W)) + (x - x_hi) * f16(W), computed as FP8 (E4M3) products with power-of-two
 * scales into the same FP32 accumulator: weights and activations act as if kept to about 15
 * significant bits, at twice the tensor-core work of F16 (the FP8 rate is twice the FP16 rate).
 * It is the mode that meets the 1e-2 * scale forecast bound at Chronos-2's full shape (F16
 * alone does not). Chronos-2 only for now. */
typedef enum tsfm_compute {
    TSFM_COMPUTE_BF16 = 0,
    TSFM_COMPUTE_TF32 = 1,
    TSFM_COMPUTE_F16 = 2,
    TSFM_COMPUTE_F16C = 3
} tsfm_compute;

/* Timestral layer kinds, the entries of `block_schedule` (timestral/config.zig:94-100). */
typedef enum tsfm_layer_kind {
    TSFM_LAYER_TIME = 0,
    TSFM_LAYER_VARIATE = 1,
    TSFM_LAYER_TIME_VARIATE = 2,
    TSFM_LAYER_VARIATE_TIME = 3
} tsfm_layer_kind;

/* One named checkpoint tensor: `data` points at `numel` elements of `dtype` (host memory, e.g.
 * the safetensors mapping). The table is read during tsfm_model_create only. */
typedef struct tsfm_tensor {
    const char *name;
    const void *data;
    int32_t dtype;   /* tsfm_dtype */
    uint64_t numel;
} tsfm_tensor;

/* The inference configuration of one checkpoint. The fields mirror the reference's Config
 * structs (chronos2/config.zig:9-30, chronos_bolt/config.zig:10-32, timestral/config.zig:6-28);
 * fields a family does not use are ignored. `validate()` of each family is applied by
 * tsfm_model_create. */
typedef struct tsfm_config {
    int32_t family;              /* tsfm_family */
    /* shared transformer shape */
    int32_t d_model;
    int32_t d_ff;                /* Chronos d_ff; Timestral mlp_hidden_dim */
    int32_t num_heads;
    int32_t d_kv;                /* Chronos head width; Timestral uses d_model / num_heads */
    int32_t num_layers;          /* Chronos encoder layers (Timestral: n_layer_kinds) */
    int32_t num_decoder_layers;  /* Chronos-Bolt */
    int32_t patch_size;          /* input_patch_size (== stride, == output_patch_size) */
    int32_t context_length;
    int32_t max_output_patches;  /* Chronos-2 */
    int32_t prediction_length;   /* Chronos-Bolt */
    int32_t num_quantiles;
    const double *quantiles;     /* Chronos quantiles / Timestral quantile_knots */
    double layer_norm_epsilon;   /* Timestral norm_eps */
    double rope_theta;
    double time_encoding_scale;  /* Chronos-2 */
    int32_t use_arcsinh;         /* Chronos-2 use_arcsinh; Timestral use_asinh */
    int32_t use_reg_token;
    /* Chronos-Bolt T5 specifics */
    int32_t relative_attention_num_buckets;
    int32_t relative_attention_max_distance;
    int32_t decoder_start_token_id;
    int32_t reg_token_id;
    /* Timestral */
    int32_t block_size;
    int32_t n_layer_kinds;
    const int32_t *layer_kinds;  /* tsfm_layer_kind per layer */
    double rope_partial_factor;
    double minimum_scale;
    double quantile_width_factor;
    int32_t covariate_enabled;
    int32_t attend_missing_patches;
    int32_t time_attn_gate;      /* 1 = "sdpa_sigmoid" gate present */
    int32_t variate_attn_gate;
} tsfm_config;

typedef struct tsfm_model tsfm_model;

/* Timestral covariates (timestral/forecaster.zig:37-46): numeric arrays are (B, C, len) f32 with
 * NaN for missing, categorical ones (B, C, len) f64 codes; past arrays have len T, known ones
 * T + horizon. A null pointer means "none". */
typedef struct tsfm_covariates {
    const float *past;      size_t n_past;
    const float *known;     size_t n_known;
    const double *cat_past; size_t n_cat_past;
    const double *cat_known; size_t n_cat_known;
} tsfm_covariates;

/* Timestral forecaster options (timestral/forecaster.zig:21-32). */
typedef struct tsfm_timestral_options {
    size_t max_context;               /* 0 = the trained context length */
    size_t per_shot_horizon_patches;  /* default 32, capped at block_size */
    float quantile_real_cap_k;        /* default 1e4; 0 disables */
    float extreme_value_threshold;    /* default 1e30 */
    int32_t symmetric_averaging;      /* default 1 */
    int32_t clip_nonnegative;         /* default 1 */
} tsfm_timestral_options;

/* ---------------------------------------------------------------------------------------------
 * Library */

/* Message of the last failure on the calling thread ("" if none). Never null. */
const char *tsfm_last_error(void);
/* Name of a status code. */
const char *tsfm_status_string(int32_t status);
/* Number of visible CUDA devices. */
int32_t tsfm_device_count(int32_t *count);
/* Library version string. */
const char *tsfm_version(void);

/* ---------------------------------------------------------------------------------------------
 * Models. A model holds one weight replica per device in `devices` (n_devices >= 1). Forecasts
 * shard series across the replicas (contiguous ranges, one host thread per device, no
 * collective); the output does not depend on the number of devices. Replaces `Model.load` of
 * each family plus nn.Weight.initWith's upload (core/nn.zig:35-38). */
int32_t tsfm_model_create(const tsfm_config *config, const tsfm_tensor *tensors, size_t n_tensors,
                          int32_t compute, const int32_t *devices, int32_t n_devices,
                          tsfm_model **out);
void tsfm_model_destroy(tsfm_model *model);
/* Device bytes held by the weights of one replica. */
int32_t tsfm_model_weight_bytes(const tsfm_model *model, uint64_t *bytes);

/* ---------------------------------------------------------------------------------------------
 * Forecasts (host pointers). */

/* chronos2/forecaster.zig:14-22: `inputs` (b, t) f32 with NaN = missing; writes (b, horizon, Q)
 * quantiles in the config's quantile order. horizon <= max_output_patches * patch_size. */
int32_t tsfm_forecast_chronos2(tsfm_model *model, const float *inputs, size_t b, size_t t,
                               size_t horizon, float *out);

/* chronos_bolt/forecaster.zig:22: as above; horizons beyond prediction_length feed every quantile
 * path back (chronos_bolt/forecaster.zig:45-78). */
int32_t tsfm_forecast_bolt(tsfm_model *model, const float *inputs, size_t b, size_t t,
                           size_t horizon, float *out);

/* timestral/forecaster.zig:57-69: `inputs` (b, v, t) f32, zero where unobserved, `observed`
 * (b, v, t) 0/1 bytes; writes (b, v, horizon, Q). `cov` and `opts` may be null (none / defaults). */
int32_t tsfm_forecast_timestral(tsfm_model *model, const float *inputs, const uint8_t *observed,
                                size_t b, size_t v, size_t t, size_t horizon,
                                const tsfm_covariates *cov, const tsfm_timestral_options *opts,
                                float *out);

/* Default Timestral options (timestral/forecaster.zig:21-32). */
void tsfm_timestral_default_options(tsfm_timestral_options *opts);

/* ---------------------------------------------------------------------------------------------
 * Forecasts on device-resident data (first replica's device only): `inputs` and `out` are device
 * pointers, `stream` a cudaStream_t or null for the legacy default stream. */
int32_t tsfm_forecast_chronos2_device(tsfm_model *model, const float *inputs, size_t b, size_t t,
                                      size_t horizon, float *out, void *stream);
int32_t tsfm_forecast_bolt_device(tsfm_model *model, const float *inputs, size_t b, size_t t,
                                  size_t horizon, float *out, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Per-kernel timing of the device forward. When enabled, every kernel launch of a forecast is
 * bracketed by CUDA events on the launching stream; tsfm_profile_read returns, per kernel class,
 * the launch count, the summed device time (ms) and the algorithmic work (FLOPs for contractions,
 * bytes for memory-bound kernels). Class names: "gemm", "attention", "rmsnorm", "patch", "head",
 * "other". */
int32_t tsfm_profile_enable(tsfm_model *model, int32_t enable);
int32_t tsfm_profile_reset(tsfm_model *model);
int32_t tsfm_profile_read(tsfm_model *model, const char *kernel_class, uint64_t *launches,
                          double *ms, double *work);
/* Kernel launches made by the most recent forecast on the first replica. */
int32_t tsfm_last_launch_count(tsfm_model *model, uint64_t *launches);

/* ---------------------------------------------------------------------------------------------
 * The reference's CUDA GEMM seam (platform/cuda/gemm.c:232-330), same signatures and semantics:
 * host pointers, row-major, 0 = success. The device is the current CUDA device (gemm.c uses
 * device 0). Products run on the tensor cores with 3xTF32 splitting, which keeps them within
 * FP32 SGEMM accuracy (the reference's own test uses tolerance 1e-4). */
void *tsfm_weight_register(const float *data, size_t len);                    /* gemm.c:232 */
void tsfm_weight_release(void *handle);                                      /* gemm.c:244 */
int tsfm_sgemm_nt(int m, int n, int k, float alpha, const float *A, int lda,  /* gemm.c:316 */
                  const float *B, int ldb, float *C, int ldc, void *b_buf);
int tsfm_sgemm_nn(int m, int n, int k, const float *A, int lda,               /* gemm.c:323 */
                  const float *B, int ldb, float *C, int ldc, void *b_buf);

/* tsfm_sgemm_nt_noalloc has no counterpart in the reference. It computes the same FP32-accurate
 * C[m, n] = alpha * A[m, k] * B[n, k]^T as tsfm_sgemm_nt, but on DEVICE pointers A, B, C (row
 * strides lda, ldb, ldc in elements) and without allocating anything, for callers that cannot
 * call cudaMalloc once running: latency-bound loops that cannot afford the device-wide
 * synchronisation of cudaMalloc/cudaFree, real-time hosts that forbid allocation after start-up,
 * and processes whose own pool owns all device memory. Its scratch is a fixed 16 MiB array inside
 * the library (held by every GPU that loads it) with room for the hi/lo splits of A and B:
 * round_up(m * round_up(k, 4), 64) + round_up(n * round_up(k, 4), 64) must not exceed 2^21 - 64
 * floats (for k a multiple of 64: m + n <= 32767), else TSFM_ERR_INVALID_ARGUMENT and nothing
 * runs. All calls share that array: calls that overlap on the GPU race. Runs on `stream` (null =
 * legacy default stream) and is synchronous: it reads its device error word back and waits for
 * `stream` before returning, so C is written on return; it must therefore never be called on a
 * stream that is being captured into a CUDA graph. The first call on each device looks up the
 * array's address (which may load the library's device code). 0 = success, else a tsfm_status. */
int32_t tsfm_sgemm_nt_noalloc(int m, int n, int k, float alpha, const float *A, int lda,
                              const float *B, int ldb, float *C, int ldc, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Kernel-level entry points on device pointers (what the family forwards are built from; used by
 * the kernel parity tests). All return after enqueueing on `stream`.
 *
 * tsfm_kernel_linear: y[M, N] (+)= act(x[M, K] · W[N, K]^T + bias) on the tensor cores.
 *   x_dtype/w_dtype: TSFM_DTYPE_BF16 or TSFM_DTYPE_F16 (kind::f16), or TSFM_DTYPE_F32 (read as
 *   TF32, kind::tf32); both equal.
 *   out_mode: 0 = store in the 16-bit operand type, 1 = store f32, 2 = accumulate into f32.
 *   act: 0 none, 1 relu, 3 gated pairs (W's rows in 256-row blocks [g (128) | u (128)], y of
 *   N / 2 columns with y[:, 128 t + c] = g[c] * silu(u[c]) for block t; N % 256 == 0, out_mode 0,
 *   16-bit operands, no bias: mulSilu of core/nn.zig:302-563 fused into the product).
 *   bias may be null. Replaces nn.linear (core/nn.zig:270-293). */
int32_t tsfm_kernel_linear(const void *x, int32_t x_dtype, const void *w, int32_t w_dtype,
                           const float *bias, void *y, int32_t out_mode, int32_t act,
                           int64_t M, int64_t N, int64_t K, int64_t ldx, int64_t ldw, int64_t ldy,
                           void *stream);

/* tsfm_kernel_linear_corrected: the corrected product of TSFM_COMPUTE_F16C on FP32 device inputs
 * x [M, K] and W [N, K] (dense rows, K % 8 == 0): both are split into FP16 operands and FP8
 * correction companions exactly as a TSFM_COMPUTE_F16C model holds them, then
 * y[M, N] (dense) = act(x W^T + bias) with out_mode 0 = FP16 (and, when y8 is not null, its FP8
 * companion [M, 2N] bytes: e4m3(y16 / 32) then e4m3((y - y16) * 128)), 1 = store f32,
 * 2 = accumulate into f32; act 0 none, 1 relu. terms = 2 adds both correction terms, 1 only the
 * weight term x_hi (W - f16(W)). Allocates its temporaries on `stream` and returns after the
 * product is enqueued. The kernel-level test of nn.linear's corrected form (core/nn.zig:270-293). */
int32_t tsfm_kernel_linear_corrected(const float *x, const float *w, const float *bias, void *y,
                                     void *y8, int32_t out_mode, int32_t act, int64_t M, int64_t N,
                                     int64_t K, int32_t terms, void *stream);

/* tsfm_test_bounded_wait: the failure-detection check of the device waits. Every wait of the
 * warp-specialised kernels (TMA and tensor-core barriers) gives up after 2 s, records its site in
 * the device error word and lets the kernel return, and the host reports
 * TSFM_ERR_DEVICE_TIMEOUT; this entry runs that same bounded wait on a barrier that nothing
 * arrives on, with a limit of limit_ns (1 us .. 2 s), and returns what the host then reports
 * (TSFM_ERR_DEVICE_TIMEOUT). The context stays usable. No counterpart in the reference (its GPU
 * seam has no device waits).
 * Host-side failure injection: with the environment variable TSFM_FAIL_REPLICA=<i>, the forecast
 * worker of replica i of a multi-device model fails before touching its device while the other
 * workers run and are joined (the forecast returns TSFM_ERR_INVALID_ARGUMENT); unset in normal
 * use. */
int32_t tsfm_test_bounded_wait(int64_t limit_ns, void *stream);

/* The corrected product's pieces on device pointers, for benches and tests that time the product
 * alone: tsfm_kernel_split_f16c writes x16 = f16(x) [rows, cols] and its FP8 companion x8
 * [rows, 2 cols]; tsfm_kernel_weight_f16c writes w16 = f16(w) * 2^s and w8 [rows, 2 cols] and
 * returns *acc_scale = 2^-s (it waits for `stream`); tsfm_kernel_linear_f16c runs
 * tsfm_kernel_linear_corrected's product on such operands (dense rows). */
int32_t tsfm_kernel_split_f16c(const float *x, int64_t rows, int64_t cols, void *x16, void *x8,
                               void *stream);
int32_t tsfm_kernel_weight_f16c(const float *w, int64_t rows, int64_t cols, void *w16, void *w8,
                                float *acc_scale, void *stream);
int32_t tsfm_kernel_linear_f16c(const void *x16, const void *x8, const void *w16, const void *w8,
                                float acc_scale, const float *bias, void *y, void *y8,
                                int32_t out_mode, int32_t act, int64_t M, int64_t N, int64_t K,
                                int32_t terms, void *stream);

/* The indexing work of the forecasters, exposed for bit-exact parity tests. All return after
 * enqueueing on `stream`; pointers are device pointers.
 *
 * tsfm_relative_bucket: relativeBucket (chronos_bolt/model.zig:74-85), the T5 bucket of key - query
 *   offset `rel` that the Bolt encoder's bias table is built from (host function; -1 on bad
 *   arguments).
 * tsfm_kernel_patch: the instance norm and context-patch features of one forecast call, as the
 *   forward computes them before its first product (features here in exact FP32, not rounded to
 *   the TF32 operand): family TSFM_CHRONOS2 (chronos2/forecaster.zig:94-143; features
 *   [time, value, mask] of 3 * patch per patch, key_valid (b, n_ctx)) or TSFM_CHRONOS_BOLT
 *   (chronos_bolt/forecaster.zig:150-197; [value, mask] of 2 * patch, key_valid (b, n_ctx + reg)
 *   with the REG slot valid); inputs (b, t_in) with NaN = missing, the last context_length steps
 *   used, left-padded to a multiple of patch; loc, scale (b).
 * tsfm_kernel_timestral_block_inputs: predictBlock's window statistics (f64 causal Welford, f32
 *   results), features [asinh((x - loc) / scale), missing] per step (exact FP32), key validity and
 *   first observed patch per group (timestral/model.zig:253-362; a value >= n for a group without
 *   an observed patch, which the forward reads as 0) over rows of t context steps, then with
 *   covariates hl known-future steps (rows of role 2 normalised by their whole-row statistics);
 *   roles: one int8 per row of a group of vall rows (0 target, 1 past, 2 known). loc / scale /
 *   key_valid (rows, n), feats (rows, n, 2 * patch), n = (t + hl) / patch. Allocates a few bytes per
 *   row of temporaries on `stream`. */
int32_t tsfm_relative_bucket(int64_t rel, int32_t num_buckets, int32_t max_distance);
int32_t tsfm_kernel_patch(int32_t family, const float *inputs, int64_t b, int64_t t_in,
                          int64_t context_length, int32_t patch, float time_encoding_scale,
                          int32_t use_arcsinh, int32_t use_reg_token, float *loc, float *scale,
                          float *feats, uint8_t *key_valid, void *stream);
int32_t tsfm_kernel_timestral_block_inputs(const float *ctx, const uint8_t *observed, int64_t rows,
                                           int64_t t, const float *known_future,
                                           const uint8_t *known_future_observed, int64_t hl,
                                           int32_t patch, int32_t vall, const int8_t *roles,
                                           int32_t covariates, double minimum_scale,
                                           int32_t use_asinh, int32_t attend_missing, float *loc,
                                           float *scale, float *feats, uint8_t *key_valid,
                                           int32_t *first_obs, void *stream);

/* tsfm_kernel_attention: o = softmax(mask(scale · q k^T + bias)) v per (group, head) over `n`
 * tokens of head width 64, q/k/v bf16 with row stride ld_qkv (elements), o bf16 with row stride
 * ld_o; group g's tokens are rows [g*n, (g+1)*n). key_valid: (groups, n) bytes, or null = all
 * valid. mask_mode: 0 = T5 additive (invalid keys excluded; a row with no valid key averages all
 * keys, as -floatMax addition does), 1 = causal over valid keys with the diagonal open,
 * 2 = bidirectional over valid keys with the diagonal open. rel_bias: (heads, 2n-1) f32 added
 * at [h][j - i + n - 1], or null. Replaces attn.selfAttend (core/attn.zig:72-96). */
int32_t tsfm_kernel_attention(const void *q, const void *k, const void *v, int64_t ld_qkv,
                              void *o, int64_t ld_o, const uint8_t *key_valid,
                              const float *rel_bias, int32_t groups, int32_t heads, int32_t n,
                              float scale, int32_t mask_mode, int32_t dtype, void *stream);

/* tsfm_kernel_attention_ex: tsfm_kernel_attention with Timestral's time-attention masks in full
 * (timestral/model.zig:558-635): for mask_mode 1-2, queries i < ne are encoder rows (causal over
 * valid keys below ne, diagonal open; bidirectional for mode 2 or where group_bidir[g] != 0) and
 * queries i >= ne decoder rows reading the valid keys below l plus their chain [ne, i]; key_valid
 * has row stride kv_stride (0: n). o32 (row stride ld_o32 floats), when not null, receives an FP32
 * output instead of o. o8 (row stride ld_o8 bytes), when not null, receives the FP8 companion of
 * the FP16 output (tcgen05 kernel; the layout of tsfm_kernel_split_f16c's x8). rel_bias as in
 * tsfm_kernel_attention (mode 0). force_path: 0 automatic, 1 the tcgen05 kernel (UNSUPPORTED if it
 * cannot take the call), 2 the mma.sync kernel, 3 the tcgen05 kernel with two softmax threads per
 * query row. */
int32_t tsfm_kernel_attention_ex(const void *q, const void *k, const void *v, int64_t ld_qkv,
                                 void *o, int64_t ld_o, float *o32, int64_t ld_o32, uint8_t *o8,
                                 int64_t ld_o8, const uint8_t *key_valid, int64_t kv_stride,
                                 const float *rel_bias, const uint8_t *group_bidir, int32_t groups,
                                 int32_t heads, int32_t n,
                                 float scale, int32_t mask_mode, int32_t ne, int32_t l,
                                 int32_t dtype, int32_t force_path, void *stream);

/* tsfm_kernel_target_encode: Timestral's categorical target encoding (timestral/forecaster.zig:
 * 201-238) on device pointers: inputs (b, t) f32 and observed (b, t) u8 of a univariate target,
 * codes (b, nc, len) f64 with len = t (past) or t + horizon (known); out (b, nc, len) f32.
 * have_target == 0 only rounds the codes. The forecaster runs the same kernels. */
int32_t tsfm_kernel_target_encode(const float *inputs, const uint8_t *observed, int64_t b, int64_t t,
                                  int64_t max_context, const double *codes, int64_t nc, int64_t len,
                                  int32_t have_target, float *out, void *stream);

/* tsfm_kernel_rmsnorm: out[r, :] = x[r, :] / sqrt(mean(x^2) + eps) * scale, x f32, out bf16 or
 * f32 (out_dtype). Replaces nn.rmsNorm (core/nn.zig:367-396). */
int32_t tsfm_kernel_rmsnorm(const float *x, const float *scale, void *out, int32_t out_dtype,
                            int64_t rows, int64_t dim, float eps, void *stream);

/* tsfm_kernel_rmsnorm_ex: tsfm_kernel_rmsnorm (out_dtype bf16, f16 or f32) plus, for an f16
 * output, the FP8 companion the corrected mode (TSFM_COMPUTE_F16C) feeds to the next product:
 * out8 (null for none) row r at out8 + r * ld8 bytes, byte c = e4m3(f16(y[r, c]) / 32) and byte
 * dim + c = e4m3((y[r, c] - f16(y[r, c])) * 128), y the FP32 result. dim % 4 == 0,
 * ld8 >= 2 * dim. The same kernels as the forecasts' norms. Replaces nn.rmsNorm
 * (core/nn.zig:367-396); the companion has no counterpart in the reference. */
int32_t tsfm_kernel_rmsnorm_ex(const float *x, const float *scale, void *out, int32_t out_dtype, void *out8,
                               int64_t ld8, int64_t rows, int64_t dim, float eps, void *stream);

/* ---------------------------------------------------------------------------------------------
 * CSV output of a forecast. Replaces the CLI's writeCsv (src/main.zig:181-198): a header
 * "series,variate,step" followed by ",q<level>" per quantile level, then one line per
 * (series, variate, step) of values (series, variates, horizon, num_levels) f32 row-major:
 * "s,v,step+1" followed by ",<value>" per level, each line ended by '\n'. Numbers are printed as
 * Zig's "{d}": integers in decimal, floats in decimal notation (no exponent) with the shortest
 * digits that read back to the same value (f32 values, f64 levels); "nan", "inf", "-inf", "-0"
 * as Zig prints them. The text is rendered on the GPU.
 *
 * tsfm_csv_format: values in host memory; the text goes to out[0, capacity). *length receives
 * the text's byte count; when it exceeds capacity (out may then be NULL with capacity 0) the
 * call returns TSFM_ERR_BUFFER_TOO_SMALL and writes nothing past the header.
 * tsfm_csv_write: values in host memory; the text is written to the file descriptor fd (the
 * reference writes stdout), *length = bytes written.
 * tsfm_csv_format_device: values and out in the current device's memory, ordered on stream;
 * returns after the text is complete. At most 1000 levels. */
int32_t tsfm_csv_format(const float *values, size_t series, size_t variates, size_t horizon,
                        const double *levels, size_t num_levels, int32_t device, char *out,
                        size_t capacity, size_t *length);
int32_t tsfm_csv_write(const float *values, size_t series, size_t variates, size_t horizon,
                       const double *levels, size_t num_levels, int32_t device, int32_t fd,
                       size_t *length);
int32_t tsfm_csv_format_device(const float *values, size_t series, size_t variates, size_t horizon,
                               const double *levels, size_t num_levels, char *out, size_t capacity,
                               size_t *length, void *stream);

/* ---------------------------------------------------------------------------------------------
 * Series CSV input. Replaces the reader's parseBlocks (core/series.zig:21-68): blank-line-
 * separated blocks of equal-length rows; '#' lines skipped; comma-separated tokens when a line
 * holds a comma, else space / tab separated; each token trimmed of " \t\r" and parsed as f64
 * (correctly rounded; NaN when empty or not a number). The values are (blocks, rows, len)
 * row-major. Errors: TSFM_ERR_RAGGED_INPUT, TSFM_ERR_RAGGED_BLOCKS, TSFM_ERR_EMPTY_INPUT, in the
 * reference's order. The text is split and parsed on the GPU.
 *
 * tsfm_parse_blocks: text in host memory, values to host memory. values == NULL only returns
 * the shape; a capacity (in values) below blocks * rows * len returns TSFM_ERR_BUFFER_TOO_SMALL.
 * tsfm_parse_blocks_device: text and outputs in the current device's memory, ordered on stream;
 * values (f64) and values_f32 (toF32, core/series.zig:78-82: round to nearest) may each be NULL;
 * returns after the values are complete. */
int32_t tsfm_parse_blocks(const char *text, size_t length, int32_t device, double *values,
                          size_t capacity, size_t *blocks, size_t *rows, size_t *len);
int32_t tsfm_parse_blocks_device(const char *text, size_t length, double *values, float *values_f32,
                                 size_t capacity, size_t *blocks, size_t *rows, size_t *len,
                                 void *stream);

/* Per-kernel device time of the CSV kernels on a device ("describe", "scan", "text"): launches and
 * milliseconds since the last enable (CUDA events around each launch while enabled). */
int32_t tsfm_csv_profile_enable(int32_t device, int32_t enable);
int32_t tsfm_csv_profile_read(int32_t device, const char *kernel, uint64_t *launches, double *ms);

#ifdef __cplusplus
}
#endif

#endif /* TSFM_B200_H */
