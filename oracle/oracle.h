/*
 * ORACLE — test infrastructure only. Not part of the product.
 *
 * A CPU restatement of tsfm-zig's forecast path (the reference is Zig 0.17.1 and cannot be built
 * here). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and
 * only as the checker or the timed CPU baseline; the CUDA library never links or calls it.
 *
 * Parity status: pinned to the reference's own known-answer tests (the T5 bucket table of
 * chronos_bolt/model.zig:695-703, quantileLinear of chronos_bolt/forecaster.zig:222-228, the
 * mask-vs-float64 attention property of core/attn.zig:156-189, the CSV cases of
 * core/series.zig:95-112). The reference publishes no forecast-level golden outputs, so
 * forecast-level parity of this restatement is unpinned beyond those pieces.
 *
 * Arithmetic follows the reference: FP32 compute, FP64 for instance-norm and Welford statistics,
 * the same operation order per element; matrix products use a fixed per-element reduction order,
 * so results do not depend on the thread count (the reference's core/nn.zig:285-288 property).
 */
#ifndef TSFM_ORACLE_H
#define TSFM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#include "../include/tsfm_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct oracle_model oracle_model;

int32_t oracle_set_threads(int32_t n);
int32_t oracle_get_threads(void);
/* Precision study only (oracle_emul.cpp): 0 (default) = the reference's FP32 arithmetic; 1-7 =
 * the Chronos-2 forward with operands rounded as a reduced-precision device product consumes
 * them (schemes listed in oracle_emul.cpp). Process-wide; not for concurrent forecasts. */
int32_t oracle_set_operand_emulation(int32_t scheme);
/* Overrides the scheme for one class of products (1 q/k/v, 2 attention output, 3 group v, 4 group
 * o, 5 MLP wi, 6 MLP wo, 7 patch-embedding output; -1 = back to the global scheme). */
int32_t oracle_set_operand_emulation_class(int32_t cls, int32_t scheme);
/* Rounds the operands of TF32-operand products (the patch features' products) to TF32 in every
 * scheme, not only in 1 and 5 (reset by oracle_set_operand_emulation). */
int32_t oracle_set_operand_emulation_tf32(int32_t round);
const char *oracle_last_error(void);

int32_t oracle_model_create(const tsfm_config *cfg, const tsfm_tensor *tensors, size_t n_tensors,
                            oracle_model **out);
void oracle_model_destroy(oracle_model *m);

int32_t oracle_forecast_chronos2(oracle_model *m, const float *inputs, size_t b, size_t t,
                                 size_t horizon, float *out);
int32_t oracle_forecast_bolt(oracle_model *m, const float *inputs, size_t b, size_t t,
                             size_t horizon, float *out);
int32_t oracle_forecast_timestral(oracle_model *m, const float *inputs, const uint8_t *observed,
                                  size_t b, size_t v, size_t t, size_t horizon,
                                  const tsfm_covariates *cov, const tsfm_timestral_options *opts,
                                  float *out);

/* Known-answer pieces, exposed so the tests can pin them against the reference's own vectors. */
int32_t oracle_relative_bucket(int64_t rel, uint32_t num_buckets, uint32_t max_distance);
float oracle_quantile_linear(const float *sorted, size_t n, float level);
/* attn.selfAttend for one head; mask: 0 full, 1 keys_additive, 2 causal, 3 causal_keys,
 * 4 full_keys (the order of core/attn.zig:10-21). */
int32_t oracle_self_attend(int32_t mask, const float *q, const float *k, const float *v, float *o,
                           size_t ldq, size_t ldk, size_t ldv, size_t ldo, size_t n, size_t hd,
                           float scale, const uint8_t *key_valid, const float *bias);
int32_t oracle_mask_pick(int32_t causal, int32_t all_keys_valid, int32_t additive);
/* core/series.zig parseBlocks: returns 0 and fills blocks/rows/len, writing up to cap values;
 * nonzero error codes: 1 RaggedInput, 2 RaggedBlocks, 3 EmptyInput, 4 capacity. */
int32_t oracle_parse_blocks(const char *text, double *values, size_t cap, size_t *blocks,
                            size_t *rows, size_t *len);
/* Timestral's categorical target encoding (forecaster.zig:201-238) for one kind of covariate. */
int32_t oracle_target_encode(const float *inputs, const uint8_t *observed, size_t b, size_t t,
                             size_t max_context, const double *codes, size_t nc, size_t len,
                             int32_t have_target, float *out);
/* nn.linear (y = x W^T + b) and nn.rmsNorm, for kernel-level parity tests. */
int32_t oracle_linear(const float *x, const float *w, const float *bias, float *y, size_t rows,
                      size_t out, size_t in);
int32_t oracle_rmsnorm(const float *x, const float *scale, float *out, size_t rows, size_t dim,
                       float eps);
/* The indexing work of the three forecasters, for the bit-exact tests: Chronos-2's instance norm
 * and context-patch features [time, value, mask] with patch validity (chronos2/forecaster.zig:
 * 94-143; feats (b, n_ctx, 3 ps), key_valid (b, n_ctx)); Chronos-Bolt's [value, mask] features and
 * validity with the REG slot (chronos_bolt/forecaster.zig:150-197; key_valid (b, n_patch + reg));
 * Timestral's window statistics, features, key validity and first observed patch per group
 * (timestral/model.zig:253-362; roles: one per row of a group, 0 target, 1 past, 2 known). */
int32_t oracle_chronos2_patch(const float *inputs, size_t b, size_t t_in, size_t context_length, size_t ps,
                              float tscale, int32_t arcsinh, float *loc, float *scale, float *feats,
                              uint8_t *key_valid);
int32_t oracle_bolt_patch(const float *inputs, size_t b, size_t t_in, size_t context_length, size_t ps,
                          int32_t use_reg, float *loc, float *scale, float *feats, uint8_t *key_valid);
int32_t oracle_timestral_block_inputs(const float *full, const uint8_t *full_obs, size_t rows, size_t w, size_t ps,
                                      size_t vall, const int8_t *roles, int32_t cov, double min_scale,
                                      int32_t use_asinh, int32_t attend_missing, float *loc, float *scale,
                                      float *feats, uint8_t *key_valid, int32_t *first_obs);

/* CSV output (oracle_csv.cpp): writeCsv of src/main.zig:181-198 and Zig's "{d}" rendering.
 * oracle_csv_format returns the text's length and fills out when capacity allows. */
void oracle_f32_digits(float x, uint32_t *digits, int32_t *exponent);
void oracle_f32_digits_search(float x, uint64_t *digits, int32_t *exponent);
void oracle_f32_digits_batch(const float *x, size_t n, uint32_t *digits, int32_t *exponent);
void oracle_f32_digits_search_batch(const float *x, size_t n, uint64_t *digits, int32_t *exponent);
size_t oracle_f32_text(float x, char *out);
size_t oracle_f64_text(double x, char *out);
size_t oracle_csv_format(const float *values, size_t series, size_t variates, size_t horizon,
                         const double *levels, size_t num_levels, char *out, size_t capacity);

#ifdef __cplusplus
}
#endif

#endif
