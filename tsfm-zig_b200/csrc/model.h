// The model object behind the C ABI and the per-family device forwards.
#pragma once

#include <memory>
#include <vector>

#include "runtime.h"

namespace tsfm {

// Chronos-2 weights on one device (chronos2/model.zig:77-125).
struct C2Dev {
    DResBlock in_embed;
    // The quantile head runs FP32-accurate (split TF32): its output passes through sinh, which
    // amplifies errors by cosh(v) at the tails.
    DLin3 head_hidden, head_output, head_residual;
    struct Layer {
        float *time_norm = nullptr, *group_norm = nullptr, *mlp_norm = nullptr;
        DLin qkv, o, gvo, wi, wo;  // gvo = W_o W_v of the singleton-group attention
    };
    std::vector<Layer> layers;
    float *final_norm = nullptr, *reg = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;  // [max_seq, 32]
    float *fut_emb = nullptr;                        // [max_output_patches, d]: shared future-patch embeddings
    int64_t max_seq = 0;
    int act = E_F16;  // element type of GEMM operands / 16-bit activations
    // Corrected products (TSFM_COMPUTE_F16C): every 16-bit weight carries its FP8 companion and
    // every 16-bit GEMM input is written with one.
    bool corr = false;
};

// Chronos-Bolt weights on one device (chronos_bolt/model.zig:101-172).
struct BoltDev {
    DResBlock in_embed;
    DLin3 head_hidden, head_output, head_residual;  // FP32-accurate quantile head
    struct Enc {
        float *attn_norm = nullptr, *ffn_norm = nullptr;
        DLin qkv, o, wi, wo;
    };
    struct Dec {
        float *self_norm = nullptr, *cross_norm = nullptr, *ffn_norm = nullptr;
        DLin self_v, self_o, cross_q, cross_kv, cross_o, wi, wo;
    };
    std::vector<Enc> enc;
    std::vector<Dec> dec;
    float *enc_final = nullptr, *dec_final = nullptr, *reg = nullptr, *start = nullptr;
    float *rel = nullptr;  // [heads, 2 * max_seq - 1]: bias by key - query offset (offset 0 at max_seq - 1)
    int64_t max_seq = 0;
    float *levels = nullptr;  // quantile levels (f32) for the long-horizon loop
    int act = E_F16;
};

// Timestral weights on one device (timestral/model.zig:26-70).
struct TsDev {
    DResBlock patch_proj;                           // 2P -> 4d (SiLU) -> d, with bias
    DLin3 head_hidden, head_output, head_residual;  // FP32-accurate quantile head, no bias
    float *fq_rep = nullptr;                        // forecast query replicated block_size times
    float *out_norm = nullptr, *inv_freq = nullptr, *widths = nullptr;
    struct Attn {
        bool is_time = true, gate = false;
        float *norm = nullptr;
        DLin qkvg;  // rows [q | k | v | gate]: q, k, v permuted to head-major; gate when enabled
        DLin o;
    };
    struct Layer {
        int n_attn = 1;
        Attn attns[2];
        float *mlp_norm = nullptr;
        DLin w12, w3;
        bool glu = false;  // w12 rows interleaved in 128-row [gate | up] blocks for the fused epilogue
    };
    std::vector<Layer> layers;
    int64_t max_qkv_cols = 0;
    int act = E_F16;
    bool corr = false;  // corrected products (TSFM_COMPUTE_F16C), as C2Dev::corr
    // Per-forecast roles of one series' rows (0 target, 1 past covariate, 2 known covariate).
    const int8_t *roles = nullptr;
};

struct tsfm_model_impl {
    tsfm_config cfg{};
    std::vector<double> quantiles;
    std::vector<int32_t> kinds;
    int compute = TSFM_COMPUTE_BF16;
    std::vector<std::unique_ptr<Replica>> reps;
    std::vector<std::unique_ptr<C2Dev>> c2;
    std::vector<std::unique_ptr<BoltDev>> bolt;
    std::vector<std::unique_ptr<TsDev>> ts;
    uint64_t weight_bytes = 0;
};

Status c2_validate(const tsfm_config &c);
Status c2_check_tensors(const tsfm_config &c, const TensorTable &t);
Status c2_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, C2Dev &w);
// Device forecast of b series (inputs/out on the device), chunked to fit the workspace budget.
Status c2_forecast(Replica &r, const tsfm_config &c, const C2Dev &w, const float *d_in, int64_t b, int64_t t_in,
                   int64_t horizon, float *d_out, cudaStream_t s);

// relativeBucket (chronos_bolt/model.zig:74-85): the bucket of key - query offset `rel`; the bias
// table of the Bolt encoder is built from it at load.
int64_t relative_bucket(int64_t rel, uint32_t num_buckets, uint32_t max_distance);
Status bolt_validate(const tsfm_config &c);
Status bolt_check_tensors(const tsfm_config &c, const TensorTable &t);
Status bolt_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, BoltDev &w);
Status bolt_forecast(Replica &r, const tsfm_config &c, const BoltDev &w, const float *d_in, int64_t b, int64_t t_in,
                     int64_t horizon, float *d_out, cudaStream_t s);

Status ts_validate(const tsfm_config &c);
Status ts_check_tensors(const tsfm_config &c, const TensorTable &t);
Status ts_load(Replica &r, const tsfm_config &c, const TensorTable &t, int act, TsDev &w);
// Host-memory forecast of b series with v target variates each: out is (b, v, horizon, q).
Status ts_forecast(Replica &r, const tsfm_config &c, TsDev &w, const float *inputs, const uint8_t *observed, size_t b,
                   size_t v, size_t t0, size_t horizon, const tsfm_covariates *cov, const tsfm_timestral_options &opts,
                   float *out);

// Bytes of device memory a forward may use for workspace (60 % of what is free plus the
// workspace already held).
size_t workspace_budget(Replica &r);

}  // namespace tsfm

struct tsfm_model : tsfm::tsfm_model_impl {};
