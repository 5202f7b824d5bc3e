// The model object behind the C ABI and the per-family device forwards.
#pragma once

#include <memory>
#include <vector>

#include "runtime.h"

namespace tsfm {

// Chronos-2 weights on one device (chronos2/model.zig:77-125).
struct C2Dev {
    DResBlock in_embed, out_embed;
    struct Layer {
        float *time_norm = nullptr, *group_norm = nullptr, *mlp_norm = nullptr;
        DLin qkv, o, gv, go, wi, wo;
    };
    std::vector<Layer> layers;
    float *final_norm = nullptr, *reg = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;  // [max_seq, 32]
    float *fut_emb = nullptr;                        // [max_output_patches, d]: shared future-patch embeddings
    int64_t max_seq = 0;
};

// Chronos-Bolt weights on one device (chronos_bolt/model.zig:101-172).
struct BoltDev {
    DResBlock in_embed, out_embed;
    struct Enc {
        float *attn_norm = nullptr, *ffn_norm = nullptr;
        DLin qkv, o, wi, wo;
    };
    struct Dec {
        float *self_norm = nullptr, *cross_norm = nullptr, *ffn_norm = nullptr;
        DLin self_vo, cross_q, cross_kv, cross_o, wi, wo;  // self_vo = o·v folded (one key)
        float *x_after_self = nullptr;  // decoder state after the token-only self-attention of layer 0
    };
    std::vector<Enc> enc;
    std::vector<Dec> dec;
    float *enc_final = nullptr, *dec_final = nullptr, *reg = nullptr, *start = nullptr;
    float *rel_bias = nullptr;  // [heads, 2 * max_seq - 1] by relative offset
    int64_t max_seq = 0;
};

struct tsfm_model_impl {
    tsfm_config cfg{};
    std::vector<double> quantiles;
    std::vector<int32_t> kinds;
    int compute = TSFM_COMPUTE_BF16;
    std::vector<std::unique_ptr<Replica>> reps;
    std::vector<std::unique_ptr<C2Dev>> c2;
    std::vector<std::unique_ptr<BoltDev>> bolt;
    uint64_t weight_bytes = 0;
};

Status c2_validate(const tsfm_config &c);
Status c2_check_tensors(const tsfm_config &c, const TensorTable &t);
Status c2_load(Replica &r, const tsfm_config &c, const TensorTable &t, C2Dev &w);
// Forecast b series of length t_in (device pointers) into out (b, horizon, Q).
Status c2_forward(Replica &r, const tsfm_config &c, const C2Dev &w, const float *d_in, int64_t b, int64_t t_in,
                  int64_t horizon, float *d_out, cudaStream_t s);
// Workspace bytes for a chunk of nb series.
size_t c2_workspace(const tsfm_config &c, int64_t nb, int64_t t_in, int64_t horizon);

}  // namespace tsfm

struct tsfm_model : tsfm::tsfm_model_impl {};
