// Persistent batch-1 decode engine: one cooperative kernel runs a whole
// generation (prefill token by token, then greedy decode) with one CTA per SM.
#pragma once

#include <cuda_bf16.h>

#include <string>
#include <vector>

#include "decode.cuh"
#include "lsx_internal.h"

namespace lsx {

class PersistentDecoder {
public:
    ~PersistentDecoder();
    static bool eligible(const FusedConfig& c, const lsx_ctx* ctx, std::string* why);
    int build(lsx_ctx* ctx, const FusedConfig& config, const std::vector<FusedLayer>& layers);
    // Runs up to `steps` decode steps under the state already uploaded to state().
    int run(int steps);
    DecodeState* state() const { return state_; }
    int slots() const { return slots_; }

private:
    lsx_ctx* ctx_ = nullptr;
    FusedConfig config_{};
    DecodeState* state_ = nullptr;
    void* layers_dev_ = nullptr;
    float2* rope_ = nullptr;
    unsigned long long *t_resid_ = nullptr, *t_qkv_ = nullptr, *t_attn_ = nullptr, *t_feat_ = nullptr,
                       *t_arg_ = nullptr, *t_part_ = nullptr;
    size_t smem_ = 0;
    int slots_ = 0;
    int inflight_ = 0;
    int inflight_layers_ = 0;
    int ns_ = 0, split_min_ = 0;  // split attention: slots per KV group, first position + 1
    int grid_ = 0;
    int layer_count_ = 0;
    std::vector<void*> owned_;
};

}  // namespace lsx
