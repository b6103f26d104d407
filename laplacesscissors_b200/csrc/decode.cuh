// Fused batch-1 decode engine: the B200 execution plan for Model::decode
// (src/model.rs:729-853) when the checkpoint has the common dense layout
// (bf16 projections, RMS norms, head_dim a multiple of 32).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include <vector>

#include "lsx_internal.h"

namespace lsx {

// Device-resident control block of the decode loop.  Kernels read the cursor and
// the token source from here, so one captured graph serves every step.
struct DecodeState {
    int position;       // cursor of the step being executed
    int step;           // step index within the current call
    int prompt_length;  // tokens taken from `prompt` before greedy argmax takes over
    int maximum;        // tokens to generate (src/diagnosis.rs:106-149)
    int mode;           // 0: token input, 1: injected residual (Model::inject)
    int stopped;        // set once generation is complete; later kernels return at once
    int generated;
    int nonfinite;      // any non-finite logit or hidden value (src/model.rs:845-848)
    int status;         // device error code (timeouts), 0 when healthy
    int frames;         // write per-token frames into hidden_frames/logits_frames
    int n_stop;
    int rot_kind;  // 0 none, 1 plane, 2 joint
    int rot_rank;
    int frame_back;     // frames start this many steps before the last prompt step (teacher forcing)
    uint32_t argmax;  // argmax of the latest logits
    uint32_t token;   // token consumed by the latest step
    unsigned int head_counter;
    unsigned int pad1;
    float rot_a, rot_b;
    const uint32_t* prompt;
    uint32_t* tokens_out;
    const float* inject;
    float* hidden_frames;
    float* logits_frames;
    float* hidden_scratch;
    float* logits_scratch;
    const float* rot_u;
    const float* rot_v;
    const float* rot_basis;  // [rank x hidden]
    const float* rot_delta;  // [rank x rank] = R - I
    uint32_t stop[16];
    unsigned int attn_counter[64];
    unsigned int epoch;  // last publication epoch of the persistent engine's tagged buffers
    unsigned int pad2;
    // Failure-path test hook of the persistent engine (0 in normal runs): CTA
    // hold_cta - 1 skips publishing its argmax partial at step hold_step, and every
    // exchange wait gives up after spin_limit clock cycles instead of about two
    // seconds, so the other CTAs' waits expire and the kernel records a status.
    int hold_cta;
    int hold_step;
    long long spin_limit;
};

struct FusedLayer {
    const __nv_bfloat16* wqkv;  // [(qheads + 2 kvheads) * head_dim, hidden]: q rows, k rows, v rows
    const __nv_bfloat16* wo;    // [hidden, qheads * head_dim]
    const __nv_bfloat16* wgu;   // [2 * intermediate, hidden]: gate_f, up_f interleaved
    const __nv_bfloat16* wd;    // [hidden, intermediate]
    const float *bqkv, *bo, *bgu, *bd;  // optional biases in the same row order
    const float *input_gain, *post_gain, *q_gain, *k_gain;
    float *keys, *values;  // f32 [capacity, kvheads * head_dim] as the reference keeps them
};

struct FusedConfig {
    int hidden, vocab, layers, qheads, kvheads, head_dim, intermediate, rotary, interleaved, activation;
    int capacity;
    float eps, qk_eps, scale, embedding_scale;
    double theta;
    const void* embedding;
    int embedding_kind;
    const __nv_bfloat16* head;
    const float* head_bias;
    const float* final_gain;
};

class FusedDecoder {
public:
    ~FusedDecoder();
    // Allocates work buffers and the RoPE table; validates the configuration.
    int build(lsx_ctx* ctx, const FusedConfig& config, const std::vector<FusedLayer>& layers);
    // Enqueues one decode step (embedding/inject -> layers -> head) on the stream;
    // uses a captured CUDA graph when available.
    int enqueue_step();
    // Enqueues `count` steps.
    int enqueue_steps(int count);
    DecodeState* state() const { return state_; }
    float* residual() const { return residual_; }
    bool supports_graph() const { return graph_exec_ != nullptr; }
    int kernels_per_step() const { return 2 + 5 * config_.layers; }
    static bool eligible(const FusedConfig& c, std::string* why);

private:
    int launch_all();
    int capture();
    lsx_ctx* ctx_ = nullptr;
    FusedConfig config_{};
    std::vector<FusedLayer> layers_;
    DecodeState* state_ = nullptr;
    float* residual_ = nullptr;
    float* qkv_ = nullptr;
    float* attn_partial_ = nullptr;
    float* attn_out_ = nullptr;
    float* feature_ = nullptr;
    float2* rope_ = nullptr;
    unsigned long long* head_partials_ = nullptr;
    int splits_ = 1;
    int grid_ = 148;
    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
    bool graph_tried_ = false;
    std::vector<void*> owned_;
};

}  // namespace lsx
