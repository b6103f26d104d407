// Batched teacher-forced forward (batched.cu): equal-length cases through the
// decoder together, with tensor-core GEMMs per layer.
#pragma once

#include <string>
#include <vector>

#include "decode.cuh"
#include "lsx_internal.h"

namespace lsx {

class BatchedScorer {
public:
    // Host destinations of the scores, [cases, count] each ([cases, count, vocab]
    // for logits); any may be NULL.
    struct Outputs {
        double* nll = nullptr;
        uint32_t* argmax = nullptr;
        double* margin = nullptr;
        float* logits = nullptr;
    };
    ~BatchedScorer();
    static bool eligible(const FusedConfig& c, std::string* why);
    int build(lsx_ctx* ctx, const FusedConfig& config, const std::vector<FusedLayer>& layers);
    // tokens [cases, T] (host): each case's fed tokens.  Scores rows first ..
    // first + count - 1 of every case against targets [cases, count] (host),
    // through the edited readout when `rotation` is given.
    int score(const uint32_t* tokens, size_t cases, size_t T, size_t first, size_t count, const uint32_t* targets,
              const lsx_rotation* rotation, const Outputs& out);
    // The first n tokens of a generation (host) through the decoder at once: fills
    // positions 0 .. n-1 of the layers' KV caches as n decode steps would.
    int prefill(const uint32_t* tokens, size_t n);
    // Greedy decode of `batch` sequences together (prompts [batch, P] host, P >= 2):
    // the first P - 1 prompt tokens of every sequence in one batched forward into
    // per-sequence KV caches, then one row per sequence per step through the GEMMs and
    // an attention over each sequence's own cache; tokens_out [batch, maximum] (host).
    int generate_batch(const uint32_t* prompts, size_t batch, size_t P, size_t maximum, uint32_t* tokens_out);

private:
    struct Layout {
        size_t x, work, planes, logits, rope, tokens, targets, rows, nll, argmax, margin, status, total;
    };
    int reserve(size_t rows, size_t scored, size_t T);
    int run(const uint32_t* tokens, size_t cases, size_t T, size_t first, size_t count, const uint32_t* targets,
            const lsx_rotation* rotation, const Outputs& out, bool write_cache);
    // Per-sequence KV caches of generate_batch: per layer keys [batch, cap, kvheads *
    // head_dim] then values; run() writes prefill rows there while batch_keys_ is set.
    float* batch_cache_ = nullptr;
    size_t batch_cache_bytes_ = 0;
    float* batch_keys_ = nullptr;
    size_t batch_case_stride_ = 0, batch_layer_stride_ = 0;
    lsx_ctx* ctx_ = nullptr;
    FusedConfig config_{};
    std::vector<FusedLayer> layers_;
    void* block_ = nullptr;
    size_t capacity_ = 0;
    Layout layout_{};
};

}  // namespace lsx
