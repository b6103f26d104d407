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

private:
    struct Layout {
        size_t x, work, planes, logits, rope, tokens, targets, rows, nll, argmax, margin, status, total;
    };
    int reserve(size_t rows, size_t scored, size_t T);
    int run(const uint32_t* tokens, size_t cases, size_t T, size_t first, size_t count, const uint32_t* targets,
            const lsx_rotation* rotation, const Outputs& out, bool write_cache);
    lsx_ctx* ctx_ = nullptr;
    FusedConfig config_{};
    std::vector<FusedLayer> layers_;
    void* block_ = nullptr;
    size_t capacity_ = 0;
    Layout layout_{};
};

}  // namespace lsx
