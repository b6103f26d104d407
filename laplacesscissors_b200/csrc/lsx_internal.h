// Internal declarations shared by the CUDA/C++ sources of liblsx.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "lsx.h"

namespace lsx {

// Records `message` as this thread's last error and returns `status`.
int fail(int status, const std::string& message);
void clear_error();
std::string cuda_message(const char* what, cudaError_t error);

#define LSX_ENSURE(cond, msg)                                              \
    do {                                                                   \
        if (!(cond)) return ::lsx::fail(LSX_E_ARGUMENT, (msg));            \
    } while (0)
#define LSX_CUDA(call, what)                                               \
    do {                                                                   \
        cudaError_t lsx_e_ = (call);                                       \
        if (lsx_e_ != cudaSuccess)                                         \
            return ::lsx::fail(LSX_E_CUDA, ::lsx::cuda_message((what), lsx_e_)); \
    } while (0)
#define LSX_TRY(call)                                                      \
    do {                                                                   \
        int lsx_s_ = (call);                                               \
        if (lsx_s_ != LSX_OK) return lsx_s_;                               \
    } while (0)

inline size_t dtype_bytes(int kind) { return kind == LSX_F32 ? 4 : 2; }

// Caching device allocator: blocks are kept on release and reused by size, so
// steady-state op sequences make no cudaMalloc/cudaFree calls (the reference
// allocates and frees one buffer per op, src/gpu.rs:204-216).
class Pool {
public:
    explicit Pool(int device) : device_(device) {}
    ~Pool();
    int allocate(size_t bytes, void** out);
    void release(void* pointer);
    void trim();
    size_t cached_bytes() const { return cached_; }

private:
    int device_;
    std::multimap<size_t, void*> free_;
    std::map<void*, size_t> sizes_;
    size_t cached_ = 0;
};

}  // namespace lsx

struct lsx_ctx {
    int device = 0;
    int sm_count = 0;
    int architecture = 0;
    size_t smem_optin = 0;
    std::string name;
    cudaStream_t stream = nullptr;
    lsx::Pool* pool = nullptr;
    // Pinned host staging for synchronous reads of large tensors.
    void* pinned = nullptr;
    size_t pinned_bytes = 0;
    int staging(size_t bytes, void** out);
    // Live tensors keep the context: lsx_ctx_destroy defers the release until the
    // last tensor is freed, so destruction order does not matter to callers.
    int refs = 0;
    bool destroyed = false;
};

struct lsx_tensor {
    lsx_ctx* ctx = nullptr;
    void* data = nullptr;
    size_t count = 0;
    lsx_dtype kind = LSX_F32;
    bool owned = true;
};

namespace lsx {

// Allocates an owned tensor from the context pool (Gpu::reserve, src/gpu.rs:204-216:
// 1..=i32::MAX elements).
int reserve(lsx_ctx* ctx, size_t count, lsx_dtype kind, lsx_tensor** out);
int device_alloc(lsx_ctx* ctx, size_t bytes, void** out);
void device_release(lsx_ctx* ctx, void* p);

// ---- kernel launchers (ops.cu) ----
cudaError_t launch_take_row(cudaStream_t s, const void* w, int kind, size_t row, size_t width, float* out);
// `stable_weight`: no kernel writes w (it was uploaded from the host), so a large
// GEMV may start streaming it while the preceding kernel on the stream still runs.
cudaError_t launch_matvec(cudaStream_t s, int sm_count, const void* w, int kind, const float* x,
                          const float* bias, size_t rows, size_t cols, float* out, bool stable_weight = false);
cudaError_t launch_norm(cudaStream_t s, const float* x, const float* gain, const float* bias,
                        size_t groups, size_t width, float eps, int center, float* out);
cudaError_t launch_rope(cudaStream_t s, const float* x, size_t position, size_t heads, size_t dim,
                        float theta, size_t rotary, int interleaved, float* out);
cudaError_t launch_cache_write(cudaStream_t s, const float* k, const float* v, float* keys,
                               float* values, size_t position, size_t width);
cudaError_t launch_attention(cudaStream_t s, const float* q, const float* keys, const float* values,
                             size_t position, size_t qheads, size_t kvheads, size_t dim, float scale,
                             float* out);
cudaError_t launch_gated(cudaStream_t s, const float* gate, const float* up, size_t n, int kind, float* out);
cudaError_t launch_combine(cudaStream_t s, const float* x, const float* y, float factor, size_t n, float* out);
cudaError_t launch_rotate(cudaStream_t s, const float* h, const float* u, const float* v, float a, float b,
                          size_t width, float* out);
cudaError_t launch_all_finite(cudaStream_t s, const float* x, size_t n, int* flag);

// ---- large host <-> device copies through the context's pinned staging (runtime.cu) ----
// staged_upload: enqueued on ctx->stream; returns once the host data has been
// consumed.  staged_download: returns once the host holds the data (synchronises
// ctx->stream).  Copies below 8 MiB go directly.
int staged_upload(lsx_ctx* ctx, void* dst, const void* src, size_t bytes);
int staged_download(lsx_ctx* ctx, void* dst, const void* src, size_t bytes);

// ---- head images on the tensor cores (readout.cu) ----
size_t head_images_scratch(size_t count, size_t width);
int head_images_enqueue(lsx_ctx* ctx, const lsx_tensor* weight, size_t vocab, size_t width, const float* dirs_host,
                        size_t count, float* out, void* scratch);

}  // namespace lsx

// Rotation kept on the device in the form DeviceRotation uses (src/model.rs:285-299),
// plus the f64 host copy the fused readout needs to build its rank-r correction.
struct lsx_rotation {
    lsx_ctx* ctx = nullptr;
    bool joint = false;
    size_t width = 0, rank = 0;
    // Plane: u, v (f32 device), coefficients.
    lsx_tensor* u = nullptr;
    lsx_tensor* v = nullptr;
    float cosine_minus_one = 0.f, sine = 0.f;
    // Joint: basis [rank x width], transpose [width x rank], delta = R - I [rank x rank].
    // A plane also carries basis = [u; v] and delta = R - I (2 x 2), which the fused
    // readout reads from the device for its rank-r correction.
    lsx_tensor* basis = nullptr;
    lsx_tensor* transpose = nullptr;
    lsx_tensor* delta = nullptr;
    // Host f64 copies: rows of the edit's basis and (R - I), as SubspaceRotation holds them
    // (a plane is the rank-2 subspace of ReadoutEdit::subspace, src/response.rs:240-251).
    std::vector<double> basis64, delta64;
};
