// Context, caching pool, tensors and error reporting of liblsx.
// Replaces the reference's Device layer (src/device.rs) and Tensor ownership
// (src/gpu.rs:55-76, 204-247) with the CUDA runtime on one stream per context.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cstring>
#include <string>

#include "lsx_internal.h"

namespace lsx {

static thread_local std::string g_last_error;

int fail(int status, const std::string& message) {
    g_last_error = message;
    return status;
}
void clear_error() { g_last_error.clear(); }

std::string cuda_message(const char* what, cudaError_t error) {
    return std::string(what) + ": " + cudaGetErrorName(error) + " (" + cudaGetErrorString(error) + ")";
}

Pool::~Pool() { trim(); }

int Pool::allocate(size_t bytes, void** out) {
    size_t rounded = (bytes + 511) & ~size_t(511);
    if (rounded == 0) rounded = 512;
    auto it = free_.lower_bound(rounded);
    if (it != free_.end() && it->first <= rounded * 2) {
        *out = it->second;
        cached_ -= it->first;
        free_.erase(it);
        return LSX_OK;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, rounded);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        trim();
        e = cudaMalloc(&p, rounded);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            return fail(LSX_E_MEMORY, "device allocation of " + std::to_string(rounded) + " bytes failed");
        }
    }
    sizes_[p] = rounded;
    *out = p;
    return LSX_OK;
}

void Pool::release(void* pointer) {
    if (!pointer) return;
    auto it = sizes_.find(pointer);
    if (it == sizes_.end()) return;
    free_.emplace(it->second, pointer);
    cached_ += it->second;
}

void Pool::trim() {
    int previous = 0;
    cudaGetDevice(&previous);
    cudaSetDevice(device_);
    for (auto& kv : free_) {
        cudaFree(kv.second);
        sizes_.erase(kv.second);
    }
    free_.clear();
    cached_ = 0;
    cudaSetDevice(previous);
}

int device_alloc(lsx_ctx* ctx, size_t bytes, void** out) { return ctx->pool->allocate(bytes, out); }
void device_release(lsx_ctx* ctx, void* p) { ctx->pool->release(p); }

int reserve(lsx_ctx* ctx, size_t count, lsx_dtype kind, lsx_tensor** out) {
    LSX_ENSURE(count > 0 && count <= 2147483647ull, "buffer element count must be in 1..=i32::MAX");
    void* p = nullptr;
    LSX_TRY(ctx->pool->allocate(count * dtype_bytes(kind), &p));
    lsx_tensor* t = new lsx_tensor;
    t->ctx = ctx;
    t->data = p;
    t->count = count;
    t->kind = kind;
    t->owned = true;
    ctx->refs += 1;
    *out = t;
    return LSX_OK;
}

static void release_context(lsx_ctx* ctx) {
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    delete ctx->pool;
    if (ctx->pinned) cudaFreeHost(ctx->pinned);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
}

}  // namespace lsx

int lsx_ctx::staging(size_t bytes, void** out) {
    if (bytes > pinned_bytes) {
        if (pinned) cudaFreeHost(pinned);
        pinned = nullptr;
        pinned_bytes = 0;
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        LSX_CUDA(cudaHostAlloc(&pinned, want, cudaHostAllocDefault), "pinned staging allocation");
        pinned_bytes = want;
    }
    *out = pinned;
    return LSX_OK;
}

namespace lsx {
namespace {

constexpr size_t kStageChunk = size_t(4) << 20;  // bytes per staged piece (two in flight)

// memcpy with the host's threads (pageable source or destination, pinned other side).
void parallel_copy(void* dst, const void* src, size_t bytes) {
    constexpr size_t kPiece = size_t(256) << 10;
    const long long pieces = (long long)((bytes + kPiece - 1) / kPiece);
#pragma omp parallel for schedule(static) if (pieces > 1)
    for (long long i = 0; i < pieces; ++i) {
        const size_t off = (size_t)i * kPiece;
        std::memcpy((uint8_t*)dst + off, (const uint8_t*)src + off, std::min(kPiece, bytes - off));
    }
}

}  // namespace

int staged_upload(lsx_ctx* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes < 2 * kStageChunk) {
        LSX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "host to device copy");
        return LSX_OK;
    }
    void* pin = nullptr;
    LSX_TRY(ctx->staging(2 * kStageChunk, &pin));
    cudaEvent_t done[2];
    LSX_CUDA(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming), "staging event");
    LSX_CUDA(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming), "staging event");
    cudaError_t e = cudaSuccess;
    size_t i = 0;
    for (size_t off = 0; off < bytes && e == cudaSuccess; off += kStageChunk, ++i) {
        const size_t len = std::min(kStageChunk, bytes - off);
        uint8_t* half = (uint8_t*)pin + (i & 1) * kStageChunk;
        if (i >= 2) e = cudaEventSynchronize(done[i & 1]);  // that half's previous copy has left it
        if (e != cudaSuccess) break;
        parallel_copy(half, (const uint8_t*)src + off, len);
        e = cudaMemcpyAsync((uint8_t*)dst + off, half, len, cudaMemcpyHostToDevice, ctx->stream);
        if (e == cudaSuccess) e = cudaEventRecord(done[i & 1], ctx->stream);
    }
    // the staging buffer is free again once the last copies have left it
    if (e == cudaSuccess) e = cudaEventSynchronize(done[(i - 1) & 1]);
    if (e == cudaSuccess && i >= 2) e = cudaEventSynchronize(done[i & 1]);
    cudaEventDestroy(done[0]);
    cudaEventDestroy(done[1]);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("staged host to device copy", e));
    return LSX_OK;
}

int staged_download(lsx_ctx* ctx, void* dst, const void* src, size_t bytes) {
    if (bytes < 2 * kStageChunk) {
        LSX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "device to host copy");
        LSX_CUDA(cudaStreamSynchronize(ctx->stream), "device to host copy");
        return LSX_OK;
    }
    void* pin = nullptr;
    LSX_TRY(ctx->staging(2 * kStageChunk, &pin));
    cudaEvent_t done[2];
    LSX_CUDA(cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming), "staging event");
    LSX_CUDA(cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming), "staging event");
    const size_t n = (bytes + kStageChunk - 1) / kStageChunk;
    auto issue = [&](size_t i) {
        const size_t off = i * kStageChunk, len = std::min(kStageChunk, bytes - off);
        cudaError_t r = cudaMemcpyAsync((uint8_t*)pin + (i & 1) * kStageChunk, (const uint8_t*)src + off, len,
                                        cudaMemcpyDeviceToHost, ctx->stream);
        return r == cudaSuccess ? cudaEventRecord(done[i & 1], ctx->stream) : r;
    };
    cudaError_t e = issue(0);
    for (size_t i = 0; i < n && e == cudaSuccess; ++i) {
        if (i + 1 < n) e = issue(i + 1);  // the next piece lands while this one is copied out
        if (e == cudaSuccess) e = cudaEventSynchronize(done[i & 1]);
        if (e != cudaSuccess) break;
        const size_t off = i * kStageChunk;
        parallel_copy((uint8_t*)dst + off, (uint8_t*)pin + (i & 1) * kStageChunk, std::min(kStageChunk, bytes - off));
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaEventDestroy(done[0]);
    cudaEventDestroy(done[1]);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("staged device to host copy", e));
    return LSX_OK;
}

}  // namespace lsx

using namespace lsx;

extern "C" {

const char* lsx_last_error(void) { return g_last_error.c_str(); }
const char* lsx_version(void) { return "liblsx 0.1.0 (sm_100a)"; }

int lsx_ctx_create(int device, lsx_ctx** out) {
    LSX_ENSURE(out != nullptr, "output pointer is NULL");
    int count = 0;
    LSX_CUDA(cudaGetDeviceCount(&count), "CUDA device count");
    LSX_ENSURE(device >= 0 && device < count, "device ordinal out of range");
    LSX_CUDA(cudaSetDevice(device), "select device");
    cudaDeviceProp prop;
    LSX_CUDA(cudaGetDeviceProperties(&prop, device), "device properties");
    if (prop.major != 10)
        return fail(LSX_E_UNSUPPORTED, std::string("this build targets sm_100a (B200); device is ") +
                                           prop.name + " cc " + std::to_string(prop.major) + "." +
                                           std::to_string(prop.minor));
    lsx_ctx* c = new lsx_ctx;
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    c->architecture = prop.major * 10 + prop.minor;
    c->smem_optin = prop.sharedMemPerBlockOptin;
    c->name = prop.name;
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return fail(LSX_E_CUDA, cuda_message("stream creation", e));
    }
    c->pool = new Pool(device);
    *out = c;
    return LSX_OK;
}

int lsx_ctx_destroy(lsx_ctx* ctx) {
    if (!ctx || ctx->destroyed) return LSX_OK;
    ctx->destroyed = true;
    if (ctx->refs == 0) release_context(ctx);
    return LSX_OK;
}

int lsx_ctx_synchronize(lsx_ctx* ctx) {
    LSX_ENSURE(ctx, "context is NULL");
    LSX_CUDA(cudaStreamSynchronize(ctx->stream), "device synchronize");
    return LSX_OK;
}

int lsx_ctx_name(lsx_ctx* ctx, char* buffer, size_t length) {
    LSX_ENSURE(ctx && buffer && length > 0, "invalid name buffer");
    snprintf(buffer, length, "%s", ctx->name.c_str());
    return LSX_OK;
}

int lsx_ctx_architecture(lsx_ctx* ctx, int* architecture) {
    LSX_ENSURE(ctx && architecture, "invalid argument");
    *architecture = ctx->architecture;
    return LSX_OK;
}

int lsx_ctx_stream(lsx_ctx* ctx, void** stream) {
    LSX_ENSURE(ctx && stream, "invalid argument");
    *stream = (void*)ctx->stream;
    return LSX_OK;
}

int lsx_upload_raw(lsx_ctx* ctx, const void* data, size_t bytes, lsx_dtype kind, lsx_tensor** out) {
    LSX_ENSURE(ctx && out && (data || bytes == 0), "invalid argument");
    LSX_ENSURE(kind == LSX_F32 || kind == LSX_F16 || kind == LSX_BF16, "unknown storage kind");
    LSX_ENSURE(bytes > 0 && bytes % dtype_bytes(kind) == 0,
               "weight storage kind and byte size do not agree");
    cudaSetDevice(ctx->device);
    lsx_tensor* t = nullptr;
    LSX_TRY(reserve(ctx, bytes / dtype_bytes(kind), kind, &t));
    cudaError_t e = cudaMemcpyAsync(t->data, data, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        lsx_tensor_free(t);
        return fail(LSX_E_CUDA, cuda_message("host to device copy", e));
    }
    *out = t;
    return LSX_OK;
}

int lsx_upload_f32(lsx_ctx* ctx, const float* data, size_t count, lsx_tensor** out) {
    return lsx_upload_raw(ctx, data, count * 4, LSX_F32, out);
}

int lsx_zeros(lsx_ctx* ctx, size_t count, lsx_tensor** out) {
    LSX_ENSURE(ctx && out, "invalid argument");
    cudaSetDevice(ctx->device);
    lsx_tensor* t = nullptr;
    LSX_TRY(reserve(ctx, count, LSX_F32, &t));
    cudaError_t e = cudaMemsetAsync(t->data, 0, count * 4, ctx->stream);
    if (e != cudaSuccess) {
        lsx_tensor_free(t);
        return fail(LSX_E_CUDA, cuda_message("zero fill", e));
    }
    *out = t;
    return LSX_OK;
}

int lsx_read(lsx_ctx* ctx, const lsx_tensor* tensor, float* out, size_t count) {
    LSX_ENSURE(ctx && tensor && out, "invalid argument");
    LSX_ENSURE(tensor->kind == LSX_F32, "an F32 result buffer is required");
    LSX_ENSURE(count == tensor->count, "read length does not match the tensor");
    cudaSetDevice(ctx->device);
    size_t bytes = count * 4;
    if (bytes <= (64u << 20)) {
        void* stage = nullptr;
        LSX_TRY(ctx->staging(bytes, &stage));
        LSX_CUDA(cudaMemcpyAsync(stage, tensor->data, bytes, cudaMemcpyDeviceToHost, ctx->stream),
                 "device to host copy");
        LSX_CUDA(cudaStreamSynchronize(ctx->stream), "device to host copy");
        memcpy(out, stage, bytes);
    } else {
        LSX_CUDA(cudaMemcpyAsync(out, tensor->data, bytes, cudaMemcpyDeviceToHost, ctx->stream),
                 "device to host copy");
        LSX_CUDA(cudaStreamSynchronize(ctx->stream), "device to host copy");
    }
    return LSX_OK;
}

int lsx_tensor_free(lsx_tensor* tensor) {
    if (!tensor) return LSX_OK;
    lsx_ctx* ctx = tensor->ctx;
    if (tensor->owned && tensor->data) device_release(ctx, tensor->data);
    delete tensor;
    if (ctx && --ctx->refs == 0 && ctx->destroyed) release_context(ctx);
    return LSX_OK;
}

size_t lsx_tensor_len(const lsx_tensor* tensor) { return tensor ? tensor->count : 0; }
int lsx_tensor_dtype(const lsx_tensor* tensor) { return tensor ? (int)tensor->kind : -1; }
void* lsx_tensor_data(const lsx_tensor* tensor) { return tensor ? tensor->data : nullptr; }

int lsx_tensor_wrap(lsx_ctx* ctx, void* device_pointer, size_t count, lsx_dtype kind, lsx_tensor** out) {
    LSX_ENSURE(ctx && out && device_pointer, "invalid argument");
    LSX_ENSURE(kind == LSX_F32 || kind == LSX_F16 || kind == LSX_BF16, "unknown storage kind");
    LSX_ENSURE(count > 0 && count <= 2147483647ull, "buffer element count must be in 1..=i32::MAX");
    lsx_tensor* t = new lsx_tensor;
    t->ctx = ctx;
    t->data = device_pointer;
    t->count = count;
    t->kind = kind;
    t->owned = false;
    ctx->refs += 1;
    *out = t;
    return LSX_OK;
}

}  // extern "C"
