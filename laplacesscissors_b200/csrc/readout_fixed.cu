// Readout margin with fixed, statically placed scratch.
//
// Some callers cannot allocate device memory at the moment they validate: a host
// that has handed every byte of HBM to its own caching allocator, or code running
// where an allocation would be illegal or would stall other streams (a real-time
// serving loop that has already sized its memory).  lsx_readout_margin_device needs
// a caller-provided workspace; this variant instead uses one scratch area that is
// part of the library's own device image, so it makes no allocation at all.
//
// Limits and rules of use:
//  - The scratch is kReadoutFixedScratch bytes per device.  A call whose working
//    set (per-row best-other keys and target logits, plus the bf16 hi/lo split of
//    F32 hidden states) exceeds it is rejected with LSX_E_ARGUMENT before anything
//    is enqueued.
//  - Nothing in the scratch has to start at zero: every call's first kernel writes
//    each word the later kernels read, the two status words included.
//  - The scratch is shared by every call on the same device.  Two calls whose work
//    can overlap on the GPU (different streams or contexts of one device, without
//    ordering between them) race on it and give wrong results; serialise them.
//  - The kernels' status words (a device wait that gave up, non-finite scores) stay
//    in the scratch until the next call on the device: lsx_readout_status(ctx, NULL)
//    waits for the context's stream and reports them.
//  - The first call on each device looks up the scratch's device address, which
//    may make the CUDA runtime load this module onto that device.  Make the first
//    call on each device before any stream capture begins and before any section
//    of the program that must not trigger such setup.
//  - The edit (rotation) path is not available here: it stages host-side edit
//    factors and builds a vocab-sized extension, which does not fit the scratch.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "lsx_internal.h"

namespace lsx {

int readout_margin_enqueue(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab, size_t width,
                           const void* hidden, int hidden_kind, size_t rows, const uint32_t* targets,
                           const lsx_rotation* rotation, double* margin, uint32_t* argmax, float* target_logit,
                           void* workspace, size_t workspace_bytes, int* host_status);
size_t readout_workspace_need(size_t vocab, size_t width, size_t rows, size_t rank, bool f32_hidden);

namespace {

constexpr size_t kReadoutFixedScratch = size_t(4) << 20;  // 4 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char readout_fixed_scratch[kReadoutFixedScratch];

std::mutex g_scratch_mutex;
void* g_scratch[kMaxDevices] = {};

// Device address of the scratch on the current device (`device`), looked up once.
int scratch_for(int device, void** out) {
    LSX_ENSURE(device >= 0 && device < kMaxDevices, "device ordinal out of range for the fixed scratch");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch[device]) {
        void* p = nullptr;
        LSX_CUDA(cudaGetSymbolAddress(&p, readout_fixed_scratch), "fixed readout scratch lookup");
        LSX_ENSURE(p && (uintptr_t)p % 256 == 0, "fixed readout scratch is not 256-byte aligned");
        g_scratch[device] = p;
    }
    *out = g_scratch[device];
    return LSX_OK;
}

}  // namespace

// Device address of this device's fixed scratch (the status words sit at its start).
int fixed_scratch_address(lsx_ctx* ctx, void** out) {
    LSX_CUDA(cudaSetDevice(ctx->device), "select device");
    return scratch_for(ctx->device, out);
}

}  // namespace lsx

using namespace lsx;

extern "C" {

int lsx_readout_margin_fixed(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab,
                             size_t width, const void* hidden, lsx_dtype hidden_kind, size_t rows,
                             const uint32_t* targets, double* margin_out, uint32_t* argmax_out,
                             float* target_logit_out) {
    LSX_ENSURE(ctx && weight && hidden && targets, "invalid argument");
    LSX_ENSURE(hidden_kind == LSX_F32 || hidden_kind == LSX_BF16, "hidden states are F32 or BF16");
    // The checks readout_enqueue makes, here before the scratch size is computed
    // from these sizes, so that no product below can wrap.
    LSX_ENSURE(weight->kind == LSX_BF16, "the readout weight must be a BF16 tensor");
    LSX_ENSURE(rows > 0 && rows <= 2147483647ull && vocab > 1 && vocab <= 2147483647ull, "check the row count");
    LSX_ENSURE(width > 0 && width % 8 == 0, "the readout width must be a multiple of 8");
    size_t cells = 0, plane_bytes = 0;
    LSX_ENSURE(!__builtin_mul_overflow(vocab, width, &cells) && weight->count == cells,
               "check the readout weight dimensions");
    LSX_ENSURE(!__builtin_mul_overflow(rows, width, &cells) && !__builtin_mul_overflow(cells, (size_t)4, &plane_bytes),
               "check the row count");
    const size_t need = readout_workspace_need(vocab, width, rows, 0, hidden_kind == LSX_F32);
    if (need > kReadoutFixedScratch)
        return fail(LSX_E_ARGUMENT, "lsx_readout_margin_fixed needs " + std::to_string(need) +
                                        " scratch bytes for these sizes; its fixed scratch holds " +
                                        std::to_string(kReadoutFixedScratch) +
                                        " (use lsx_readout_margin_device with a workspace)");
    LSX_CUDA(cudaSetDevice(ctx->device), "select device");
    void* scratch = nullptr;
    LSX_TRY(scratch_for(ctx->device, &scratch));
    return readout_margin_enqueue(ctx, weight, bias, vocab, width, hidden, hidden_kind, rows, targets, nullptr,
                                  margin_out, argmax_out, target_logit_out, scratch, kReadoutFixedScratch, nullptr);
}

}  // extern "C"
