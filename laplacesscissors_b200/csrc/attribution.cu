// Attribution of a readout edit's loss change to vocabulary rows
// (src/attribution.rs:49-123): the straight chord z(t) = (1 - t) before + t after
// between a point's logits before and after the edit, the softmax along it
// integrated by Simpson's rule over `panels` panels, and per vocabulary row j
//     integral_j = sum_k w_k (softmax(z(t_k))_j - [j == target])
//     credit_j  -= weight (after_j - before_j) integral_j      (summed over points)
// The reference evaluates (panels + 1) softmaxes over the vocabulary per point in
// f64 on one host core.  Here, in f64 with the reference's operation order:
//   chord_stats_kernel   per (point, panel node) the maximum and the sum of
//                        exponentials, as partials of 32 x kEntries entries per warp;
//   chord_merge_kernel   merges the partials (in partial order) per (point, node);
//   chord_credit_kernel  one thread per vocabulary row: every point in order, every
//                        node in order, so each credit accumulates as the reference's;
//   chord_gradient_kernel integral_j of chosen rows per point;
//   restored_loss_kernel  src/attribution.rs:61-78 for chosen rows, and the plain
//                        loss (src/attribution.rs:49-60) of before and after.
// exp and log are CUDA's f64 functions; sums over the vocabulary are reassociated
// (partials), so results agree with the reference to rounding, not bit for bit.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "lsx_internal.h"

namespace lsx {
namespace {

constexpr int kEntries = 8;                  // vocabulary entries per lane in chord_stats_kernel
constexpr int kWarpSpan = 32 * kEntries;     // entries per warp partial
constexpr size_t kStatsBatch = 256;          // points per partial-statistics pass

__device__ __forceinline__ double chord(float b, float a, double t) {
    // f64::from(before) * (1. - t) + f64::from(after) * t, without contraction
    return __dadd_rn(__dmul_rn((double)b, __dsub_rn(1.0, t)), __dmul_rn((double)a, t));
}

__device__ __forceinline__ double node_weight(int k, int panels) {
    const double c = (k == 0 || k == panels) ? 1.0 : ((k % 2 == 0) ? 2.0 : 4.0);
    return __ddiv_rn(c, __dmul_rn(3.0, (double)panels));
}

__device__ __forceinline__ double node_t(int k, int panels) { return __ddiv_rn((double)k, (double)panels); }

// grid (warp-partials / 8, points), 256 threads: partial (max, sum exp(z - max)) of
// each warp's kWarpSpan entries for every node k.
__global__ void __launch_bounds__(256) chord_stats_kernel(const float* __restrict__ before,
                                                           const float* __restrict__ after, int vocab, int panels,
                                                           int parts, double2* __restrict__ partial) {
    const int p = blockIdx.y;
    const int warp_global = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (warp_global >= parts) return;
    const float* b = before + (size_t)p * vocab;
    const float* a = after + (size_t)p * vocab;
    float bv[kEntries], av[kEntries];
    const int j0 = warp_global * kWarpSpan;
#pragma unroll
    for (int e = 0; e < kEntries; ++e) {
        const int j = j0 + e * 32 + lane;
        bv[e] = j < vocab ? b[j] : 0.f;
        av[e] = j < vocab ? a[j] : 0.f;
    }
    for (int k = 0; k <= panels; ++k) {
        const double t = node_t(k, panels);
        double m = -INFINITY;
#pragma unroll
        for (int e = 0; e < kEntries; ++e)
            if (j0 + e * 32 + lane < vocab) m = fmax(m, chord(bv[e], av[e], t));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        double s = 0.0;
#pragma unroll
        for (int e = 0; e < kEntries; ++e)
            if (j0 + e * 32 + lane < vocab) s += exp(chord(bv[e], av[e], t) - m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) partial[((size_t)p * (panels + 1) + k) * parts + warp_global] = make_double2(m, s);
    }
}

// One thread per (point, node): maximum over the partials, then their sums rescaled.
__global__ void chord_merge_kernel(const double2* __restrict__ partial, int points, int panels, int parts,
                                   double2* __restrict__ stats) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= points * (panels + 1)) return;
    const double2* q = partial + (size_t)i * parts;
    double m = -INFINITY;
    for (int c = 0; c < parts; ++c) m = fmax(m, q[c].x);
    double s = 0.0;
    for (int c = 0; c < parts; ++c) s += q[c].y * exp(q[c].x - m);
    stats[i] = make_double2(m, s);
}

__device__ __forceinline__ double integral_at(const float* __restrict__ before, const float* __restrict__ after,
                                              const double2* __restrict__ stats, int vocab, int panels, int p, int j,
                                              uint32_t target) {
    const float bj = before[(size_t)p * vocab + j], aj = after[(size_t)p * vocab + j];
    const double2* st = stats + (size_t)p * (panels + 1);
    const double delta = (uint32_t)j == target ? 1.0 : 0.0;
    double integral = 0.0;
    for (int k = 0; k <= panels; ++k) {
        const double t = node_t(k, panels);
        const double2 mk = st[k];
        const double pr = exp(chord(bj, aj, t) - mk.x);
        integral = __dadd_rn(integral, __dmul_rn(node_weight(k, panels), __dsub_rn(__ddiv_rn(pr, mk.y), delta)));
    }
    return integral;
}

// One thread per vocabulary row: credits[j] = -sum over points (in order) of
// weight (after_j - before_j) integral_j.
__global__ void __launch_bounds__(256) chord_credit_kernel(const float* __restrict__ before,
                                                            const float* __restrict__ after,
                                                            const uint32_t* __restrict__ targets,
                                                            const double* __restrict__ weights,
                                                            const double2* __restrict__ stats, int vocab, int points,
                                                            int panels, double* __restrict__ credits) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= vocab) return;
    double credit = 0.0;
    for (int p = 0; p < points; ++p) {
        const double integral = integral_at(before, after, stats, vocab, panels, p, j, targets[p]);
        const double change = __dsub_rn((double)after[(size_t)p * vocab + j], (double)before[(size_t)p * vocab + j]);
        credit = __dsub_rn(credit, __dmul_rn(__dmul_rn(weights[p], change), integral));
    }
    credits[j] = credit;
}

// gradients[p, r] = integral_{rows[r]} of point p.
__global__ void chord_gradient_kernel(const float* __restrict__ before, const float* __restrict__ after,
                                      const uint32_t* __restrict__ targets, const double2* __restrict__ stats,
                                      const uint32_t* __restrict__ rows, int row_count, int vocab, int points,
                                      int panels, double* __restrict__ gradients) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= points * row_count) return;
    const int p = i / row_count, r = i - p * row_count;
    gradients[i] = integral_at(before, after, stats, vocab, panels, p, (int)rows[r], targets[p]);
}

// Block per (point, slot): slot 0 loss(before), slot 1 loss(after), slot 2 + r
// restored_loss(after, rows[r], before[rows[r]], target).  f64 max, then the sum of
// exponentials, then max + ln(sum) - z[target].
__global__ void __launch_bounds__(512) restored_loss_kernel(const float* __restrict__ before,
                                                            const float* __restrict__ after,
                                                            const uint32_t* __restrict__ targets,
                                                            const uint32_t* __restrict__ rows, int vocab,
                                                            double* __restrict__ out, int slots) {
    __shared__ double red[16];
    const int p = blockIdx.y, slot = blockIdx.x;
    const float* z = (slot == 0 ? before : after) + (size_t)p * vocab;
    const int row = slot >= 2 ? (int)rows[slot - 2] : -1;
    const float replaced = row >= 0 ? before[(size_t)p * vocab + row] : 0.f;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto value = [&](int j) -> double { return (double)(j == row ? replaced : z[j]); };
    double top = -INFINITY;
    for (int j = tid; j < vocab; j += blockDim.x) top = fmax(top, value(j));
    for (int o = 16; o > 0; o >>= 1) top = fmax(top, __shfl_xor_sync(0xffffffffu, top, o));
    if (lane == 0) red[warp] = top;
    __syncthreads();
    top = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) top = fmax(top, red[w]);
    __syncthreads();
    double sum = 0.0;
    for (int j = tid; j < vocab; j += blockDim.x) sum += exp(value(j) - top);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        double total = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += red[w];
        out[(size_t)p * slots + slot] = top + log(total) - value((int)targets[p]);
    }
}

}  // namespace
}  // namespace lsx

using namespace lsx;

extern "C" {

int lsx_integrated_credits(lsx_ctx* ctx, const float* before, const float* after, const uint32_t* targets,
                           const double* weights, size_t points, size_t vocab, size_t panels, double* credits_out,
                           const uint32_t* rows, size_t row_count, double* gradients_out, double* losses_out) {
    LSX_ENSURE(ctx && before && after && targets && weights && credits_out, "invalid argument");
    LSX_ENSURE(points > 0 && points <= 2147483647ull && vocab > 0 && vocab <= 2147483647ull,
               "check the attribution sizes");
    LSX_ENSURE(panels >= 2 && panels % 2 == 0 && panels <= 65536, "Simpson's rule needs an even panel count");
    LSX_ENSURE(row_count == 0 || rows, "invalid argument");
    for (size_t p = 0; p < points; ++p) {
        LSX_ENSURE(targets[p] < vocab, "check the attribution observation conditions");
        LSX_ENSURE(std::isfinite(weights[p]) && weights[p] >= 0.0, "check the attribution observation conditions");
    }
    for (size_t r = 0; r < row_count; ++r) LSX_ENSURE(rows[r] < vocab, "check the attribution row range");
    cudaSetDevice(ctx->device);
    const int V = (int)vocab, P = (int)points, K = (int)panels;
    const int parts = (V + kWarpSpan - 1) / kWarpSpan;
    const size_t lbytes = points * vocab * 4;
    const size_t slots = 2 + row_count;
    auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t batch = std::min<size_t>(points, kStatsBatch);  // points per partial pass
    const size_t n_partial = batch * (panels + 1) * (size_t)parts;
    const size_t need = 2 * a256(lbytes) + a256(points * 4) + a256(points * 8) + a256(n_partial * 16) +
                        a256(points * (panels + 1) * 16) + a256(vocab * 8) + a256(row_count * 4 + 4) +
                        a256(points * row_count * 8 + 8) + a256(points * slots * 8);
    void* block = nullptr;
    LSX_TRY(device_alloc(ctx, need, &block));
    uint8_t* base = (uint8_t*)block;
    size_t at = 0;
    auto take = [&](size_t bytes) {
        uint8_t* q = base + at;
        at += a256(bytes);
        return q;
    };
    float* d_before = (float*)take(lbytes);
    float* d_after = (float*)take(lbytes);
    uint32_t* d_targets = (uint32_t*)take(points * 4);
    double* d_weights = (double*)take(points * 8);
    double2* d_partial = (double2*)take(n_partial * 16);
    double2* d_stats = (double2*)take(points * (panels + 1) * 16);
    double* d_credits = (double*)take(vocab * 8);
    uint32_t* d_rows = (uint32_t*)take(row_count * 4 + 4);
    double* d_grad = (double*)take(points * row_count * 8 + 8);
    double* d_losses = (double*)take(points * slots * 8);
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaMemcpyAsync(d_before, before, lbytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_after, after, lbytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_targets, targets, points * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_weights, weights, points * 8, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && row_count)
        e = cudaMemcpyAsync(d_rows, rows, row_count * 4, cudaMemcpyHostToDevice, s);
    for (size_t p0 = 0; p0 < points && e == cudaSuccess; p0 += batch) {
        const int nb = (int)std::min(batch, points - p0);
        chord_stats_kernel<<<dim3((unsigned)((parts + 7) / 8), (unsigned)nb), 256, 0, s>>>(
            d_before + p0 * vocab, d_after + p0 * vocab, V, K, parts, d_partial);
        e = cudaGetLastError();
        if (e == cudaSuccess) {
            const int n = nb * (K + 1);
            chord_merge_kernel<<<(n + 127) / 128, 128, 0, s>>>(d_partial, nb, K, parts, d_stats + p0 * (K + 1));
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess) {
        chord_credit_kernel<<<(V + 255) / 256, 256, 0, s>>>(d_before, d_after, d_targets, d_weights, d_stats, V, P,
                                                            K, d_credits);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && row_count && gradients_out) {
        const int n = P * (int)row_count;
        chord_gradient_kernel<<<(n + 127) / 128, 128, 0, s>>>(d_before, d_after, d_targets, d_stats, d_rows,
                                                              (int)row_count, V, P, K, d_grad);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && losses_out) {
        for (size_t p0 = 0; p0 < points && e == cudaSuccess; p0 += 65535) {
            const unsigned nb = (unsigned)std::min<size_t>(65535, points - p0);
            restored_loss_kernel<<<dim3((unsigned)slots, nb), 512, 0, s>>>(
                d_before + p0 * vocab, d_after + p0 * vocab, d_targets + p0, d_rows, V, d_losses + p0 * slots,
                (int)slots);
            e = cudaGetLastError();
        }
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(credits_out, d_credits, vocab * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && row_count && gradients_out)
        e = cudaMemcpyAsync(gradients_out, d_grad, points * row_count * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && losses_out)
        e = cudaMemcpyAsync(losses_out, d_losses, points * slots * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    device_release(ctx, block);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("integrated credits", e));
    return LSX_OK;
}

}  // extern "C"
