// Device helpers shared by the fused decode and readout kernels: mbarriers,
// 1-D bulk copies (cp.async.bulk, no multicast), programmatic dependent launch
// controls and bounded waits that report a timeout instead of hanging.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace lsx {

// Error codes a kernel may record in its status word.
enum : int {
    kDeviceOk = 0,
    kDeviceTimeoutWeights = 1,  // a weight-stage mbarrier did not complete in time
    kDeviceTimeoutMma = 2,      // an MMA/TMA pipeline barrier did not complete in time
    kDeviceTimeoutEpilogue = 3,
};

// The gate activations of the MLPs (kernels/ops.py gated: 0 SiLU, 1 GELU (erf),
// 2 ReLU, 3 GELU (tanh)).
__device__ __forceinline__ float act_fn(float x, int kind) {
    switch (kind) {
    case 0: return x / (1.f + expf(-x));
    case 1: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
    case 2: return fmaxf(x, 0.f);
    default: return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
    }
}

// About one second at B200 clocks; a healthy wait completes in microseconds.
constexpr long long kWaitCycles = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of `bar` to complete; gives up after kWaitCycles and
// returns false (the caller records a status and leaves).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    long long start = clock64();
    while (!mbar_try_wait(a, parity)) {
        if (clock64() - start > kWaitCycles) return false;
    }
    return true;
}

// Orders this thread's (and, after a block barrier, the block's) earlier generic
// accesses to shared memory before its later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared completing on `bar` (bytes % 16 == 0, both
// addresses 16-byte aligned).  The source is this GPU's own memory.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for data read exactly once (streamed weights): evict it first so it
// does not displace small, hot data (norm gains, KV cache, exchange buffers).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_load with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait until every kernel this one depends on has completed.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Order-preserving key for f32 under IEEE total order (f32::total_cmp): a larger
// key is a larger value.  Combined with the complemented index, the u64 maximum
// picks the largest value and, among equal values, the lowest index.
__device__ __forceinline__ uint32_t total_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float total_order_value(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}
__device__ __forceinline__ unsigned long long pack_arg(float v, uint32_t index) {
    return ((unsigned long long)total_order_key(v) << 32) | (unsigned long long)(0xffffffffu - index);
}
__device__ __forceinline__ uint32_t packed_index(unsigned long long p) {
    return 0xffffffffu - (uint32_t)(p & 0xffffffffull);
}
__device__ __forceinline__ float packed_value(unsigned long long p) { return total_order_value((uint32_t)(p >> 32)); }

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

}  // namespace lsx

namespace lsx {

// Eight bf16 weights (one 16-byte chunk) dotted with eight f32 activations.
__device__ __forceinline__ float dot8_bf16(uint4 w, float4 a, float4 b) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    float2 p0 = __bfloat1622float2(h[0]);
    float2 p1 = __bfloat1622float2(h[1]);
    float2 p2 = __bfloat1622float2(h[2]);
    float2 p3 = __bfloat1622float2(h[3]);
    float s = p0.x * a.x;
    s = fmaf(p0.y, a.y, s);
    s = fmaf(p1.x, a.z, s);
    s = fmaf(p1.y, a.w, s);
    s = fmaf(p2.x, b.x, s);
    s = fmaf(p2.y, b.y, s);
    s = fmaf(p3.x, b.z, s);
    s = fmaf(p3.y, b.w, s);
    return s;
}

}  // namespace lsx
