// Per-op kernels of liblsx: the parity surface of the reference's Gpu methods
// (src/gpu.rs:360-559) over the ops of kernels/ops.py.  Activations are f32,
// stored weights are F32/F16/BF16 and widened exactly; accumulation is f32.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include <cmath>
#include <vector>

#include "device_common.cuh"
#include "lsx_internal.h"

namespace lsx {

// ----------------------------------------------------------------- helpers --
__device__ __forceinline__ float widen(const void* base, int kind, size_t i) {
    if (kind == LSX_F32) return ((const float*)base)[i];
    if (kind == LSX_BF16) return __bfloat162float(((const __nv_bfloat16*)base)[i]);
    return __half2float(((const __half*)base)[i]);
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 load_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum for blockDim.x <= 1024; every thread receives the result.
__device__ float block_sum(float v, float* scratch /* >= 33 floats */) {
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < warps ? scratch[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) scratch[32] = t;
    }
    __syncthreads();
    return scratch[32];
}

// Eight packed bf16/f16 values (one 16-byte chunk) dotted with eight f32 values.
template <int KIND>
__device__ __forceinline__ float dot8(uint4 w, float4 a, float4 b) {
    float f[8];
    if (KIND == LSX_BF16) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 p = __bfloat1622float2(h[i]);
            f[2 * i] = p.x;
            f[2 * i + 1] = p.y;
        }
    } else {
        const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 p = __half22float2(h[i]);
            f[2 * i] = p.x;
            f[2 * i + 1] = p.y;
        }
    }
    float s = f[0] * a.x;
    s = fmaf(f[1], a.y, s);
    s = fmaf(f[2], a.z, s);
    s = fmaf(f[3], a.w, s);
    s = fmaf(f[4], b.x, s);
    s = fmaf(f[5], b.y, s);
    s = fmaf(f[6], b.z, s);
    s = fmaf(f[7], b.w, s);
    return s;
}

// ------------------------------------------------------------------- GEMV --
// y[r] = sum_c W[r,c] x[c] (+ b[r]).  G threads cooperate on one row; each thread
// keeps UNROLL independent 16-byte weight loads in flight.  Requires 16-byte
// aligned W and x and cols a multiple of 8 (2-byte kinds) or 4 (f32).
template <int KIND, int G>
__global__ void __launch_bounds__(256) gemv_vector_kernel(const void* __restrict__ W,
                                                          const float* __restrict__ x,
                                                          const float* __restrict__ bias, int rows,
                                                          int cols, float* __restrict__ out) {
    constexpr int RPC = 256 / G;
    constexpr int UNROLL = 4;
    __shared__ float partial[256 / 32];
    const int t = threadIdx.x;
    const int r = blockIdx.x * RPC + t / G;
    const int g = t % G;
    float acc = 0.f;
    if (threadIdx.x == 0) pdl_launch_dependents();
    // x and the output depend on earlier kernels; the weights do not, so the first
    // weight loads are issued before waiting for the preceding grid (a no-op unless
    // launched as a programmatic dependent)
    bool waited = false;
    if (r < rows) {
        if (KIND == LSX_F32) {
            const int chunks = cols >> 2;
            const char* row = (const char*)W + (size_t)r * cols * 4;
            for (int base = g; base < chunks; base += UNROLL * G) {
                uint4 w[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    int c = base + u * G;
                    w[u] = c < chunks ? load_stream(row + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
                }
                if (!waited) {
                    pdl_wait();
                    waited = true;
                }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    int c = base + u * G;
                    if (c < chunks) {
                        float4 a = __ldg(reinterpret_cast<const float4*>(x) + c);
                        acc = fmaf(__uint_as_float(w[u].x), a.x, acc);
                        acc = fmaf(__uint_as_float(w[u].y), a.y, acc);
                        acc = fmaf(__uint_as_float(w[u].z), a.z, acc);
                        acc = fmaf(__uint_as_float(w[u].w), a.w, acc);
                    }
                }
            }
        } else {
            const int chunks = cols >> 3;
            const char* row = (const char*)W + (size_t)r * cols * 2;
            for (int base = g; base < chunks; base += UNROLL * G) {
                uint4 w[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    int c = base + u * G;
                    w[u] = c < chunks ? load_stream(row + (size_t)c * 16) : make_uint4(0, 0, 0, 0);
                }
                if (!waited) {
                    pdl_wait();
                    waited = true;
                }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    int c = base + u * G;
                    if (c < chunks) {
                        float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * c);
                        float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * c + 1);
                        acc += dot8<KIND>(w[u], a, b);
                    }
                }
            }
        }
    }
    if (!waited) pdl_wait();  // before the output write
    acc = warp_sum(acc);
    if (G > 32) {
        if ((t & 31) == 0) partial[t >> 5] = acc;
        __syncthreads();
        if (g == 0) {
            acc = 0.f;
#pragma unroll
            for (int i = 0; i < G / 32; ++i) acc += partial[(t >> 5) + i];
        }
    }
    if (g == 0 && r < rows) out[r] = bias ? acc + bias[r] : acc;
}

// Streaming bf16 GEMV for matrices that span the GPU (kernels/ops.py:14-28 with W
// bf16 and x f32): one CTA per SM owns a contiguous block of rows, which is one
// contiguous byte range of W, and streams it through a ring of shared-memory
// stages with 1-D bulk copies issued by a producer warp, so each SM keeps up to
// kStreamStages x 32 KB of weights in flight whatever the compute warps are doing.
// x is staged once per CTA in shared memory; each compute warp takes two rows of a
// stage at a time, so every x load serves two rows.  Waits are bounded: a stage
// that never lands (a failed copy) ends the CTA's work and its rows read NaN.
constexpr int kStreamWarps = 8;
constexpr int kStreamThreads = (kStreamWarps + 1) * 32;
constexpr int kStreamChunk = 32768;  // bytes per stage at most
constexpr int kStreamStages = 6;

struct StreamPlan {
    int rows_per_stage, stages;
    size_t smem;
};

StreamPlan stream_plan(int cols, size_t smem_limit) {
    StreamPlan p{};
    p.rows_per_stage = (kStreamChunk / (2 * cols)) & ~1;  // even: the warps take rows in pairs
    const size_t stage = (size_t)p.rows_per_stage * cols * 2;
    const size_t fixed = (size_t)cols * 4 + 2 * kStreamStages * 8 + 128;
    p.stages = 0;
    for (int st = kStreamStages; st >= 2; --st)
        if (fixed + st * stage <= smem_limit) {
            p.stages = st;
            break;
        }
    p.smem = fixed + (size_t)p.stages * stage;
    return p;
}

__global__ void __launch_bounds__(kStreamThreads, 1)
    gemv_stream_kernel(const __nv_bfloat16* __restrict__ W, const float* __restrict__ x,
                       const float* __restrict__ bias, int rows, int cols, int rows_per_stage, int stages,
                       float* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t smem[];
    const size_t stage_bytes = (size_t)rows_per_stage * cols * 2;
    float* xs = reinterpret_cast<float*>(smem + (size_t)stages * stage_bytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(xs + cols);
    uint64_t* empty = full + kStreamStages;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (int)(((long long)blockIdx.x * rows) / gridDim.x);
    const int r1 = (int)(((long long)(blockIdx.x + 1) * rows) / gridDim.x);
    const int nchunks = (r1 - r0 + rows_per_stage - 1) / rows_per_stage;
    if (threadIdx.x == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kStreamWarps);
        }
        fence_barrier_init();
        pdl_launch_dependents();  // the next kernel may start fetching its own weights
    }
    __syncthreads();
    if (warp == kStreamWarps) {  // ------------------------------ producer
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            for (int ch = 0; ch < nchunks; ++ch) {
                const int slot = ch % stages;
                if (ch >= stages && !mbar_wait_bounded(&empty[slot], (uint32_t)(((ch / stages) - 1) & 1))) break;
                const int a = r0 + ch * rows_per_stage, n = min(rows_per_stage, r1 - a);
                const uint32_t bytes = (uint32_t)n * (uint32_t)cols * 2u;
                mbar_expect_tx(&full[slot], bytes);
                bulk_load_hint(smem + (size_t)slot * stage_bytes, W + (size_t)a * cols, bytes, &full[slot], policy);
            }
        }
        return;
    }
    // -------------------------------------------------------------- compute
    // x is staged while the first weight stages are already in flight (named
    // barrier 1 joins the compute warps only).  Weights never depend on earlier
    // kernels; x and the outputs do, so they wait for the preceding grid here (a
    // no-op unless this kernel was launched as a programmatic dependent).
    pdl_wait();
    for (int i = threadIdx.x; i < cols / 4; i += kStreamWarps * 32)
        reinterpret_cast<float4*>(xs)[i] = __ldg(reinterpret_cast<const float4*>(x) + i);
    asm volatile("bar.sync 1, %0;" ::"n"(kStreamWarps * 32) : "memory");
    // Row pairs are dealt to the warps round-robin across stages (rows_per_stage is
    // even), so wide rows (a few per stage) still keep every warp busy.  Every warp
    // waits for every stage before it releases it: a release then always belongs
    // to the stage's current use.
    const int nk = cols >> 3;  // 16-byte chunks per row
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    const int pairs_per_stage = rows_per_stage / 2;
    bool ok = true;
    for (int ch = 0; ch < nchunks; ++ch) {
        const int slot = ch % stages;
        const int a = r0 + ch * rows_per_stage, n = min(rows_per_stage, r1 - a);
        ok = ok && mbar_wait_bounded(&full[slot], (uint32_t)((ch / stages) & 1));
        const uint8_t* base = smem + (size_t)slot * stage_bytes;
        const int first = (kStreamWarps + warp - (ch * pairs_per_stage) % kStreamWarps) % kStreamWarps;
        for (int i = 2 * first; i < n; i += 2 * kStreamWarps) {
            const bool two = i + 1 < n;
            const uint4* w0 = reinterpret_cast<const uint4*>(base + (size_t)i * cols * 2);
            const uint4* w1 = reinterpret_cast<const uint4*>(base + (size_t)(two ? i + 1 : i) * cols * 2);
            float s0 = 0.f, s1 = 0.f;
            if (ok) {
                for (int c = lane; c < nk; c += 32) {
                    const float4 xa = x4[2 * c], xb = x4[2 * c + 1];
                    s0 += dot8<LSX_BF16>(w0[c], xa, xb);
                    s1 += dot8<LSX_BF16>(w1[c], xa, xb);
                }
            }
            s0 = warp_sum(s0);
            s1 = warp_sum(s1);
            if (lane == 0) {
                const int r = a + i;
                out[r] = ok ? (bias ? s0 + bias[r] : s0) : __int_as_float(0x7fc00000);
                if (two) out[r + 1] = ok ? (bias ? s1 + bias[r + 1] : s1) : __int_as_float(0x7fc00000);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (!ok) return;
}

// Any shape or alignment: one warp per row, scalar loads.
__global__ void gemv_scalar_kernel(const void* __restrict__ W, int kind, const float* __restrict__ x,
                                   const float* __restrict__ bias, int rows, int cols,
                                   float* __restrict__ out) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= rows) return;
    float acc = 0.f;
    size_t base = (size_t)warp * cols;
    for (int c = lane; c < cols; c += 32) acc = fmaf(widen(W, kind, base + c), x[c], acc);
    acc = warp_sum(acc);
    if (lane == 0) out[warp] = bias ? acc + bias[warp] : acc;
}

template <int KIND, int G>
static cudaError_t launch_gemv_g(cudaStream_t s, const void* w, const float* x, const float* b, int rows,
                                 int cols, float* out, bool stable_weight) {
    constexpr int RPC = 256 / G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows + RPC - 1) / RPC);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = stable_weight ? 1 : 0;  // early weight loads need weights no kernel writes
    return cudaLaunchKernelEx(&cfg, gemv_vector_kernel<KIND, G>, w, x, b, rows, cols, out);
}

template <int KIND>
static cudaError_t launch_gemv_kind(cudaStream_t s, int sm, const void* w, const float* x, const float* b,
                                    int rows, int cols, float* out, bool stable_weight) {
    int chunks = KIND == LSX_F32 ? cols / 4 : cols / 8;
    int G = 32;
    while (G < 256 && (long)rows * G / 256 < 2L * sm && chunks >= 4 * G) G *= 2;
    switch (G) {
    case 32: return launch_gemv_g<KIND, 32>(s, w, x, b, rows, cols, out, stable_weight);
    case 64: return launch_gemv_g<KIND, 64>(s, w, x, b, rows, cols, out, stable_weight);
    case 128: return launch_gemv_g<KIND, 128>(s, w, x, b, rows, cols, out, stable_weight);
    default: return launch_gemv_g<KIND, 256>(s, w, x, b, rows, cols, out, stable_weight);
    }
}

// Matrices of at least this many bytes stream through the shared-memory ring.
constexpr size_t kStreamMinBytes = size_t(32) << 20;

cudaError_t launch_matvec(cudaStream_t s, int sm, const void* w, int kind, const float* x, const float* bias,
                          size_t rows, size_t cols, float* out, bool stable_weight) {
    bool aligned = ((uintptr_t)w % 16 == 0) && ((uintptr_t)x % 16 == 0);
    bool vector = aligned && (kind == LSX_F32 ? cols % 4 == 0 : cols % 8 == 0);
    if (vector && kind == LSX_BF16 && rows * cols * 2 >= kStreamMinBytes && cols <= 8192 &&
        rows >= (size_t)4 * sm) {
        int device = 0, limit = 0;
        cudaError_t e = cudaGetDevice(&device);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        if (e != cudaSuccess) return e;
        const StreamPlan plan = stream_plan((int)cols, (size_t)limit);
        if (plan.stages >= 2 && plan.rows_per_stage >= 2) {
            e = cudaFuncSetAttribute((const void*)gemv_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)plan.smem);
            if (e != cudaSuccess) return e;
            // programmatic dependent launch: the weight stream starts while the
            // previous kernel on the stream finishes; x is read after it completes
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(sm);
            cfg.blockDim = dim3(kStreamThreads);
            cfg.dynamicSmemBytes = plan.smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = stable_weight ? 1 : 0;
            return cudaLaunchKernelEx(&cfg, gemv_stream_kernel, (const __nv_bfloat16*)w, x, bias, (int)rows,
                                      (int)cols, plan.rows_per_stage, plan.stages, out);
        }
    }
    if (vector) {
        if (kind == LSX_BF16) return launch_gemv_kind<LSX_BF16>(s, sm, w, x, bias, (int)rows, (int)cols, out, stable_weight);
        if (kind == LSX_F16) return launch_gemv_kind<LSX_F16>(s, sm, w, x, bias, (int)rows, (int)cols, out, stable_weight);
        return launch_gemv_kind<LSX_F32>(s, sm, w, x, bias, (int)rows, (int)cols, out, stable_weight);
    }
    int warps_per_block = 8;
    int grid = (int)((rows + warps_per_block - 1) / warps_per_block);
    gemv_scalar_kernel<<<grid, 256, 0, s>>>(w, kind, x, bias, (int)rows, (int)cols, out);
    return cudaGetLastError();
}

// ------------------------------------------------------------ other ops -----
__global__ void take_row_kernel(const void* W, int kind, size_t row, size_t width, float* out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < width) out[i] = widen(W, kind, row * width + i);
}

cudaError_t launch_take_row(cudaStream_t s, const void* w, int kind, size_t row, size_t width, float* out) {
    take_row_kernel<<<(unsigned)((width + 255) / 256), 256, 0, s>>>(w, kind, row, width, out);
    return cudaGetLastError();
}

// kernels/ops.py:31-45: one block per group.
__global__ void norm_kernel(const float* __restrict__ x, const float* __restrict__ gain,
                            const float* __restrict__ bias, int width, float eps, int center,
                            float* __restrict__ out) {
    __shared__ float scratch[33];
    const float* row = x + (size_t)blockIdx.x * width;
    float mean = 0.f;
    if (center) {
        float s = 0.f;
        for (int i = threadIdx.x; i < width; i += blockDim.x) s += row[i];
        mean = block_sum(s, scratch) / (float)width;
    }
    float q = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        float d = row[i] - mean;
        q = fmaf(d, d, q);
    }
    float inverse = rsqrtf(block_sum(q, scratch) / (float)width + eps);
    float* o = out + (size_t)blockIdx.x * width;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        float y = (row[i] - mean) * inverse * gain[i];
        if (bias) y += bias[i];
        o[i] = y;
    }
}

cudaError_t launch_norm(cudaStream_t s, const float* x, const float* gain, const float* bias, size_t groups,
                        size_t width, float eps, int center, float* out) {
    norm_kernel<<<(unsigned)groups, 256, 0, s>>>(x, gain, bias, (int)width, eps, center, out);
    return cudaGetLastError();
}

// kernels/ops.py:48-66.  The phase is formed in f64 (position * theta^(-2 pair/rotary))
// so that long positions keep f32-level accuracy in the rotated values.
__global__ void rope_kernel(const float* __restrict__ x, size_t position, int dim, int width, double theta,
                            int rotary, int interleaved, float* __restrict__ out) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= width) return;
    int local = i % dim;
    float original = x[i];
    if (local >= rotary) {
        out[i] = original;
        return;
    }
    int pair, other;
    double sign;
    if (interleaved) {
        pair = local / 2;
        other = (local % 2 == 0) ? local + 1 : local - 1;
        sign = (local % 2 == 0) ? -1.0 : 1.0;
    } else {
        int half = rotary / 2;
        pair = local % half;
        other = local < half ? local + half : local - half;
        sign = local < half ? -1.0 : 1.0;
    }
    double angle = (double)position * pow(theta, -2.0 * (double)pair / (double)rotary);
    double sn, cs;
    sincos(angle, &sn, &cs);
    float partner = x[i - local + other];
    out[i] = (float)((double)original * cs + sign * (double)partner * sn);
}

cudaError_t launch_rope(cudaStream_t s, const float* x, size_t position, size_t heads, size_t dim, float theta,
                        size_t rotary, int interleaved, float* out) {
    int width = (int)(heads * dim);
    rope_kernel<<<(width + 255) / 256, 256, 0, s>>>(x, position, (int)dim, width, (double)theta, (int)rotary,
                                                    interleaved, out);
    return cudaGetLastError();
}

// kernels/ops.py:69-73
__global__ void cache_write_kernel(const float* k, const float* v, float* keys, float* values, size_t position,
                                   int width) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < width) {
        keys[position * width + i] = k[i];
        values[position * width + i] = v[i];
    }
}

cudaError_t launch_cache_write(cudaStream_t s, const float* k, const float* v, float* keys, float* values,
                               size_t position, size_t width) {
    cache_write_kernel<<<(unsigned)((width + 255) / 256), 256, 0, s>>>(k, v, keys, values, position, (int)width);
    return cudaGetLastError();
}

// kernels/ops.py:76-101: one block per query head, one warp per key position,
// online softmax per warp and an exact merge of the warp states.
constexpr int kAttnWarps = 4;
constexpr int kMaxDimPerLane = 8;  // head_dim <= 256

__global__ void __launch_bounds__(kAttnWarps * 32) attention_kernel(const float* __restrict__ q,
                                                                    const float* __restrict__ keys,
                                                                    const float* __restrict__ values,
                                                                    int position, int qheads, int kvheads,
                                                                    int dim, float scale,
                                                                    float* __restrict__ out) {
    __shared__ float s_m[kAttnWarps], s_l[kAttnWarps];
    __shared__ float s_acc[kAttnWarps][kMaxDimPerLane * 32];
    const int head = blockIdx.x;
    const int kv = head / (qheads / kvheads);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int width = kvheads * dim;
    float qd[kMaxDimPerLane], acc[kMaxDimPerLane];
#pragma unroll
    for (int j = 0; j < kMaxDimPerLane; ++j) {
        int d = lane + 32 * j;
        qd[j] = d < dim ? q[head * dim + d] : 0.f;
        acc[j] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int t = warp; t <= position; t += kAttnWarps) {
        const float* kt = keys + (size_t)t * width + kv * dim;
        const float* vt = values + (size_t)t * width + kv * dim;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxDimPerLane; ++j) {
            int d = lane + 32 * j;
            if (d < dim) s = fmaf(qd[j], kt[d], s);
        }
        s = warp_sum(s) * scale;
        float mn = fmaxf(m, s);
        float carry = expf(m - mn);
        float p = expf(s - mn);
        l = l * carry + p;
#pragma unroll
        for (int j = 0; j < kMaxDimPerLane; ++j) {
            int d = lane + 32 * j;
            if (d < dim) acc[j] = fmaf(p, vt[d], acc[j] * carry);
        }
        m = mn;
    }
    if (lane == 0) {
        s_m[warp] = m;
        s_l[warp] = l;
    }
#pragma unroll
    for (int j = 0; j < kMaxDimPerLane; ++j) s_acc[warp][lane + 32 * j] = acc[j];
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) L += s_m[w] == -INFINITY ? 0.f : s_l[w] * expf(s_m[w] - M);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        float o = 0.f;
        for (int w = 0; w < kAttnWarps; ++w)
            if (s_m[w] != -INFINITY) o = fmaf(s_acc[w][d], expf(s_m[w] - M), o);
        out[head * dim + d] = o / L;
    }
}

cudaError_t launch_attention(cudaStream_t s, const float* q, const float* keys, const float* values,
                             size_t position, size_t qheads, size_t kvheads, size_t dim, float scale, float* out) {
    attention_kernel<<<(unsigned)qheads, kAttnWarps * 32, 0, s>>>(q, keys, values, (int)position, (int)qheads,
                                                                  (int)kvheads, (int)dim, scale, out);
    return cudaGetLastError();
}

// kernels/ops.py:104-116
__device__ __forceinline__ float activate(float x, int kind) {
    switch (kind) {
    case 0: return x / (1.f + expf(-x));
    case 1: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
    case 2: return fmaxf(x, 0.f);
    default: return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
    }
}

__global__ void gated_kernel(const float* gate, const float* up, int n, int kind, float* out) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = activate(gate[i], kind) * up[i];
}

cudaError_t launch_gated(cudaStream_t s, const float* gate, const float* up, size_t n, int kind, float* out) {
    gated_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(gate, up, (int)n, kind, out);
    return cudaGetLastError();
}

// kernels/ops.py:119-122; no FMA contraction, as the reference compiles it
// (kernels/compile.py:35), so x + f*y rounds the product and the sum separately.
__global__ void combine_kernel(const float* x, const float* y, float factor, int n, float* out) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(x[i], __fmul_rn(factor, y[i]));
}

cudaError_t launch_combine(cudaStream_t s, const float* x, const float* y, float factor, size_t n, float* out) {
    combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, y, factor, (int)n, out);
    return cudaGetLastError();
}

// kernels/ops.py:125-135: one block.
__global__ void rotate_kernel(const float* h, const float* u, const float* v, float a, float b, int width,
                              float* out) {
    __shared__ float scratch[33];
    float hu = 0.f, hv = 0.f;
    for (int i = threadIdx.x; i < width; i += blockDim.x) {
        hu = fmaf(h[i], u[i], hu);
        hv = fmaf(h[i], v[i], hv);
    }
    hu = block_sum(hu, scratch);
    hv = block_sum(hv, scratch);
    for (int i = threadIdx.x; i < width; i += blockDim.x)
        out[i] = h[i] + u[i] * (a * hu + b * hv) + v[i] * (a * hv - b * hu);
}

cudaError_t launch_rotate(cudaStream_t s, const float* h, const float* u, const float* v, float a, float b,
                          size_t width, float* out) {
    rotate_kernel<<<1, 1024, 0, s>>>(h, u, v, a, b, (int)width, out);
    return cudaGetLastError();
}

__global__ void all_finite_kernel(const float* x, size_t n, int* flag) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (; i < n; i += stride) bad |= !isfinite(x[i]);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1);
}

cudaError_t launch_all_finite(cudaStream_t s, const float* x, size_t n, int* flag) {
    unsigned grid = (unsigned)((n + 255) / 256);
    if (grid > 1024) grid = 1024;
    all_finite_kernel<<<grid, 256, 0, s>>>(x, n, flag);
    return cudaGetLastError();
}

}  // namespace lsx

using namespace lsx;

namespace {

int finish(lsx_ctx* ctx, cudaError_t e, lsx_tensor* out, lsx_tensor** result, const char* what) {
    if (e != cudaSuccess) {
        lsx_tensor_free(out);
        return fail(LSX_E_CUDA, cuda_message(what, e));
    }
    *result = out;
    return LSX_OK;
}

bool is_f32(const lsx_tensor* t) { return t && t->kind == LSX_F32; }

// ReadoutRotation::validate (src/rotation.rs:28-49)
int validate_plane(const double* u, const double* v, double tangent, size_t width) {
    LSX_ENSURE(width > 1 && u && v, "check the rotation vector dimensions");
    double uu = 0, vv = 0, uv = 0;
    for (size_t i = 0; i < width; ++i) {
        LSX_ENSURE(std::isfinite(u[i]) && std::isfinite(v[i]), "finite rotation coordinates are required");
        uu += u[i] * u[i];
        vv += v[i] * v[i];
        uv += u[i] * v[i];
    }
    LSX_ENSURE(std::isfinite(tangent), "finite rotation coordinates are required");
    LSX_ENSURE(std::fabs(uu - 1) < 1e-8 && std::fabs(vv - 1) < 1e-8 && std::fabs(uv) < 1e-8,
               "the rotation plane needs orthonormal unit vectors");
    LSX_ENSURE(std::fabs(tangent) <= 1e6, "the half-angle coordinate must be within 1e6 in magnitude");
    return LSX_OK;
}

double determinant(std::vector<double> a, size_t n) {
    double det = 1.0;
    for (size_t c = 0; c < n; ++c) {
        size_t p = c;
        for (size_t r = c + 1; r < n; ++r)
            if (std::fabs(a[r * n + c]) > std::fabs(a[p * n + c])) p = r;
        if (a[p * n + c] == 0.0) return 0.0;
        if (p != c) {
            for (size_t k = 0; k < n; ++k) std::swap(a[p * n + k], a[c * n + k]);
            det = -det;
        }
        det *= a[c * n + c];
        for (size_t r = c + 1; r < n; ++r) {
            double f = a[r * n + c] / a[c * n + c];
            for (size_t k = c; k < n; ++k) a[r * n + k] -= f * a[c * n + k];
        }
    }
    return det;
}

// SubspaceRotation::validate (src/response.rs:33-60)
int validate_joint(const double* basis, const double* transform, size_t rank, size_t width) {
    LSX_ENSURE(basis && transform, "invalid argument");
    LSX_ENSURE(rank > 0 && rank <= width && rank <= 256, "check the joint rotation rank and inner matrix size");
    for (size_t i = 0; i < rank * width; ++i)
        LSX_ENSURE(std::isfinite(basis[i]), "the joint rotation needs a finite basis and square matrix");
    for (size_t i = 0; i < rank * rank; ++i)
        LSX_ENSURE(std::isfinite(transform[i]), "the joint rotation needs a finite basis and square matrix");
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j <= i; ++j) {
            double d = 0;
            for (size_t k = 0; k < width; ++k) d += basis[i * width + k] * basis[j * width + k];
            LSX_ENSURE(std::fabs(d - (i == j ? 1.0 : 0.0)) < 1e-8, "check the orthogonality of the joint basis");
        }
    double worst = 0;
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < rank; ++j) {
            double d = 0;
            for (size_t k = 0; k < rank; ++k) d += transform[k * rank + i] * transform[k * rank + j];
            worst = std::fmax(worst, std::fabs(d - (i == j ? 1.0 : 0.0)));
        }
    std::vector<double> copy(transform, transform + rank * rank);
    LSX_ENSURE(worst < 1e-8 && determinant(copy, rank) > 0.0,
               "check the orthogonality and orientation of the joint rotation");
    return LSX_OK;
}

}  // namespace

extern "C" {

int lsx_embedding(lsx_ctx* ctx, const lsx_tensor* weight, size_t row, size_t width, lsx_tensor** out) {
    LSX_ENSURE(ctx && weight && out, "invalid argument");
    LSX_ENSURE(width > 0 && row < weight->count / width, "check the embedding row range");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, width, LSX_F32, &o));
    return finish(ctx, launch_take_row(ctx->stream, weight->data, weight->kind, row, width, (float*)o->data), o,
                  out, "take_row");
}

int lsx_linear_into(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* w, const lsx_tensor* bias, size_t rows,
                    size_t cols, lsx_tensor* out) {
    LSX_ENSURE(ctx && x && w && out, "invalid argument");
    LSX_ENSURE(is_f32(x) && (!bias || is_f32(bias)) && is_f32(out), "linear inputs, bias and output are F32 tensors");
    LSX_ENSURE(rows > 0 && cols > 0 && x->count == cols && w->count / rows == cols && w->count % rows == 0 &&
                   (!bias || bias->count == rows) && out->count == rows,
               "check the dimensions of the linear op");
    cudaSetDevice(ctx->device);
    // a BF16 tensor the library owns was uploaded from the host (every op output is
    // F32), so no kernel writes it; wrapped caller memory might be
    LSX_CUDA(launch_matvec(ctx->stream, ctx->sm_count, w->data, w->kind, (const float*)x->data,
                           bias ? (const float*)bias->data : nullptr, rows, cols, (float*)out->data, w->owned),
             "matvec");
    return LSX_OK;
}

int lsx_linear(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* w, const lsx_tensor* bias, size_t rows,
               size_t cols, lsx_tensor** out) {
    LSX_ENSURE(ctx && x && w && out, "invalid argument");
    LSX_ENSURE(is_f32(x) && (!bias || is_f32(bias)), "linear inputs and bias are F32 tensors");
    LSX_ENSURE(rows > 0 && cols > 0 && x->count == cols && w->count / rows == cols && w->count % rows == 0 &&
                   (!bias || bias->count == rows),
               "check the dimensions of the linear op");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, rows, LSX_F32, &o));
    return finish(ctx,
                  launch_matvec(ctx->stream, ctx->sm_count, w->data, w->kind, (const float*)x->data,
                                bias ? (const float*)bias->data : nullptr, rows, cols, (float*)o->data, w->owned),
                  o, out, "matvec");
}

int lsx_norm(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* gain, const lsx_tensor* bias, size_t groups,
             size_t width, float epsilon, int center, lsx_tensor** out) {
    LSX_ENSURE(ctx && x && gain && out, "invalid argument");
    LSX_ENSURE(is_f32(x) && is_f32(gain) && (!bias || is_f32(bias)), "norm operands are F32 tensors");
    LSX_ENSURE(width > 0 && groups * width == x->count && gain->count == width && (!bias || bias->count == width) &&
                   std::isfinite(epsilon) && epsilon > 0.f,
               "check the normalization dimensions");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, x->count, LSX_F32, &o));
    return finish(ctx,
                  launch_norm(ctx->stream, (const float*)x->data, (const float*)gain->data,
                              bias ? (const float*)bias->data : nullptr, groups, width, epsilon, center,
                              (float*)o->data),
                  o, out, "normalization");
}

int lsx_rope(lsx_ctx* ctx, const lsx_tensor* x, size_t position, size_t heads, size_t dim, float theta,
             size_t rotary, int interleaved, lsx_tensor** out) {
    LSX_ENSURE(ctx && x && out && is_f32(x), "invalid argument");
    LSX_ENSURE(heads * dim == x->count && rotary > 0 && rotary <= dim && rotary % 2 == 0 &&
                   position <= 2147483647ull && std::isfinite(theta) && theta > 0.f,
               "check the RoPE dimensions");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, x->count, LSX_F32, &o));
    return finish(ctx,
                  launch_rope(ctx->stream, (const float*)x->data, position, heads, dim, theta, rotary, interleaved,
                              (float*)o->data),
                  o, out, "rotary_position");
}

int lsx_attention(lsx_ctx* ctx, const lsx_tensor* q, const lsx_tensor* k, const lsx_tensor* v, lsx_tensor* keys,
                  lsx_tensor* values, size_t position, size_t qheads, size_t kvheads, size_t dim, float scale,
                  lsx_tensor** out) {
    LSX_ENSURE(ctx && q && k && v && keys && values && out, "invalid argument");
    LSX_ENSURE(is_f32(q) && is_f32(k) && is_f32(v) && is_f32(keys) && is_f32(values),
               "attention buffers are F32 tensors");
    size_t width = kvheads * dim;
    LSX_ENSURE(width > 0 && qheads * dim == q->count && k->count == width && v->count == width &&
                   kvheads > 0 && qheads % kvheads == 0 && (position + 1) * width <= keys->count &&
                   keys->count == values->count && std::isfinite(scale) && scale > 0.f,
               "check the attention buffer dimensions");
    if (dim > (size_t)(kMaxDimPerLane * 32))
        return fail(LSX_E_UNSUPPORTED, "attention head_dim above 256 is not built");
    cudaSetDevice(ctx->device);
    cudaError_t e = launch_cache_write(ctx->stream, (const float*)k->data, (const float*)v->data,
                                       (float*)keys->data, (float*)values->data, position, width);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("cache_write", e));
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, q->count, LSX_F32, &o));
    return finish(ctx,
                  launch_attention(ctx->stream, (const float*)q->data, (const float*)keys->data,
                                   (const float*)values->data, position, qheads, kvheads, dim, scale,
                                   (float*)o->data),
                  o, out, "causal_attention");
}

int lsx_gated(lsx_ctx* ctx, const lsx_tensor* gate, const lsx_tensor* up, uint32_t kind, lsx_tensor** out) {
    LSX_ENSURE(ctx && gate && up && out && is_f32(gate) && is_f32(up), "invalid argument");
    LSX_ENSURE(gate->count == up->count && kind <= 3, "check the MLP gate conditions");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, gate->count, LSX_F32, &o));
    return finish(ctx,
                  launch_gated(ctx->stream, (const float*)gate->data, (const float*)up->data, gate->count,
                               (int)kind, (float*)o->data),
                  o, out, "gated_product");
}

int lsx_combine(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* y, float factor, lsx_tensor** out) {
    LSX_ENSURE(ctx && x && y && out && is_f32(x) && is_f32(y), "invalid argument");
    LSX_ENSURE(x->count == y->count && std::isfinite(factor), "check the vector combine conditions");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, x->count, LSX_F32, &o));
    return finish(ctx,
                  launch_combine(ctx->stream, (const float*)x->data, (const float*)y->data, factor, x->count,
                                 (float*)o->data),
                  o, out, "vector_sum");
}

int lsx_rotate(lsx_ctx* ctx, const lsx_tensor* h, const lsx_tensor* u, const lsx_tensor* v, float a, float b,
               lsx_tensor** out) {
    LSX_ENSURE(ctx && h && u && v && out && is_f32(h) && is_f32(u) && is_f32(v), "invalid argument");
    LSX_ENSURE(h->count == u->count && h->count == v->count && std::isfinite(a) && std::isfinite(b),
               "check the readout rotation conditions");
    cudaSetDevice(ctx->device);
    lsx_tensor* o = nullptr;
    LSX_TRY(reserve(ctx, h->count, LSX_F32, &o));
    return finish(ctx,
                  launch_rotate(ctx->stream, (const float*)h->data, (const float*)u->data, (const float*)v->data,
                                a, b, h->count, (float*)o->data),
                  o, out, "plane_rotation");
}

int lsx_rotation_plane(lsx_ctx* ctx, const double* u, const double* v, double tangent, size_t width,
                       lsx_rotation** out) {
    LSX_ENSURE(ctx && out, "invalid argument");
    LSX_TRY(validate_plane(u, v, tangent, width));
    std::vector<float> uf(width), vf(width);
    for (size_t i = 0; i < width; ++i) {
        uf[i] = (float)u[i];
        vf[i] = (float)v[i];
    }
    lsx_rotation* r = new lsx_rotation;
    r->ctx = ctx;
    r->joint = false;
    r->width = width;
    r->rank = 2;
    double t = tangent, a = -2.0 * t * t / (1.0 + t * t), b = 2.0 * t / (1.0 + t * t);
    r->cosine_minus_one = (float)a;
    r->sine = (float)b;
    // ReadoutEdit::subspace (src/response.rs:240-251): basis [u; v], transform
    // [[1+a, b], [-b, 1+a]], so R - I = [[a, b], [-b, a]].
    r->basis64.assign(u, u + width);
    r->basis64.insert(r->basis64.end(), v, v + width);
    r->delta64 = {a, b, -b, a};
    std::vector<float> uv(uf);
    uv.insert(uv.end(), vf.begin(), vf.end());
    const float dr[4] = {(float)a, (float)b, (float)-b, (float)a};
    int s = lsx_upload_f32(ctx, uf.data(), width, &r->u);
    if (s == LSX_OK) s = lsx_upload_f32(ctx, vf.data(), width, &r->v);
    if (s == LSX_OK) s = lsx_upload_f32(ctx, uv.data(), uv.size(), &r->basis);
    if (s == LSX_OK) s = lsx_upload_f32(ctx, dr, 4, &r->delta);
    if (s != LSX_OK) {
        lsx_rotation_free(r);
        return s;
    }
    *out = r;
    return LSX_OK;
}

int lsx_rotation_joint(lsx_ctx* ctx, const double* basis, const double* transform, size_t rank, size_t width,
                       lsx_rotation** out) {
    LSX_ENSURE(ctx && out, "invalid argument");
    LSX_TRY(validate_joint(basis, transform, rank, width));
    // DeviceRotation::upload_edit (src/model.rs:311-341)
    std::vector<float> b(rank * width), tr(width * rank), d(rank * rank);
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < width; ++j) {
            b[i * width + j] = (float)basis[i * width + j];
            tr[j * rank + i] = (float)basis[i * width + j];
        }
    lsx_rotation* r = new lsx_rotation;
    r->ctx = ctx;
    r->joint = true;
    r->width = width;
    r->rank = rank;
    r->basis64.assign(basis, basis + rank * width);
    r->delta64.resize(rank * rank);
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < rank; ++j) {
            double v = transform[i * rank + j] - (i == j ? 1.0 : 0.0);
            d[i * rank + j] = (float)v;
            r->delta64[i * rank + j] = v;
        }
    int s = lsx_upload_f32(ctx, b.data(), b.size(), &r->basis);
    if (s == LSX_OK) s = lsx_upload_f32(ctx, tr.data(), tr.size(), &r->transpose);
    if (s == LSX_OK) s = lsx_upload_f32(ctx, d.data(), d.size(), &r->delta);
    if (s != LSX_OK) {
        lsx_rotation_free(r);
        return s;
    }
    *out = r;
    return LSX_OK;
}

int lsx_rotation_apply(lsx_ctx* ctx, const lsx_rotation* rotation, const lsx_tensor* hidden, lsx_tensor** out) {
    LSX_ENSURE(ctx && rotation && hidden && out && is_f32(hidden), "invalid argument");
    LSX_ENSURE(hidden->count == rotation->width, "the hidden width does not match the rotation");
    if (!rotation->joint)
        return lsx_rotate(ctx, hidden, rotation->u, rotation->v, rotation->cosine_minus_one, rotation->sine, out);
    // DeviceRotation::apply Joint (src/model.rs:350-361): three matvecs and a combine.
    lsx_tensor *coordinates = nullptr, *shift = nullptr, *lifted = nullptr;
    int s = lsx_linear(ctx, hidden, rotation->basis, nullptr, rotation->rank, rotation->width, &coordinates);
    if (s == LSX_OK) s = lsx_linear(ctx, coordinates, rotation->delta, nullptr, rotation->rank, rotation->rank, &shift);
    if (s == LSX_OK) s = lsx_linear(ctx, shift, rotation->transpose, nullptr, rotation->width, rotation->rank, &lifted);
    if (s == LSX_OK) s = lsx_combine(ctx, hidden, lifted, 1.f, out);
    lsx_tensor_free(coordinates);
    lsx_tensor_free(shift);
    lsx_tensor_free(lifted);
    return s;
}

int lsx_rotation_free(lsx_rotation* rotation) {
    if (!rotation) return LSX_OK;
    lsx_tensor_free(rotation->u);
    lsx_tensor_free(rotation->v);
    lsx_tensor_free(rotation->basis);
    lsx_tensor_free(rotation->transpose);
    lsx_tensor_free(rotation->delta);
    delete rotation;
    return LSX_OK;
}

}  // extern "C"
