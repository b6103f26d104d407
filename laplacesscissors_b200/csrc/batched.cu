// Batched teacher-forced forward: many cases of equal length through the decoder
// at once, each layer's projections as tensor-core GEMMs over all tokens.
//
// Teacher forcing (src/scaling.rs:181-216) knows every input token in advance: a
// case feeds its prompt and then each target but the last, and scores the frames
// from the last prompt position on.  The reference feeds them one decode step at a
// time (Model::advance, src/model.rs:694-853); here the T = prompt + count - 1
// tokens of every case go through each layer together, so a layer's weights are
// read once per batch of cases instead of once per token.  Per layer:
//
//   x [M, H] f32 (M = cases x T rows, case-major)
//   RMSNorm(x) -> A planes (bf16 hi/lo of the f32 activations)
//   [q; k; v] = A Wqkv^T              (tcgen05 GEMM, f32 out)
//   QK-norm + RoPE per head, in place (position = row within the case)
//   causal attention within each case -> A planes
//   x += A Wo^T                       (GEMM, residual add in the epilogue)
//   RMSNorm(x) -> A planes
//   [g0 u0 g1 u1 ...] = A Wgu^T       (GEMM)
//   act(g) * u -> A planes
//   x += A Wd^T                       (GEMM, residual add)
//
// then the final RMSNorm of the scored rows, the lm_head GEMM into f32 logits and
// per row attribution::loss (src/attribution.rs:49-60) and the first argmax
// (src/diagnosis.rs:58-70).  The f32 activations enter the tensor cores as two
// bf16 terms (hi + lo carries 16 significant bits), each multiplied by the bf16
// weights with f32 accumulation.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include "batched.cuh"
#include "device_common.cuh"

namespace lsx {

int gemm_planes_enqueue(lsx_ctx* ctx, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int M, int K,
                        const __nv_bfloat16* w, int N, const float* bias, float* out, int ldo, bool accumulate,
                        int* status);
int gemm_gated_enqueue(lsx_ctx* ctx, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int M, int K,
                       const __nv_bfloat16* w, int N, const float* bias, int act_kind, __nv_bfloat16* out_hi,
                       __nv_bfloat16* out_lo, int* status, bool* fused);

namespace {

__device__ __forceinline__ void split_store(__nv_bfloat16* hi, __nv_bfloat16* lo, size_t i, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = h;
    lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < warps; ++i) t += red[i];
    return t;
}

// x[m] = embedding row of tokens[m] (Model::embedding_tensor, src/model.rs:620-631).
__global__ void embed_rows_kernel(const void* __restrict__ emb, int kind, float scale, const uint32_t* __restrict__ tokens,
                                  int H, float* __restrict__ x) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t m = blockIdx.x;
    const size_t base = (size_t)tokens[m] * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        float v;
        if (kind == LSX_BF16) v = __bfloat162float(((const __nv_bfloat16*)emb)[base + i]);
        else if (kind == LSX_F32) v = ((const float*)emb)[base + i];
        else v = __half2float(((const __half*)emb)[base + i]);
        if (scale != 1.f) v = __fadd_rn(v, __fmul_rn(scale - 1.f, v));
        x[m * H + i] = v;
    }
}

// A planes of RMSNorm(x[rows[r]]) * gain (kernels/ops.py:31-45); rows == nullptr: r.
// With `out` the normalised rows are written there in f32 instead.
__global__ void rms_planes_kernel(const float* __restrict__ x, const int* __restrict__ rows, int H,
                                  const float* __restrict__ gain, float eps, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo, float* __restrict__ out = nullptr) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float red[32];
    const size_t r = blockIdx.x;
    const float* xr = x + (size_t)(rows ? rows[r] : (int)r) * H;
    if ((H & 3) == 0 && !out) {  // 16-byte loads, 8-byte plane stores
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const float4* g4 = reinterpret_cast<const float4*>(gain);
        float ss = 0.f;
        for (int i = threadIdx.x; i < (H >> 2); i += blockDim.x) {
            const float4 v = x4[i];
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        const float inverse = rsqrtf(block_sum(ss, red) / (float)H + eps);
        for (int i = threadIdx.x; i < (H >> 2); i += blockDim.x) {
            const float4 v = x4[i], g = g4[i];
            const float y[4] = {v.x * inverse * g.x, v.y * inverse * g.y, v.z * inverse * g.z, v.w * inverse * g.w};
            __align__(8) __nv_bfloat16 h4[4], l4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h4[e] = __float2bfloat16_rn(y[e]);
                l4[e] = __float2bfloat16_rn(y[e] - __bfloat162float(h4[e]));
            }
            *reinterpret_cast<uint2*>(hi + r * H + 4 * i) = *reinterpret_cast<const uint2*>(h4);
            *reinterpret_cast<uint2*>(lo + r * H + 4 * i) = *reinterpret_cast<const uint2*>(l4);
        }
        return;
    }
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    const float inverse = rsqrtf(block_sum(ss, red) / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = xr[i] * inverse * gain[i];
        if (out) out[r * H + i] = v;
        else split_store(hi, lo, r * H + i, v);
    }
}

// The readout edit on each final hidden row, then its A planes: a plane rotation
// h + u (a hu + b hv) + v (a hv - b hu) (kernels/ops.py:125-135 with
// ReadoutRotation::coefficients, src/rotation.rs:50-53), or a joint rotation
// h + basis^T ((R - I) (basis h)) (DeviceRotation::apply, src/model.rs:350-361).
__global__ void edit_rows_kernel(const float* __restrict__ h, int H, int kind, float a, float b,
                                 const float* __restrict__ u, const float* __restrict__ v, int rank,
                                 const float* __restrict__ basis, const float* __restrict__ delta,
                                 __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    __shared__ float red[32];
    __shared__ float coords[256], shift[256];
    const size_t r = blockIdx.x;
    const float* hr = h + r * H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    if (kind == 1) {
        float pu = 0.f, pv = 0.f;
        for (int i = threadIdx.x; i < H; i += blockDim.x) {
            pu = fmaf(hr[i], u[i], pu);
            pv = fmaf(hr[i], v[i], pv);
        }
        const float hu = block_sum(pu, red);
        const float hv = block_sum(pv, red);
        for (int i = threadIdx.x; i < H; i += blockDim.x)
            split_store(hi, lo, r * H + i, hr[i] + u[i] * (a * hu + b * hv) + v[i] * (a * hv - b * hu));
        return;
    }
    for (int k = warp; k < rank; k += warps) {
        float d = 0.f;
        for (int j = lane; j < H; j += 32) d = fmaf(basis[(size_t)k * H + j], hr[j], d);
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) coords[k] = d;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rank; i += blockDim.x) {
        float d = 0.f;
        for (int j = 0; j < rank; ++j) d = fmaf(delta[i * rank + j], coords[j], d);
        shift[i] = d;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < H; j += blockDim.x) {
        float d = 0.f;
        for (int k = 0; k < rank; ++k) d = fmaf(basis[(size_t)k * H + j], shift[k], d);
        split_store(hi, lo, r * H + j, __fadd_rn(hr[j], d));
    }
}

// QK-norm and rotate-half RoPE in place on the q and k heads of every row; one
// warp per (row, head).  rope: [T, D/2] (cos, sin) per position.
template <int DPL>
__global__ void qk_rope_kernel(float* __restrict__ qkv, int M, int T, int QH, int KVH, const float* __restrict__ q_gain,
                               const float* __restrict__ k_gain, float eps, const float2* __restrict__ rope) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int D = DPL * 32;
    const int lane = threadIdx.x & 31;
    const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int heads = QH + KVH;
    if (wid >= (long long)M * heads) return;
    const int m = (int)(wid / heads), h = (int)(wid % heads);
    const int t = m % T;
    const bool is_q = h < QH;
    const float* gain = is_q ? q_gain : k_gain;
    float* v = qkv + (size_t)m * (QH + 2 * KVH) * D + (size_t)h * D;
    float e[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) e[j] = v[lane + 32 * j];
    if (gain) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss = fmaf(e[j], e[j], ss);
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inverse = rsqrtf(ss / (float)D + eps);
#pragma unroll
        for (int j = 0; j < DPL; ++j) e[j] = e[j] * inverse * gain[lane + 32 * j];
    }
#pragma unroll
    for (int j = 0; j < DPL / 2; ++j) {
        const float2 cs = rope[(size_t)t * (D / 2) + lane + 32 * j];
        const float a = e[j], b = e[j + DPL / 2];
        e[j] = a * cs.x + -1.f * b * cs.y;
        e[j + DPL / 2] = b * cs.x + 1.f * a * cs.y;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) v[lane + 32 * j] = e[j];
}

// Causal attention within each case (kernels/ops.py:76-101): one warp per (row,
// query head), keys s <= t of the row's case in batches of 8 (online softmax).
// Output: A planes [M, QH * D].
template <int DPL>
__global__ void causal_attention_kernel(const float* __restrict__ qkv, int M, int T, int QH, int KVH, float scale,
                                        __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    constexpr int D = DPL * 32;
    constexpr int PB = 8, LPV = 32 / PB;
    const int lane = threadIdx.x & 31;
    const long long wid = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= (long long)M * QH) return;
    const int m = (int)(wid / QH), h = (int)(wid % QH);
    const int t = m % T, first = m - t;
    const int g = h / (QH / KVH);
    const size_t stride = (size_t)(QH + 2 * KVH) * D;
    const float* kbase = qkv + (size_t)QH * D + (size_t)g * D;
    const float* vbase = kbase + (size_t)KVH * D;
    float q[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) q[j] = qkv[(size_t)m * stride + (size_t)h * D + lane + 32 * j];
    float mx = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    const int my_b = lane / LPV;
    for (int s0 = 0; s0 <= t; s0 += PB) {
        float kv[PB][DPL], vv[PB][DPL], sc[PB];
#pragma unroll
        for (int b = 0; b < PB; ++b) {
            const int s = s0 + b;
            const size_t row = (size_t)(first + (s <= t ? s : t)) * stride;
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                kv[b][j] = kbase[row + lane + 32 * j];
                vv[b][j] = vbase[row + lane + 32 * j];
            }
            float x = 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) x = fmaf(q[j], kv[b][j], x);
            sc[b] = x;
        }
        // transposing butterfly: lane l ends with the total of key l / LPV
#pragma unroll
        for (int cnt = PB, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
            const bool up = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < cnt / 2; ++i) {
                const float keep = up ? sc[i + cnt / 2] : sc[i];
                const float send = up ? sc[i] : sc[i + cnt / 2];
                sc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        for (int off = LPV / 2; off > 0; off >>= 1) sc[0] += __shfl_xor_sync(0xffffffffu, sc[0], off);
        const bool valid = s0 + my_b <= t;
        const float sv = valid ? sc[0] * scale : -INFINITY;
        float mb = sv;
        for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        const float mn = fmaxf(mx, mb);
        const float carry = expf(mx - mn);
        const float p = valid ? expf(sv - mn) : 0.f;
        float ps = (lane % LPV) == 0 ? p : 0.f;
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l = l * carry + ps;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] *= carry;
#pragma unroll
        for (int b = 0; b < PB; ++b) {
            const float pb = __shfl_sync(0xffffffffu, p, b * LPV);
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[j] = fmaf(pb, vv[b][j], acc[j]);
        }
        mx = mn;
    }
    const size_t o = (size_t)m * QH * D + (size_t)h * D;
#pragma unroll
    for (int j = 0; j < DPL; ++j) split_store(hi, lo, o + lane + 32 * j, acc[j] / l);
}

// The same attention with the keys and values staged in shared memory: a block
// takes one case, one KV group and kQT consecutive query rows (one warp per row);
// each kKT-key tile of the group's K and V is loaded once and serves every warp,
// and each warp carries all R query heads of the group, so a tile is read once per
// warp instead of once per (row, head) from L2.  Per (row, head) the arithmetic is
// that of causal_attention_kernel (the same key batches in the same order), so the
// outputs are identical.
constexpr int kQT = 8;   // query rows per block
constexpr int kKT = 32;  // keys per staged tile (a multiple of the 8-key batch)

template <int DPL, int R>
__global__ void __launch_bounds__(32 * kQT, 1) causal_attention_tiled_kernel(const float* __restrict__ qkv, int M,
                                                                          int T, int QH, int KVH, float scale,
                                                                          __nv_bfloat16* __restrict__ hi,
                                                                          __nv_bfloat16* __restrict__ lo) {
    constexpr int D = DPL * 32;
    constexpr int PB = 8, LPV = 32 / PB;
    __shared__ float ks[kKT * D], vs[kKT * D];
    const int qtiles = (T + kQT - 1) / kQT;
    int bid = blockIdx.x;
    const int qt = bid % qtiles;
    bid /= qtiles;
    const int g = bid % KVH, c = bid / KVH;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = qt * kQT + warp;  // query position within the case
    const bool active = t < T;
    const int first = c * T;
    const size_t stride = (size_t)(QH + 2 * KVH) * D;
    const float* kbase = qkv + (size_t)QH * D + (size_t)g * D;
    const float* vbase = kbase + (size_t)KVH * D;
    float q[R][DPL], mx[R], l[R], acc[R][DPL];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        mx[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            q[i][j] = active ? qkv[(size_t)(first + t) * stride + (size_t)(g * R + i) * D + lane + 32 * j] : 0.f;
            acc[i][j] = 0.f;
        }
    }
    const int my_b = lane / LPV;
    const int kv_end = min(T, qt * kQT + kQT);  // keys the block's last row needs
    for (int k0 = 0; k0 < kv_end; k0 += kKT) {
        __syncthreads();  // every warp is done with the previous tile
        for (int i = threadIdx.x; i < kKT * D; i += blockDim.x) {
            const int sk = k0 + i / D, col = i % D;
            const size_t row = (size_t)(first + (sk < T ? sk : T - 1)) * stride + col;
            ks[i] = kbase[row];
            vs[i] = vbase[row];
        }
        __syncthreads();
        if (!active) continue;
        for (int s0 = k0; s0 < k0 + kKT && s0 <= t; s0 += PB) {
            float kv[PB][DPL], vv[PB][DPL];
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                const int sk = (s0 + b <= t ? s0 + b : t) - k0;
#pragma unroll
                for (int j = 0; j < DPL; ++j) {
                    kv[b][j] = ks[sk * D + lane + 32 * j];
                    vv[b][j] = vs[sk * D + lane + 32 * j];
                }
            }
            const bool valid = s0 + my_b <= t;
#pragma unroll
            for (int i = 0; i < R; ++i) {
                float sc[PB];
#pragma unroll
                for (int b = 0; b < PB; ++b) {
                    float x = 0.f;
#pragma unroll
                    for (int j = 0; j < DPL; ++j) x = fmaf(q[i][j], kv[b][j], x);
                    sc[b] = x;
                }
#pragma unroll
                for (int cnt = PB, off = 16; cnt > 1; cnt >>= 1, off >>= 1) {
                    const bool up = (lane & off) != 0;
#pragma unroll
                    for (int e = 0; e < cnt / 2; ++e) {
                        const float keep = up ? sc[e + cnt / 2] : sc[e];
                        const float send = up ? sc[e] : sc[e + cnt / 2];
                        sc[e] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                    }
                }
                for (int off = LPV / 2; off > 0; off >>= 1) sc[0] += __shfl_xor_sync(0xffffffffu, sc[0], off);
                const float sv = valid ? sc[0] * scale : -INFINITY;
                float mb = sv;
                for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
                const float mn = fmaxf(mx[i], mb);
                const float carry = expf(mx[i] - mn);
                const float p = valid ? expf(sv - mn) : 0.f;
                float ps = (lane % LPV) == 0 ? p : 0.f;
                for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                l[i] = l[i] * carry + ps;
#pragma unroll
                for (int j = 0; j < DPL; ++j) acc[i][j] *= carry;
#pragma unroll
                for (int b = 0; b < PB; ++b) {
                    const float pb = __shfl_sync(0xffffffffu, p, b * LPV);
#pragma unroll
                    for (int j = 0; j < DPL; ++j) acc[i][j] = fmaf(pb, vv[b][j], acc[i][j]);
                }
                mx[i] = mn;
            }
        }
    }
    if (!active) return;
    const int m = first + t;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const size_t o = (size_t)m * QH * D + (size_t)(g * R + i) * D;
#pragma unroll
        for (int j = 0; j < DPL; ++j) split_store(hi, lo, o + lane + 32 * j, acc[i][j] / l[i]);
    }
}

// ---- tensor-core attention for head_dim 128 -------------------------------
// Flash-style causal attention on mma.sync (bf16 inputs, f32 accumulation): a
// block takes one case, one KV group and 16 query positions, one warp per query
// head of the group.  f32 operands enter as two bf16 terms (hi + lo, 16
// significant bits), and each product is formed as hi.hi + hi.lo + lo.hi, so S =
// Q K^T and O = P V keep about 16 bits like the batched GEMMs.  K and V^T tiles of
// kFaKeys keys are staged in shared memory once per block (split into hi/lo) and
// serve every warp; S stays in registers and becomes the A operand of P V
// directly (the m16n8 accumulator layout is the m16k16 operand layout).  The
// online softmax (running row maximum and sum, rescaled output) follows
// kernels/ops.py:88-99 per key tile.
constexpr int kFaD = 128;
constexpr int kFaKeys = 64;
constexpr int kFaKStride = kFaD + 8;     // bf16 per staged K row (padding: conflict-free fragment loads)
constexpr int kFaVStride = kFaKeys + 8;  // bf16 per staged V^T row

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo_half, __nv_bfloat16 hi_half) {
    return (uint32_t)__bfloat16_as_ushort(lo_half) | ((uint32_t)__bfloat16_as_ushort(hi_half) << 16);
}
// (x, y) -> packed bf16 hi terms and lo terms
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat16 hx = __float2bfloat16_rn(x), hy = __float2bfloat16_rn(y);
    hi = pack_bf16x2(hx, hy);
    lo = pack_bf16x2(__float2bfloat16_rn(x - __bfloat162float(hx)), __float2bfloat16_rn(y - __bfloat162float(hy)));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Q fragments (hi, lo) of the 16 query rows q0 .. q0 + 15 of head h (rows past T - 1
// repeat row T - 1): 8 k-steps of 16 dims.
__device__ __forceinline__ void fa_load_q(const float* qkv, size_t stride, int first, int q0, int T, int h, int r,
                                          int cq, uint32_t (&qa_hi)[8][4], uint32_t (&qa_lo)[8][4]) {
    const int ra = min(q0 + r, T - 1), rb = min(q0 + r + 8, T - 1);
    const float* qa = qkv + (size_t)(first + ra) * stride + (size_t)h * kFaD;
    const float* qb = qkv + (size_t)(first + rb) * stride + (size_t)h * kFaD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
        const int d0 = kk * 16 + cq;
        const float2 x0 = *reinterpret_cast<const float2*>(qa + d0);
        const float2 x1 = *reinterpret_cast<const float2*>(qb + d0);
        const float2 x2 = *reinterpret_cast<const float2*>(qa + d0 + 8);
        const float2 x3 = *reinterpret_cast<const float2*>(qb + d0 + 8);
        split2(x0.x, x0.y, qa_hi[kk][0], qa_lo[kk][0]);
        split2(x1.x, x1.y, qa_hi[kk][1], qa_lo[kk][1]);
        split2(x2.x, x2.y, qa_hi[kk][2], qa_lo[kk][2]);
        split2(x3.x, x3.y, qa_hi[kk][3], qa_lo[kk][3]);
    }
}

// One warp's online-softmax update of its 16 query rows q0 .. q0 + 15 by the 64 keys
// k0 .. k0 + 63, staged as K rows krow0 .. krow0 + 63 of (k_hi, k_lo) [key][kFaKStride]
// and V^T columns vcol0 .. vcol0 + 63 of (v_hi, v_lo) [dim][vstride]: S = Q K^T, the
// causal mask, the running maxima and sums, then O += P V (kernels/ops.py:88-99 per
// tile).  Groups of 8 keys past q0 + 15 (or past T) are masked for every row of the
// warp, so their S and P V products are skipped: their probabilities are exactly 0
// and their terms would add exactly 0.  q0 is the same in all lanes, as every lane
// takes part in each mma.sync.
__device__ __forceinline__ void fa_tile(const uint32_t (&qa_hi)[8][4], const uint32_t (&qa_lo)[8][4],
                                        float (&o)[16][4], float& m_a, float& m_b, float& l_a, float& l_b,
                                        const __nv_bfloat16* k_hi, const __nv_bfloat16* k_lo,
                                        const __nv_bfloat16* v_hi, const __nv_bfloat16* v_lo, int krow0, int vstride,
                                        int vcol0, int k0, int q0, int T, float scale, int r, int cq) {
    const int q_a = q0 + r, q_b = q0 + r + 8;
    const int live = min(8, (min(q0 + 16, T) - k0 + 7) >> 3);  // n-tiles some row may see
    // S = Q K^T over this tile: 8 n-tiles of 8 keys.
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        if (nt >= live) continue;
        const int key = krow0 + nt * 8 + r;  // B fragment column (key) of this lane
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int d0 = kk * 16 + cq;
            const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(k_hi + key * kFaKStride + d0);
            const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(k_hi + key * kFaKStride + d0 + 8);
            const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(k_lo + key * kFaKStride + d0);
            const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(k_lo + key * kFaKStride + d0 + 8);
            mma_bf16(sc[nt], qa_lo[kk], bh0, bh1);
            mma_bf16(sc[nt], qa_hi[kk], bl0, bl1);
            mma_bf16(sc[nt], qa_hi[kk], bh0, bh1);
        }
    }
    // causal mask, scale, running maxima of rows r and r + 8
    float tile_a = -INFINITY, tile_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int key = k0 + nt * 8 + cq + e;
            sc[nt][e] = key <= q_a && key < T ? sc[nt][e] * scale : -INFINITY;
            sc[nt][2 + e] = key <= q_b && key < T ? sc[nt][2 + e] * scale : -INFINITY;
            tile_a = fmaxf(tile_a, sc[nt][e]);
            tile_b = fmaxf(tile_b, sc[nt][2 + e]);
        }
    }
    tile_a = fmaxf(tile_a, __shfl_xor_sync(0xffffffffu, tile_a, 1));
    tile_a = fmaxf(tile_a, __shfl_xor_sync(0xffffffffu, tile_a, 2));
    tile_b = fmaxf(tile_b, __shfl_xor_sync(0xffffffffu, tile_b, 1));
    tile_b = fmaxf(tile_b, __shfl_xor_sync(0xffffffffu, tile_b, 2));
    const float mn_a = fmaxf(m_a, tile_a), mn_b = fmaxf(m_b, tile_b);
    const float carry_a = expf(m_a - mn_a), carry_b = expf(m_b - mn_b);
    m_a = mn_a;
    m_b = mn_b;
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            sc[nt][e] = expf(sc[nt][e] - mn_a);
            sc[nt][2 + e] = expf(sc[nt][2 + e] - mn_b);
            sum_a += sc[nt][e];
            sum_b += sc[nt][2 + e];
        }
    }
    l_a = l_a * carry_a + sum_a;
    l_b = l_b * carry_b + sum_b;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
        o[n][0] *= carry_a;
        o[n][1] *= carry_a;
        o[n][2] *= carry_b;
        o[n][3] *= carry_b;
    }
    // O += P V: P's accumulator tiles (2j, 2j + 1) form the A operand of k-step j.
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (2 * j >= live) continue;  // P is exactly 0 on these keys
        uint32_t pa_hi[4], pa_lo[4];
        split2(sc[2 * j][0], sc[2 * j][1], pa_hi[0], pa_lo[0]);
        split2(sc[2 * j][2], sc[2 * j][3], pa_hi[1], pa_lo[1]);
        split2(sc[2 * j + 1][0], sc[2 * j + 1][1], pa_hi[2], pa_lo[2]);
        split2(sc[2 * j + 1][2], sc[2 * j + 1][3], pa_hi[3], pa_lo[3]);
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            const int d = n * 8 + r;  // B fragment column (dim) of this lane
            const int kb = vcol0 + j * 16 + cq;
            const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(v_hi + d * vstride + kb);
            const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(v_hi + d * vstride + kb + 8);
            const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(v_lo + d * vstride + kb);
            const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(v_lo + d * vstride + kb + 8);
            mma_bf16(o[n], pa_lo, bh0, bh1);
            mma_bf16(o[n], pa_hi, bl0, bl1);
            mma_bf16(o[n], pa_hi, bh0, bh1);
        }
    }
}

// The attention output of one warp's 16 query rows, normalised, as bf16 hi/lo.
__device__ __forceinline__ void fa_store(const float (&o)[16][4], float l_a, float l_b, int first, int q0, int T,
                                         int QH, int h, int r, int cq, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int q_a = q0 + r, q_b = q0 + r + 8;
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
#pragma unroll
    for (int n = 0; n < 16; ++n) {
        const int d = n * 8 + cq;
        if (q_a < T) {
            const size_t at = (size_t)(first + q_a) * QH * kFaD + (size_t)h * kFaD + d;
            uint32_t hh, ll;
            split2(o[n][0] / l_a, o[n][1] / l_a, hh, ll);
            *reinterpret_cast<uint32_t*>(hi + at) = hh;
            *reinterpret_cast<uint32_t*>(lo + at) = ll;
        }
        if (q_b < T) {
            const size_t at = (size_t)(first + q_b) * QH * kFaD + (size_t)h * kFaD + d;
            uint32_t hh, ll;
            split2(o[n][2] / l_b, o[n][3] / l_b, hh, ll);
            *reinterpret_cast<uint32_t*>(hi + at) = hh;
            *reinterpret_cast<uint32_t*>(lo + at) = ll;
        }
    }
}

// Keys src0 .. src0 + n - 1 (rows past T - 1 repeat row T - 1) of one case and KV group,
// split into bf16 hi/lo: K rows from krow0 of (k_hi, k_lo) [key][kFaKStride], V^T
// columns from vcol0 of (v_hi, v_lo) [dim][vstride].  All threads of the block.
__device__ __forceinline__ void fa_stage(const float* kbase, const float* vbase, size_t stride, int first, int src0,
                                         int n, int T, __nv_bfloat16* k_hi, __nv_bfloat16* k_lo,
                                         __nv_bfloat16* v_hi, __nv_bfloat16* v_lo, int krow0, int vstride,
                                         int vcol0) {
    for (int i = threadIdx.x; i < n * (kFaD / 2); i += blockDim.x) {
        const int key = i / (kFaD / 2), d = (i % (kFaD / 2)) * 2;
        const int src = first + min(src0 + key, T - 1);
        const float2 kv = *reinterpret_cast<const float2*>(kbase + (size_t)src * stride + d);
        const float2 vv = *reinterpret_cast<const float2*>(vbase + (size_t)src * stride + d);
        uint32_t kh, kl;
        split2(kv.x, kv.y, kh, kl);
        *reinterpret_cast<uint32_t*>(k_hi + (krow0 + key) * kFaKStride + d) = kh;
        *reinterpret_cast<uint32_t*>(k_lo + (krow0 + key) * kFaKStride + d) = kl;
        const __nv_bfloat16 v0 = __float2bfloat16_rn(vv.x), v1 = __float2bfloat16_rn(vv.y);
        v_hi[d * vstride + vcol0 + key] = v0;
        v_hi[(d + 1) * vstride + vcol0 + key] = v1;
        v_lo[d * vstride + vcol0 + key] = __float2bfloat16_rn(vv.x - __bfloat162float(v0));
        v_lo[(d + 1) * vstride + vcol0 + key] = __float2bfloat16_rn(vv.y - __bfloat162float(v1));
    }
}

__global__ void __launch_bounds__(256, 1) causal_attention_mma_kernel(const float* __restrict__ qkv, int M, int T,
                                                                     int QH, int KVH, float scale,
                                                                     __nv_bfloat16* __restrict__ hi,
                                                                     __nv_bfloat16* __restrict__ lo) {
    extern __shared__ __align__(16) __nv_bfloat16 fa_smem[];
    __nv_bfloat16* k_hi = fa_smem;                        // [kFaKeys][kFaKStride]
    __nv_bfloat16* k_lo = k_hi + kFaKeys * kFaKStride;
    __nv_bfloat16* v_hi = k_lo + kFaKeys * kFaKStride;    // V^T [kFaD][kFaVStride]
    __nv_bfloat16* v_lo = v_hi + kFaD * kFaVStride;
    const int R = QH / KVH;
    const int qtiles = (T + 15) / 16;
    int bid = blockIdx.x;
    const int qt = bid % qtiles;
    bid /= qtiles;
    const int g = bid % KVH, c = bid / KVH;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g * R + warp;
    const int first = c * T, q0 = qt * 16;
    const int r = lane >> 2, cq = (lane & 3) * 2;  // fragment row and column pair
    const size_t stride = (size_t)(QH + 2 * KVH) * kFaD;
    const float* kbase = qkv + (size_t)QH * kFaD + (size_t)g * kFaD;
    const float* vbase = kbase + (size_t)KVH * kFaD;
    uint32_t qa_hi[8][4], qa_lo[8][4];
    fa_load_q(qkv, stride, first, q0, T, h, r, cq, qa_hi, qa_lo);
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;  // rows r and r + 8
    const int key_end = min(T, q0 + 16);
    for (int k0 = 0; k0 < key_end; k0 += kFaKeys) {
        __syncthreads();  // the previous tile is no longer read
        fa_stage(kbase, vbase, stride, first, k0, kFaKeys, T, k_hi, k_lo, v_hi, v_lo, 0, kFaVStride, 0);
        __syncthreads();
        if (warp >= R) continue;
        fa_tile(qa_hi, qa_lo, o, m_a, m_b, l_a, l_b, k_hi, k_lo, v_hi, v_lo, 0, kFaVStride, 0, k0, q0, T, scale, r,
                cq);
    }
    if (warp >= R) return;
    fa_store(o, l_a, l_b, first, q0, T, QH, h, r, cq, hi, lo);
}

// Short cases (T <= kFaShortKeys, the scoring workload's cases): one block per case
// and KV group stages all of the case's keys once, and its eight warps take the
// (16-query tile, query head) tasks of the group in turn, with the per-tile
// arithmetic of causal_attention_mma_kernel (so the results are the same bits).
constexpr int kFaShortKeys = 128;
constexpr int kFaShortVStride = kFaShortKeys + 8;

__global__ void __launch_bounds__(256, 1) causal_attention_mma_case_kernel(const float* __restrict__ qkv, int M,
                                                                          int T, int QH, int KVH, float scale,
                                                                          __nv_bfloat16* __restrict__ hi,
                                                                          __nv_bfloat16* __restrict__ lo) {
    extern __shared__ __align__(16) __nv_bfloat16 fa_smem[];
    __nv_bfloat16* k_hi = fa_smem;                             // [kFaShortKeys][kFaKStride]
    __nv_bfloat16* k_lo = k_hi + kFaShortKeys * kFaKStride;
    __nv_bfloat16* v_hi = k_lo + kFaShortKeys * kFaKStride;    // V^T [kFaD][kFaShortVStride]
    __nv_bfloat16* v_lo = v_hi + kFaD * kFaShortVStride;
    const int R = QH / KVH;
    const int qtiles = (T + 15) / 16;
    const int g = blockIdx.x % KVH, c = blockIdx.x / KVH;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    const int first = c * T;
    const int r = lane >> 2, cq = (lane & 3) * 2;
    const size_t stride = (size_t)(QH + 2 * KVH) * kFaD;
    const float* kbase = qkv + (size_t)QH * kFaD + (size_t)g * kFaD;
    const float* vbase = kbase + (size_t)KVH * kFaD;
    const int staged = ((T + kFaKeys - 1) / kFaKeys) * kFaKeys;  // whole 64-key tiles, <= kFaShortKeys
    fa_stage(kbase, vbase, stride, first, 0, staged, T, k_hi, k_lo, v_hi, v_lo, 0, kFaShortVStride, 0);
    __syncthreads();
    for (int task = warp; task < qtiles * R; task += warps) {  // the same in all lanes of a warp
        const int qt = task / R, h = g * R + task % R;
        const int q0 = qt * 16;
        uint32_t qa_hi[8][4], qa_lo[8][4];
        fa_load_q(qkv, stride, first, q0, T, h, r, cq, qa_hi, qa_lo);
        float o[16][4];
#pragma unroll
        for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
        const int key_end = min(T, q0 + 16);
        for (int k0 = 0; k0 < key_end; k0 += kFaKeys)
            fa_tile(qa_hi, qa_lo, o, m_a, m_b, l_a, l_b, k_hi, k_lo, v_hi, v_lo, k0, kFaShortVStride, k0, k0, q0, T,
                    scale, r, cq);
        fa_store(o, l_a, l_b, first, q0, T, QH, h, r, cq, hi, lo);
    }
}

constexpr size_t kFaShortSmem = (size_t)(2 * kFaShortKeys * kFaKStride + 2 * kFaD * kFaShortVStride) * 2;

constexpr size_t kFaSmem = (size_t)(2 * kFaKeys * kFaKStride + 2 * kFaD * kFaVStride) * 2;

// Tensor-core attention when head_dim is 128 and a group has at most eight query heads.
bool launch_attention_mma(cudaStream_t s, const float* qkv, int M, int T, int QH, int KVH, int D, float scale,
                          __nv_bfloat16* hi, __nv_bfloat16* lo) {
    if (D != kFaD || QH % KVH != 0 || QH / KVH > 8 || M % T != 0) return false;
    // set on every call: the attribute belongs to the current device
    if (cudaFuncSetAttribute((const void*)causal_attention_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kFaSmem) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    const int R = QH / KVH;
    // short cases: one block per case and KV group (LSX_ATTENTION_PER_CASE=0: per 16-query tile)
    const char* per_case = getenv("LSX_ATTENTION_PER_CASE");
    if (T <= kFaShortKeys && !(per_case && per_case[0] == '0') &&
        cudaFuncSetAttribute((const void*)causal_attention_mma_case_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaShortSmem) == cudaSuccess) {
        causal_attention_mma_case_kernel<<<(M / T) * KVH, 256, kFaShortSmem, s>>>(qkv, M, T, QH, KVH, scale, hi,
                                                                                  lo);
        return true;
    }
    (void)cudaGetLastError();
    const int blocks = (M / T) * KVH * ((T + 15) / 16);
    causal_attention_mma_kernel<<<blocks, 32 * std::max(R, 4), kFaSmem, s>>>(qkv, M, T, QH, KVH, scale, hi, lo);
    return true;
}

// Tiled attention when the group ratio has an instantiation (q and the
// accumulators of all R heads stay in registers); false otherwise.
template <int DPL>
bool launch_attention_tiled(cudaStream_t s, const float* qkv, int M, int T, int QH, int KVH, float scale,
                            __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int R = QH / KVH;
    const int blocks = (M / T) * KVH * ((T + kQT - 1) / kQT);
    if (M % T != 0 || QH % KVH != 0) return false;
    if (R == 1) causal_attention_tiled_kernel<DPL, 1><<<blocks, 32 * kQT, 0, s>>>(qkv, M, T, QH, KVH, scale, hi, lo);
    else if (R == 2) causal_attention_tiled_kernel<DPL, 2><<<blocks, 32 * kQT, 0, s>>>(qkv, M, T, QH, KVH, scale, hi, lo);
    else if (R == 4 && DPL <= 4)
        causal_attention_tiled_kernel<DPL, 4><<<blocks, 32 * kQT, 0, s>>>(qkv, M, T, QH, KVH, scale, hi, lo);
    else return false;
    return true;
}

// A planes of act(gate) * up from the interleaved [g0 u0 g1 u1 ...] rows.
// Four features per thread (two 16-byte loads, 8-byte plane stores) when I % 4 == 0.
__global__ void gated_planes_kernel(const float* __restrict__ gu, size_t total, int I, int kind,
                                    __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t step = (size_t)gridDim.x * blockDim.x;
    if ((I & 3) == 0) {
        const size_t quads = total >> 2;
        const int per_row = I >> 2;
        for (size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x; q < quads; q += step) {
            const size_t m = q / per_row;
            const int f = (int)(q - m * per_row) * 4;
            const float4* src = reinterpret_cast<const float4*>(gu + m * 2 * I + 2 * f);
            const float4 a = src[0], b = src[1];  // (g0 u0 g1 u1) (g2 u2 g3 u3)
            const float v[4] = {act_fn(a.x, kind) * a.y, act_fn(a.z, kind) * a.w, act_fn(b.x, kind) * b.y,
                                act_fn(b.z, kind) * b.w};
            __align__(8) __nv_bfloat16 h4[4], l4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h4[e] = __float2bfloat16_rn(v[e]);
                l4[e] = __float2bfloat16_rn(v[e] - __bfloat162float(h4[e]));
            }
            const size_t o = m * I + f;
            *reinterpret_cast<uint2*>(hi + o) = *reinterpret_cast<const uint2*>(h4);
            *reinterpret_cast<uint2*>(lo + o) = *reinterpret_cast<const uint2*>(l4);
        }
        return;
    }
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
        const size_t m = i / I, f = i % I;
        const float2 v = *reinterpret_cast<const float2*>(gu + m * 2 * I + 2 * f);
        split_store(hi, lo, i, act_fn(v.x, kind) * v.y);
    }
}

// Appends every row's k (after QK-norm and RoPE) and v to the f32 KV cache at
// position = row (kernels/ops.py:69-73 for a whole prompt).
// Row m = c T + t goes to position pos0 + t of case c's cache (case_stride floats
// apart; one case: case_stride is unused); element d of KV group g of position p
// sits at g group_stride + p pos_stride + d. The engine's cache is position-major
// (group_stride D, pos_stride KVH D); the caches of batched generation are
// group-major (group_stride capacity D, pos_stride D).
__global__ void kv_store_kernel(const float* __restrict__ qkv, size_t total, int QH, int KVH, int D,
                                float* __restrict__ keys, float* __restrict__ values, int T, int pos0,
                                size_t case_stride, size_t group_stride, size_t pos_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t kw = (size_t)KVH * D, stride = (size_t)(QH + 2 * KVH) * D;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / kw, e = i % kw;
        const size_t c = m / T, t = m % T;
        const size_t dst = c * case_stride + (e / D) * group_stride + (pos0 + t) * pos_stride + e % D;
        keys[dst] = qkv[m * stride + (size_t)QH * D + e];
        values[dst] = qkv[m * stride + (size_t)(QH + KVH) * D + e];
    }
}

// ---- batched decode: one new row per sequence, attention over its cache ----
// The caches are group-major: case c's KV group g holds its positions' D-float rows
// contiguously (group_stride = case_stride / KVH floats apart), so a block's walk
// reads one contiguous stretch of memory.
// Block (case c, KV group g, split s) takes positions [s chunk, (s + 1) chunk) of
// 0 .. pos of case c's cache. Each half-warp is one walker: walker w of the block
// takes positions start + w, start + w + walkers, ...; lane hl of a half owns the
// D / 16 elements 64 u + 4 hl .. 64 u + 4 hl + 3 (u < D / 64) of a row, so every
// 16-byte copy or load instruction of the half covers 256 contiguous bytes, and one
// 4-step butterfly reduces two positions' dot products at once. Each walker carries the R query heads of the group (the K
// and V rows are read once for all of them) with a running softmax per head
// (kernels/ops.py:88-99); the walkers' states merge in shared memory, and the block
// writes per head a partial state (max, sum, unnormalised output[D]) for
// cached_attention_merge_kernel.
//
// A warp keeps its next positions' K and V rows in flight with cp.async into its
// own ring in shared memory; a lane copies and reads back only its own elements,
// so the ring needs no cross-lane synchronisation.
template <int DPL>
struct AttentionWalk {
    static constexpr int kWarps = DPL == 8 ? 4 : 8;
    // ring slots of two positions per warp: 96 KB of ring per block (dynamic shared
    // memory), so each warp has ten or more rows of K and V in flight
    static constexpr int kDepth = 98304 / (kWarps * 16 * DPL * 32);
};

template <int DPL, int R>
constexpr size_t attention_walk_smem() {
    constexpr int D = DPL * 32, W = AttentionWalk<DPL>::kWarps;
    constexpr size_t ring = (size_t)W * AttentionWalk<DPL>::kDepth * 4 * D, state = (size_t)2 * W * R * (D + 2);
    return 4 * (ring > state ? ring : state);
}

// this lane's E floats of one row (four at every 64 floats from src), global ->
// shared at the same offsets from dst, asynchronously
template <int E>
__device__ __forceinline__ void lane_row_async(float* dst, const float* src) {
    static_assert(E % 4 == 0, "16-byte copies");
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
#pragma unroll
    for (int u = 0; u < E / 4; ++u)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + 256 * u), "l"(src + 64 * u) : "memory");
}

__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// this lane's E floats of one row (four at every 64 floats), element order as copied
template <int E>
__device__ __forceinline__ void lane_row_load(const float* src, float (&x)[E]) {
#pragma unroll
    for (int u = 0; u < E / 4; ++u) {
        const float4 t = *reinterpret_cast<const float4*>(src + 64 * u);
        x[4 * u] = t.x;
        x[4 * u + 1] = t.y;
        x[4 * u + 2] = t.z;
        x[4 * u + 3] = t.w;
    }
}

// Row offset of a lane's local element e (0 <= e < E): lane hl owns 64 u + 4 hl + r.
__device__ __forceinline__ int lane_elem(int e, int hl) { return ((e >> 2) << 6) + 4 * hl + (e & 3); }

// Packed f32 pairs: Blackwell's fma.rn.f32x2 does two multiply-adds per instruction.
__device__ __forceinline__ unsigned long long pair_of(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void pair_fma(unsigned long long& acc, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float pair_lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float pair_hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }

// Sums CNT per-lane values over the 16 lanes of a half-warp at once: each halving
// round exchanges half of the values with the lane OFF apart, so after log2(CNT)
// rounds each lane carries one value and the plain rounds complete its sum.  Lane
// hl of the half ends with the total of value hl / (16 / CNT).
template <int CNT, int OFF>
struct HalfReduce {
    static __device__ __forceinline__ void run(float* v, int lane) {
        if constexpr (OFF > 0) {
            if constexpr (CNT > 1) {
                constexpr int half = CNT / 2;
                const bool up = (lane & OFF) != 0;
#pragma unroll
                for (int i = 0; i < half; ++i) {
                    const float keep = up ? v[i + half] : v[i];
                    const float send = up ? v[i] : v[i + half];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
                }
                HalfReduce<half, OFF / 2>::run(v, lane);
            } else {
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
                HalfReduce<1, OFF / 2>::run(v, lane);
            }
        }
    }
};

template <int DPL, int R>
__global__ void __launch_bounds__(32 * AttentionWalk<DPL>::kWarps) cached_attention_part_kernel(
    const float* __restrict__ qkv, const float* __restrict__ keys, const float* __restrict__ values, int QH, int KVH,
    int pos, size_t case_stride, int splits, float scale, float* __restrict__ part) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int D = DPL * 32, E = D / 16, W = AttentionWalk<DPL>::kWarps, S = AttentionWalk<DPL>::kDepth;
    constexpr int kWalkers = 2 * W;
    extern __shared__ __align__(16) float smem[];  // attention_walk_smem<DPL, R>() bytes
    const int s = blockIdx.x % splits, g = (blockIdx.x / splits) % KVH, c = blockIdx.x / (splits * KVH);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
    const int walker = 2 * warp + half;
    const int n = pos + 1, chunk = (n + splits - 1) / splits;
    const int t0 = s * chunk, t1 = min(n, t0 + chunk);
    const size_t group = (size_t)c * case_stride + (size_t)g * (case_stride / KVH);
    const float* kb = keys + group + hl * 4;
    const float* vb = values + group + hl * 4;
    const float* qrow = qkv + (size_t)c * (QH + 2 * KVH) * D;
    // ring slot: [K of the two halves' positions | V of the same], D floats each
    float* ring = smem + warp * (S * 4 * D) + half * D + hl * 4;
    // q and the output accumulators as packed pairs of this lane's E elements
    unsigned long long q2[R][E / 2], acc2[R][E / 2];
    float m[R], l[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
        const float* qh = qrow + (size_t)(g * R + i) * D;
#pragma unroll
        for (int j = 0; j < E / 2; ++j) {
            q2[i][j] = pair_of(qh[lane_elem(2 * j, hl)], qh[lane_elem(2 * j + 1, hl)]);
            acc2[i][j] = 0ull;
        }
    }
    const int first = t0 + walker;
    const int count = first < t1 ? (t1 - first + kWalkers - 1) / kWalkers : 0;
    const int trips = max(count, __shfl_xor_sync(0xffffffffu, count, 16));  // uniform over the warp
#pragma unroll
    for (int i = 0; i < S - 1; ++i) {
        if (i < count) {
            const size_t row = (size_t)(first + i * kWalkers) * D;
            lane_row_async<E>(ring + i * 4 * D, kb + row);
            lane_row_async<E>(ring + i * 4 * D + 2 * D, vb + row);
        }
        async_commit();
    }
    int rd = 0, wr = S - 1;  // ring slots of position i and of position i + S - 1
    for (int i = 0; i < trips; ++i) {
        if (i + S - 1 < count) {
            const size_t row = (size_t)(first + (i + S - 1) * kWalkers) * D;
            lane_row_async<E>(ring + wr * 4 * D, kb + row);
            lane_row_async<E>(ring + wr * 4 * D + 2 * D, vb + row);
        }
        async_commit();
        async_wait<S - 1>();  // position i's rows have landed
        const bool live = i < count;  // the same in all lanes of a half
        const int slot = rd;
        rd = rd + 1 == S ? 0 : rd + 1;
        wr = wr + 1 == S ? 0 : wr + 1;
        float k[E], v[E];
        lane_row_load<E>(ring + slot * 4 * D, k);
        lane_row_load<E>(ring + slot * 4 * D + 2 * D, v);
        // the R heads' partial dots, then one transposed butterfly over the half:
        // lane hl holds head hl / (16 / R)'s score, which the other lanes read back
        float sc[R];
#pragma unroll
        for (int h = 0; h < R; ++h) {
            unsigned long long a = 0ull;
#pragma unroll
            for (int j = 0; j < E / 2; ++j) pair_fma(a, q2[h][j], pair_of(k[2 * j], k[2 * j + 1]));
            sc[h] = pair_lo(a) + pair_hi(a);
        }
        HalfReduce<R, 8>::run(sc, hl);
        const float mine = sc[0];
#pragma unroll
        for (int h = 0; h < R; ++h) sc[h] = __shfl_sync(0xffffffffu, mine, (lane & 16) | (h * (16 / R)));
        if (live) {  // the same in all lanes of a half
#pragma unroll
            for (int h = 0; h < R; ++h) {
                const float sv = sc[h] * scale;
                if (sv > m[h]) {
                    const float carry = expf(m[h] - sv);
                    l[h] *= carry;
                    const unsigned long long c2 = pair_of(carry, carry);
#pragma unroll
                    for (int j = 0; j < E / 2; ++j) {
                        unsigned long long z = 0ull;
                        pair_fma(z, acc2[h][j], c2);
                        acc2[h][j] = z;
                    }
                    m[h] = sv;
                }
                const float p = expf(sv - m[h]);
                l[h] += p;
                const unsigned long long p2 = pair_of(p, p);
#pragma unroll
                for (int j = 0; j < E / 2; ++j) pair_fma(acc2[h][j], p2, pair_of(v[2 * j], v[2 * j + 1]));
            }
        }
    }
    async_wait<0>();
    __syncthreads();  // every warp is done with its ring: the states reuse the space
    float* st = smem;  // [walker][R][D + 2]
#pragma unroll
    for (int i = 0; i < R; ++i) {
        float* w = st + (walker * R + i) * (D + 2);
        if (hl == 0) {
            w[0] = m[i];
            w[1] = l[i];
        }
#pragma unroll
        for (int j = 0; j < E / 2; ++j) {
            w[2 + lane_elem(2 * j, hl)] = pair_lo(acc2[i][j]);
            w[2 + lane_elem(2 * j + 1, hl)] = pair_hi(acc2[i][j]);
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < R * (D + 2); idx += blockDim.x) {
        const int i = idx / (D + 2), e = idx % (D + 2);
        float M = -INFINITY;
        for (int w = 0; w < kWalkers; ++w) M = fmaxf(M, st[(w * R + i) * (D + 2)]);
        float val;
        if (e == 0) {
            val = M;
        } else {
            val = 0.f;
            for (int w = 0; w < kWalkers; ++w) {
                const float* ws = st + (w * R + i) * (D + 2);
                if (ws[0] != -INFINITY) val = fmaf(ws[e], expf(ws[0] - M), val);
            }
        }
        part[(((size_t)c * QH + g * R + i) * splits + s) * (D + 2) + e] = val;
    }
}

// Per (case, query head): merges the splits' partial states and writes the output as
// the bf16 hi/lo A planes of the o projection, row c.
template <int DPL>
__global__ void cached_attention_merge_kernel(const float* __restrict__ part, int QH, int splits,
                                              __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int D = DPL * 32;
    const int c = blockIdx.x / QH, h = blockIdx.x % QH;
    const float* p = part + ((size_t)c * QH + h) * splits * (D + 2);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float M = -INFINITY;
        for (int s = 0; s < splits; ++s) M = fmaxf(M, p[(size_t)s * (D + 2)]);
        float L = 0.f, O = 0.f;
        for (int s = 0; s < splits; ++s) {
            const float* q = p + (size_t)s * (D + 2);
            if (q[0] == -INFINITY) continue;
            const float ex = expf(q[0] - M);
            L = fmaf(q[1], ex, L);
            O = fmaf(q[2 + d], ex, O);
        }
        split_store(hi, lo, ((size_t)c * QH + h) * D + d, O / L);
    }
}

// First argmax of each logit row (src/diagnosis.rs:58-70) into tokens[row] and
// history[row]; a non-finite logit raises status[1].
__global__ void __launch_bounds__(1024) row_argmax_tokens_kernel(const float* __restrict__ logits, int V,
                                                                 uint32_t* __restrict__ tokens,
                                                                 uint32_t* __restrict__ history, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long kbest[32];
    const float* z = logits + (size_t)blockIdx.x * V;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
    unsigned long long best = 0ull;
    bool bad = false;
    for (int j = tid; j < V; j += blockDim.x) {
        const unsigned long long k = pack_arg(z[j], (uint32_t)j);
        best = k > best ? k : best;
        bad |= !isfinite(z[j]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long b2 = __shfl_xor_sync(0xffffffffu, best, o);
        best = b2 > best ? b2 : best;
    }
    if (lane == 0) kbest[warp] = best;
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&status[1], 1);
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < warps; ++w) best = kbest[w] > best ? kbest[w] : best;
        const uint32_t token = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
        tokens[blockIdx.x] = token;
        history[blockIdx.x] = token;
    }
}

// Per logit row: attribution::loss (src/attribution.rs:49-60, f64 logsumexp minus
// the target's logit), the first argmax (src/diagnosis.rs:58-70) and the target
// margin f64(z_t) - f64(max over j != t, lowest index on ties) (src/diagnosis.rs:
// 71-80, 490-492), from packed (value, index) keys.
__global__ void __launch_bounds__(1024) row_scores_kernel(const float* __restrict__ logits, int V,
                                                          const uint32_t* __restrict__ targets,
                                                          double* __restrict__ nll, uint32_t* __restrict__ argmax,
                                                          double* __restrict__ margin) {
    __shared__ unsigned long long kbest[32], kother[32];
    __shared__ double red[32];
    const float* z = logits + (size_t)blockIdx.x * V;
    const uint32_t t = targets[blockIdx.x];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
    unsigned long long best = 0ull, other = 0ull;
    for (int j = tid; j < V; j += blockDim.x) {
        const unsigned long long k = pack_arg(z[j], (uint32_t)j);
        best = k > best ? k : best;
        if ((uint32_t)j != t) other = k > other ? k : other;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long b2 = __shfl_xor_sync(0xffffffffu, best, o);
        const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, other, o);
        best = b2 > best ? b2 : best;
        other = o2 > other ? o2 : other;
    }
    if (lane == 0) {
        kbest[warp] = best;
        kother[warp] = other;
    }
    __syncthreads();
    best = kbest[0];
    other = kother[0];
    for (int w = 1; w < warps; ++w) {
        best = kbest[w] > best ? kbest[w] : best;
        other = kother[w] > other ? kother[w] : other;
    }
    const double top = (double)z[0xffffffffu - (uint32_t)(best & 0xffffffffull)];
    double sum = 0.0;
    for (int j = tid; j < V; j += blockDim.x) sum += exp((double)z[j] - top);
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    __syncthreads();
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    if (tid == 0) {
        double total = 0.0;
        for (int w = 0; w < warps; ++w) total += red[w];
        const double zt = (double)z[t];
        nll[blockIdx.x] = top + log(total) - zt;
        argmax[blockIdx.x] = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
        margin[blockIdx.x] = other ? zt - (double)z[0xffffffffu - (uint32_t)(other & 0xffffffffull)] : INFINITY;
    }
}

}  // namespace

BatchedScorer::~BatchedScorer() {
    if (block_) cudaFree(block_);
    if (batch_cache_) cudaFree(batch_cache_);
}

bool BatchedScorer::eligible(const FusedConfig& c, std::string* why) {
    const int dpl = c.head_dim / 32;
    if (c.head_dim % 32 != 0 || (dpl != 2 && dpl != 4 && dpl != 8)) {
        if (why) *why = "head_dim must be 64, 128 or 256";
        return false;
    }
    if (c.rotary != c.head_dim || c.interleaved) {
        if (why) *why = "only full-width rotate-half RoPE";
        return false;
    }
    if (c.hidden % 8 != 0 || c.intermediate % 8 != 0 || c.kvheads <= 0 || c.qheads % c.kvheads != 0) {
        if (why) *why = "widths must be multiples of 8";
        return false;
    }
    return true;
}

int BatchedScorer::reserve(size_t rows, size_t scored, size_t T) {
    const FusedConfig& c = config_;
    const size_t H = c.hidden, V = c.vocab, D = c.head_dim;
    const size_t qkvw = (size_t)(c.qheads + 2 * c.kvheads) * D;
    const size_t widest = std::max(H, std::max((size_t)c.qheads * D, (size_t)c.intermediate));
    auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
    Layout L{};
    size_t at = 0;
    L.x = at;
    at = up(at + rows * H * 4);
    L.work = at;  // [q; k; v] rows, then gate/up rows
    at = up(at + rows * std::max(std::max(qkvw, 2 * (size_t)c.intermediate), H) * 4);
    L.planes = at;
    at = up(at + 2 * std::max(rows, scored) * widest * 2);
    L.logits = at;
    at = up(at + scored * V * 4);
    L.rope = at;
    at = up(at + T * (D / 2) * 8);
    L.tokens = at;
    at = up(at + rows * 4);
    L.targets = at;
    at = up(at + scored * 4);
    L.rows = at;
    at = up(at + scored * 4);
    L.nll = at;
    at = up(at + scored * 8);
    L.argmax = at;
    at = up(at + scored * 4);
    L.margin = at;
    at = up(at + scored * 8);
    L.status = at;
    at = up(at + 16);
    L.total = at;
    if (L.total > capacity_) {
        if (block_) cudaFree(block_);
        block_ = nullptr;
        capacity_ = 0;
        LSX_CUDA(cudaMalloc(&block_, L.total), "batched scoring buffers");
        capacity_ = L.total;
    }
    layout_ = L;
    return LSX_OK;
}

int BatchedScorer::build(lsx_ctx* ctx, const FusedConfig& config, const std::vector<FusedLayer>& layers) {
    std::string why;
    if (!eligible(config, &why)) return fail(LSX_E_UNSUPPORTED, "batched scoring: " + why);
    ctx_ = ctx;
    config_ = config;
    layers_ = layers;
    return LSX_OK;
}

int BatchedScorer::prefill(const uint32_t* tokens, size_t n) {
    LSX_ENSURE(n > 0 && n <= (size_t)config_.capacity, "check the prefill length");
    return run(tokens, 1, n, 0, 0, nullptr, nullptr, Outputs{}, true);
}

// Launches `kernel` on `s` as a programmatic dependent of the kernel before it: its
// CTAs may be scheduled while that kernel finishes, and its first instruction waits
// for it (pdl_wait), so only the launch latency overlaps.  Used for the chain of
// small kernels of a batched decode step.
template <typename... Params, typename... Args>
static cudaError_t chain_launch(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int DPL>
static bool launch_cached_attention(cudaStream_t s, const float* qkv, const float* keys, const float* values, int B,
                                    int QH, int KVH, int pos, size_t case_stride, int splits, float scale,
                                    float* part, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int R = QH / KVH;
    const int blocks = B * KVH * splits, threads = 32 * AttentionWalk<DPL>::kWarps;
    auto launch = [&](auto kernel, size_t smem) {
        if (cudaFuncSetAttribute((const void*)kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return false;
        return chain_launch(kernel, dim3(blocks), dim3(threads), smem, s, qkv, keys, values, QH, KVH, pos,
                            case_stride, splits, scale, part) == cudaSuccess;
    };
    bool ok;
    if (R == 1)
        ok = launch(cached_attention_part_kernel<DPL, 1>, attention_walk_smem<DPL, 1>());
    else if (R == 2)
        ok = launch(cached_attention_part_kernel<DPL, 2>, attention_walk_smem<DPL, 2>());
    else if (R == 4 && DPL <= 4)
        ok = launch(cached_attention_part_kernel<DPL, 4>, attention_walk_smem<DPL, 4>());
    else
        return false;
    if (!ok) return false;
    return chain_launch(cached_attention_merge_kernel<DPL>, dim3(B * QH), dim3(128), 0, s, (const float*)part, QH,
                        splits, hi, lo) == cudaSuccess;
}

int BatchedScorer::generate_batch(const uint32_t* prompts, size_t batch, size_t P, size_t maximum,
                                  uint32_t* tokens_out) {
    const FusedConfig& c = config_;
    LSX_ENSURE(prompts && tokens_out && batch > 0 && batch <= 1024 && P >= 2 && maximum > 0,
               "check the batched generation shape");
    for (size_t i = 0; i < batch * P; ++i) LSX_ENSURE(prompts[i] < (uint32_t)c.vocab, "check the prompt token range");
    const int H = c.hidden, D = c.head_dim, QH = c.qheads, KVH = c.kvheads, I = c.intermediate, V = c.vocab;
    const int R = QH / KVH, dpl = D / 32;
    LSX_ENSURE(R == 1 || R == 2 || (R == 4 && dpl <= 4), "batched generation: unsupported group ratio");
    const size_t cap = P + maximum, kw = (size_t)KVH * D, B = batch;
    // per layer: keys, then values, each [batch][kvheads][capacity][head_dim]
    const size_t case_stride = cap * kw, layer_stride = 2 * B * case_stride;
    // about eight attention blocks per SM at any batch: each warp's cache walk is
    // latency-bound, so parallel blocks carry the bandwidth
    int splits = std::max(1, std::min(64, (8 * ctx_->sm_count + (int)(B * KVH) - 1) / (int)(B * KVH)));
    if (const char* v = std::getenv("LSX_BATCH_ATTENTION_SPLITS")) splits = std::max(1, std::min(64, std::atoi(v)));
    const size_t part_floats = B * QH * (size_t)splits * (D + 2);
    const size_t need = (layer_stride * layers_.size() + part_floats) * 4 + maximum * B * 4 + 256;
    cudaStream_t s = ctx_->stream;
    LSX_CUDA(cudaStreamSynchronize(s), "batched generation");
    if (need > batch_cache_bytes_) {
        if (batch_cache_) cudaFree(batch_cache_);
        batch_cache_ = nullptr;
        batch_cache_bytes_ = 0;
        LSX_CUDA(cudaMalloc(&batch_cache_, need), "batched generation caches");
        batch_cache_bytes_ = need;
    }
    float* part = batch_cache_ + layer_stride * layers_.size();
    uint32_t* history = (uint32_t*)(part + part_floats);

    // the prompts less their last token: one batched forward into the sequences' caches
    std::vector<uint32_t> head_tokens(B * (P - 1));
    for (size_t b = 0; b < B; ++b)
        for (size_t t = 0; t + 1 < P; ++t) head_tokens[b * (P - 1) + t] = prompts[b * P + t];
    batch_keys_ = batch_cache_;
    batch_case_stride_ = case_stride;
    batch_layer_stride_ = layer_stride;
    const int rc = run(head_tokens.data(), B, P - 1, 0, 0, nullptr, nullptr, Outputs{}, true);
    batch_keys_ = nullptr;
    LSX_TRY(rc);

    // decode: one row per sequence and step, the whole loop on the device
    LSX_TRY(reserve(B, B, cap));
    const Layout& L = layout_;
    uint8_t* base = (uint8_t*)block_;
    float* x = (float*)(base + L.x);
    float* work = (float*)(base + L.work);
    const size_t widest = std::max((size_t)H, std::max((size_t)QH * D, (size_t)I));
    __nv_bfloat16* hi = (__nv_bfloat16*)(base + L.planes);
    __nv_bfloat16* lo = hi + B * widest;
    float* logits = (float*)(base + L.logits);
    float2* rope = (float2*)(base + L.rope);
    uint32_t* d_tokens = (uint32_t*)(base + L.tokens);
    int* status = (int*)(base + L.status);
    const int half = D / 2, qkvw = (QH + 2 * KVH) * D;
    std::vector<float2> table(cap * half);
    for (size_t p = 0; p < cap; ++p)
        for (int i = 0; i < half; ++i) {
            const double angle = (double)p * std::pow(c.theta, -2.0 * i / (double)c.rotary);
            table[p * half + i] = make_float2((float)std::cos(angle), (float)std::sin(angle));
        }
    std::vector<uint32_t> last(B);
    for (size_t b = 0; b < B; ++b) last[b] = prompts[b * P + P - 1];
    LSX_CUDA(cudaMemcpyAsync(rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice, s),
             "rope upload");
    LSX_CUDA(cudaMemcpyAsync(d_tokens, last.data(), B * 4, cudaMemcpyHostToDevice, s), "token upload");
    LSX_CUDA(cudaMemsetAsync(status, 0, 16, s), "status clear");
    LSX_CUDA(cudaStreamSynchronize(s), "batched generation upload");  // host tables go out of scope
    const int M = (int)B;
    const int qk_blocks = (M * (QH + KVH) + 7) / 8;
    const int kv_blocks = (int)((B * kw + 255) / 256);
    for (size_t step = 0; step < maximum; ++step) {
        const int pos = (int)(P - 1 + step);
        LSX_CUDA(chain_launch(embed_rows_kernel, dim3(M), dim3(256), 0, s, c.embedding, c.embedding_kind,
                              c.embedding_scale, (const uint32_t*)d_tokens, H, x),
                 "embedding rows");
        for (size_t li = 0; li < layers_.size(); ++li) {
            const FusedLayer& Ly = layers_[li];
            float* bk = batch_cache_ + li * layer_stride;
            float* bv = bk + layer_stride / 2;
            LSX_CUDA(chain_launch(rms_planes_kernel, dim3(M), dim3(256), 0, s, (const float*)x, (const int*)nullptr, H,
                                  Ly.input_gain, c.eps, hi, lo, (float*)nullptr),
                     "batched decode norm");
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, H, Ly.wqkv, qkvw, Ly.bqkv, work, qkvw, false, status));
            const float2* rp = rope + (size_t)pos * half;
            bool ok;
            if (D == 128) {
                LSX_CUDA(chain_launch(qk_rope_kernel<4>, dim3(qk_blocks), dim3(256), 0, s, work, M, 1, QH, KVH,
                                      Ly.q_gain, Ly.k_gain, c.qk_eps, rp),
                         "batched decode rope");
                LSX_CUDA(chain_launch(kv_store_kernel, dim3(kv_blocks), dim3(256), 0, s, (const float*)work, B * kw, QH,
                                      KVH, D, bk, bv, 1, pos, case_stride, cap * D, (size_t)D),
                         "batched decode cache append");
                ok = launch_cached_attention<4>(s, work, bk, bv, M, QH, KVH, pos, case_stride, splits, c.scale, part,
                                                hi, lo);
            } else if (D == 64) {
                LSX_CUDA(chain_launch(qk_rope_kernel<2>, dim3(qk_blocks), dim3(256), 0, s, work, M, 1, QH, KVH,
                                      Ly.q_gain, Ly.k_gain, c.qk_eps, rp),
                         "batched decode rope");
                LSX_CUDA(chain_launch(kv_store_kernel, dim3(kv_blocks), dim3(256), 0, s, (const float*)work, B * kw, QH,
                                      KVH, D, bk, bv, 1, pos, case_stride, cap * D, (size_t)D),
                         "batched decode cache append");
                ok = launch_cached_attention<2>(s, work, bk, bv, M, QH, KVH, pos, case_stride, splits, c.scale, part,
                                                hi, lo);
            } else {
                LSX_CUDA(chain_launch(qk_rope_kernel<8>, dim3(qk_blocks), dim3(256), 0, s, work, M, 1, QH, KVH,
                                      Ly.q_gain, Ly.k_gain, c.qk_eps, rp),
                         "batched decode rope");
                LSX_CUDA(chain_launch(kv_store_kernel, dim3(kv_blocks), dim3(256), 0, s, (const float*)work, B * kw, QH,
                                      KVH, D, bk, bv, 1, pos, case_stride, cap * D, (size_t)D),
                         "batched decode cache append");
                ok = launch_cached_attention<8>(s, work, bk, bv, M, QH, KVH, pos, case_stride, splits, c.scale, part,
                                                hi, lo);
            }
            LSX_ENSURE(ok, "batched generation: attention launch (group ratio, shared memory)");
            LSX_CUDA(cudaGetLastError(), "batched decode attention");
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, QH * D, Ly.wo, H, Ly.bo, x, H, true, status));
            LSX_CUDA(chain_launch(rms_planes_kernel, dim3(M), dim3(256), 0, s, (const float*)x, (const int*)nullptr, H,
                                  Ly.post_gain, c.eps, hi, lo, (float*)nullptr),
                     "batched decode norm");
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, H, Ly.wgu, 2 * I, Ly.bgu, work, 2 * I, false, status));
            const size_t feats = (size_t)M * I;
            LSX_CUDA(chain_launch(gated_planes_kernel, dim3((unsigned)std::min<size_t>((feats + 255) / 256, 148 * 16)),
                                  dim3(256), 0, s, (const float*)work, feats, I, c.activation, hi, lo),
                     "batched decode gate");
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, I, Ly.wd, H, Ly.bd, x, H, true, status));
        }
        LSX_CUDA(chain_launch(rms_planes_kernel, dim3(M), dim3(256), 0, s, (const float*)x, (const int*)nullptr, H,
                              c.final_gain, c.eps, hi, lo, (float*)nullptr),
                 "batched decode norm");
        LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, H, c.head, V, c.head_bias, logits, V, false, status));
        LSX_CUDA(chain_launch(row_argmax_tokens_kernel, dim3(M), dim3(1024), 0, s, (const float*)logits, V, d_tokens,
                              history + step * B, status),
                 "batched decode step");
    }
    std::vector<uint32_t> hist(maximum * B);
    int host_status[2] = {0, 0};
    LSX_CUDA(cudaMemcpyAsync(hist.data(), history, hist.size() * 4, cudaMemcpyDeviceToHost, s), "token download");
    LSX_CUDA(cudaMemcpyAsync(host_status, status, 8, cudaMemcpyDeviceToHost, s), "status download");
    LSX_CUDA(cudaStreamSynchronize(s), "batched generation");
    if (host_status[0] != 0) return fail(LSX_E_CUDA, "batched generation: a device wait timed out");
    if (host_status[1] != 0) return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
    for (size_t b = 0; b < B; ++b)
        for (size_t k = 0; k < maximum; ++k) tokens_out[b * maximum + k] = hist[k * B + b];
    return LSX_OK;
}

int BatchedScorer::score(const uint32_t* tokens, size_t cases, size_t T, size_t first, size_t count,
                         const uint32_t* targets, const lsx_rotation* rotation, const Outputs& out) {
    LSX_ENSURE(cases > 0 && T > 0 && count > 0 && first + count <= T && targets, "check the case shape");
    if (rotation) LSX_ENSURE(rotation->width == (size_t)config_.hidden && rotation->rank <= 256,
                             "the edit must match the model width (rank at most 256)");
    return run(tokens, cases, T, first, count, targets, rotation, out, false);
}

int BatchedScorer::run(const uint32_t* tokens, size_t cases, size_t T, size_t first, size_t count,
                       const uint32_t* targets, const lsx_rotation* rotation, const Outputs& out, bool write_cache) {
    const FusedConfig& c = config_;
    const size_t rows = cases * T, scored = cases * count;
    LSX_ENSURE(rows <= 2147483647ull / 4 && scored * (size_t)c.vocab <= (size_t)1 << 40, "too many rows");
    LSX_TRY(reserve(rows, scored, T));
    const Layout& L = layout_;
    uint8_t* base = (uint8_t*)block_;
    float* x = (float*)(base + L.x);
    float* work = (float*)(base + L.work);
    const size_t widest = std::max((size_t)c.hidden, std::max((size_t)c.qheads * c.head_dim, (size_t)c.intermediate));
    __nv_bfloat16* hi = (__nv_bfloat16*)(base + L.planes);
    __nv_bfloat16* lo = hi + std::max(rows, scored) * widest;
    float* logits = (float*)(base + L.logits);
    float2* rope = (float2*)(base + L.rope);
    uint32_t* d_tokens = (uint32_t*)(base + L.tokens);
    uint32_t* d_targets = (uint32_t*)(base + L.targets);
    int* d_rows = (int*)(base + L.rows);
    double* d_nll = (double*)(base + L.nll);
    uint32_t* d_argmax = (uint32_t*)(base + L.argmax);
    double* d_margin = (double*)(base + L.margin);
    int* status = (int*)(base + L.status);
    cudaStream_t s = ctx_->stream;
    const int H = c.hidden, D = c.head_dim, QH = c.qheads, KVH = c.kvheads, I = c.intermediate, V = c.vocab;
    const int qkvw = (QH + 2 * KVH) * D;
    const int M = (int)rows;

    // host-side tables: RoPE for positions < T (as the decode engines build it),
    // and the scored rows (first .. first + count - 1 of each case)
    const int half = D / 2;
    std::vector<float2> table((size_t)T * half);
    for (size_t p = 0; p < T; ++p)
        for (int i = 0; i < half; ++i) {
            const double angle = (double)p * std::pow(c.theta, -2.0 * i / (double)c.rotary);
            table[p * half + i] = make_float2((float)std::cos(angle), (float)std::sin(angle));
        }
    std::vector<int> scored_rows(scored);
    for (size_t b = 0; b < cases; ++b)
        for (size_t k = 0; k < count; ++k) scored_rows[b * count + k] = (int)(b * T + first + k);
    LSX_CUDA(cudaMemcpyAsync(rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice, s),
             "rope upload");
    if (scored) {
        LSX_CUDA(cudaMemcpyAsync(d_rows, scored_rows.data(), scored * 4, cudaMemcpyHostToDevice, s), "row upload");
        LSX_CUDA(cudaMemcpyAsync(d_targets, targets, scored * 4, cudaMemcpyHostToDevice, s), "target upload");
    }
    LSX_CUDA(cudaMemcpyAsync(d_tokens, tokens, rows * 4, cudaMemcpyHostToDevice, s), "token upload");
    LSX_CUDA(cudaMemsetAsync(status, 0, 16, s), "status clear");
    LSX_CUDA(cudaStreamSynchronize(s), "batched scoring upload");  // host tables go out of scope

    embed_rows_kernel<<<M, 256, 0, s>>>(c.embedding, c.embedding_kind, c.embedding_scale, d_tokens, H, x);
    LSX_CUDA(cudaGetLastError(), "embedding rows");
    const int warps_per_block = 8;
    for (size_t li = 0; li < layers_.size(); ++li) {
        const FusedLayer& Ly = layers_[li];
        rms_planes_kernel<<<M, 256, 0, s>>>(x, nullptr, H, Ly.input_gain, c.eps, hi, lo);
        LSX_CUDA(cudaGetLastError(), "input norm");
        LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, H, Ly.wqkv, qkvw, Ly.bqkv, work, qkvw, false, status));
        const long long qk_warps = (long long)M * (QH + KVH);
        const int qk_blocks = (int)((qk_warps + warps_per_block - 1) / warps_per_block);
        const long long at_warps = (long long)M * QH;
        const int at_blocks = (int)((at_warps + warps_per_block - 1) / warps_per_block);
        if (D == 128) {
            qk_rope_kernel<4><<<qk_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH, Ly.q_gain,
                                                                         Ly.k_gain, c.qk_eps, rope);
            if (!launch_attention_mma(s, work, M, (int)T, QH, KVH, D, c.scale, hi, lo) &&
                !launch_attention_tiled<4>(s, work, M, (int)T, QH, KVH, c.scale, hi, lo))
                causal_attention_kernel<4><<<at_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH,
                                                                                      c.scale, hi, lo);
        } else if (D == 64) {
            qk_rope_kernel<2><<<qk_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH, Ly.q_gain,
                                                                         Ly.k_gain, c.qk_eps, rope);
            if (!launch_attention_tiled<2>(s, work, M, (int)T, QH, KVH, c.scale, hi, lo))
                causal_attention_kernel<2><<<at_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH,
                                                                                      c.scale, hi, lo);
        } else {
            qk_rope_kernel<8><<<qk_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH, Ly.q_gain,
                                                                         Ly.k_gain, c.qk_eps, rope);
            causal_attention_kernel<8><<<at_blocks, 32 * warps_per_block, 0, s>>>(work, M, (int)T, QH, KVH, c.scale,
                                                                                  hi, lo);
        }
        LSX_CUDA(cudaGetLastError(), "attention");
        if (write_cache) {
            const size_t kv = (size_t)M * KVH * D;
            if (batch_keys_) {  // per-sequence caches of generate_batch
                float* bk = batch_keys_ + li * batch_layer_stride_;
                float* bv = bk + batch_layer_stride_ / 2;
                kv_store_kernel<<<(int)std::min<size_t>((kv + 255) / 256, 148 * 16), 256, 0, s>>>(
                    work, kv, QH, KVH, D, bk, bv, (int)T, 0, batch_case_stride_, batch_case_stride_ / KVH, D);
            } else {
                kv_store_kernel<<<(int)std::min<size_t>((kv + 255) / 256, 148 * 16), 256, 0, s>>>(
                    work, kv, QH, KVH, D, Ly.keys, Ly.values, (int)T, 0, 0, D, (size_t)KVH * D);
            }
            LSX_CUDA(cudaGetLastError(), "KV append");
        }
        LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, QH * D, Ly.wo, H, Ly.bo, x, H, true, status));
        rms_planes_kernel<<<M, 256, 0, s>>>(x, nullptr, H, Ly.post_gain, c.eps, hi, lo);
        LSX_CUDA(cudaGetLastError(), "post norm");
        // gate/up with the gated product in the GEMM's epilogue: the features' planes
        // go to the work buffer (free until the next layer's q/k/v), which holds the
        // f32 gate/up product otherwise
        const size_t feats = (size_t)M * I;
        __nv_bfloat16* f_hi = reinterpret_cast<__nv_bfloat16*>(work);
        __nv_bfloat16* f_lo = f_hi + feats;
        bool fused = false;
        LSX_TRY(gemm_gated_enqueue(ctx_, hi, lo, M, H, Ly.wgu, 2 * I, Ly.bgu, c.activation, f_hi, f_lo, status,
                                   &fused));
        if (fused) {
            LSX_TRY(gemm_planes_enqueue(ctx_, f_hi, f_lo, M, I, Ly.wd, H, Ly.bd, x, H, true, status));
        } else {
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, H, Ly.wgu, 2 * I, Ly.bgu, work, 2 * I, false, status));
            gated_planes_kernel<<<(int)std::min<size_t>((feats + 255) / 256, 148 * 16), 256, 0, s>>>(
                work, feats, I, c.activation, hi, lo);
            LSX_CUDA(cudaGetLastError(), "gated product");
            LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, M, I, Ly.wd, H, Ly.bd, x, H, true, status));
        }
    }
    int host_status[2] = {0, 0};
    if (scored == 0) {  // prefill: the KV cache is the result
        LSX_CUDA(cudaMemcpyAsync(host_status, status, 8, cudaMemcpyDeviceToHost, s), "status download");
        LSX_CUDA(cudaStreamSynchronize(s), "batched prefill");
        if (host_status[0] != 0) return fail(LSX_E_CUDA, "batched prefill: a device wait timed out");
        if (host_status[1] != 0) return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
        return LSX_OK;
    }
    if (rotation) {  // the edited readout of the unedited hidden state
        rms_planes_kernel<<<(int)scored, 256, 0, s>>>(x, d_rows, H, c.final_gain, c.eps, hi, lo, work);
        const bool joint = rotation->joint;
        edit_rows_kernel<<<(int)scored, 256, 0, s>>>(
            work, H, joint ? 2 : 1, rotation->cosine_minus_one, rotation->sine,
            joint ? nullptr : (const float*)rotation->u->data, joint ? nullptr : (const float*)rotation->v->data,
            (int)rotation->rank, joint ? (const float*)rotation->basis->data : nullptr,
            joint ? (const float*)rotation->delta->data : nullptr, hi, lo);
    } else {
        rms_planes_kernel<<<(int)scored, 256, 0, s>>>(x, d_rows, H, c.final_gain, c.eps, hi, lo);
    }
    LSX_CUDA(cudaGetLastError(), "final norm");
    LSX_TRY(gemm_planes_enqueue(ctx_, hi, lo, (int)scored, H, c.head, V, c.head_bias, logits, V, false, status));
    row_scores_kernel<<<(int)scored, 1024, 0, s>>>(logits, V, d_targets, d_nll, d_argmax, d_margin);
    LSX_CUDA(cudaGetLastError(), "scores");
    if (out.nll) LSX_CUDA(cudaMemcpyAsync(out.nll, d_nll, scored * 8, cudaMemcpyDeviceToHost, s), "nll download");
    if (out.argmax)
        LSX_CUDA(cudaMemcpyAsync(out.argmax, d_argmax, scored * 4, cudaMemcpyDeviceToHost, s), "argmax download");
    if (out.margin)
        LSX_CUDA(cudaMemcpyAsync(out.margin, d_margin, scored * 8, cudaMemcpyDeviceToHost, s), "margin download");
    if (out.logits)
        LSX_CUDA(cudaMemcpyAsync(out.logits, logits, scored * (size_t)V * 4, cudaMemcpyDeviceToHost, s),
                 "logits download");
    LSX_CUDA(cudaMemcpyAsync(host_status, status, 8, cudaMemcpyDeviceToHost, s), "status download");
    LSX_CUDA(cudaStreamSynchronize(s), "batched scoring");
    if (host_status[0] != 0) return fail(LSX_E_CUDA, "batched scoring: a device wait timed out");
    if (host_status[1] != 0) return fail(LSX_E_NONFINITE, "check the finiteness of the model outputs");
    return LSX_OK;
}

}  // namespace lsx
