// Fused batch-1 decode engine for B200 (sm_100a).
//
// One decode step (Model::decode, src/model.rs:729-853) runs as 2 + 5*layers
// kernels chained with programmatic dependent launch:
//   embed  : token (prompt, or argmax of the previous step) -> residual
//   per layer:
//     qkv  : RMSNorm(residual) -> [q;k;v] = Wqkv x                (one GEMV over concatenated rows)
//     attn : QK-norm, RoPE, KV append, GQA attention split over positions
//     o    : residual += Wo attn
//     gu   : RMSNorm(residual) -> act(Wg x) * (Wu x)              (gate/up rows interleaved)
//     down : residual += Wd h
//   head   : final RMSNorm, optional readout edit, logits = Wh x, first argmax
// Every GEMV kernel issues bulk copies of its weight rows into shared memory
// BEFORE griddepcontrol.wait, so weight streaming of the next kernels overlaps the
// dependent chain; weights never depend on activations.  Activations are f32 and
// weights bf16 with f32 accumulation, as in the reference (src/gpu.rs:365,
// src/model.rs:148); the KV cache is f32 as in src/model.rs:492.
#include <math.h>

#include <cmath>
#include <string>

#include "decode.cuh"
#include "device_common.cuh"

namespace lsx {

enum { kPlain = 0, kNorm = 1, kNormRotate = 2 };
enum { kStore = 0, kResidual = 1, kGated = 2, kHead = 3 };

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kStageBytes = 16384;
constexpr int kRingBudget = 98304;
constexpr int kRedFloats = 64 + 512;  // block reductions + joint-edit coordinates

struct GemvArgs {
    const __nv_bfloat16* w;
    const float* bias;
    int n, k, rows_per_stage, nstage;
    const float* x;
    const float* gain;
    float eps;
    float* out;
    int act;
    DecodeState* state;
    unsigned long long* partials;
};

__device__ __forceinline__ float activation(float x, int kind) {
    switch (kind) {
    case 0: return x / (1.f + expf(-x));
    case 1: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
    case 2: return fmaxf(x, 0.f);
    default: return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
    }
}

__device__ float block_allsum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_allsum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kGemvWarps; ++i) t += red[i];
    return t;
}

// Row dot product of one staged bf16 row with x.  KCH > 0: x chunks live in
// registers (K == 256*KCH); KCH == 0: x is read from shared memory (K % 8 == 0).
template <int KCH>
__device__ __forceinline__ float row_dot(const unsigned char* row, const float4* xr, const float* xs, int K,
                                         int lane) {
    const uint4* w = reinterpret_cast<const uint4*>(row);
    float acc = 0.f;
    if (KCH > 0) {
#pragma unroll
        for (int j = 0; j < KCH; ++j) acc += dot8_bf16(w[lane + 32 * j], xr[2 * j], xr[2 * j + 1]);
    } else {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        for (int c = lane; c < (K >> 3); c += 32) acc += dot8_bf16(w[c], x4[2 * c], x4[2 * c + 1]);
    }
    return warp_allsum(acc);
}

template <int PRO, int EPI, int KCH>
__global__ void __launch_bounds__(kGemvThreads) fused_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.k;
    const size_t row_bytes = (size_t)K * 2;
    const int unit = (EPI == kGated) ? 2 : 1;
    const int units = a.n / unit;
    const int lo = (int)(((long long)blockIdx.x * units) / gridDim.x) * unit;
    const int hi = (int)(((long long)(blockIdx.x + 1) * units) / gridDim.x) * unit;
    const int SR = a.rows_per_stage;
    const int nst = (hi - lo + SR - 1) / SR;
    const size_t stage_bytes = (size_t)SR * row_bytes;
    unsigned char* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)a.nstage * stage_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + K);
    float* red = reinterpret_cast<float*>(bars + a.nstage);
    __shared__ int s_flag;

    if (tid == 0) {
        for (int i = 0; i < a.nstage; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int s) {
        const int r0 = lo + s * SR;
        const int nr = min(SR, hi - r0);
        const uint32_t bytes = (uint32_t)(nr * row_bytes);
        uint64_t* bar = &bars[s % a.nstage];
        mbar_expect_tx(bar, bytes);
        bulk_load(ring + (size_t)(s % a.nstage) * stage_bytes, a.w + (size_t)r0 * K, bytes, bar);
    };
    const int first = min(a.nstage, nst);
    if (tid == 0)
        for (int s = 0; s < first; ++s) issue(s);

    pdl_launch_dependents();
    pdl_wait();

    DecodeState* st = a.state;
    // Waits (bounded) for the stages issued but not consumed, so no copy is in
    // flight into this block's shared memory when it exits.
    auto drain = [&](int consumed, int issued) {
        if (tid == 0)
            for (int s = consumed; s < issued; ++s) mbar_wait_bounded(&bars[s % a.nstage], (s / a.nstage) & 1);
    };
    if (st->stopped) {
        drain(0, first);
        return;
    }

    // ---- prologue: the input vector into shared memory ----
    if (PRO == kPlain) {
        for (int i = tid; i < K; i += kGemvThreads) xs[i] = a.x[i];
    } else {
        float ss = 0.f;
        for (int i = tid; i < K; i += kGemvThreads) {
            float v = a.x[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
        ss = block_allsum(ss, red);
        const float inverse = rsqrtf(ss / (float)K + a.eps);
        for (int i = tid; i < K; i += kGemvThreads) xs[i] = xs[i] * inverse * a.gain[i];
    }
    __syncthreads();
    float* logits = nullptr;
    if (PRO == kNormRotate) {
        const int slot = st->step - (st->prompt_length - 1 - st->frame_back);
        const bool framed = st->frames && slot >= 0;
        float* hid = framed ? st->hidden_frames + (size_t)slot * K : st->hidden_scratch;
        logits = framed ? st->logits_frames + (size_t)slot * a.n : st->logits_scratch;
        if (blockIdx.x == 0) {
            bool bad = false;
            for (int i = tid; i < K; i += kGemvThreads) {
                hid[i] = xs[i];
                bad |= !isfinite(xs[i]);
            }
            if (__syncthreads_or(bad) && tid == 0) st->nonfinite = 1;
        }
        if (st->rot_kind == 1) {  // kernels/ops.py:125-135
            const float* u = st->rot_u;
            const float* v = st->rot_v;
            float hu = 0.f, hv = 0.f;
            for (int i = tid; i < K; i += kGemvThreads) {
                hu = fmaf(xs[i], u[i], hu);
                hv = fmaf(xs[i], v[i], hv);
            }
            hu = block_allsum(hu, red);
            hv = block_allsum(hv, red + 16);
            const float A = st->rot_a, B = st->rot_b;
            for (int i = tid; i < K; i += kGemvThreads)
                xs[i] = xs[i] + u[i] * (A * hu + B * hv) + v[i] * (A * hv - B * hu);
        } else if (st->rot_kind == 2) {  // DeviceRotation::apply Joint (src/model.rs:350-361)
            const int r = st->rot_rank;
            const float* basis = st->rot_basis;
            const float* delta = st->rot_delta;
            float* coords = red + 64;
            float* shift = coords + 256;
            for (int k = warp; k < r; k += kGemvWarps) {
                float d = 0.f;
                for (int j = lane; j < K; j += 32) d = fmaf(basis[(size_t)k * K + j], xs[j], d);
                d = warp_allsum(d);
                if (lane == 0) coords[k] = d;
            }
            __syncthreads();
            for (int i = tid; i < r; i += kGemvThreads) {
                float d = 0.f;
                for (int j = 0; j < r; ++j) d = fmaf(delta[i * r + j], coords[j], d);
                shift[i] = d;
            }
            __syncthreads();
            for (int j = tid; j < K; j += kGemvThreads) {
                float d = 0.f;
                for (int k = 0; k < r; ++k) d = fmaf(basis[(size_t)k * K + j], shift[k], d);
                xs[j] = __fadd_rn(xs[j], d);
            }
        }
        __syncthreads();
    }
    float4 xr[KCH > 0 ? 2 * KCH : 1];
    if (KCH > 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            xr[2 * j] = x4[2 * (lane + 32 * j)];
            xr[2 * j + 1] = x4[2 * (lane + 32 * j) + 1];
        }
    }

    // ---- main loop over weight stages ----
    unsigned long long best = 0ull;
    bool bad = false;
    for (int s = 0; s < nst; ++s) {
        const int buf = s % a.nstage;
        const bool ok = mbar_wait_bounded(&bars[buf], (s / a.nstage) & 1);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicExch(&st->status, kDeviceTimeoutWeights);
            drain(s, min(nst, s + a.nstage));
            return;
        }
        const unsigned char* sb = ring + (size_t)buf * stage_bytes;
        const int r0 = lo + s * SR;
        const int nr = min(SR, hi - r0);
        if (EPI == kGated) {
            for (int p = warp; p < (nr >> 1); p += kGemvWarps) {
                float g = row_dot<KCH>(sb + (size_t)(2 * p) * row_bytes, xr, xs, K, lane);
                float u = row_dot<KCH>(sb + (size_t)(2 * p + 1) * row_bytes, xr, xs, K, lane);
                if (lane == 0) {
                    const int row = r0 + 2 * p;
                    if (a.bias) {
                        g += a.bias[row];
                        u += a.bias[row + 1];
                    }
                    a.out[row >> 1] = activation(g, a.act) * u;
                }
            }
        } else {
            for (int ri = warp; ri < nr; ri += kGemvWarps) {
                float d = row_dot<KCH>(sb + (size_t)ri * row_bytes, xr, xs, K, lane);
                if (lane == 0) {
                    const int row = r0 + ri;
                    if (a.bias) d += a.bias[row];
                    if (EPI == kStore) {
                        a.out[row] = d;
                    } else if (EPI == kResidual) {
                        a.out[row] = __fadd_rn(a.out[row], d);
                    } else {  // kHead
                        logits[row] = d;
                        bad |= !isfinite(d);
                        unsigned long long key = pack_arg(d, (uint32_t)row);
                        best = key > best ? key : best;
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && s + a.nstage < nst) issue(s + a.nstage);
    }

    if (EPI == kHead) {
        unsigned long long* rbest = reinterpret_cast<unsigned long long*>(red);
        if (__syncthreads_or(bad) && tid == 0) st->nonfinite = 1;
        if (lane == 0) rbest[warp] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int i = 0; i < kGemvWarps; ++i) b = rbest[i] > b ? rbest[i] : b;
            a.partials[blockIdx.x] = b;
            __threadfence();
            unsigned int previous = atomicAdd(&st->head_counter, 1u);
            s_flag = (previous == gridDim.x - 1) ? 1 : 0;
        }
        __syncthreads();
        if (s_flag) {  // last block: global first argmax, then advance the cursor
            __threadfence();
            unsigned long long b = 0ull;
            for (int i = tid; i < (int)gridDim.x; i += kGemvThreads) {
                unsigned long long v = __ldcg(&a.partials[i]);
                b = v > b ? v : b;
            }
            b = warp_max_u64(b);
            __syncthreads();
            if (lane == 0) rbest[warp] = b;
            __syncthreads();
            if (tid == 0) {
                for (int i = 0; i < kGemvWarps; ++i) b = rbest[i] > b ? rbest[i] : b;
                const uint32_t token = packed_index(b);
                st->argmax = token;
                st->head_counter = 0u;
                const int index = st->step - (st->prompt_length - 1 - st->frame_back);
                if (index >= 0) {
                    st->tokens_out[index] = token;
                    st->generated = index + 1;
                    bool stop = index + 1 >= st->maximum;
                    for (int i = 0; i < st->n_stop; ++i) stop |= st->stop[i] == token;
                    if (stop) st->stopped = 1;
                }
                st->position += 1;
                st->step += 1;
            }
        }
    }
}

// ------------------------------------------------------------------ embed --
struct EmbedArgs {
    const void* table;
    int kind;
    int hidden;
    float scale;
    float* residual;
    DecodeState* state;
};

__global__ void __launch_bounds__(256) embed_kernel(const EmbedArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    DecodeState* st = a.state;
    if (st->stopped) return;
    if (st->mode == 1) {
        for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) a.residual[i] = st->inject[i];
        return;
    }
    const uint32_t token = st->step < st->prompt_length ? st->prompt[st->step] : st->argmax;
    const size_t base = (size_t)token * a.hidden;
    for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) {
        float v;
        if (a.kind == LSX_BF16) v = __bfloat162float(((const __nv_bfloat16*)a.table)[base + i]);
        else if (a.kind == LSX_F32) v = ((const float*)a.table)[base + i];
        else v = __half2float(((const __half*)a.table)[base + i]);
        // Model::embedding_tensor (src/model.rs:620-631): combine(row, row, scale - 1)
        if (a.scale != 1.f) v = __fadd_rn(v, __fmul_rn(a.scale - 1.f, v));
        a.residual[i] = v;
    }
    if (threadIdx.x == 0) st->token = token;
}

// -------------------------------------------------------------- attention --
struct AttnArgs {
    const float* qkv;
    const float* q_gain;
    const float* k_gain;
    float qk_eps;
    float* keys;
    float* values;
    float* partial;
    float* out;
    const float2* rope;  // [capacity][rotary/2] (cos, sin) of position * theta^(-2 pair/rotary)
    int qheads, kvheads, dim, rotary, interleaved, splits;
    float scale;
    DecodeState* state;
};

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;

// Grid (kvheads, splits).  Block (g, s) handles the RATIO query heads of KV group
// g over its share of positions 0..position; partial softmax states merge exactly
// (max, sum, weighted values), in this block when splits == 1, else in the last
// block of the group to finish.
template <int RATIO, int DPL>
__global__ void __launch_bounds__(kAttnThreads) fused_attention_kernel(const AttnArgs a) {
    constexpr int D = DPL * 32;
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    float* raw = sm;                    // (RATIO + 1) * D
    float* qs = raw + (RATIO + 1) * D;  // RATIO * D
    float* ks = qs + RATIO * D;         // D
    float* vs = ks + D;                 // D
    float* merge = vs + D;              // kAttnWarps * RATIO * (D + 2)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = blockIdx.x, split = blockIdx.y;

    pdl_launch_dependents();
    pdl_wait();
    DecodeState* st = a.state;
    if (st->stopped) return;
    const int pos = st->position;
    const int kw = a.kvheads * D;

    const float* qraw = a.qkv + (size_t)g * RATIO * D;
    const float* kraw = a.qkv + (size_t)a.qheads * D + (size_t)g * D;
    const float* vraw = kraw + kw;
    for (int i = tid; i < RATIO * D; i += kAttnThreads) raw[i] = qraw[i];
    for (int i = tid; i < D; i += kAttnThreads) {
        raw[RATIO * D + i] = kraw[i];
        vs[i] = vraw[i];
    }
    __syncthreads();
    // Per-head RMSNorm (Qwen3 q_norm / k_norm: groups of head_dim).
    for (int h = warp; h < RATIO + 1; h += kAttnWarps) {
        const float* gain = h < RATIO ? a.q_gain : a.k_gain;
        if (!gain) continue;
        float* row = raw + h * D;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss = fmaf(row[lane + 32 * j], row[lane + 32 * j], ss);
        ss = warp_allsum(ss);
        const float inverse = rsqrtf(ss / (float)D + a.qk_eps);
#pragma unroll
        for (int j = 0; j < DPL; ++j) row[lane + 32 * j] = row[lane + 32 * j] * inverse * gain[lane + 32 * j];
    }
    __syncthreads();
    // RoPE (kernels/ops.py:48-66).
    const int half = a.rotary / 2;
    for (int i = tid; i < (RATIO + 1) * D; i += kAttnThreads) {
        const int h = i / D, local = i % D;
        const float x = raw[i];
        float y = x;
        if (local < a.rotary) {
            int pair, other;
            float sign;
            if (a.interleaved) {
                pair = local >> 1;
                other = (local & 1) ? local - 1 : local + 1;
                sign = (local & 1) ? 1.f : -1.f;
            } else {
                pair = local % half;
                other = local < half ? local + half : local - half;
                sign = local < half ? -1.f : 1.f;
            }
            const float2 cs = a.rope[(size_t)pos * half + pair];
            y = x * cs.x + sign * raw[h * D + other] * cs.y;
        }
        if (h < RATIO) qs[i] = y;
        else ks[local] = y;
    }
    __syncthreads();

    const int n = pos + 1;
    const int chunk = (n + a.splits - 1) / a.splits;
    const int t0 = split * chunk;
    const int t1 = min(n, t0 + chunk);
    if (t0 <= pos && pos < t1) {  // kernels/ops.py:69-73 cache_write, by the block that owns `pos`
        float* kd = a.keys + (size_t)pos * kw + (size_t)g * D;
        float* vd = a.values + (size_t)pos * kw + (size_t)g * D;
        for (int i = tid; i < D; i += kAttnThreads) {
            kd[i] = ks[i];
            vd[i] = vs[i];
        }
    }

    float q[RATIO][DPL], acc[RATIO][DPL], m[RATIO], l[RATIO];
#pragma unroll
    for (int h = 0; h < RATIO; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            q[h][j] = qs[h * D + lane + 32 * j];
            acc[h][j] = 0.f;
        }
    }
    for (int t = t0 + warp; t < t1; t += kAttnWarps) {
        const float* kt = t == pos ? ks : a.keys + (size_t)t * kw + (size_t)g * D;
        const float* vt = t == pos ? vs : a.values + (size_t)t * kw + (size_t)g * D;
        float kv[DPL], vv[DPL];
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            kv[j] = kt[lane + 32 * j];
            vv[j] = vt[lane + 32 * j];
        }
#pragma unroll
        for (int h = 0; h < RATIO; ++h) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) s = fmaf(q[h][j], kv[j], s);
            s = warp_allsum(s) * a.scale;
            const float mn = fmaxf(m[h], s);
            const float carry = expf(m[h] - mn);
            const float p = expf(s - mn);
            l[h] = l[h] * carry + p;
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[h][j] = fmaf(p, vv[j], acc[h][j] * carry);
            m[h] = mn;
        }
    }
    // Merge the warps of this block.
    const int stride = D + 2;
#pragma unroll
    for (int h = 0; h < RATIO; ++h) {
        float* slot = merge + (size_t)(warp * RATIO + h) * stride;
        if (lane == 0) {
            slot[0] = m[h];
            slot[1] = l[h];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) slot[2 + lane + 32 * j] = acc[h][j];
    }
    __syncthreads();
    float* part = a.partial + (size_t)((g * a.splits + split) * RATIO) * stride;
    for (int i = tid; i < RATIO * D; i += kAttnThreads) {
        const int h = i / D, d = i % D;
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, merge[(w * RATIO + h) * stride]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < kAttnWarps; ++w) {
                const float* sl = merge + (size_t)(w * RATIO + h) * stride;
                if (sl[0] == -INFINITY) continue;
                const float e = expf(sl[0] - M);
                L = fmaf(sl[1], e, L);
                O = fmaf(sl[2 + d], e, O);
            }
        }
        if (a.splits == 1) {
            a.out[(size_t)(g * RATIO + h) * D + d] = O / L;
        } else {
            float* ph = part + (size_t)h * stride;
            if (d == 0) {
                ph[0] = M;
                ph[1] = L;
            }
            ph[2 + d] = O;
        }
    }
    if (a.splits == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned int previous = atomicAdd(&st->attn_counter[g], 1u);
        s_last = previous == (unsigned)a.splits - 1 ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* group = a.partial + (size_t)(g * a.splits * RATIO) * stride;
    for (int i = tid; i < RATIO * D; i += kAttnThreads) {
        const int h = i / D, d = i % D;
        float M = -INFINITY;
        for (int s = 0; s < a.splits; ++s) M = fmaxf(M, __ldcg(group + (size_t)(s * RATIO + h) * stride));
        float L = 0.f, O = 0.f;
        for (int s = 0; s < a.splits; ++s) {
            const float* ph = group + (size_t)(s * RATIO + h) * stride;
            const float ms = __ldcg(ph);
            if (ms == -INFINITY) continue;
            const float e = expf(ms - M);
            L = fmaf(__ldcg(ph + 1), e, L);
            O = fmaf(__ldcg(ph + 2 + d), e, O);
        }
        a.out[(size_t)(g * RATIO + h) * D + d] = O / L;
    }
    if (tid == 0) st->attn_counter[g] = 0u;
}

// ------------------------------------------------------------ host side ----
namespace {

using GemvKernel = void (*)(const GemvArgs);

template <int PRO, int EPI>
GemvKernel pick_gemv(int kch) {
    switch (kch) {
    case 4: return fused_gemv_kernel<PRO, EPI, 4>;
    case 8: return fused_gemv_kernel<PRO, EPI, 8>;
    case 10: return fused_gemv_kernel<PRO, EPI, 10>;
    case 12: return fused_gemv_kernel<PRO, EPI, 12>;
    default: return fused_gemv_kernel<PRO, EPI, 0>;
    }
}

int register_path(int k) {
    if (k % 256 != 0) return 0;
    int kch = k / 256;
    return (kch == 4 || kch == 8 || kch == 10 || kch == 12) ? kch : 0;
}

GemvKernel gemv_kernel_for(int pro, int epi, int k) {
    int kch = register_path(k);
    if (pro == kNorm && epi == kStore) return pick_gemv<kNorm, kStore>(kch);
    if (pro == kPlain && epi == kResidual) return pick_gemv<kPlain, kResidual>(kch);
    if (pro == kNorm && epi == kGated) return pick_gemv<kNorm, kGated>(kch);
    return pick_gemv<kNormRotate, kHead>(kch);
}

using AttnKernel = void (*)(const AttnArgs);
AttnKernel attention_kernel_for(int ratio, int dpl) {
#define LSX_ATTN_CASE(R)                                          \
    if (ratio == R) {                                             \
        if (dpl == 2) return fused_attention_kernel<R, 2>;        \
        if (dpl == 4) return fused_attention_kernel<R, 4>;        \
        if (dpl == 8) return fused_attention_kernel<R, 8>;        \
    }
    LSX_ATTN_CASE(1)
    LSX_ATTN_CASE(2)
    LSX_ATTN_CASE(4)
    LSX_ATTN_CASE(8)
#undef LSX_ATTN_CASE
    return nullptr;
}

struct GemvPlan {
    GemvKernel kernel;
    GemvArgs args;
    int grid;
    size_t smem;
};

// Rows per stage and ring depth for a GEMV of n rows x k columns on `grid` blocks.
void plan_stages(int n, int k, int unit, int grid, int* rows_per_stage, int* nstage) {
    int sr = kStageBytes / (2 * k);
    sr = (sr / unit) * unit;
    if (sr < unit) sr = unit;
    int rows = ((n / unit + grid - 1) / grid) * unit;
    int stages = (rows + sr - 1) / sr;
    int budget = kRingBudget / (sr * 2 * k);
    if (budget < 2) budget = 2;
    *rows_per_stage = sr;
    *nstage = stages < budget ? (stages < 1 ? 1 : stages) : budget;
}

size_t gemv_smem(int k, int rows_per_stage, int nstage) {
    return (size_t)nstage * rows_per_stage * 2 * k + (size_t)k * 4 + (size_t)nstage * 8 + kRedFloats * 4;
}

cudaError_t launch_pdl(const void* kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = s;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    return cudaLaunchKernelExC(&config, kernel, args);
}

}  // namespace

bool FusedDecoder::eligible(const FusedConfig& c, std::string* why) {
    auto no = [&](const char* m) {
        if (why) *why = m;
        return false;
    };
    if (c.hidden % 8 || c.intermediate % 8 || (c.qheads * c.head_dim) % 8) return no("widths not multiples of 8");
    if (c.head_dim % 32 || c.head_dim > 256 || c.head_dim / 32 == 3 || c.head_dim / 32 > 8 ||
        (c.head_dim / 32) & ((c.head_dim / 32) - 1))
        return no("head_dim must be 64, 128 or 256");
    if (c.kvheads <= 0 || c.qheads % c.kvheads) return no("query heads must be a multiple of KV heads");
    int ratio = c.qheads / c.kvheads;
    if (ratio != 1 && ratio != 2 && ratio != 4 && ratio != 8) return no("GQA ratio must be 1, 2, 4 or 8");
    if (c.kvheads > 64) return no("at most 64 KV heads");
    if (c.rotary % 2 || c.rotary > c.head_dim) return no("rotary dim");
    if (c.hidden > 16384 || c.intermediate > 65536) return no("widths too large for the fused plan");
    if (c.embedding_kind != LSX_BF16 && c.embedding_kind != LSX_F32 && c.embedding_kind != LSX_F16)
        return no("embedding kind");
    return true;
}

FusedDecoder::~FusedDecoder() {
    if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
    if (graph_) cudaGraphDestroy(graph_);
    for (void* p : owned_) cudaFree(p);
}

int FusedDecoder::build(lsx_ctx* ctx, const FusedConfig& c, const std::vector<FusedLayer>& layers) {
    std::string why;
    if (!eligible(c, &why)) return fail(LSX_E_UNSUPPORTED, "fused decode plan: " + why);
    ctx_ = ctx;
    config_ = c;
    layers_ = layers;
    grid_ = ctx->sm_count;
    int ratio = c.qheads / c.kvheads;
    int cap_splits = (c.capacity + 15) / 16;
    int max_splits = grid_ / c.kvheads;
    if (max_splits < 1) max_splits = 1;
    splits_ = cap_splits < max_splits ? cap_splits : max_splits;
    if (splits_ < 1) splits_ = 1;
    auto alloc = [&](size_t bytes, void** p) -> int {
        LSX_CUDA(cudaMalloc(p, bytes), "decode buffer allocation");
        owned_.push_back(*p);
        return LSX_OK;
    };
    int qw = c.qheads * c.head_dim, kw = c.kvheads * c.head_dim;
    LSX_TRY(alloc(sizeof(DecodeState), (void**)&state_));
    LSX_TRY(alloc((size_t)c.hidden * 4, (void**)&residual_));
    LSX_TRY(alloc((size_t)(qw + 2 * kw) * 4, (void**)&qkv_));
    LSX_TRY(alloc((size_t)c.kvheads * splits_ * ratio * (c.head_dim + 2) * 4, (void**)&attn_partial_));
    LSX_TRY(alloc((size_t)qw * 4, (void**)&attn_out_));
    LSX_TRY(alloc((size_t)c.intermediate * 4, (void**)&feature_));
    LSX_TRY(alloc((size_t)grid_ * 8, (void**)&head_partials_));
    LSX_CUDA(cudaMemset(state_, 0, sizeof(DecodeState)), "decode state");
    int half = c.rotary / 2;
    if (half > 0) {
        std::vector<float2> table((size_t)c.capacity * half);
        for (int p = 0; p < c.capacity; ++p)
            for (int i = 0; i < half; ++i) {
                double angle = (double)p * std::pow(c.theta, -2.0 * i / (double)c.rotary);
                table[(size_t)p * half + i] = make_float2((float)std::cos(angle), (float)std::sin(angle));
            }
        LSX_TRY(alloc(table.size() * sizeof(float2), (void**)&rope_));
        LSX_CUDA(cudaMemcpy(rope_, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice),
                 "rope table upload");
    }
    // Opt every kernel in to the shared memory it needs.
    const int ks[4] = {c.hidden, qw, c.hidden, c.intermediate};
    const int pros[4] = {kNorm, kPlain, kNorm, kPlain};
    const int epis[4] = {kStore, kResidual, kGated, kResidual};
    const int ns[4] = {qw + 2 * kw, c.hidden, 2 * c.intermediate, c.hidden};
    for (int i = 0; i < 4; ++i) {
        int sr, nstage;
        plan_stages(ns[i], ks[i], epis[i] == kGated ? 2 : 1, grid_, &sr, &nstage);
        size_t smem = gemv_smem(ks[i], sr, nstage);
        if (smem > ctx->smem_optin) return fail(LSX_E_UNSUPPORTED, "fused decode plan: shared memory");
        LSX_CUDA(cudaFuncSetAttribute((const void*)gemv_kernel_for(pros[i], epis[i], ks[i]),
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "gemv shared memory attribute");
    }
    {
        int sr, nstage;
        plan_stages(c.vocab, c.hidden, 1, grid_, &sr, &nstage);
        size_t smem = gemv_smem(c.hidden, sr, nstage);
        if (smem > ctx->smem_optin) return fail(LSX_E_UNSUPPORTED, "fused decode plan: shared memory");
        LSX_CUDA(cudaFuncSetAttribute((const void*)gemv_kernel_for(kNormRotate, kHead, c.hidden),
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "head shared memory attribute");
    }
    AttnKernel ak = attention_kernel_for(ratio, c.head_dim / 32);
    if (!ak) return fail(LSX_E_UNSUPPORTED, "fused decode plan: attention shape");
    size_t attn_smem = (size_t)((ratio + 1) * c.head_dim + ratio * c.head_dim + 2 * c.head_dim +
                                kAttnWarps * ratio * (c.head_dim + 2)) * 4;
    LSX_CUDA(cudaFuncSetAttribute((const void*)ak, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem),
             "attention shared memory attribute");
    return LSX_OK;
}

int FusedDecoder::launch_all() {
    const FusedConfig& c = config_;
    cudaStream_t s = ctx_->stream;
    const int qw = c.qheads * c.head_dim, kw = c.kvheads * c.head_dim;
    const int ratio = c.qheads / c.kvheads;
    {
        EmbedArgs e{c.embedding, c.embedding_kind, c.hidden, c.embedding_scale, residual_, state_};
        void* args[] = {&e};
        LSX_CUDA(launch_pdl((const void*)embed_kernel, dim3(1), dim3(256), 0, s, args), "embed launch");
    }
    auto gemv = [&](int pro, int epi, const __nv_bfloat16* w, const float* bias, int n, int k, const float* x,
                    const float* gain, float* out) -> int {
        GemvArgs g{};
        g.w = w;
        g.bias = bias;
        g.n = n;
        g.k = k;
        plan_stages(n, k, epi == kGated ? 2 : 1, grid_, &g.rows_per_stage, &g.nstage);
        g.x = x;
        g.gain = gain;
        g.eps = c.eps;
        g.out = out;
        g.act = c.activation;
        g.state = state_;
        g.partials = head_partials_;
        size_t smem = gemv_smem(k, g.rows_per_stage, g.nstage);
        void* args[] = {&g};
        LSX_CUDA(launch_pdl((const void*)gemv_kernel_for(pro, epi, k), dim3(grid_), dim3(kGemvThreads), smem, s,
                            args),
                 "gemv launch");
        return LSX_OK;
    };
    AttnKernel ak = attention_kernel_for(ratio, c.head_dim / 32);
    size_t attn_smem = (size_t)((ratio + 1) * c.head_dim + ratio * c.head_dim + 2 * c.head_dim +
                                kAttnWarps * ratio * (c.head_dim + 2)) * 4;
    for (int l = 0; l < c.layers; ++l) {
        const FusedLayer& L = layers_[l];
        LSX_TRY(gemv(kNorm, kStore, L.wqkv, L.bqkv, qw + 2 * kw, c.hidden, residual_, L.input_gain, qkv_));
        AttnArgs at{};
        at.qkv = qkv_;
        at.q_gain = L.q_gain;
        at.k_gain = L.k_gain;
        at.qk_eps = c.qk_eps;
        at.keys = L.keys;
        at.values = L.values;
        at.partial = attn_partial_;
        at.out = attn_out_;
        at.rope = rope_;
        at.qheads = c.qheads;
        at.kvheads = c.kvheads;
        at.dim = c.head_dim;
        at.rotary = c.rotary;
        at.interleaved = c.interleaved;
        at.splits = splits_;
        at.scale = c.scale;
        at.state = state_;
        void* args[] = {&at};
        LSX_CUDA(launch_pdl((const void*)ak, dim3(c.kvheads, splits_), dim3(kAttnThreads), attn_smem, s, args),
                 "attention launch");
        LSX_TRY(gemv(kPlain, kResidual, L.wo, L.bo, c.hidden, qw, attn_out_, nullptr, residual_));
        LSX_TRY(gemv(kNorm, kGated, L.wgu, L.bgu, 2 * c.intermediate, c.hidden, residual_, L.post_gain, feature_));
        LSX_TRY(gemv(kPlain, kResidual, L.wd, L.bd, c.hidden, c.intermediate, feature_, nullptr, residual_));
    }
    LSX_TRY(gemv(kNormRotate, kHead, c.head, c.head_bias, c.vocab, c.hidden, residual_, c.final_gain, nullptr));
    return LSX_OK;
}

int FusedDecoder::capture() {
    graph_tried_ = true;
    cudaStream_t s = ctx_->stream;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        (void)cudaGetLastError();
        return LSX_OK;
    }
    int status = launch_all();
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &graph);
    if (status != LSX_OK || e != cudaSuccess || !graph) {
        (void)cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        return LSX_OK;  // fall back to direct launches
    }
    cudaGraphExec_t exec = nullptr;
    if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
        (void)cudaGetLastError();
        cudaGraphDestroy(graph);
        return LSX_OK;
    }
    graph_ = graph;
    graph_exec_ = exec;
    return LSX_OK;
}

int FusedDecoder::enqueue_step() {
    if (!graph_tried_) LSX_TRY(capture());
    if (graph_exec_) {
        LSX_CUDA(cudaGraphLaunch(graph_exec_, ctx_->stream), "decode graph launch");
        return LSX_OK;
    }
    return launch_all();
}

int FusedDecoder::enqueue_steps(int count) {
    for (int i = 0; i < count; ++i) LSX_TRY(enqueue_step());
    return LSX_OK;
}

}  // namespace lsx
