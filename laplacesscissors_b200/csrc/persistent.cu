// Persistent batch-1 decode engine for B200 (sm_100a).
//
// One cooperative launch runs a whole generation (diagnosis::generate_frames,
// src/diagnosis.rs:106-149: prompt tokens one at a time, then greedy argmax),
// each step in the op order of Model::decode (src/model.rs:729-853).  One CTA per
// SM; 8 compute warps and 1 producer warp.
//
// Weights: every GEMV op gives each CTA a fixed contiguous row range.  The
// producer warp walks the whole sequence of (step, layer, op, chunk) and streams
// each chunk of those rows into a shared-memory ring with 1-D bulk copies, as far
// ahead as the ring allows.  Weights never depend on activations, so HBM keeps
// streaming while the compute warps wait for the previous op's outputs.
//
// Activations: op outputs are published as 64-bit words (epoch << 32 | f32 bits)
// with single-copy-atomic stores.  A consumer polls the words it needs until every
// one carries the current epoch, so the data read IS the synchronisation (one L2
// round trip per op boundary, no separate barrier).  Each residual row is owned by
// one CTA for the whole generation, so residual updates need no read-back.
// Every wait is bounded; on timeout the kernel records a status, raises a global
// abort flag that all other waits observe, drains its copies and returns.
#include <math.h>

#include <cmath>
#include <string>

#include "device_common.cuh"
#include "persistent.cuh"

namespace lsx {
namespace {

constexpr int kWarps = 7;                       // compute warps (2 warps per SM sub-partition with the producer)
constexpr int kThreads = (kWarps + 1) * 32;     // + producer warp
constexpr int kCompute = kWarps * 32;
constexpr long long kSpin = 4000000000ll;        // ~2 s at B200 clocks

struct PArgs {
    int H, V, L, QH, KVH, D, I, rotary, interleaved, act;
    float eps, qk_eps, scale, emb_scale;
    const void* embedding;
    int emb_kind;
    const __nv_bfloat16* head;
    const float* head_bias;
    const float* final_gain;
    const FusedLayer* layers;
    const float2* rope;
    unsigned long long *t_resid, *t_qkv, *t_attn, *t_feat, *t_arg;
    DecodeState* state;
    int steps;
    int slots;
    int slot_bytes;
    int xmax;
    int scratch;  // floats of attention / edit scratch
    int rmax;     // residual rows owned per CTA, upper bound
    int prefetch; // chunks of L2 prefetch ahead of the ring copies
    int layers_offset;  // byte offset of the layer table in shared memory
};

// ------------------------------------------------------------ primitives --
__device__ __forceinline__ unsigned long long ld_relaxed(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_relaxed_int(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long tagged(uint32_t epoch, float v) {
    return ((unsigned long long)epoch << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCompute) : "memory"); }
// AND-reduction over the compute warps (named barrier 1; the producer warp never joins it).
__device__ __forceinline__ bool compute_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kCompute)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void raise_abort(DecodeState* st, int code) {
    atomicCAS(&st->status, 0, code);
}
__device__ __forceinline__ bool aborted(DecodeState* st) { return ld_relaxed_int(&st->status) != 0; }

// Argmax partial: total-order value (32) | 0x7FFFF - index (19) | epoch (13).
__device__ __forceinline__ unsigned long long arg_word(unsigned long long key, uint32_t epoch) {
    const uint32_t value = (uint32_t)(key >> 32);
    const uint32_t index = 0xffffffffu - (uint32_t)(key & 0xffffffffull);
    return ((unsigned long long)value << 32) | ((unsigned long long)((0x7FFFFu - index) & 0x7FFFFu) << 13) |
           (unsigned long long)(epoch & 0x1FFFu);
}

// Polls n tagged words until each carries `epoch`; values land in dst[0..n).
// Every stale word of a thread is re-read in the same round, so a poll costs one
// L2 round trip per round rather than one per word.  Called by all compute
// threads; false on timeout or abort.
__device__ bool poll_vector(const unsigned long long* src, int n, uint32_t epoch, float* dst, DecodeState* st) {
    const int tid = threadIdx.x;
    constexpr int kBatch = 16;
    bool ok = true;
    for (int base = 0; base < n && ok; base += kBatch * kCompute) {
        unsigned long long v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = base + tid + j * kCompute;
            v[j] = i < n ? ld_relaxed(src + i) : ((unsigned long long)epoch << 32);
        }
        long long start = 0;
        while (true) {
            bool stale = false;
#pragma unroll
            for (int j = 0; j < kBatch; ++j) stale |= (uint32_t)(v[j] >> 32) != epoch;
            if (!stale) break;
            if (start == 0) {
                start = clock64();
            } else if (clock64() - start > kSpin || aborted(st)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const int i = base + tid + j * kCompute;
                if ((uint32_t)(v[j] >> 32) != epoch) v[j] = ld_relaxed(src + i);
            }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = base + tid + j * kCompute;
            if (i < n) dst[i] = __uint_as_float((uint32_t)v[j]);
        }
    }
    if (!ok) raise_abort(st, kDeviceTimeoutEpilogue);
    return ok;
}

// Three segments polled in one round (q heads, k and v of one KV group).
__device__ bool poll_segments(const unsigned long long* s0, int n0, float* d0, const unsigned long long* s1, int n1,
                              float* d1, const unsigned long long* s2, int n2, float* d2, uint32_t epoch,
                              DecodeState* st) {
    const int tid = threadIdx.x;
    const int n = n0 + n1 + n2;
    bool ok = true;
    for (int base = 0; base < n && ok; base += 4 * kCompute) {
        unsigned long long v[4];
        const unsigned long long* src[4];
        float* dst[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = base + tid + j * kCompute;
            if (i < n0) { src[j] = s0 + i; dst[j] = d0 + i; }
            else if (i < n0 + n1) { src[j] = s1 + (i - n0); dst[j] = d1 + (i - n0); }
            else if (i < n) { src[j] = s2 + (i - n0 - n1); dst[j] = d2 + (i - n0 - n1); }
            else { src[j] = nullptr; dst[j] = nullptr; }
            v[j] = src[j] ? ld_relaxed(src[j]) : ((unsigned long long)epoch << 32);
        }
        long long start = 0;
        while (true) {
            bool stale = false;
#pragma unroll
            for (int j = 0; j < 4; ++j) stale |= (uint32_t)(v[j] >> 32) != epoch;
            if (!stale) break;
            if (start == 0) {
                start = clock64();
            } else if (clock64() - start > kSpin || aborted(st)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if ((uint32_t)(v[j] >> 32) != epoch) v[j] = ld_relaxed(src[j]);
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (dst[j]) *dst[j] = __uint_as_float((uint32_t)v[j]);
    }
    if (!ok) raise_abort(st, kDeviceTimeoutEpilogue);
    return ok;
}

struct Range {
    int lo, hi, sr, nch;
};

__device__ __forceinline__ Range range_of(int n, int unit, int K, int c, int G, int slot_bytes) {
    Range r;
    const int units = n / unit;
    r.lo = (int)(((long long)c * units) / G) * unit;
    r.hi = (int)(((long long)(c + 1) * units) / G) * unit;
    int sr = slot_bytes / (2 * K);
    sr = (sr / unit) * unit;
    if (sr < unit) sr = unit;
    r.sr = sr;
    r.nch = (r.hi - r.lo + sr - 1) / sr;
    return r;
}

// Op table: 0 qkv, 1 o, 2 gate/up, 3 down, 4 head.
__device__ __forceinline__ void op_shape(const PArgs& a, const FusedLayer* table, int op, int layer,
                                         const __nv_bfloat16** w, int* n, int* K, int* unit) {
    const FusedLayer& L = table[layer];
    switch (op) {
    case 0: *w = L.wqkv; *n = (a.QH + 2 * a.KVH) * a.D; *K = a.H; *unit = 1; break;
    case 1: *w = L.wo; *n = a.H; *K = a.QH * a.D; *unit = 1; break;
    case 2: *w = L.wgu; *n = 2 * a.I; *K = a.H; *unit = 2; break;
    case 3: *w = L.wd; *n = a.H; *K = a.I; *unit = 1; break;
    default: *w = a.head; *n = a.V; *K = a.H; *unit = 1; break;
    }
}

// Walks this CTA's weight chunks in consumption order: for every step, the four
// GEMV ops of each layer, then the head.
struct ChunkCursor {
    int step = 0, op_i = 0, ch = 0;
    const __nv_bfloat16* w = nullptr;
    int K = 0, r0 = 0, nr = 0;
    Range R{};
    bool valid = false;
    // Positions on the first chunk of the current (or next non-empty) op.
    const FusedLayer* table = nullptr;  // the shared-memory copy of the layer table
    __device__ void load(const PArgs& a, int c, int G) {
        valid = false;
        while (step < a.steps) {
            const int layer = op_i < 4 * a.L ? op_i / 4 : 0;
            const int op = op_i < 4 * a.L ? op_i % 4 : 4;
            int n, unit;
            op_shape(a, table, op, layer, &w, &n, &K, &unit);
            R = range_of(n, unit, K, c, G, a.slot_bytes);
            if (R.nch > 0) {
                ch = 0;
                r0 = R.lo;
                nr = min(R.sr, R.hi - r0);
                valid = true;
                return;
            }
            if (++op_i > 4 * a.L) {
                op_i = 0;
                ++step;
            }
        }
    }
    __device__ void advance(const PArgs& a, int c, int G) {
        if (++ch < R.nch) {  // next chunk of the same op: no range arithmetic
            r0 += R.sr;
            nr = min(R.sr, R.hi - r0);
            return;
        }
        if (++op_i > 4 * a.L) {
            op_i = 0;
            ++step;
        }
        load(a, c, G);
    }
};

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float activation(float x, int kind) {
    switch (kind) {
    case 0: return x / (1.f + expf(-x));
    case 1: return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
    case 2: return fmaxf(x, 0.f);
    default: return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
    }
}

__device__ float compute_allsum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_allsum(v);
    compute_sync();
    if (lane == 0) red[warp] = v;
    compute_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) t += red[i];
    compute_sync();
    return t;
}

struct Ring {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    int slots;
    int slot_bytes;
};

enum { kEpiStore = 0, kEpiResidual = 1, kEpiGated = 2, kEpiHead = 3 };

struct EpiCtx {
    unsigned long long* out;  // tagged destination (store, residual, gated)
    uint32_t epoch;
    float* resid;             // this CTA's residual rows (shared memory), residual epilogue
    int resid_lo;
    float* logits;            // head
    unsigned long long best;  // head, per warp (lane 0)
    bool bad;
    int act;
};

// Partial dot of one 16-byte chunk of bf16 weights with eight f32 values, as two
// independent FMA chains (shorter dependency chains than one running sum).
__device__ __forceinline__ void dot8_split(uint4 w, float4 x0, float4 x1, float& s0, float& s1) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    const float2 p0 = __bfloat1622float2(h[0]);
    const float2 p1 = __bfloat1622float2(h[1]);
    const float2 p2 = __bfloat1622float2(h[2]);
    const float2 p3 = __bfloat1622float2(h[3]);
    s0 = fmaf(p0.x, x0.x, s0);
    s1 = fmaf(p0.y, x0.y, s1);
    s0 = fmaf(p1.x, x0.z, s0);
    s1 = fmaf(p1.y, x0.w, s1);
    s0 = fmaf(p2.x, x1.x, s0);
    s1 = fmaf(p2.y, x1.y, s1);
    s0 = fmaf(p3.x, x1.z, s0);
    s1 = fmaf(p3.y, x1.w, s1);
}

// Dot products of two staged rows with x, interleaved for instruction-level
// parallelism; both results are reduced across the warp together.
template <int KCH>
__device__ __forceinline__ float2 row_dot2(const uint8_t* ra, const uint8_t* rb, const float4* xr, const float* xs,
                                           int K, int lane) {
    const uint4* wa = reinterpret_cast<const uint4*>(ra);
    const uint4* wb = reinterpret_cast<const uint4*>(rb);
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
    if (KCH > 0) {
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            const uint4 ua = wa[lane + 32 * j];
            const uint4 ub = wb[lane + 32 * j];
            dot8_split(ua, xr[2 * j], xr[2 * j + 1], a0, a1);
            dot8_split(ub, xr[2 * j], xr[2 * j + 1], b0, b1);
        }
    } else {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
        for (int c = lane; c < (K >> 3); c += 32) {
            const float4 x0 = x4[2 * c], x1 = x4[2 * c + 1];
            dot8_split(wa[c], x0, x1, a0, a1);
            dot8_split(wb[c], x0, x1, b0, b1);
        }
    }
    float a = a0 + a1, b = b0 + b1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    return make_float2(a, b);
}

__device__ __forceinline__ void epilogue(int EPI, int r, float d, const float* bias, EpiCtx& e) {
    if (bias) d += bias[r];
    if (EPI == kEpiStore) {
        st_relaxed(e.out + r, tagged(e.epoch, d));
    } else if (EPI == kEpiResidual) {
        const float v = __fadd_rn(e.resid[r - e.resid_lo], d);
        e.resid[r - e.resid_lo] = v;
        st_relaxed(e.out + r, tagged(e.epoch, v));
    } else {
        e.logits[r] = d;
        e.bad |= !isfinite(d);
        const unsigned long long key = pack_arg(d, (uint32_t)r);
        e.best = key > e.best ? key : e.best;
    }
}

// One GEMV op over this CTA's rows; consumes its chunks from the ring in order
// and releases them window by window.
// KCH > 0: K == 256 * KCH and each lane keeps its x chunks in registers;
// KCH == 0: any K % 8 == 0, x read from shared memory.
template <int EPI, int KCH>
__device__ __forceinline__ bool run_gemv(const Ring& ring, unsigned long long& q, const float* bias, int n, int K, int unit,
                         const float* xs, EpiCtx& e) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Range R = range_of(n, unit, K, blockIdx.x, gridDim.x, ring.slot_bytes);
    float4 xr[KCH > 0 ? 2 * KCH : 1];
    if (KCH > 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            xr[2 * j] = x4[2 * (lane + 32 * j)];
            xr[2 * j + 1] = x4[2 * (lane + 32 * j) + 1];
        }
    }
    const size_t row_bytes = (size_t)K * 2;
    // Ops that fit half the ring run as one window; longer ones (the head) stream
    // in short windows so freed slots are refilled continuously.
    const int half = ring.slots / 2 > 0 ? ring.slots / 2 : 1;
    const int win = R.nch <= half ? half : (half >= 4 ? 4 : half);
    const int slot0 = (int)(q % (unsigned long long)ring.slots);
    const uint32_t round0 = (uint32_t)(q / (unsigned long long)ring.slots);
    bool ok = true;
    for (int w0 = 0; w0 < R.nch && ok; w0 += win) {
        const int wn = min(win, R.nch - w0);
        const int rs = R.lo + w0 * R.sr;
        const int re = min(R.hi, R.lo + (w0 + wn) * R.sr);
        // Wait once for every chunk of the window (immediate when already landed).
        bool landed = true;
        for (int ch = w0; ch < w0 + wn; ++ch) {
            const int lin = slot0 + ch;
            const int slot = lin % ring.slots;
            const uint32_t parity = (round0 + (uint32_t)(lin / ring.slots)) & 1u;
            landed &= mbar_wait_bounded(&ring.full[slot], parity);
        }
        ok = __all_sync(0xffffffffu, landed);
        auto row_at = [&](int r) -> const uint8_t* {
            const int local = r - R.lo;
            const int ch = local / R.sr;
            const int slot = (slot0 + ch) % ring.slots;
            return ring.base + (size_t)slot * ring.slot_bytes + (size_t)(local - ch * R.sr) * row_bytes;
        };
        if (ok) {
            if (EPI == kEpiGated) {
                for (int p = warp; p < (re - rs) / 2; p += kWarps) {
                    const int r = rs + 2 * p;
                    const uint8_t* g_row = row_at(r);  // even rows per chunk: pairs stay whole
                    const float2 gu = row_dot2<KCH>(g_row, g_row + row_bytes, xr, xs, K, lane);
                    if (lane == 0) {
                        float g = gu.x, u = gu.y;
                        if (bias) {
                            g += bias[r];
                            u += bias[r + 1];
                        }
                        st_relaxed(e.out + (r >> 1), tagged(e.epoch, activation(g, e.act) * u));
                    }
                }
            } else {
                for (int r = rs + warp; r < re; r += 2 * kWarps) {
                    const int r2 = r + kWarps;
                    const uint8_t* pa = row_at(r);
                    const uint8_t* pb = r2 < re ? row_at(r2) : pa;
                    const float2 d = row_dot2<KCH>(pa, pb, xr, xs, K, lane);
                    if (lane == 0) {
                        epilogue(EPI, r, d.x, bias, e);
                        if (r2 < re) epilogue(EPI, r2, d.y, bias, e);
                    }
                }
            }
        }
        ok = compute_and(ok);
        if (tid == 0)
            for (int ch = w0; ch < w0 + wn; ++ch) mbar_arrive(&ring.empty[(slot0 + ch) % ring.slots]);
    }
    q += (unsigned long long)R.nch;
    return ok;
}

// Attention of KV group g at `pos` (kernels/ops.py:69-101 after QK-norm and RoPE):
// polls the group's q/k/v, normalises and rotates them, appends k/v to the f32
// cache, attends over positions 0..pos and publishes the group's output heads.
template <int RATIO, int DPL>
__device__ __forceinline__ bool attention_group(const PArgs& a, const FusedLayer& L, int g, int pos, uint32_t e_qkv, uint32_t e_attn,
                                float* sm) {
    constexpr int D = DPL * 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float* raw = sm;                    // (RATIO + 2) * D: q heads, k, v
    float* qs = raw + (RATIO + 2) * D;  // RATIO * D (normed, rotated)
    float* ks = qs + RATIO * D;         // D
    float* merge = ks + D;              // kWarps * RATIO * (D + 2)
    const int qw = a.QH * D, kw = a.KVH * D;
    // The cached positions 0..pos-1 do not depend on this step: start loading this
    // warp's first batch of them before waiting for q, k and v.
    constexpr int PB = 4;
    const float* kbase = L.keys + (size_t)g * D;
    const float* vbase = L.values + (size_t)g * D;
    float kpre[PB][DPL], vpre[PB][DPL];
#pragma unroll
    for (int b = 0; b < PB; ++b) {
        const int t = warp + kWarps * b;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            kpre[b][j] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * j) : 0.f;
            vpre[b][j] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * j) : 0.f;
        }
    }
    // Gains and the RoPE row of this position are also independent of the step's
    // activations: fetch them now.
    float qg[DPL], kg[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        qg[j] = L.q_gain ? __ldg(L.q_gain + lane + 32 * j) : 1.f;
        kg[j] = L.k_gain ? __ldg(L.k_gain + lane + 32 * j) : 1.f;
    }
    const int half = a.rotary / 2;
    constexpr int kRopeRegs = 4;  // rotary pairs up to 4 * kCompute
    float2 cs_pre[kRopeRegs];
#pragma unroll
    for (int j = 0; j < kRopeRegs; ++j) {
        const int i = tid + j * kCompute;
        cs_pre[j] = i < half ? a.rope[(size_t)pos * half + i] : make_float2(1.f, 0.f);
    }
    bool ok = poll_segments(a.t_qkv + (size_t)g * RATIO * D, RATIO * D, raw, a.t_qkv + qw + (size_t)g * D, D,
                            raw + RATIO * D, a.t_qkv + qw + kw + (size_t)g * D, D, raw + (RATIO + 1) * D, e_qkv,
                            a.state);
    if (!compute_and(ok)) return false;
    float* cs_s = merge;  // RoPE row for this position, shared by the heads
#pragma unroll
    for (int j = 0; j < kRopeRegs; ++j) {
        const int i = tid + j * kCompute;
        if (i < half) reinterpret_cast<float2*>(cs_s)[i] = cs_pre[j];
    }
    for (int h = warp; h < RATIO + 1; h += kWarps) {  // Qwen3 q_norm / k_norm per head
        const bool has = h < RATIO ? L.q_gain != nullptr : L.k_gain != nullptr;
        if (!has) continue;
        float* row = raw + h * D;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss = fmaf(row[lane + 32 * j], row[lane + 32 * j], ss);
        ss = warp_allsum(ss);
        const float inverse = rsqrtf(ss / (float)D + a.qk_eps);
#pragma unroll
        for (int j = 0; j < DPL; ++j)
            row[lane + 32 * j] = row[lane + 32 * j] * inverse * (h < RATIO ? qg[j] : kg[j]);
    }
    compute_sync();
    for (int i = tid; i < (RATIO + 1) * D; i += kCompute) {  // kernels/ops.py:48-66
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
            const float2 cs = reinterpret_cast<const float2*>(cs_s)[pair];
            y = x * cs.x + sign * raw[h * D + other] * cs.y;
        }
        if (h < RATIO) qs[i] = y;
        else ks[local] = y;
    }
    compute_sync();
    const float* vs = raw + (RATIO + 1) * D;
    float* kd = L.keys + (size_t)pos * kw + (size_t)g * D;
    float* vd = L.values + (size_t)pos * kw + (size_t)g * D;
    for (int i = tid; i < D; i += kCompute) {  // kernels/ops.py:69-73
        kd[i] = ks[i];
        vd[i] = vs[i];
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
    // Scores of a batch of positions are formed and reduced together, then one
    // online-softmax update folds the whole batch in (kernels/ops.py:88-99).
    auto attend_batch = [&](const float (*kv)[DPL], const float (*vv)[DPL], int nb) {
        float sc[PB][RATIO];
#pragma unroll
        for (int b = 0; b < PB; ++b)
#pragma unroll
            for (int h = 0; h < RATIO; ++h) {
                float t = 0.f;
#pragma unroll
                for (int j = 0; j < DPL; ++j) t = fmaf(q[h][j], kv[b][j], t);
                sc[b][h] = t;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int b = 0; b < PB; ++b)
#pragma unroll
                for (int h = 0; h < RATIO; ++h) sc[b][h] += __shfl_xor_sync(0xffffffffu, sc[b][h], o);
#pragma unroll
        for (int h = 0; h < RATIO; ++h) {
            float mn = m[h];
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                sc[b][h] = b < nb ? sc[b][h] * a.scale : -INFINITY;
                mn = fmaxf(mn, sc[b][h]);
            }
            const float carry = expf(m[h] - mn);
            float pr[PB], psum = 0.f;
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                pr[b] = b < nb ? expf(sc[b][h] - mn) : 0.f;
                psum += pr[b];
            }
            l[h] = l[h] * carry + psum;
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                float v = acc[h][j] * carry;
#pragma unroll
                for (int b = 0; b < PB; ++b) v = fmaf(pr[b], vv[b][j], v);
                acc[h][j] = v;
            }
            m[h] = mn;
        }
    };
    // Cached positions in batches of PB per warp, every batch's loads issued together.
    for (int i0 = 0; warp + kWarps * i0 < pos; i0 += PB) {
        if (i0 > 0) {
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                const int t = warp + kWarps * (i0 + b);
#pragma unroll
                for (int j = 0; j < DPL; ++j) {
                    kpre[b][j] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * j) : 0.f;
                    vpre[b][j] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * j) : 0.f;
                }
            }
        }
        int nb = 0;
#pragma unroll
        for (int b = 0; b < PB; ++b) nb += warp + kWarps * (i0 + b) < pos ? 1 : 0;
        attend_batch(kpre, vpre, nb);
    }
    if (warp == 0) {  // the current position, from shared memory
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            kpre[0][j] = ks[lane + 32 * j];
            vpre[0][j] = vs[lane + 32 * j];
        }
        attend_batch(kpre, vpre, 1);
    }
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
    compute_sync();
    for (int i = tid; i < RATIO * D; i += kCompute) {
        const int h = i / D, d = i % D;
        float M = -INFINITY;
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, merge[(w * RATIO + h) * stride]);
        float Lsum = 0.f, O = 0.f;
        for (int w = 0; w < kWarps; ++w) {
            const float* sl = merge + (size_t)(w * RATIO + h) * stride;
            if (sl[0] == -INFINITY) continue;
            const float ex = expf(sl[0] - M);
            Lsum = fmaf(sl[1], ex, Lsum);
            O = fmaf(sl[2 + d], ex, O);
        }
        st_relaxed(a.t_attn + (size_t)(g * RATIO + h) * D + d, tagged(e_attn, O / Lsum));
    }
    compute_sync();
    return true;
}

// Norm gains of one width, fetched into registers before the activations they
// scale are waited for (hides the load behind the poll).
constexpr int kGainRegs = 24;  // widths up to 24 * kCompute
struct GainRegs {
    float g[kGainRegs];
    __device__ __forceinline__ void load(const float* gain, int n) {
#pragma unroll
        for (int j = 0; j < kGainRegs; ++j) {
            const int i = threadIdx.x + j * kCompute;
            g[j] = i < n ? __ldg(gain + i) : 0.f;
        }
    }
};

// RMSNorm of xs in place (kernels/ops.py:31-45): x * rsqrt(mean(x^2) + eps) * gain.
__device__ void rms_norm_inplace(float* xs, int n, const GainRegs& gain, float eps, float* red) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kGainRegs; ++j) {
        const int i = threadIdx.x + j * kCompute;
        if (i < n) ss = fmaf(xs[i], xs[i], ss);
    }
    ss = compute_allsum(ss, red);
    const float inverse = rsqrtf(ss / (float)n + eps);
#pragma unroll
    for (int j = 0; j < kGainRegs; ++j) {
        const int i = threadIdx.x + j * kCompute;
        if (i < n) xs[i] = xs[i] * inverse * gain.g[j];
    }
    compute_sync();
}

// KH, KQ, KI: 16-byte chunks per lane of x for the hidden, query and
// intermediate widths (0: x stays in shared memory).
template <int KH, int KQ, int KI, int RATIO, int DPL>
__global__ void __launch_bounds__(kThreads, 1) persistent_decode_kernel(const PArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    Ring ring;
    ring.base = smem;
    ring.slots = a.slots;
    ring.slot_bytes = a.slot_bytes;
    float* xs = reinterpret_cast<float*>(smem + (size_t)a.slots * a.slot_bytes);
    float* scratch = xs + a.xmax;
    float* resid = scratch + a.scratch;
    float* red = resid + a.rmax;
    ring.full = reinterpret_cast<uint64_t*>(red + 64);
    ring.empty = ring.full + a.slots;
    volatile int* s_stop = reinterpret_cast<volatile int*>(ring.empty + a.slots);
    int* s_issued = const_cast<int*>(s_stop) + 1;
    FusedLayer* layers = reinterpret_cast<FusedLayer*>(smem + a.layers_offset);
    DecodeState* st = a.state;
    // The per-layer pointer table lives in shared memory: reading it from global
    // memory would miss L2 (the weight stream evicts it) on every op.
    for (int i = tid; i < a.L * (int)(sizeof(FusedLayer) / 8); i += kThreads)
        reinterpret_cast<unsigned long long*>(layers)[i] = reinterpret_cast<const unsigned long long*>(a.layers)[i];

    if (tid == 0) {
        for (int i = 0; i < a.slots; ++i) {
            mbar_init(&ring.full[i], 1);
            mbar_init(&ring.empty[i], 1);
        }
        *s_stop = 0;
        *s_issued = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const int P = st->prompt_length, maximum = st->maximum, mode = st->mode;
    const int pos0 = st->position;
    const uint32_t base = st->epoch;
    const uint32_t per_step = 5u * (uint32_t)a.L + 1u;

    if (warp == kWarps) {  // ---------------------------------- producer warp
        if (lane == 0) {
            unsigned long long q = 0;
            bool go = true;
            // Copies into the ring follow `cur`; L2 prefetches run `a.prefetch` chunks
            // ahead of it so HBM reads start about a layer before the ring can hold them.
            const uint64_t policy = l2_evict_first_policy();
            ChunkCursor cur, pre;
            cur.table = layers;
            pre.table = layers;
            cur.load(a, c, G);
            pre.load(a, c, G);
            for (int i = 0; i < a.prefetch && pre.valid; ++i) {
                prefetch_l2(pre.w + (size_t)pre.r0 * pre.K, (uint32_t)((size_t)pre.nr * pre.K * 2));
                pre.advance(a, c, G);
            }
            for (; cur.valid && go; ++q) {
                const int slot = (int)(q % (unsigned long long)a.slots);
                const unsigned long long round = q / (unsigned long long)a.slots;
                if (round > 0) {
                    // wait until the consumers released this slot's previous chunk
                    const uint32_t addr = smem_u32(&ring.empty[slot]);
                    const uint32_t parity = (uint32_t)((round - 1) & 1ull);
                    long long start = 0;
                    while (!mbar_try_wait(addr, parity)) {
                        if (*s_stop) {
                            go = false;
                            break;
                        }
                        if (start == 0) start = clock64();
                        else if (clock64() - start > kSpin) {
                            raise_abort(st, kDeviceTimeoutWeights);
                            go = false;
                            break;
                        }
                    }
                    if (!go) break;
                }
                const uint32_t bytes = (uint32_t)((size_t)cur.nr * cur.K * 2);
                mbar_expect_tx(&ring.full[slot], bytes);
                bulk_load_hint(ring.base + (size_t)slot * a.slot_bytes, cur.w + (size_t)cur.r0 * cur.K, bytes,
                               &ring.full[slot], policy);
                cur.advance(a, c, G);
                if (pre.valid) {
                    prefetch_l2(pre.w + (size_t)pre.r0 * pre.K, (uint32_t)((size_t)pre.nr * pre.K * 2));
                    pre.advance(a, c, G);
                }
            }
            *s_issued = (int)q;
        }
        __syncwarp();
    } else {  // ------------------------------------------------ compute warps
        unsigned long long q = 0;
        const Range RH = range_of(a.H, 1, a.H, c, G, a.slot_bytes);  // residual rows owned by this CTA
        bool ok = true;
        int steps_done = 0;
        uint32_t token = 0, next_token = 0;
        int generated = st->generated, stopped = 0;
        const bool frames = st->frames != 0;
        for (int step = 0; step < a.steps && ok; ++step) {
            const uint32_t e0 = base + (uint32_t)step * per_step;  // epochs of this step: e0 + 1 ..
            const int pos = pos0 + step;
            // ---- token: prompt, injected vector, or the previous step's argmax
            if (!(mode == 1 && step == 0)) token = step < P ? st->prompt[step] : next_token;
            // ---- residual = embedding row (Model::embedding_tensor, src/model.rs:620-631) or injection
            for (int i = tid; i < a.H; i += kCompute) {
                float v;
                if (mode == 1 && step == 0) {
                    v = st->inject[i];
                } else {
                    const size_t off = (size_t)token * a.H + i;
                    if (a.emb_kind == LSX_BF16) v = __bfloat162float(((const __nv_bfloat16*)a.embedding)[off]);
                    else if (a.emb_kind == LSX_F32) v = ((const float*)a.embedding)[off];
                    else v = __half2float(((const __half*)a.embedding)[off]);
                    if (a.emb_scale != 1.f) v = __fadd_rn(v, __fmul_rn(a.emb_scale - 1.f, v));
                }
                xs[i] = v;
            }
            compute_sync();
            for (int i = tid; i < RH.hi - RH.lo; i += kCompute) resid[i] = xs[RH.lo + i];
            for (int layer = 0; layer < a.L && ok; ++layer) {
                const FusedLayer& Lr = layers[layer];
                const uint32_t e_qkv = e0 + 5u * layer + 1u, e_attn = e_qkv + 1u, e_o = e_qkv + 2u,
                               e_gu = e_qkv + 3u, e_down = e_qkv + 4u;
                // qkv: RMSNorm(residual) -> [q; k; v]
                GainRegs gain;
                gain.load(Lr.input_gain, a.H);
                if (layer > 0) ok = compute_and(poll_vector(a.t_resid, a.H, e_qkv - 1u, xs, st));
                if (!ok) break;
                rms_norm_inplace(xs, a.H, gain, a.eps, red);
                EpiCtx e{};
                e.out = a.t_qkv;
                e.epoch = e_qkv;
                e.act = a.act;
                ok = run_gemv<kEpiStore, KH>(ring, q, Lr.bqkv, (a.QH + 2 * a.KVH) * a.D, a.H, 1, xs, e);
                if (!ok) break;
                // attention: KV groups on CTAs 0..KVH-1
                if (c < a.KVH) {
                    ok = attention_group<RATIO, DPL>(a, Lr, c, pos, e_qkv, e_attn, scratch);
                    if (!ok) break;
                }
                // o: residual += Wo attn
                ok = compute_and(poll_vector(a.t_attn, a.QH * a.D, e_attn, xs, st));
                if (!ok) break;
                e.out = a.t_resid;
                e.epoch = e_o;
                e.resid = resid;
                e.resid_lo = RH.lo;
                ok = run_gemv<kEpiResidual, KQ>(ring, q, Lr.bo, a.H, a.QH * a.D, 1, xs, e);
                if (!ok) break;
                // gate/up: RMSNorm(residual) -> act(gate) * up
                gain.load(Lr.post_gain, a.H);
                ok = compute_and(poll_vector(a.t_resid, a.H, e_o, xs, st));
                if (!ok) break;
                rms_norm_inplace(xs, a.H, gain, a.eps, red);
                e.out = a.t_feat;
                e.epoch = e_gu;
                ok = run_gemv<kEpiGated, KH>(ring, q, Lr.bgu, 2 * a.I, a.H, 2, xs, e);
                if (!ok) break;
                // down: residual += Wd feature
                ok = compute_and(poll_vector(a.t_feat, a.I, e_gu, xs, st));
                if (!ok) break;
                e.out = a.t_resid;
                e.epoch = e_down;
                ok = run_gemv<kEpiResidual, KI>(ring, q, Lr.bd, a.H, a.I, 1, xs, e);
            }
            if (!ok) break;
            // ---- head: final RMSNorm, optional edit, logits and first argmax
            const uint32_t e_last = e0 + 5u * (uint32_t)a.L, e_head = e_last + 1u;
            GainRegs fgain;
            fgain.load(a.final_gain, a.H);
            ok = compute_and(poll_vector(a.t_resid, a.H, e_last, xs, st));
            if (!ok) break;
            rms_norm_inplace(xs, a.H, fgain, a.eps, red);
            const int slot_idx = step - (P - 1);
            const bool framed = frames && slot_idx >= 0;
            float* hid = framed ? st->hidden_frames + (size_t)slot_idx * a.H : st->hidden_scratch;
            float* logits = framed ? st->logits_frames + (size_t)slot_idx * a.V : st->logits_scratch;
            if (c == 0) {
                bool bad = false;
                for (int i = tid; i < a.H; i += kCompute) {
                    hid[i] = xs[i];
                    bad |= !isfinite(xs[i]);
                }
                if (!compute_and(!bad) && tid == 0) atomicOr(&st->nonfinite, 1);
            }
            if (st->rot_kind == 1) {  // kernels/ops.py:125-135
                const float* u = st->rot_u;
                const float* v = st->rot_v;
                float hu = 0.f, hv = 0.f;
                for (int i = tid; i < a.H; i += kCompute) {
                    hu = fmaf(xs[i], u[i], hu);
                    hv = fmaf(xs[i], v[i], hv);
                }
                hu = compute_allsum(hu, red);
                hv = compute_allsum(hv, red + 16);
                const float A = st->rot_a, B = st->rot_b;
                for (int i = tid; i < a.H; i += kCompute)
                    xs[i] = xs[i] + u[i] * (A * hu + B * hv) + v[i] * (A * hv - B * hu);
                compute_sync();
            } else if (st->rot_kind == 2) {  // DeviceRotation::apply Joint (src/model.rs:350-361)
                const int r = st->rot_rank;
                float* coords = scratch;
                float* shift = scratch + 256;
                for (int k = warp; k < r; k += kWarps) {
                    float d = 0.f;
                    for (int j = lane; j < a.H; j += 32) d = fmaf(st->rot_basis[(size_t)k * a.H + j], xs[j], d);
                    d = warp_allsum(d);
                    if (lane == 0) coords[k] = d;
                }
                compute_sync();
                for (int i = tid; i < r; i += kCompute) {
                    float d = 0.f;
                    for (int j = 0; j < r; ++j) d = fmaf(st->rot_delta[i * r + j], coords[j], d);
                    shift[i] = d;
                }
                compute_sync();
                for (int j = tid; j < a.H; j += kCompute) {
                    float d = 0.f;
                    for (int k = 0; k < r; ++k) d = fmaf(st->rot_basis[(size_t)k * a.H + j], shift[k], d);
                    xs[j] = __fadd_rn(xs[j], d);
                }
                compute_sync();
            }
            EpiCtx e{};
            e.logits = logits;
            e.best = 0ull;
            ok = run_gemv<kEpiHead, KH>(ring, q, a.head_bias, a.V, a.H, 1, xs, e);
            if (!ok) break;
            unsigned long long* rb = reinterpret_cast<unsigned long long*>(red);
            if (lane == 0) rb[warp] = e.best;
            if (!compute_and(!e.bad) && tid == 0) atomicOr(&st->nonfinite, 1);
            if (tid == 0) {
                unsigned long long b = 0ull;
                for (int i = 0; i < kWarps; ++i) b = rb[i] > b ? rb[i] : b;
                st_relaxed(a.t_arg + c, arg_word(b, e_head));
            }
            // ---- gather the step's argmax from every CTA's partial
            unsigned long long* gathered = reinterpret_cast<unsigned long long*>(scratch);
            if (tid < G) {
                const unsigned long long* src = a.t_arg + tid;
                unsigned long long v = ld_relaxed(src);
                long long start = 0;
                while ((uint32_t)(v & 0x1FFFull) != (e_head & 0x1FFFu)) {
                    if (start == 0) start = clock64();
                    else if (clock64() - start > kSpin || aborted(st)) {
                        ok = false;
                        break;
                    }
                    v = ld_relaxed(src);
                }
                gathered[tid] = v;
            }
            ok = compute_and(ok);
            if (!ok) {
                raise_abort(st, kDeviceTimeoutEpilogue);
                break;
            }
            unsigned long long best = 0ull;
            for (int i = 0; i < G; ++i) best = gathered[i] > best ? gathered[i] : best;
            const uint32_t arg = 0x7FFFFu - (uint32_t)((best >> 13) & 0x7FFFFu);
            compute_sync();  // everyone has read the gathered partials before scratch is reused
            steps_done = step + 1;
            if (slot_idx >= 0) {  // generate_frames bookkeeping (src/diagnosis.rs:122-145)
                if (c == 0 && tid == 0) st->tokens_out[slot_idx] = arg;
                generated = slot_idx + 1;
                bool stop = generated >= maximum;
                for (int i = 0; i < st->n_stop; ++i) stop |= st->stop[i] == arg;
                if (stop) stopped = 1;
            }
            if (c == 0 && tid == 0) st->argmax = arg;
            next_token = arg;  // every thread of every CTA computed the same maximum
            if (stopped) break;
        }
        // tell the producer to stop and record the final state
        if (tid == 0) *s_stop = 1;
        if (c == 0 && tid == 0) {
            st->position = pos0 + steps_done;
            st->generated = generated;
            st->stopped = stopped;
            st->epoch = base + (uint32_t)(steps_done + 1) * per_step;
        }
    }
    __syncthreads();
    // Drain: no bulk copy may still be in flight into this block's shared memory.
    if (tid == 0) {
        const long long issued = *s_issued;
        for (long long qq = issued > a.slots ? issued - a.slots : 0; qq < issued; ++qq) {
            const int slot = (int)(qq % a.slots);
            mbar_wait_bounded(&ring.full[slot], (uint32_t)((qq / a.slots) & 1));
        }
    }
}

using PKernel = void (*)(const PArgs);

PKernel kernel_for(const FusedConfig& c) {
    const int qw = c.qheads * c.head_dim;
    const int ratio = c.qheads / c.kvheads, dpl = c.head_dim / 32;
    // Register-resident x needs compile-time widths; attention shapes likewise.
    if (c.hidden == 1024 && qw == 2048 && c.intermediate == 3072 && ratio == 2 && dpl == 4)
        return persistent_decode_kernel<4, 8, 12, 2, 4>;  // Qwen3-0.6B
    if (c.hidden == 2560 && ratio == 4 && dpl == 4) return persistent_decode_kernel<10, 0, 0, 4, 4>;  // Qwen3-4B
    if (ratio == 4 && dpl == 4) return persistent_decode_kernel<0, 0, 0, 4, 4>;  // Qwen3-8B and others
    if (ratio == 2 && dpl == 4) return persistent_decode_kernel<0, 0, 0, 2, 4>;
    if (ratio == 2 && dpl == 2) return persistent_decode_kernel<0, 0, 0, 2, 2>;
    if (ratio == 1 && dpl == 4) return persistent_decode_kernel<0, 0, 0, 1, 4>;
    if (ratio == 8 && dpl == 4) return persistent_decode_kernel<0, 0, 0, 8, 4>;
    return nullptr;
}

}  // namespace

PersistentDecoder::~PersistentDecoder() {
    for (void* p : owned_) cudaFree(p);
}

bool PersistentDecoder::eligible(const FusedConfig& c, const lsx_ctx* ctx, std::string* why) {
    if (!FusedDecoder::eligible(c, why)) return false;
    if (!kernel_for(c)) {
        if (why) *why = "no persistent kernel instantiation for this GQA ratio / head_dim";
        return false;
    }
    const int ratio = c.qheads / c.kvheads;
    if (ratio == 8 && c.head_dim == 256) {
        if (why) *why = "GQA ratio 8 with head_dim 256";
        return false;
    }
    if (c.vocab > 0x7FFFF) {
        if (why) *why = "vocabulary above 524287";
        return false;
    }
    if (c.kvheads > ctx->sm_count) {
        if (why) *why = "more KV heads than SMs";
        return false;
    }
    return true;
}

int PersistentDecoder::build(lsx_ctx* ctx, const FusedConfig& c, const std::vector<FusedLayer>& layers) {
    std::string why;
    if (!eligible(c, ctx, &why)) return fail(LSX_E_UNSUPPORTED, "persistent decode plan: " + why);
    ctx_ = ctx;
    config_ = c;
    grid_ = ctx->sm_count;
    auto alloc = [&](size_t bytes, void** p) -> int {
        LSX_CUDA(cudaMalloc(p, bytes), "persistent decode buffer");
        LSX_CUDA(cudaMemset(*p, 0, bytes), "persistent decode buffer");
        owned_.push_back(*p);
        return LSX_OK;
    };
    const int qw = c.qheads * c.head_dim, kw = c.kvheads * c.head_dim;
    LSX_TRY(alloc(sizeof(DecodeState), (void**)&state_));
    LSX_TRY(alloc(layers.size() * sizeof(FusedLayer), &layers_dev_));
    LSX_CUDA(cudaMemcpy(layers_dev_, layers.data(), layers.size() * sizeof(FusedLayer), cudaMemcpyHostToDevice),
             "layer table upload");
    LSX_TRY(alloc((size_t)c.hidden * 8, (void**)&t_resid_));
    LSX_TRY(alloc((size_t)(qw + 2 * kw) * 8, (void**)&t_qkv_));
    LSX_TRY(alloc((size_t)qw * 8, (void**)&t_attn_));
    LSX_TRY(alloc((size_t)c.intermediate * 8, (void**)&t_feat_));
    LSX_TRY(alloc((size_t)grid_ * 8, (void**)&t_arg_));
    const int half = c.rotary / 2;
    if (half > 0) {
        std::vector<float2> table((size_t)c.capacity * half);
        for (int p = 0; p < c.capacity; ++p)
            for (int i = 0; i < half; ++i) {
                const double angle = (double)p * std::pow(c.theta, -2.0 * i / (double)c.rotary);
                table[(size_t)p * half + i] = make_float2((float)std::cos(angle), (float)std::sin(angle));
            }
        LSX_TRY(alloc(table.size() * sizeof(float2), (void**)&rope_));
        LSX_CUDA(cudaMemcpy(rope_, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice),
                 "rope table upload");
    }
    // Shared memory: ring slots, x buffer, attention/edit scratch, owned residual rows.
    int slot_bytes = 16384;
    const int ks[4] = {c.hidden, qw, c.hidden, c.intermediate};
    const int units[4] = {1, 1, 2, 1};
    for (int i = 0; i < 4; ++i) slot_bytes = std::max(slot_bytes, units[i] * ks[i] * 2);
    slot_bytes = (slot_bytes + 127) & ~127;
    const int ratio = c.qheads / c.kvheads;
    const int xmax = (std::max(std::max(c.hidden, qw), c.intermediate) + 3) & ~3;
    const int scratch = (std::max((2 * ratio + 3) * c.head_dim + 8 * ratio * (c.head_dim + 2), 512) + 3) & ~3;
    const int rmax = ((c.hidden + grid_ - 1) / grid_ + 1 + 3) & ~3;
    const size_t fixed = (size_t)(xmax + scratch + rmax + 64) * 4 + 16 + 16 + layers.size() * sizeof(FusedLayer);
    const size_t limit = ctx->smem_optin;
    if (fixed + 2 * (size_t)slot_bytes + 32 > limit) return fail(LSX_E_UNSUPPORTED, "persistent decode plan: smem");
    slots_ = (int)((limit - fixed - 64) / ((size_t)slot_bytes + 16));
    if (slots_ > 16) slots_ = 16;
    smem_ = (size_t)slots_ * slot_bytes + fixed + (size_t)slots_ * 16 + 16;
    PKernel k = kernel_for(c);
    LSX_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_),
             "persistent smem attribute");
    int per_sm = 0;
    LSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem_), "persistent occupancy");
    if (per_sm < 1) return fail(LSX_E_UNSUPPORTED, "persistent decode plan: one block per SM does not fit");
    return LSX_OK;
}

int PersistentDecoder::run(int steps) {
    const FusedConfig& c = config_;
    PArgs a{};
    a.H = c.hidden;
    a.V = c.vocab;
    a.L = c.layers;
    a.QH = c.qheads;
    a.KVH = c.kvheads;
    a.D = c.head_dim;
    a.I = c.intermediate;
    a.rotary = c.rotary;
    a.interleaved = c.interleaved;
    a.act = c.activation;
    a.eps = c.eps;
    a.qk_eps = c.qk_eps;
    a.scale = c.scale;
    a.emb_scale = c.embedding_scale;
    a.embedding = c.embedding;
    a.emb_kind = c.embedding_kind;
    a.head = c.head;
    a.head_bias = c.head_bias;
    a.final_gain = c.final_gain;
    a.layers = (const FusedLayer*)layers_dev_;
    a.rope = rope_;
    a.t_resid = t_resid_;
    a.t_qkv = t_qkv_;
    a.t_attn = t_attn_;
    a.t_feat = t_feat_;
    a.t_arg = t_arg_;
    a.state = state_;
    a.steps = steps;
    a.slots = slots_;
    const int qw = c.qheads * c.head_dim;
    int slot_bytes = 16384;
    const int ks[4] = {c.hidden, qw, c.hidden, c.intermediate};
    const int units[4] = {1, 1, 2, 1};
    for (int i = 0; i < 4; ++i) slot_bytes = std::max(slot_bytes, units[i] * ks[i] * 2);
    a.slot_bytes = (slot_bytes + 127) & ~127;
    const int ratio = c.qheads / c.kvheads;
    a.xmax = (std::max(std::max(c.hidden, qw), c.intermediate) + 3) & ~3;
    a.scratch = (std::max((2 * ratio + 3) * c.head_dim + 8 * ratio * (c.head_dim + 2), 512) + 3) & ~3;
    a.rmax = ((c.hidden + grid_ - 1) / grid_ + 1 + 3) & ~3;
    // About one layer of this CTA's chunks: 4 GEMV ops of roughly 16 KB chunks.
    {
        const size_t layer_bytes = (size_t)2 * c.hidden * ((size_t)(c.qheads + 2 * c.kvheads) * c.head_dim + 2 * c.intermediate) +
                                   (size_t)2 * c.hidden * ((size_t)c.qheads * c.head_dim + c.intermediate);
        const size_t per_cta = layer_bytes / grid_;
        (void)per_cta;
        a.prefetch = 0;  // measured: L2 prefetch through the bulk-copy engine slows the stream
    }
    // Layer table after the barriers and flags, 8-byte aligned.
    a.layers_offset = (int)(((size_t)a.slots * a.slot_bytes + (size_t)(a.xmax + a.scratch + a.rmax + 64) * 4 +
                             (size_t)a.slots * 16 + 16 + 15) & ~(size_t)15);
    void* args[] = {&a};
    LSX_CUDA(cudaLaunchCooperativeKernel((const void*)kernel_for(c), dim3(grid_), dim3(kThreads), args, smem_,
                                         ctx_->stream),
             "persistent decode launch");
    return LSX_OK;
}

}  // namespace lsx
