// Persistent batch-1 decode engine for B200 (sm_100a).
//
// One cooperative launch runs a whole generation (diagnosis::generate_frames,
// src/diagnosis.rs:106-149: prompt tokens one at a time, then greedy argmax),
// each step in the op order of Model::decode (src/model.rs:729-853).  One CTA per
// SM; 7 compute warps and 1 producer warp.
//
// Weights: every GEMV op gives each CTA a fixed contiguous row range, cut into
// chunks of a power-of-two number of rows.  The producer warp walks the whole
// sequence of (step, layer, op, chunk) and streams each chunk into a shared-memory
// ring with 1-D bulk copies, as far ahead as the ring allows.  Weights never depend
// on activations, so HBM keeps streaming while the compute warps wait for the
// previous op's outputs; a chunk typically lands several microseconds before use.
//
// Compute: a GEMV op is latency-bound at batch 1 (a CTA holds only tens of rows),
// so each warp takes NR rows at once: all NR x KCH 16-byte weight loads issue
// together against x held in registers, and the NR partial sums are reduced across
// the warp with one transposing butterfly (log2(NR) halving rounds, then plain
// rounds), which leaves every row's total in 32/NR lanes.  RMSNorm is folded into
// the register load of x: every warp holds all of x, so each forms the sum of
// squares itself and no block-wide reduction is needed.
//
// Activations: op outputs are published as 64-bit words (epoch << 32 | f32 bits)
// with single-copy-atomic stores.  A consumer polls the words it needs until every
// one carries the current epoch, so the data read IS the synchronisation (one L2
// round trip per op boundary, no separate barrier).  Each residual row is owned by
// one CTA for the whole generation, so residual updates need no read-back.
// Attention runs one query head per CTA (CTAs 0..qheads-1), with QK-norm and RoPE in
// registers.  Every wait is bounded; on timeout the kernel records a status, raises a
// global abort flag that all other waits observe, drains its copies and returns.
#include <math.h>

#include <cmath>
#include <cstdlib>
#include <string>

#include "device_common.cuh"
#include "persistent.cuh"

// Phase marks for timing builds; empty in the library.
#ifndef LSX_PHASE_MARK
#define LSX_PHASE_MARK(k)
#endif
#ifndef LSX_HEAD_MARK
#define LSX_HEAD_MARK(k)
#endif
#ifndef LSX_WINDOW_MARK
#define LSX_WINDOW_MARK(k)
#endif

namespace lsx {
namespace {

constexpr int kWarps = 7;                    // compute warps (2 warps per SM sub-partition with the producer)
constexpr int kThreads = (kWarps + 1) * 32;  // + producer warp
constexpr int kCompute = kWarps * 32;
constexpr long long kSpin = 4000000000ll;     // ~2 s at B200 clocks
// Argmax partials sit one per 128-byte line: every CTA polls every partial, and
// packed into a few lines those polls queued on a handful of L2 slices.
constexpr int kArgStride = 16;

// Clock cycles an exchange wait may spin before it gives up: kSpin, or the
// failure-path test hook's shorter limit (DecodeState::spin_limit).  Set by thread 0
// before the block's first barrier.
__shared__ long long s_spin;

enum { kOpQkv = 0, kOpO = 1, kOpGu = 2, kOpDown = 3, kOpHead = 4, kOps = 5 };

// This CTA's share of one GEMV op.
struct OpDesc {
    int lo, hi;  // rows [lo, hi)
    int shift;   // rows per chunk = 1 << shift
    int nch;     // chunks
    int K;       // row length in elements
    int win;     // chunks per window (a window is waited for, computed and released together)
};

// Byte offsets of the shared-memory regions (host-computed).
struct SmemLayout {
    int xs, scratch, resid, red, full, empty, flags, ops, layers, total;
};

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
    unsigned long long* t_part;  // split attention: per query head, ns partial states of D + 2 words
    int ns, bs, split_min;       // slots per KV group, positions per block, first split position + 1
    DecodeState* state;
    int steps;
    int slots;
    int slot_bytes;
    int inflight;  // chunks the producer keeps in flight at most (0: every free slot)
    int inflight_layers;  // the same during the layers' ops (the head streams with `inflight`)
    SmemLayout sm;
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

__device__ __forceinline__ void raise_abort(DecodeState* st, int code) { atomicCAS(&st->status, 0, code); }
__device__ __forceinline__ bool aborted(DecodeState* st) { return ld_relaxed_int(&st->status) != 0; }

// Clock cycles a wait spins before it also watches the abort flag (~10 us; a
// healthy exchange completes in about one).  Reading the one abort word on every
// polling round of every warp of every CTA queued a thousand requests per round
// on a single L2 line, in front of the exchange data that shares its slice.
constexpr long long kAbortWatchAfter = 20000;

// True when a wait that started at `start` should give up: past its spin limit,
// or past kAbortWatchAfter with another CTA having aborted the run.
__device__ __forceinline__ bool give_up(long long start, DecodeState* st) {
    const long long waited = clock64() - start;
    if (waited < kAbortWatchAfter) return false;
    return waited > s_spin || aborted(st);
}

// Argmax partial: total-order value (32) | 0x7FFFF - index (19) | epoch (13).
__device__ __forceinline__ unsigned long long arg_word(unsigned long long key, uint32_t epoch) {
    const uint32_t value = (uint32_t)(key >> 32);
    const uint32_t index = 0xffffffffu - (uint32_t)(key & 0xffffffffull);
    return ((unsigned long long)value << 32) | ((unsigned long long)((0x7FFFFu - index) & 0x7FFFFu) << 13) |
           (unsigned long long)(epoch & 0x1FFFu);
}

// Activation layout in shared memory for the GEMVs: element i of an n-vector is
// stored at xperm(i, n) so that the two 16-byte halves of every lane's 8-element
// slice sit in two arrays of consecutive slices, and each warp-wide 16-byte load
// of x reads 512 contiguous bytes (one conflict-free pass).
__device__ __forceinline__ int xperm(int i, int n) { return ((i & 4) ? (n >> 1) : 0) + ((i >> 3) << 2) + (i & 3); }

// Polls n tagged words until each carries `epoch`; values land in dst[0..n)
// (at xperm positions when `perm`).
// Every stale word of a thread is re-read in the same round, so a poll costs one
// L2 round trip per round rather than one per word.  Called by all compute
// threads; false on timeout or abort.
__device__ bool poll_vector(const unsigned long long* src, int n, uint32_t epoch, float* dst, DecodeState* st,
                            bool perm = false) {
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
            // re-read first: the abort flag's load then overlaps the round trip
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const int i = base + tid + j * kCompute;
                if ((uint32_t)(v[j] >> 32) != epoch) v[j] = ld_relaxed(src + i);
            }
            if (start == 0) {
                start = clock64();
            } else if (give_up(start, st)) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = base + tid + j * kCompute;
            if (i < n) dst[perm ? xperm(i, n) : i] = __uint_as_float((uint32_t)v[j]);
        }
    }
    if (!ok) raise_abort(st, kDeviceTimeoutEpilogue);
    return ok;
}

// Three segments polled in one round (one query head, the key and the value of its group).
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
            if (i < n0) {
                src[j] = s0 + i;
                dst[j] = d0 + i;
            } else if (i < n0 + n1) {
                src[j] = s1 + (i - n0);
                dst[j] = d1 + (i - n0);
            } else if (i < n) {
                src[j] = s2 + (i - n0 - n1);
                dst[j] = d2 + (i - n0 - n1);
            } else {
                src[j] = nullptr;
                dst[j] = nullptr;
            }
            v[j] = src[j] ? ld_relaxed(src[j]) : ((unsigned long long)epoch << 32);
        }
        long long start = 0;
        while (true) {
            bool stale = false;
#pragma unroll
            for (int j = 0; j < 4; ++j) stale |= (uint32_t)(v[j] >> 32) != epoch;
            if (!stale) break;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if ((uint32_t)(v[j] >> 32) != epoch) v[j] = ld_relaxed(src[j]);
            if (start == 0) {
                start = clock64();
            } else if (give_up(start, st)) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (dst[j]) *dst[j] = __uint_as_float((uint32_t)v[j]);
    }
    if (!ok) raise_abort(st, kDeviceTimeoutEpilogue);
    return ok;
}

// This CTA's rows of an op of n rows in units of `unit` rows, chunked for the ring.
__device__ OpDesc make_op(int n, int unit, int K, int c, int G, int slot_bytes, int slots) {
    OpDesc d;
    const int units = n / unit;
    d.lo = (int)(((long long)c * units) / G) * unit;
    d.hi = (int)(((long long)(c + 1) * units) / G) * unit;
    const int fit = slot_bytes / (2 * K);
    int shift = 0;
    while ((2 << shift) <= fit) ++shift;
    while ((1 << shift) < unit) ++shift;
    d.shift = shift;
    d.nch = (d.hi - d.lo + (1 << shift) - 1) >> shift;
    d.K = K;
    const int half = slots / 2 > 0 ? slots / 2 : 1;
    d.win = d.nch <= half ? (d.nch > 0 ? d.nch : 1) : half;
    return d;
}

__device__ __forceinline__ const __nv_bfloat16* op_weight(const PArgs& a, const FusedLayer& L, int op) {
    switch (op) {
    case kOpQkv: return L.wqkv;
    case kOpO: return L.wo;
    case kOpGu: return L.wgu;
    case kOpDown: return L.wd;
    default: return a.head;
    }
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

// Position of the next chunk in the ring: slot and the parity of its use.
struct Cursor {
    int slot = 0;
    uint32_t phase = 0;
    long long consumed = 0;  // chunks consumed so far
    __device__ __forceinline__ void at(int ahead, int slots, int* s, uint32_t* p) const {
        int t = slot + ahead;
        uint32_t q = phase;
        if (t >= slots) {
            t -= slots;
            q ^= 1u;
        }
        *s = t;
        *p = q;
    }
    __device__ __forceinline__ void advance(int n, int slots) {
        consumed += n;
        slot += n;
        if (slot >= slots) {
            slot -= slots;
            phase ^= 1u;
        }
    }
};

enum { kEpiStore = 0, kEpiResidual = 1, kEpiGated = 2, kEpiHead = 3 };

struct EpiCtx {
    unsigned long long* out;  // tagged destination (store, residual, gated)
    uint32_t epoch;
    float* resid;             // this CTA's residual rows (shared memory), residual epilogue
    int resid_lo;
    float* logits;            // head
    unsigned long long best;  // head, per lane
    bool bad;
    int act;
};

// Partial dot of one 16-byte chunk of bf16 weights with eight f32 values, with
// packed f32x2 FMAs (two multiply-adds per instruction):
// each 32-bit word of w holds two bf16 weights, widened to an f32 pair by a shift
// and a mask; s0 accumulates words 0 and 2, s1 words 1 and 3, two lanes each.
__device__ __forceinline__ unsigned long long pack_f32x2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ unsigned long long widen_bf16x2(uint32_t u) {
    unsigned long long r;
    asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r)
        : "r"(u));
    return r;
}
__device__ __forceinline__ void fma_f32x2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float sum_f32x2(unsigned long long v) {
    return __uint_as_float((uint32_t)v) + __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ void dot8_x2(uint4 w, float4 x0, float4 x1, unsigned long long& s0,
                                        unsigned long long& s1) {
    fma_f32x2(s0, widen_bf16x2(w.x), pack_f32x2(x0.x, x0.y));
    fma_f32x2(s1, widen_bf16x2(w.y), pack_f32x2(x0.z, x0.w));
    fma_f32x2(s0, widen_bf16x2(w.z), pack_f32x2(x1.x, x1.y));
    fma_f32x2(s1, widen_bf16x2(w.w), pack_f32x2(x1.z, x1.w));
}

// Sums CNT per-lane partials across the warp.  Each halving round exchanges half
// of the values with the lane OFF apart, so after log2(CNT) rounds every lane
// carries one value; the remaining rounds complete the sum.  Lane l ends with
// the total of value l / (32 / CNT).
template <int CNT, int OFF>
struct RowReduce {
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
                RowReduce<half, OFF / 2>::run(v, lane);
            } else {
                v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
                RowReduce<1, OFF / 2>::run(v, lane);
            }
        }
    }
};

// x of one GEMV in registers, lane-interleaved as the weight loads use it:
// lane l holds elements [8 (l + 32 j), 8 (l + 32 j) + 8) for j < KCH.
template <int KCH>
struct XRegs {
    float4 v[2 * (KCH > 0 ? KCH : 1)];
    // perm: xs holds x at xperm positions (K = 256 KCH); otherwise in natural order.
    __device__ __forceinline__ void load(const float* xs, int lane, bool perm) {
        const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            const int c = lane + 32 * j;
            v[2 * j] = perm ? x4[c] : x4[2 * c];
            v[2 * j + 1] = perm ? x4[KCH * 32 + c] : x4[2 * c + 1];
        }
    }
};

// RMSNorm gains in the XRegs layout, fetched before the activations are waited for.
template <int KCH>
// Two 16-byte loads per 8-element slice (gains are 16-byte aligned library
// allocations): scalar loads at a 32-byte lane stride touched 32 sectors per
// instruction and delayed the residual polls behind them.
struct GainX {
    float g[8 * (KCH > 0 ? KCH : 1)];
    __device__ __forceinline__ void load(const float* gain, int lane) {
        const float4* g4 = reinterpret_cast<const float4*>(gain);
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            const float4 a = gain ? __ldg(g4 + 2 * (lane + 32 * j)) : make_float4(1.f, 1.f, 1.f, 1.f);
            const float4 b = gain ? __ldg(g4 + 2 * (lane + 32 * j) + 1) : make_float4(1.f, 1.f, 1.f, 1.f);
            g[8 * j + 0] = a.x;
            g[8 * j + 1] = a.y;
            g[8 * j + 2] = a.z;
            g[8 * j + 3] = a.w;
            g[8 * j + 4] = b.x;
            g[8 * j + 5] = b.y;
            g[8 * j + 6] = b.z;
            g[8 * j + 7] = b.w;
        }
    }
};

// RMSNorm (kernels/ops.py:31-45) split for latency: x * gain feeds the dot
// products at once, and rsqrt(mean(x^2) + eps) (four independent chains, then one
// warp reduction) multiplies each row total in the epilogue, off the critical path.
template <int KCH>
__device__ __forceinline__ float gain_regs_rms(XRegs<KCH>& x, const GainX<KCH>& g, int n, float eps) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int j = 0; j < 2 * KCH; ++j) {
        s0 = fmaf(x.v[j].x, x.v[j].x, s0);
        s1 = fmaf(x.v[j].y, x.v[j].y, s1);
        s2 = fmaf(x.v[j].z, x.v[j].z, s2);
        s3 = fmaf(x.v[j].w, x.v[j].w, s3);
        x.v[j].x *= g.g[4 * j + 0];
        x.v[j].y *= g.g[4 * j + 1];
        x.v[j].z *= g.g[4 * j + 2];
        x.v[j].w *= g.g[4 * j + 3];
    }
    const float ss = warp_allsum((s0 + s1) + (s2 + s3));
    return rsqrtf(ss / (float)n + eps);
}

// Waits for the chunks of the window starting at the cursor: one pass of
// independent tests, then bounded waits only if some chunk has not landed.
__device__ __forceinline__ bool window_landed(const Ring& ring, const Cursor& cur, int wn) {
    bool all = true;
    for (int ch = 0; ch < wn; ++ch) {
        int s;
        uint32_t p;
        cur.at(ch, ring.slots, &s, &p);
        all &= mbar_try_wait(smem_u32(&ring.full[s]), p);
    }
    if (!all) {
        all = true;
        for (int ch = 0; ch < wn; ++ch) {
            int s;
            uint32_t p;
            cur.at(ch, ring.slots, &s, &p);
            all &= mbar_wait_bounded(&ring.full[s], p);
        }
    }
    return __all_sync(0xffffffffu, all);
}

// The first window of an op, waited for ahead of the activations it multiplies.
__device__ __forceinline__ bool first_window_landed(const Ring& ring, const Cursor& cur, const OpDesc& op) {
    return op.nch == 0 || window_landed(ring, cur, min(op.win, op.nch));
}

// One GEMV op over this CTA's rows: consumes its chunks from the ring window by
// window and releases each window's slots when done.  Each warp takes NV <= NR rows
// per pass (NR, a power of two, is the width of the cross-lane reduction; NV < NR
// evens out a CTA's rows over its warps).  KCH > 0: K == 256 * KCH and x lives in
// registers (normalised there when `gain` is given); KCH == 0: any K % 8 == 0, x
// read from shared memory.
template <int EPI, int KCH, int NR, int NV = NR>
__device__ __forceinline__ bool run_gemv(const Ring& ring, Cursor& cur, const OpDesc& op, const float* bias,
                                         const float* xs, const GainX<KCH>* gain, float eps, EpiCtx& e,
                                         bool first_ready, bool perm) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = op.K;
    const uint32_t row_bytes = (uint32_t)K * 2u;
    const int mask = (1 << op.shift) - 1;
    XRegs<KCH> x;
    float inverse = 1.f;
    if (KCH > 0) {
        x.load(xs, lane, perm);
        if (gain) inverse = gain_regs_rms<KCH>(x, *gain, K, eps);
    }
    constexpr int kLanesPerRow = 32 / NR;
    const int my_row = lane / kLanesPerRow;  // row of the pass this lane ends up holding
    const bool owner = (lane % kLanesPerRow) == 0;
    bool ok = true;
    for (int w0 = 0; w0 < op.nch && ok; w0 += op.win) {
        const int wn = min(op.win, op.nch - w0);
        const int rs = op.lo + (w0 << op.shift);
        const int re = min(op.hi, op.lo + ((w0 + wn) << op.shift));
        // Wait once for every chunk of the window (the first one usually before the
        // activations were polled).
        LSX_WINDOW_MARK(0);
        ok = (w0 == 0 && first_ready) || window_landed(ring, cur, wn);
        LSX_WINDOW_MARK(1);
        if (ok) {
            for (int r0 = rs + warp * NV; r0 < re; r0 += kWarps * NV) {
                const uint8_t* rp[NV];
#pragma unroll
                for (int i = 0; i < NV; ++i) {
                    const int local = min(r0 + i, re - 1) - rs;  // the window starts on a chunk boundary
                    int s;
                    uint32_t p;
                    cur.at(local >> op.shift, ring.slots, &s, &p);
                    rp[i] = ring.base + (size_t)s * ring.slot_bytes + (uint32_t)(local & mask) * row_bytes;
                }
                float acc[NR];
                {
                    unsigned long long a0[NR], a1[NR];
#pragma unroll
                    for (int i = 0; i < NR; ++i) a0[i] = a1[i] = 0ull;
                    if (KCH > 0) {
#pragma unroll
                        for (int j = 0; j < KCH; ++j) {
                            uint4 w[NV];
#pragma unroll
                            for (int i = 0; i < NV; ++i) w[i] = reinterpret_cast<const uint4*>(rp[i])[lane + 32 * j];
#pragma unroll
                            for (int i = 0; i < NV; ++i) dot8_x2(w[i], x.v[2 * j], x.v[2 * j + 1], a0[i], a1[i]);
                        }
                    } else {
                        const float4* x4 = reinterpret_cast<const float4*>(xs);
                        for (int cc = lane; cc < (K >> 3); cc += 32) {
                            const float4 x0 = perm ? x4[cc] : x4[2 * cc];
                            const float4 x1 = perm ? x4[(K >> 3) + cc] : x4[2 * cc + 1];
#pragma unroll
                            for (int i = 0; i < NV; ++i)
                                dot8_x2(reinterpret_cast<const uint4*>(rp[i])[cc], x0, x1, a0[i], a1[i]);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < NR; ++i) acc[i] = sum_f32x2(a0[i]) + sum_f32x2(a1[i]);
                }
                RowReduce<NR, 16>::run(acc, lane);
                float d = gain ? acc[0] * inverse : acc[0];
                const int r = r0 + my_row;
                const bool valid = owner && my_row < NV && r < re;
                if (EPI == kEpiGated) {
                    // rows come in (gate, up) pairs; the up total sits kLanesPerRow lanes higher
                    const float u = __shfl_down_sync(0xffffffffu, d, kLanesPerRow);
                    if (valid && (my_row & 1) == 0) {
                        float g = d, uu = u;
                        if (bias) {
                            g += bias[r];
                            uu += bias[r + 1];
                        }
                        st_relaxed(e.out + (r >> 1), tagged(e.epoch, activation(g, e.act) * uu));
                    }
                } else if (valid) {
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
            }
        }
        LSX_WINDOW_MARK(4);
        ok = compute_and(ok);
        LSX_WINDOW_MARK(2);
        if (tid == 0)
            for (int ch = 0; ch < wn; ++ch) {
                int s;
                uint32_t p;
                cur.at(ch, ring.slots, &s, &p);
                mbar_arrive(&ring.empty[s]);
            }
        cur.advance(wn, ring.slots);
    }
    return ok;
}

// Attention of query head h at `pos` (kernels/ops.py:69-101 after QK-norm and
// RoPE): polls the head's q and its group's k and v, normalises and rotates them
// in registers, appends k/v to the f32 cache (first head of the group), attends
// over positions 0..pos and publishes the head's output.  Warp w takes positions
// w, w + kWarps, ... in batches of PB; partial softmax states merge in shared memory.
template <int DPL, int PB>
__device__ __forceinline__ bool attention_head(const PArgs& a, const FusedLayer& L, int h, int pos, uint32_t e_qkv,
                                               uint32_t e_attn, float* sm) {
    constexpr int D = DPL * 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ratio = a.QH / a.KVH, g = h / ratio;
    const int qw = a.QH * D, kw = a.KVH * D;
    float* raw = sm;                        // 3 D: q, k, v
    float* merge = raw + 3 * D;             // kWarps * (D + 2)
    float* rot = merge + kWarps * (D + 2);  // general RoPE path: q, k and the table row (3 D)
    const bool fast_rope = a.rotary == D && !a.interleaved;
    // The cached positions 0..pos-1 do not depend on this step: load this warp's
    // first batch before waiting for q, k and v.
    const float* kbase = L.keys + (size_t)g * D;
    const float* vbase = L.values + (size_t)g * D;
    float kv[PB][DPL], vv[PB][DPL];
#pragma unroll
    for (int b = 0; b < PB; ++b) {
        const int t = warp + kWarps * b;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            kv[b][j] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * j) : 0.f;
            vv[b][j] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * j) : 0.f;
        }
    }
    float qg[DPL], kg[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        qg[j] = L.q_gain ? __ldg(L.q_gain + lane + 32 * j) : 1.f;
        kg[j] = L.k_gain ? __ldg(L.k_gain + lane + 32 * j) : 1.f;
    }
    const int half = a.rotary / 2;
    float2 cs[DPL / 2 > 0 ? DPL / 2 : 1];
    if (fast_rope) {
#pragma unroll
        for (int j = 0; j < DPL / 2; ++j) cs[j] = a.rope[(size_t)pos * half + lane + 32 * j];
    }
    bool ok = poll_segments(a.t_qkv + (size_t)h * D, D, raw, a.t_qkv + qw + (size_t)g * D, D, raw + D,
                            a.t_qkv + qw + kw + (size_t)g * D, D, raw + 2 * D, e_qkv, a.state);
    if (!compute_and(ok)) return false;
    float q[DPL], k[DPL], v[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        q[j] = raw[lane + 32 * j];
        k[j] = raw[D + lane + 32 * j];
        v[j] = raw[2 * D + lane + 32 * j];
    }
    // Qwen3 q_norm / k_norm per head (kernels/ops.py:31-45 over head_dim)
    if (L.q_gain) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss = fmaf(q[j], q[j], ss);
        const float inverse = rsqrtf(warp_allsum(ss) / (float)D + a.qk_eps);
#pragma unroll
        for (int j = 0; j < DPL; ++j) q[j] = q[j] * inverse * qg[j];
    }
    if (L.k_gain) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss = fmaf(k[j], k[j], ss);
        const float inverse = rsqrtf(warp_allsum(ss) / (float)D + a.qk_eps);
#pragma unroll
        for (int j = 0; j < DPL; ++j) k[j] = k[j] * inverse * kg[j];
    }
    // RoPE (kernels/ops.py:48-66).  Full-width rotate-half pairs d with d + D/2,
    // i.e. register j with register j + DPL/2 of the same lane.
    if (fast_rope) {
#pragma unroll
        for (int j = 0; j < DPL / 2; ++j) {
            const float q1 = q[j], q2 = q[j + DPL / 2], k1 = k[j], k2 = k[j + DPL / 2];
            q[j] = q1 * cs[j].x + -1.f * q2 * cs[j].y;
            q[j + DPL / 2] = q2 * cs[j].x + 1.f * q1 * cs[j].y;
            k[j] = k1 * cs[j].x + -1.f * k2 * cs[j].y;
            k[j + DPL / 2] = k2 * cs[j].x + 1.f * k1 * cs[j].y;
        }
    } else if (a.rotary > 0) {
        float* qn = rot;
        float* kn = rot + D;
        float2* cs_s = reinterpret_cast<float2*>(rot + 2 * D);
        if (warp == 0) {
#pragma unroll
            for (int j = 0; j < DPL; ++j) {
                qn[lane + 32 * j] = q[j];
                kn[lane + 32 * j] = k[j];
            }
        }
        for (int i = tid; i < half; i += kCompute) cs_s[i] = a.rope[(size_t)pos * half + i];
        compute_sync();
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            const int local = lane + 32 * j;
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
                const float2 c2 = cs_s[pair];
                q[j] = qn[local] * c2.x + sign * qn[other] * c2.y;
                k[j] = kn[local] * c2.x + sign * kn[other] * c2.y;
            }
        }
    }
    if (h % ratio == 0 && warp == 0) {  // kernels/ops.py:69-73: append this position's k, v
        float* kd = L.keys + (size_t)pos * kw + (size_t)g * D;
        float* vd = L.values + (size_t)pos * kw + (size_t)g * D;
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
            kd[lane + 32 * j] = k[j];
            vd[lane + 32 * j] = v[j];
        }
    }
    // Online softmax over this warp's positions, a batch of PB at a time
    // (kernels/ops.py:88-99): the batch's scores are reduced together.
    constexpr int kLanesPerPos = 32 / PB;
    const int my_b = lane / kLanesPerPos;
    float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
    for (int i0 = 0; warp + kWarps * i0 <= pos; i0 += PB) {
        if (i0 > 0) {
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                const int t = warp + kWarps * (i0 + b);
#pragma unroll
                for (int j = 0; j < DPL; ++j) {
                    kv[b][j] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * j) : 0.f;
                    vv[b][j] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * j) : 0.f;
                }
            }
        }
        float sc[PB];
#pragma unroll
        for (int b = 0; b < PB; ++b) {
            const int t = warp + kWarps * (i0 + b);
            if (t == pos) {  // the current position, from registers
#pragma unroll
                for (int j = 0; j < DPL; ++j) {
                    kv[b][j] = k[j];
                    vv[b][j] = v[j];
                }
            }
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) s = fmaf(q[j], kv[b][j], s);
            sc[b] = s;
        }
        RowReduce<PB, 16>::run(sc, lane);
        const bool valid = warp + kWarps * (i0 + my_b) <= pos;
        const float s = valid ? sc[0] * a.scale : -INFINITY;
        // the kLanesPerPos lanes of a position hold the same score, so the maximum and
        // the sum over positions need only the rounds across position groups (the sum
        // adds the same values in the same order as a full-warp sum of one lane each)
        float mb = s;
#pragma unroll
        for (int o = 16; o >= kLanesPerPos; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        const float mn = fmaxf(m, mb);
        const float carry = expf(m - mn);
        const float p = valid ? expf(s - mn) : 0.f;
        float psum = p;
#pragma unroll
        for (int o = 16; o >= kLanesPerPos; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l = l * carry + psum;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] *= carry;
#pragma unroll
        for (int b = 0; b < PB; ++b) {
            const float pb = __shfl_sync(0xffffffffu, p, b * kLanesPerPos);
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[j] = fmaf(pb, vv[b][j], acc[j]);
        }
        m = mn;
    }
    const int stride = D + 2;
    float* slot = merge + (size_t)warp * stride;
    if (lane == 0) {
        slot[0] = m;
        slot[1] = l;
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) slot[2 + lane + 32 * j] = acc[j];
    compute_sync();
    for (int d = tid; d < D; d += kCompute) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, merge[w * stride]);
        float Lsum = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float* sl = merge + (size_t)w * stride;
            if (sl[0] == -INFINITY) continue;
            const float ex = expf(sl[0] - M);
            Lsum = fmaf(sl[1], ex, Lsum);
            O = fmaf(sl[2 + d], ex, O);
        }
        st_relaxed(a.t_attn + (size_t)h * D + d, tagged(e_attn, O / Lsum));
    }
    // The merge area is rewritten only after later block-wide barriers.
    return true;
}

// ---- long contexts: attention split over the CTAs ---------------------------
// Past `split_min` positions one query head per CTA leaves most SMs idle while
// the K/V reads grow with the context.  Instead the CTAs of slot s of KV group g
// (CTA g + KVH s, s < ns) each own the position blocks b = s, s + ns, s + 2 ns ...
// (BS positions per block) of group g for the whole generation.  The CTA reads
// each cached K/V row once for all R query heads of the group, and publishes per
// head a partial softmax state (running max m, sum l, unnormalised output o[D]).
// CTA h then merges the ns partials of query head h and publishes its attention
// output (kernels/ops.py:88-101 evaluated in another order: the same exp/max
// rescaling, summed over blocks).  The owner of the current position's block
// appends its k and v to the cache, so each cached position is written and later
// read by one CTA.

// Position of local index j of slot s.
__device__ __forceinline__ int split_position(int j, int s, int ns, int bs) {
    return ((j / bs) * ns + s) * bs + (j % bs);
}

// Number of local positions of slot s at or before `pos`.
__device__ __forceinline__ int split_count(int pos, int s, int ns, int bs) {
    int n = 0;
    for (int b = s; b * bs <= pos; b += ns) n += min(bs, pos + 1 - b * bs);
    return n;
}

template <int DPL, int PB, int R>
__device__ __forceinline__ bool attention_part(const PArgs& a, const FusedLayer& L, int g, int s, int pos,
                                               uint32_t e_qkv, uint32_t e_attn, float* sm) {
    constexpr int D = DPL * 32;
    constexpr int CNT = R * PB;          // scores reduced together per batch
    constexpr int LPV = 32 / CNT;        // lanes holding each reduced score
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qw = a.QH * D, kw = a.KVH * D;
    const int ns = a.ns, bs = a.bs;
    float* raw = sm;                 // (R + 2) D: the group's q heads, k, v
    float* merge = raw + (R + 2) * D;  // kWarps R (D + 2)
    const float* kbase = L.keys + (size_t)g * D;
    const float* vbase = L.values + (size_t)g * D;
    const int n = split_count(pos, s, ns, bs);
    // the first batch of cached positions does not depend on this step
    float kv[PB][DPL], vv[PB][DPL];
#pragma unroll
    for (int b = 0; b < PB; ++b) {
        const int j = warp + kWarps * b;
        const int t = j < n ? split_position(j, s, ns, bs) : pos;
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
            kv[b][d] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * d) : 0.f;
            vv[b][d] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * d) : 0.f;
        }
    }
    float qg[DPL], kg[DPL];
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
        qg[d] = L.q_gain ? __ldg(L.q_gain + lane + 32 * d) : 1.f;
        kg[d] = L.k_gain ? __ldg(L.k_gain + lane + 32 * d) : 1.f;
    }
    const int half = a.rotary / 2;
    float2 cs[DPL / 2 > 0 ? DPL / 2 : 1];
#pragma unroll
    for (int d = 0; d < DPL / 2; ++d) cs[d] = a.rope[(size_t)pos * half + lane + 32 * d];
    bool ok = poll_segments(a.t_qkv + (size_t)g * R * D, R * D, raw, a.t_qkv + qw + (size_t)g * D, D, raw + R * D,
                            a.t_qkv + qw + kw + (size_t)g * D, D, raw + (R + 1) * D, e_qkv, a.state);
    if (!compute_and(ok)) return false;
    float q[R][DPL], k[DPL], v[DPL];
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
#pragma unroll
        for (int i = 0; i < R; ++i) q[i][d] = raw[i * D + lane + 32 * d];
        k[d] = raw[R * D + lane + 32 * d];
        v[d] = raw[(R + 1) * D + lane + 32 * d];
    }
    // QK-norm (kernels/ops.py:31-45 over head_dim) and rotate-half RoPE in registers
    if (L.q_gain) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
            float ss = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; ++d) ss = fmaf(q[i][d], q[i][d], ss);
            const float inverse = rsqrtf(warp_allsum(ss) / (float)D + a.qk_eps);
#pragma unroll
            for (int d = 0; d < DPL; ++d) q[i][d] = q[i][d] * inverse * qg[d];
        }
    }
    if (L.k_gain) {
        float ss = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) ss = fmaf(k[d], k[d], ss);
        const float inverse = rsqrtf(warp_allsum(ss) / (float)D + a.qk_eps);
#pragma unroll
        for (int d = 0; d < DPL; ++d) k[d] = k[d] * inverse * kg[d];
    }
#pragma unroll
    for (int d = 0; d < DPL / 2; ++d) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const float q1 = q[i][d], q2 = q[i][d + DPL / 2];
            q[i][d] = q1 * cs[d].x + -1.f * q2 * cs[d].y;
            q[i][d + DPL / 2] = q2 * cs[d].x + 1.f * q1 * cs[d].y;
        }
        const float k1 = k[d], k2 = k[d + DPL / 2];
        k[d] = k1 * cs[d].x + -1.f * k2 * cs[d].y;
        k[d + DPL / 2] = k2 * cs[d].x + 1.f * k1 * cs[d].y;
    }
    if (((pos / bs) % ns) == s && warp == 0) {  // kernels/ops.py:69-73: append this position's k, v
        float* kd = L.keys + (size_t)pos * kw + (size_t)g * D;
        float* vd = L.values + (size_t)pos * kw + (size_t)g * D;
#pragma unroll
        for (int d = 0; d < DPL; ++d) {
            kd[lane + 32 * d] = k[d];
            vd[lane + 32 * d] = v[d];
        }
    }
    // Online softmax per head over this warp's positions, PB at a time.  After the
    // reduction lane l holds score (l / LPV): head (l / LPV) / PB, position (l / LPV) % PB.
    const int vi = lane / LPV, my_head = vi / PB, my_b = vi % PB;
    float m[R], l[R], acc[R][DPL];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[i][d] = 0.f;
    }
    for (int i0 = 0; warp + kWarps * i0 < n; i0 += PB) {
        if (i0 > 0) {
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                const int j = warp + kWarps * (i0 + b);
                const int t = j < n ? split_position(j, s, ns, bs) : pos;
#pragma unroll
                for (int d = 0; d < DPL; ++d) {
                    kv[b][d] = t < pos ? __ldcg(kbase + (size_t)t * kw + lane + 32 * d) : 0.f;
                    vv[b][d] = t < pos ? __ldcg(vbase + (size_t)t * kw + lane + 32 * d) : 0.f;
                }
            }
        }
        float sc[CNT];
#pragma unroll
        for (int b = 0; b < PB; ++b) {
            const int j = warp + kWarps * (i0 + b);
            if (j < n && split_position(j, s, ns, bs) == pos) {  // the current position, from registers
#pragma unroll
                for (int d = 0; d < DPL; ++d) {
                    kv[b][d] = k[d];
                    vv[b][d] = v[d];
                }
            }
#pragma unroll
            for (int i = 0; i < R; ++i) {
                float x = 0.f;
#pragma unroll
                for (int d = 0; d < DPL; ++d) x = fmaf(q[i][d], kv[b][d], x);
                sc[i * PB + b] = x;
            }
        }
        RowReduce<CNT, 16>::run(sc, lane);
        const bool valid = warp + kWarps * (i0 + my_b) < n;
        const float sv = valid ? sc[0] * a.scale : -INFINITY;
        // per-head maximum and sum over the batch: xor within the head's lane segment
        float mb = sv;
#pragma unroll
        for (int o = LPV; o < PB * LPV; o <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        float mn[R], carry[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            mn[i] = fmaxf(m[i], __shfl_sync(0xffffffffu, mb, i * PB * LPV));
            carry[i] = expf(m[i] - mn[i]);
        }
        float mine = mn[0];
#pragma unroll
        for (int i = 1; i < R; ++i) mine = my_head == i ? mn[i] : mine;
        const float p = valid ? expf(sv - mine) : 0.f;
        float ps = p;
#pragma unroll
        for (int o = LPV; o < PB * LPV; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            l[i] = l[i] * carry[i] + __shfl_sync(0xffffffffu, ps, i * PB * LPV);
#pragma unroll
            for (int d = 0; d < DPL; ++d) acc[i][d] *= carry[i];
#pragma unroll
            for (int b = 0; b < PB; ++b) {
                const float pb = __shfl_sync(0xffffffffu, p, (i * PB + b) * LPV);
#pragma unroll
                for (int d = 0; d < DPL; ++d) acc[i][d] = fmaf(pb, vv[b][d], acc[i][d]);
            }
            m[i] = mn[i];
        }
    }
    // merge the warps' states per head, then publish this slot's partial per head
    const int stride = D + 2;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        float* slot = merge + (size_t)(warp * R + i) * stride;
        if (lane == 0) {
            slot[0] = m[i];
            slot[1] = l[i];
        }
#pragma unroll
        for (int d = 0; d < DPL; ++d) slot[2 + lane + 32 * d] = acc[i][d];
    }
    compute_sync();
    for (int idx = tid; idx < R * stride; idx += kCompute) {
        const int i = idx / stride, e = idx % stride;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, merge[(w * R + i) * stride]);
        float val;
        if (e == 0) {
            val = M;
        } else {
            val = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float* sl = merge + (size_t)(w * R + i) * stride;
                if (sl[0] == -INFINITY) continue;
                val = fmaf(sl[e], expf(sl[0] - M), val);
            }
        }
        const int h = g * R + i;
        st_relaxed(a.t_part + ((size_t)h * ns + s) * stride + e, tagged(e_attn, val));
    }
    // The merge area is rewritten only after later block-wide barriers.
    return true;
}

// Merges the ns partial states of query head h and publishes its attention output.
template <int DPL>
__device__ __forceinline__ bool attention_merge(const PArgs& a, int h, uint32_t e_attn, float* sm) {
    constexpr int D = DPL * 32;
    const int tid = threadIdx.x;
    const int ns = a.ns, stride = D + 2;
    bool ok = poll_vector(a.t_part + (size_t)h * ns * stride, ns * stride, e_attn, sm, a.state);
    if (!compute_and(ok)) return false;
    for (int d = tid; d < D; d += kCompute) {
        float M = -INFINITY;
        for (int s = 0; s < ns; ++s) M = fmaxf(M, sm[s * stride]);
        float Lsum = 0.f, O = 0.f;
        for (int s = 0; s < ns; ++s) {
            const float* sl = sm + (size_t)s * stride;
            if (sl[0] == -INFINITY) continue;
            const float ex = expf(sl[0] - M);
            Lsum = fmaf(sl[1], ex, Lsum);
            O = fmaf(sl[2 + d], ex, O);
        }
        st_relaxed(a.t_attn + (size_t)h * D + d, tagged(e_attn, O / Lsum));
    }
    return true;
}

template <int DPL>
__device__ bool attention_split(const PArgs& a, const FusedLayer& L, int c, int pos, uint32_t e_qkv,
                                uint32_t e_attn, float* sm) {
    bool ok = true;
    if (c < a.KVH * a.ns) {
        const int g = c % a.KVH, s = c / a.KVH;
        // the host enables the split only for these ratios (head_dim 256: up to 2)
        const int ratio = a.QH / a.KVH;
        if (ratio == 1) ok = attention_part<DPL, 8, 1>(a, L, g, s, pos, e_qkv, e_attn, sm);
        else if (ratio == 2) ok = attention_part<DPL, 8, 2>(a, L, g, s, pos, e_qkv, e_attn, sm);
        if constexpr (DPL < 8) {
            if (ratio == 4) ok = attention_part<DPL, 8, 4>(a, L, g, s, pos, e_qkv, e_attn, sm);
            else if (ratio == 8) ok = attention_part<DPL, 4, 8>(a, L, g, s, pos, e_qkv, e_attn, sm);
        }
        compute_sync();  // the part's scratch is read before the merge reuses it
    }
    if (ok && c < a.QH) ok = attention_merge<DPL>(a, c, e_attn, sm);
    return ok;
}

// Norm gains of one width in a strided layout (i = tid + j * kCompute), for the
// shared-memory RMSNorm used by the generic widths and the final norm.
constexpr int kGainRegs = 24;  // widths up to 24 * kCompute
struct GainRegs {
    float g[kGainRegs];
    __device__ __forceinline__ void load(const float* gain, int n) {
#pragma unroll
        for (int j = 0; j < kGainRegs; ++j) {
            const int i = threadIdx.x + j * kCompute;
            g[j] = i < n ? (gain ? __ldg(gain + i) : 1.f) : 0.f;
        }
    }
};

// RMSNorm of xs in place (kernels/ops.py:31-45): x * rsqrt(mean(x^2) + eps) * gain.
__device__ void rms_norm_inplace(float* xs, int n, const GainRegs& gain, float eps, float* red, bool perm = false) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kGainRegs; ++j) {
        const int i = threadIdx.x + j * kCompute;
        if (i < n) {
            const float x = xs[perm ? xperm(i, n) : i];
            ss = fmaf(x, x, ss);
        }
    }
    ss = compute_allsum(ss, red);
    const float inverse = rsqrtf(ss / (float)n + eps);
#pragma unroll
    for (int j = 0; j < kGainRegs; ++j) {
        const int i = threadIdx.x + j * kCompute;
        if (i < n) {
            const int k = perm ? xperm(i, n) : i;
            xs[k] = xs[k] * inverse * gain.g[j];
        }
    }
    compute_sync();
}

// Rows per warp pass for a register-resident x of KCH chunks (0: x in shared memory).
constexpr int rows_for(int kch) { return kch == 0 ? 2 : (kch <= 4 ? 4 : (kch <= 8 ? 2 : 1)); }

// KH, KQ, KI: 16-byte chunks per lane of x for the hidden, query and
// intermediate widths (0: x stays in shared memory).  DPL: head_dim / 32.
template <int KH, int KQ, int KI, int DPL>
__global__ void __launch_bounds__(kThreads, 1) persistent_decode_kernel(const PArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int NRH = rows_for(KH);               // qkv and head
    // gate/up: whole (gate, up) pairs; at H = 1024 a CTA holds 40-42 rows, six per warp
    constexpr int NRG = KH > 0 && KH <= 4 ? 8 : 2;
    constexpr int NVG = KH > 0 && KH <= 4 ? 6 : 2;
    // o and down own ~7 rows per CTA at hidden 1024: one row per warp (four rows
    // per warp, x read twice instead of seven times, measured 1.8x slower rows)
    constexpr int NRQ = KQ > 4 ? 1 : rows_for(KQ);  // o
    constexpr int NRI = KI > 4 ? 1 : rows_for(KI);  // down
    constexpr int PB = DPL >= 8 ? 4 : 8;            // attention positions per warp batch
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    Ring ring;
    ring.base = smem;
    ring.slots = a.slots;
    ring.slot_bytes = a.slot_bytes;
    float* xs = reinterpret_cast<float*>(smem + a.sm.xs);
    float* scratch = reinterpret_cast<float*>(smem + a.sm.scratch);
    float* resid = reinterpret_cast<float*>(smem + a.sm.resid);
    float* red = reinterpret_cast<float*>(smem + a.sm.red);
    ring.full = reinterpret_cast<uint64_t*>(smem + a.sm.full);
    ring.empty = reinterpret_cast<uint64_t*>(smem + a.sm.empty);
    volatile int* s_stop = reinterpret_cast<volatile int*>(smem + a.sm.flags);
    long long* s_issued = reinterpret_cast<long long*>(smem + a.sm.flags + 8);
    OpDesc* ops = reinterpret_cast<OpDesc*>(smem + a.sm.ops);
    FusedLayer* layers = reinterpret_cast<FusedLayer*>(smem + a.sm.layers);
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
        s_spin = a.state->spin_limit > 0 ? a.state->spin_limit : kSpin;
        const int qkv_rows = (a.QH + 2 * a.KVH) * a.D;
        ops[kOpQkv] = make_op(qkv_rows, 1, a.H, c, G, a.slot_bytes, a.slots);
        ops[kOpO] = make_op(a.H, 1, a.QH * a.D, c, G, a.slot_bytes, a.slots);
        ops[kOpGu] = make_op(2 * a.I, 2, a.H, c, G, a.slot_bytes, a.slots);
        ops[kOpDown] = make_op(a.H, 1, a.I, c, G, a.slot_bytes, a.slots);
        ops[kOpHead] = make_op(a.V, 1, a.H, c, G, a.slot_bytes, a.slots);
        fence_barrier_init();
    }
    __syncthreads();

    const int P = st->prompt_length, maximum = st->maximum, mode = st->mode;
    const int first_frame = P - 1 - st->frame_back;  // step of the first recorded frame
    const int pos0 = st->position;
    const uint32_t base = st->epoch;
    const int hold_cta = st->hold_cta - 1, hold_step = st->hold_step;
    // per-generation constants, read once: a global read on every step would sit on
    // the step's critical path (the head phase and the end-of-step bookkeeping)
    const int rot_kind = st->rot_kind, n_stop = st->n_stop;
    const uint32_t emb_row_bytes = (uint32_t)a.H * (a.emb_kind == LSX_F32 ? 4u : 2u);
    const bool emb_prefetch = emb_row_bytes % 16 == 0 && (uintptr_t)a.embedding % 16 == 0;
    const uint32_t per_step = 5u * (uint32_t)a.L + 1u;

    if (warp == kWarps) {  // ---------------------------------- producer warp
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            int slot = 0;
            uint32_t phase = 0;
            bool wrapped = false, go = true;
            long long issued = 0;
            // the oldest chunk that may still be in flight
            int lslot = 0;
            uint32_t lphase = 0;
            long long landed = 0;
            for (int step = 0; step < a.steps && go; ++step) {
                for (int oi = 0; oi <= 4 * a.L && go; ++oi) {
                    const int op = oi < 4 * a.L ? (oi & 3) : kOpHead;
                    const OpDesc d = ops[op];
                    const __nv_bfloat16* w = op_weight(a, layers[oi < 4 * a.L ? oi >> 2 : 0], op);
                    for (int ch = 0; ch < d.nch; ++ch) {
                        if (wrapped) {
                            // wait until the consumers released this slot's previous chunk
                            const uint32_t addr = smem_u32(&ring.empty[slot]);
                            long long start = 0;
                            while (!mbar_try_wait(addr, phase ^ 1u)) {
                                if (*s_stop) {
                                    go = false;
                                    break;
                                }
                                if (start == 0) {
                                    start = clock64();
                                } else if (clock64() - start > s_spin) {
                                    raise_abort(st, kDeviceTimeoutWeights);
                                    go = false;
                                    break;
                                }
                            }
                            if (!go) break;
                        }
                        // bound the bytes in flight per SM: a deep queue of bulk copies
                        // delays the small exchange loads behind it
                        const int cap = oi < 4 * a.L ? a.inflight_layers : a.inflight;
                        while (cap > 0 && issued - landed >= cap && go) {
                            if (!mbar_wait_bounded(&ring.full[lslot], lphase)) {
                                raise_abort(st, kDeviceTimeoutWeights);
                                go = false;
                                break;
                            }
                            ++landed;
                            if (++lslot == a.slots) {
                                lslot = 0;
                                lphase ^= 1u;
                            }
                        }
                        if (!go) break;
                        const int r0 = d.lo + (ch << d.shift);
                        const int nr = min(1 << d.shift, d.hi - r0);
                        const uint32_t bytes = (uint32_t)nr * (uint32_t)d.K * 2u;
                        mbar_expect_tx(&ring.full[slot], bytes);
                        bulk_load_hint(ring.base + (size_t)slot * a.slot_bytes, w + (size_t)r0 * d.K, bytes,
                                       &ring.full[slot], policy);
                        ++issued;
                        if (++slot == a.slots) {
                            slot = 0;
                            phase ^= 1u;
                            wrapped = true;
                        }
                    }
                }
            }
            *s_issued = issued;
        }
        __syncwarp();
    } else {  // ------------------------------------------------ compute warps
        Cursor cur;
        const OpDesc op_qkv = ops[kOpQkv], op_o = ops[kOpO], op_gu = ops[kOpGu], op_down = ops[kOpDown],
                     op_head = ops[kOpHead];
        const int r_lo = op_o.lo, r_hi = op_o.hi;  // residual rows owned by this CTA
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
                xs[xperm(i, a.H)] = v;
            }
            compute_sync();
            for (int i = tid; i < r_hi - r_lo; i += kCompute) resid[i] = xs[xperm(r_lo + i, a.H)];
            for (int layer = 0; layer < a.L && ok; ++layer) {
                const FusedLayer& Lr = layers[layer];
                const uint32_t e_qkv = e0 + 5u * layer + 1u, e_attn = e_qkv + 1u, e_o = e_qkv + 2u,
                               e_gu = e_qkv + 3u, e_down = e_qkv + 4u;
                EpiCtx e{};
                e.act = a.act;
                LSX_PHASE_MARK(0);
                // qkv: RMSNorm(residual) -> [q; k; v]
                {
                    GainX<KH> gx;
                    GainRegs gs;
                    if (KH > 0) gx.load(Lr.input_gain, lane);
                    else gs.load(Lr.input_gain, a.H);
                    // the op's first weight window before the exchange: the wait also
                    // delays the start of polling, which keeps the polls' L2 traffic down
                    // (polling first measured 9% slower)
                    const bool ready = first_window_landed(ring, cur, op_qkv);
                    if (layer > 0) ok = compute_and(poll_vector(a.t_resid, a.H, e_qkv - 1u, xs, st, true));
                    if (!ok) break;
                    LSX_PHASE_MARK(1);
                    if (KH == 0) rms_norm_inplace(xs, a.H, gs, a.eps, red, true);
                    e.out = a.t_qkv;
                    e.epoch = e_qkv;
                    ok = run_gemv<kEpiStore, KH, NRH>(ring, cur, op_qkv, Lr.bqkv, xs, KH > 0 ? &gx : nullptr,
                                                      a.eps, e, ready, true);
                    if (!ok) break;
                    LSX_PHASE_MARK(3);
                }
                // attention: one query head per CTA, or split over the CTAs at long contexts
                if (a.ns > 0 && pos + 1 >= a.split_min) {
                    ok = attention_split<DPL>(a, Lr, c, pos, e_qkv, e_attn, scratch);
                    if (!ok) break;
                } else if (c < a.QH) {
                    ok = attention_head<DPL, PB>(a, Lr, c, pos, e_qkv, e_attn, scratch);
                    if (!ok) break;
                }
                LSX_PHASE_MARK(4);
                // o: residual += Wo attn
                bool ready = first_window_landed(ring, cur, op_o);
                ok = compute_and(poll_vector(a.t_attn, a.QH * a.D, e_attn, xs, st, true));
                if (!ok) break;
                LSX_PHASE_MARK(5);
                e.out = a.t_resid;
                e.epoch = e_o;
                e.resid = resid;
                e.resid_lo = r_lo;
                ok = run_gemv<kEpiResidual, KQ, NRQ>(ring, cur, op_o, Lr.bo, xs, nullptr, a.eps, e, ready, true);
                if (!ok) break;
                LSX_PHASE_MARK(6);
                // gate/up: RMSNorm(residual) -> act(gate) * up
                {
                    GainX<KH> gx;
                    GainRegs gs;
                    if (KH > 0) gx.load(Lr.post_gain, lane);
                    else gs.load(Lr.post_gain, a.H);
                    ready = first_window_landed(ring, cur, op_gu);
                    ok = compute_and(poll_vector(a.t_resid, a.H, e_o, xs, st, true));
                    if (!ok) break;
                    LSX_PHASE_MARK(7);
                    if (KH == 0) rms_norm_inplace(xs, a.H, gs, a.eps, red, true);
                    e.out = a.t_feat;
                    e.epoch = e_gu;
                    ok = run_gemv<kEpiGated, KH, NRG, NVG>(ring, cur, op_gu, Lr.bgu, xs, KH > 0 ? &gx : nullptr,
                                                      a.eps, e, ready, true);
                    if (!ok) break;
                    LSX_PHASE_MARK(9);
                }
                // down: residual += Wd feature
                ready = first_window_landed(ring, cur, op_down);
                ok = compute_and(poll_vector(a.t_feat, a.I, e_gu, xs, st, true));
                if (!ok) break;
                LSX_PHASE_MARK(10);
                e.out = a.t_resid;
                e.epoch = e_down;
                ok = run_gemv<kEpiResidual, KI, NRI>(ring, cur, op_down, Lr.bd, xs, nullptr, a.eps, e, ready, true);
                LSX_PHASE_MARK(11);
            }
            if (!ok) break;
            // ---- head: final RMSNorm, optional edit, logits and first argmax
            const uint32_t e_last = e0 + 5u * (uint32_t)a.L, e_head = e_last + 1u;
            GainRegs fgain;
            fgain.load(a.final_gain, a.H);
            LSX_HEAD_MARK(0);
            ok = compute_and(poll_vector(a.t_resid, a.H, e_last, xs, st));
            if (!ok) break;
            LSX_HEAD_MARK(1);
            rms_norm_inplace(xs, a.H, fgain, a.eps, red);
            const int slot_idx = step - first_frame;
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
            if (rot_kind == 1) {  // kernels/ops.py:125-135
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
            } else if (rot_kind == 2) {  // DeviceRotation::apply Joint (src/model.rs:350-361)
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
            LSX_HEAD_MARK(2);
            ok = run_gemv<kEpiHead, KH, NRH>(ring, cur, op_head, a.head_bias, xs, nullptr, a.eps, e, false, false);
            if (!ok) break;
            LSX_HEAD_MARK(3);
            unsigned long long* rb = reinterpret_cast<unsigned long long*>(red);
            const unsigned long long wbest = warp_max_u64(e.best);
            if (lane == 0) rb[warp] = wbest;
            if (!compute_and(!e.bad) && tid == 0) atomicOr(&st->nonfinite, 1);
            if (tid == 0 && !(c == hold_cta && step == hold_step)) {
                unsigned long long b = 0ull;
                for (int i = 0; i < kWarps; ++i) b = rb[i] > b ? rb[i] : b;
                st_relaxed(a.t_arg + (size_t)c * kArgStride, arg_word(b, e_head));
                // the next step embeds the winner, which is one of the CTAs' local
                // bests: each CTA pulls its candidate's embedding row into L2 (the
                // head stream read it with evict-first, or not at all)
                const uint32_t cand = 0xffffffffu - (uint32_t)(b & 0xffffffffull);
                if (emb_prefetch && step + 1 < a.steps && step + 1 >= P && cand < (uint32_t)a.V)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                                     (const uint8_t*)a.embedding + (size_t)cand * emb_row_bytes),
                                 "r"(emb_row_bytes)
                                 : "memory");
            }
            // ---- gather the step's argmax from every CTA's partial
            unsigned long long* gathered = reinterpret_cast<unsigned long long*>(scratch);
            if (tid < G) {
                const unsigned long long* src = a.t_arg + (size_t)tid * kArgStride;
                unsigned long long v = ld_relaxed(src);
                long long start = 0;
                while ((uint32_t)(v & 0x1FFFull) != (e_head & 0x1FFFu)) {
                    v = ld_relaxed(src);
                    if (start == 0) start = clock64();
                    else if (give_up(start, st)) {
                        ok = false;
                        break;
                    }
                }
                gathered[tid] = v;
            }
            ok = compute_and(ok);
            LSX_HEAD_MARK(4);
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
                for (int i = 0; i < n_stop; ++i) stop |= st->stop[i] == arg;
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
    const int dpl = c.head_dim / 32;
    // Register-resident x needs compile-time widths; attention likewise.
    if (c.hidden == 1024 && qw == 2048 && c.intermediate == 3072 && dpl == 4)
        return persistent_decode_kernel<4, 8, 12, 4>;  // Qwen3-0.6B
    if (c.hidden == 2560 && dpl == 4) return persistent_decode_kernel<10, 0, 0, 4>;  // Qwen3-4B
    if (dpl == 4) return persistent_decode_kernel<0, 0, 0, 4>;
    if (dpl == 2) return persistent_decode_kernel<0, 0, 0, 2>;
    if (dpl == 8) return persistent_decode_kernel<0, 0, 0, 8>;
    return nullptr;
}

// Split attention: slots per KV group (0: never split), at most 32.  It needs the
// full-width rotate-half RoPE and a group ratio of 1, 2, 4 or 8 (1 or 2 at head_dim 256).
int split_slots(const FusedConfig& c, int grid) {
    const int ratio = c.kvheads > 0 ? c.qheads / c.kvheads : 0;
    const bool fast_rope = c.rotary == c.head_dim && !c.interleaved;
    const int max_ratio = c.head_dim >= 256 ? 2 : 8;
    if (!fast_rope || ratio * c.kvheads != c.qheads || ratio > max_ratio ||
        (ratio != 1 && ratio != 2 && ratio != 4 && ratio != 8))
        return 0;
    const int ns = std::min(grid / c.kvheads, 32);
    return ns >= 2 ? ns : 0;
}

int scratch_floats(const FusedConfig& c, int grid) {
    const int D = c.head_dim;
    int attention = 3 * D + kWarps * (D + 2) + 3 * D;
    const int ns = split_slots(c, grid);
    if (ns > 0) {
        const int ratio = c.qheads / c.kvheads;
        attention = std::max(attention, (ratio + 2) * D + kWarps * ratio * (D + 2));
        attention = std::max(attention, ns * (D + 2));
    }
    return (std::max(attention, 512 + 2 * 256) + 3) & ~3;
}

// Shared-memory layout for `slots` ring slots.
SmemLayout layout_for(const FusedConfig& c, int slots, int slot_bytes, int grid, size_t layers) {
    const int qw = c.qheads * c.head_dim;
    const int xmax = (std::max(std::max(c.hidden, qw), c.intermediate) + 3) & ~3;
    const int rmax = ((c.hidden + grid - 1) / grid + 1 + 3) & ~3;
    SmemLayout s{};
    size_t at = (size_t)slots * slot_bytes;
    s.xs = (int)at;
    at += (size_t)xmax * 4;
    s.scratch = (int)at;
    at += (size_t)scratch_floats(c, grid) * 4;
    s.resid = (int)at;
    at += (size_t)rmax * 4;
    s.red = (int)at;
    at += 64 * 4;
    s.full = (int)at;
    at += (size_t)slots * 8;
    s.empty = (int)at;
    at += (size_t)slots * 8;
    s.flags = (int)at;
    at += 16;
    s.ops = (int)at;
    at += (kOps * sizeof(OpDesc) + 15) & ~(size_t)15;
    s.layers = (int)at;
    at += layers * sizeof(FusedLayer);
    s.total = (int)at;
    return s;
}

int slot_bytes_for(const FusedConfig& c) {
    const int qw = c.qheads * c.head_dim;
    int slot_bytes = 16384;
    const int ks[4] = {c.hidden, qw, c.hidden, c.intermediate};
    const int units[4] = {1, 1, 2, 1};
    for (int i = 0; i < 4; ++i) slot_bytes = std::max(slot_bytes, units[i] * ks[i] * 2);
    return (slot_bytes + 127) & ~127;
}

}  // namespace

PersistentDecoder::~PersistentDecoder() {
    for (void* p : owned_) cudaFree(p);
}

bool PersistentDecoder::eligible(const FusedConfig& c, const lsx_ctx* ctx, std::string* why) {
    if (!FusedDecoder::eligible(c, why)) return false;
    if (!kernel_for(c)) {
        if (why) *why = "no persistent kernel instantiation for this head_dim";
        return false;
    }
    if (c.vocab > 0x7FFFF) {
        if (why) *why = "vocabulary above 524287";
        return false;
    }
    if (c.qheads > ctx->sm_count) {
        if (why) *why = "more query heads than SMs";
        return false;
    }
    if (c.hidden > kGainRegs * kCompute) {
        if (why) *why = "hidden width above the register-gain limit";
        return false;
    }
    return true;
}

int PersistentDecoder::build(lsx_ctx* ctx, const FusedConfig& c, const std::vector<FusedLayer>& layers) {
    std::string why;
    if (!eligible(c, ctx, &why)) return fail(LSX_E_UNSUPPORTED, "persistent decode plan: " + why);
    for (const FusedLayer& L : layers)  // the register-resident RMSNorm gains are read 16 bytes at a time
        LSX_ENSURE((uintptr_t)L.input_gain % 16 == 0 && (uintptr_t)L.post_gain % 16 == 0,
                   "persistent decode plan: norm gains must be 16-byte aligned");
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
    LSX_TRY(alloc((size_t)grid_ * kArgStride * 8, (void**)&t_arg_));
    // Split attention from position split_min_ - 1 on (LSX_DECODE_SPLIT_MIN overrides;
    // 0 turns it off).
    ns_ = split_slots(c, grid_);
    split_min_ = 128;
    if (const char* v = std::getenv("LSX_DECODE_SPLIT_MIN")) split_min_ = std::max(0, std::atoi(v));
    if (split_min_ == 0) ns_ = 0;
    if (ns_ > 0) LSX_TRY(alloc((size_t)c.qheads * ns_ * (c.head_dim + 2) * 8, (void**)&t_part_));
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
    // Shared memory: ring slots first, then x, scratch, owned residual rows,
    // barriers and the tables.  As many slots as fit, at most 16.
    const int slot_bytes = slot_bytes_for(c);
    cudaFuncAttributes fattr{};
    LSX_CUDA(cudaFuncGetAttributes(&fattr, (const void*)kernel_for(c)), "persistent kernel attributes");
    const size_t limit = ctx->smem_optin - fattr.sharedSizeBytes;  // the static s_spin word included
    slots_ = 0;
    for (int s = 16; s >= 2; --s)
        if ((size_t)layout_for(c, s, slot_bytes, grid_, layers.size()).total <= limit) {
            slots_ = s;
            break;
        }
    if (slots_ == 0) return fail(LSX_E_UNSUPPORTED, "persistent decode plan: shared memory");
    // Weight chunks each SM keeps in flight: six 16 KB chunks per SM (14 MB over
    // the GPU) saturate HBM; a cap of 0 (every free slot), 6 or 8 measures within 1%.
    // LSX_DECODE_INFLIGHT overrides.
    inflight_ = std::min(6, slots_ - 1);
    if (const char* v = std::getenv("LSX_DECODE_INFLIGHT")) inflight_ = std::max(0, std::min(std::atoi(v), slots_ - 1));
    // At hidden 1024 two chunks per SM carry the layers' weights (they need about a
    // third of HBM's bandwidth): 1% faster generations than six, one was 9% slower
    // (measured at that width only; wider models keep the head's cap).
    // LSX_DECODE_INFLIGHT_LAYERS overrides.
    inflight_layers_ = c.hidden <= 1024 ? std::min(2, slots_ - 1) : inflight_;
    if (const char* v = std::getenv("LSX_DECODE_INFLIGHT_LAYERS"))
        inflight_layers_ = std::max(0, std::min(std::atoi(v), slots_ - 1));
    layer_count_ = (int)layers.size();
    smem_ = (size_t)layout_for(c, slots_, slot_bytes, grid_, layers.size()).total;
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
    a.t_part = t_part_;
    a.ns = ns_;
    a.bs = 16;
    a.split_min = split_min_;
    a.state = state_;
    a.steps = steps;
    a.slots = slots_;
    a.slot_bytes = slot_bytes_for(c);
    a.inflight = inflight_;
    a.inflight_layers = inflight_layers_;
    a.sm = layout_for(c, slots_, a.slot_bytes, grid_, (size_t)layer_count_);
    void* args[] = {&a};
    LSX_CUDA(cudaLaunchCooperativeKernel((const void*)kernel_for(c), dim3(grid_), dim3(kThreads), args, smem_,
                                         ctx_->stream),
             "persistent decode launch");
    return LSX_OK;
}

}  // namespace lsx
