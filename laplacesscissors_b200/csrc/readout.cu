// Fused readout-margin validation on B200 tensor cores.
//
// For many hidden states h_i and target tokens t_i this computes, without ever
// storing logits,
//     z_i        = W (Q h_i) + b                        (W: [V, H] bf16 lm_head)
//     margin_i   = f64(z_i[t_i]) - f64(max_{j != t_i} z_i[j])   (lowest index on ties)
//     argmax_i   = first index of max_j z_i[j]
// which is what verify_cached does per prefix with Model::readout, argmax and
// minimum_margin (src/diagnosis.rs:493-580, 490-492, 58-70; src/model.rs:664-685).
//
// The edit Q = I + U^T (R - I) U (rank r, U orthonormal rows; a plane is r = 2)
// enters as a rank-r correction, the identity CompactReadout uses
// (src/diagnosis.rs:608-666):
//     W Q h = W h + F c,   F = W U^T  [V, r],   c = (R - I) U h  [r]
// The main product W h runs on tcgen05 with bf16 operands and f32 accumulation in
// TMEM: a bf16 hidden state is exact; an f32 hidden state is split into hi + lo
// bf16 planes (two MMAs).  F c is appended as one extra K block of split-bf16
// terms [c_hi | c_lo | c_hi] x [F_hi | F_hi | F_lo], so the correction keeps
// ~16 more bits than a bf16 rounding of Q h would.
//
// Kernel structure (one persistent CTA per SM, 6 warps):
//   warp 0     TMA producer: A (hidden) and B (lm_head) tiles, 128B swizzle
//   warp 1     TMEM owner and single-thread MMA issuer (tcgen05.mma kind::f16)
//   warps 2-5  epilogue: tcgen05.ld of the 128 x 256 f32 accumulator, per-row
//              best-other / target logit, one 64-bit atomicMax per row and tile
// Two TMEM accumulators (2 x 256 columns) let the epilogue of one tile overlap
// the MMAs of the next.  Tiles are ordered with the hidden-row block fastest so
// concurrently running CTAs share each lm_head block through L2.
// No load uses cluster multicast; every TMA source is this GPU's own memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <math.h>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <vector>

#include "device_common.cuh"
#include "lsx_internal.h"

namespace lsx {

constexpr int RM = 128;  // hidden rows per tile (TMEM lanes)
constexpr int RN = 256;  // vocab columns per tile
constexpr int RK = 64;   // K per stage: 64 bf16 = 128 bytes = one swizzle atom row
constexpr int kReadoutThreads = 192;
constexpr int kTileBytesA = RM * RK * 2;  // 16 KB
constexpr int kTileBytesB = RN * RK * 2;  // 32 KB

struct ReadoutParams {
    int M, V, H;
    int k_blocks, ext_blocks, m_tiles, n_tiles;
    const uint32_t* targets;
    int vocab_offset;               // global index of column 0 (a vocabulary shard's first row)
    const float* bias;
    unsigned long long* other_key;  // [M] packed (value, index) of the best non-target
    float* target_logit;            // [M]
    int* status;                    // [0] device error code, [1] non-finite flag
    // store mode: out[M, ldo] (=|+=) A B^T + bias, columns [0, V)
    float* out;
    int ldo, accumulate;
    // store mode, split over K: ksplits > 1 writes K-slice s's product to
    // partial + s * M * V (row stride V, no bias), summed by split_reduce_kernel
    int ksplits;
    float* partial;
    // store mode, gated (gated = activation kind + 1; 0: off): the columns are
    // interleaved (gate, up) pairs, and instead of out the epilogue writes
    // act(gate + bias) * (up + bias) for column pair j as bf16 hi and lo terms at
    // g_hi / g_lo [row * ldg + j] (the next GEMM's A planes)
    int gated;
    __nv_bfloat16* g_hi;
    __nv_bfloat16* g_lo;
    int ldg;
};

enum { kModeMargin = 0, kModeStore = 2 };

// ---------------------------------------------------------------- PTX ------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Prefetch a tile of this GPU's memory into L2 (no shared-memory destination).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile whose rows are 128 bytes,
// stored by TMA with 128-byte swizzle: 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);        // start address
    d |= (uint64_t)1 << 16;                        // leading byte offset (unused with swizzle)
    d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                        // descriptor version for sm_100
    d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16, bf16 A and B (K-major), f32 accumulate, M x N.
constexpr uint32_t kIdesc = (1u << 4)            // D format f32
                            | (1u << 7)          // A format bf16
                            | (1u << 10)         // B format bf16
                            | ((RN >> 3) << 17)  // N
                            | ((RM >> 4) << 24); // M

// Waits for this thread's tcgen05.ld results; the registers are tied to the wait
// so no use of them can be scheduled before it.
__device__ __forceinline__ void tc_wait_ld_regs(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// Running margin state of one hidden row over one tile.
struct RowScan {
    float best = -INFINITY;  // best non-target logit so far
    int best_col = -1;       // its tile column (lowest on ties)
    float tval = 0.f;        // the target's logit when it lies in this tile
    float probe = 0.f;       // becomes NaN once any logit is non-finite (z * 0)
};

// Folds 32 accumulator columns [c0, c0 + 32) of one row into the scan: the target
// column is set aside, the rest reduce by a max tree, and the (rare) chunk that
// beats the running best is searched for its first maximal column.
template <bool BIAS, bool TAIL>
__device__ __forceinline__ void scan_chunk(const uint32_t (&r)[32], int c0, int tcol, int n0, const ReadoutParams& p,
                                           RowScan& st) {
    float z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        float v = __uint_as_float(r[i]);
        if (BIAS) v += __ldg(&p.bias[min(n0 + c0 + i, p.V - 1)]);
        if (TAIL && n0 + c0 + i >= p.V) v = -INFINITY;
        else st.probe = fmaf(v, 0.f, st.probe);
        if (c0 + i == tcol) {
            st.tval = v;
            v = -INFINITY;
        }
        z[i] = v;
    }
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = fmaxf(fmaxf(z[4 * j], z[4 * j + 1]), fmaxf(z[4 * j + 2], z[4 * j + 3]));
    const float mx = fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
    if (mx > st.best) {
        int idx = 31;
#pragma unroll
        for (int i = 30; i >= 0; --i) idx = z[i] == mx ? i : idx;
        st.best = mx;
        st.best_col = c0 + idx;
    }
}

// One row's pass over a 256-column accumulator: TMEM loads run one 32-column
// chunk ahead of the scan.
__device__ __forceinline__ void scan_tile(uint32_t taddr, int tcol, int n0, const ReadoutParams& p, RowScan& st) {
    uint32_t ra[32], rb[32];
    const bool bias = p.bias != nullptr, tail = n0 + RN > p.V;
    tc_ld32(taddr, ra);
    tc_wait_ld_regs(ra);
#pragma unroll 1
    for (int c = 0; c < RN / 32; c += 2) {
        tc_ld32(taddr + (uint32_t)((c + 1) * 32), rb);
        if (bias) scan_chunk<true, true>(ra, c * 32, tcol, n0, p, st);
        else if (tail) scan_chunk<false, true>(ra, c * 32, tcol, n0, p, st);
        else scan_chunk<false, false>(ra, c * 32, tcol, n0, p, st);
        tc_wait_ld_regs(rb);
        if (c + 2 < RN / 32) tc_ld32(taddr + (uint32_t)((c + 2) * 32), ra);
        if (bias) scan_chunk<true, true>(rb, (c + 1) * 32, tcol, n0, p, st);
        else if (tail) scan_chunk<false, true>(rb, (c + 1) * 32, tcol, n0, p, st);
        else scan_chunk<false, false>(rb, (c + 1) * 32, tcol, n0, p, st);
        if (c + 2 < RN / 32) tc_wait_ld_regs(ra);
    }
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    long long start = clock64();
    while (!mbar_try_wait(a, parity)) {
        if (*abort_flag) return false;
        if (clock64() - start > kWaitCycles) return false;
    }
    return true;
}

// Store epilogue of one accumulator tile: this thread's row of out (=|+=) the
// tile's 256 columns (+ bias), 32 columns per TMEM load.  With `accumulate` the
// row's current values for the next 32 columns are loaded while the present ones
// are summed, so each chunk costs one memory round trip at most.
// The gated form of store_tile: 16 (gate, up) column pairs per 32-column chunk.
__device__ __forceinline__ void store_tile_gated(uint32_t taddr, int row, bool live, int n0, const ReadoutParams& p,
                                                 bool& nonfinite) {
    const int kind = p.gated - 1;
    const bool vec = (p.ldg & 7) == 0;
#pragma unroll 1
    for (int c = 0; c < RN / 32; ++c) {
        uint32_t r[32];
        tc_ld32(taddr + (uint32_t)(c * 32), r);
        tc_wait_ld();
        const int nb = n0 + c * 32;
        if (!live || nb >= p.V) continue;
        uint32_t hw[8], lw[8];  // bf16 pairs: feature 2 j in the low half, 2 j + 1 in the high half
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int col = nb + 2 * i;
            float g = __uint_as_float(r[2 * i]), u = __uint_as_float(r[2 * i + 1]);
            if (p.bias && col + 1 < p.V) {
                g += p.bias[col];
                u += p.bias[col + 1];
            }
            if (col + 1 < p.V) nonfinite |= !(isfinite(g) && isfinite(u));
            const float v = act_fn(g, kind) * u;
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            const uint32_t hb = __bfloat16_as_ushort(h);
            const uint32_t lb = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
            if (i & 1) {
                hw[i >> 1] |= hb << 16;
                lw[i >> 1] |= lb << 16;
            } else {
                hw[i >> 1] = hb;
                lw[i >> 1] = lb;
            }
        }
        const size_t o = (size_t)row * p.ldg + (size_t)(nb >> 1);
        if (vec && nb + 32 <= p.V) {
            reinterpret_cast<uint4*>(p.g_hi + o)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            reinterpret_cast<uint4*>(p.g_hi + o)[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            reinterpret_cast<uint4*>(p.g_lo + o)[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            reinterpret_cast<uint4*>(p.g_lo + o)[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (nb + 2 * i + 1 < p.V) {
                    p.g_hi[o + i] = __ushort_as_bfloat16((unsigned short)(hw[i >> 1] >> (16 * (i & 1))));
                    p.g_lo[o + i] = __ushort_as_bfloat16((unsigned short)(lw[i >> 1] >> (16 * (i & 1))));
                }
            }
        }
    }
}

__device__ __forceinline__ void store_tile(uint32_t taddr, int row, bool live, int n0, const ReadoutParams& p,
                                           bool& nonfinite) {
    if (p.gated) {
        store_tile_gated(taddr, row, live, n0, p, nonfinite);
        return;
    }
    float* orow = p.out + (size_t)(live ? row : 0) * p.ldo;
    const bool vec = (p.ldo & 3) == 0;
    float4 cur[8], nxt[8];
    auto fetch = [&](int c, float4 (&dst)[8]) {
        const int nb = n0 + c * 32;
        if (p.accumulate && live && vec && nb + 32 <= p.V) {
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = __ldcg(reinterpret_cast<const float4*>(orow + nb) + i);
        }
    };
    fetch(0, cur);
#pragma unroll 1
    for (int c = 0; c < RN / 32; ++c) {
        uint32_t r[32];
        tc_ld32(taddr + (uint32_t)(c * 32), r);
        if (c + 1 < RN / 32) fetch(c + 1, nxt);
        tc_wait_ld();
        const int nb = n0 + c * 32;
        if (live && nb < p.V) {
            if (nb + 32 <= p.V && vec) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 v = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                           __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
                    if (p.bias) {
                        v.x += p.bias[nb + 4 * i];
                        v.y += p.bias[nb + 4 * i + 1];
                        v.z += p.bias[nb + 4 * i + 2];
                        v.w += p.bias[nb + 4 * i + 3];
                    }
                    if (p.accumulate) {
                        v.x = cur[i].x + v.x;
                        v.y = cur[i].y + v.y;
                        v.z = cur[i].z + v.z;
                        v.w = cur[i].w + v.w;
                    }
                    nonfinite |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
                    reinterpret_cast<float4*>(orow + nb)[i] = v;
                }
            } else {
                for (int i = 0; i < 32 && nb + i < p.V; ++i) {
                    float v = __uint_as_float(r[i]) + (p.bias ? p.bias[nb + i] : 0.f);
                    if (p.accumulate) v = orow[nb + i] + v;
                    nonfinite |= !isfinite(v);
                    orow[nb + i] = v;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
    }
}

// MODE kModeMargin: the margin epilogue above.
// MODE kModeStore: a plain GEMM, out = A B^T (+ bias), or out += ... with
// `accumulate` (a residual add: each output element belongs to one tile).
template <int PLANES, int STAGES, int MODE>
__global__ void __launch_bounds__(kReadoutThreads, 1)
    readout_margin_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                          const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_ea,
                          const __grid_constant__ CUtensorMap map_eb, const ReadoutParams p) {
    constexpr int kStageBytes = PLANES * kTileBytesA + kTileBytesB;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_count = const_cast<int*>(abort_flag) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.m_tiles * p.n_tiles;
    const int k_total = p.k_blocks + p.ext_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4 * 32);
        }
        *abort_flag = 0;
        *issued_count = 0;
        fence_barrier_init();
    }
    if (warp == 1) {  // TMEM: two 256-column f32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            // CTAs that share an lm_head block start it together, so without a
            // prefetch every K stage of it is a DRAM miss for all of them; warm
            // L2 one tile ahead instead.
            if (blockIdx.x < total)
                for (int kb = 0; kb < p.k_blocks; ++kb)
                    tma_prefetch_2d(&map_b, kb * RK, (blockIdx.x / p.m_tiles) * RN);
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const int m0 = (tile % p.m_tiles) * RM;
                const int n0 = (tile / p.m_tiles) * RN;
                const int next = tile + gridDim.x;
                if (next < total && (next / p.m_tiles) != (tile / p.m_tiles))
                    for (int kb = 0; kb < p.k_blocks; ++kb)
                        tma_prefetch_2d(&map_b, kb * RK, (next / p.m_tiles) * RN);
                // Tiles that share an operand block run side by side; each starts its
                // K sweep at a different block so they do not all request the same
                // lines at once.
                const int rot = tile % k_total;
                for (int kq = 0; kq < k_total; ++kq) {
                    const int kb = kq + rot < k_total ? kq + rot : kq + rot - k_total;
                    if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * kStageBytes;
                    uint8_t* sb = sa + PLANES * kTileBytesA;
                    if (kb < p.k_blocks) {
                        mbar_expect_tx(&full[stage], kStageBytes);
                        tma_load_2d(sa, &map_a, kb * RK, m0, &full[stage]);
                        if (PLANES == 2) tma_load_2d(sa + kTileBytesA, &map_a2, kb * RK, m0, &full[stage]);
                        tma_load_2d(sb, &map_b, kb * RK, n0, &full[stage]);
                    } else {
                        const int e = kb - p.k_blocks;
                        mbar_expect_tx(&full[stage], kTileBytesA + kTileBytesB);
                        tma_load_2d(sa, &map_ea, e * RK, m0, &full[stage]);
                        tma_load_2d(sb, &map_eb, e * RK, n0, &full[stage]);
                    }
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            *issued_count = issued;
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // ---------------- MMA issuer ----------------
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                if (!wait_or_abort(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * RN);
                const int rot = tile % k_total;  // the producer's K order
                for (int kq = 0; kq < k_total; ++kq) {
                    const int kb = kq + rot < k_total ? kq + rot : kq + rot - k_total;
                    if (!wait_or_abort(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * kStageBytes);
                    const uint32_t sb = sa + PLANES * kTileBytesA;
                    const uint64_t bdesc = smem_desc_sw128(sb);
                    const int planes = kb < p.k_blocks ? PLANES : 1;
                    for (int pl = 0; pl < planes; ++pl) {
                        const uint64_t adesc = smem_desc_sw128(sa + pl * kTileBytesA);
#pragma unroll
                        for (int k = 0; k < RK / 16; ++k) {
                            // +32 bytes along K inside the swizzle atom per 16-element step
                            const uint32_t accumulate = (kq | pl | k) != 0;
                            tc_mma(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kIdesc, accumulate);
                        }
                    }
                    tc_commit(&empty[stage]);  // frees the stage once these MMAs have read it
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else {  // ---------------- epilogue warps 2..5 ----------------
        const int quarter = warp & 3;  // TMEM lane group this warp may access
        const int row_local = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool nonfinite = false;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            const int m0 = (tile % p.m_tiles) * RM;
            const int n0 = (tile / p.m_tiles) * RN;
            const bool ok = wait_or_abort(&tmem_full[acc], acc_phase, abort_flag);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) {
                    atomicExch(&p.status[0], kDeviceTimeoutEpilogue);
                    *abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            if (MODE == kModeStore) {
                const int row = m0 + row_local;
                store_tile(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * RN), row, row < p.M, n0, p,
                           nonfinite);
                tc_fence_before();
                mbar_arrive(&tmem_empty[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
                continue;
            }
            const int row = m0 + row_local;
            const bool live = row < p.M;
            const int tcol = live ? (int)((long long)p.targets[row] - p.vocab_offset - n0) : -1;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * RN);
            RowScan scan;
            scan_tile(taddr, tcol, n0, p, scan);
            nonfinite |= scan.probe != 0.f;  // NaN (non-finite logit) or never 0 otherwise
            const float best = scan.best, tval = scan.tval;
            const int best_col = scan.best_col;
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
            if (live) {
                if (best_col >= 0)
                    atomicMax(&p.other_key[row], pack_arg(best, (uint32_t)(p.vocab_offset + n0 + best_col)));
                if (tcol >= 0 && tcol < RN && n0 + tcol < p.V) p.target_logit[row] = tval;
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(&p.status[1], 1);
    }

    __syncthreads();
    if (*abort_flag) {
        // Leave nothing in flight: wait (bounded) for every TMA stage that was issued.
        if (threadIdx.x == 0) {
            const int issued = *issued_count;
            for (int s = 0; s < STAGES && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % STAGES);  // latest use of stage s
                mbar_wait_bounded(&full[s], (uint32_t)((last / STAGES) & 1));
            }
        }
        __syncthreads();
    }
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
}

// ------------------------------------------------- CTA-pair margin kernel --
// The same margin GEMM on CTA pairs (a cluster of 2, tcgen05 cta_group::2, M = 256
// per MMA): each CTA of the pair loads its own 128 hidden rows and its half (128
// rows) of the 256-row lm_head block, and the pair's MMA reads both halves, so each
// CTA moves 32 KB per K block instead of 48 KB for the same 128 x 256 outputs.
// The margin path is bound by operand traffic out of L2, so this is the lever.
// Protocol (the one CUTLASS's 2-SM pipelines use):
//   - both CTAs allocate TMEM with cta_group::2; the even CTA (leader) issues MMAs;
//   - each producer waits for its own stage to be released, the leader expects the
//     pair's bytes on its own `full` barrier and both producers' TMA loads (never
//     multicast; sources are this GPU's memory) complete on that barrier;
//   - the leader's commits arrive on both CTAs' `empty` / `tmem_full` barriers;
//   - both CTAs' epilogue warps release an accumulator on the leader's `tmem_empty`;
//   - cluster barriers after initialisation and before TMEM is freed.
constexpr int kPairRows = 2 * RM;       // rows per pair tile
constexpr int kHalfN = RN / 2;          // lm_head rows loaded by each CTA
constexpr int kHalfBytesB = kHalfN * RK * 2;  // 16 KB
constexpr uint32_t kIdescPair = (1u << 4) | (1u << 7) | (1u << 10) | ((RN >> 3) << 17) | ((kPairRows >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory object in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA 2-D load into this CTA's shared memory, completing on a barrier of the pair
// (given as a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
// Arrive (once, when the issued MMAs complete) on `bar` in both CTAs of the pair.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}

template <int PLANES, int STAGES, int MODE = kModeMargin>
__global__ void __launch_bounds__(kReadoutThreads, 1)
    readout_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_a2,
                        const __grid_constant__ CUtensorMap map_b, const __grid_constant__ CUtensorMap map_ea,
                        const __grid_constant__ CUtensorMap map_eb, const ReadoutParams p) {
    constexpr int kStageBytes = PLANES * kTileBytesA + kHalfBytesB;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_count = const_cast<int*>(abort_flag) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();  // 0: leader
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int m_pairs = (p.M + kPairRows - 1) / kPairRows;
    const int ksplits = (MODE == kModeStore && p.ksplits > 1) ? p.ksplits : 1;
    const int base_tiles = m_pairs * p.n_tiles;
    const int total = base_tiles * ksplits;
    const int k_total = p.k_blocks + p.ext_blocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);   // the leader's expect_tx arrival (+ the pair's bytes)
            mbar_init(&empty[s], 1);  // the leader's MMA commit
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);   // the leader's commit after a tile's MMAs
            mbar_init(&tmem_empty[a], 8);  // the 4 epilogue warps of both CTAs (leader's copy)
        }
        *abort_flag = 0;
        *issued_count = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---------------- TMA producer (both CTAs) ----------------
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            const uint32_t full0 = map_to_rank(smem_u32(&full[0]), 0);
            for (int tile = pair; tile < total && ok; tile += pairs) {
                const int ks = tile / base_tiles, bt = tile - ks * base_tiles;
                const int m0 = (bt % m_pairs) * kPairRows + (int)rank * RM;
                const int n0 = (bt / m_pairs) * RN + (int)rank * kHalfN;
                const int kb0 = ks * k_total / ksplits, kb1 = (ks + 1) * k_total / ksplits;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * kStageBytes;
                    uint8_t* sb = sa + PLANES * kTileBytesA;
                    const uint32_t fb = full0 + (uint32_t)(stage * 8);
                    if (kb < p.k_blocks) {
                        if (rank == 0) mbar_expect_tx(&full[stage], 2 * kStageBytes);
                        tma_load_2d_pair(sa, &map_a, kb * RK, m0, fb);
                        if (PLANES == 2) tma_load_2d_pair(sa + kTileBytesA, &map_a2, kb * RK, m0, fb);
                        tma_load_2d_pair(sb, &map_b, kb * RK, n0, fb);
                    } else {
                        const int e = kb - p.k_blocks;
                        if (rank == 0) mbar_expect_tx(&full[stage], 2 * (kTileBytesA + kHalfBytesB));
                        tma_load_2d_pair(sa, &map_ea, e * RK, m0, fb);
                        tma_load_2d_pair(sb, &map_eb, e * RK, n0, fb);
                    }
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            *issued_count = issued;
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // ---------------- MMA issuer (leader) ----------------
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = pair; tile < total && ok; tile += pairs) {
                if (!wait_or_abort(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * RN);
                const int ks = tile / base_tiles;
                const int kb0 = ks * k_total / ksplits, kb1 = (ks + 1) * k_total / ksplits;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!wait_or_abort(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * kStageBytes);
                    const uint32_t sb = sa + PLANES * kTileBytesA;
                    const uint64_t bdesc = smem_desc_sw128(sb);
                    const int planes = kb < p.k_blocks ? PLANES : 1;
                    for (int pl = 0; pl < planes; ++pl) {
                        const uint64_t adesc = smem_desc_sw128(sa + pl * kTileBytesA);
#pragma unroll
                        for (int k = 0; k < RK / 16; ++k) {
                            const uint32_t accumulate = ((kb - kb0) | pl | k) != 0;
                            tc_mma_pair(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kIdescPair,
                                        accumulate);
                        }
                    }
                    tc_commit_pair(&empty[stage]);  // frees the stage in both CTAs
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit_pair(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else {  // ---------------- epilogue warps 2..5 (both CTAs) ----------------
        const int quarter = warp & 3;
        const int row_local = quarter * 32 + lane;
        const uint32_t tmem_empty0 = map_to_rank(smem_u32(&tmem_empty[0]), 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        bool nonfinite = false;
        for (int tile = pair; tile < total; tile += pairs) {
            const int ks = tile / base_tiles, bt = tile - ks * base_tiles;
            const int m0 = (bt % m_pairs) * kPairRows + (int)rank * RM;
            const int n0 = (bt / m_pairs) * RN;
            const bool ok = wait_or_abort(&tmem_full[acc], acc_phase, abort_flag);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) {
                    atomicExch(&p.status[0], kDeviceTimeoutEpilogue);
                    *abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const int row = m0 + row_local;
            const bool live = row < p.M;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * RN);
            if (MODE == kModeStore) {
                if (ksplits > 1) {  // this K slice's product, plain, into its partial plane
                    ReadoutParams q = p;
                    q.out = p.partial + (size_t)ks * p.M * p.V;
                    q.ldo = p.V;
                    q.accumulate = 0;
                    q.bias = nullptr;
                    bool unused = false;
                    store_tile(taddr, row, live, n0, q, unused);
                } else {
                    store_tile(taddr, row, live, n0, p, nonfinite);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(tmem_empty0 + (uint32_t)(acc * 8));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
                continue;
            }
            const int tcol = live ? (int)((long long)p.targets[row] - p.vocab_offset - n0) : -1;
            RowScan scan;
            scan_tile(taddr, tcol, n0, p, scan);
            nonfinite |= scan.probe != 0.f;  // NaN (non-finite logit) or never 0 otherwise
            const float best = scan.best, tval = scan.tval;
            const int best_col = scan.best_col;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tmem_empty0 + (uint32_t)(acc * 8));
            if (live) {
                if (best_col >= 0)
                    atomicMax(&p.other_key[row], pack_arg(best, (uint32_t)(p.vocab_offset + n0 + best_col)));
                if (tcol >= 0 && tcol < RN && n0 + tcol < p.V) p.target_logit[row] = tval;
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(&p.status[1], 1);
    }

    __syncthreads();
    if (*abort_flag) {
        // Leave nothing in flight: wait (bounded) for every TMA stage this CTA issued
        // whose completion the leader's barrier would show.
        if (threadIdx.x == 0 && rank == 0) {
            const int issued = *issued_count;
            for (int s = 0; s < STAGES && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % STAGES);
                mbar_wait_bounded(&full[s], (uint32_t)((last / STAGES) & 1));
            }
        }
        __syncthreads();
    }
    tc_fence_before();
    cluster_sync();  // the pair's MMAs and epilogues are done with both CTAs' memory
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
}

// Sum of the K slices of a split store GEMM, in slice order: out[m, n] (=|+=)
// sum_s partial[s, m, n] (+ bias[n]); a non-finite result raises status[1].
__global__ void split_reduce_kernel(const float* __restrict__ partial, int ksplits, int M, int N,
                                    const float* __restrict__ bias, float* __restrict__ out, int ldo, int accumulate,
                                    int* status) {
    pdl_wait();  // a no-op unless launched as a programmatic dependent of the GEMM
    const size_t total = (size_t)M * N, plane = total;
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i - (size_t)m * N);
        float v = partial[i];
        for (int sl = 1; sl < ksplits; ++sl) v += partial[(size_t)sl * plane + i];
        if (bias) v += bias[n];
        float* o = out + (size_t)m * ldo + n;
        if (accumulate) v = *o + v;
        bad |= !isfinite(v);
        *o = v;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(&status[1], 1);
}

// ------------------------------------------------------------ prep kernels --
// The edit basis U [rank, H] f32 as the A operand of the image GEMM: rows 2k and
// 2k + 1 hold bf16 hi and lo of U's row k0 + k.
__global__ void basis_split_kernel(const float* __restrict__ basis, int H, int k0, int kc,
                                   __nv_bfloat16* __restrict__ out) {
    const int total = kc * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int k = i / H, j = i - k * H;
        const float u = basis[(size_t)(k0 + k) * H + j];
        const __nv_bfloat16 hi = __float2bfloat16_rn(u);
        out[(size_t)(2 * k) * H + j] = hi;
        out[(size_t)(2 * k + 1) * H + j] = __float2bfloat16_rn(u - __bfloat162float(hi));
    }
}

// Directions [count, H] f32 as the B operand of the f32 image pass: rows 4k .. 4k + 3
// hold bf16 hi, mid, lo of direction k0 + k (their sum is the f32 value exactly)
// and a zero row.
__global__ void direction_split_kernel(const float* __restrict__ dirs, int H, int k0, int kc,
                                       __nv_bfloat16* __restrict__ out) {
    const int total = kc * H;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int k = i / H, j = i - k * H;
        const float u = dirs[(size_t)(k0 + k) * H + j];
        const __nv_bfloat16 hi = __float2bfloat16_rn(u);
        const float r1 = u - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        out[(size_t)(4 * k) * H + j] = hi;
        out[(size_t)(4 * k + 1) * H + j] = mid;
        out[(size_t)(4 * k + 2) * H + j] = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        out[(size_t)(4 * k + 3) * H + j] = __float2bfloat16_rn(0.f);
    }
}

// ------------------------------------------------------- edit image kernel --
// F = W U^T for ranks [k0, k0 + kc) of the edit, written as the B extension of
// the margin GEMM: row n of `image` holds [F_hi | F_hi | F_lo] (each `rank` wide)
// and zeros up to `ext_k`.  The lm_head is the A operand here (128 vocab rows per
// tile, one per TMEM lane) and the basis, as interleaved (hi, lo) bf16 rows, the B
// operand (N = np columns, 2 kc rounded up to 32; rows past 2 kc read as zero), so
// each epilogue thread owns one vocab row and writes it contiguously.  One pass
// reads the lm_head once and is bound by HBM.
//   warp 0     TMA producer (W tile 128 x 64, basis tile np x 64 per stage)
//   warp 1     TMEM owner, single-thread MMA issuer (M = 128, N = np, K = 16)
//   warps 2-5  epilogue: F_k = lane 2k + lane 2k + 1 of the accumulator, hi/lo split
constexpr int kImageM = 128;
constexpr int kImageMaxN = 128;        // 64 ranks per pass
constexpr int kImageRanks = kImageMaxN / 2;
constexpr int kImageThreads = 192;

struct ImageParams {
    int V, k_blocks, n_tiles, np, stages;
    int rank, k0, kc, ext_k;
    __nv_bfloat16* image;  // extension mode: [V, ext_k] bf16
    float* out;            // f32 mode: [rank, V] f32, row k = W u_k
    int accumulate;        // f32 mode: out += instead of out =
    int* status;
};

// Epilogue forms of edit_image_kernel.
//   kImageExtension: basis rows interleaved (hi, lo); writes [F_hi | F_hi | F_lo].
//   kImageF32: direction rows in groups of four (hi, mid, lo, 0), which hold an f32
//              direction exactly; writes W u_k in f32 (the head image of u_k).
enum { kImageExtension = 0, kImageF32 = 1 };

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* dst, const float* v) {
    __align__(16) __nv_bfloat16 b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = __float2bfloat16_rn(v[e]);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(b);
}

template <int MODE>
__global__ void __launch_bounds__(kImageThreads, 1)
    edit_image_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_u,
                      const ImageParams p) {
    constexpr int kTileW = kImageM * RK * 2;  // 16 KB
    const int tile_u = p.np * RK * 2;
    const int stage_bytes = kTileW + tile_u;
    const int S = p.stages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* tmem_full = empty + S;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_count = const_cast<int*>(abort_flag) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4 * 32);
        }
        *abort_flag = 0;
        *issued_count = 0;
        fence_barrier_init();
    }
    if (warp == 1) {  // TMEM: two accumulators of np <= 128 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---------------- TMA producer ----------------
            int stage = 0, issued = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sw = smem + (size_t)stage * stage_bytes;
                    mbar_expect_tx(&full[stage], (uint32_t)stage_bytes);
                    tma_load_2d(sw, &map_w, kb * RK, tile * kImageM, &full[stage]);
                    tma_load_2d(sw + kTileW, &map_u, kb * RK, 0, &full[stage]);
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            *issued_count = issued;
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // ---------------- MMA issuer ----------------
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.np >> 3) << 17) |
                                   ((uint32_t)(kImageM >> 4) << 24);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
                if (!wait_or_abort(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * p.np);
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!wait_or_abort(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sw = smem_u32(smem + (size_t)stage * stage_bytes);
                    const uint64_t adesc = smem_desc_sw128(sw), bdesc = smem_desc_sw128(sw + kTileW);
#pragma unroll
                    for (int k = 0; k < RK / 16; ++k)
                        tc_mma(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0);
                    tc_commit(&empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else {  // ---------------- epilogue warps 2..5 ----------------
        const int quarter = warp & 3;
        const int R = p.rank, k0 = p.k0, kc = p.kc;
        const bool vec = (R % 8) == 0 && (k0 % 8) == 0 && (kc % 8) == 0 && (p.ext_k % 8) == 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
            const bool ok = wait_or_abort(&tmem_full[acc], acc_phase, abort_flag);
            if (__any_sync(0xffffffffu, !ok)) {
                if (lane == 0) {
                    atomicExch(&p.status[0], kDeviceTimeoutEpilogue);
                    *abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const int n = tile * kImageM + quarter * 32 + lane;
            const bool live = n < p.V;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.np);
            if constexpr (MODE == kImageF32) {
                // eight directions per 32-column chunk: columns 4j .. 4j + 3 of direction j
#pragma unroll 1
                for (int c = 0; c < p.np / 32; ++c) {
                    uint32_t r[32];
                    tc_ld32(taddr + (uint32_t)(c * 32), r);
                    tc_wait_ld_regs(r);
                    if (live) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int k = 8 * c + j;
                            if (k < kc) {
                                const float f = (__uint_as_float(r[4 * j + 2]) + __uint_as_float(r[4 * j + 1])) +
                                                __uint_as_float(r[4 * j]);
                                float* o = p.out + (size_t)(k0 + k) * p.V + n;
                                *o = p.accumulate ? *o + f : f;
                            }
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&tmem_empty[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
                continue;
            }
            __nv_bfloat16* dst = p.image + (size_t)(live ? n : 0) * p.ext_k;
#pragma unroll 1
            for (int c = 0; c < p.np / 32; ++c) {
                uint32_t r[32];
                tc_ld32(taddr + (uint32_t)(c * 32), r);
                tc_wait_ld_regs(r);
                float hi[16], lo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float f = __uint_as_float(r[2 * j]) + __uint_as_float(r[2 * j + 1]);
                    const __nv_bfloat16 h = __float2bfloat16_rn(f);
                    hi[j] = __bfloat162float(h);
                    lo[j] = f - hi[j];
                }
                if (!live) continue;
                const int kb = 16 * c;  // first rank of this chunk, relative to k0
                if (vec) {
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        if (kb + 8 * g + 8 <= kc) {
                            const int k = k0 + kb + 8 * g;
                            store_bf16x8(dst + k, hi + 8 * g);
                            store_bf16x8(dst + R + k, hi + 8 * g);
                            store_bf16x8(dst + 2 * R + k, lo + 8 * g);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (kb + j < kc) {
                            const int k = k0 + kb + j;
                            dst[k] = __float2bfloat16_rn(hi[j]);
                            dst[R + k] = __float2bfloat16_rn(hi[j]);
                            dst[2 * R + k] = __float2bfloat16_rn(lo[j]);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
            if (live && k0 == 0)  // the padding columns of the extension block
                for (int k = 3 * R; k < p.ext_k; ++k) dst[k] = __float2bfloat16_rn(0.f);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) {
            const int issued = *issued_count;
            for (int i = 0; i < S && i < issued; ++i) {
                const int last = issued - 1 - ((issued - 1 - i) % S);
                mbar_wait_bounded(&full[i], (uint32_t)((last / S) & 1));
            }
        }
        __syncthreads();
    }
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem_base) : "memory");
}

// ---------------------------------------------------- few-row store GEMM ----
// out[M, ldo] (=|+=) (A_hi + A_lo) W^T (+ bias) for M <= 32 activation rows (a
// batched decode step): the weight is the A operand of the MMA (128 rows of W per
// tile, one per TMEM lane) and the activations' two bf16 planes are the B operand
// (N = 2 Mp columns: Mp hi rows, then Mp lo rows, Mp = M rounded up to 16), so a
// tile's tensor work is 128 x 2Mp per K step instead of a 256-row MMA with 16 live
// rows, and the pass is bound by streaming W from HBM.  Work items are (weight
// tile, K slice); with few tiles the K loop is split so every SM streams a share,
// each slice's product goes plain into its own partial plane, and
// split_reduce_kernel sums the slices in order (then bias, then the accumulate).
//   warp 0     TMA producer: W tile 128 x 64, hi and lo tiles Mp x 64 per stage
//   warp 1     TMEM owner, single-thread MMA issuer (M = 128, N = 2 Mp, K = 16)
//   warps 2-5  epilogue: lane = weight row n, column m + column Mp + m = out[m, n]
constexpr int kFewThreads = 192;
constexpr int kFewMaxRows = 32;

struct FewParams {
    int M, Mp, N, k_blocks, n_tiles, ksplits, stages;
    const float* bias;
    float* out;        // out[m * ldo + n] (=|+=) value + bias
    int ldo, accumulate;
    float* partial;    // ksplits > 1: partial[(s * M + m) * N + n] = slice s's product
    int* status;
};

__global__ void __launch_bounds__(kFewThreads, 1)
    few_rows_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_hi,
                    const __grid_constant__ CUtensorMap map_lo, const FewParams p) {
    constexpr int kTileW = 128 * RK * 2;  // 16 KB
    const int tile_a = p.Mp * RK * 2;     // one plane's tile
    const int stage_bytes = kTileW + 2 * tile_a;
    const int S = p.stages;
    const int ncol = 2 * p.Mp;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
    uint64_t* empty = full + S;
    uint64_t* tmem_full = empty + S;
    uint64_t* tmem_empty = tmem_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* issued_count = const_cast<int*>(abort_flag) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = p.n_tiles * p.ksplits;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4 * 32);
        }
        *abort_flag = 0;
        *issued_count = 0;
        fence_barrier_init();
        pdl_launch_dependents();
    }
    if (warp == 1) {  // TMEM: two accumulators of 2 Mp <= 64 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {  // ---------------- TMA producer ----------------
            // The weight tiles of the first S stages do not depend on earlier kernels:
            // they are requested before waiting for the preceding grid (a no-op
            // unless launched as a programmatic dependent); the activation tiles,
            // which the preceding kernel writes, after it.
            int pre = 0;
            for (int item = blockIdx.x; item < items && pre < S; item += gridDim.x) {
                const int tile = item / p.ksplits, slice = item % p.ksplits;
                const int kb0 = (int)((long long)slice * p.k_blocks / p.ksplits);
                const int kb1 = (int)((long long)(slice + 1) * p.k_blocks / p.ksplits);
                for (int kb = kb0; kb < kb1 && pre < S; ++kb, ++pre) {
                    mbar_expect_tx(&full[pre], (uint32_t)stage_bytes);
                    tma_load_2d(smem + (size_t)pre * stage_bytes, &map_w, kb * RK, tile * 128, &full[pre]);
                }
            }
            pdl_wait();
            int stage = 0, issued = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                const int tile = item / p.ksplits, slice = item % p.ksplits;
                const int kb0 = (int)((long long)slice * p.k_blocks / p.ksplits);
                const int kb1 = (int)((long long)(slice + 1) * p.k_blocks / p.ksplits);
                for (int kb = kb0; kb < kb1; ++kb) {
                    uint8_t* sw = smem + (size_t)stage * stage_bytes;
                    if (issued >= pre) {  // a stage's first use was prefilled with its weight tile
                        if (!wait_or_abort(&empty[stage], phase ^ 1u, abort_flag)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(&full[stage], (uint32_t)stage_bytes);
                        tma_load_2d(sw, &map_w, kb * RK, tile * 128, &full[stage]);
                    }
                    tma_load_2d(sw + kTileW, &map_hi, kb * RK, 0, &full[stage]);
                    tma_load_2d(sw + kTileW + tile_a, &map_lo, kb * RK, 0, &full[stage]);
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            *issued_count = issued;
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // ---------------- MMA issuer ----------------
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(ncol >> 3) << 17) |
                                   ((uint32_t)(128 >> 4) << 24);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                const int slice = item % p.ksplits;
                const int kb0 = (int)((long long)slice * p.k_blocks / p.ksplits);
                const int kb1 = (int)((long long)(slice + 1) * p.k_blocks / p.ksplits);
                if (!wait_or_abort(&tmem_empty[acc], acc_phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * 64);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!wait_or_abort(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sw = smem_u32(smem + (size_t)stage * stage_bytes);
                    const uint64_t adesc = smem_desc_sw128(sw), bdesc = smem_desc_sw128(sw + kTileW);
#pragma unroll
                    for (int k = 0; k < RK / 16; ++k)
                        tc_mma(d, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb > kb0 || k > 0));
                    tc_commit(&empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) {
                atomicExch(&p.status[0], kDeviceTimeoutMma);
                *abort_flag = 1;
            }
        }
        __syncwarp();
    } else {  // ---------------- epilogue warps 2..5 ----------------
        pdl_wait();  // out (accumulated into) and bias may come from earlier kernels
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool nonfinite = false;
        for (int item = blockIdx.x; item < items; item += gridDim.x) {
            const int tile = item / p.ksplits, slice = item % p.ksplits;
            const bool ok = wait_or_abort(&tmem_full[acc], acc_phase, abort_flag);
            // one decision for all four epilogue warps, which meet at named barriers below
            uint32_t bad;
            asm volatile(
                "{\n\t.reg .pred p, q;\n\tsetp.eq.u32 p, %1, 0;\n\tbar.red.or.pred q, 3, 128, p;\n\t"
                "selp.u32 %0, 1, 0, q;\n\t}"
                : "=r"(bad)
                : "r"((uint32_t)ok)
                : "memory");
            if (bad) {
                if (quarter == 0 && lane == 0) {
                    atomicExch(&p.status[0], kDeviceTimeoutEpilogue);
                    *abort_flag = 1;
                }
                break;
            }
            tc_fence_after();
            const int n = tile * 128 + quarter * 32 + lane;
            const bool live = n < p.N;
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * 64);
            uint32_t hi[32], lo[32];
            tc_ld32(taddr, hi);
            tc_wait_ld_regs(hi);
            if (p.Mp > 16) {
                tc_ld32(taddr + 32u, lo);
                tc_wait_ld_regs(lo);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) lo[j] = hi[16 + j];
            }
            tc_fence_before();
            mbar_arrive(&tmem_empty[acc]);
            const float b = (live && p.bias) ? p.bias[n] : 0.f;
            if (p.ksplits == 1) {
                if (live) {
#pragma unroll
                    for (int m = 0; m < kFewMaxRows; ++m) {
                        if (m < p.M) {
                            const float v = __uint_as_float(hi[m]) + __uint_as_float(lo[m]);
                            float* o = p.out + (size_t)m * p.ldo + n;
                            const float r = p.accumulate ? *o + (v + b) : v + b;
                            nonfinite |= !isfinite(r);
                            *o = r;
                        }
                    }
                }
            } else if (live) {  // this slice's product; split_reduce_kernel sums the slices in order
#pragma unroll
                for (int m = 0; m < kFewMaxRows; ++m)
                    if (m < p.M)
                        p.partial[((size_t)slice * p.M + m) * p.N + n] = __uint_as_float(hi[m]) + __uint_as_float(lo[m]);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(&p.status[1], 1);
    }

    __syncthreads();
    if (*abort_flag) {
        if (threadIdx.x == 0) {
            const int issued = *issued_count;
            for (int i = 0; i < S && i < issued; ++i) {
                const int last = issued - 1 - ((issued - 1 - i) % S);
                mbar_wait_bounded(&full[i], (uint32_t)((last / S) & 1));
            }
        }
        __syncthreads();
    }
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tmem_base) : "memory");
}

constexpr int kMaxEditRank = 256;

// c = (R - I) U h per hidden row (one warp per row) from the edit coordinates
// coords[k, row] = U_k . h_row ([rank, M], as the f32 image pass leaves them),
// written as [c_hi | c_lo | c_hi | 0 ...] into the extension block of A; with F32
// hidden rows also the bf16 hi/lo planes of the main product (coords NULL: the
// split only).
__global__ void __launch_bounds__(256) edit_coefficients_kernel(const void* __restrict__ hidden, int hidden_kind,
                                                                int M, int H, const float* __restrict__ coords,
                                                                const float* __restrict__ delta, int rank,
                                                                __nv_bfloat16* __restrict__ ext_a, int ext_k,
                                                                __nv_bfloat16* __restrict__ plane_hi,
                                                                __nv_bfloat16* __restrict__ plane_lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * 8 + warp;
    if (i >= M) return;
    if (plane_hi && hidden_kind == LSX_F32) {
        const float4* src = reinterpret_cast<const float4*>((const float*)hidden + (size_t)i * H);
        for (int v = lane; v < (H >> 3); v += 32) {
            const float4 a = __ldg(src + 2 * v), b = __ldg(src + 2 * v + 1);
            const float h[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            __align__(16) __nv_bfloat16 hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                hi[e] = __float2bfloat16_rn(h[e]);
                lo[e] = __float2bfloat16_rn(h[e] - __bfloat162float(hi[e]));
            }
            reinterpret_cast<uint4*>(plane_hi + (size_t)i * H)[v] = *reinterpret_cast<const uint4*>(hi);
            reinterpret_cast<uint4*>(plane_lo + (size_t)i * H)[v] = *reinterpret_cast<const uint4*>(lo);
        }
    }
    if (!coords) return;
    __nv_bfloat16* dst = ext_a + (size_t)i * ext_k;
    for (int k = 3 * rank + lane; k < ext_k; k += 32) dst[k] = __float2bfloat16_rn(0.f);
    for (int k = lane; k < rank; k += 32) {
        float c = 0.f;
        for (int q = 0; q < rank; ++q) c = fmaf(delta[k * rank + q], coords[(size_t)q * M + i], c);
        const __nv_bfloat16 hi = __float2bfloat16_rn(c);
        const __nv_bfloat16 lo = __float2bfloat16_rn(c - __bfloat162float(hi));
        dst[k] = hi;
        dst[rank + k] = lo;
        dst[2 * rank + k] = hi;
    }
}

// A target logit starts as NaN (never set: a target outside the vocabulary), or
// as -inf for a vocabulary shard, whose merge takes the maximum over shards.
__global__ void readout_init_kernel(unsigned long long* other_key, float* target_logit, int M, int* status,
                                    bool shard) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < M) {
        other_key[i] = 0ull;
        target_logit[i] = shard ? -INFINITY : __int_as_float(0x7fc00000);
    }
    if (i < 2) status[i] = 0;
}

// margin and first argmax from (best other, target logit): argmax is the target
// when it beats the best other, or ties it with a lower index.
__global__ void readout_finalize_kernel(const unsigned long long* other_key, const float* target_logit,
                                        const uint32_t* targets, int M, double* margin, uint32_t* argmax,
                                        float* target_out, uint32_t* other_out = nullptr) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M) return;
    const unsigned long long k = other_key[i];
    const float ov = packed_value(k);
    const uint32_t oi = packed_index(k);
    const float tv = target_logit[i];
    const uint32_t t = targets[i];
    if (margin) margin[i] = (double)tv - (double)ov;
    if (argmax) argmax[i] = (tv > ov || (tv == ov && t < oi)) ? t : oi;
    if (target_out) target_out[i] = tv;
    if (other_out) other_out[i] = oi;
}

// Vocabulary-shard partials in one signed-orderable int64 buffer [2 x M]: the
// best-other key with its top bit flipped (so signed order is the key's unsigned
// order), then the target logit's total-order key (non-negative).  An element-wise
// signed maximum over the shards -- one all-reduce MAX -- merges them.
__device__ __forceinline__ long long logit_order(float v) {
    const uint32_t b = __float_as_uint(v);
    return (long long)((b & 0x80000000u) ? ~b : (b | 0x80000000u));
}
__device__ __forceinline__ float order_logit(long long o) {
    const uint32_t u = (uint32_t)o;
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__global__ void shard_pack_kernel(long long* partials, const float* target_logit, int M) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M) return;
    partials[i] = (long long)((unsigned long long)partials[i] ^ 0x8000000000000000ull);
    partials[M + i] = logit_order(target_logit[i]);
}

__global__ void shard_merge_kernel(const long long* partials, const uint32_t* targets, int M, double* margin,
                                   uint32_t* argmax, float* target_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M) return;
    const unsigned long long k = (unsigned long long)partials[i] ^ 0x8000000000000000ull;
    const float ov = packed_value(k);
    const uint32_t oi = packed_index(k);
    const float tv = order_logit(partials[M + i]);
    const uint32_t t = targets[i];
    if (margin) margin[i] = (double)tv - (double)ov;
    if (argmax) argmax[i] = (tv > ov || (tv == ov && t < oi)) ? t : oi;
    if (target_out) target_out[i] = tv;
}

// ------------------------------------------------------ compact readout ----
// CompactReadout::evaluate (src/diagnosis.rs:643-665) fused with the margin rules:
// for observation o, z_o = image c_o + baseline_o (image [V, r] f32 row-major, the
// transposed head images; c_o the observation's (R - I) coordinates; baseline_o its
// current logits), reduced at once to the target logit and the best other column
// (packed key, lowest index on ties) instead of being stored.  A block scores
// kCompactObs observations over a grid-stride share of the vocabulary, so each
// image row it reads (from L2) serves all of them; baselines stream from HBM once.
constexpr int kCompactObs = 8;
constexpr int kCompactThreads = 256;

__global__ void __launch_bounds__(kCompactThreads) compact_margin_kernel(
    const float* __restrict__ image, const float* __restrict__ baseline, const float* __restrict__ coefficients,
    const uint32_t* __restrict__ targets, int V, int r, int n, unsigned long long* other_key, float* target_logit,
    int* status) {
    __shared__ float cs[kCompactObs][kMaxEditRank];
    __shared__ unsigned long long red[kCompactThreads / 32][kCompactObs];
    const int o0 = blockIdx.y * kCompactObs;
    const int no = min(kCompactObs, n - o0);
    for (int i = threadIdx.x; i < kCompactObs * r; i += blockDim.x) {
        const int o = i / r, k = i - o * r;
        cs[o][k] = o < no ? coefficients[(size_t)(o0 + o) * r + k] : 0.f;
    }
    __syncthreads();
    uint32_t tg[kCompactObs];
#pragma unroll
    for (int o = 0; o < kCompactObs; ++o) tg[o] = o < no ? targets[o0 + o] : 0xffffffffu;
    unsigned long long best[kCompactObs];
#pragma unroll
    for (int o = 0; o < kCompactObs; ++o) best[o] = 0ull;
    bool bad = false;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        float acc[kCompactObs];
#pragma unroll
        for (int o = 0; o < kCompactObs; ++o) acc[o] = 0.f;
        const float* row = image + (size_t)i * r;
        for (int k = 0; k < r; ++k) {
            const float w = __ldg(row + k);
#pragma unroll
            for (int o = 0; o < kCompactObs; ++o) acc[o] = fmaf(w, cs[o][k], acc[o]);
        }
#pragma unroll
        for (int o = 0; o < kCompactObs; ++o) {
            if (o < no) {
                const float z = acc[o] + __ldcs(baseline + (size_t)(o0 + o) * V + i);
                bad |= !isfinite(z);
                if ((uint32_t)i == tg[o]) {
                    target_logit[o0 + o] = z;
                } else {
                    const unsigned long long key = pack_arg(z, (uint32_t)i);
                    best[o] = key > best[o] ? key : best[o];
                }
            }
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 0; o < kCompactObs; ++o) {
        const unsigned long long b = warp_max_u64(best[o]);
        if (lane == 0) red[warp][o] = b;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&status[1], 1);
    __syncthreads();
    if (threadIdx.x < no) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kCompactThreads / 32; ++w) b = red[w][threadIdx.x] > b ? red[w][threadIdx.x] : b;
        if (b) atomicMax(&other_key[o0 + threadIdx.x], b);
    }
}

// ------------------------------------------------------------ host side ----
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
        else
            (void)cudaGetLastError();
    }
    return fn;
}

// 2-D bf16 tensor map of a row-major [rows, cols] matrix with a (64 x box_rows)
// box and 128-byte swizzle; out-of-range elements read as zero.
int make_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(LSX_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
    LSX_ENSURE((uintptr_t)base % 16 == 0 && row_bytes % 16 == 0, "tensor map operands must be 16-byte aligned");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)RK, box_rows};
    cuuint32_t elem[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(LSX_E_CUDA, "cuTensorMapEncodeTiled failed with " + std::to_string((int)r));
    return LSX_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }


struct Layout {
    size_t ext_k, planes_off, planes_bytes, ext_a_off, ext_b_off, basis_off, delta_off, image_a_off, coords_off, key_off,
        tlog_off, status_off, total;
};

// The two status words sit at the start of every layout, so lsx_readout_status can
// read them from any workspace without knowing the sizes of the call that used it.
Layout layout_for(size_t vocab, size_t width, size_t rows, size_t rank, bool f32_hidden) {
    Layout L{};
    L.ext_k = rank ? ((3 * rank + RK - 1) / RK) * RK : 0;
    size_t at = 0;
    L.status_off = at;
    at = align256(at + 16);
    L.planes_off = at;
    L.planes_bytes = f32_hidden ? rows * width * 2 : 0;
    at = align256(at + 2 * L.planes_bytes);
    L.ext_a_off = at;
    at = align256(at + rows * L.ext_k * 2);
    L.ext_b_off = at;
    at = align256(at + vocab * L.ext_k * 2);
    L.basis_off = at;
    at = align256(at + rank * width * 4);
    L.delta_off = at;
    at = align256(at + rank * rank * 4);
    L.image_a_off = at;
    at = align256(at + (rank ? std::max(2 * std::min(rank, (size_t)kImageRanks), (size_t)kImageMaxN) : 0) * width * 2);
    L.coords_off = at;
    at = align256(at + rows * rank * 4);
    L.key_off = at;
    at = align256(at + rows * 8);
    L.tlog_off = at;
    at = align256(at + rows * 4);
    L.total = at;
    return L;
}

template <int PLANES, int STAGES>
size_t readout_smem() {
    return (size_t)STAGES * (PLANES * kTileBytesA + kTileBytesB) + 1024 + (2 * STAGES + 4) * 8 + 16;
}

template <int PLANES, int STAGES>
size_t pair_smem() {
    return (size_t)STAGES * (PLANES * kTileBytesA + kHalfBytesB) + 1024 + (2 * STAGES + 4) * 8 + 16;
}

// Launches the CTA-pair margin kernel as clusters of 2.
template <int PLANES, int STAGES, int MODE = kModeMargin>
cudaError_t launch_pair(lsx_ctx* ctx, const CUtensorMap& ma, const CUtensorMap& ma2, const CUtensorMap& mb,
                        const CUtensorMap& mea, const CUtensorMap& meb, const ReadoutParams& p) {
    auto k = readout_pair_kernel<PLANES, STAGES, MODE>;
    const size_t smem = pair_smem<PLANES, STAGES>();
    cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int m_pairs = (p.M + kPairRows - 1) / kPairRows;
    const int total = m_pairs * p.n_tiles * (MODE == kModeStore && p.ksplits > 1 ? p.ksplits : 1);
    const int pairs = std::max(1, std::min(total, ctx->sm_count / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kReadoutThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, ma, ma2, mb, mea, meb, p);
}

}  // namespace

// The few-row store GEMM (few_rows_kernel): K slices chosen so the (tile, slice)
// items cover the SMs in whole waves, the cost being waves x K blocks per item
// with a small charge per extra slice for the partial planes and their reduce.
int few_rows_enqueue(lsx_ctx* ctx, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int M, int K,
                     const __nv_bfloat16* w, int N, const float* bias, float* out, int ldo, bool accumulate,
                     int* status) {
    const int Mp = M <= 16 ? 16 : 32;
    CUtensorMap mw, mhi, mlo;
    LSX_TRY(make_map(&mw, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, 128));
    LSX_TRY(make_map(&mhi, a_hi, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, (uint32_t)Mp));
    LSX_TRY(make_map(&mlo, a_lo, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, (uint32_t)Mp));
    FewParams p{};
    p.M = M;
    p.Mp = Mp;
    p.N = N;
    p.k_blocks = (K + RK - 1) / RK;
    p.n_tiles = (N + 127) / 128;
    p.bias = bias;
    p.out = out;
    p.ldo = ldo;
    p.accumulate = accumulate ? 1 : 0;
    p.status = status;
    const int G = ctx->sm_count;
    int best_ks = 1;
    double best_cost = 1e300;
    for (int ks = 1; ks <= 16 && ks <= std::max(1, p.k_blocks / 2); ++ks) {
        const double waves = std::ceil((double)p.n_tiles * ks / G);
        const double cost = waves * std::ceil((double)p.k_blocks / ks) * (1.0 + 0.03 * (ks - 1));
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best_ks = ks;
        }
    }
    if (const char* v = getenv("LSX_FEW_ROWS_SPLITS")) best_ks = std::max(1, std::min(16, atoi(v)));
    p.ksplits = best_ks;
    const int stage_bytes = 128 * RK * 2 + 2 * Mp * RK * 2;
    const size_t fixed = 1024 + 8 * 8 * 2 + 64;
    p.stages = (int)std::min<size_t>(8, (ctx->smem_optin - fixed) / stage_bytes);
    LSX_ENSURE(p.stages >= 2, "few-row GEMM: shared memory");
    const size_t smem = (size_t)p.stages * stage_bytes + 1024 + (2 * p.stages + 4) * 8 + 16;
    void* part = nullptr;
    if (p.ksplits > 1) {
        LSX_TRY(device_alloc(ctx, (size_t)p.ksplits * M * N * 4, &part));
        p.partial = (float*)part;
    }
    cudaError_t e = cudaFuncSetAttribute((const void*)few_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e == cudaSuccess) {
        // as a programmatic dependent of the kernel before it: the weight tiles stream
        // while that kernel finishes (the activations are read after it completes)
        const int items = p.n_tiles * p.ksplits;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(std::min(items, G));
        cfg.blockDim = dim3(kFewThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = ctx->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, few_rows_kernel, mw, mhi, mlo, p);
    }
    if (e == cudaSuccess && p.ksplits > 1) {
        // the in-order sum of the slices, launched as a programmatic dependent so its
        // launch overlaps the GEMM's tail (it waits for the GEMM before reading)
        const size_t total = (size_t)M * N;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)std::min<size_t>((total + 255) / 256, 4096));
        cfg.blockDim = dim3(256);
        cfg.stream = ctx->stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, split_reduce_kernel, (const float*)part, p.ksplits, M, N, bias, out, ldo,
                               accumulate ? 1 : 0, status);
    }
    if (part) device_release(ctx, part);  // stream-ordered: later users of the block run after the reduce
    LSX_CUDA(e, "few-row GEMM launch");
    return LSX_OK;
}

// out[M, ldo] (=|+=) (A_hi + A_lo) W^T (+ bias) on the tensor cores: A as two bf16
// planes [M, K] (an f32 operand split hi/lo), W bf16 [N, K]; f32 accumulate.
// status[0] receives a device error code, status[1] the non-finite flag.
int gemm_planes_enqueue(lsx_ctx* ctx, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int M, int K,
                        const __nv_bfloat16* w, int N, const float* bias, float* out, int ldo, bool accumulate,
                        int* status) {
    LSX_ENSURE(M > 0 && N > 0 && K > 0 && K % 8 == 0 && ldo >= N, "check the GEMM dimensions");
    CUtensorMap ma, ma2, mb;
    LSX_TRY(make_map(&ma, a_hi, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, RM));
    LSX_TRY(make_map(&ma2, a_lo, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, RM));
    LSX_TRY(make_map(&mb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, RN));
    ReadoutParams p{};
    p.M = M;
    p.V = N;
    p.H = K;
    p.k_blocks = (K + RK - 1) / RK;
    p.ext_blocks = 0;
    p.m_tiles = (M + RM - 1) / RM;
    p.n_tiles = (N + RN - 1) / RN;
    p.bias = bias;
    p.status = status;
    p.out = out;
    p.ldo = ldo;
    p.accumulate = accumulate ? 1 : 0;
    // A batched decode step (a few activation rows): the weight as the 128-row
    // operand (LSX_GEMM_FEW_ROWS=0 keeps the CTA-pair path).
    const char* few = getenv("LSX_GEMM_FEW_ROWS");
    if (M <= kFewMaxRows && !(few && few[0] == '0'))
        return few_rows_enqueue(ctx, a_hi, a_lo, M, K, w, N, bias, out, ldo, accumulate, status);
    const char* single = getenv("LSX_GEMM_SINGLE");
    if (!(single && single[0] == '1') && ctx->sm_count >= 2) {
        // CTA pairs (cta_group::2): each CTA loads half of the weight tile
        CUtensorMap mbh;
        LSX_TRY(make_map(&mbh, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, kHalfN));
        // Few rows (a batched decode step): too few output tiles to occupy the
        // pairs, so the K loop is split over otherwise idle pairs and the slices'
        // products are summed in order afterwards.
        const int pairs = ctx->sm_count / 2;
        const int tiles = ((M + kPairRows - 1) / kPairRows) * p.n_tiles;
        const int ksplits = tiles * 2 <= pairs ? std::min(std::min(pairs / tiles, p.k_blocks / 4), 16) : 1;
        if (ksplits > 1) {
            const size_t bytes = (size_t)ksplits * M * N * 4;
            void* part = nullptr;
            LSX_TRY(device_alloc(ctx, bytes, &part));
            p.ksplits = ksplits;
            p.partial = (float*)part;
            cudaError_t e = launch_pair<2, 4, kModeStore>(ctx, ma, ma2, mbh, ma, mbh, p);
            if (e == cudaSuccess) {
                const size_t total = (size_t)M * N;
                split_reduce_kernel<<<(int)std::min<size_t>((total + 255) / 256, 4096), 256, 0, ctx->stream>>>(
                    (const float*)part, ksplits, M, N, bias, out, ldo, accumulate ? 1 : 0, status);
                e = cudaGetLastError();
            }
            device_release(ctx, part);  // stream-ordered: later users of the block run after the reduce
            LSX_CUDA(e, "split GEMM launch");
            return LSX_OK;
        }
        LSX_CUDA((launch_pair<2, 4, kModeStore>(ctx, ma, ma2, mbh, ma, mbh, p)), "GEMM launch");
        return LSX_OK;
    }
    auto k = readout_margin_kernel<2, 3, kModeStore>;
    const size_t smem = readout_smem<2, 3>();
    LSX_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
             "GEMM smem attribute");
    const int total = p.m_tiles * p.n_tiles;
    k<<<std::min(total, ctx->sm_count), kReadoutThreads, smem, ctx->stream>>>(ma, ma2, mb, ma, mb, p);
    LSX_CUDA(cudaGetLastError(), "GEMM launch");
    return LSX_OK;
}

// The gate/up GEMM with the gated product in its epilogue: out_hi / out_lo
// [M, N / 2] receive act(gate) * up as the next GEMM's bf16 A planes (the columns
// of W are interleaved (gate, up) rows), so the f32 [M, N] product is never
// written.  Only the CTA-pair and single-CTA paths without a K split carry the
// gated epilogue: *fused is false (and nothing is enqueued) for the shapes that
// would take the few-row or split path, and the caller runs the two-kernel form.
int gemm_gated_enqueue(lsx_ctx* ctx, const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, int M, int K,
                       const __nv_bfloat16* w, int N, const float* bias, int act_kind, __nv_bfloat16* out_hi,
                       __nv_bfloat16* out_lo, int* status, bool* fused) {
    LSX_ENSURE(fused != nullptr, "check the GEMM arguments");
    *fused = false;
    LSX_ENSURE(M > 0 && N > 0 && K > 0 && K % 8 == 0 && N % 2 == 0, "check the GEMM dimensions");
    const char* few = getenv("LSX_GEMM_FEW_ROWS");
    if (M <= kFewMaxRows && !(few && few[0] == '0')) return LSX_OK;
    if (const char* g = getenv("LSX_GEMM_GATED")) {
        if (g[0] == '0') return LSX_OK;
    }
    if ((uintptr_t)out_hi % 16 != 0 || (uintptr_t)out_lo % 16 != 0) return LSX_OK;
    const char* single = getenv("LSX_GEMM_SINGLE");
    const bool pair = !(single && single[0] == '1') && ctx->sm_count >= 2;
    const int n_tiles = (N + RN - 1) / RN;
    if (pair) {
        const int pairs = ctx->sm_count / 2, k_blocks = (K + RK - 1) / RK;
        const int tiles = ((M + kPairRows - 1) / kPairRows) * n_tiles;
        const int ksplits = tiles * 2 <= pairs ? std::min(std::min(pairs / tiles, k_blocks / 4), 16) : 1;
        if (ksplits > 1) return LSX_OK;
    }
    CUtensorMap ma, ma2, mb;
    LSX_TRY(make_map(&ma, a_hi, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, RM));
    LSX_TRY(make_map(&ma2, a_lo, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, RM));
    LSX_TRY(make_map(&mb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, RN));
    ReadoutParams p{};
    p.M = M;
    p.V = N;
    p.H = K;
    p.k_blocks = (K + RK - 1) / RK;
    p.ext_blocks = 0;
    p.m_tiles = (M + RM - 1) / RM;
    p.n_tiles = n_tiles;
    p.bias = bias;
    p.status = status;
    p.out = nullptr;
    p.ldo = N;
    p.accumulate = 0;
    p.ksplits = 1;
    p.gated = act_kind + 1;
    p.g_hi = out_hi;
    p.g_lo = out_lo;
    p.ldg = N / 2;
    if (pair) {
        CUtensorMap mbh;
        LSX_TRY(make_map(&mbh, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, kHalfN));
        LSX_CUDA((launch_pair<2, 4, kModeStore>(ctx, ma, ma2, mbh, ma, mbh, p)), "gated GEMM launch");
    } else {
        auto k = readout_margin_kernel<2, 3, kModeStore>;
        const size_t smem = readout_smem<2, 3>();
        LSX_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "GEMM smem attribute");
        const int total = p.m_tiles * p.n_tiles;
        k<<<std::min(total, ctx->sm_count), kReadoutThreads, smem, ctx->stream>>>(ma, ma2, mb, ma, mb, p);
        LSX_CUDA(cudaGetLastError(), "gated GEMM launch");
    }
    *fused = true;
    return LSX_OK;
}

// Workspace bytes readout_margin_enqueue needs for exactly this hidden dtype.
size_t readout_workspace_need(size_t vocab, size_t width, size_t rows, size_t rank, bool f32_hidden) {
    return layout_for(vocab, width, rows, rank, f32_hidden).total;
}

int image_f32_enqueue(lsx_ctx* ctx, const void* a, size_t rows, size_t width, const float* dirs, size_t count,
                      float* out, bool accumulate, __nv_bfloat16* split, int* status);

// One vocabulary shard's outputs: per-row partials instead of margins.
struct ShardOut {
    size_t vocab_offset;
    unsigned long long* other_key;
    float* target_logit;
    long long* partials;  // packed form [2 x rows] (other_key and target_logit unused), or NULL
};

// Enqueues the whole validation on ctx->stream.  All pointers are device pointers.
// With `shard`, `weight` holds lm_head rows [vocab_offset, vocab_offset + vocab),
// targets are global ids, and the per-row partials land in the shard's buffers
// (no finalize).
int readout_enqueue(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab, size_t width,
                    const void* hidden, int hidden_kind, size_t rows, const uint32_t* targets,
                    const lsx_rotation* rotation, double* margin, uint32_t* argmax, float* target_logit,
                    void* workspace, size_t workspace_bytes, int* host_status, const ShardOut* shard) {
    LSX_ENSURE(weight && weight->kind == LSX_BF16, "the readout weight must be a BF16 tensor");
    LSX_ENSURE(vocab > 1 && width > 0 && weight->count == vocab * width, "check the readout weight dimensions");
    LSX_ENSURE(!bias || (bias->kind == LSX_F32 && bias->count == vocab), "the readout bias is F32 [vocab]");
    LSX_ENSURE(hidden_kind == LSX_F32 || hidden_kind == LSX_BF16, "hidden states are F32 or BF16");
    LSX_ENSURE(rows > 0 && rows <= 2147483647ull && vocab <= 2147483647ull, "check the row count");
    LSX_ENSURE(width % 8 == 0, "the readout width must be a multiple of 8");
    if (rotation) LSX_ENSURE(rotation->width == width, "the rotation width does not match the readout");
    if (rotation) LSX_ENSURE(rotation->rank >= 1 && rotation->rank <= (size_t)kMaxEditRank, "the edit rank is 1..256");
    LSX_ENSURE((uintptr_t)hidden % 16 == 0, "hidden states must be 16-byte aligned");
    const size_t rank = rotation ? rotation->rank : 0;
    const bool f32_hidden = hidden_kind == LSX_F32;
    Layout L = layout_for(vocab, width, rows, rank, f32_hidden);
    LSX_ENSURE(workspace && workspace_bytes >= L.total, "the readout workspace is too small");
    uint8_t* ws = (uint8_t*)workspace;
    cudaStream_t s = ctx->stream;
    int* status = (int*)(ws + L.status_off);
    const bool packed = shard && shard->partials;
    unsigned long long* keys = packed  ? (unsigned long long*)shard->partials
                               : shard ? shard->other_key
                                       : (unsigned long long*)(ws + L.key_off);
    float* tlog = shard && !packed ? shard->target_logit : (float*)(ws + L.tlog_off);
    if (shard)
        LSX_ENSURE(shard->vocab_offset + vocab <= 2147483647ull, "check the vocabulary shard range");
    __nv_bfloat16* plane_hi = f32_hidden ? (__nv_bfloat16*)(ws + L.planes_off) : nullptr;
    __nv_bfloat16* plane_lo = f32_hidden ? plane_hi + rows * width : nullptr;
    __nv_bfloat16* ext_a = (__nv_bfloat16*)(ws + L.ext_a_off);
    __nv_bfloat16* ext_b = (__nv_bfloat16*)(ws + L.ext_b_off);
    const int M = (int)rows, V = (int)vocab, H = (int)width;

    readout_init_kernel<<<(M + 255) / 256, 256, 0, s>>>(keys, tlog, M, status, shard != nullptr);
    LSX_CUDA(cudaGetLastError(), "readout init");
    if (rank > 0) {
        // Edit basis and R - I in f32: the rotation's device copies when it lives
        // on this device, else uploaded from its f64 host copies.
        const float* dbasis;
        const float* ddelta;
        if (rotation->basis && rotation->delta && rotation->ctx && rotation->ctx->device == ctx->device) {
            dbasis = (const float*)rotation->basis->data;
            ddelta = (const float*)rotation->delta->data;
        } else {
            std::vector<float> b(rank * width), d(rank * rank);
            for (size_t i = 0; i < b.size(); ++i) b[i] = (float)rotation->basis64[i];
            for (size_t i = 0; i < d.size(); ++i) d[i] = (float)rotation->delta64[i];
            float* ub = (float*)(ws + L.basis_off);
            float* ud = (float*)(ws + L.delta_off);
            LSX_CUDA(cudaMemcpyAsync(ub, b.data(), b.size() * 4, cudaMemcpyHostToDevice, s), "edit upload");
            LSX_CUDA(cudaMemcpyAsync(ud, d.data(), d.size() * 4, cudaMemcpyHostToDevice, s), "edit upload");
            LSX_CUDA(cudaStreamSynchronize(s), "edit upload");  // host vectors go out of scope
            dbasis = ub;
            ddelta = ud;
        }
        // F = W U^T on the tensor cores, up to kImageRanks ranks per pass; the
        // passes also write the extension block's zero padding.
        __nv_bfloat16* image_a = (__nv_bfloat16*)(ws + L.image_a_off);
        CUtensorMap mw;
        LSX_TRY(make_map(&mw, weight->data, width, vocab, width * 2, kImageM));
        const int n_tiles = (V + kImageM - 1) / kImageM;
        for (int k0 = 0; k0 < (int)rank; k0 += kImageRanks) {
            const int kc = std::min(kImageRanks, (int)rank - k0);
            basis_split_kernel<<<std::min(ctx->sm_count, (kc * H + 255) / 256), 256, 0, s>>>(dbasis, H, k0, kc,
                                                                                           image_a);
            LSX_CUDA(cudaGetLastError(), "edit basis split");
            ImageParams q{};
            q.V = V;
            q.k_blocks = (H + RK - 1) / RK;
            q.n_tiles = n_tiles;
            q.np = ((2 * kc + 31) / 32) * 32;
            q.rank = (int)rank;
            q.k0 = k0;
            q.kc = kc;
            q.ext_k = (int)L.ext_k;
            q.image = ext_b;
            q.status = status;
            const int stage_bytes = kImageM * RK * 2 + q.np * RK * 2;
            q.stages = std::min(8, (int)((200u << 10) / stage_bytes));
            const size_t ismem = (size_t)q.stages * stage_bytes + 1024 + (2 * q.stages + 4) * 8 + 16;
            CUtensorMap mu;
            LSX_TRY(make_map(&mu, image_a, width, 2 * (size_t)kc, width * 2, (uint32_t)q.np));
            LSX_CUDA(cudaFuncSetAttribute((const void*)edit_image_kernel<kImageExtension>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ismem),
                     "edit image smem attribute");
            edit_image_kernel<kImageExtension>
                <<<std::min(n_tiles, ctx->sm_count), kImageThreads, ismem, s>>>(mw, mu, q);
            LSX_CUDA(cudaGetLastError(), "edit image");
        }
        // Edit coordinates U h of every row ([rank, M] f32) on the tensor cores: the
        // rows (bf16, or the hi and lo planes of f32 rows) against U as exact
        // three-term bf16 directions.
        float* coords = (float*)(ws + L.coords_off);
        __nv_bfloat16* split = (__nv_bfloat16*)(ws + L.image_a_off);
        if (f32_hidden) {
            edit_coefficients_kernel<<<(M + 7) / 8, 256, 0, s>>>(hidden, hidden_kind, M, H, nullptr, nullptr, 0,
                                                                 nullptr, 0, plane_hi, plane_lo);
            LSX_CUDA(cudaGetLastError(), "hidden split");
            LSX_TRY(image_f32_enqueue(ctx, plane_hi, rows, width, dbasis, rank, coords, false, split, status));
            LSX_TRY(image_f32_enqueue(ctx, plane_lo, rows, width, dbasis, rank, coords, true, split, status));
        } else {
            LSX_TRY(image_f32_enqueue(ctx, hidden, rows, width, dbasis, rank, coords, false, split, status));
        }
        edit_coefficients_kernel<<<(M + 7) / 8, 256, 0, s>>>(hidden, hidden_kind, M, H, coords, ddelta, (int)rank,
                                                             ext_a, (int)L.ext_k, nullptr, nullptr);
        LSX_CUDA(cudaGetLastError(), "edit coefficients");
    } else if (f32_hidden) {
        edit_coefficients_kernel<<<(M + 7) / 8, 256, 0, s>>>(hidden, hidden_kind, M, H, nullptr, nullptr, 0, nullptr,
                                                             0, plane_hi, plane_lo);
        LSX_CUDA(cudaGetLastError(), "hidden split");
    }

    CUtensorMap ma, ma2, mb, mea, meb;
    const void* a_base = f32_hidden ? (const void*)plane_hi : hidden;
    LSX_TRY(make_map(&ma, a_base, width, rows, width * 2, RM));
    LSX_TRY(make_map(&ma2, f32_hidden ? (const void*)plane_lo : a_base, width, rows, width * 2, RM));
    LSX_TRY(make_map(&mb, weight->data, width, vocab, width * 2, RN));
    if (rank > 0) {
        LSX_TRY(make_map(&mea, ext_a, L.ext_k, rows, L.ext_k * 2, RM));
        LSX_TRY(make_map(&meb, ext_b, L.ext_k, vocab, L.ext_k * 2, RN));
    } else {
        mea = ma;
        meb = mb;
    }
    ReadoutParams p{};
    p.M = M;
    p.V = V;
    p.H = H;
    p.k_blocks = (H + RK - 1) / RK;
    p.ext_blocks = (int)(L.ext_k / RK);
    p.m_tiles = (M + RM - 1) / RM;
    p.n_tiles = (V + RN - 1) / RN;
    p.targets = targets;
    p.vocab_offset = shard ? (int)shard->vocab_offset : 0;
    p.bias = bias ? (const float*)bias->data : nullptr;
    p.other_key = keys;
    p.target_logit = tlog;
    p.status = status;
    const int total = p.m_tiles * p.n_tiles;
    const int grid = std::min(total, ctx->sm_count);
    // CTA pairs (cta_group::2) unless LSX_READOUT_SINGLE=1 asks for one CTA per tile.
    const char* single = getenv("LSX_READOUT_SINGLE");
    if (!(single && single[0] == '1') && ctx->sm_count >= 2) {
        CUtensorMap mbh, mebh;
        LSX_TRY(make_map(&mbh, weight->data, width, vocab, width * 2, kHalfN));
        if (rank > 0) LSX_TRY(make_map(&mebh, ext_b, L.ext_k, vocab, L.ext_k * 2, kHalfN));
        else mebh = mbh;
        cudaError_t e = f32_hidden ? launch_pair<2, 4>(ctx, ma, ma2, mbh, mea, mebh, p)
                                   : launch_pair<1, 6>(ctx, ma, ma2, mbh, mea, mebh, p);
        LSX_CUDA(e, "readout margin launch");
    } else if (f32_hidden) {
        auto k = readout_margin_kernel<2, 3, kModeMargin>;
        size_t smem = readout_smem<2, 3>();
        LSX_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "readout smem attribute");
        k<<<grid, kReadoutThreads, smem, s>>>(ma, ma2, mb, mea, meb, p);
    } else {  // single CTA per tile
        auto k = readout_margin_kernel<1, 4, kModeMargin>;
        size_t smem = readout_smem<1, 4>();
        LSX_CUDA(cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                 "readout smem attribute");
        k<<<grid, kReadoutThreads, smem, s>>>(ma, ma2, mb, mea, meb, p);
    }
    LSX_CUDA(cudaGetLastError(), "readout margin launch");
    if (!shard) {
        readout_finalize_kernel<<<(M + 255) / 256, 256, 0, s>>>(keys, tlog, targets, M, margin, argmax, target_logit);
        LSX_CUDA(cudaGetLastError(), "readout finalize");
    } else if (packed) {
        shard_pack_kernel<<<(M + 255) / 256, 256, 0, s>>>(shard->partials, tlog, M);
        LSX_CUDA(cudaGetLastError(), "shard partials pack");
    }
    if (host_status) {
        LSX_CUDA(cudaMemcpyAsync(host_status, status, 8, cudaMemcpyDeviceToHost, s), "status download");
    }
    return LSX_OK;
}

// Device scratch head_images_enqueue needs for `count` directions of width H.
size_t head_images_scratch(size_t count, size_t width) {
    return align256(count * width * 4) + align256((size_t)kImageMaxN * width * 2) + 256;
}

// out[k, :] (=|+=) A u_k in f32 for the f32 directions dirs [count, width] (device):
// one tcgen05 pass over A (BF16 [rows, width]) per 32 directions (kImageF32);
// `split` holds kImageMaxN x width bf16 for the split directions.  Enqueued only.
int image_f32_enqueue(lsx_ctx* ctx, const void* a, size_t rows, size_t width, const float* dirs, size_t count,
                      float* out, bool accumulate, __nv_bfloat16* split, int* status) {
    LSX_ENSURE(count > 0 && width % 8 == 0 && rows > 0 && rows <= 2147483647ull, "check the image sizes");
    cudaStream_t s = ctx->stream;
    CUtensorMap mw;
    LSX_TRY(make_map(&mw, a, width, rows, width * 2, kImageM));
    const int V = (int)rows, H = (int)width;
    const int n_tiles = (V + kImageM - 1) / kImageM;
    constexpr int kDirs = kImageMaxN / 4;  // directions per pass
    for (int k0 = 0; k0 < (int)count; k0 += kDirs) {
        const int kc = std::min(kDirs, (int)count - k0);
        direction_split_kernel<<<std::min(ctx->sm_count, (kc * H + 255) / 256), 256, 0, s>>>(dirs, H, k0, kc, split);
        LSX_CUDA(cudaGetLastError(), "direction split");
        ImageParams q{};
        q.V = V;
        q.k_blocks = (H + RK - 1) / RK;
        q.n_tiles = n_tiles;
        q.np = ((4 * kc + 31) / 32) * 32;
        q.rank = (int)count;
        q.k0 = k0;
        q.kc = kc;
        q.out = out;
        q.accumulate = accumulate ? 1 : 0;
        q.status = status;
        const int stage_bytes = kImageM * RK * 2 + q.np * RK * 2;
        q.stages = std::min(8, (int)((200u << 10) / stage_bytes));
        const size_t ismem = (size_t)q.stages * stage_bytes + 1024 + (2 * q.stages + 4) * 8 + 16;
        CUtensorMap mu;
        LSX_TRY(make_map(&mu, split, width, 4 * (size_t)kc, width * 2, (uint32_t)q.np));
        LSX_CUDA(cudaFuncSetAttribute((const void*)edit_image_kernel<kImageF32>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ismem),
                 "image smem attribute");
        edit_image_kernel<kImageF32><<<std::min(n_tiles, ctx->sm_count), kImageThreads, ismem, s>>>(mw, mu, q);
        LSX_CUDA(cudaGetLastError(), "f32 image");
    }
    return LSX_OK;
}

// out[k, :] = W u_k (f32) for the f32 directions dirs_host [count, width]: one
// tcgen05 pass over W per 32 directions (kImageF32).  W is BF16 [vocab, width].
// Runs on ctx->stream and waits for it; `scratch` holds head_images_scratch() bytes.
int head_images_enqueue(lsx_ctx* ctx, const lsx_tensor* weight, size_t vocab, size_t width, const float* dirs_host,
                        size_t count, float* out, void* scratch) {
    LSX_ENSURE(weight && weight->kind == LSX_BF16 && weight->count == vocab * width, "the head weight must be BF16");
    LSX_ENSURE(count > 0 && count <= 4096 && width % 8 == 0 && vocab <= 2147483647ull, "check the head image sizes");
    uint8_t* b = (uint8_t*)scratch;
    float* dirs = (float*)b;
    __nv_bfloat16* split = (__nv_bfloat16*)(b + align256(count * width * 4));
    int* status = (int*)(b + align256(count * width * 4) + align256((size_t)kImageMaxN * width * 2));
    cudaStream_t s = ctx->stream;
    LSX_CUDA(cudaMemcpyAsync(dirs, dirs_host, count * width * 4, cudaMemcpyHostToDevice, s), "direction upload");
    LSX_CUDA(cudaMemsetAsync(status, 0, 8, s), "status clear");
    LSX_TRY(image_f32_enqueue(ctx, weight->data, vocab, width, dirs, count, out, false, split, status));
    int host_status[2] = {0, 0};
    LSX_CUDA(cudaMemcpyAsync(host_status, status, 8, cudaMemcpyDeviceToHost, s), "status download");
    LSX_CUDA(cudaStreamSynchronize(s), "head images");
    if (host_status[0] != 0)
        return fail(LSX_E_CUDA, "head image kernel reported status " + std::to_string(host_status[0]));
    return LSX_OK;
}

int fixed_scratch_address(lsx_ctx* ctx, void** out);

int readout_margin_enqueue(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab, size_t width,
                           const void* hidden, int hidden_kind, size_t rows, const uint32_t* targets,
                           const lsx_rotation* rotation, double* margin, uint32_t* argmax, float* target_logit,
                           void* workspace, size_t workspace_bytes, int* host_status) {
    return readout_enqueue(ctx, weight, bias, vocab, width, hidden, hidden_kind, rows, targets, rotation, margin,
                           argmax, target_logit, workspace, workspace_bytes, host_status, nullptr);
}

}  // namespace lsx

using namespace lsx;

extern "C" {

int lsx_readout_shard_device(lsx_ctx* ctx, const lsx_tensor* weight_shard, const lsx_tensor* bias_shard,
                             size_t vocab_offset, size_t shard_vocab, size_t width, const void* hidden,
                             lsx_dtype hidden_kind, size_t rows, const uint32_t* targets,
                             const lsx_rotation* rotation, uint64_t* other_key_out, float* target_logit_out,
                             void* workspace, size_t workspace_bytes) {
    LSX_ENSURE(ctx && hidden && targets && other_key_out && target_logit_out, "invalid argument");
    cudaSetDevice(ctx->device);
    const ShardOut shard{vocab_offset, (unsigned long long*)other_key_out, target_logit_out, nullptr};
    return readout_enqueue(ctx, weight_shard, bias_shard, shard_vocab, width, hidden, hidden_kind, rows, targets,
                           rotation, nullptr, nullptr, nullptr, workspace, workspace_bytes, nullptr, &shard);
}

int lsx_readout_partials_device(lsx_ctx* ctx, const lsx_tensor* weight_shard, const lsx_tensor* bias_shard,
                                size_t vocab_offset, size_t shard_vocab, size_t width, const void* hidden,
                                lsx_dtype hidden_kind, size_t rows, const uint32_t* targets,
                                const lsx_rotation* rotation, int64_t* partials, void* workspace,
                                size_t workspace_bytes) {
    LSX_ENSURE(ctx && hidden && targets && partials, "invalid argument");
    LSX_ENSURE(rows > 0 && rows <= 1073741823ull, "check the row count");  // 2 x rows indexes an int
    LSX_CUDA(cudaSetDevice(ctx->device), "select device");
    const ShardOut shard{vocab_offset, nullptr, nullptr, (long long*)partials};
    return readout_enqueue(ctx, weight_shard, bias_shard, shard_vocab, width, hidden, hidden_kind, rows, targets,
                           rotation, nullptr, nullptr, nullptr, workspace, workspace_bytes, nullptr, &shard);
}

int lsx_readout_partials_merge_device(lsx_ctx* ctx, const int64_t* partials, const uint32_t* targets, size_t rows,
                                      double* margin_out, uint32_t* argmax_out, float* target_logit_out) {
    LSX_ENSURE(ctx && partials && targets, "invalid argument");
    LSX_ENSURE(rows > 0 && rows <= 1073741823ull, "check the row count");
    LSX_CUDA(cudaSetDevice(ctx->device), "select device");
    const int M = (int)rows;
    shard_merge_kernel<<<(M + 255) / 256, 256, 0, ctx->stream>>>((const long long*)partials, targets, M, margin_out,
                                                                 argmax_out, target_logit_out);
    LSX_CUDA(cudaGetLastError(), "shard partials merge");
    return LSX_OK;
}

int lsx_readout_merge_device(lsx_ctx* ctx, const uint64_t* other_key, const float* target_logit,
                             const uint32_t* targets, size_t rows, double* margin_out, uint32_t* argmax_out,
                             float* target_logit_out) {
    LSX_ENSURE(ctx && other_key && target_logit && targets, "invalid argument");
    LSX_ENSURE(rows > 0 && rows <= 2147483647ull, "check the row count");
    cudaSetDevice(ctx->device);
    const int M = (int)rows;
    readout_finalize_kernel<<<(M + 255) / 256, 256, 0, ctx->stream>>>((const unsigned long long*)other_key,
                                                                      target_logit, targets, M, margin_out,
                                                                      argmax_out, target_logit_out);
    LSX_CUDA(cudaGetLastError(), "readout merge");
    return LSX_OK;
}

int lsx_compact_margin(lsx_ctx* ctx, const lsx_tensor* image, const lsx_tensor* baseline, size_t vocab,
                       size_t rank, size_t count, const float* coefficients, const uint32_t* targets,
                       double* margin_out, uint32_t* other_out, uint32_t* argmax_out) {
    LSX_ENSURE(ctx && image && baseline && coefficients && targets, "invalid argument");
    LSX_ENSURE(image->kind == LSX_F32 && baseline->kind == LSX_F32, "the compact image and baselines are F32");
    LSX_ENSURE(rank >= 1 && rank <= (size_t)kMaxEditRank && vocab > 1 && vocab <= 2147483647ull && count > 0 &&
                   count <= 2147483647ull,
               "check the compact readout sizes");
    LSX_ENSURE(image->count == vocab * rank && baseline->count == count * vocab,
               "check the compact image and baseline dimensions");
    for (size_t i = 0; i < count; ++i) LSX_ENSURE(targets[i] < vocab, "check the target token range");
    for (size_t i = 0; i < count * rank; ++i)
        LSX_ENSURE(std::isfinite(coefficients[i]), "check the finiteness of the compact coefficients");
    cudaSetDevice(ctx->device);
    const size_t n = count;
    const size_t total = align256(n * rank * 4) + align256(n * 4) + align256(n * 8) + align256(n * 4) +
                         align256(n * 8) + align256(n * 4) + align256(n * 4) + 256;
    void* block = nullptr;
    LSX_TRY(device_alloc(ctx, total, &block));
    uint8_t* b = (uint8_t*)block;
    size_t at = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = b + at;
        at += align256(bytes);
        return p;
    };
    float* d_coef = (float*)take(n * rank * 4);
    uint32_t* d_targets = (uint32_t*)take(n * 4);
    unsigned long long* d_keys = (unsigned long long*)take(n * 8);
    float* d_tlog = (float*)take(n * 4);
    double* d_margin = (double*)take(n * 8);
    uint32_t* d_other = (uint32_t*)take(n * 4);
    uint32_t* d_argmax = (uint32_t*)take(n * 4);
    int* d_status = (int*)take(16);
    cudaStream_t s = ctx->stream;
    int status[2] = {0, 0};
    cudaError_t e = cudaMemcpyAsync(d_coef, coefficients, n * rank * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_targets, targets, n * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        readout_init_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(d_keys, d_tlog, (int)n, d_status, false);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        const int V = (int)vocab;
        dim3 grid((unsigned)std::min<size_t>((vocab + kCompactThreads * 4 - 1) / (kCompactThreads * 4), 4096),
                  (unsigned)((n + kCompactObs - 1) / kCompactObs));
        compact_margin_kernel<<<grid, kCompactThreads, 0, s>>>((const float*)image->data,
                                                              (const float*)baseline->data, d_coef, d_targets, V,
                                                              (int)rank, (int)n, d_keys, d_tlog, d_status);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        readout_finalize_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(d_keys, d_tlog, d_targets, (int)n, d_margin,
                                                                      d_argmax, nullptr, d_other);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && margin_out) e = cudaMemcpyAsync(margin_out, d_margin, n * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && other_out) e = cudaMemcpyAsync(other_out, d_other, n * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && argmax_out) e = cudaMemcpyAsync(argmax_out, d_argmax, n * 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(status, d_status, 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    device_release(ctx, block);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("compact readout", e));
    if (status[1] != 0) return fail(LSX_E_NONFINITE, "check the finite scores of the compact readout");
    return LSX_OK;
}

int lsx_readout_status(lsx_ctx* ctx, const void* workspace) {
    LSX_ENSURE(ctx, "invalid argument");
    LSX_CUDA(cudaSetDevice(ctx->device), "select device");
    const void* words = workspace;
    if (!words) {
        void* fixed = nullptr;
        LSX_TRY(fixed_scratch_address(ctx, &fixed));
        words = fixed;
    }
    int status[2] = {0, 0};
    LSX_CUDA(cudaMemcpyAsync(status, words, 8, cudaMemcpyDeviceToHost, ctx->stream), "readout status download");
    LSX_CUDA(cudaStreamSynchronize(ctx->stream), "readout status");
    if (status[0] != 0) return fail(LSX_E_CUDA, "readout kernel reported status " + std::to_string(status[0]));
    if (status[1] != 0) return fail(LSX_E_NONFINITE, "check the finiteness of the readout scores");
    return LSX_OK;
}

size_t lsx_readout_workspace_bytes(size_t vocab, size_t width, size_t rows, const lsx_rotation* rotation) {
    // Sized for F32 hidden states (the larger case).
    return layout_for(vocab, width, rows, rotation ? rotation->rank : 0, true).total;
}

int lsx_readout_margin_device(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab,
                              size_t width, const void* hidden, lsx_dtype hidden_kind, size_t rows,
                              const uint32_t* targets, const lsx_rotation* rotation, double* margin_out,
                              uint32_t* argmax_out, float* target_logit_out, void* workspace,
                              size_t workspace_bytes) {
    LSX_ENSURE(ctx && hidden && targets, "invalid argument");
    cudaSetDevice(ctx->device);
    return readout_margin_enqueue(ctx, weight, bias, vocab, width, hidden, hidden_kind, rows, targets, rotation,
                                  margin_out, argmax_out, target_logit_out, workspace, workspace_bytes, nullptr);
}

int lsx_readout_margin(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab, size_t width,
                       const void* hidden, lsx_dtype hidden_kind, size_t rows, const uint32_t* targets,
                       const lsx_rotation* rotation, double* margin_out, uint32_t* argmax_out,
                       float* target_logit_out) {
    LSX_ENSURE(ctx && weight && hidden && targets, "invalid argument");
    LSX_ENSURE(hidden_kind == LSX_F32 || hidden_kind == LSX_BF16, "hidden states are F32 or BF16");
    LSX_ENSURE(rows > 0 && vocab > 1, "check the row count");
    for (size_t i = 0; i < rows; ++i) LSX_ENSURE(targets[i] < vocab, "check the target token range");
    cudaSetDevice(ctx->device);
    const size_t hbytes = rows * width * (hidden_kind == LSX_F32 ? 4 : 2);
    const size_t ws_bytes = lsx_readout_workspace_bytes(vocab, width, rows, rotation);
    const size_t out_bytes = rows * (8 + 4 + 4);
    const size_t total = align256(hbytes) + align256(rows * 4) + align256(out_bytes) + ws_bytes;
    void* block = nullptr;
    LSX_TRY(device_alloc(ctx, total, &block));
    uint8_t* b = (uint8_t*)block;
    void* d_hidden = b;
    uint32_t* d_targets = (uint32_t*)(b + align256(hbytes));
    uint8_t* d_out = b + align256(hbytes) + align256(rows * 4);
    double* d_margin = (double*)d_out;
    uint32_t* d_argmax = (uint32_t*)(d_out + rows * 8);
    float* d_tlog = (float*)(d_out + rows * 12);
    void* ws = d_out + align256(out_bytes);
    cudaStream_t s = ctx->stream;
    int status[2] = {0, 0};
    int rc = LSX_OK;
    rc = staged_upload(ctx, d_hidden, hidden, hbytes);
    cudaError_t e = cudaSuccess;
    if (rc == LSX_OK) e = cudaMemcpyAsync(d_targets, targets, rows * 4, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) rc = fail(LSX_E_CUDA, cuda_message("readout upload", e));
    if (rc == LSX_OK)
        rc = readout_margin_enqueue(ctx, weight, bias, vocab, width, d_hidden, hidden_kind, rows, d_targets, rotation,
                                    d_margin, d_argmax, d_tlog, ws, ws_bytes, status);
    if (rc == LSX_OK) {
        e = cudaSuccess;
        if (margin_out) e = cudaMemcpyAsync(margin_out, d_margin, rows * 8, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess && argmax_out) e = cudaMemcpyAsync(argmax_out, d_argmax, rows * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess && target_logit_out)
            e = cudaMemcpyAsync(target_logit_out, d_tlog, rows * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = fail(LSX_E_CUDA, cuda_message("readout margin", e));
    }
    device_release(ctx, block);
    if (rc != LSX_OK) return rc;
    if (status[0] != 0) return fail(LSX_E_CUDA, "readout kernel reported status " + std::to_string(status[0]));
    if (status[1] != 0) return fail(LSX_E_NONFINITE, "check the finiteness of the readout scores");
    return LSX_OK;
}

}  // extern "C"
