// Plane-candidate feasibility (src/diagnosis.rs:1113-1143, src/interval.rs).
//
// For a plane (u, v) the reference tests every target point against every
// vocabulary entry j: with du = wu[t] - wu[j], dv = wv[t] - wv[j] (wu = W u,
// wv = W v, the head images), alpha = du hv - dv hu, beta = du hu + dv hv and
// c = z[t] - z[j] - margin - guard, the rotation's half-angle tangent t must keep
// (c - 2 beta) t^2 + 2 alpha t + c >= 0.  FeasibleSet merges the forbidden
// intervals on the host, one constraint at a time, and first screens each
// constraint: one that is certainly non-negative on the current hull [left,
// right] (both ends, and the vertex outside or a non-negative discriminant)
// changes nothing and is only counted.  Nearly all of the points x vocab
// constraints are screened, so this is an O(points x vocab) scan on the host.
//
// Here plane_screen_kernel forms every constraint on the GPU in f64 with the
// reference's exact operation order (no contraction; fma only where the
// reference calls mul_add) and evaluates the same screening test against a given
// hull, leaving one bit per (point, j) for the constraints that need the host.
// The host walks the constraints in the reference's order: a screened one is
// counted as the reference counts it; the others are rebuilt on the host
// (bit-identical f64) and merged.  The screening test depends on the hull, so
// whenever a merge moves the hull the kernel rescreens the rest against the new
// one.  The merged set, the nearest tangent and the work counters equal the
// reference's.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <iterator>
#include <map>
#include <vector>

#include "lsx_internal.h"

namespace lsx {
namespace {

// f64::total_cmp order, with equal values (including -0.0 == 0.0) equal: the
// Endpoint key order of src/interval.rs:13-33.
inline long long total_key(double x) {
    long long b;
    std::memcpy(&b, &x, 8);
    return b ^ (long long)((unsigned long long)(b >> 63) >> 1);
}
struct EndpointLess {
    bool operator()(double x, double y) const { return x != y && total_key(x) < total_key(y); }
};

constexpr double kEps8 = 8.0 * 2.220446049250313e-16;  // 8 f64::EPSILON

}  // namespace
}  // namespace lsx

// FeasibleSet (src/interval.rs:47-212).
struct lsx_feasible {
    double bound = 1.0;
    std::map<double, double, lsx::EndpointLess> forbidden;  // lower -> upper of open forbidden intervals
    uint64_t constraints = 0, screened = 0, square_roots = 0, inserted = 0;

    // the interval with the largest key below x, when x lies inside it
    bool containing(double x, double* a, double* b) const {
        auto it = forbidden.lower_bound(x);  // first key >= x
        if (it == forbidden.begin()) return false;
        --it;
        if (x < it->second) {
            *a = it->first;
            *b = it->second;
            return true;
        }
        return false;
    }
    bool hull(double* left, double* right) const {
        double a, b;
        *left = containing(-bound, &a, &b) ? b : -bound;
        *right = containing(bound, &a, &b) ? a : bound;
        return *left <= *right;
    }
    bool empty() const {
        double l, r;
        return !hull(&l, &r);
    }
    void exclude(double a, double b) {
        if (a >= b || b <= -bound || a >= bound) return;
        ++inserted;
        auto it = forbidden.upper_bound(a);  // first key > a; the one before is the largest key <= a
        if (it != forbidden.begin()) {
            auto prev = std::prev(it);
            if (prev->second > a) {
                a = prev->first;
                b = std::fmax(b, prev->second);
                forbidden.erase(prev);
            }
        }
        for (auto next = forbidden.lower_bound(a); next != forbidden.end() && !(next->first >= b);
             next = forbidden.lower_bound(a)) {
            b = std::fmax(b, next->second);
            forbidden.erase(next);
        }
        forbidden[a] = b;
    }
    // FeasibleSet::constrain; false for non-finite coefficients.
    bool constrain(double a, double b, double c) {
        if (!(std::isfinite(a) && std::isfinite(b) && std::isfinite(c))) return false;
        ++constraints;
        double left, right;
        if (!hull(&left, &right)) return true;
        const double magnitude = std::fmax(std::fmax(std::fabs(a), std::fabs(b)), std::fabs(c));
        if (magnitude == 0.0) {
            ++screened;
            return true;
        }
        unsigned long long bits;
        std::memcpy(&bits, &magnitude, 8);
        unsigned long long exponent = (bits >> 52) & 0x7ff;
        if (exponent < 1) exponent = 1;
        const unsigned long long sbits = exponent << 52;
        double scale;
        std::memcpy(&scale, &sbits, 8);
        a = a / scale;
        b = b / scale;
        c = c / scale;
        auto certain = [&](double t) {
            const double tt = t * t;
            const double value = std::fma(a, tt, std::fma(b, t, c));
            const double aa = std::fabs(a) * t;
            const double e1 = aa * t;
            const double e2 = std::fabs(b) * std::fabs(t);
            const double error = lsx::kEps8 * ((e1 + e2) + std::fabs(c));
            return value >= error || (a == 0.0 && b == 0.0 && c >= 0.0);
        };
        bool vertex_ok = true;
        if (a > 0.0) {
            const double vertex = -b / (2.0 * a);
            const double ac4 = (4.0 * a) * c;
            const double bb = b * b;
            vertex_ok = vertex <= left || vertex >= right || ac4 - bb >= 0.0;
        }
        if (certain(left) && certain(right) && vertex_ok) {
            ++screened;
            return true;
        }
        const double inf = INFINITY;
        if (a == 0.0) {
            if (b > 0.0) exclude(-inf, -c / b);
            else if (b < 0.0) exclude(-c / b, inf);
            else if (c < 0.0) exclude(-inf, inf);
            return true;
        }
        const double ac4n = (-4.0 * a) * c;
        const double discriminant = std::fma(b, b, ac4n);
        if (discriminant < 0.0) {
            if (a < 0.0) exclude(-inf, inf);
        } else if (discriminant == 0.0) {
            if (a < 0.0) {
                const double root = -b / (2.0 * a);
                exclude(-inf, root);
                exclude(root, inf);
            }
        } else {
            ++square_roots;
            double first, second;
            if (b == 0.0) {
                const double root = std::sqrt(-c / a);
                first = -root;
                second = root;
            } else {
                const double q = -0.5 * (b + std::copysign(std::sqrt(discriminant), b));
                first = q / a;
                second = c / q;
            }
            const double lo = std::fmin(first, second), hi = std::fmax(first, second);
            if (a > 0.0) {
                exclude(lo, hi);
            } else {
                exclude(-inf, lo);
                exclude(hi, inf);
            }
        }
        return true;
    }
    bool nearest(double* t) const {
        double l, r;
        if (!hull(&l, &r)) return false;
        double a, b;
        if (!containing(0.0, &a, &b)) {
            *t = 0.0;
            return true;
        }
        bool have = false;
        double best = 0.0;
        for (double cand : {a, b}) {
            if (!(std::fabs(cand) <= bound)) continue;
            // |x|.total_cmp(|y|).then(x.total_cmp(y))
            const bool less = !have || lsx::total_key(std::fabs(cand)) < lsx::total_key(std::fabs(best)) ||
                              (lsx::total_key(std::fabs(cand)) == lsx::total_key(std::fabs(best)) &&
                               lsx::total_key(cand) < lsx::total_key(best));
            if (less) best = cand;
            have = true;
        }
        if (have) *t = best;
        return have;
    }
    size_t intervals(double* out, size_t capacity) const {
        double cursor = -bound;
        size_t n = 0;
        for (const auto& [a, b] : forbidden) {
            if (a >= cursor) {
                if (n < capacity) {
                    out[2 * n] = cursor;
                    out[2 * n + 1] = std::fmin(a, bound);
                }
                ++n;
            }
            cursor = std::fmax(cursor, b);
            if (cursor > bound) return n;
        }
        if (n < capacity) {
            out[2 * n] = cursor;
            out[2 * n + 1] = bound;
        }
        return n + 1;
    }
};

namespace lsx {
namespace {

// The constraint of point p and vocabulary entry j, in the reference's f64 order
// (src/diagnosis.rs:1127-1140).  Device and host share this body; the explicit
// __d*_rn / fma forms keep nvcc from contracting products into FMAs.
struct Coefficients {
    double a, b, c;
};

__host__ __device__ inline double mul_rn(double x, double y) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(x, y);
#else
    return x * y;
#endif
}
__host__ __device__ inline double add_rn(double x, double y) {
#ifdef __CUDA_ARCH__
    return __dadd_rn(x, y);
#else
    return x + y;
#endif
}
__host__ __device__ inline double sub_rn(double x, double y) {
#ifdef __CUDA_ARCH__
    return __dsub_rn(x, y);
#else
    return x - y;
#endif
}

__host__ __device__ inline Coefficients constraint_of(float wut, float wuj, float wvt, float wvj, float zt, float zj,
                                                      double hu, double hv, double margin, double guard) {
    const double du = sub_rn((double)wut, (double)wuj);
    const double dv = sub_rn((double)wvt, (double)wvj);
    const double alpha = sub_rn(mul_rn(du, hv), mul_rn(dv, hu));
    const double beta = add_rn(mul_rn(du, hu), mul_rn(dv, hv));
    const double c = sub_rn(sub_rn(sub_rn((double)zt, (double)zj), margin), guard);
    return {sub_rn(c, mul_rn(2.0, beta)), mul_rn(2.0, alpha), c};
}

// The screening test of FeasibleSet::constrain against the hull [left, right]
// (src/interval.rs:110-132): true when the constraint changes nothing.
// Non-finite coefficients are left to the host, which reports them.
__device__ inline bool screened_at(Coefficients k, double left, double right) {
    double a = k.a, b = k.b, c = k.c;
    if (!(isfinite(a) && isfinite(b) && isfinite(c))) return false;
    const double magnitude = fmax(fmax(fabs(a), fabs(b)), fabs(c));
    if (magnitude == 0.0) return true;
    const unsigned long long bits = (unsigned long long)__double_as_longlong(magnitude);
    unsigned long long exponent = (bits >> 52) & 0x7ff;
    if (exponent < 1) exponent = 1;
    const double scale = __longlong_as_double((long long)(exponent << 52));
    a = __ddiv_rn(a, scale);
    b = __ddiv_rn(b, scale);
    c = __ddiv_rn(c, scale);
    auto certain = [&](double t) {
        const double tt = __dmul_rn(t, t);
        const double value = __fma_rn(a, tt, __fma_rn(b, t, c));
        const double e1 = __dmul_rn(__dmul_rn(fabs(a), t), t);
        const double e2 = __dmul_rn(fabs(b), fabs(t));
        const double error = __dmul_rn(kEps8, __dadd_rn(__dadd_rn(e1, e2), fabs(c)));
        return value >= error || (a == 0.0 && b == 0.0 && c >= 0.0);
    };
    bool vertex_ok = true;
    if (a > 0.0) {
        const double vertex = __ddiv_rn(-b, __dmul_rn(2.0, a));
        vertex_ok = vertex <= left || vertex >= right ||
                    __dsub_rn(__dmul_rn(__dmul_rn(4.0, a), c), __dmul_rn(b, b)) >= 0.0;
    }
    return certain(left) && certain(right) && vertex_ok;
}

// One thread per 32 vocabulary entries of one point: bit j of the word is set
// when constraint (p, 32 w + j) needs the host (not screened against [left,
// right]); the target's own bit and bits past the vocabulary stay clear.
// Words [word0, total_words) of the [points, words_per_point] mask.
__global__ void plane_screen_kernel(const float* __restrict__ wu, const float* __restrict__ wv,
                                    const float* __restrict__ logits, const uint32_t* __restrict__ targets,
                                    const double* __restrict__ hu, const double* __restrict__ hv, int vocab,
                                    int words_per_point, long long word0, long long total_words, double margin,
                                    double guard, double left, double right, uint32_t* __restrict__ mask) {
    for (long long w = word0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; w < total_words;
         w += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(w / words_per_point);
        const int j0 = (int)(w - (long long)p * words_per_point) * 32;
        const uint32_t t = targets[p];
        const float* z = logits + (size_t)p * vocab;
        const float wut = wu[t], wvt = wv[t], zt = z[t];
        const double hup = hu[p], hvp = hv[p];
        uint32_t bitsw = 0;
        for (int i = 0; i < 32; ++i) {
            const int j = j0 + i;
            if (j >= vocab || (uint32_t)j == t) continue;
            const Coefficients k = constraint_of(wut, wu[j], wvt, wv[j], zt, z[j], hup, hvp, margin, guard);
            if (!screened_at(k, left, right)) bitsw |= 1u << i;
        }
        mask[w] = bitsw;
    }
}

}  // namespace
}  // namespace lsx

using namespace lsx;

extern "C" {

int lsx_feasible_create(double bound, lsx_feasible** out) {
    LSX_ENSURE(out, "invalid argument");
    LSX_ENSURE(std::isfinite(bound) && bound > 0.0 && bound <= 1e6, "the half-angle bound must lie in (0, 1e6]");
    lsx_feasible* f = new lsx_feasible;
    f->bound = bound;
    *out = f;
    return LSX_OK;
}

int lsx_feasible_free(lsx_feasible* set) {
    delete set;
    return LSX_OK;
}

int lsx_feasible_constrain(lsx_feasible* set, double a, double b, double c) {
    LSX_ENSURE(set, "invalid argument");
    if (!set->constrain(a, b, c)) return fail(LSX_E_ARGUMENT, "finite quadratic coefficients are required");
    return LSX_OK;
}

int lsx_feasible_is_empty(const lsx_feasible* set) { return set && set->empty() ? 1 : 0; }

int lsx_feasible_nearest(const lsx_feasible* set, double* tangent, int* found) {
    LSX_ENSURE(set && tangent && found, "invalid argument");
    *found = set->nearest(tangent) ? 1 : 0;
    return LSX_OK;
}

size_t lsx_feasible_intervals(const lsx_feasible* set, double* out, size_t capacity) {
    return set ? set->intervals(out, out ? capacity : 0) : 0;
}

int lsx_feasible_work(const lsx_feasible* set, uint64_t* work) {
    LSX_ENSURE(set && work, "invalid argument");
    work[0] = set->constraints;
    work[1] = set->screened;
    work[2] = set->square_roots;
    work[3] = set->inserted;
    return LSX_OK;
}

int lsx_plane_feasible(lsx_ctx* ctx, lsx_feasible* set, const float* wu, const float* wv, size_t vocab,
                       const float* logits, const uint32_t* targets, const double* hu, const double* hv,
                       size_t points, double margin, double guard) {
    LSX_ENSURE(ctx && set && wu && wv && logits && targets && hu && hv, "invalid argument");
    LSX_ENSURE(vocab > 1 && vocab <= 2147483647ull && points > 0 && points <= 2147483647ull,
               "check the plane constraint sizes");
    for (size_t p = 0; p < points; ++p) LSX_ENSURE(targets[p] < vocab, "check the target token range");
    cudaSetDevice(ctx->device);
    const int V = (int)vocab;
    const long long wpp = (V + 31) / 32;
    const long long total_words = wpp * (long long)points;
    const size_t lbytes = points * vocab * 4;
    auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t need = a256(vocab * 4) * 2 + a256(lbytes) + a256(points * 4) + a256(points * 8) * 2 +
                        a256((size_t)total_words * 4);
    void* block = nullptr;
    LSX_TRY(device_alloc(ctx, need, &block));
    uint8_t* base = (uint8_t*)block;
    size_t at = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base + at;
        at += a256(bytes);
        return p;
    };
    float* d_wu = (float*)take(vocab * 4);
    float* d_wv = (float*)take(vocab * 4);
    float* d_logits = (float*)take(lbytes);
    uint32_t* d_targets = (uint32_t*)take(points * 4);
    double* d_hu = (double*)take(points * 8);
    double* d_hv = (double*)take(points * 8);
    uint32_t* d_mask = (uint32_t*)take((size_t)total_words * 4);
    cudaStream_t s = ctx->stream;
    std::vector<uint32_t> mask((size_t)total_words);
    int rc = LSX_OK;
    cudaError_t e = cudaMemcpyAsync(d_wu, wu, vocab * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_wv, wv, vocab * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_logits, logits, lbytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_targets, targets, points * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_hu, hu, points * 8, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_hv, hv, points * 8, cudaMemcpyHostToDevice, s);
    long long word = 0;  // first mask word of the next screening pass
    bool done = false;
    while (e == cudaSuccess && rc == LSX_OK && !done && word < total_words) {
        double left, right;
        if (!set->hull(&left, &right)) break;
        const long long words = total_words - word;
        const int grid = (int)std::min<long long>((words + 255) / 256, (long long)ctx->sm_count * 16);
        plane_screen_kernel<<<grid, 256, 0, s>>>(d_wu, d_wv, d_logits, d_targets, d_hu, d_hv, V, (int)wpp, word,
                                                 total_words, margin, guard, left, right, d_mask);
        e = cudaGetLastError();
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(mask.data() + word, d_mask + word, (size_t)words * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) break;
        // Walk the constraints from this pass's first word in the reference's order.
        long long next = total_words;
        for (long long w = word; w < total_words && !done; ++w) {
            const size_t p = (size_t)(w / wpp);
            const int j0 = (int)(w - (long long)p * wpp) * 32;
            const int jn = std::min(32, V - j0);
            const uint32_t t = targets[p];
            const uint32_t needs = mask[w];
            // screened constraints of this word: counted as FeasibleSet::constrain counts them
            const int own = (t >= (uint32_t)j0 && t < (uint32_t)(j0 + jn)) ? 1 : 0;
            const int screened_here = jn - own - __builtin_popcount(needs);
            if (needs == 0) {
                set->constraints += (uint64_t)screened_here;
                set->screened += (uint64_t)screened_here;
                continue;
            }
            bool moved = false;
            for (int i = 0; i < jn; ++i) {
                const int j = j0 + i;
                if ((uint32_t)j == t) continue;
                if (!(needs >> i & 1u)) {
                    ++set->constraints;
                    ++set->screened;
                    continue;
                }
                const float* z = logits + p * vocab;
                const Coefficients k = constraint_of(wu[t], wu[j], wv[t], wv[j], z[t], z[j], hu[p], hv[p], margin,
                                                     guard);
                double l0, r0;
                set->hull(&l0, &r0);
                if (!set->constrain(k.a, k.b, k.c)) {
                    rc = fail(LSX_E_ARGUMENT, "finite quadratic coefficients are required");
                    done = true;
                    break;
                }
                if (set->empty()) {  // src/diagnosis.rs:1141-1143
                    done = true;
                    break;
                }
                double l1, r1;
                set->hull(&l1, &r1);
                if (l1 != l0 || r1 != r0) {
                    // The rest of this word and all later words were screened against the old hull.
                    for (int i2 = i + 1; i2 < jn; ++i2) {
                        const int j2 = j0 + i2;
                        if ((uint32_t)j2 == t) continue;
                        const Coefficients k2 = constraint_of(wu[t], wu[j2], wv[t], wv[j2], z[t], z[j2], hu[p],
                                                              hv[p], margin, guard);
                        if (!set->constrain(k2.a, k2.b, k2.c)) {
                            rc = fail(LSX_E_ARGUMENT, "finite quadratic coefficients are required");
                            done = true;
                            break;
                        }
                        if (set->empty()) {
                            done = true;
                            break;
                        }
                    }
                    moved = true;
                    break;
                }
            }
            if (moved && !done) {
                next = w + 1;
                break;
            }
        }
        if (done || next >= total_words) break;
        word = next;
    }
    device_release(ctx, block);
    if (e != cudaSuccess) return fail(LSX_E_CUDA, cuda_message("plane constraints", e));
    return rc;
}

}  // extern "C"
