/*
 * lsx_oracle.c -- TEST INFRASTRUCTURE ONLY (see lsx_oracle.h).
 *
 * CPU restatement of the reference's decode and readout-validation path.  Each
 * function names the reference lines it follows.  Products of stored weights and
 * f32 activations are formed exactly in f64 and summed in f64; vectors between
 * ops are rounded to f32 as the reference's device tensors are.
 */
#include "lsx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

const char* lsxo_version(void) { return "lsx-oracle 1"; }

static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16 -> f32, exact (half 2.7.1's widening, Cargo.lock of the reference). */
static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400u));
            man &= 0x3ffu;
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline double load(const void* m, int kind, size_t i) {
    switch (kind) {
    case LSXO_F32: return (double)((const float*)m)[i];
    case LSXO_F16: return (double)f16_to_f32(((const uint16_t*)m)[i]);
    default: return (double)bf16_to_f32(((const uint16_t*)m)[i]);
    }
}

/* kernels/ops.py:7-11 */
void lsxo_take_row(const void* matrix, int kind, size_t row, size_t width, float* out) {
    for (size_t i = 0; i < width; ++i) out[i] = (float)load(matrix, kind, row * width + i);
}

static double dot_row(const void* matrix, int kind, size_t row, const float* x, size_t cols) {
    double s = 0.0;
    size_t base = row * cols;
    if (kind == LSXO_BF16) {
        const uint16_t* w = (const uint16_t*)matrix + base;
        for (size_t c = 0; c < cols; ++c) s += (double)bf16_to_f32(w[c]) * (double)x[c];
    } else if (kind == LSXO_F32) {
        const float* w = (const float*)matrix + base;
        for (size_t c = 0; c < cols; ++c) s += (double)w[c] * (double)x[c];
    } else {
        const uint16_t* w = (const uint16_t*)matrix + base;
        for (size_t c = 0; c < cols; ++c) s += (double)f16_to_f32(w[c]) * (double)x[c];
    }
    return s;
}

/* kernels/ops.py:14-28 (f64 accumulation of exact products) */
void lsxo_matvec(const void* matrix, int kind, const float* x, const float* bias, size_t rows,
                 size_t cols, float* out, int threads) {
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for num_threads(threads) schedule(static) if (rows * cols > (1u << 16))
#else
    (void)threads;
#endif
    for (long r = 0; r < (long)rows; ++r) {
        double s = dot_row(matrix, kind, (size_t)r, x, cols);
        if (bias) s += (double)bias[r];
        out[r] = (float)s;
    }
}

/* kernels/ops.py:31-45 */
void lsxo_norm(const float* x, const float* gain, const float* bias, size_t groups, size_t width,
               float epsilon, int center, float* out) {
    for (size_t g = 0; g < groups; ++g) {
        const float* row = x + g * width;
        double mean = 0.0;
        if (center) {
            for (size_t i = 0; i < width; ++i) mean += row[i];
            mean /= (double)width;
        }
        double sq = 0.0;
        for (size_t i = 0; i < width; ++i) {
            double d = (double)row[i] - mean;
            sq += d * d;
        }
        double inverse = 1.0 / sqrt(sq / (double)width + (double)epsilon);
        for (size_t i = 0; i < width; ++i) {
            double y = ((double)row[i] - mean) * inverse * (double)gain[i];
            if (bias) y += (double)bias[i];
            out[g * width + i] = (float)y;
        }
    }
}

/* kernels/ops.py:48-66; phase = position * theta^(-2 pair / rotary) in f64 as
   tests/qwen_reference.rs:61-76 and tests/gpu.rs:118-131 state it. */
void lsxo_rope(const float* x, size_t heads, size_t dim, double theta, size_t rotary,
               int interleaved, size_t position, float* out) {
    size_t width = heads * dim;
    memcpy(out, x, width * sizeof(float));
    size_t half = rotary / 2;
    for (size_t h = 0; h < heads; ++h) {
        for (size_t pair = 0; pair < half; ++pair) {
            size_t a, b;
            if (interleaved) {
                a = h * dim + 2 * pair;
                b = a + 1;
            } else {
                a = h * dim + pair;
                b = a + half;
            }
            double phase = (double)position / pow(theta, 2.0 * (double)pair / (double)rotary);
            double s = sin(phase), c = cos(phase);
            double xa = x[a], xb = x[b];
            out[a] = (float)(xa * c - xb * s);
            out[b] = (float)(xb * c + xa * s);
        }
    }
}

/* kernels/ops.py:69-73 */
void lsxo_cache_write(const float* k, const float* v, float* keys, float* values, size_t position,
                      size_t width) {
    memcpy(keys + position * width, k, width * sizeof(float));
    memcpy(values + position * width, v, width * sizeof(float));
}

/* kernels/ops.py:76-101 with f64 scores and softmax (tests/gpu.rs:210-239) */
void lsxo_attention(const float* q, const float* keys, const float* values, size_t position,
                    size_t qheads, size_t kvheads, size_t dim, double scale, float* out) {
    size_t width = kvheads * dim;
    size_t ratio = qheads / kvheads;
    double* scores = (double*)malloc((position + 1) * sizeof(double));
    for (size_t head = 0; head < qheads; ++head) {
        size_t kv = head / ratio;
        double m = -INFINITY;
        for (size_t t = 0; t <= position; ++t) {
            double s = 0.0;
            for (size_t d = 0; d < dim; ++d)
                s += (double)q[head * dim + d] * (double)keys[t * width + kv * dim + d];
            s *= scale;
            scores[t] = s;
            if (s > m) m = s;
        }
        double denom = 0.0;
        for (size_t t = 0; t <= position; ++t) {
            scores[t] = exp(scores[t] - m);
            denom += scores[t];
        }
        for (size_t d = 0; d < dim; ++d) {
            double acc = 0.0;
            for (size_t t = 0; t <= position; ++t)
                acc += scores[t] * (double)values[t * width + kv * dim + d];
            out[head * dim + d] = (float)(acc / denom);
        }
    }
    free(scores);
}

/* kernels/ops.py:104-116 */
void lsxo_gated(const float* gate, const float* up, size_t n, int kind, float* out) {
    for (size_t i = 0; i < n; ++i) {
        double x = gate[i], a;
        switch (kind) {
        case 0: a = x / (1.0 + exp(-x)); break;
        case 1: a = 0.5 * x * (1.0 + erf(x * 0.7071067811865476)); break;
        case 2: a = x > 0.0 ? x : 0.0; break;
        default: a = 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x))); break;
        }
        out[i] = (float)(a * (double)up[i]);
    }
}

/* kernels/ops.py:119-122; the reference compiles without FMA contraction
   (kernels/compile.py:35), so the product and the sum round separately. */
void lsxo_combine(const float* x, const float* y, float factor, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) {
        volatile float p = factor * y[i];
        out[i] = x[i] + p;
    }
}

/* kernels/ops.py:125-135 */
void lsxo_plane_rotation(const float* h, const float* u, const float* v, float cosine_minus_one,
                         float sine, size_t width, float* out) {
    double hu = 0.0, hv = 0.0;
    for (size_t i = 0; i < width; ++i) {
        hu += (double)h[i] * (double)u[i];
        hv += (double)h[i] * (double)v[i];
    }
    double a = cosine_minus_one, b = sine;
    for (size_t i = 0; i < width; ++i)
        out[i] = (float)((double)h[i] + (double)u[i] * (a * hu + b * hv) +
                         (double)v[i] * (a * hv - b * hu));
}

/* src/rotation.rs:50-53 */
void lsxo_plane_coefficients(double t, double* a, double* b) {
    *a = -2.0 * t * t / (1.0 + t * t);
    *b = 2.0 * t / (1.0 + t * t);
}

/* src/rotation.rs:54-68 */
void lsxo_plane_apply(const double* u, const double* v, double tangent, size_t width,
                      const double* h, double* out) {
    double a, b;
    lsxo_plane_coefficients(tangent, &a, &b);
    double x = 0.0, y = 0.0;
    for (size_t i = 0; i < width; ++i) {
        x += u[i] * h[i];
        y += v[i] * h[i];
    }
    for (size_t i = 0; i < width; ++i) out[i] = h[i] + u[i] * (a * x + b * y) + v[i] * (a * y - b * x);
}

/* src/response.rs:61-77 */
void lsxo_subspace_apply(const double* basis, const double* transform, size_t rank, size_t width,
                         const double* h, double* out) {
    double* x = (double*)calloc(rank, sizeof(double));
    double* delta = (double*)calloc(rank, sizeof(double));
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < width; ++j) x[i] += basis[i * width + j] * h[j];
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < rank; ++j)
            delta[i] += (transform[i * rank + j] - (i == j ? 1.0 : 0.0)) * x[j];
    memcpy(out, h, width * sizeof(double));
    for (size_t i = 0; i < rank; ++i)
        for (size_t j = 0; j < width; ++j) out[j] += delta[i] * basis[i * width + j];
    free(x);
    free(delta);
}

/* src/diagnosis.rs:58-70 */
uint32_t lsxo_argmax(const float* z, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (z[i] > z[best]) best = i;
    return (uint32_t)best;
}

/* f32::total_cmp key: larger key <=> larger in IEEE total order. */
static inline int64_t total_key(float f) {
    int32_t i;
    memcpy(&i, &f, 4);
    return (int64_t)(i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1));
}

/* src/diagnosis.rs:71-80: max_by(total_cmp).then(b.cmp(a)) keeps the lowest index. */
size_t lsxo_other(const float* z, size_t n, uint32_t target) {
    size_t best = (size_t)-1;
    int64_t key = 0;
    for (size_t i = 0; i < n; ++i) {
        if (i == target) continue;
        int64_t k = total_key(z[i]);
        if (best == (size_t)-1 || k > key) {
            best = i;
            key = k;
        }
    }
    return best;
}

/* src/diagnosis.rs:490-492 */
double lsxo_minimum_margin(const float* z, size_t n, uint32_t target) {
    return (double)z[target] - (double)z[lsxo_other(z, n, target)];
}

/* src/attribution.rs:49-60 */
double lsxo_loss(const float* z, size_t n, uint32_t target) {
    double top = -INFINITY;
    for (size_t i = 0; i < n; ++i)
        if ((double)z[i] > top) top = z[i];
    double s = 0.0;
    for (size_t i = 0; i < n; ++i) s += exp((double)z[i] - top);
    return top + log(s) - (double)z[target];
}

/* src/model.rs:620-631 */
void lsxo_embedding(const lsxo_model* m, uint32_t token, float* out) {
    lsxo_take_row(m->embedding, m->embedding_kind, token, m->hidden, out);
    if (m->embedding_scale != 1.0f) lsxo_combine(out, out, m->embedding_scale - 1.0f, m->hidden, out);
}

/* src/model.rs:729-853 */
void lsxo_decode(const lsxo_model* m, size_t position, const float* residual_in, float* hidden,
                 float* logits, int threads) {
    size_t H = m->hidden, qw = m->qheads * m->head_dim, kw = m->kvheads * m->head_dim;
    size_t I = m->intermediate;
    size_t big = qw > H ? qw : H;
    if (I > big) big = I;
    float* residual = (float*)malloc(H * sizeof(float));
    float* norm = (float*)malloc(big * sizeof(float));
    float* q = (float*)malloc(qw * sizeof(float));
    float* k = (float*)malloc(kw * sizeof(float));
    float* v = (float*)malloc(kw * sizeof(float));
    float* t = (float*)malloc(big * sizeof(float));
    float* mixed = (float*)malloc(qw * sizeof(float));
    float* gate = (float*)malloc(I * sizeof(float));
    float* up = (float*)malloc(I * sizeof(float));
    float* feature = (float*)malloc(I * sizeof(float));
    float* proj = (float*)malloc(H * sizeof(float));
    memcpy(residual, residual_in, H * sizeof(float));
    for (size_t l = 0; l < m->layers; ++l) {
        const lsxo_block* b = &m->blocks[l];
        lsxo_norm(residual, b->input_gain, b->input_bias, 1, H, m->epsilon, m->center, norm);
        lsxo_matvec(b->q, b->kind, norm, b->q_bias, qw, H, q, threads);
        lsxo_matvec(b->k, b->kind, norm, b->k_bias, kw, H, k, threads);
        lsxo_matvec(b->v, b->kind, norm, b->v_bias, kw, H, v, threads);
        if (b->q_gain) {
            lsxo_norm(q, b->q_gain, NULL, m->qheads, m->head_dim, m->qk_epsilon, 0, t);
            memcpy(q, t, qw * sizeof(float));
        }
        if (b->k_gain) {
            lsxo_norm(k, b->k_gain, NULL, m->kvheads, m->head_dim, m->qk_epsilon, 0, t);
            memcpy(k, t, kw * sizeof(float));
        }
        if (m->rotary > 0) {
            lsxo_rope(q, m->qheads, m->head_dim, m->theta, m->rotary, m->interleaved, position, t);
            memcpy(q, t, qw * sizeof(float));
            lsxo_rope(k, m->kvheads, m->head_dim, m->theta, m->rotary, m->interleaved, position, t);
            memcpy(k, t, kw * sizeof(float));
        }
        lsxo_cache_write(k, v, b->keys, b->values, position, kw);
        lsxo_attention(q, b->keys, b->values, position, m->qheads, m->kvheads, m->head_dim,
                       m->score_scale, mixed);
        lsxo_matvec(b->o, b->kind, mixed, b->o_bias, H, qw, proj, threads);
        lsxo_combine(residual, proj, 1.0f, H, residual);
        lsxo_norm(residual, b->post_gain, b->post_bias, 1, H, m->epsilon, m->center, norm);
        lsxo_matvec(b->gate, b->kind, norm, b->gate_bias, I, H, gate, threads);
        lsxo_matvec(b->up, b->kind, norm, b->up_bias, I, H, up, threads);
        lsxo_gated(gate, up, I, m->activation, feature);
        lsxo_matvec(b->down, b->kind, feature, b->down_bias, H, I, proj, threads);
        lsxo_combine(residual, proj, 1.0f, H, residual);
    }
    lsxo_norm(residual, m->final_gain, m->final_bias, 1, H, m->epsilon, m->center, hidden);
    if (logits)
        lsxo_matvec(m->head, m->head_kind, hidden, m->head_bias, m->vocab, H, logits, threads);
    free(residual); free(norm); free(q); free(k); free(v); free(t); free(mixed);
    free(gate); free(up); free(feature); free(proj);
}

/* Blocked readout: stream the head once per block of rows (the reference re-reads it
   once per row, src/diagnosis.rs:512-537; the result per row is the same). */
#define ORACLE_ROW_BLOCK 8
void lsxo_readout_rows(const void* head, int kind, const float* bias, size_t vocab, size_t width,
                       const float* inputs, size_t n, const uint32_t* targets, double* margin,
                       uint32_t* argmax, float* target_logit, int threads) {
    float* z = (float*)malloc(vocab * ORACLE_ROW_BLOCK * sizeof(float));
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#else
    (void)threads;
#endif
    for (size_t r0 = 0; r0 < n; r0 += ORACLE_ROW_BLOCK) {
        size_t rb = n - r0 < ORACLE_ROW_BLOCK ? n - r0 : ORACLE_ROW_BLOCK;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
        for (long j = 0; j < (long)vocab; ++j) {
            double acc[ORACLE_ROW_BLOCK] = {0};
            if (kind == LSXO_BF16) {
                const uint16_t* w = (const uint16_t*)head + (size_t)j * width;
                for (size_t c = 0; c < width; ++c) {
                    double wc = (double)bf16_to_f32(w[c]);
                    for (size_t r = 0; r < rb; ++r) acc[r] += wc * (double)inputs[(r0 + r) * width + c];
                }
            } else {
                for (size_t c = 0; c < width; ++c) {
                    double wc = load(head, kind, (size_t)j * width + c);
                    for (size_t r = 0; r < rb; ++r) acc[r] += wc * (double)inputs[(r0 + r) * width + c];
                }
            }
            for (size_t r = 0; r < rb; ++r) {
                double s = acc[r] + (bias ? (double)bias[j] : 0.0);
                z[r * vocab + (size_t)j] = (float)s;
            }
        }
        for (size_t r = 0; r < rb; ++r) {
            const float* zr = z + r * vocab;
            uint32_t t = targets[r0 + r];
            if (margin) margin[r0 + r] = lsxo_minimum_margin(zr, vocab, t);
            if (argmax) argmax[r0 + r] = lsxo_argmax(zr, vocab);
            if (target_logit) target_logit[r0 + r] = zr[t];
        }
    }
    free(z);
}


/* ------------------------------------------------------------ FeasibleSet --
 * src/interval.rs:47-212.  Every operation below keeps the reference's f64
 * evaluation order; the Makefile compiles with -ffp-contract=off so that only the
 * explicit fma() calls (the reference's mul_add) fuse. */
static int endpoint_cmp(double x, double y) {
    if (x == y) return 0;
    /* f64::total_cmp */
    int64_t a, b;
    memcpy(&a, &x, 8);
    memcpy(&b, &y, 8);
    a ^= (int64_t)(((uint64_t)(a >> 63)) >> 1);
    b ^= (int64_t)(((uint64_t)(b >> 63)) >> 1);
    return a < b ? -1 : (a > b ? 1 : 0);
}

int lsxo_feasible_init(lsxo_feasible* f, double bound) {
    memset(f, 0, sizeof(*f));
    if (!(isfinite(bound) && bound > 0. && bound <= 1e6)) return -1;
    f->bound = bound;
    return 0;
}

void lsxo_feasible_free(lsxo_feasible* f) {
    free(f->lower);
    free(f->upper);
    f->lower = f->upper = NULL;
    f->count = f->capacity = 0;
}

/* number of keys strictly below x (Endpoint order) */
static size_t keys_below(const lsxo_feasible* f, double x) {
    size_t lo = 0, hi = f->count;
    while (lo < hi) {
        size_t mid = (lo + hi) / 2;
        if (endpoint_cmp(f->lower[mid], x) < 0) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

/* FeasibleSet::containing: the forbidden interval with the largest key < x, if x < its upper. */
static int containing(const lsxo_feasible* f, double x, double* a, double* b) {
    size_t n = keys_below(f, x);
    if (n == 0) return 0;
    if (x < f->upper[n - 1]) {
        *a = f->lower[n - 1];
        *b = f->upper[n - 1];
        return 1;
    }
    return 0;
}

static int hull(const lsxo_feasible* f, double* left, double* right) {
    double a, b;
    *left = containing(f, -f->bound, &a, &b) ? b : -f->bound;
    *right = containing(f, f->bound, &a, &b) ? a : f->bound;
    return *left <= *right;
}

int lsxo_feasible_is_empty(const lsxo_feasible* f) {
    double l, r;
    return !hull(f, &l, &r);
}

static void remove_at(lsxo_feasible* f, size_t i) {
    memmove(f->lower + i, f->lower + i + 1, (f->count - i - 1) * sizeof(double));
    memmove(f->upper + i, f->upper + i + 1, (f->count - i - 1) * sizeof(double));
    f->count--;
}

static void insert_key(lsxo_feasible* f, double a, double b) {
    size_t i = keys_below(f, a);
    if (i < f->count && endpoint_cmp(f->lower[i], a) == 0) {  /* BTreeMap::insert replaces the value */
        f->upper[i] = b;
        return;
    }
    if (f->count == f->capacity) {
        f->capacity = f->capacity ? 2 * f->capacity : 16;
        f->lower = (double*)realloc(f->lower, f->capacity * sizeof(double));
        f->upper = (double*)realloc(f->upper, f->capacity * sizeof(double));
    }
    memmove(f->lower + i + 1, f->lower + i, (f->count - i) * sizeof(double));
    memmove(f->upper + i + 1, f->upper + i, (f->count - i) * sizeof(double));
    f->lower[i] = a;
    f->upper[i] = b;
    f->count++;
}

static double fmax_rs(double x, double y) { return isnan(x) ? y : (isnan(y) ? x : (x > y ? x : y)); }

static void exclude(lsxo_feasible* f, double a, double b) {
    if (a >= b || b <= -f->bound || a >= f->bound) return;
    f->work[3]++;
    /* the largest key <= a whose interval reaches past a */
    size_t n = keys_below(f, a);
    if (n < f->count && endpoint_cmp(f->lower[n], a) == 0) n++;
    if (n > 0 && f->upper[n - 1] > a) {
        a = f->lower[n - 1];
        b = fmax_rs(b, f->upper[n - 1]);
        remove_at(f, n - 1);
    }
    for (;;) {
        size_t i = keys_below(f, a); /* smallest key >= a */
        if (i >= f->count || f->lower[i] >= b) break;
        b = fmax_rs(b, f->upper[i]);
        remove_at(f, i);
    }
    insert_key(f, a, b);
}

int lsxo_feasible_constrain(lsxo_feasible* f, double a, double b, double c) {
    if (!(isfinite(a) && isfinite(b) && isfinite(c))) return -1;
    f->work[0]++;
    double left, right;
    if (!hull(f, &left, &right)) return 0;
    double magnitude = fmax_rs(fmax_rs(fabs(a), fabs(b)), fabs(c));
    if (magnitude == 0.) {
        f->work[1]++;
        return 0;
    }
    uint64_t bits;
    memcpy(&bits, &magnitude, 8);
    uint64_t exponent = (bits >> 52) & 0x7ff;
    if (exponent < 1) exponent = 1;
    uint64_t sbits = exponent << 52;
    double scale;
    memcpy(&scale, &sbits, 8);
    a = a / scale;
    b = b / scale;
    c = c / scale;
    const double eps8 = 8. * 2.220446049250313e-16;
#define CERTAIN(t)                                                                                   \
    ((fma(a, (t) * (t), fma(b, (t), c)) >= eps8 * (fabs(a) * (t) * (t) + fabs(b) * fabs(t) + fabs(c))) || \
     (a == 0. && b == 0. && c >= 0.))
    int vertex_ok = 1;
    if (a > 0.) {
        double vertex = -b / (2. * a);
        vertex_ok = vertex <= left || vertex >= right || 4. * a * c - b * b >= 0.;
    }
    if (CERTAIN(left) && CERTAIN(right) && vertex_ok) {
        f->work[1]++;
        return 0;
    }
#undef CERTAIN
    const double inf = INFINITY;
    if (a == 0.) {
        if (b > 0.) exclude(f, -inf, -c / b);
        else if (b < 0.) exclude(f, -c / b, inf);
        else if (c < 0.) exclude(f, -inf, inf);
        return 0;
    }
    double discriminant = fma(b, b, -4. * a * c);
    if (discriminant < 0.) {
        if (a < 0.) exclude(f, -inf, inf);
    } else if (discriminant == 0.) {
        if (a < 0.) {
            double root = -b / (2. * a);
            exclude(f, -inf, root);
            exclude(f, root, inf);
        }
    } else {
        f->work[2]++;
        double first, second;
        if (b == 0.) {
            double root = sqrt(-c / a);
            first = -root;
            second = root;
        } else {
            double q = -0.5 * (b + copysign(sqrt(discriminant), b));
            first = q / a;
            second = c / q;
        }
        double lo = first < second ? first : second, hi = first < second ? second : first;
        /* f64::min / f64::max of two non-NaN values */
        if (a > 0.) {
            exclude(f, lo, hi);
        } else {
            exclude(f, -inf, lo);
            exclude(f, hi, inf);
        }
    }
    return 0;
}

/* |x|.total_cmp(|y|).then(x.total_cmp(y)) == Less */
static int abs_then_value_less(double x, double y) {
    double ax = fabs(x), ay = fabs(y);
    int64_t ia, ib;
    memcpy(&ia, &ax, 8);
    memcpy(&ib, &ay, 8);
    if (ia != ib) return ia < ib; /* non-negative doubles order like their bits */
    int64_t a, b;
    memcpy(&a, &x, 8);
    memcpy(&b, &y, 8);
    a ^= (int64_t)(((uint64_t)(a >> 63)) >> 1);
    b ^= (int64_t)(((uint64_t)(b >> 63)) >> 1);
    return a < b;
}

int lsxo_feasible_nearest(const lsxo_feasible* f, double* t) {
    double l, r, a, b;
    if (!hull(f, &l, &r)) return 0;
    if (!containing(f, 0., &a, &b)) {
        *t = 0.;
        return 1;
    }
    int have = 0;
    double best = 0.;
    double cand[2] = {a, b};
    for (int i = 0; i < 2; ++i) {
        if (!(fabs(cand[i]) <= f->bound)) continue;
        if (!have || abs_then_value_less(cand[i], best)) best = cand[i];
        have = 1;
    }
    if (have) *t = best;
    return have;
}

size_t lsxo_feasible_intervals(const lsxo_feasible* f, double* out, size_t capacity) {
    double cursor = -f->bound;
    size_t n = 0;
    for (size_t i = 0; i < f->count; ++i) {
        if (f->lower[i] >= cursor) {
            if (n < capacity) {
                out[2 * n] = cursor;
                out[2 * n + 1] = f->lower[i] < f->bound ? f->lower[i] : f->bound;
            }
            n++;
        }
        cursor = fmax_rs(cursor, f->upper[i]);
        if (cursor > f->bound) return n;
    }
    if (n < capacity) {
        out[2 * n] = cursor;
        out[2 * n + 1] = f->bound;
    }
    return n + 1;
}

int lsxo_plane_feasible(lsxo_feasible* f, const float* wu, const float* wv, size_t vocab, const float* logits,
                        const uint32_t* targets, const double* hu, const double* hv, size_t points, double margin,
                        double guard) {
    for (size_t p = 0; p < points; ++p) {
        const float* z = logits + p * vocab;
        const size_t t = targets[p];
        for (size_t j = 0; j < vocab; ++j) {
            if (j == t) continue;
            const double du = (double)wu[t] - (double)wu[j];
            const double dv = (double)wv[t] - (double)wv[j];
            const double alpha = du * hv[p] - dv * hu[p];
            const double beta = du * hu[p] + dv * hv[p];
            const double c = (double)z[t] - (double)z[j] - margin - guard;
            if (lsxo_feasible_constrain(f, c - 2. * beta, 2. * alpha, c) != 0) return -1;
            if (lsxo_feasible_is_empty(f)) return 0;
        }
    }
    return 0;
}


/* ------------------------------------------------------------ attribution --
 * src/attribution.rs:61-123, in the reference's f64 order (sequential sums,
 * -ffp-contract=off). */
double lsxo_restored_loss(const float* z, size_t n, size_t row, float original, uint32_t target) {
    double maximum = -INFINITY;
    for (size_t j = 0; j < n; ++j) maximum = fmax_rs(maximum, (double)(j == row ? original : z[j]));
    double total = 0.0;
    for (size_t j = 0; j < n; ++j) total += exp((double)(j == row ? original : z[j]) - maximum);
    return maximum + log(total) - (double)(row == target ? original : z[target]);
}

void lsxo_integrated_credits(const float* before, const float* after, const uint32_t* targets,
                             const double* weights, size_t points, size_t vocab, size_t panels, double* credits,
                             double* gradients) {
    double* integral = (double*)malloc(vocab * sizeof(double));
    double* prob = (double*)malloc(vocab * sizeof(double));
    for (size_t j = 0; j < vocab; ++j) credits[j] = 0.0;
    for (size_t p = 0; p < points; ++p) {
        const float* b = before + p * vocab;
        const float* a = after + p * vocab;
        for (size_t j = 0; j < vocab; ++j) integral[j] = 0.0;
        for (size_t k = 0; k <= panels; ++k) {
            const double t = (double)k / (double)panels;
            double maximum = -INFINITY;
            for (size_t j = 0; j < vocab; ++j) {
                prob[j] = (double)b[j] * (1. - t) + (double)a[j] * t;
                maximum = fmax_rs(maximum, prob[j]);
            }
            double total = 0.0;
            for (size_t j = 0; j < vocab; ++j) {
                prob[j] = exp(prob[j] - maximum);
                total += prob[j];
            }
            const double weight = (k == 0 || k == panels ? 1. : (k % 2 == 0 ? 2. : 4.)) / (3. * (double)panels);
            for (size_t j = 0; j < vocab; ++j)
                integral[j] += weight * (prob[j] / total - (j == targets[p] ? 1. : 0.));
        }
        for (size_t j = 0; j < vocab; ++j)
            credits[j] -= weights[p] * ((double)a[j] - (double)b[j]) * integral[j];
        if (gradients) memcpy(gradients + p * vocab, integral, vocab * sizeof(double));
    }
    free(integral);
    free(prob);
}

/* ------------------------------------------------------------ input generator -- */
static uint64_t synth_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
#define SYNTH_STEP 0x9E3779B97F4A7C15ull

static uint64_t synth_bits(uint64_t key, uint64_t i) { return synth_mix(key + (i + 1) * SYNTH_STEP); }

static uint16_t synth_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

void lsxo_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, double std, int kind,
                       void* out) {
    const uint64_t key = synth_mix(seed ^ synth_mix(stream + SYNTH_STEP));
    const long long n = (long long)count;
#pragma omp parallel for schedule(static) if (count > (1u << 16))
    for (long long j = 0; j < n; ++j) {
        const uint64_t i = offset + (uint64_t)j, pair = i >> 1;
        const double u1 = (double)((synth_bits(key, 2 * pair) >> 11) + 1) * 0x1.0p-53;
        const double u2 = (double)(synth_bits(key, 2 * pair + 1) >> 11) * 0x1.0p-53;
        const double radius = sqrt(-2.0 * log(u1)), angle = 6.283185307179586476925286766559 * u2;
        const float v = (float)(std * ((i & 1) ? radius * sin(angle) : radius * cos(angle)));
        if (kind == LSXO_BF16) ((uint16_t*)out)[j] = synth_bf16(v);
        else ((float*)out)[j] = v;
    }
}

void lsxo_synth_uniform_u32(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, uint32_t bound,
                            uint32_t* out) {
    const uint64_t key = synth_mix(seed ^ synth_mix(stream + SYNTH_STEP));
    for (size_t j = 0; j < count; ++j) out[j] = (uint32_t)(((synth_bits(key, offset + j) >> 32) * (uint64_t)bound) >> 32);
}
