/*
 * lsx_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of LaplacesScissors' decode and readout-validation path, used
 * as the checker for the CUDA implementation in laplacesscissors_b200.  Only the
 * test suite, __graft_entry__.smoke() and the CPU-baseline leg of bench.py load
 * this library; the product path never does.
 *
 * Arithmetic contract (follows tests/qwen_reference.rs:39-202 of the reference,
 * which is the reference's own independent CPU forward): stored weights are
 * widened exactly to f32 (bf16 -> f32 is a 16-bit shift), every vector that
 * crosses an op boundary is f32 as in the reference's device tensors, and every
 * reduction (dot products, norms, RoPE phases, softmax) is carried in f64.
 *
 * Parity pinning: tests/test_oracle_golden.py checks these functions against
 * (a) the known-answer cases of the reference's tests/gpu.rs:19-264 and
 * src/rotation.rs:312-329, and (b) golden vectors produced by running the
 * reference's own kernels/ops.py through Triton's CPU interpreter, driven in
 * the op order of src/model.rs:729-853 (tests/golden/make_golden.py).
 */
#ifndef LSX_ORACLE_H
#define LSX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage kinds: same codes as lsx_dtype (src/gpu.rs:15-20). */
enum { LSXO_F32 = 0, LSXO_F16 = 1, LSXO_BF16 = 2 };

/* kernels/ops.py:7-11 take_row */
void lsxo_take_row(const void* matrix, int kind, size_t row, size_t width, float* out);
/* kernels/ops.py:14-28 matvec: out[r] = sum_c W[r,c] x[c] (+ bias[r]) */
void lsxo_matvec(const void* matrix, int kind, const float* x, const float* bias,
                 size_t rows, size_t cols, float* out, int threads);
/* kernels/ops.py:31-45 normalization (RMSNorm, or LayerNorm when center != 0) */
void lsxo_norm(const float* x, const float* gain, const float* bias, size_t groups,
               size_t width, float epsilon, int center, float* out);
/* kernels/ops.py:48-66 rotary_position (neox half split or interleaved pairs) */
void lsxo_rope(const float* x, size_t heads, size_t dim, double theta, size_t rotary,
               int interleaved, size_t position, float* out);
/* kernels/ops.py:69-73 cache_write */
void lsxo_cache_write(const float* k, const float* v, float* keys, float* values,
                      size_t position, size_t width);
/* kernels/ops.py:76-101 causal_attention over positions 0..position */
void lsxo_attention(const float* q, const float* keys, const float* values, size_t position,
                    size_t qheads, size_t kvheads, size_t dim, double scale, float* out);
/* kernels/ops.py:104-116 gated_product; kind 0 SiLU, 1 erf-GELU, 2 ReLU, 3 tanh-GELU */
void lsxo_gated(const float* gate, const float* up, size_t n, int kind, float* out);
/* kernels/ops.py:119-122 vector_sum: out = x + factor*y, both roundings kept (no FMA) */
void lsxo_combine(const float* x, const float* y, float factor, size_t n, float* out);
/* kernels/ops.py:125-135 plane_rotation on f32 data, f64 inner products */
void lsxo_plane_rotation(const float* h, const float* u, const float* v, float cosine_minus_one,
                         float sine, size_t width, float* out);

/* src/rotation.rs:50-53 ReadoutRotation::coefficients */
void lsxo_plane_coefficients(double tangent, double* a, double* b);
/* src/rotation.rs:54-68 ReadoutRotation::apply (f64) */
void lsxo_plane_apply(const double* u, const double* v, double tangent, size_t width,
                      const double* h, double* out);
/* src/response.rs:67-77 SubspaceRotation::apply (f64); basis is rank x width rows,
   transform is rank x rank row-major */
void lsxo_subspace_apply(const double* basis, const double* transform, size_t rank,
                         size_t width, const double* h, double* out);

/* src/diagnosis.rs:58-70 argmax: first maximum (strict >) */
uint32_t lsxo_argmax(const float* z, size_t n);
/* src/diagnosis.rs:71-80 other: max over j != target, total order, lowest index on ties */
size_t lsxo_other(const float* z, size_t n, uint32_t target);
/* src/diagnosis.rs:490-492 minimum_margin */
double lsxo_minimum_margin(const float* z, size_t n, uint32_t target);
/* attribution.rs:49-60 loss: logsumexp(z) - z[target] in f64 */
double lsxo_loss(const float* z, size_t n, uint32_t target);

/* Decoder description in the shape of GraphSpec (src/graph.rs:93-107) restricted to
   what src/model.rs executes.  Matrices are row-major [out, in] in `kind` storage. */
typedef struct lsxo_block {
    const void *q, *k, *v, *o, *gate, *up, *down;
    const float *q_bias, *k_bias, *v_bias, *o_bias, *gate_bias, *up_bias, *down_bias;
    int kind;                                   /* storage kind of the seven matrices */
    const float *input_gain, *post_gain;        /* f32, gain_offset already added */
    const float *input_bias, *post_bias;        /* LayerNorm biases or NULL */
    const float *q_gain, *k_gain;               /* per-head norms or NULL */
    float *keys, *values;                       /* f32 [capacity, kv_heads*head_dim] */
} lsxo_block;

typedef struct lsxo_model {
    size_t hidden, vocab, layers, qheads, kvheads, head_dim, intermediate, rotary, capacity;
    double theta, score_scale;
    float epsilon, qk_epsilon;
    int center;              /* LayerNorm (NormKind::Layer) for the residual norms */
    int interleaved, activation;
    float embedding_scale;
    const void* embedding; int embedding_kind;
    const void* head; int head_kind; const float* head_bias;
    const float* final_gain; const float* final_bias;
    lsxo_block* blocks;
} lsxo_model;

/* Model::decode (src/model.rs:729-853) for one position.  `residual` is the decoder
   input (embedding row or injected vector, f32[hidden]); writes the final-normed
   hidden state and, when `logits` is non-NULL, the readout logits of `readout_input`
   (the hidden state when NULL) -- callers apply an edit between the two by calling
   lsxo_decode with logits NULL and then lsxo_matvec. */
void lsxo_decode(const lsxo_model* m, size_t position, const float* residual, float* hidden,
                 float* logits, int threads);
/* Model::embedding_tensor (src/model.rs:620-631): row, then combine(row,row,scale-1). */
void lsxo_embedding(const lsxo_model* m, uint32_t token, float* out);

/* Readout validation rows (src/model.rs:664-685 + src/diagnosis.rs:490-492, 58-70):
   for each of n f32 inputs (already edited), logits = W x + b, then margin of
   target vs the best other token, first argmax and the target logit. */
void lsxo_readout_rows(const void* head, int kind, const float* bias, size_t vocab, size_t width,
                       const float* inputs, size_t n, const uint32_t* targets, double* margin,
                       uint32_t* argmax, float* target_logit, int threads);

/* FeasibleSet (src/interval.rs:47-212): open forbidden intervals of the half-angle
   tangent t in [-bound, bound], merged as quadratic constraints a t^2 + b t + c >= 0
   arrive.  Sorted array of (lower, upper) with the Endpoint order (equal when ==,
   otherwise f64::total_cmp). */
typedef struct lsxo_feasible {
    double bound;
    double *lower, *upper;
    size_t count, capacity;
    uint64_t work[4]; /* constraints, screened, square_roots, inserted_intervals */
} lsxo_feasible;
/* 0 on success, -1 for an invalid bound (FeasibleSet::new). */
int lsxo_feasible_init(lsxo_feasible* f, double bound);
void lsxo_feasible_free(lsxo_feasible* f);
/* FeasibleSet::constrain: 0, or -1 for non-finite coefficients. */
int lsxo_feasible_constrain(lsxo_feasible* f, double a, double b, double c);
int lsxo_feasible_is_empty(const lsxo_feasible* f);
/* FeasibleSet::nearest: 1 and *t when some, else 0. */
int lsxo_feasible_nearest(const lsxo_feasible* f, double* t);
/* FeasibleSet::intervals: writes up to `capacity` (lower, upper) pairs and returns
   the number of feasible intervals. */
size_t lsxo_feasible_intervals(const lsxo_feasible* f, double* out, size_t capacity);
/* The plane candidate's constraint loop (src/diagnosis.rs:1118-1143): for each point
   p (target t_p, frame logits z_p [vocab], projections hu_p, hv_p) and each j != t_p,
   the constraint (c - 2 beta, 2 alpha, c) with du = wu[t] - wu[j], dv = wv[t] - wv[j],
   alpha = du hv - dv hu, beta = du hu + dv hv, c = z[t] - z[j] - margin - guard, all
   f64; stops once the set is empty.  0, or -1 on non-finite coefficients. */
int lsxo_plane_feasible(lsxo_feasible* f, const float* wu, const float* wv, size_t vocab, const float* logits,
                        const uint32_t* targets, const double* hu, const double* hv, size_t points, double margin,
                        double guard);

/* restored_loss (src/attribution.rs:61-78): loss of z with z[row] replaced by `original`. */
double lsxo_restored_loss(const float* z, size_t n, size_t row, float original, uint32_t target);
/* integrated_probabilities (src/attribution.rs:79-123), sequential f64 as the
   reference: credits [vocab] and, when non-NULL, the per-point integrals
   gradients [points x vocab]. */
void lsxo_integrated_credits(const float* before, const float* after, const uint32_t* targets,
                             const double* weights, size_t points, size_t vocab, size_t panels, double* credits,
                             double* gradients);

/* The benchmark inputs' counter-based generator (SplitMix64 finaliser; Box-Muller
   normals rounded to f32, then to bf16 when kind is LSXO_BF16; uniform integers by
   multiply-shift), written independently of the library's so that the CPU
   baseline and the reference arms can build their inputs without it, and so that
   a test can check the two generators against each other. */
void lsxo_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, double std, int kind,
                       void* out);
void lsxo_synth_uniform_u32(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, uint32_t bound,
                            uint32_t* out);

/* Version string of the oracle build. */
const char* lsxo_version(void);

#ifdef __cplusplus
}
#endif
#endif
