/*
 * lsx.h -- C ABI of the B200 decode and readout-validation path of LaplacesScissors.
 *
 * The reference runs this path from Rust through a Triton compile bridge
 * (src/gpu.rs, src/device.rs, kernels/compile.py, kernels/ops.py).  This header is
 * the boundary that replaces it: plain pointers and sizes, status codes, no
 * framework types.  Each entry names the reference function whose contract it
 * keeps (file:line in the reference tree).
 *
 * Conventions
 *  - Every call returns an int status (LSX_OK == 0).  On failure the calling
 *    thread's message is available from lsx_last_error(), in the spirit of the
 *    reference's anyhow messages (src/device.rs:233-255).
 *  - Argument checks follow the reference's `ensure!`s: the same shapes are
 *    rejected, with LSX_E_ARGUMENT.
 *  - A context owns one device and one stream.  Calls are synchronous with respect
 *    to host buffers they take (like every Gpu::read in the reference) unless the
 *    name says `_device`, in which case all pointers are device pointers and the
 *    call only enqueues work on the context's stream.
 *  - A context is not thread-safe (the reference's Gpu is used through &mut self).
 */
#ifndef LSX_H
#define LSX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage kinds; same members and order as DType (src/gpu.rs:15-20). */
typedef enum lsx_dtype { LSX_F32 = 0, LSX_F16 = 1, LSX_BF16 = 2 } lsx_dtype;

/* Status codes. */
enum lsx_status {
    LSX_OK = 0,
    LSX_E_ARGUMENT = 1,    /* a shape, range or finiteness check failed */
    LSX_E_MEMORY = 2,      /* device or host allocation failed */
    LSX_E_CUDA = 3,        /* a CUDA runtime/driver call failed */
    LSX_E_NONFINITE = 4,   /* non-finite outputs (src/model.rs:680-683, 845-848) */
    LSX_E_IO = 5,          /* file access failed while loading a checkpoint */
    LSX_E_FORMAT = 6,      /* malformed safetensors / config.json / graph */
    LSX_E_UNSUPPORTED = 7, /* valid input this build does not execute */
    LSX_E_STATE = 8        /* call not valid in the object's current state */
};

typedef struct lsx_ctx lsx_ctx;           /* Gpu + Device (src/gpu.rs:133-190) */
typedef struct lsx_tensor lsx_tensor;     /* Tensor (src/gpu.rs:55-76) */
typedef struct lsx_rotation lsx_rotation; /* DeviceRotation (src/model.rs:285-364) */
typedef struct lsx_model lsx_model;       /* Model (src/model.rs:383-853) */

/* Message of the last failed call on this thread ("" when none). */
const char* lsx_last_error(void);
/* Library version string. */
const char* lsx_version(void);

/* ---------------------------------------------------------------- context -- */
/* Gpu::new + Device::open (src/gpu.rs:142-190, src/device.rs:101-181): binds CUDA
   device `device` (the reference's LAPLACE_DEVICE ordinal) and creates a stream. */
int lsx_ctx_create(int device, lsx_ctx** out);
/* Drop for Gpu (src/gpu.rs:561-566): synchronises, then releases everything. */
int lsx_ctx_destroy(lsx_ctx* ctx);
/* Gpu::synchronize (src/gpu.rs:200-203). */
int lsx_ctx_synchronize(lsx_ctx* ctx);
/* Gpu::name (src/gpu.rs:191-193). */
int lsx_ctx_name(lsx_ctx* ctx, char* buffer, size_t length);
/* Gpu::architecture (src/gpu.rs:197-199): compute capability as major*10+minor. */
int lsx_ctx_architecture(lsx_ctx* ctx, int* architecture);
/* The context's cudaStream_t, for callers that order their own work after ours. */
int lsx_ctx_stream(lsx_ctx* ctx, void** stream);

/* ---------------------------------------------------------------- tensors -- */
/* Gpu::upload_raw (src/gpu.rs:217-226): copies `bytes` of `kind` storage. */
int lsx_upload_raw(lsx_ctx* ctx, const void* data, size_t bytes, lsx_dtype kind, lsx_tensor** out);
/* Gpu::upload_f32 (src/gpu.rs:227-235). */
int lsx_upload_f32(lsx_ctx* ctx, const float* data, size_t count, lsx_tensor** out);
/* Gpu::zeros (src/gpu.rs:236-240). */
int lsx_zeros(lsx_ctx* ctx, size_t count, lsx_tensor** out);
/* Gpu::read (src/gpu.rs:241-247): F32 tensors only; `count` must equal the length. */
int lsx_read(lsx_ctx* ctx, const lsx_tensor* tensor, float* out, size_t count);
/* Drop for Tensor (src/gpu.rs:72-76).  NULL is accepted. */
int lsx_tensor_free(lsx_tensor* tensor);
/* Tensor::len / Tensor::dtype (src/gpu.rs:61-70). */
size_t lsx_tensor_len(const lsx_tensor* tensor);
int lsx_tensor_dtype(const lsx_tensor* tensor);
/* Device address of the tensor's first element. */
void* lsx_tensor_data(const lsx_tensor* tensor);
/* Non-owning tensor over caller device memory (no counterpart in the reference;
   lets a caller hand its own device buffers to the per-op entries). */
int lsx_tensor_wrap(lsx_ctx* ctx, void* device_pointer, size_t count, lsx_dtype kind, lsx_tensor** out);

/* ------------------------------------------------------------ per-op API -- */
/* Each entry returns a new F32 tensor, as every Gpu op does. */
/* Gpu::embedding (src/gpu.rs:360-377), kernels/ops.py:7-11. */
int lsx_embedding(lsx_ctx* ctx, const lsx_tensor* weight, size_t row, size_t width, lsx_tensor** out);
/* Gpu::linear (src/gpu.rs:378-405), kernels/ops.py:14-28.  bias may be NULL. */
int lsx_linear(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* w, const lsx_tensor* bias,
               size_t rows, size_t cols, lsx_tensor** out);
/* Gpu::linear into a caller-provided F32 tensor `out` of `rows` elements (no
   allocation and no synchronisation; the reference always returns a new tensor).
   Enqueued on the context's stream, so it can be captured into a CUDA graph. */
int lsx_linear_into(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* w, const lsx_tensor* bias,
                    size_t rows, size_t cols, lsx_tensor* out);
/* Gpu::norm (src/gpu.rs:406-431), kernels/ops.py:31-45.  center != 0 is LayerNorm. */
int lsx_norm(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* gain, const lsx_tensor* bias,
             size_t groups, size_t width, float epsilon, int center, lsx_tensor** out);
/* Gpu::rope (src/gpu.rs:432-453), kernels/ops.py:48-66. */
int lsx_rope(lsx_ctx* ctx, const lsx_tensor* x, size_t position, size_t heads, size_t dim,
             float theta, size_t rotary, int interleaved, lsx_tensor** out);
/* Gpu::attention (src/gpu.rs:454-501), kernels/ops.py:69-101: writes k, v at
   `position` of the f32 caches, then attends over positions 0..position. */
int lsx_attention(lsx_ctx* ctx, const lsx_tensor* q, const lsx_tensor* k, const lsx_tensor* v,
                  lsx_tensor* keys, lsx_tensor* values, size_t position, size_t qheads,
                  size_t kvheads, size_t dim, float scale, lsx_tensor** out);
/* Gpu::gated (src/gpu.rs:502-519), kernels/ops.py:104-116; kind 0 SiLU, 1 GELU(erf),
   2 ReLU, 3 GELU(tanh) (Activation::code, src/graph.rs:41-50). */
int lsx_gated(lsx_ctx* ctx, const lsx_tensor* gate, const lsx_tensor* up, uint32_t kind, lsx_tensor** out);
/* Gpu::combine (src/gpu.rs:520-538), kernels/ops.py:119-122: x + factor*y. */
int lsx_combine(lsx_ctx* ctx, const lsx_tensor* x, const lsx_tensor* y, float factor, lsx_tensor** out);
/* Gpu::rotate (src/gpu.rs:539-559), kernels/ops.py:125-135. */
int lsx_rotate(lsx_ctx* ctx, const lsx_tensor* h, const lsx_tensor* u, const lsx_tensor* v,
               float cosine_minus_one, float sine, lsx_tensor** out);

/* --------------------------------------------------------- readout edits -- */
/* DeviceRotation::upload (src/model.rs:300-310): plane (u, v, tangent), validated as
   ReadoutRotation::validate (src/rotation.rs:28-49). */
int lsx_rotation_plane(lsx_ctx* ctx, const double* u, const double* v, double tangent, size_t width,
                       lsx_rotation** out);
/* DeviceRotation::upload_edit Joint (src/model.rs:311-341): basis rank x width rows,
   transform rank x rank row-major, validated as SubspaceRotation::validate
   (src/response.rs:33-60). */
int lsx_rotation_joint(lsx_ctx* ctx, const double* basis, const double* transform, size_t rank,
                       size_t width, lsx_rotation** out);
/* DeviceRotation::apply (src/model.rs:342-363) on an F32 tensor. */
int lsx_rotation_apply(lsx_ctx* ctx, const lsx_rotation* rotation, const lsx_tensor* hidden, lsx_tensor** out);
int lsx_rotation_free(lsx_rotation* rotation);

/* ------------------------------------------------------------------ model -- */
typedef struct lsx_model_info {
    uint64_t hidden_size, vocab_size, layers, capacity, position;
    uint64_t query_heads, kv_heads, head_dim, intermediate_size, rotary_dim;
    uint64_t parameters, tensors;
    uint64_t eos_count;
    uint32_t eos_token_ids[8];
    uint64_t fused;        /* 1: fused decode engine; 0: per-op kernels */
    uint64_t graph;        /* 1: the fused step replays a captured CUDA graph */
    uint64_t kernels_per_step; /* kernel launches of one fused decode step (kernel-chain engine) */
    uint64_t persistent;   /* 1: one persistent kernel runs each generate/advance call */
} lsx_model_info;

/* Model::load (src/model.rs:411-529): reads `root`/laplace.graph.json or the HF
   config.json (GraphSpec::load, src/graph.rs:151-163) and its safetensors weights
   (hub::weight_files, src/hub.rs:120-128); allocates f32 K/V caches of `capacity`. */
int lsx_model_load(lsx_ctx* ctx, const char* root, size_t capacity, lsx_model** out);
int lsx_model_free(lsx_model* model);
int lsx_model_info_get(const lsx_model* model, lsx_model_info* out);
/* 1 when the fused decode engine runs this checkpoint, 0 when the per-op kernels do
   (checkpoints with F32/F16 projections, LayerNorm or other head sizes). */
int lsx_model_fused(const lsx_model* model);
/* Model::reset / Model::rewind (src/model.rs:632-642). */
int lsx_model_reset(lsx_model* model);
int lsx_model_rewind(lsx_model* model, size_t position);
/* Model::advance (src/model.rs:694-706): one token at the cursor; returns the Frame
   (hidden = final-normed state before the edit, logits after it).  hidden_out,
   logits_out and argmax_out may each be NULL. */
int lsx_model_advance(lsx_model* model, uint32_t token, const lsx_rotation* rotation,
                      float* hidden_out, float* logits_out, uint32_t* argmax_out);
/* Model::inject without intervention or trace (src/model.rs:707-728). */
int lsx_model_inject(lsx_model* model, const float* vector, const lsx_rotation* rotation,
                     float* hidden_out, float* logits_out, uint32_t* argmax_out);
/* Model::embedding_vector (src/model.rs:611-619). */
int lsx_model_embedding_vector(lsx_model* model, uint32_t token, float* out);
/* Model::readout (src/model.rs:664-685): logits of a host f32 hidden state. */
int lsx_model_readout(lsx_model* model, const float* hidden, const lsx_rotation* rotation, float* logits_out);
/* Model::head_image (src/model.rs:643-652): W u without bias for an f64 direction. */
int lsx_model_head_image(lsx_model* model, const double* vector, float* out);
/* Model::head_image for `count` directions at once, as the joint search calls it
   once per basis axis (src/diagnosis.rs:777-781): out[k * vocab + i] = (W f32(u_k))[i]
   for vectors [count x hidden] (f64, row-major).  One tensor-core pass over the
   lm_head per 32 directions, each f32 direction entering exactly as three bf16
   terms; results equal lsx_model_head_image's up to f32 summation order. */
int lsx_model_head_images(lsx_model* model, const double* vectors, size_t count, float* out);
/* Model::head_row (src/model.rs:653-663). */
int lsx_model_head_row(lsx_model* model, uint32_t token, float* out);
/* Readout weight and bias of the model (non-owning; bias NULL when absent). */
int lsx_model_head(lsx_model* model, const lsx_tensor** weight, const lsx_tensor** bias);
/* diagnosis::generate_frames (src/diagnosis.rs:106-149): prefill `prompt`
   token by token, then greedy decode up to `maximum` tokens, stopping after a stop
   token.  tokens_out holds `maximum` entries; *generated receives the count.  When
   non-NULL, hidden_frames [maximum x hidden] and logits_frames [maximum x vocab]
   receive the Frame of each generated token.  The cursor ends where the reference's
   does (prompt length + generated - 1). */
int lsx_model_generate(lsx_model* model, const uint32_t* prompt, size_t prompt_length, size_t maximum,
                       const uint32_t* stop_tokens, size_t stop_count, const lsx_rotation* rotation,
                       uint32_t* tokens_out, size_t* generated, int* stopped,
                       float* hidden_frames, float* logits_frames);

/* Teacher-forced case scoring (src/scaling.rs:181-216): prefill `prompt` token by
   token, then for each of the `count` targets score the Frame that predicts it and
   advance with the target.  Per scored position k: nll_out[k] = attribution::loss
   (src/attribution.rs:49-60) of the Frame's logits for targets[k] (f64),
   argmax_out[k] = the logits' first argmax.  With `rotation` the logits are the
   edited readout of the unedited hidden state (the reference's "after" scores:
   Model::readout with the edit); hidden states and the advance are unchanged.
   hidden_frames [count x hidden] and logits_frames [count x vocab] may be NULL, as
   may nll_out and argmax_out.  The cursor ends at prompt_length + count - 1. */
int lsx_model_score(lsx_model* model, const uint32_t* prompt, size_t prompt_length, const uint32_t* targets,
                    size_t count, const lsx_rotation* rotation, double* nll_out, uint32_t* argmax_out,
                    float* hidden_frames, float* logits_frames);

/* Greedy generation of `batch` independent sequences at once (batch > 1 decode; the
   reference decodes one sequence at a time, diagnosis::generate_frames,
   src/diagnosis.rs:106-149, so a batch equals that many separate generations):
   prompts [batch x prompt_length] (prompt_length >= 2), tokens_out [batch x maximum].
   The first prompt_length - 1 tokens of every sequence go through one batched
   forward into per-sequence KV caches; then each step feeds one row per sequence
   through the tensor-core GEMMs (each weight read once for the whole batch) and an
   attention over each sequence's own cache.  No stop tokens, no frames; does not
   touch the model's own cursor or cache. */
int lsx_model_generate_batch(lsx_model* model, const uint32_t* prompts, size_t batch, size_t prompt_length,
                             size_t maximum, uint32_t* tokens_out);
/* lsx_model_score over `cases` independent cases of equal shape at once (the
   per-case loop of scaling::evaluate, src/scaling.rs:181-216, batched): prompts
   [cases x prompt_length], targets [cases x count].  Per scored position:
   nll_out (attribution::loss), argmax_out (first argmax), margin_out
   (minimum_margin of the target, src/diagnosis.rs:490-492), all [cases x count],
   and logits_out [cases x count x vocab] (host, each may be NULL).  With
   `rotation` (rank at most 256) the scores come from the edited readout of the
   unedited hidden states, as lsx_model_score's.  The fed tokens of all cases go
   through each layer together (tensor-core GEMMs with the f32 activations as two
   bf16 terms); results agree with lsx_model_score within the decode tolerances.
   The model's decode cursor and KV cache are not touched. */
int lsx_model_score_batch(lsx_model* model, const uint32_t* prompts, size_t cases, size_t prompt_length,
                          const uint32_t* targets, size_t count, const lsx_rotation* rotation, double* nll_out,
                          uint32_t* argmax_out, double* margin_out, float* logits_out);

/* ------------------------------------------------------ readout validation -- */
/* Fused readout margin over many hidden states (verify_cached's target rows,
   src/diagnosis.rs:512-537 with minimum_margin src/diagnosis.rs:490-492 and argmax
   src/diagnosis.rs:58-70): for each row i, z = W (Q h_i) + b with Q the optional
   edit, then
     margin_out[i]       = f64(z[t_i]) - f64(max_{j != t_i} z[j])  (lowest index on ties)
     argmax_out[i]       = first index of max_j z[j]
     target_logit_out[i] = z[t_i]
   Logits are never stored.  `hidden` is [rows x width] of `hidden_kind` (F32 or
   BF16).  Host pointers; any output may be NULL. */
int lsx_readout_margin(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias, size_t vocab,
                       size_t width, const void* hidden, lsx_dtype hidden_kind, size_t rows,
                       const uint32_t* targets, const lsx_rotation* rotation, double* margin_out,
                       uint32_t* argmax_out, float* target_logit_out);
/* Same computation on device-resident inputs and outputs (no host copies, no
   synchronisation).  workspace must hold lsx_readout_workspace_bytes() bytes.  The
   kernels' status (a device wait that gave up; non-finite scores, which the
   reference rejects, src/model.rs:680-683) stays in the workspace: read it with
   lsx_readout_status. */
int lsx_readout_margin_device(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias,
                              size_t vocab, size_t width, const void* hidden, lsx_dtype hidden_kind,
                              size_t rows, const uint32_t* targets, const lsx_rotation* rotation,
                              double* margin_out, uint32_t* argmax_out, float* target_logit_out,
                              void* workspace, size_t workspace_bytes);
size_t lsx_readout_workspace_bytes(size_t vocab, size_t width, size_t rows, const lsx_rotation* rotation);
/* Status of the last readout call that used `workspace` (lsx_readout_margin_device,
   lsx_readout_shard_device), or, with workspace NULL, of the last
   lsx_readout_margin_fixed call on the context's device: waits for the context's
   stream, then returns LSX_E_CUDA when a kernel's bounded device wait gave up,
   LSX_E_NONFINITE when a score was not finite (Model::readout's rejection,
   src/model.rs:680-683), else LSX_OK.  The host-buffer entries check this
   themselves. */
int lsx_readout_status(lsx_ctx* ctx, const void* workspace);
/* CompactReadout::evaluate (src/diagnosis.rs:643-665) fused with minimum_margin,
   other and argmax (src/diagnosis.rs:58-80, 490-492): for observation o the scores
   z_o = image c_o + baseline_o are reduced on the device, never stored, to
     margin_out[o] = f64(z_o[t_o]) - f64(max_{j != t_o} z_o[j]),
     other_out[o]  = that competitor (lowest index on ties),
     argmax_out[o] = first index of max_j z_o[j].
   image: F32 tensor [vocab x rank] (the transposed head images, rank <= 256);
   baseline: F32 tensor [count x vocab] (each observation's current logits);
   coefficients [count x rank] f32 and targets [count] are host arrays, outputs
   host arrays (any may be NULL).  A non-finite score fails with LSX_E_NONFINITE,
   as the reference rejects it. */
int lsx_compact_margin(lsx_ctx* ctx, const lsx_tensor* image, const lsx_tensor* baseline, size_t vocab,
                       size_t rank, size_t count, const float* coefficients, const uint32_t* targets,
                       double* margin_out, uint32_t* other_out, uint32_t* argmax_out);
/* Vocabulary-sharded validation (the multi-GPU split of the lm_head by rows; the
   reference runs the whole readout on one device, src/model.rs:664-685).  One
   shard's part: `weight_shard` holds lm_head rows [vocab_offset, vocab_offset +
   shard_vocab) ([shard_vocab x width] BF16), `bias_shard` the same slice of the
   bias or NULL, targets are global token ids.  Per row it writes, to device
   buffers, the packed key of the shard's best column other than the target
   (total-order f32 value << 32 | (0xFFFFFFFF - global index), so the larger key
   is the larger logit and, on equal logits, the lower index: the rule of other(),
   src/diagnosis.rs:71-80) and the target's logit (-inf when the target lies
   outside the shard).  The shards' partials combine by an element-wise maximum
   (an all-reduce MAX of the keys as unsigned 64-bit integers and of the target
   logits); lsx_readout_merge_device then gives margins and first argmaxes equal
   to lsx_readout_margin_device's over the whole vocabulary.  workspace must hold
   lsx_readout_workspace_bytes(shard_vocab, ...) bytes.  Asynchronous on the
   context's stream. */
int lsx_readout_shard_device(lsx_ctx* ctx, const lsx_tensor* weight_shard, const lsx_tensor* bias_shard,
                             size_t vocab_offset, size_t shard_vocab, size_t width, const void* hidden,
                             lsx_dtype hidden_kind, size_t rows, const uint32_t* targets,
                             const lsx_rotation* rotation, uint64_t* other_key_out, float* target_logit_out,
                             void* workspace, size_t workspace_bytes);
/* Margins (f64(z_t) - f64(z_competitor), minimum_margin, src/diagnosis.rs:490-492),
   first argmaxes (src/diagnosis.rs:58-70) and target logits from merged partials;
   device pointers, any output may be NULL. */
int lsx_readout_merge_device(lsx_ctx* ctx, const uint64_t* other_key, const float* target_logit,
                             const uint32_t* targets, size_t rows, double* margin_out, uint32_t* argmax_out,
                             float* target_logit_out);
/* lsx_readout_shard_device with the shard's per-row partials written in one
   signed-orderable int64 buffer partials [2 x rows]: element i < rows is the
   packed best-other key with its top bit flipped, element rows + i the target
   logit's total-order key (-inf, the lowest, when the target lies outside the
   shard).  An element-wise signed maximum merges shards, so the whole exchange is
   one all-reduce MAX of 16 bytes per row (ncclInt64) with no conversion before or
   after it; lsx_readout_partials_merge_device then gives margins, first argmaxes
   and target logits equal to lsx_readout_margin_device's over the whole
   vocabulary.  Asynchronous on the context's stream; status as
   lsx_readout_shard_device's (lsx_readout_status on the workspace). */
int lsx_readout_partials_device(lsx_ctx* ctx, const lsx_tensor* weight_shard, const lsx_tensor* bias_shard,
                                size_t vocab_offset, size_t shard_vocab, size_t width, const void* hidden,
                                lsx_dtype hidden_kind, size_t rows, const uint32_t* targets,
                                const lsx_rotation* rotation, int64_t* partials, void* workspace,
                                size_t workspace_bytes);
/* Margins (minimum_margin, src/diagnosis.rs:490-492), first argmaxes
   (src/diagnosis.rs:58-70) and target logits from merged packed partials; device
   pointers, any output may be NULL. */
int lsx_readout_partials_merge_device(lsx_ctx* ctx, const int64_t* partials, const uint32_t* targets, size_t rows,
                                      double* margin_out, uint32_t* argmax_out, float* target_logit_out);
/* The device-pointer readout margin without an edit, for callers that must not
   allocate device memory (their memory is already fully committed, or an
   allocation at that point would be illegal or would stall other work).  It has
   no counterpart in the reference.
   Scratch is a fixed 4 MiB area inside the library's device image, one per device:
   calls needing more (bf16 hidden: about 12 bytes per row; F32 hidden: a further
   4 x width bytes per row) fail with LSX_E_ARGUMENT and enqueue nothing.  No
   scratch word needs to start at zero.  Calls that may overlap on one device share
   that scratch and race: order them on one stream.  The kernels' status words stay
   in the scratch until the next call on the device: lsx_readout_status(ctx, NULL)
   reports them.  The first call on a device looks the scratch up (which may load
   the library's device code): make it before any stream capture begins. */
int lsx_readout_margin_fixed(lsx_ctx* ctx, const lsx_tensor* weight, const lsx_tensor* bias,
                             size_t vocab, size_t width, const void* hidden, lsx_dtype hidden_kind,
                             size_t rows, const uint32_t* targets, double* margin_out,
                             uint32_t* argmax_out, float* target_logit_out);

/* ------------------------------------------------ plane-candidate feasibility -- */
/* FeasibleSet (src/interval.rs:47-212): the open forbidden intervals of a plane
   rotation's half-angle tangent t in [-bound, bound], merged as quadratic
   constraints a t^2 + b t + c >= 0 arrive, with the reference's screening and work
   counters.  Host code; needs no GPU. */
typedef struct lsx_feasible lsx_feasible;
/* FeasibleSet::new: bound in (0, 1e6]. */
int lsx_feasible_create(double bound, lsx_feasible** out);
int lsx_feasible_free(lsx_feasible* set);
/* FeasibleSet::constrain; LSX_E_ARGUMENT for non-finite coefficients. */
int lsx_feasible_constrain(lsx_feasible* set, double a, double b, double c);
/* FeasibleSet::is_empty: 1 when no tangent is feasible. */
int lsx_feasible_is_empty(const lsx_feasible* set);
/* FeasibleSet::nearest: *found = 0 when empty, else the feasible tangent nearest 0
   (ties: the smaller magnitude, then the smaller value). */
int lsx_feasible_nearest(const lsx_feasible* set, double* tangent, int* found);
/* FeasibleSet::intervals: writes up to `capacity` (lower, upper) pairs and returns
   how many feasible intervals there are. */
size_t lsx_feasible_intervals(const lsx_feasible* set, double* out, size_t capacity);
/* Work counters: constraints, screened, square_roots, inserted_intervals. */
int lsx_feasible_work(const lsx_feasible* set, uint64_t* work);
/* The plane candidate's constraint loop (src/diagnosis.rs:1118-1143) into `set`:
   for each point p (target t_p, frame logits [points x vocab] row p, f64 projections
   hu_p = u.h_p, hv_p = v.h_p) and each j != t_p, the constraint (c - 2 beta, 2 alpha,
   c) with du = wu[t] - wu[j], dv = wv[t] - wv[j], alpha = du hv - dv hu,
   beta = du hu + dv hv, c = z[t] - z[j] - margin - guard (wu, wv the head images of
   u and v); stops as soon as the set is empty.  Every constraint is formed and
   screened on the GPU against the current hull; the host merges the rest in the
   reference's order, so the set and its counters equal the sequential loop's.
   Host arrays. */
int lsx_plane_feasible(lsx_ctx* ctx, lsx_feasible* set, const float* wu, const float* wv, size_t vocab,
                       const float* logits, const uint32_t* targets, const double* hu, const double* hv,
                       size_t points, double margin, double guard);

/* ------------------------------------------------------------ attribution -- */
/* integrated_probabilities (src/attribution.rs:79-123) with the losses analyze needs
   (src/attribution.rs:49-78), on the GPU in f64.  For point p (before/after logits
   rows of [points x vocab] f32, target, weight >= 0) the softmax along the chord
   z(t) = (1 - t) before + t after is integrated by Simpson's rule over `panels`
   (even) panels; credits_out[j] = -sum_p weight_p (after_pj - before_pj) integral_pj.
   For the `row_count` rows given, gradients_out[p * row_count + r] = integral_p at
   rows[r] (may be NULL).  losses_out (may be NULL) is [points x (2 + row_count)]:
   loss(before_p), loss(after_p), then restored_loss(after_p, rows[r], before_p[rows[r]],
   target_p).  Host arrays; sums over the vocabulary are reassociated, so results
   match the sequential loop to f64 rounding. */
int lsx_integrated_credits(lsx_ctx* ctx, const float* before, const float* after, const uint32_t* targets,
                           const double* weights, size_t points, size_t vocab, size_t panels, double* credits_out,
                           const uint32_t* rows, size_t row_count, double* gradients_out, double* losses_out);

/* ---------------------------------------------------- synthetic checkpoints -- */
/* Seeded N(0, std^2) values rounded to `kind` (BF16 or F32): element i of stream
   `stream` under `seed` is a pure function of (seed, stream, i), so any slice can
   be generated independently.  Host code; needs no GPU. */
int lsx_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, double std,
                     lsx_dtype kind, void* out);
/* Seeded uniform integers in [0, bound). */
int lsx_synth_uniform_u32(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, uint32_t bound,
                          uint32_t* out);

#ifdef __cplusplus
}
#endif
#endif
