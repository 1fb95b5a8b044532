/*
 * krystal_cuda.h — C ABI of the B200 backend for Krystal's frame forward.
 *
 * This is the drop-in boundary. The reference session talks to a device
 * through the `BrainBackend` seam (packages/krystal/src/host/backend.ts:
 * 146-180); `@krystal/webgpu` implements it in packages/webgpu/src/
 * backend.ts:91-181. A `@krystal/cuda` adapter binds the functions below
 * through bun:ffi and implements the same seam:
 *
 *   BrainBackendFactory (backend.ts:177-180)  -> kc_create
 *   BrainBackend.encode (backend.ts:149)      -> kc_encode
 *   BrainBackend.sync   (backend.ts:167)      -> kc_sync
 *   BrainBackend.backward (backend.ts:158)    -> kc_backward
 *   GradientSource.backward over many frames (gradients.ts:15-24, learn.ts:
 *     318-400)                                -> kc_backward_batch_device
 *   BrainBackend.destroy(backend.ts:168)      -> kc_destroy
 *   selectorOracle in choose() (session.ts:149-176, forward/oracle.ts:332-382)
 *                                             -> kc_select (optional seam
 *                                                extension `select?`)
 *   packed ragged batches of think()          -> kc_forward_batch /
 *                                                kc_forward_batch_device
 *   think() turns arriving one at a time      -> kc_stream_* (rolling batches)
 *
 * Conventions. All arrays are row-major fp32 / u32, exactly the typed arrays
 * the TypeScript side holds. Host pointers unless a function says "device".
 * The library owns its device buffers; the caller owns every pointer it
 * passes. Every call returns a kc_status; kc_last_error() gives the message.
 * Calls on one handle are serialised by an internal mutex (the reference
 * serialises device work per engine, webgpu/src/backend.ts:84-89). One CUDA
 * stream per handle. Nothing here allocates host memory the caller must free.
 *
 * Numerics. The forward reproduces the reference CPU oracle's arithmetic:
 * f64 accumulation in the reference's loop order, rounding to f32 wherever
 * the oracle stores into a Float32Array. Selected indices match the oracle
 * bit for bit; distributions agree to far inside 1e-4.
 */
#ifndef KRYSTAL_CUDA_H
#define KRYSTAL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KC_ABI_VERSION 1u
#define KC_RECORD_WIDTH 8u        /* BRAIN_LIMITS.recordWidth (schema/src/krystal-engine-schema.ts:97) */
#define KC_QUERY_BAND 5u          /* index of "query" in BRAIN_FRAME_BANDS (:150-172) */
#define KC_NO_SELECTION 0xffffffffu /* index of an all-blocked row (forward/oracle.ts:364-365) */
#define KC_MAX_BANK 4096u         /* largest bank one frame may hold */
#define KC_NO_WORD 0xffffffffu    /* INVALID_WORD_ID (forward/masks.ts:145) */

/* Precision of the batch entry points (kc_forward_batch[_device]).
 * EXACT: the oracle's arithmetic (f64 accumulation in its order, f32 stores).
 * CERTIFIED (default): tensor cores at fp32-class accuracy; every score
 *   carries a margin B_qj = kappa_q * |sq_q| * |sk_j| / sqrt(H) + 4u|s_qj|
 *   (kappa_q = kappa0 * (1 + sqrt(max_j |s_qj| / 2)), kappa0 = 2e-5, u = 2^-24)
 *   and every question whose selection those margins cannot settle (the top
 *   score's interval touching another's, a sampled draw within the cumulative
 *   p's error of an edge, non-finite values) has its frame recomputed on the
 *   exact path, so selections match the exact path and distributions agree
 *   to ~1e-6. The recomputed frames audit the margin (kc_stage_times).
 * FAST: the tensor-core path without the recomputation (diagnostics).
 * kc_backward_batch_device runs its products on the tensor cores at CERTIFIED
 * and FAST (gradients to fp32-class accuracy; the backward makes no discrete
 * choice to certify) and in the oracle's arithmetic at EXACT.
 * kc_encode, kc_select and kc_backward always compute exactly. */
#define KC_PRECISION_EXACT 0
#define KC_PRECISION_CERTIFIED 1
#define KC_PRECISION_FAST 2

typedef enum kc_status {
  KC_OK = 0,
  KC_ERR_INVALID_ARG = 1, /* malformed frame, weights or arguments */
  KC_ERR_CAPACITY = 2,    /* a size beyond what the library supports, or device memory exhausted */
  KC_ERR_CUDA = 3,        /* a CUDA runtime error */
  KC_ERR_TIMEOUT = 4,     /* a bounded device-side wait expired */
  KC_ERR_NONFINITE = 5,   /* non-finite values where finite ones are required */
  KC_ERR_NO_DEVICE = 6    /* no usable CUDA device */
} kc_status;

typedef struct kc_handle kc_handle;

/* BrainForwardConfig (forward/model.ts:27-53). The six embedding table row
 * counts are parameters; the reference's defaults are 4352, 4352, 256, 8, 2, 8.
 * token_rows maps a token (or field-role) id to its embedding row (model.ts:52). */
typedef struct kc_config {
  uint32_t hidden_size, head_count, head_dim, ffn_size, encoder_blocks, mixer_blocks;
  uint32_t token_space, field_space, schema_space, band_space, stream_space, pos_space;
  uint32_t route_kind_count;
  const uint32_t* token_rows;
  uint32_t token_rows_len;
} kc_config;

/* BlockWeights (model.ts:131-137): wq, wk, wv [H,H], w1 [FFN,H], w2 [H,FFN]. */
typedef struct kc_block_view {
  const float *wq, *wk, *wv, *w1, *w2;
} kc_block_view;

/* BrainForwardWeights (model.ts:145-183). */
typedef struct kc_weights_view {
  const float* embeddings;      /* concatenated tables, embeddingTableBases order */
  const kc_block_view* enc;     /* encoder_blocks entries */
  const float* pool;            /* [2,H] */
  const kc_block_view* mixer;   /* mixer_blocks entries */
  const float* selector_wq;     /* [H,H] */
  const float* selector_wk;     /* [H,H] */
  const float* decision_head_wh;/* [route_kind_count, 3H] */
  const float* value_head_wv;   /* [3H] */
} kc_weights_view;

/* WeightChanges (host/backend.ts:134-145). embedding_rows are element
 * offsets into the embeddings page, each hidden_size long. */
typedef struct kc_changes {
  int32_t selector, pool, value_head, decision_head, blocks;
  const uint32_t* embedding_rows;
  uint32_t embedding_rows_count;
} kc_changes;

/* One packed frame: BrainFrameGpu (schema/src/krystal-engine-schema.ts:
 * 203-209) as built by packHostFrame (host/frame.ts:72-115). */
typedef struct kc_frame_view {
  uint32_t slots;
  const uint32_t* token_ids;             /* [slots*8], PAD = 0 */
  const uint32_t* field_roles;           /* [slots*8] */
  const uint32_t* schema_ids;            /* [slots] */
  const uint32_t* band_ids;              /* [slots]; band 5 marks a question */
  const uint32_t* active_record_indices; /* [slots], ascending, 0xffffffff ends the list */
} kc_frame_view;

/* EncodedFrame (host/backend.ts:33-39). */
typedef struct kc_encoded_view {
  uint32_t q, r;
  const float* query_output; /* [Q,H] */
  const float* bank_keys;    /* [R,H] */
  const float* bank_values;  /* [R,H] */
} kc_encoded_view;

/* Device form of the host grammar `allows(query, record)` that selectionMask
 * (host/learn.ts:215-232) turns into a [Q,R] mask: question i admits bank
 * record s iff bit schema_ids[s] of schema_allow[i*8..i*8+8) (256 bits) and
 * bit band_ids[s] of band_allow[i] are set. A question that admits nothing is
 * reopened to the whole bank (learn.ts:229). */
typedef struct kc_mask_rule {
  const uint32_t* schema_allow;    /* [Q*8] */
  const uint32_t* band_allow;      /* [Q] */
  const uint32_t* bank_schema_ids; /* [R] schema of each bank row (kc_select only) */
  const uint32_t* bank_band_ids;   /* [R] band of each bank row (kc_select only) */
} kc_mask_rule;

/* A packed ragged batch: frame f owns records rec_off[f] .. rec_off[f+1]-1,
 * every record active and in order (packHostFrame's layout). Questions are
 * numbered across the batch in frame order, then slot order. */
typedef struct kc_batch_view {
  uint32_t frames;
  uint64_t records;              /* rec_off[frames] */
  const uint64_t* rec_off;       /* [frames+1] */
  const uint32_t* token_ids;     /* [records*8] */
  const uint32_t* field_roles;   /* [records*8] */
  const uint32_t* schema_ids;    /* [records] */
  const uint32_t* band_ids;      /* [records] */
  const uint32_t* schema_allow;  /* optional rule, [batch questions * 8] */
  const uint32_t* band_allow;    /* optional rule, [batch questions] */
  const double* uniforms;        /* optional: sample instead of argmax, [batch questions] */
  /* Optional same-word bias on the encoder's record-local attention (WordBias,
   * forward/masks.ts:145-198): word_ids [records*8] parallel to token_ids,
   * 0xffffffff = no word; two tokens of one record with the same word id get
   * word_alpha (stored f32) added to their attention logit. word_alpha = 0 or
   * word_ids NULL: no bias. The backward entry points ignore it, as the
   * session's gradient source passes no record mask (host/gradients.ts:30-66),
   * and so does the streaming packer. */
  const uint32_t* word_ids;
  float word_alpha;
  /* Optional explicit selection mask laid out like p ([sum_f Q_f R_f], frame
   * f's [Q_f, R_f] block at p_off[f]): added to every score, as selectorOracle
   * adds selectionMask's rows (forward/oracle.ts:340-345; NEG_INF -1e30 =
   * blocked, 0 = open; host/learn.ts:215-232 builds it from any allows(q, r)
   * closure, a row nothing admits reopened). For grammars that are not a
   * schema x band product. Exclusive with schema_allow / band_allow. Not taken
   * by the streaming packer. */
  const float* mask;
} kc_batch_view;

/* Outputs of a batch. p of frame f is a [Q_f, R_f] block at p_off[f]; the
 * indices of its questions start at q_off[f]. Questions of a frame whose bank
 * is empty get KC_NO_SELECTION (the session returns no selection for them,
 * session.ts:133). */
typedef struct kc_batch_out {
  float* p;                /* [total_p] */
  uint64_t p_capacity;
  uint32_t* index;         /* [total_q] */
  uint64_t q_capacity;
  uint64_t* p_off;         /* optional [frames+1] */
  uint64_t* q_off;         /* optional [frames+1] */
  float* query_output;     /* optional [total_q, H] */
  uint64_t total_p, total_q, total_r, total_t; /* written by the call */
} kc_batch_out;

/* Library-owned device results of kc_forward_batch_device, valid until the
 * next call on the handle. */
typedef struct kc_device_result {
  const float* p;
  const uint32_t* index;
  const uint64_t* p_off;
  const uint64_t* q_off;
  uint64_t total_p, total_q, total_r, total_t;
} kc_device_result;

/* Per-stage device time, accumulated while profiling is on. */
typedef struct kc_stage_times {
  double pack_ms, embed_ms, enc_gemm_ms, enc_attn_ms, pool_ms, mixer_ms, selector_ms, total_ms;
  uint64_t enc_gemm_launches, launches, batches;
  double enc_gemm_flops;    /* algorithmic FLOPs of the encoder GEMMs timed */
  double fallback_ms;       /* exact recomputation of uncertified frames */
  uint64_t fallback_frames; /* frames recomputed (counted whether or not profiling is on) */
  double enc_gemm_bytes;    /* algorithmic bytes of the encoder GEMMs timed (A read, C written) */
  /* the fused feed-forward kernel (W1, ReLU, W2, residual in one launch) */
  double enc_ffn_ms;
  uint64_t enc_ffn_launches;
  double enc_ffn_flops, enc_ffn_bytes;
  /* the fused attention kernel (q|k|v projection, record-local attention,
     residual in one launch): its time, launches and algorithmic FLOPs
     (the projection) and bytes (x read and written) */
  double enc_attn_tc_ms;
  uint64_t enc_attn_tc_launches;
  double enc_attn_tc_flops, enc_attn_tc_bytes;
  /* the certificate's audit: every frame recomputed exactly has each fast
     score compared with its exact score; the largest |s^ - s| / B seen
     (B the margin the selector allowed), the batches where it exceeded 1
     (each raises the margin fourfold for later batches), the frames audited,
     and the base margin kappa0 in force (counted whether or not profiling is on) */
  double cert_audit_max;
  uint64_t cert_audit_violations;
  uint64_t cert_audit_frames;
  double cert_kappa0;
  /* the exact path's products on the int8 tensor cores (counted whether or
     not profiling is on): products run, their outputs, the outputs whose
     error interval straddled an f32 rounding boundary (recomputed by the
     sequential chain), and forwards sent again through the FP64 kernel
     because a product listed more outputs than its list holds */
  uint64_t oz_products;
  double oz_outputs;
  uint64_t oz_listed;
  uint64_t oz_reruns;
} kc_stage_times;

uint32_t kc_abi_version(void);

/* BrainBackendFactory (host/backend.ts:177-180): copy the weights to `device`
 * and return a handle. */
kc_status kc_create(const kc_config* config, const kc_weights_view* weights, int device, kc_handle** out);

/* BrainBackend.sync (host/backend.ts:167). changes == NULL means everything. */
kc_status kc_sync(kc_handle* h, const kc_weights_view* weights, const kc_changes* changes);

/* BrainBackend.encode (host/backend.ts:149) for one frame. Outputs are
 * [Q,H], [R,H], [R,H]; *q_out / *r_out receive Q and R. q_cap / r_cap are the
 * rows the output buffers hold. A frame without a question is refused, as
 * the WebGPU runner refuses it (webgpu/src/krystal-forward.ts:216). */
kc_status kc_encode(kc_handle* h, const kc_frame_view* frame, float* query_output, float* bank_keys,
                    float* bank_values, uint32_t q_cap, uint32_t r_cap, uint32_t* q_out, uint32_t* r_out);

/* selectorOracle (forward/oracle.ts:332-382) on the device: score, mask,
 * softmax, first-max argmax (or an inverse-CDF draw when uniforms != NULL,
 * forward/sampling.ts:41-57), soft gather. mask: [Q,R] (NEG_INF -1e30 =
 * blocked) or NULL; rule: the device form of the grammar or NULL; both NULL
 * = open. p: [Q,R]; index: [Q]; gather: [Q,H] or NULL. */
kc_status kc_select(kc_handle* h, const kc_encoded_view* encoded, const float* mask, const kc_mask_rule* rule,
                    const double* uniforms, float* p, uint32_t* index, float* gather);

/* The selector of kc_select over DEVICE pointers, allocating no device memory.
 * No counterpart in the reference: it exists for callers that cannot call
 * cudaMalloc at the point they select — code running inside CUDA stream
 * capture, real-time loops that forbid allocation, or hosts whose memory is
 * handed out by their own pool. Its scratch is one static device array of
 * about 2.2 MB that every GPU loading this library holds until exit; it caps
 * a call at 256 questions and KC_MAX_BANK bank rows (KC_ERR_CAPACITY above).
 * Inputs [Q,H], [R,H], [R,H] (bank_values only needed for the gather), mask
 * [Q,R] or NULL; outputs p [Q,R], index [Q], gather [Q,H] or NULL. Work is
 * queued on the handle's stream and the call returns without waiting. The
 * first call on a device looks up the scratch's device address; make that
 * first call before any stream capture. All calls share the one scratch
 * array, so calls whose GPU work overlaps (two streams, two handles on one
 * device) race: serialise them. */
kc_status kc_select_noalloc(kc_handle* h, uint32_t q, uint32_t r, const float* query_output, const float* bank_keys,
                            const float* bank_values, const float* mask, float* p, uint32_t* index, float* gather);

/* Whole-batch think: pack on the GPU, encode, select. Host buffers; the
 * host<->device copies are part of the call. */
kc_status kc_forward_batch(kc_handle* h, const kc_batch_view* batch, kc_batch_out* out);

/* consider / choose reuse at batch scale (host/session.ts:128-176: consider()
 * encodes once, each choose() selects again under its own mask): the last
 * batch kc_forward_batch ran on this handle, selected again under a new mask
 * rule (per question, laid out as in kc_batch_view) and/or new uniforms
 * (NULL: argmax), without encoding it again. At the batch's precision; in
 * the certified mode frames it cannot certify are recomputed on the exact
 * path as in kc_forward_batch. The batch is resident until any other call on
 * the handle that packs or selects (kc_forward_batch again, kc_encode,
 * kc_select, the backward and learn calls, a stream's batches) or changes
 * weights (kc_sync, kc_load_checkpoint); KC_ERR_INVALID_ARG otherwise.
 * Results as for kc_forward_batch. */
typedef struct kc_batch_select_view {
  const uint32_t* schema_allow;  /* [Q * 8] or NULL (the open mask) */
  const uint32_t* band_allow;    /* [Q], NULL with schema_allow */
  const double* uniforms;        /* [Q] or NULL */
  const float* mask;             /* [total_p] explicit mask laid out like p, or NULL; exclusive with the rule */
} kc_batch_select_view;

kc_status kc_select_batch(kc_handle* h, const kc_batch_select_view* select, kc_batch_out* out);

/* As kc_forward_batch, but every array in `batch` is a DEVICE pointer on the
 * handle's device. Work is queued on the handle's stream; the call returns
 * once the result is queued (one short host wait inside, for the batch's
 * sizes). Results are library-owned device arrays. */
kc_status kc_forward_batch_device(kc_handle* h, const kc_batch_view* batch, kc_device_result* out);

/* BackwardRequest (host/backend.ts:74-94) targets: a bank row, KC_NO_TARGET
 * (NO_TARGET, :42), or a bank row | KC_AWAY_TARGET (AWAY, :58: push
 * probability away from that row). */
#define KC_NO_TARGET 0xffffffffu
#define KC_AWAY_TARGET 0x80000000u

/* BackwardResult (host/backend.ts:105-123) of one frame, host buffers the
 * caller sizes from the frame: Q questions, R bank records, T non-PAD tokens
 * of the active records (active-token order, compileActiveFrame). */
typedef struct kc_backward_out {
  float* policy;            /* [Q*R] */
  float* value_prediction;  /* [Q] */
  double value_loss;        /* written by the call */
  float* d_selector_wq;     /* [H*H] */
  float* d_selector_wk;     /* [H*H] */
  float* d_pool;            /* [2*H] */
  float* d_field_states;    /* [T*H], may be NULL */
  float* d_value_wv;        /* [3*H] */
  uint64_t p_capacity, q_capacity, t_capacity; /* elements of policy, value_prediction, d_field_states/H */
  uint32_t q, r, t;         /* written by the call */
} kc_backward_out;

/* BrainBackend.backward (host/backend.ts:158) for one frame:
 * brainBackwardOracle (forward/backward.ts:751-982) as host/gradients.ts:
 * 30-66 requests it (context "available", open mixer mask, the argument slot
 * aimed at nothing). selection: [Q,R] mask (-1e30 blocked, 0 open), NULL =
 * open. targets: [Q] or NULL. has_valence = 0: no value target. Computed in
 * the reference's exact arithmetic. */
kc_status kc_backward(kc_handle* h, const kc_frame_view* frame, const float* selection, const uint32_t* targets,
                      int has_valence, double valence, kc_backward_out* out);

/* Library-owned device results of kc_backward_batch_device, valid until the
 * next call on the handle. Per-frame arrays are indexed by frame. */
typedef struct kc_backward_result {
  const float* policy;            /* [total_p], frame f at p_off[f] */
  const float* value_prediction;  /* [total_q] */
  const double* value_loss;       /* [frames] */
  const float* d_selector_wq;     /* [frames, H, H] */
  const float* d_selector_wk;     /* [frames, H, H] */
  const float* d_pool;            /* [frames, 2H] */
  const float* d_field_states;    /* [total_t, H], frame f at t_off[f] */
  const float* d_value_wv;        /* [frames, 3H] */
  const uint64_t *p_off, *q_off, *r_off, *t_off; /* [frames+1] */
  uint64_t total_p, total_q, total_r, total_t;
} kc_backward_result;

/* The backward of every frame of a packed batch at once (learn and teach
 * differentiate many frames against one set of weights, host/learn.ts:
 * 318-400). DEVICE pointers: `batch` as for kc_forward_batch_device;
 * selection [total_p] laid out like p, or NULL (then the batch's mask rule,
 * or open when it has none); targets [total_q] or NULL; valence [frames] with
 * NaN = no value target, or NULL = none. Work is queued on the handle's
 * stream; the call waits for the batch's sizes and, on the tensor-core path,
 * for the pipeline's error word (a split overflow reruns the batch exactly). */
kc_status kc_backward_batch_device(kc_handle* h, const kc_batch_view* batch, const float* selection,
                                   const uint32_t* targets, const double* valence, kc_backward_result* out);

/* learnFromExperience's per-frame readings (host/learn.ts:318-400) of the
 * last batch kc_backward_batch_device differentiated on this handle. stats:
 * DEVICE [frames * KC_LEARN_STATS] f64, per frame: questions, bank rows,
 * baseline (mean valuePrediction), valueLoss, entropy total and rows,
 * confidence total and rows (the report's terms, learn.ts:372-389; targets:
 * DEVICE [total_q] bank rows or KC_NO_TARGET, NULL = none). Queued on the
 * handle's stream. */
#define KC_LEARN_STATS 8
kc_status kc_learn_frame_stats(kc_handle* h, const uint32_t* targets, double* stats);

/* The batch gradients the update applies (host/learn.ts:440-470), over the
 * last batch differentiated: sums = [sum_f step[f]*dSelectorWq_f (H*H) |
 * sum_f step[f]*dSelectorWk_f (H*H) | sum_f step[f]*dPool_f (2H) |
 * sum_f value_weight[f]*dValueWv_f (3H)], f64. step / value_weight: DEVICE
 * [frames] f64 (0 leaves a frame out); sums: DEVICE [2H*H + 5H] f64. With
 * several GPUs, these per-rank sums are what an all-reduce adds. */
kc_status kc_learn_accumulate(kc_handle* h, const double* step, const double* value_weight, double* sums);

/* The update half of learnFromExperience (host/learn.ts:318-512) on the
 * device, in stream order, so that a learn step needs no host round trip
 * between the backward and the next forward. All pointers are DEVICE
 * pointers unless named host. The options are LearnOptions (learn.ts:61-139)
 * with the reference's defaults (:292-299): learning_rate 0.05, policy_scale
 * 1, advantage_clip 3, max_parameter_abs +inf, token_rate 0.1 (unfreeze.
 * tokenRate), unfreeze_pool / unfreeze_tokens 0. */
typedef struct kc_learn_options {
  double learning_rate, policy_scale, advantage_clip, max_parameter_abs, token_rate;
  int32_t unfreeze_pool, unfreeze_tokens;
} kc_learn_options;
#define KC_LEARN_ROW 10    /* the KC_LEARN_STATS readings, the reward (NaN = none), answered (0 / 1) */
#define KC_LEARN_REPORT 9  /* seen, actor moved, reinforced, discouraged, mean advantage, mean value loss,
                              mean entropy, mean confidence, frames pending */
#define KC_LEARN_RESULT 19 /* applied, rejected (0 none, 1 "non-finite", 2 "parameter-limit"), finite, health
                              maxima (table rows, selector, value head, pool, selector Wq, selector Wk),
                              table rows touched, then the plan's KC_LEARN_REPORT values */
/* The plan (learn.ts:318-470) over every frame of a batch in frame order —
 * with several GPUs, the all-gathered rows of every rank, so that every rank
 * plans the same update: rows [frames, KC_LEARN_ROW] f64 -> step,
 * value_weight (kc_learn_accumulate's weights) and pending (the frames whose
 * gradients the actor takes) [frames] f64, report [KC_LEARN_REPORT] f64.
 * Every sum is a running sum in frame order, as the reference's loop. */
kc_status kc_learn_plan(kc_handle* h, const double* rows, uint32_t frames, const kc_learn_options* options,
                        double* step, double* value_weight, double* pending, double* report);
/* Unfrozen tables (scatterEmbeddings, learn.ts:242-263, as one sum per
 * row): over the last batch differentiated (whose token_ids / field_roles
 * are passed again), row_sums [token_space + field_space, H] f64 gain
 * step[f] * dFieldStates of every token of a pending frame at its token row
 * and at token_space + its field row; touched [token_space + field_space]
 * is set to 1 for those rows. Both must start at zero; several GPUs add
 * them with one all-reduce. step / pending: this rank's frames. */
kc_status kc_learn_accumulate_rows(kc_handle* h, const uint32_t* token_ids, const uint32_t* field_roles,
                                   const double* step, const double* pending, double* row_sums, double* touched);
/* The update itself on the device's weight page (learn.ts:427-470) from the
 * (all-reduced) sums of kc_learn_accumulate, and of kc_learn_accumulate_rows
 * when unfreeze_tokens (else NULL), and kc_learn_plan's report; then
 * parameterHealth (:187-205), the rejection rule and the rollback
 * (:477-495). Waits for the device; result (HOST, [KC_LEARN_RESULT] f64)
 * reports it, its health that of the arrays as left, followed by a copy of
 * the report. The weights the caller
 * holds on the host are not touched: read them back with kc_copy_weights. */
kc_status kc_learn_apply(kc_handle* h, const double* sums, const double* row_sums, const double* touched,
                         const double* report, const kc_learn_options* options, double* result);
/* count floats of the device weight page from offset (createBrainForwardWeights
 * order) into host memory; waits for the device. */
kc_status kc_copy_weights(kc_handle* h, uint64_t offset, uint64_t count, float* host);

/* KRY1 checkpoints (host/checkpoint.ts:17-116): 11 little-endian u32 header
 * words (magic "KRY1" = 0x4b525931, version 1, hiddenSize, ffnSize,
 * encoderBlocks, mixerBlocks, headCount, headDim, routeKindCount, tokenRows
 * length, weight element count), the tokenRows, then every weight array in
 * createBrainForwardWeights order, which is the device page's order. */
#define KC_CHECKPOINT_MAGIC 0x4b525931u
#define KC_CHECKPOINT_VERSION 1u
typedef enum kc_checkpoint_refusal {  /* CheckpointRefusal (checkpoint.ts:44-49) */
  KC_CHECKPOINT_FITS = 0,
  KC_CHECKPOINT_NOT_KRYSTAL = 1,      /* "not a krystal checkpoint" */
  KC_CHECKPOINT_LATER_FORMAT = 2,     /* "a later checkpoint format" */
  KC_CHECKPOINT_GEOMETRY = 3,         /* "a different geometry" */
  KC_CHECKPOINT_VOCABULARY = 4,       /* "a different vocabulary" */
  KC_CHECKPOINT_TRUNCATED = 5         /* "truncated" */
} kc_checkpoint_refusal;

/* decodeCheckpoint (checkpoint.ts:78-116) straight into the device weight
 * page: the same checks against the handle's geometry and tokenRows, then one
 * host-to-device copy; `bytes` may start anywhere. A refusal leaves the
 * device weights untouched and returns KC_OK with *refusal set; the host's own
 * arrays are the caller's to decode. */
kc_status kc_load_checkpoint(kc_handle* h, const void* bytes, uint64_t len, int* refusal);
/* encodeCheckpoint (checkpoint.ts:51-69) from the device weight page:
 * *written = the checkpoint's size; nothing is written when cap is smaller
 * (KC_ERR_CAPACITY), so a NULL out with cap 0 asks for the size. */
kc_status kc_save_checkpoint(kc_handle* h, void* out, uint64_t cap, uint64_t* written);

/* Streaming packer: frames that arrive one at a time (one think() per turn
 * of many sessions, host/session.ts:128-181) leave in rolling packed batches.
 * kc_stream_push copies a frame's active records into the open pinned staging
 * buffer and validates them there (a malformed frame is refused alone);
 * kc_stream_flush seals that buffer and queues it; a worker thread runs sealed
 * buffers back to back through the batch path (the handle's precision) while
 * the caller keeps pushing into the next buffer; kc_stream_poll hands back the
 * oldest finished batch. No counterpart in the reference, which thinks about
 * one frame per call. Destroy a stream before its handle. */
typedef struct kc_stream kc_stream;

typedef struct kc_stream_result {
  uint64_t first_ticket;   /* the batch holds tickets first_ticket .. first_ticket + frames - 1 */
  uint32_t frames;         /* 0: nothing finished */
  uint64_t questions, total_p;
  const uint64_t* p_off;   /* [frames+1] */
  const uint64_t* q_off;   /* [frames+1] */
  const float* p;          /* [total_p] */
  const uint32_t* index;   /* [questions] */
  kc_status status;        /* the batch's own status; error: its message or NULL */
  const char* error;
  double sealed_ms, done_ms; /* kc_stream_clock_ms() at flush and when the results landed */
  double started_ms;       /* kc_stream_clock_ms() when the worker took the batch up */
  double sync_wait_ms;     /* of done_ms - started_ms, the worker's time blocked until the device finished */
} kc_stream_result;

/* Placement and helpers of a stream (kc_stream_create uses {0, 1}).
 * push_threads: the threads a large kc_stream_push_many call validates and
 * stages with, the caller's included; 0 picks one per 4 CPUs local to the GPU,
 * at most 8; 1 is the caller alone. bind_cpus != 0: the worker and the helpers
 * run on the CPUs sysfs lists as local to the GPU (local_cpulist, as far as
 * this process may use them), and the worker allocates the pinned staging, so
 * that its pages lie on the GPU's NUMA node. */
typedef struct kc_stream_options {
  uint32_t push_threads;
  int32_t bind_cpus;
} kc_stream_options;

/* Where a stream's host time went (kc_stream_read_stats; the counters since
 * the last reset). Fault and switch counts are getrusage(RUSAGE_THREAD)
 * differences over the worker's batches and the callers' push_many calls. */
typedef struct kc_stream_stats {
  uint64_t batches;                    /* batches the worker finished */
  uint64_t push_calls, frames_pushed;  /* kc_stream_push / _push_many calls and the frames they queued */
  uint64_t bytes_staged;               /* record and rule bytes copied into the staging */
  double push_ms;                      /* time inside push calls (checks and staging copies) */
  double run_ms;                       /* worker: time inside batches */
  double sync_wait_ms;                 /* worker: of run_ms, blocked until the device finished */
  double idle_ms;                      /* worker: waiting for a sealed buffer */
  uint64_t workspace_grows;            /* device workspace reallocations inside batches */
  double workspace_grow_ms;
  uint64_t worker_minor_faults, worker_major_faults;
  uint64_t worker_voluntary_switches, worker_involuntary_switches;
  uint64_t worker_cpu_moves;           /* batches that ended on another CPU than they began on */
  uint64_t caller_minor_faults, caller_involuntary_switches;
  int32_t gpu_numa_node;               /* sysfs numa_node of the GPU; -1 unknown */
  int32_t staging_numa_node;           /* node of the first staging page; -1 unknown */
  int32_t worker_numa_node;            /* node of the worker's CPU at its last batch */
  int32_t caller_numa_node;            /* node of the CPU of the last push_many call */
  uint32_t push_threads;               /* threads a large push_many uses */
  uint32_t bound_cpus;                 /* CPUs the worker and helpers are bound to (0: unbound) */
} kc_stream_stats;

/* depth >= 2 staging buffers, each for up to max_frames frames, max_records
 * records and max_p p entries (0: 64 per record). Pinned host memory only. */
kc_status kc_stream_create(kc_handle* h, uint32_t max_frames, uint64_t max_records, uint64_t max_p, uint32_t depth,
                           kc_stream** out);
/* kc_stream_create with the placement and helpers of *opts (NULL: {0, 1}). */
kc_status kc_stream_create_ex(kc_handle* h, uint32_t max_frames, uint64_t max_records, uint64_t max_p,
                              uint32_t depth, const kc_stream_options* opts, kc_stream** out);
/* Queue one packed frame (kc_frame_view as for kc_encode). schema_allow /
 * band_allow: the frame's questions' rule ([Q*8], [Q]) or both NULL (open).
 * *ticket numbers the frame (consecutive from 0). KC_ERR_CAPACITY when the
 * open buffer is full (flush) or every buffer is in flight (poll). */
kc_status kc_stream_push(kc_stream* s, const kc_frame_view* frame, const uint32_t* schema_allow,
                         const uint32_t* band_allow, uint64_t* ticket);
/* Queue a run of packed frames in one call, as kc_stream_push would one by
 * one: frame f is records rec_off[f] .. rec_off[f+1]-1 of the arrays
 * (rec_off[0] need not be 0), every record active; the rule, if given, is per
 * question of these frames in order. *pushed counts the frames queued before
 * a refusal; their tickets start at *first_ticket. */
kc_status kc_stream_push_many(kc_stream* s, const kc_batch_view* frames, uint64_t* first_ticket, uint32_t* pushed);
/* Seal the open buffer and queue it for the device; returns at once. */
kc_status kc_stream_flush(kc_stream* s);
/* Batches sealed but not finished. */
uint32_t kc_stream_pending(kc_stream* s);
/* The oldest finished batch (wait != 0: block until one finishes, unless none
 * is queued). Its arrays stay valid until the next poll. */
kc_status kc_stream_poll(kc_stream* s, int wait, kc_stream_result* out);
/* The stream's host-side counters (reset != 0: zeroed after reading; the
 * placement fields stay). */
kc_status kc_stream_read_stats(kc_stream* s, int reset, kc_stream_stats* out);
/* The steady clock the stream's timestamps use, in milliseconds. */
double kc_stream_clock_ms(void);
const char* kc_stream_last_error(kc_stream* s);
/* Finishes the batch running, discards the rest. */
void kc_stream_destroy(kc_stream* s);

/* Precision of the batch entry points (KC_PRECISION_*); tau > 0 also sets the
 * certificate's base relative margin kappa0 (default 2e-5; 0 keeps it). */
kc_status kc_set_precision(kc_handle* h, int mode, float tau);

/* Test hook for the failure path, no counterpart in the reference: the next
 * launch of one tensor-core kernel (KC_INJECT_ATTN: the fused encoder
 * attention; KC_INJECT_FFN: the fused feed-forward; KC_INJECT_GEMM: the
 * projection GEMM; KC_INJECT_EXACT_GEMM: the exact path's int8 product)
 * behaves as if its producer's first bounded wait had
 * expired, before it issues any copy: the kernel raises the error word,
 * every warp role leaves, TMEM is freed, and the batch call returns
 * KC_ERR_TIMEOUT with kc_last_error naming the expired wait. One shot; the
 * handle stays usable. Nothing faults or hangs: no wait actually runs out. */
#define KC_INJECT_ATTN 0
#define KC_INJECT_FFN 1
#define KC_INJECT_GEMM 2
#define KC_INJECT_EXACT_GEMM 3  /* the exact path's int8 tensor-core product */
kc_status kc_inject_wait_expiry(kc_handle* h, int kernel);

/* Stream control: run on `stream` (a cudaStream_t; NULL = the handle's own). */
kc_status kc_set_stream(kc_handle* h, void* stream);
void* kc_get_stream(kc_handle* h);
kc_status kc_synchronize(kc_handle* h);

/* Profiling: per-stage CUDA-event timing (adds events between stages). */
kc_status kc_profile(kc_handle* h, int enable);
kc_status kc_profile_read(kc_handle* h, kc_stage_times* out, int reset);
/* Kernel launches the handle has issued since creation. */
uint64_t kc_launch_count(kc_handle* h);

/* BrainBackend.destroy (host/backend.ts:168). */
void kc_destroy(kc_handle* h);

/* Last error message for the handle (or the last failed kc_create if NULL). */
const char* kc_last_error(kc_handle* h);

#ifdef __cplusplus
}
#endif
#endif
