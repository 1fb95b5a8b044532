/*
 * krystal_oracle.h — CPU restatement of Krystal's frame forward and selector.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker: the parity tests,
 * the smoke check and the benchmark's CPU-baseline leg call it to say what the
 * right answer is, and to time the reference algorithm on host cores. Nothing
 * in the product links, loads or calls it.
 *
 * It restates the reference TypeScript oracle line for line (packages/krystal/
 * src/forward/{model,masks,oracle,sampling}.ts and host/learn.ts selectionMask)
 * with the JavaScript numeric semantics kept exactly:
 *   - every intermediate is an IEEE f64 ("number");
 *   - every store into a Float32Array rounds to f32 (round to nearest even);
 *   - the loop orders are the reference's, so f64 sums associate identically;
 *   - the build uses -ffp-contract=off so no a*b+c is fused behind our back.
 * The reference's Math.exp/log/sin/cos are f64 library calls; glibc's are
 * used here and may differ from V8's by at most 1 ulp in f64, which the f32
 * store hides except with probability ~1e-8 per value.
 *
 * Parity pin: the reference's own TypeScript (weights, packing, forward,
 * selection with masks and sampling, the same-word bias, the session
 * backward, learn and teach) was executed on the inputs of the golden
 * fixtures by a runner that keeps JavaScript's number semantics
 * (tests/golden/tsrun.py, tests/golden/make_reference_golden.py); this
 * restatement reproduces those outputs bit for bit
 * (tests/test_reference_golden.py). It is also checked against every
 * known-answer test the reference's test files hold and against an
 * independent numpy re-implementation of the forward.
 */
#ifndef KRYSTAL_ORACLE_H
#define KRYSTAL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* BrainForwardConfig geometry (packages/krystal/src/forward/model.ts:27-80).
 * The six table row counts are parameters here; the reference fixes them at
 * module load from the default profile (model.ts:92-99). */
typedef struct ko_dims {
  uint32_t hidden, heads, head_dim, ffn, enc_blocks, mixer_blocks;
  uint32_t token_space, field_space, schema_space, band_space, stream_space, pos_space;
  uint32_t route_kinds;
} ko_dims;

/* Flat weight page, in createBrainForwardWeights generation order
 * (model.ts:233-265): embeddings page, enc[b].{wq,wk,wv,w1,w2}, pool,
 * mixer[b].{...}, selector.wq, selector.wk, decisionHeadWh, valueHeadWv. */
uint64_t ko_weight_count(const ko_dims* d);
void ko_create_weights(const ko_dims* d, uint32_t seed, float* out);
/* Element offset of each named array inside the flat page. which:
 * 0 embeddings, 1 enc, 2 pool, 3 mixer, 4 sel_wq, 5 sel_wk, 6 decision, 7 value.
 * For 1/3 the offset is of block 0; blocks follow each other. */
uint64_t ko_weight_offset(const ko_dims* d, int which);

/* mulberry32 draws (model.ts:186-195), for KATs. */
void ko_mulberry32(uint32_t seed, uint32_t n, double* out);

/* y = x · Wᵀ, W [out,in] row-major (oracle.ts:114-125). */
void ko_matmul(const float* x, const float* w, uint32_t rows, uint32_t out_dim, uint32_t in_dim, float* y);
/* In-place softmaxRow (oracle.ts:38-49). */
void ko_softmax_row(float* v, uint32_t count);
/* sampleRow (sampling.ts:41-57). */
int32_t ko_sample_row(const float* p, uint32_t count, double uniform);

/* compileActiveFrame (masks.ts:65-101). Outputs are sized by `slots`
 * (active_tokens by slots*8). Returns T; *r_out / *q_out get R / Q. */
uint32_t ko_compile_active(uint32_t slots, const uint32_t* token_ids, const uint32_t* band_ids,
                           const uint32_t* active_record_indices, uint32_t* active_tokens,
                           uint32_t* rec_offset, uint32_t* rec_count, uint32_t* stream_ids,
                           uint32_t* bank_records, uint32_t* query_records, uint32_t* r_out,
                           uint32_t* q_out, uint32_t* active_count_out);

/* brainForwardOracle (oracle.ts:231-299) for one packed frame.
 * mixer_mask: [Q,R] or NULL for the open (all-zero) mask the session uses.
 * Outputs sized [T,H], [R,H], [R,H], [Q,H], [Q,H], [Q,H]; any may be NULL
 * except query_output/bank_keys/bank_values. word_ids [slots*8] (frame token
 * order, 0xffffffff = no word) with alpha != 0 adds the same-word bias to the
 * encoder's record mask (WordBias, masks.ts:145-198); NULL / 0 for none.
 * Returns 0, or -1 on a bad frame. */
int ko_forward(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
               uint32_t slots, const uint32_t* token_ids, const uint32_t* field_roles,
               const uint32_t* schema_ids, const uint32_t* band_ids, const uint32_t* active_record_indices,
               const float* mixer_mask, float* field_states, float* bank_keys, float* bank_values,
               float* query_keys, float* query_values_premix, float* query_output, const uint32_t* word_ids,
               float alpha);

/* selectorOracle (oracle.ts:332-382). uniforms: [Q] or NULL (argmax).
 * gather may be NULL. */
void ko_selector(const float* query, const float* bank_keys, const float* bank_values, const float* mask,
                 const float* sel_wq, const float* sel_wk, uint32_t q, uint32_t r, uint32_t h,
                 const double* uniforms, float* p, float* gather, uint32_t* index);

/* selectionMask (host/learn.ts:215-232) for the device-side rule form of
 * `allows`: question i admits bank slot s iff bit schema[s] of
 * schema_allow[i*8 .. i*8+8) and bit band[s] of band_allow[i] are set. */
void ko_selection_mask_rule(uint32_t q, uint32_t r, const uint32_t* bank_records, const uint32_t* schema_ids,
                            const uint32_t* band_ids, const uint32_t* schema_allow, const uint32_t* band_allow,
                            float* mask);

/* Packed ragged batch, packHostFrame form (host/frame.ts:72-115: every slot
 * active, in order). Frame f owns records [rec_off[f], rec_off[f+1]).
 * Per frame: forward (open mixer mask), then selector under the rule mask
 * (or open mask when schema_allow is NULL); sampling when uniforms != NULL
 * (one per question, in batch question order).
 * p_off[f] / q_off[f] (size F+1) are written: frame f's p rows start at
 * p_off[f] (Q_f*R_f floats) and its indices at q_off[f].
 * Frames run in parallel over `threads` host threads (0 = all). word_ids
 * [records*8] and alpha: the same-word bias as for ko_forward.
 * Returns 0, or -1 on a bad frame. */
int ko_forward_batch(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
                     uint32_t frames, const uint64_t* rec_off, const uint32_t* token_ids,
                     const uint32_t* field_roles, const uint32_t* schema_ids, const uint32_t* band_ids,
                     const uint32_t* schema_allow, const uint32_t* band_allow, const double* uniforms,
                     int threads, uint64_t* p_off, uint64_t* q_off, float* p, uint32_t* index,
                     float* query_output, const uint32_t* word_ids, float alpha);

/* Sizes of a batch without running it: fills p_off/q_off/t_off (F+1 each). */
void ko_batch_offsets(uint32_t frames, const uint64_t* rec_off, const uint32_t* token_ids,
                      const uint32_t* band_ids, uint64_t* p_off, uint64_t* q_off, uint64_t* r_off, uint64_t* t_off);

/* brainBackwardOracle (forward/backward.ts:751-982) as host/gradients.ts:
 * 30-66 runs it for a session: context "available", the argument slot given
 * nothing to aim at, no route-kind labels. selection: [Q,R] mask; targets:
 * [Q] (0xffffffff = none, top bit = push away) or NULL; has_valence selects
 * whether the value head has a target. Outputs are BackwardResult
 * (host/backend.ts:220-238): policy [Q,R], value_prediction [Q], value_loss,
 * d_selector_wq/wk [H,H], d_pool [2,H], d_field_states [T,H], d_value_wv [3H]. */
int ko_backward(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
                uint32_t slots, const uint32_t* token_ids, const uint32_t* field_roles, const uint32_t* schema_ids,
                const uint32_t* band_ids, const uint32_t* active_record_indices, const float* selection,
                const uint32_t* targets, int has_valence, double valence, float* policy, float* value_prediction,
                double* value_loss, float* d_selector_wq, float* d_selector_wk, float* d_pool,
                float* d_field_states, float* d_value_wv);

int ko_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
