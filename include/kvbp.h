/*
 * kvbp.h -- C ABI of the B200 (sm_100a) capped-KV decode path.
 *
 * One decode step of GQA attention over a globally capped KV cache, fused with the
 * eviction policy's per-slot score update, the structural prefix/suffix protection,
 * victim selection and the scatter of the new K/V into a free slot.  The reference
 * (Gpgabriel25/KVCacheBoundaryProtection) has no FFI; these entry points are what its
 * JAX decode loop would bind through a jax.ffi / XLA custom call.  Each declaration
 * names the reference code it replaces (paths inside the reference project).
 *
 * Conventions
 *  - Every entry point is stateless and enqueue-only on ``stream`` (a cudaStream_t):
 *    no host synchronisation, no device allocation.  The caller owns every buffer.
 *  - Return value: KVBP_OK, or a KVBP_ERR_* code for an argument / shape / launch
 *    error detected on the host before or at launch; kvbp_last_error() then holds a
 *    message (thread-local).
 *  - Problems found on the device are OR-ed into the caller's int32 ``dev_err`` word
 *    (KVBP_DEV_* bits; may be NULL).  Kernels never trap; every wait is bounded.
 *  - Tensors are dense row-major; "bf16" means IEEE bfloat16 bit patterns.
 *  - Slot layout: a sequence's cache holds S slots.  slot_pos[b][s] is the absolute
 *    position stored in slot s, or -1 when the slot is free.  After step 0 the retained
 *    prompt positions fill slots 0..R-1 in ascending order; each decode step's new
 *    position takes the lowest free slot before that step's eviction; victims' slots
 *    become free.
 */
#ifndef KVBP_H
#define KVBP_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kvbp_stream_t; /* == cudaStream_t */

#define KVBP_OK 0
#define KVBP_ERR_ARG 1
#define KVBP_ERR_UNSUPPORTED 2
#define KVBP_ERR_CUDA 3

#define KVBP_DEV_NO_FREE_SLOT 1
#define KVBP_DEV_NAN_SCORE 2
#define KVBP_DEV_INDEX 4
#define KVBP_DEV_WAIT_TIMEOUT 8
#define KVBP_DEV_NO_VALID_SLOT 16
#define KVBP_DEV_LOG_OVERFLOW 32
#define KVBP_DEV_PEER_TIMEOUT 64

/* Policy ids: the reference CLI names (scripts/run_v3_jax.py:145-148, built at
 * :500-518); "attention-mass" is an alias of "h2o_faithful". */
#define KVBP_POLICY_LRU 0
#define KVBP_POLICY_H2O_FAITHFUL 1
#define KVBP_POLICY_H2O 2
#define KVBP_POLICY_SNAPKV 3
#define KVBP_POLICY_SNAPKV_FAITHFUL 4
#define KVBP_POLICY_ADAKV 5
#define KVBP_POLICY_QUEST 6
#define KVBP_POLICY_STREAMINGLLM 7
#define KVBP_POLICY_RANDOM 8 /* victims sampled on the host: kvbp_append_evict_listed */

const char* kvbp_version(void);
const char* kvbp_last_error(void);
/* Policy id for a reference policy name, or -1. */
int kvbp_policy_id(const char* name);

/* Per-sequence eviction state (device pointers).  Arrays are [B][S] except posmap,
 * which is [B][W]: bit p of sequence b is set while position p is retained. */
typedef struct kvbp_state {
  int32_t B, S, W;
  int32_t* slot_pos;
  int32_t* insert_step;
  int32_t* last_access;
  int32_t* access_count;
  float* attn;      /* latest per-step score                  (KVBlockMetadata.attention_score) */
  float* max_attn;  /* running max of per-step scores         (.max_attention_score) */
  double* cumul;    /* float64 sum of per-step scores         (.cumulative_attention_score) */
  float* prefill;   /* prefill score                          (.prefill_attention_score) */
  uint32_t* posmap;
} kvbp_state;

/* Eviction configuration.  n_prefix / n_suffix are the ProtectedPolicyWrapper sizes
 * max(4, int(capacity * frac)) (0 when frac == 0), see kvbp_protection_sizes(). */
typedef struct kvbp_evict_cfg {
  int32_t capacity;      /* --capacity */
  int32_t evict_every;   /* --evict-every */
  int32_t policy;        /* KVBP_POLICY_* */
  int32_t protect;       /* --protect-prefix-suffix */
  int32_t n_prefix;
  int32_t n_suffix;
  int32_t decode_regime; /* 1: --eviction-regime decode, 0: prefill (evict at step 0 only) */
} kvbp_evict_cfg;

/* Protection sizes of ProtectedPolicyWrapper (scripts/run_v3_jax.py:119-121). */
void kvbp_protection_sizes(int32_t capacity, double prefix_frac, double suffix_frac, int32_t* n_prefix,
                           int32_t* n_suffix);

/* K1 -- decode attention over the slot cache + per-slot eviction score, one layer.
 * Replaces the GQA einsum/mask/softmax/PV of _attention_layer
 * (src/counterfact_kv_eviction/jax_inference.py:1018-1050) and the per-key score
 * reduction (max over heads :1345, over layers :1670-1673).
 * q [B][Hq][128] bf16; kcache/vcache [B][Hkv][S][128] bf16 (16-byte aligned);
 * slot_pos [B][S]; out [B][Hq][128] bf16; step_score [B][S] float (non-negative,
 * updated with max(existing, max over this layer's heads of p)).  Hq/Hkv <= 8.
 * write_slot [B] may be NULL.  When given, it names the one cache slot per sequence
 * (< 0: none) that the kvbp kernels immediately before this call on the stream write
 * this step (kvbp_decode_qkv_gemm / kvbp_qkv_rope_scatter with one row per sequence);
 * the kernel then starts reading the other rows before those kernels finish.  Every
 * row such a kernel writes must be listed. */
int kvbp_decode_attn_score(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim, int32_t S,
                           const void* q, const void* kcache, const void* vcache, const int32_t* slot_pos,
                           const int32_t* write_slot, void* out, float* step_score, int32_t* dev_err);

/* K4 + K1 + K2 fused -- one layer's decode attention that also scatters this step's new
 * K/V row and, as the last kernel of the step to touch the scores, runs the per-step score
 * update (kv_coupled_generator.py:504-516).  As kvbp_decode_attn_score, and:
 *  - k_new / v_new [B][Hkv][128] bf16 (16-byte aligned; both NULL = the row is already in
 *    the cache): stored into slot write_slot[b] (< 0: not stored) and used in place of the
 *    cache row in this call (jax_inference.py:1011-1012);
 *  - st, seq_step: the score update's state; the last CTA to finish each sequence updates
 *    attn / max_attn / cumul / last_access / access_count of its valid slots from the
 *    completed step_score (pass the layer that completes the max over layers: the last)
 *    and clears step_score, as kvbp_score_update does;
 *  - seq_counter [B] int32, all zero before the first call; the kernel leaves it zero.
 * st == NULL (seq_step, seq_counter ignored): attention + scatter only, for callers that
 * run the score update at the start of the next step (kvbp_update_append_evict). */
int kvbp_decode_attn_score_update(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                  int32_t S, const void* q, const void* k_new, const void* v_new, void* kcache,
                                  void* vcache, const int32_t* slot_pos, const int32_t* write_slot, void* out,
                                  float* step_score, const kvbp_state* st, const int32_t* seq_step,
                                  int32_t* seq_counter, int32_t* dev_err);

/* K5 -- causal prefill attention of one sequence and layer on the tcgen05 tensor cores,
 * with the per-key score.  q [P][Hq][128] bf16 (after RoPE), kcache/vcache
 * [Hkv][P][128] bf16 (16-byte aligned), out [P][Hq][128] bf16 = the attention output
 * (jax_inference.py:1018-1050 with the causal mask :1169-1179).  colmax [P] float (may
 * be NULL, non-negative on entry) is max-accumulated with each key's largest probability
 * over the heads and query rows (jax_inference.py:1754-1760; pass the same buffer for
 * every layer to get the max over layers). */
int kvbp_prefill_attn_score(kvbp_stream_t stream, int32_t P, int32_t Hq, int32_t Hkv, int32_t head_dim,
                            const void* q, const void* kcache, const void* vcache, void* out, float* colmax,
                            int32_t* dev_err);

/* K4 -- QKV epilogue + scatter of the new K/V into its slot.  Replaces the bias add
 * (jax_inference.py:953-956), q/k RMSNorm (:975-978), RoPE (:621-637,1000-1001) and the
 * cache write dynamic_update_slice (:1011-1012).  qkv [rows][ldq] bf16 holds the Hq
 * query heads, then Hkv key heads, then Hkv value heads (128 each); bias may be NULL
 * (Qwen3), q_norm_w/k_norm_w may be NULL (Qwen2).  Row r belongs to sequence
 * r / rows_per_seq and is written to slot write_slot[r] (skipped when < 0) of
 * kcache/vcache [seq][Hkv][S][128].  inv_freq [64] float: RoPE inverse frequencies. */
int kvbp_qkv_rope_scatter(kvbp_stream_t stream, int32_t rows, int32_t rows_per_seq, int32_t Hq, int32_t Hkv,
                          int32_t head_dim, int32_t S, const void* qkv, int32_t ldq, const void* bias,
                          const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                          const int32_t* positions, const int32_t* write_slot, void* q_out, void* kcache,
                          void* vcache, int32_t* dev_err);

/* K2 -- per-step score update of every retained slot from step_score, then clears
 * step_score.  Replaces kv_coupled_generator.py:504-516 (attn/max/cumul update, 5 %
 * relative access threshold, last_access_step / access_count).  seq_step [B] device. */
int kvbp_score_update(kvbp_stream_t stream, const kvbp_state* st, const int32_t* seq_step, float* step_score,
                      int32_t* dev_err);

/* K3 -- one decode step's bookkeeping: advances seq_step/next_pos, puts the new
 * position into the lowest free slot (kv_coupled_generator.py:350-364) and, every
 * evict_every steps, selects and frees victims: ProtectedPolicyWrapper
 * (scripts/run_v3_jax.py:113-136) + the policy's composite-key top-k
 * (policies.py:12-63 and the policy classes) + the hard-capacity guardrail
 * (kv_coupled_generator.py:549-604).  Outputs cur_pos[b] (position to forward) and
 * write_slot[b] (its slot, -1 if evicted at this step); appends victims to
 * evlog [B][evcap] (evcount [B]); logs tokens[b] into token_log[B][log_steps] and the
 * retained count into retained_log[B][log_steps+1] when those are non-NULL.
 * KVBP_POLICY_RANDOM is rejected here (KVBP_ERR_ARG): use kvbp_append_evict_listed. */
int kvbp_append_evict(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg, int32_t* seq_step,
                      int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot, const int32_t* tokens,
                      int32_t* token_log, int32_t log_steps, int32_t* evlog, int32_t* evcount, int32_t evcap,
                      int32_t* retained_log, int32_t* dev_err);

/* K2 + K3 in one launch: the previous step's score update (as kvbp_score_update, with
 * last_access = that step, seq_step[b] on entry) runs first, then this step's
 * kvbp_append_evict -- the reference's order (kv_coupled_generator.py:504-516 at the end
 * of step t, then :350-364 and _maybe_evict :549-604 of step t + 1).  step_score [B][S]
 * holds the scores the previous step's layers max-accumulated; the kernel applies them
 * where pending[b] != 0, clears step_score for this step's layers and sets pending[b] = 1.
 * pending [B] int32 is 0 before the first decode step after prefill (no scores yet); after
 * the last step, kvbp_score_update applies the scores still pending. */
int kvbp_update_append_evict(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg,
                             int32_t* seq_step, int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot,
                             const int32_t* tokens, int32_t* token_log, int32_t log_steps, int32_t* evlog,
                             int32_t* evcount, int32_t evcap, int32_t* retained_log, float* step_score,
                             int32_t* pending, int32_t* dev_err);

/* K3 with the victims chosen on the host -- the random policy's path.
 * RandomEvictionPolicy (src/counterfact_kv_eviction/policies.py:1553-1582) draws its
 * victims with Python's random.Random(42).sample over the eligible keys in dict order,
 * so they are computed by the host (bit-exact with the reference's generator) and
 * handed in here.  Same as kvbp_append_evict, except that at a cadence step the victims
 * are victim_pos[b][0..victim_count[b]) (absolute positions, in eviction order, each
 * retained after this step's append; victim_pos is [B][victim_stride]) instead of the
 * kernel's protection + top-k; the hard-capacity guardrail (kv_coupled_generator.py:
 * 588-604) still runs after them unless flags has KVBP_LISTED_NO_HARDCAP.  Unknown or
 * repeated positions are skipped (KVBP_DEV_INDEX for unknown).  Off-cadence steps ignore
 * the list.  The per-KV-head policies use the same path: their selection (per-head top-k,
 * union, trim by votes then signal, kv_coupled_generator.py:373-433) lists the positions
 * no head keeps, with KVBP_LISTED_NO_HARDCAP (that branch of the reference has no
 * guardrail). */
#define KVBP_LISTED_NO_HARDCAP 1
int kvbp_append_evict_listed(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg,
                             int32_t* seq_step, int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot,
                             const int32_t* tokens, int32_t* token_log, int32_t log_steps, int32_t* evlog,
                             int32_t* evcount, int32_t evcap, int32_t* retained_log, const int32_t* victim_pos,
                             const int32_t* victim_count, int32_t victim_stride, int32_t flags, int32_t* dev_err);

/* K1 with per-KV-head retention (faithful Ada-KV / QUEST, kv_coupled_generator.py:
 * 436-447 builds the per-head mask, jax_inference.py:1534-1573 applies it per KV head).
 * As kvbp_decode_attn_score, and: head_keep [B][Hkv][S] u8 -- slot s is visible to kv
 * head h only when head_keep[b][h][s] != 0 (and slot_pos >= 0); head_score [B][Hkv][S]
 * float (non-negative on entry) is max-accumulated with query head r's probability for
 * r < Hkv: the rows of the per-head (Hq, C) attention output the reference's generator
 * takes as its per-head signals (kv_coupled_generator.py:470-492).  Pass the same buffer
 * for every layer to get the max over layers (jax_inference.py:1666-1673). */
int kvbp_decode_attn_score_heads(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                 int32_t S, const void* q, const void* kcache, const void* vcache,
                                 const int32_t* slot_pos, const int32_t* write_slot, const uint8_t* head_keep,
                                 void* out, float* step_score, float* head_score, int32_t* dev_err);

/* Per-head signal update after a step's forward (kv_coupled_generator.py:482-492):
 * head_cumul [B][Hkv][S] float64 += head_score (the slot write_slot[b] names starts from
 * 0: it holds this step's new position), head_current = head_score, then head_score is
 * cleared. */
int kvbp_head_signal_update(kvbp_stream_t stream, int32_t B, int32_t Hkv, int32_t S, const int32_t* write_slot,
                            float* head_score, double* head_cumul, float* head_current, int32_t* dev_err);

/* K3 at step 0 -- victim selection over the P prompt positions after prefill
 * (kv_coupled_generator.py:229-239 with force_if_over_capacity).  scores [B][P] are the
 * prefill per-key scores (NULL = zeros, as for LRU).  Writes victim [B][P] flags and the
 * policy victims, in eviction order, to evlog [B][evcap][0..n).  *n_policy_victims
 * receives n (identical for every sequence).  KVBP_POLICY_RANDOM is rejected
 * (KVBP_ERR_ARG): its step-0 victims come from the host, which writes the flags and the
 * eviction-ordered log itself and calls kvbp_prefill_compact. */
int kvbp_prefill_select(kvbp_stream_t stream, int32_t B, int32_t P, const kvbp_evict_cfg* cfg, const float* scores,
                        uint8_t* victim, int32_t* evlog, int32_t evcap, int32_t* n_policy_victims,
                        int32_t* dev_err);

/* K6 -- step-0 compaction: applies the hard-capacity guardrail, lays the retained prompt
 * positions into slots 0..R-1, initialises their metadata (kv_coupled_generator.py:179-209)
 * and gather_src [B][S] (prompt position per slot, -1 = none); resets seq_step to 0,
 * next_pos to P and clears step_score [B][S]. */
int kvbp_prefill_compact(kvbp_stream_t stream, const kvbp_state* st, int32_t P, int32_t capacity,
                         int32_t n_policy_victims, const uint8_t* victim, const float* scores, int32_t* gather_src,
                         int32_t* evlog, int32_t evcap, int32_t* evcount, int32_t* seq_step, int32_t* next_pos,
                         int32_t* retained_log, int32_t log_steps, float* step_score, int32_t* dev_err);

/* Step-0 eviction for callers that cannot allocate device memory (no counterpart in
 * the reference).  Same result as kvbp_prefill_select followed by kvbp_prefill_compact,
 * but the per-position victim flags live in a fixed array inside this library instead of
 * a caller buffer: a jax.ffi / XLA custom-call handler may only use the buffers XLA
 * assigns it (XLA pre-allocates most of the GPU, so a cudaMalloc of its own can fail).
 * Limit: batch * prompt <= 1,048,576 positions, else KVBP_ERR_ARG.  The array costs
 * 1 MiB on every GPU that loads the library, until the process exits.  The first call
 * in a CUDA context looks up the array's device address (with that context current) and
 * caches it under the context's unique ID, so a context made after cudaDeviceReset or a
 * non-primary context gets its own lookup; make that first call before any stream
 * capture.  All calls share the array: calls that overlap
 * on the GPU (e.g. on two streams) race; calls on one stream are ordered and safe.  Each
 * call rewrites every flag it uses, so no clearing is needed. */
int kvbp_prefill_evict_noalloc(kvbp_stream_t stream, const kvbp_state* st, int32_t P, const kvbp_evict_cfg* cfg,
                               const float* scores, int32_t* gather_src, int32_t* evlog, int32_t evcap,
                               int32_t* evcount, int32_t* seq_step, int32_t* next_pos, int32_t* retained_log,
                               int32_t log_steps, float* step_score, int32_t* dev_err);

/* K6 -- copies prompt K/V rows src [layers][B][Hkv][P][128] into the slot caches
 * dst [layers][B][Hkv][S][128] following gather_src. */
int kvbp_gather_kv(kvbp_stream_t stream, const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                   const int32_t* gather_src, int32_t layers, int32_t B, int32_t Hkv, int32_t P, int32_t S);

/* Dense-step helpers (reference: _forward_jittable, jax_inference.py:1182-1348). */
/* out[r] = table[ids[r]] (bf16 rows of ``hidden``), jax_inference.py:1208. */
int kvbp_embed(kvbp_stream_t stream, int32_t rows, int32_t vocab, int32_t hidden, const void* table,
               const int32_t* ids, void* out, int32_t* dev_err);
/* h = bf16(h + delta) (delta may be NULL); out = bf16(rms_norm(h) * w), jax_inference.py:609-618. */
int kvbp_add_rmsnorm(kvbp_stream_t stream, int32_t rows, int32_t hidden, void* h, const void* delta, const void* w,
                     void* out, float eps);
/* act = bf16(bf16(g * bf16(sigmoid(g))) * u) for gu = [g | u] rows, jax_inference.py:702-704,1103-1107. */
int kvbp_silu_mul(kvbp_stream_t stream, int32_t rows, int32_t ffn, const void* gu, void* act);
/* ss_out[r] = sum over the row of h[r][:]^2 (fp32), rows <= 32: the RMSNorm statistics of
 * the embedding output for the first decode GEMM's norm prologue. */
int kvbp_row_sumsq(kvbp_stream_t stream, int32_t rows, int32_t hidden, const void* h, float* ss_out);

/* Weight-streaming decode GEMM out[M][N] = X[M][K] . W[N][K]^T (bf16, fp32 accumulate),
 * M <= 32, N and K multiples of 128 -- the q/k/v, o, gate/up, down and lm_head products
 * of _forward_jittable (jax_inference.py:949-956,1081,1095-1107,1330-1333).
 * w_packed is W in the packed layout written by kvbp_pack_weight.
 * Prologue: with norm_w != NULL, X is bf16((x * inv_rms[m]) * norm_w[k]) where x (ldx) is
 *   the residual stream and inv_rms[m] = 1/sqrt(sum_t ss_parts[t][m] / K + eps) over the
 *   n_parts partial sums ([n_parts][32] floats) -- RMSNorm (jax_inference.py:609-618).
 * Epilogue 0 (plain): out = bf16(acc).
 * Epilogue 1 (residual): out (the residual stream, ldo == N) = bf16(out + bf16(acc)) in
 *   place, and ss_out[N/128][32] receives each 128-column tile's per-row sum of squares of
 *   the new stream (the next norm's n_parts = N/128) -- jax_inference.py:1280,1325.
 * Epilogue 3 (fp32): out is float [M][ldo] and receives the unrounded sums (a tensor-
 *   parallel shard's partial of a row-parallel projection, before the allreduce).
 * Epilogue 2 (SwiGLU): W rows hold gate and up features interleaved in blocks of 64
 *   (rows 128t..128t+63 = gate features 64t.., rows 128t+64.. = the matching up features);
 *   out[M][N/2] = bf16(bf16(g * bf16(sigmoid(g))) * u) with g, u the bf16 GEMM outputs
 *   (jax_inference.py:702-704,1103-1107).
 * splits (1..min(16, K/128)) CTAs share each 128-column tile's K range as one thread-block
 * cluster and reduce their partial sums in shared memory, in a fixed order: the result
 * does not depend on timing.  No workspace. */
int kvbp_decode_gemm(kvbp_stream_t stream, int32_t epilogue, int32_t M, int32_t N, int32_t K, const void* w_packed,
                     const void* x, int32_t ldx, const float* ss_parts, int32_t n_parts, const void* norm_w, float eps,
                     void* out, int32_t ldo, float* ss_out, int32_t splits, int32_t* dev_err);

/* kvbp_decode_gemm for the stacked q/k/v projection (N = (n_heads + 2 n_kv_heads) * 128,
 * norm prologue as above) fused with kvbp_qkv_rope_scatter's per-head work: each
 * 128-feature tile is one head, finished in the epilogue with bias, q/k RMSNorm, RoPE
 * and the store of q to q_out[M][n_heads][128] or of k/v to kcache/vcache
 * [M][n_kv_heads][S][128] at slot write_slot[m] (skipped when < 0; >= S sets
 * KVBP_ERR_INDEX).  jax_inference.py:949-956,975-978,1000-1012. */
int kvbp_decode_qkv_gemm(kvbp_stream_t stream, int32_t M, int32_t n_heads, int32_t n_kv_heads, int32_t K,
                         const void* w_packed, const void* x, int32_t ldx, const float* ss_parts, int32_t n_parts,
                         const void* norm_w, float eps, const void* bias, const void* q_norm, const void* k_norm,
                         const float* inv_freq, const int32_t* positions, const int32_t* write_slot, int32_t S,
                         void* q_out, void* kcache, void* vcache, int32_t splits, int32_t* dev_err);

/* Tensor-parallel row-parallel projection with the allreduce fused in: this rank's
 * partial Y = X . W^T (fp32, W packed) is pushed tile by tile into the symmetric buffer
 * of every other rank of the group (peer_bases[q] = rank q's buffer, mapped into this
 * process; a device array), and each tile is finished as h = bf16(h + bf16(sum over
 * ranks, in rank order)) with ss_out as in epilogue 1 -- identical on every rank.  Each
 * fp32 value travels with a tag in the same 8 bytes (16-byte slots {x, tag, y, tag} per
 * column pair), so receivers spin on the data itself: no fences or flag round trips.
 * Buffer layout (buffer_bytes each, >= 2 * world * M * N * 8): slots
 * [2 (call_index & 1)][world (source rank)][M][N / 2]; N <= 8192.  The buffer is zeroed
 * (and the ranks synchronised) before a run.  call_index (0..254) numbers the allreduces
 * of one step and *epoch must differ between steps (tags are epoch * 256 + call_index +
 * 1).  Every rank must make the same calls in the same order; waits are bounded
 * (KVBP_DEV_PEER_TIMEOUT).  One rank per GPU: the ranks' kernels wait on each other and
 * must run concurrently; the call is rejected when the whole grid cannot be resident at
 * once. */
int kvbp_decode_gemm_allreduce(kvbp_stream_t stream, int32_t M, int32_t N, int32_t K, const void* w_packed,
                               const void* x, int32_t ldx, void* h, float* ss_out, int32_t splits,
                               const uint64_t* peer_bases, int32_t world, int32_t rank, int32_t call_index,
                               const int32_t* epoch, int64_t buffer_bytes, int32_t* dev_err);

/* Prefill projection on the tcgen05 tensor cores: out = X[M][K] . W[N][K]^T for the
 * prompt rows of every sequence at once (the q/k/v, o, gate/up and down products of
 * _forward_jittable over the prompt, jax_inference.py:949-956,1081,1095-1107 as the
 * prefill branch :1684-1790 runs them).  w_packed is W in the kvbp_pack_weight layout
 * (read directly, no unpacking); x [M][ldx] bf16 (ldx >= K, a multiple of 8, 16-byte
 * aligned); bf16 output rounded from fp32 accumulators.  Epilogue 0: out [M][ldo] =
 * bf16(acc).  Epilogue 2 (SwiGLU, gate/up interleaved in blocks of 64 rows as for
 * kvbp_decode_gemm): out [M][ldo] holds the N/2 features bf16(bf16(g * bf16(sigmoid(g)))
 * * u) (jax_inference.py:702-704,1103-1107).  Epilogue 3: out float [M][ldo] = acc (the
 * row-parallel partial sums of tensor parallelism, rounded after the reduction over the
 * ranks).  N, K multiples of 128. */
int kvbp_prefill_gemm(kvbp_stream_t stream, int32_t epilogue, int32_t M, int32_t N, int32_t K, const void* w_packed,
                      const void* x, int32_t ldx, void* out, int32_t ldo, int32_t* dev_err);

/* Converts a row-major bf16 weight W[N][K] (N, K multiples of 128) to the decode GEMM's
 * packed layout and back: each 128-row x 128-column block becomes one contiguous 32 KiB
 * run of two 128 x 64 halves whose 16-byte chunks are XOR-swizzled by row (chunk
 * c of row r stored at c ^ (r % 8)), the image of a 128-byte-swizzled shared-memory
 * tile.  src and dst must not overlap.  (No counterpart in the reference, whose weights
 * stay row-major.) */
int kvbp_pack_weight(kvbp_stream_t stream, int32_t N, int32_t K, const void* src, void* dst);
int kvbp_unpack_weight(kvbp_stream_t stream, int32_t N, int32_t K, const void* src, void* dst);

/* Greedy sampling: first index of the row maximum (numpy.argmax), kv_coupled_generator.py:344.
 * logits [rows][ld] bf16, 16-byte aligned with ld a multiple of 8 (else status 1, nothing
 * launched); rows <= 65535. */
int kvbp_argmax(kvbp_stream_t stream, int32_t rows, int32_t vocab, int64_t ld, const void* logits, int32_t* out_ids);

/* Greedy sampling over a vocabulary shard (tensor parallelism): keys_out[r] encodes the
 * shard's (maximum value, index_offset + first index of it) so that the largest key over
 * all shards (an allreduce-MAX on int64) is the global numpy.argmax; kvbp_key_to_token
 * turns the reduced keys back into token ids. */
int kvbp_argmax_key(kvbp_stream_t stream, int32_t rows, int32_t vocab, int64_t ld, const void* logits,
                    int32_t index_offset, int64_t* keys_out);
int kvbp_key_to_token(kvbp_stream_t stream, int32_t rows, const int64_t* keys, int32_t* tokens);

/* Residual add of a reduced fp32 projection (tensor parallelism: after the allreduce of
 * the o / down shards' partial sums): h = bf16(h + bf16(delta)) for rows <= 32, and
 * ss_out[hidden/128][32] = each 128-column tile's per-row sum of squares of the new h
 * (the next decode GEMM's norm statistics) -- jax_inference.py:1280,1325. */
int kvbp_residual_add(kvbp_stream_t stream, int32_t rows, int32_t hidden, void* h, const float* delta,
                      float* ss_out);

/* Lossy int8 demotion of cache rows (online_credit_generator.py:643-704,
 * _demote_kv_positions): for every layer and kv head, the K and V rows of slots
 * slots[b][0..counts[b]) (slots is [B][stride]; < 0 or >= S sets KVBP_DEV_INDEX) of the
 * caches [layers][B][Hkv][S][128] bf16 get an absmax int8 round trip in place, with the
 * reference's bf16 arithmetic: scale = bf16(max|x| / 127), q = clip(round-half-even(
 * bf16(x / max(scale, bf16(1e-10)))), -127, 127), x = bf16(q * scale).  Slots are
 * the caller's map of the positions to demote (slot_pos); skipping positions already
 * demoted is the caller's bookkeeping, as in the reference. */
int kvbp_demote_int8(kvbp_stream_t stream, void* kcache, void* vcache, int32_t layers, int32_t B, int32_t Hkv,
                     int32_t S, const int32_t* slots, int32_t stride, const int32_t* counts, int32_t* dev_err);

#ifdef __cplusplus
}
#endif

#endif /* KVBP_H */
