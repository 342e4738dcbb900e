/*
 * moe_oracle.h -- CPU restatement of the reference's MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library, and
 * only as the checker or as the timed CPU baseline -- never as the product
 * path.  The product (moe_prefetch_b200/libmoeb200.so) never links it.
 *
 * What it restates (file:line in the reference tree, everett6/moe-prefetch):
 *   - ggml block formats Q4_K / Q6_K (layout from the upstream ggml-common.h,
 *     visible only through the patches; decode cross-checked against gguf-py
 *     0.19.0's dequantizers in tests/test_oracle_codecs.py);
 *   - the router of build_moe_ffn (softmax -> +cache prior (patches/0007:109-124)
 *     -> top-k by selection prob, ties to the lower id (patches/0010:433-441,
 *     cpp/moe-predictor.cpp:231-237) -> weights gathered from the UNBIASED
 *     probabilities and renormalised);
 *   - the fused CPU rows op ggml_cpu_moe_rows (patches/0008:186-251): up, gate,
 *     swiglu(gate, up), down, unweighted rows out; the weighted sum follows;
 *   - the slot-table state machine of llama-moecache.cpp as patched by
 *     patches/0006 (slots, free pool, LRU victim, early issue), 0007 (admission
 *     gates, probation, batched tables, cache prior, heat file) and 0008
 *     (deterministic publication, map record format, freeze).
 *
 * Parity status: the slot table, admission and router are restated exactly.
 * The Q4_K x Q8 arithmetic of ggml itself is not in the reference tree, so the
 * quantised-dot parity against ggml is "unpinned"; the block decoders are
 * pinned against gguf-py, and the predictor hook against the reference's own
 * compiled cpp/moe-predictor.cpp (oracle/_ref).
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_QK_K 256
#define OR_Q4K_BYTES 144
#define OR_Q6K_BYTES 210
#define OR_QTYPE_Q4_K 12
#define OR_QTYPE_Q6_K 14

/* ---- scalar helpers -------------------------------------------------------- */
uint16_t or_f32_to_f16(float f);
float    or_f16_to_f32(uint16_t h);
/* exp written from the mathematics: Cody-Waite range reduction + degree-7
 * Taylor polynomial; identical operation sequence to the device version. */
float    or_expf(float x);

/* ---- block codecs ------------------------------------------------------------ */
/* Our own Q4_K / Q6_K quantisers (NOT byte-identical to ggml's
 * quantize_row_q4_K, which is not in the reference tree).  n % 256 == 0. */
void or_quantize_q4_K(const float *x, uint8_t *y, int64_t n);
void or_quantize_q6_K(const float *x, uint8_t *y, int64_t n);
void or_dequantize_q4_K(const uint8_t *y, float *x, int64_t n);
void or_dequantize_q6_K(const uint8_t *y, float *x, int64_t n);
/* Q8_1-style activation blocks of 32: d = amax/127, q = roundf(x * (1/d))
 * (the reciprocal rounded once, as ggml's CPU quantize_row_q8_1_ref),
 * s = d * sum(q), d and s kept in fp32.  n % 32 == 0. */
void or_quantize_q8_1(const float *x, int8_t *q, float *d, float *s, int64_t n);
/* Q8_K as ggml's CPU path uses it (vec_dot_type of Q4_K/Q6_K): blocks of 256,
 * d = max/-127 with the signed max.  Dequantised output only (informational). */
void or_q8_K_roundtrip(const float *x, float *out, int64_t n);

/* dot of one quantised row with Q8_1 activations, double accumulation */
double or_dot_q4_K_q8_1(const uint8_t *row, const int8_t *q, const float *d,
                        const float *s, int64_t n);
double or_dot_q6_K_q8_1(const uint8_t *row, const int8_t *q, const float *d,
                        const float *s, int64_t n);
/* the GPU kernels' combine of one token: y[h] = fma chain from 0 over the k
 * rows in rank order (w [k], rows [k][n_embd]) */
void or_combine_f32(const float *w, const float *rows, int k, int n_embd, float *y);
/* the same dots in the GPU GEMV kernels' fp32 order (unit partials, lane
 * butterfly / row-group tree): the bits those kernels produce.  Q6_K: n <= 1024. */
float or_dot_q4_K_q8_1_f32(const uint8_t *row, const int8_t *q, const float *d,
                           const float *s, int64_t n);
float or_dot_q6_K_q8_1_f32(const uint8_t *row, const int8_t *q, const float *d,
                           const float *s, int64_t n);

/* ---- router -------------------------------------------------------------------- */
/* logits = W x (canonical fp32 order), probs = softmax, sel = probs (+ prior),
 * ids = top-k of sel (descending, ties to the lower id), w = probs[ids] / sum.
 * Any of probs_out / logits_out may be NULL. n_embd % 128 == 0,
 * n_expert % 32 == 0, n_expert <= 256, k <= 16. */
void or_router(const float *W, const float *x, int n_expert, int n_embd,
               const float *prior, int k, int32_t *ids, float *w,
               float *probs_out, float *logits_out);
/* the canonical dot alone (exposed for tests) */
float or_router_dot(const float *w_row, const float *x, int n_embd);
/* Select top-k from given logits (softmax, + prior, ties to the lower id,
 * renormalised unbiased weights), the order of or_router after the logits. */
void or_router_select(const float *logits, int n_expert, const float *prior, int k,
                      int32_t *ids, float *w, float *probs_out);
/* The decode kernel's fused RMSNorm + router (canonical order of the
 * persistent kernel): the residual r [n_embd] is split in G row ranges
 * [h0[c], h1[c]); per range, partial logits P[c][e] = sum_h Wt[h][e] r[h]
 * (fma chain in h order) and S[c] = sum_h r[h]^2 (fma chain); the partials
 * are summed in fixed point: P clamped to [-2^20, 2^20], S to [.., 2^36],
 * rounded to int64 multiples of 2^-32 (P) and 2^-16 (S) with ties to even,
 * added as integers (order-free), each total converted to float once and
 * scaled back; inv = 1 / sqrtf(S / n_embd + eps); logits = total * inv;
 * x = r * inv.  Wt is the router transposed, [n_embd][n_expert].  x_out and
 * logits_out optional. */
void or_router_fused(const float *Wt, const float *r, int n_expert, int n_embd,
                     const int32_t *h0, const int32_t *h1, int G, float eps,
                     const float *prior, int k, int32_t *ids, float *w, float *x_out,
                     float *logits_out);

/* ---- expert rows / layer ---------------------------------------------------------- */
/* One expert: act = silu(gate x) * (up x) with x, act quantised to Q8_1;
 * out[n_embd] = down act.  gate/up: n_ff rows of n_embd (Q4_K);
 * down: n_embd rows of n_ff (Q6_K or Q4_K per down_type). act_out optional.
 * Every dot in the GPU GEMV kernels' fp32 order (or_dot_*_f32): the rows,
 * activations and Q8_1 blocks are those kernels' bits. */
void or_expert_row(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                   int down_type, int n_embd, int n_ff, const float *x,
                   float *out, float *act_out);
/* The same with the Q8_K activation path of ggml's CPU mul_mat_id, computed on
 * dequantised values in double (informational comparison only). */
void or_expert_row_q8K(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                       int down_type, int n_embd, int n_ff, const float *x,
                       float *out);
/* Full layer for n_tok tokens: router, k expert rows, weighted sum.
 * gate/up/down hold all n_expert experts contiguously (ggml [..., n_expert]).
 * prior may be NULL; it is applied only when n_tok == 1, as in
 * patches/0007:114.  ids_out [n_tok][k], w_out [n_tok][k], y_out [n_tok][n_embd]. */
void or_moe_layer(const float *x, int n_tok, int n_embd, int n_ff, int n_expert,
                  int k, const float *router_w, const float *prior,
                  const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                  int down_type, int32_t *ids_out, float *w_out, float *y_out,
                  int n_threads);
/* The expert half with unquantised activations and exact dequantised weights,
 * fp64 accumulation: the reference of the fp16 tensor-core GEMM path. */
void or_moe_experts_f32(const float *x, int n_tok, int n_embd, int n_ff, int n_expert, int k,
                        const int32_t *ids, const float *w, const uint8_t *gate,
                        const uint8_t *up, const uint8_t *down, int down_type, float *y_out,
                        int n_threads);
/* The expert half alone: given ids / w [n_tok][k], y = sum_i w_i row(ids_i, x),
 * the sum an fp32 fma chain from 0 in rank order (the kernels' combine; also
 * or_moe_layer's). */
void or_moe_experts(const float *x, int n_tok, int n_embd, int n_ff, int k,
                    const int32_t *ids, const float *w, const uint8_t *gate,
                    const uint8_t *up, const uint8_t *down, int down_type, float *y_out,
                    int n_threads);
/* ggml CPU path (Q8_K activations), same outputs; the timed CPU baseline. */
void or_moe_layer_q8K(const float *x, int n_tok, int n_embd, int n_ff, int n_expert,
                      int k, const float *router_w, const float *prior,
                      const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                      int down_type, int32_t *ids_out, float *w_out, float *y_out,
                      int n_threads);
/* integer-dot CPU rows path in ggml op order with Q8_K activations, OpenMP over
 * rows; this is the code timed as the CPU baseline (no double accumulation). */
void or_moe_layer_cpu_fast(const float *x, int n_embd, int n_ff, int n_expert, int k,
                           const float *router_w, const float *prior,
                           const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                           int down_type, int32_t *ids_out, float *w_out,
                           float *y_out, int n_threads);

/* ---- slot-table state machine ----------------------------------------------------- */
typedef struct or_cache_cfg {
    int32_t n_layers;
    int32_t n_expert;
    int32_t n_slots;            /* --moe-expert-cache N (default per layer)     */
    const int32_t *slot_profile;/* per-layer slots or NULL (LLAMA_MOE_SLOT_PROFILE) */
    int32_t max_inserts;        /* --moe-expert-cache-inserts, default 2         */
    int32_t admit_mode;         /* 0 off, 1 heat, 2 window (LLAMA_MOE_ADMIT)      */
    int32_t admit_window;       /* default 8                                      */
    int32_t admit_half;         /* default 64                                     */
    float   admit_floor;        /* default 1.0                                    */
    int32_t spec_probation;     /* LLAMA_MOE_SPEC_PROBATION                       */
    int32_t batch_tables;       /* LLAMA_MOE_BATCH_TABLES                         */
    float   cache_prior;        /* LLAMA_MOE_CACHE_PRIOR (delta)                  */
    int32_t early_issue;        /* LLAMA_MOE_EARLY_ISSUE                          */
    int32_t predict_top;        /* LLAMA_MOE_PREDICT_TOP (with a predictor)       */
    int32_t have_pred;          /* a predictor hook is installed                  */
    int32_t freeze;             /* LLAMA_MOE_CACHE_FREEZE                         */
    int32_t use_heat_counts;    /* a heat file is configured (use_count kept)     */
} or_cache_cfg;

typedef struct or_cache or_cache;

/* predictor hook for early issue: fill out[<=k] with ids for layer+1 given
 * this layer's observed ids and the next layer's previous ids; return count. */
typedef int (*or_predict_fn)(void *ud, int layer, const int32_t *cur, int n_cur,
                             const int32_t *next_prev, int n_next_prev,
                             int32_t *out, int k);

or_cache *or_cache_create(const or_cache_cfg *cfg);
/* moe_predictor::score (cpp/moe-predictor.cpp:165-223): W [feat_dim][E],
 * bias [E]; off: row offsets of the prev, cur, below, self_prev blocks (-1:
 * absent); any id list may be NULL. */
void      or_evict_score(const float *W, const float *bias, float prior, const int32_t off[4], int E,
                         const int32_t *prev, int n_prev, const int32_t *cur, int n_cur,
                         const int32_t *below, int n_below, const int32_t *self_prev,
                         int n_self_prev, float *out);
/* LLAMA_MOE_EVICTOR: model slot m scores layer layer_of[m]; w [n_model][feat_dim][E],
 * bias [n_model][E], prior [n_model]; copied.  0, or -1 on bad offsets. */
int       or_cache_set_evictor(or_cache *c, int n_model, const int32_t *layer_of, int feat_dim,
                               const int32_t off[4], const float *w, const float *bias,
                               const float *prior);
void      or_cache_destroy(or_cache *c);
void      or_cache_set_predictor(or_cache *c, or_predict_fn fn, void *ud);
/* moe_obs_cb for one layer: ids [n_tok][n_ids]; observed only when n_tok == 1
 * (the reference's callback returns early for batches) unless force != 0. */
void      or_cache_observe(or_cache *c, int layer, const int32_t *ids, int n_tok,
                           int n_ids, int force);
/* llama_moe_cache_step with deterministic publication */
void      or_cache_step(or_cache *c);
int32_t   or_cache_n_slots(const or_cache *c, int layer);
/* expert_slot[n_expert] (slot or -1), slot_expert[ns], slot_last_use[ns],
 * in_flight[ns], slot_protect[ns]; any pointer may be NULL. */
void      or_cache_tables(const or_cache *c, int layer, int32_t *expert_slot,
                          int32_t *slot_expert, uint64_t *last_use,
                          uint8_t *in_flight, uint64_t *protect);
/* published device table (expert -> slot or n_slots) and prior (f32) */
void      or_cache_dev_table(const or_cache *c, int layer, int32_t *table, float *prior);
/* counters, layout = enum below */
enum {
    OR_ST_STEPS = 0, OR_ST_CLOCK, OR_ST_HITS, OR_ST_MISSES, OR_ST_UPLOADS,
    OR_ST_SCHEDULED, OR_ST_COPIED, OR_ST_PUBLISHED, OR_ST_ADMIT_OK,
    OR_ST_ADMIT_DENIED, OR_ST_TABLE_FLUSHES, OR_ST_COUNT
};
void      or_cache_stats(const or_cache *c, uint64_t *out);
/* jobs scheduled and not yet published: (layer, expert, slot, spec) x n */
int       or_cache_jobs(const or_cache *c, int32_t *out, int max);
/* heat (admit_mode 1) and window state for tests; NULL allowed */
void      or_cache_gate_state(const or_cache *c, int layer, float *heat,
                              uint64_t *miss_last, uint64_t *miss_prev,
                              uint32_t *use_count);
/* "moe-map 1" header / frame text (patches/0008:417-489), written into buf;
 * returns bytes needed (excluding NUL). */
int       or_cache_map_header(const or_cache *c, char *buf, int cap);
int       or_cache_map_frame(const or_cache *c, char *buf, int cap);
/* "moe-heat 1" file (patches/0007:431-485) */
int       or_cache_save_heat(const or_cache *c, const char *path);
int64_t   or_cache_load_heat(or_cache *c, const char *path);
/* warm start from loaded use counts (patches/0007:567-618); returns placed */
int64_t   or_cache_warm_start(or_cache *c);

/* byte-priced greedy slot allocation (experiments/p7_slot_allocation.py:144-185).
 * miss8[g][L] for grid points g; returns bytes used, fills cap[L]. */
double    or_greedy_allocate_bytes(const double *miss8, const int32_t *grid, int n_grid,
                                   int n_layers, int uniform_cap,
                                   const int32_t *frozen, int n_frozen,
                                   const double *expert_bytes, int32_t *cap,
                                   double *budget_out);

#ifdef __cplusplus
}
#endif
#endif
