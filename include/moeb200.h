/*
 * moeb200.h -- C ABI of libmoeb200.so, the B200-native MoE layer with a GPU
 * expert slot cache.
 *
 * Plain pointers and sizes only; `stream` is a cudaStream_t passed as void*
 * (NULL = the legacy default stream).  Every entry point returns an int status
 * (MOE_OK = 0, negative = error) unless stated; the message of the last error
 * is available from moe_last_error().  Nothing aborts the process.
 *
 * Each declaration names the reference interface it replaces, as
 * file:line in everett6/moe-prefetch (patches are cited by line of the patch
 * file).  The reference's interface takes llama/ggml types; here the same
 * operations take plain buffers.
 */
#ifndef MOEB200_H
#define MOEB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define MOE_OK               0
#define MOE_ERR_ARG         -1   /* bad argument / shape                         */
#define MOE_ERR_CUDA        -2   /* a CUDA runtime call failed                   */
#define MOE_ERR_OOM         -3   /* device or pinned allocation failed           */
#define MOE_ERR_UNSUPPORTED -4   /* shape or mode this build does not implement  */
#define MOE_ERR_TIMEOUT     -5   /* a device-side bounded wait gave up           */
#define MOE_ERR_STATE       -6   /* call out of order (e.g. weights missing)     */
#define MOE_ERR_DEVICE      -7   /* a kernel reported a bad index                */

/* ggml type ids of the weight blocks (same numbers as ggml's enum) */
#define MOE_QTYPE_Q4_K 12
#define MOE_QTYPE_Q6_K 14

/* admission gate (LLAMA_MOE_ADMIT, patches/0007:182-188) */
#define MOE_ADMIT_OFF    0
#define MOE_ADMIT_HEAT   1
#define MOE_ADMIT_WINDOW 2

typedef struct moe_ctx moe_ctx;

/* Cache + layer configuration.  Replaces the arguments of
 * llama_moe_cache_init(model, n_slots, max_inserts) (patches/0006:482) and the
 * LLAMA_MOE_* environment switches it parses (patches/0006:501-520,
 * 0007:492-506, 0008:536-573). */
typedef struct moe_cfg {
    int32_t n_layers;          /* MoE layers in the stack                          */
    int32_t n_expert;          /* routed experts per layer: 32, 64, 128 or 256     */
    int32_t n_used;            /* experts per token (top-k, <= 8)                  */
    int32_t n_embd;            /* hidden size (2048 in this build)                 */
    int32_t n_ff;              /* expert intermediate size (multiple of 256)       */
    int32_t down_type;         /* MOE_QTYPE_Q6_K or MOE_QTYPE_Q4_K                 */
    int32_t n_slots;           /* --moe-expert-cache N, default slots per layer    */
    const int32_t *slot_profile; /* per-layer slots (LLAMA_MOE_SLOT_PROFILE) or NULL */
    int32_t max_inserts;       /* --moe-expert-cache-inserts (0 -> 2)              */
    int32_t admit_mode;        /* MOE_ADMIT_*                                      */
    int32_t admit_window;      /* LLAMA_MOE_ADMIT_WINDOW (0 -> 8)                  */
    int32_t admit_half;        /* LLAMA_MOE_ADMIT_HALF (0 -> 64)                   */
    float   admit_floor;       /* LLAMA_MOE_ADMIT_FLOOR                            */
    int32_t spec_probation;    /* LLAMA_MOE_SPEC_PROBATION                         */
    int32_t batch_tables;      /* LLAMA_MOE_BATCH_TABLES (tables always move in one
                                  device step here; kept for the stats counter)   */
    float   cache_prior;       /* LLAMA_MOE_CACHE_PRIOR, delta (0 = off)           */
    int32_t early_issue;       /* LLAMA_MOE_EARLY_ISSUE: uploads start when a layer
                                  is observed, into a free pool the step refills  */
    int32_t freeze;            /* LLAMA_MOE_CACHE_FREEZE                           */
    int32_t use_heat_counts;   /* a heat file is configured (LLAMA_MOE_HEAT_FILE)  */
    int32_t device;            /* CUDA device ordinal                              */
    int32_t n_shared;          /* always-on shared experts per layer: 0 or 1.  A
                                  shared expert joins every token after the k
                                  routed ones with weight 1; it is never cached,
                                  observed or routed (moe_set_shared_expert)      */
    int32_t predict_top;       /* LLAMA_MOE_PREDICT_TOP (0 -> 3): speculative
                                  uploads per observed layer with a predictor     */
    int32_t stream;            /* LLAMA_MOE_STREAM: just-in-time streaming (needs
                                  early_issue): after each single-token layer,
                                  the lookahead of the next two layers' routers
                                  claims slots for their best non-resident
                                  experts, copied earliest deadline first in
                                  chunks, each made visible by its table word
                                  as soon as its last byte lands               */
    int32_t stream_per_layer;  /* LLAMA_MOE_STREAM_PER_LAYER: streamed experts per
                                  target layer and token (0 -> 4)                */
    int32_t stream_reserve;    /* LLAMA_MOE_STREAM_RESERVE: extra free slots kept
                                  per layer at the token boundary (the
                                  reference's default is 2; 0 keeps none)      */
    float   stream_gbps;       /* LLAMA_MOE_STREAM_GBPS: the copy engine's rate
                                  the deadlines assume (0 -> 45.7)               */
    int32_t stream_topk;       /* LLAMA_MOE_STREAM_TOPK: lookahead candidates per
                                  target layer, best scores first (0 -> 8, <= 16) */
} moe_cfg;

/* What llama_moe_cache_lookup(up_exps) returns for one layer
 * (struct llama_moe_cache_layer, patches/0007:774-790): slot slabs
 * [n_slots + 1][...] (slot n_slots is the dummy), the device table
 * (expert -> slot, n_slots when not resident) and the slot count. */
typedef struct moe_layer_info {
    void    *gate_c;           /* device: [n_slots+1][n_ff rows of n_embd]  Q4_K  */
    void    *up_c;             /* device: same                                     */
    void    *down_c;           /* device: [n_slots+1][n_embd rows of n_ff]  down   */
    int32_t *dev_table;        /* device: [n_expert]                               */
    int64_t  gate_bytes;       /* bytes of one expert's gate (= up) matrix         */
    int64_t  down_bytes;       /* bytes of one expert's down matrix                */
    int32_t  n_slots;
    int32_t  il;
} moe_layer_info;

/* Counters (the reference's every-512-steps stderr line, patches/0006:928-953,
 * 0007:762-770), read with moe_get_stats in this order.  UPLOAD_NS is ours:
 * the time the copy stream spent on the upload batches moe_step issued (from
 * the start of a batch's first copy to the end of its last, measured with
 * events), so that UPLOAD_BYTES / UPLOAD_NS is the host-link rate while
 * uploads run. */
enum moe_stat {
    MOE_STAT_STEPS = 0, MOE_STAT_CLOCK, MOE_STAT_HITS, MOE_STAT_MISSES,
    MOE_STAT_UPLOADS, MOE_STAT_SCHEDULED, MOE_STAT_COPIED, MOE_STAT_PUBLISHED,
    MOE_STAT_ADMIT_OK, MOE_STAT_ADMIT_DENIED, MOE_STAT_TABLE_FLUSHES,
    MOE_STAT_UPLOAD_BYTES, MOE_STAT_UPLOAD_NS, MOE_STAT_COUNT
};

/* ---- lifetime ---------------------------------------------------------------- */

/* Create the cache + layer context on cfg->device: allocates the slot slabs,
 * tables and slot state on the device, all slots empty, all tables -> dummy.
 * Replaces llama_moe_cache_init (patches/0006:482-763, 0007:519-655,
 * 0008:825-573 env handling, 0009:620-658 ownership by the context). */
int moe_create(const moe_cfg *cfg, moe_ctx **out);

/* Free everything; waits for in-flight uploads.  Replaces
 * llama_moe_cache_shutdown/_claim (patches/0009:1019-1056). */
void moe_destroy(moe_ctx *ctx);

/* Text of the last error on this context ("" if none). */
const char *moe_last_error(const moe_ctx *ctx);

/* Per-layer slabs / table.  Replaces llama_moe_cache_lookup
 * (patches/0009:1184-1218, struct at 0007:774-790). */
int moe_get_layer(moe_ctx *ctx, int layer, moe_layer_info *out);

/* ---- weights ------------------------------------------------------------------- */

/* Router weight ffn_gate_inp of one layer, fp32 [n_expert][n_embd], host or
 * device memory (copied into the context).  The reference keeps it in the
 * model (build_moe_ffn, context of patches/0007:101-128). */
int moe_set_router(moe_ctx *ctx, int layer, const float *w);

/* Register the caller-owned host copies of one layer's experts, ggml layout
 * [n_expert][rows][blocks] for gate, up and down.  They are pinned and mapped
 * (cudaHostRegister) unless already pinned, and are the source of every
 * upload and of zero-copy reads for missed experts.  Replaces the host-resident
 * up_src/gate_src/down_src tensors of layer_state (patches/0006:585-590) and
 * the -ot CUDA_Host placement (patches/0006:1-17). */
int moe_set_expert_weights(moe_ctx *ctx, int layer, const void *gate, const void *up,
                           const void *down);

/* Place experts into slots without going through admission: slot_expert[ns]
 * gives the expert for each slot (-1 = empty).  With copy != 0 the bytes are
 * copied from the registered host weights, else the caller has already written
 * the slots (moe_get_layer).  Replaces the map replay frame (patches/0008:435-475)
 * and the heat warm start placement (0007:567-618). Synchronous. */
int moe_place(moe_ctx *ctx, int layer, const int32_t *slot_expert, int copy);

/* The shared expert of `layer` (cfg->n_shared == 1): gate, up [n_ff rows
 * of n_embd] Q4_K and down [n_embd rows of n_ff] in the model's layout, host
 * or device memory, copied to a device buffer of its own.  It is always
 * resident.  Replaces the ffn_*_shexp tensors of the upstream Qwen MoE
 * graphs (upstream llama.cpp, not in the reference patches); the reference's
 * 35B model has one shared expert per layer (README.md:33-36). */
int moe_set_shared_expert(moe_ctx *ctx, int layer, const void *gate, const void *up,
                          const void *down);

/* ---- the hot path -------------------------------------------------------------- */

/* One MoE layer for n_tok tokens, device buffers x [n_tok][n_embd] (the
 * ffn_norm output) -> y [n_tok][n_embd] (the weighted sum of the k expert
 * rows; the caller adds the residual).  Fused router (+cache prior when
 * n_tok == 1), slot lookup, observation (n_tok == 1 only, as the reference's
 * callback), gate/up GEMV with SiLU*mul, down GEMV with the weighted combine.
 * Missed experts are read zero-copy from the registered host weights.
 * ids/w [n_tok][n_used] are optional outputs.  Replaces build_moe_ffn's expert
 * path with the cache chain (patches/0009:659-705, 0008:372-390) and
 * ggml_cpu_moe_rows (patches/0008:186-251). */
int moe_layer_forward(moe_ctx *ctx, int layer, const float *x, float *y, int n_tok,
                      int32_t *ids, float *w, void *stream);

/* Expert paths of moe_layer_forward_path. */
#define MOE_PATH_AUTO 0   /* GEMM when n_tok * n_used >= 4 * n_expert and it applies, else GEMV */
#define MOE_PATH_GEMV 1   /* Q8_1 activations, int8 dot products: moe_layer_forward */
#define MOE_PATH_GEMM 2   /* tcgen05 grouped GEMM: fp16 weights and activations, fp32 sums */

/* moe_layer_forward with the expert arithmetic chosen by `path`.
 * MOE_PATH_GEMM is the batched / prefill path.  It groups the routed pairs
 * by expert in tiles of up to 64 tokens and dequantises each expert's
 * Q4_K/Q6_K rows to fp16 in shared memory.  The products run on the tensor
 * cores (tcgen05.mma, fp32 accumulators in tensor memory), then the same
 * combine follows.  Its outputs match exact weights times unquantised
 * activations within the layer tolerance; the GEMV path's Q8_1 activations
 * are a different rounding.  It needs Q6_K down weights.  The router,
 * prior and observation are moe_layer_forward's.  Replaces the batched
 * mul_mat_id of build_moe_ffn (patches/0009:684-695) for prefill ubatches. */
int moe_layer_forward_path(moe_ctx *ctx, int layer, const float *x, float *y, int n_tok,
                           int32_t *ids, float *w, int path, void *stream);

/* ---- expert parallelism (batched decode and prefill over several GPUs) --------- */
/* These three calls have no counterpart in the reference, which runs on one
 * GPU.  Rank g of `world` owns experts [g*E/world, (g+1)*E/world) of every
 * layer (its context holds only those in slots).  Per layer:
 *   moe_ep_route_pack -> all-to-all of send_count, then of send_ids/send_x
 *   (NCCL, by the caller) -> moe_experts_rows on the received rows ->
 *   all-to-all of the rows back -> moe_ep_combine.
 * The result equals moe_layer_forward_path on one GPU: bit for bit with
 * the GEMV path. */

/* Route the n_tok home tokens x [n_tok][n_embd] (no cache prior, no
 * observation): ids/w [n_tok][n_used].  Pack the pairs for their owners in
 * rank order, pair order within a rank:
 *   send_count [world] (device);
 *   pos [n_tok*n_used]: the send slot of pair t*n_used + r, -1 for an id
 *   out of range;
 *   send_ids / send_x: the expert id and token row of each slot.
 * capacity == 0: the slots are dense, [n_tok*n_used][...], so an exchange
 * needs send_count on the host.  capacity >= n_tok*n_used: rank d's pairs
 * fill slots [d*capacity, ...) of [world*capacity][...] and the rest keep id
 * -1 (moe_experts_rows skips them), so the exchange uses equal splits and
 * never waits for the host. */
int moe_ep_route_pack(moe_ctx *ctx, int layer, const float *x, int n_tok, int world,
                      int capacity, int32_t *ids, float *w, int32_t *send_count, int32_t *pos,
                      int32_t *send_ids, float *send_x, void *stream);

/* The expert half for n_rows received rows: y_rows[i] = expert ids[i] applied
 * to x_rows[i], unweighted (path as moe_layer_forward_path; AUTO takes the
 * GEMM from 4 rows per slot of the layer on).  Rows with id -1 (empty slots)
 * are skipped and their y_rows left as they were. */
int moe_experts_rows(moe_ctx *ctx, int layer, const float *x_rows, const int32_t *ids,
                     int n_rows, float *y_rows, int path, void *stream);

/* out[t] = sum over r in rank order of w[t][r] * y_rows[pos[t*n_used + r]],
 * then + add_rows[t] when given: the combine of moe_layer_forward over the
 * rows that came back.  With a shared expert, add_rows are its rows for the
 * home tokens (moe_experts_rows with id n_expert on every row; each rank
 * keeps a replica of the shared expert); required then, else NULL. */
int moe_ep_combine(moe_ctx *ctx, const float *y_rows, const int32_t *pos, const float *w,
                   int n_tok, const float *add_rows, float *out, void *stream);

/* ---- expert parallelism over peer memory ------------------------------------------
 * No counterpart in the reference (it runs on one GPU).  The same layer as
 * moe_ep_route_pack + all-to-all + moe_experts_rows + all-to-all +
 * moe_ep_combine, with the two exchanges done by this library's own kernels
 * over NVLink instead of a collective library: every rank owns a mailbox in
 * its device memory, mapped into the other ranks' processes with CUDA IPC,
 * and the kernels store rows straight into the owner's (then the home
 * rank's) mailbox and raise a flag there.  Only pairs that exist cross the
 * link, nothing waits for the host, and a whole step can be captured in a
 * CUDA graph.  Plain loads and stores only: no multicast, no bulk copy from
 * a peer's memory.  Waits are bounded by the context's wait limit
 * (moe_set_wait_limit); a wait that runs out sets the error word that
 * moe_sync reports as MOE_ERR_TIMEOUT.  Every rank must issue the same
 * sequence of layers (push, serve, collect), one layer after another on one
 * stream. */
#define MOE_EP_HANDLE_BYTES 64
/* Allocate this rank's mailbox for up to max_home_tokens home tokens per
 * layer and write its IPC handle (MOE_EP_HANDLE_BYTES) to handle_out.
 * world >= 2; rank g owns experts [g E / world, (g + 1) E / world). */
int moe_ep_mailbox_create(moe_ctx *ctx, int world, int rank, int max_home_tokens, void *handle_out);
/* Open the other ranks' mailboxes: handles = the world handles in rank order
 * (host memory).  Call once, on every rank, after every rank has created its
 * mailbox; keep the ranks apart from one another's mailboxes until all have
 * connected (a barrier), and again before moe_destroy. */
int moe_ep_mailbox_connect(moe_ctx *ctx, const void *handles);
/* Send this rank's routed pairs: send_count/send_ids/send_x as
 * moe_ep_route_pack wrote them with capacity 0 (compact, in owner order),
 * n_tok the home tokens of that call.  Every rank passes the same n_tok to
 * the three calls of a layer (1 .. max_home_tokens): the mailbox blocks of
 * that layer hold n_tok * n_used slots. */
int moe_ep_push(moe_ctx *ctx, int n_tok, const int32_t *send_count, const int32_t *send_ids,
                const float *send_x, void *stream);
/* Owner side: wait for every rank's pairs, run this rank's experts on them
 * (path MOE_PATH_GEMV or MOE_PATH_GEMM), send the unweighted rows back. */
int moe_ep_serve(moe_ctx *ctx, int layer, int n_tok, int path, void *stream);
/* Home side: wait for every owner's rows, then the combine of moe_ep_combine
 * (pos / w from moe_ep_route_pack; add_rows the shared expert's rows or NULL). */
int moe_ep_collect(moe_ctx *ctx, const int32_t *pos, const float *w, int n_tok, const float *add_rows,
                   float *out, void *stream);

/* moe_layer_forward that allocates no device memory.  This entry point has no
 * counterpart in the reference, whose CPU expert path allocates nothing on
 * the GPU.
 *
 * Who needs it: callers that cannot allocate device memory while they run.
 * For example, a serving process that commits all of its device memory at
 * start-up (weights, KV cache, compute buffers), or a ggml-style scheduler
 * that sizes every buffer before it runs the graph.  moe_layer_forward grows
 * its scratch with cudaMalloc the first time it sees a larger n_tok.  Growing
 * also frees the old scratch, and cudaFree waits for the whole device.  This
 * variant never does either.
 *
 * Arguments and results are those of moe_layer_forward, with two
 * differences:
 *  - contexts with a shared expert (moe_cfg.n_shared = 1) are refused with
 *    MOE_ERR_UNSUPPORTED;
 *  - a batch (n_tok > 1) always runs the per-pair kernels, which read an
 *    expert's rows once per routed (token, expert) pair, where
 *    moe_layer_forward groups the pairs by expert and reads them once per
 *    tile.  The results are the same bits; a batch is slower: 481 us vs
 *    161 us for 32 tokens of a Qwen3-30B-A3B-shape layer on one B200, 151 us
 *    vs 86 us for 8.  n_tok = 1 is the same launch sequence in both.
 * The scratch lives in one static device array of MOE_NOALLOC_SCRATCH_BYTES
 * per device, built into the library: the router ids/weights and the gate/up
 * activations.
 *
 * Limit: a call needs 2 * round_up(4 * n_tok * n_used, 256) +
 * 4 * n_tok * n_used * n_ff bytes of that array.  For n_used 8 and n_ff 768
 * that is at most 170 tokens.  A larger n_tok returns MOE_ERR_ARG, with the
 * limit in the message, before anything is launched.
 *
 * Set-up: the first call on each device looks up the array's address (with
 * that device current) and keeps it.  Make that first call before any stream
 * capture starts.
 *
 * Races: every context on a device shares the one array.  Calls whose work
 * overlaps in time race on it: other streams, other contexts, other host
 * threads.  Calls issued one after another on a single stream are safe.
 *
 * Nothing in the array has to start at zero: every entry a call reads, the
 * same call writes first. */
#define MOE_NOALLOC_SCRATCH_BYTES (4u << 20)
int moe_layer_forward_noalloc(moe_ctx *ctx, int layer, const float *x, float *y, int n_tok,
                              int32_t *ids, float *w, void *stream);

/* Optional per-(token, layer) dumps of the decode stack, device pointers or NULL:
 * x [n_tok][n_layers][n_embd] (router input), ids/w [n_tok][n_layers][n_used],
 * y [n_tok][n_layers][n_embd] (the layer's MoE output), and phase timestamps
 * prof [n_tok][n_layers][MOE_DECODE_PHASES][grid] (%globaltimer ns, one per CTA
 * at each phase boundary: 0 layer start, 1 after the first grid barrier, 2
 * router totals read, 6 selection done, 7 copies issued, 8 gate/up rows done
 * (warp 1), 9 this CTA's ranks signalled, 10 rank 0's down rows done (warp 0's
 * group), 11 combine done; 3-5 unused). */
#define MOE_DECODE_PHASES 12
typedef struct moe_decode_dbg {
    float    *x;
    int32_t  *ids;
    float    *w;
    float    *y;
    uint64_t *prof;
    int32_t   starve;   /* tests of the watchdog only: r + 1 makes rank r's first
                           activation wait target one signal more than its
                           producers give, so that it can only run out; 0 off */
    int32_t   spec;     /* the early gate/up copies (cache prior off: copies
                           requested for the top-k of the logits while the
                           softmax and the exact top-k run, re-issued where a
                           rank's id differs): 0 default (on), 1 off, 2 on with
                           a wrong rank-0 prediction in every other (token,
                           layer), for tests of the re-issue; results are the
                           same bits in every mode */
} moe_decode_dbg;

/* Batch-1 decode of n_tok tokens, strictly one after another, through all
 * n_layers: for each token t the residual starts at h[t]; every layer applies
 * RMSNorm (eps 1e-6, unit weight), the MoE layer and the residual add;
 * out[t] is the final residual.  One persistent kernel per call (one CTA per
 * SM).  Device buffers.  Replaces the per-layer decode graph of
 * llama_context::decode for the MoE part (patches/0009:620-705). */
int moe_decode(moe_ctx *ctx, const float *h, float *out, int n_tok,
               const moe_decode_dbg *dbg, void *stream);

/* The same with host buffers: h_host -> device, decode, device -> out_host,
 * all on `stream`, synchronised before returning. */
int moe_decode_host(moe_ctx *ctx, const float *h_host, float *out_host, int n_tok,
                    void *stream);

/* Limit of every device-side wait of the decode kernel (grid barrier,
 * activation signals, copy completions), in nanoseconds; 0 restores the
 * default of 2 s.  When a wait runs out, the kernel sets the error word and an
 * abort flag that ends every CTA, waits (bounded) for its own copies, and
 * returns; moe_decode_host / moe_sync then report MOE_ERR_TIMEOUT once, and the
 * context stays usable.  The reference's counterpart is the sidecar's
 * deadline, whose expiry makes llama_context::decode return -3
 * (patches/0009:652-655; cpp/test-moe-sidecar.cpp tests the dead host). */
int moe_set_wait_limit(moe_ctx *ctx, uint64_t ns);

/* Synchronise `stream` and report what the kernels flagged since the last
 * call (MOE_ERR_TIMEOUT: a bounded device wait gave up; MOE_ERR_DEVICE: an
 * id out of range).  The hot-path launches are asynchronous; this is where
 * their device-side errors surface.  Replaces the error return of
 * llama_context::decode when the sidecar times out (patches/0009:652-655). */
int moe_sync(moe_ctx *ctx, void *stream);

/* Decode-kernel geometry: grid (CTAs), shared bytes per CTA, gate/up rows and
 * down rows per CTA (max), threads per CTA; n = how many to copy. */
int moe_decode_info(const moe_ctx *ctx, int32_t *out, int n);

/* ---- the slot cache step ------------------------------------------------------- */

/* Host callbacks of the per-layer entry points (moe_layer_forward,
 * moe_layer_forward_path and moe_observe with one token), called after the
 * layer's observation on the device, with the stream synchronised.
 *
 * moe_observe_fn replaces ggml_set_moe_obs_callback's callback
 * (patches/0006:752): the layer and its routed ids (host copy, n_tok x n_ids).
 *
 * moe_predict_fn is the reference's predictor hook (cpp/moe-predictor.h:38-106
 * as called from moe_obs_cb, patches/0006:367-397, 0007:294-321): given this
 * layer's ids `cur` and the ids the next layer saw at the previous token
 * (`next_prev`), write up to k ids for the next layer to `out` and return how
 * many.  With early issue they become speculative uploads (at most
 * predict_top, keeping max_inserts slots of the pool for demand; probation
 * with spec_probation); an installed predictor also grows the free pool's
 * target by predict_top.  The persistent decode kernel (moe_decode) observes
 * on the device and issues the admitted misses early, but calls neither
 * callback: the host does not see its layers one at a time. */
typedef void (*moe_observe_fn)(void *ud, int layer, const int32_t *ids, int n_tok, int n_ids);
typedef int (*moe_predict_fn)(void *ud, int layer, const int32_t *cur, int n_cur,
                              const int32_t *next_prev, int n_next_prev, int32_t *out, int k);
int moe_set_observe_hook(moe_ctx *ctx, moe_observe_fn fn, void *ud);
int moe_set_predictor(moe_ctx *ctx, moe_predict_fn fn, void *ud);

/* LLAMA_MOE_EVICTOR (patches/0006:521-537; evict_scores 0006:402-426; the
 * victim choice 0006:790-913, 0007:680-727): a MOEP v3 model (the
 * predictor's format, cpp/moe-predictor.cpp) scores each layer's experts at
 * moe_step -- inputs: the next layer's previous-token ids, this layer's ids,
 * the previous layer's ids, this layer's previous-token ids -- and the victim
 * is the resident slot with the lowest score (recency breaking ties) instead
 * of the least recently used one, in the scheduling and the early-issue pool
 * top-up alike.  Empty, in-flight and protected slots are treated as before;
 * layers without a model keep LRU.  Scores are computed on the device
 * (moe_predictor::score, fp32, no fused multiply-adds).  n_model model slots,
 * layer_of[n_model] the stack layer of each; w [n_model][feat_dim][n_expert],
 * bias [n_model][n_expert], prior [n_model]; off[4] the row offsets of the
 * prev, cur, below and self_prev blocks in feat_dim (-1: absent).  Host
 * pointers, copied; n_model 0 removes the model. */
int moe_set_evictor(moe_ctx *ctx, int n_model, const int32_t *layer_of, int feat_dim,
                    const int32_t *off, const float *w, const float *bias, const float *prior);

/* Observe one layer's routed ids (device [n_tok][n_ids]) outside
 * moe_layer_forward: hits refresh recency, misses feed the second-miss window
 * and the pending list; with early issue the admitted misses take slots of
 * the free pool and their uploads start (then the predictor, below).  Only
 * n_tok == 1 is observed.  Replaces moe_obs_cb (patches/0006:295-400,
 * 0007:247-321). */
int moe_observe(moe_ctx *ctx, int layer, const int32_t *ids, int n_tok, int n_ids,
                void *stream);

/* Between tokens: publish every upload scheduled at the previous step in
 * (layer, slot) order, advance the step, schedule this step's admissions and
 * evictions on the device, then issue their copies on the dedicated copy
 * stream.  Deterministic publication.  Synchronises `stream` once.  Replaces
 * llama_moe_cache_step (patches/0006:765-953, 0007:655-773, 0008:607-660). */
int moe_step(moe_ctx *ctx, void *stream);

/* 1: moe_step needs the previous forward complete (always, here).  Replaces
 * llama_moe_cache_requires_sync (patches/0008:603-605). */
int moe_requires_sync(const moe_ctx *ctx);

/* Host copies of one layer's slot state (any pointer may be NULL):
 * expert_slot [n_expert] (slot or -1), slot_expert / last_use / in_flight /
 * protect [n_slots].  Synchronous. */
int moe_get_tables(moe_ctx *ctx, int layer, int32_t *expert_slot, int32_t *slot_expert,
                   uint64_t *last_use, uint8_t *in_flight, uint64_t *protect);

/* Admission-gate state of one layer (heat f32, miss_last / miss_prev u64,
 * use_count u32, each [n_expert]; NULL to skip).  Synchronous. */
int moe_get_gate_state(moe_ctx *ctx, int layer, float *heat, uint64_t *miss_last,
                       uint64_t *miss_prev, uint32_t *use_count);

/* Counters in enum moe_stat order; n = how many to copy.  Synchronous. */
int moe_get_stats(moe_ctx *ctx, uint64_t *out, int n);

/* Load use counts from a host array [n_layers][n_expert] (e.g. a parsed
 * "moe-heat 1" file, patches/0007:431-466, already halved) and place the
 * hottest experts before the first token (0007:567-618).  Returns the number
 * placed (>= 0) or an error. */
int moe_warm_start(moe_ctx *ctx, const uint32_t *use_count);

/* Just-in-time streaming counters (patches/0010's moe_stream counters and
 * its in-time / late split), cumulative, in this order: lookahead records,
 * jobs the planner accepted, chunks sent, bytes sent, table words written
 * (experts made visible within the token), jobs dropped late, jobs dropped
 * because their layer read its table first, claimed slots given back,
 * streamed experts routed and found resident by their layer (in time),
 * streamed experts routed before their table word landed (late).  Copies
 * n <= MOE_STREAM_STAT_COUNT of them to out. */
#define MOE_STREAM_STAT_COUNT 10
int moe_stream_stats(moe_ctx *ctx, uint64_t *out, int n);

/* ---- stateless kernels (device pointers) ------------------------------------------ */

/* Fused router for n_tok tokens: logits = W x in the canonical fp32 order,
 * softmax, + delta on experts with table[e] != n_slots (only when table is
 * non-NULL, delta > 0 and n_tok == 1), top-k (ties to the lower id),
 * renormalised weights from the unbiased probabilities.  logits optional.
 * Replaces the router nodes of build_moe_ffn (context of patches/0007:101-128). */
int moe_router_run(const float *W, const float *x, int n_tok, int n_expert, int n_embd,
                   const int32_t *table, int n_slots, float delta, int k,
                   int32_t *ids, float *w, float *logits, void *stream);

/* Quantise fp32 rows (n % 256 == 0) into Q4_K or Q6_K blocks on the device,
 * bit-identical to the oracle's quantiser (a synthetic-weight tool; ggml's
 * quantize_row_q4_K is not in the reference tree). */
int moe_quantize(const float *x, void *y, int64_t n, int qtype, void *stream);

/* Synthetic N(0, sigma^2) weights generated and quantised on the device in
 * one pass (element i of block b from a counter hash of (seed, b*256 + i)),
 * for the benchmark's 18.8 GB expert set; and synthetic fp32 N(0, sigma^2)
 * values.  No reference counterpart (the reference loads a GGUF). */
int moe_synth_weights(void *y, int64_t n_blocks, int qtype, uint64_t seed, float sigma,
                      void *stream);
int moe_synth_f32(float *y, int64_t n, uint64_t seed, float sigma, void *stream);

/* ---- ExpertCache (src/prefetch_engine.py:45-168) ----------------------------------- */

typedef struct moe_xc moe_xc;

/* Per-layer LRU cache of byte slabs [capacity][bytes_per_expert] in device
 * memory, refilled from a pinned host staging buffer [n_experts][bytes] on a
 * dedicated copy stream with one event per copy.  Replaces
 * ExpertCache.__init__ (src/prefetch_engine.py:48-70). */
int moe_xc_create(int n_layers, int n_experts, int capacity, int64_t bytes_per_expert,
                  const void *host_staging, int device, moe_xc **out);
void moe_xc_destroy(moe_xc *xc);
/* prefetch (src/prefetch_engine.py:89-106): start copies for the ids not yet
 * cached; returns how many started (>= 0) or an error. */
int moe_xc_prefetch(moe_xc *xc, int layer, const int32_t *ids, int n);
/* query (:108-132): status[i] = 0 hit, 1 late (copy still in flight), 2 miss. */
int moe_xc_query(moe_xc *xc, int layer, const int32_t *ids, int n, int32_t *status);
/* admit (:134-154): bring missed experts in (copies move the bytes). */
int moe_xc_admit(moe_xc *xc, int layer, const int32_t *ids, int n);
/* sync (:156-157) */
int moe_xc_sync(moe_xc *xc);
/* vram_bytes (:159-160) */
int64_t moe_xc_vram_bytes(const moe_xc *xc);
/* stats: hits, misses, late, fetches, bytes, evictions (:69-70) */
int moe_xc_stats(const moe_xc *xc, uint64_t *out6);
/* device slab of a layer and the slot an expert sits in (-1 if not cached) */
void *moe_xc_slab(moe_xc *xc, int layer);
int moe_xc_slot_of(const moe_xc *xc, int layer, int expert);

#ifdef __cplusplus
}
#endif
#endif /* MOEB200_H */
