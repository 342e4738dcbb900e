// moe_kernels.h -- internal declarations shared by the .cu files of
// libmoeb200.so (not part of the public C ABI in include/moeb200.h).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "moe_dev.cuh"

namespace moe {

// Where one layer's experts live: slot slabs on the device (slot stride =
// per-expert bytes; table[e] == ns means not resident), the registered host
// copies (expert stride), read zero-copy for misses, and the always-resident
// shared expert, addressed as expert id n_expert.
struct ExpertSrc {
    const uint8_t *gate, *up, *down;      // device slabs [ns+1][...]
    const uint8_t *hgate, *hup, *hdown;   // mapped host [n_expert][...] or null
    const uint8_t *sgate, *sup, *sdown;   // shared expert (device) or null
    const int32_t *table;                 // [n_expert] or null (= all host)
    int64_t gate_bytes, down_bytes;
    int32_t ns, n_expert;
};

// Bytes of expert `id`'s matrix (which: 0 gate, 1 up, 2 down): the shared
// expert for id == n_expert, else its slot, else (a miss) the registered host
// copy; null when there is none or the id is out of range.
__device__ __forceinline__ const uint8_t *expert_ptr(const ExpertSrc &s, int which, int id) {
    if (id == s.n_expert) return which == 0 ? s.sgate : which == 1 ? s.sup : s.sdown;
    if (id < 0 || id > s.n_expert) return nullptr;
    const int32_t slot = s.table ? s.table[id] : s.ns;
    const uint8_t *slab = which == 0 ? s.gate : which == 1 ? s.up : s.down;
    const uint8_t *host = which == 0 ? s.hgate : which == 1 ? s.hup : s.hdown;
    const int64_t bytes = which == 2 ? s.down_bytes : s.gate_bytes;
    if (slot != s.ns && slab) return slab + (int64_t)slot * bytes;
    return host ? host + (int64_t)id * bytes : nullptr;
}

// True when expert `id`'s bytes are in device memory (a slot or the shared
// expert), false for a miss read from the registered host copy.
__device__ __forceinline__ bool expert_on_device(const ExpertSrc &s, int id) {
    if (id == s.n_expert) return true;
    const int32_t slot = s.table ? s.table[id] : s.ns;
    return slot != s.ns && s.gate;
}

#define GU_ROWS 32   // gate/up rows per CTA of the stand-alone GEMVs
#define DN_ROWS 16   // down rows per CTA of the stand-alone GEMVs

cudaError_t launch_quantize(const float *x, void *y, int64_t n, int qtype, cudaStream_t s);
cudaError_t launch_synth_weights(void *y, int64_t nb, int qtype, uint64_t seed, float sigma,
                                 cudaStream_t s);
cudaError_t launch_synth_f32(float *y, int64_t n, uint64_t seed, float sigma, cudaStream_t s);
cudaError_t launch_router(const float *W, const float *x, int n_tok, int n_expert, int n_embd,
                          const int32_t *table, int ns, float delta, int use_prior, int k,
                          int32_t *ids, float *w, float *logits, const SlotState *st,
                          int observe_layer_idx, const int32_t *pub, cudaStream_t s);
cudaError_t launch_experts(const ExpertSrc &src, const float *x, const int32_t *ids,
                           const float *w, int n_tok, int k, int n_embd, int n_ff, int down_type,
                           float *act, const float *resid, float *y, int *err, cudaStream_t s);
cudaError_t launch_transpose(const float *in, float *out, int rows, int cols, cudaStream_t s);
cudaError_t launch_observe(const SlotState &st, int layer, const int32_t *ids, int n,
                           cudaStream_t s);
cudaError_t launch_step(const SlotState &st, int32_t *host_jobs, int32_t *host_njobs,
                        cudaStream_t s);
// just-in-time streaming: the lookahead scores of layers layer0 .. layer0 +
// n_targets - 1 (<= 2) on one token's x, the non-resident experts among
// their k best (out [n_targets][16], n_out [n_targets]) and the streamed
// jobs that claim pool slots for them (at most per_layer per layer and
// token); and the cancellation of streamed jobs (l, e, slot)
cudaError_t launch_ahead(const SlotState &st, const float *routers, const float *x, int layer0,
                         int n_targets, int n_embd, int k, int per_layer, float *scores, int32_t *out,
                         int32_t *n_out, cudaStream_t s);
cudaError_t launch_stream_cancel(const SlotState &st, const int32_t *jobs, int n, cudaStream_t s);
// speculative uploads of predicted ids for layer `layer` (early issue with a predictor)
cudaError_t launch_issue_spec(const SlotState &st, int layer, const int32_t *top, int n_top,
                              cudaStream_t s);

// ---- batched layer, tokens grouped by expert (moe_batched.cu) -------------

#define GROUP_TILE 8   // pairs per CTA tile of the grouped GEMVs

// Device buffers of one grouping: cnt [E], off [E + 1], pair_pos [P] (pair
// t * k + r -> position in expert order), pos_pair [P], tiles
// [group_max_tiles] ((expert << 16) | token tile), n_tiles [1].
struct GroupBufs {
    int32_t *cnt, *off, *pair_pos, *pos_pair, *tiles, *n_tiles;
};

// A wait that a kernel does before its work: until every flags[0 .. world)
// carries *epoch (acquire, system scope), bounded by wait_ns (on expiry the
// timeout bit goes into the kernel's error word and the kernel goes on).
// The expert-parallel exchange raises such flags in peer memory.
struct FlagWait {
    const unsigned long long *flags;
    int world;
    const unsigned long long *epoch;
    uint64_t wait_ns;
};

int group_max_tiles(int n_expert, int P, int tile);
// the routed pairs of each token followed by the shared expert (id n_expert, weight 1)
cudaError_t launch_append_shared(const int32_t *ids, const float *w, int n_tok, int k, int n_expert,
                                 int32_t *ids_x, float *w_x, cudaStream_t s);
cudaError_t launch_group(const int32_t *ids, int P, int n_expert, int tile, const GroupBufs &g,
                         int *err, cudaStream_t s, int div = 1, const FlagWait *wait = nullptr);
// bytes of scratch launch_experts_grouped needs for P pairs
size_t grouped_scratch_bytes(int P, int n_embd, int n_ff);
// gate/up + down over the grouped pairs (`scratch`: Q8_1 token rows and
// activations; ypair [P][n_embd]), then the combine into y.  n_embd 2048.
cudaError_t launch_experts_grouped(const ExpertSrc &src, const float *x, const GroupBufs &g,
                                   int n_tok, int k, int n_embd, int n_ff, int down_type,
                                   const float *w, void *scratch, float *ypair, const float *resid,
                                   float *y, int *err, cudaStream_t s);
cudaError_t launch_combine(const float *ypair, const int32_t *pair_pos, const float *w, int n_tok,
                           int k, int n_embd, const float *resid, float *y, cudaStream_t s,
                           const FlagWait *wait = nullptr, int *err = nullptr);

// ---- expert-parallel dispatch (moe_ep.cu) ----------------------------------

// Route pairs to ranks: the grouping `g` over `world` rank buckets (g.cnt =
// send counts, g.off[world] = pairs sent, g.pair_pos = send slot of each
// pair); send_ids [P], send_x [P][n_embd] in send-slot order.  capacity > 0:
// rank d's pairs go to slots [d * capacity, d * capacity + count), the other
// slots keep id -1, and g.pair_pos holds each pair's slot.
cudaError_t launch_ep_pack(const int32_t *ids, const float *x, int n_tok, int k, int n_expert,
                           int n_embd, int world, int capacity, const GroupBufs &g, int32_t *send_ids,
                           float *send_x, int *err, cudaStream_t s);

// The peer-memory exchange (moe_ep.cu): byte offsets of one rank's mailbox.
struct EpMail {
    int world, rank, cap, n_embd;          // cap: slots per (source, owner) block
    size_t off_fflag, off_rflag, off_meta, off_ids, off_x, off_rety, bytes;
};
// forward (send_count != null): the compact send list's blocks to every
// owner's mailbox, then meta + flags (advancing *epoch); return (send_count
// null): the owner's y rows [world][cap][n_embd] to every source's ret_y,
// then the return flags.  peer: device array of the world mailbox bases;
// done: a zeroed device counter the kernel's last CTA finds and resets.
cudaError_t launch_ep_push(const EpMail &m, uint8_t *const *peer, const int32_t *send_count,
                           const int32_t *send_ids, const float *src, unsigned long long *epoch,
                           unsigned int *done, cudaStream_t s);


// ---- tensor-core grouped GEMM (moe_gemm.cu) --------------------------------

#define GM_NT 64       // pairs per token tile of the GEMM (MMA N <= 64)

// fp16 elements of scratch the GEMM needs for P pairs (token tiles + activation tiles)
size_t gemm_scratch_halves(int n_expert, int P, int n_embd, int n_ff);
// gate/up + down on tcgen05 over pairs grouped with tile GM_NT, then the
// combine.  Q6_K down only; n_embd and n_ff multiples of 128.
cudaError_t launch_experts_gemm(const ExpertSrc &src, const float *x, const GroupBufs &g,
                                int n_tok, int k, int n_embd, int n_ff, int down_type,
                                const float *w, void *scratch, float *ypair, const float *resid,
                                float *y, int *err, cudaStream_t s);

// ---- persistent decode (moe_decode.cu) ------------------------------------

struct LayerDesc {
    const float *router_w;                 // [E][H] device
    const float *router_t;                 // [H][E] device (transposed)
    const uint8_t *gate, *up, *down;       // slot slabs
    const uint8_t *hgate, *hup, *hdown;    // mapped host or null
    const int32_t *table;                  // [E]
    const uint8_t *sgate, *sup, *sdown;    // shared expert (device) or null
    int32_t ns;
    int32_t pad_;
};

// Fixed-point router accumulators of the persistent decode kernel: one
// 128-byte line (16 int64) per total, so that the 148 CTAs' additions and
// reads of one total meet at one line each and no line becomes a hot spot.
constexpr int ACC_LINE = 16;
// one 128-byte line per rank's activation signal in the decode kernel
constexpr int READY_STRIDE = 32;

struct DecodeParams {
    int n_layers, n_expert, k, n_embd, n_ff, down_type;
    int kx;                                // experts per token: k, plus 1 with a shared expert
    int64_t gate_bytes, down_bytes;        // per expert
    const LayerDesc *layers;               // device [n_layers]
    const int32_t *gu_r0, *gu_r1;          // per CTA: flattened (k, row) range
    const int32_t *dn_h0, *dn_h1;          // per CTA: output-row range
    int gu_rows_max, dn_rows_max;          // staging sizes
    const float *h_in;                     // [n_tok][H]
    float *out;                            // [n_tok][H]
    int n_tok;
    float *resid;                          // [H]  residual stream
    float *logits;                         // [E] (unused by the 2-barrier kernel)
    long long *acc;                        // [2][E + 1][ACC_LINE]: router totals, double-buffered
    float *act;                            // [k][I]
    unsigned *bar;                         // grid barrier counter (zeroed per launch)
    unsigned *ready;                       // [MOE_KMAX][READY_STRIDE] per-rank activation signals (zeroed per launch)
    int n_prod[MOE_KMAX];                  // CTAs producing each rank's gate/up rows
    int *abort_flag;
    int *err;
    SlotState st;
    int observe;
    float delta;
    float rms_eps;
    float *dbg_x;                          // [n_tok][L][H] or null
    int32_t *dbg_ids;                      // [n_tok][L][k]
    float *dbg_w;
    float *dbg_y;                          // [n_tok][L][H]
    uint64_t *prof;                        // [n_tok][L][DEC_PHASES][grid] or null
    uint64_t wait_ns;                      // limit of every device wait (grid, rank, copies)
    int starve;                            // test hook: r + 1 starves rank r's first wait; 0 off
    int spec;                              // gate/up copies issued from the logits' top-k before the
                                           // exact selection (prior off): 1 on, 0 off, 2 on with a
                                           // wrong prediction every other (token, layer) (tests)
    // shared-memory layout (bytes from the start of dynamic smem)
    int off_xf, off_xq, off_xd, off_xs, off_aq, off_ad, off_as, off_ac, off_rt, off_tbl, off_rown,
        off_gu, off_dn, off_ys, off_prev, smem_bytes;
    int dn_stride;                         // bytes per expert chunk in the down staging
    int rt_rows;                           // router rows per CTA (ceil(E / grid))
};

int decode_smem_layout(DecodeParams &p, int grid);
cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t s);
int decode_max_grid(int smem_bytes, int device, int n_expert, int down_type);

}  // namespace moe
