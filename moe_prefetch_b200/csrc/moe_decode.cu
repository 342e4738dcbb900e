// moe_decode.cu -- persistent batch-1 decode over the whole MoE stack.
//
// One cooperative launch, one CTA per SM, 16 warps; one grid barrier per
// layer.  CTA c owns rows [h0, h1) of the residual stream for the whole
// token and, inside every layer, the flattened (rank, row) range [r0, r1)
// of the gate/up work.  Per token t and layer L:
//
//   -- grid barrier: the router totals of (t, L) and the residual rows are
//      complete --
//   1. every CTA reads the full residual (L2) and the E + 1 fixed-point
//      router totals (int64, added by every CTA with red.add: the same bits
//      whatever the order), normalises x = r * inv_rms and zeroes its share
//      of the other totals buffer;
//   2. warp 0: softmax, + cache prior from the layer's table row (prefetched
//      into shared memory), top-k and the renormalised weights in registers;
//      slots from the table; warps 1-8 quantise x to Q8_1 meanwhile; CTA 0
//      observes the routed ids (moe_obs_cb) with its counters on chip;
//   3. warp 0 issues one bulk copy (cp.async.bulk, TMA, no multicast) per
//      contiguous piece of this CTA's gate/up rows, waits for them to land,
//      then issues the down rows of its residual rows for all k experts, the
//      next layer's transposed router rows and its table row;
//   4. gate/up GEMV (Q4_K x Q8_1, dp4a) with SiLU*mul as pieces land;
//      activations to L2;
//   5. the CTA signals every rank it produced (release); warp 15 prefetches
//      the gate/up matrices of the previous token's experts of the next layer
//      into L2;
//   6. per rank, a group of warps waits for that rank's producers, quantises
//      its activations (Q8_1, padded shared-memory layout) and computes the
//      down GEMV rows (Q6_K x Q8_1) of this CTA's residual rows; then the
//      weighted combine in rank order and the residual add; the new rows go
//      to L2, and the partial logits / sum of squares of the NEXT layer over
//      these rows are added into the totals.
//
// Missed experts (table entry = n_slots) are read zero-copy from the
// registered host weights instead of the slot slabs.  Every wait (grid
// barrier, rank signal, mbarrier) is bounded by %globaltimer; on expiry the
// kernel raises an error bit and an abort flag, waits (bounded) for its own
// copies in flight, and returns.
#include "moe_kernels.h"

#include <algorithm>

namespace moe {

#define DEC_THREADS 512
#define DEC_WARPS (DEC_THREADS / 32)
#define MB_WT 0
#define MB_TBL 1
#define MB_GU 2    // 4 barriers: gate/up pieces
#define MB_DN 6    // MOE_KMAX barriers: down pieces
#define MB_FX (MB_DN + MOE_KMAX)   // 4 barriers: gate/up pieces re-issued after a wrong prediction
#define N_MB (MB_FX + 4)
#define DEC_PHASES 12

__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier in two halves, so that a CTA can do work that no other CTA
// waits for between its arrival and its wait: every CTA adds 1 (release),
// then waits (acquire) until the counter reaches epoch * gridDim.x.  Bounded
// by p.wait_ns; gives up on the shared abort flag.
__device__ __forceinline__ void grid_arrive(const DecodeParams &p, unsigned &epoch) {
    epoch += 1;
    __syncthreads();
    if (threadIdx.x == 0) red_release_add(p.bar, 1u);
}

__device__ __forceinline__ bool grid_wait(const DecodeParams &p, unsigned epoch, int *s_flag) {
    const unsigned target = epoch * gridDim.x;
    if (threadIdx.x == 0) {
        int ok = 1;
        if (ld_acquire_u32(p.bar) < target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire_u32(p.bar) < target) {
                if (ld_relaxed_i32(p.abort_flag)) { ok = 0; break; }
                if (gtimer() - t0 > p.wait_ns) {
                    atomicOr(p.err, MOE_DEV_ERR_TIMEOUT);
                    atomicExch(p.abort_flag, 1);
                    ok = 0;
                    break;
                }
            }
        }
        if (ok && ld_relaxed_i32(p.abort_flag)) ok = 0;   // a CTA gave up during the layer
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

__device__ __forceinline__ bool grid_sync(const DecodeParams &p, unsigned &epoch, int *s_flag) {
    grid_arrive(p, epoch);
    return grid_wait(p, epoch, s_flag);
}

__device__ __forceinline__ void copy_host16(uint8_t *dst, const uint8_t *src, int bytes) {
    for (int off = threadIdx.x * 16; off < bytes; off += DEC_THREADS * 16)
        *reinterpret_cast<uint4 *>(dst + off) = *reinterpret_cast<const uint4 *>(src + off);
}

__device__ __forceinline__ void red_add_u64(uint64_t *p, uint64_t v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// moe_obs_cb for one decode layer, one warp of CTA 0 (with early issue,
// lane 0 then issues the admitted misses' uploads).  Hits are stamped in
// parallel: the i-th routed id, if resident, gets clock + (hits before i) + 1,
// which is what the reference's sequential ++clock produces (the k ids are
// distinct).  Counters that only CTA 0 writes during the launch (the clock)
// live in shared memory; the others are fire-and-forget reductions.  Misses
// (window bookkeeping, the pending list) are walked in id order by lane 0.
__device__ __forceinline__ void observe_decode(const SlotState &st, int layer,
                                               const int32_t *ids, const int32_t *slots, int k,
                                               int ns, uint64_t *s_clock, int lane) {
    const int E = st.n_expert;
    const bool in = lane < k;
    const int id = in ? ids[lane] : 0;
    const int slot = in ? slots[lane] : ns;
    const bool hit = in && slot != ns;
    const unsigned hm = __ballot_sync(MOE_FULL, hit);
    const unsigned mm = __ballot_sync(MOE_FULL, in && !hit);
    const uint64_t clock = *s_clock;
    if (hit) {
        const int rank = __popc(hm & ((1u << lane) - 1u));
        st.last_use[st.slot_off[layer] + slot] = clock + (uint64_t)rank + 1;
    }
    if (in && st.heat) atomicAdd(st.heat + (size_t)layer * E + id, 1.0f);
    if (in && st.use_count) atomicAdd(st.use_count + (size_t)layer * E + id, 1u);
    if (lane == 0) {
        const int nh = __popc(hm);
        if (nh) red_add_u64(st.n_hit + layer, (uint64_t)nh);
        *s_clock = clock + (uint64_t)nh;
        if (mm) {
            const uint64_t n_steps = st.g[G_STEPS];
            int32_t *pend = st.pending + (size_t)layer * E;
            int np = st.n_pending[layer];
            unsigned m = mm;
            while (m) {
                const int i = __ffs(m) - 1;
                m &= m - 1;
                const int mid = ids[i];
                st.n_miss[layer] += 1;
                if (st.miss_last) {
                    uint64_t *ml = st.miss_last + (size_t)layer * E;
                    uint64_t *mp = st.miss_prev + (size_t)layer * E;
                    if (ml[mid] != n_steps) {
                        mp[mid] = ml[mid];
                        ml[mid] = n_steps;
                    }
                }
                bool dup = false;
                for (int q = 0; q < np; ++q)
                    if (pend[q] == mid) { dup = true; break; }
                if (!dup) pend[np++] = mid;
            }
            st.n_pending[layer] = np;
        }
    }
    // early issue: the admitted pending misses take slots of the free pool
    // now, after every lane's heat and recency updates (the clock in st.g is
    // not read there)
    __syncwarp();
    if (st.early_issue && lane == 0) early_issue_pending(st, layer);
    if (st.cur_ids && in) st.cur_ids[(size_t)layer * CUR_IDS + lane] = id;
    if (st.cur_ids && lane == 0) st.n_cur[layer] = k;
    __syncwarp();
}

// Cold path: missed experts read zero-copy from the registered host weights
// into the staging buffers (out of line to keep the hot loop's code compact;
// every argument by value or as a shared-memory pointer, so that nothing of
// the kernel's parameters has to live in local memory).
__device__ __noinline__ void host_miss_copies(const uint8_t *hgate, const uint8_t *hup,
                                              const uint8_t *hdown, int ns, int64_t gate_bytes,
                                              int64_t down_bytes, int dn_stride, int *err,
                                              const int32_t *s_ids, const int32_t *s_slot,
                                              int K, int nch, const int *ch_k, const int *ch_i0,
                                              const int *ch_n, const int *ch_off,
                                              uint8_t *gate_sm, uint8_t *up_sm, uint8_t *dn,
                                              int gurow, int drow, int h0, int h1) {
    const int tid = threadIdx.x;
    for (int q = 0; q < nch; ++q) {
        const int kk = ch_k[q];
        if (s_slot[kk] == ns) {
            const size_t off = (size_t)s_ids[kk] * gate_bytes + (size_t)ch_i0[q] * gurow;
            if (hgate && hup) {
                copy_host16(gate_sm + (size_t)ch_off[q] * gurow, hgate + off, ch_n[q] * gurow);
                copy_host16(up_sm + (size_t)ch_off[q] * gurow, hup + off, ch_n[q] * gurow);
            } else if (tid == 0) {
                atomicOr(err, MOE_DEV_ERR_INDEX);
            }
        }
    }
    for (int kk = 0; kk < K; ++kk) {
        if (h1 > h0 && s_slot[kk] == ns) {
            if (hdown) {
                const uint8_t *base = hdown + (size_t)s_ids[kk] * down_bytes;
                const uintptr_t a0 = reinterpret_cast<uintptr_t>(base + (size_t)h0 * drow);
                const uintptr_t a1 = reinterpret_cast<uintptr_t>(base + (size_t)h1 * drow);
                const uintptr_t s0 = a0 & ~uintptr_t(15), s1 = (a1 + 15) & ~uintptr_t(15);
                copy_host16(dn + (size_t)kk * dn_stride, reinterpret_cast<const uint8_t *>(s0),
                            (int)(s1 - s0));
            } else if (tid == 0) {
                atomicOr(err, MOE_DEV_ERR_INDEX);
            }
        }
    }
}

// One bulk copy (cp.async.bulk, TMA, no multicast) of gate/up piece q of
// this CTA into the staging buffers, for `slot` of the piece's rank (ld.ns:
// a miss, nothing copied here; -1: the shared expert's own buffer), completing
// on `bar`.
__device__ __forceinline__ void issue_gu_piece(const LayerDesc &ld, int slot, int q, const int *ch_i0,
                                               const int *ch_n, const int *ch_off, int gurow,
                                               int64_t gate_bytes, uint8_t *gate_sm, uint8_t *up_sm,
                                               uint64_t *bar) {
    const uint32_t bytes = (uint32_t)(ch_n[q] * gurow);
    fence_proxy_async();
    if (slot != ld.ns) {
        const size_t off = (size_t)ch_i0[q] * gurow;
        const uint8_t *gsrc = slot < 0 ? ld.sgate : ld.gate + (size_t)slot * gate_bytes;
        const uint8_t *usrc = slot < 0 ? ld.sup : ld.up + (size_t)slot * gate_bytes;
        mbar_arrive_expect_tx(bar, 2 * bytes);
        bulk_g2s(gate_sm + (size_t)ch_off[q] * gurow, gsrc + off, bytes, bar);
        bulk_g2s(up_sm + (size_t)ch_off[q] * gurow, usrc + off, bytes, bar);
    } else {
        mbar_arrive_expect_tx(bar, 0);
    }
}

// This CTA's share of the next step's fused router: partial logits over its
// residual rows (an FMA chain per expert, rows in order) and the partial sum of
// squares, added in fixed point to the step's accumulators A[e * ACC_LINE]
// (e < E) and A[E * ACC_LINE].
__device__ __forceinline__ void add_router_partials(long long *A, const float *wt, const float *rown,
                                                    int rows, int E) {
    for (int e = threadIdx.x; e < E; e += DEC_THREADS) {
        float acc = 0.0f;
        for (int i = 0; i < rows; ++i) acc = __fmaf_rn(wt[i * E + e], rown[i], acc);
        red_add_u64(reinterpret_cast<uint64_t *>(A + (size_t)e * ACC_LINE), (uint64_t)fx_logit(acc));
    }
    if (threadIdx.x == DEC_THREADS - 1) {
        float s = 0.0f;
        for (int i = 0; i < rows; ++i) s = __fmaf_rn(rown[i], rown[i], s);
        red_add_u64(reinterpret_cast<uint64_t *>(A + (size_t)E * ACC_LINE), (uint64_t)fx_sumsq(s));
    }
}

// The gate and up matrices of the previous token's experts of the next
// step's layer into L2, while the down rows of this step stream in: one bulk
// prefetch per (expert, matrix) slice of this CTA (1/G of each matrix), one
// lane each.  The next step's gate/up loads of the experts routed again then
// come from L2.  Measured and not done: prefetching the down matrices too,
// and warming with real copies into the free gate/up buffer (both slowed
// this step's down rows by more than they saved on the next).
// Resident experts only (a miss lives in host memory); pred: ids by rank,
// -1 unknown; the shared expert (rank K when kx > k) always.
__device__ __forceinline__ void prefetch_next_l2(const LayerDesc &ldn, const int32_t *pred,
                                                 const int32_t *tbl, int K, int KX, int E,
                                                 int64_t gate_bytes, int c, int G, int lane) {
    for (int item = lane; item < 2 * KX; item += 32) {
        const int r = item >> 1, m = item & 1;
        const int id = r < K ? pred[r] : E;
        if (id < 0 || id > E) continue;
        const int slot = id == E ? -1 : tbl[id];
        if (slot == ldn.ns || slot < -1) continue;
        const uint8_t *base = m == 0 ? (slot < 0 ? ldn.sgate : ldn.gate + (size_t)slot * gate_bytes)
                                     : (slot < 0 ? ldn.sup : ldn.up + (size_t)slot * gate_bytes);
        if (!base) continue;
        const int64_t o0 = ((int64_t)c * gate_bytes / G) & ~int64_t(15);
        const int64_t o1 = c + 1 == G ? gate_bytes : (((int64_t)(c + 1) * gate_bytes / G) & ~int64_t(15));
        if (o1 > o0) prefetch_l2(base + o0, (uint32_t)(o1 - o0));
    }
}

template <int E_T, bool Q6_T>
__global__ void __launch_bounds__(DEC_THREADS, 1) k_decode(DecodeParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    uint64_t *mb = reinterpret_cast<uint64_t *>(sm);
    float *xf = reinterpret_cast<float *>(sm + p.off_xf);
    int8_t *xq = reinterpret_cast<int8_t *>(sm + p.off_xq);
    float *xd = reinterpret_cast<float *>(sm + p.off_xd);
    float *xs = reinterpret_cast<float *>(sm + p.off_xs);
    int8_t *aq = reinterpret_cast<int8_t *>(sm + p.off_aq);
    float *ad = reinterpret_cast<float *>(sm + p.off_ad);
    float *as_ = reinterpret_cast<float *>(sm + p.off_as);
    int *ac = reinterpret_cast<int *>(sm + p.off_ac);          // [kx][I/16] -32 * group sums
    float *wt = reinterpret_cast<float *>(sm + p.off_rt);       // [rows][E] router^T rows
    int32_t *tbl = reinterpret_cast<int32_t *>(sm + p.off_tbl); // [E] table row
    int32_t *prev = reinterpret_cast<int32_t *>(sm + p.off_prev); // [NL][MOE_KMAX] last token's ids
    float *rown = reinterpret_cast<float *>(sm + p.off_rown);   // [rows] own residual rows
    uint8_t *gu = sm + p.off_gu;
    uint8_t *dn = sm + p.off_dn;
    float *ys = reinterpret_cast<float *>(sm + p.off_ys);

    __shared__ int32_t s_ids[MOE_KMAX];
    __shared__ float s_w[MOE_KMAX];
    __shared__ int32_t s_slot[MOE_KMAX];
    __shared__ float s_sumsq;
    __shared__ int s_flag;
    __shared__ int s_bad;
    __shared__ int s_any_miss;
    __shared__ int s_fail;
    __shared__ int s_fix;      // the gate/up pieces were requested again (wrong prediction)
    __shared__ int s_sp;       // the predicted pieces were requested
    __shared__ int s_go;       // ... and are all resident: the compute warps run ahead
    __shared__ int s_rest;     // warp 0 requested the down rows (run-ahead path)
    __shared__ uint64_t s_clock;

    const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int E = E_T;
    const int K = p.k, H = p.n_embd, I = p.n_ff, NL = p.n_layers;
    const int KX = p.kx;   // experts per token in the expert work: K, plus the shared one
    const int gurow = (H / MOE_QK) * MOE_Q4K_BYTES;
    const int drow = (I / MOE_QK) * (Q6_T ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    const int r0 = p.gu_r0[c], r1 = p.gu_r1[c];
    const int h0 = p.dn_h0[c], h1 = p.dn_h1[c];
    const int rows = h1 - h0;
    uint8_t *gate_sm = gu;
    uint8_t *up_sm = gu + (size_t)p.gu_rows_max * gurow;

    // static gate/up pieces of this CTA: [r0, r1) of the flattened (k, row);
    // the table lives in shared memory (it is indexed with run-time indices)
    __shared__ int ch_k[4], ch_i0[4], ch_n[4], ch_off[4];
    int nch = 0;
    for (int r = r0; r < r1 && nch < 4;) {
        const int kk = r / I, i0 = r % I;
        const int n = min(I - i0, r1 - r);
        if (tid == 0) { ch_k[nch] = kk; ch_i0[nch] = i0; ch_n[nch] = n; ch_off[nch] = r - r0; }
        ++nch;
        r += n;
    }

    if (tid == 0) {
        for (int i = 0; i < N_MB; ++i) mbar_init(&mb[i], 1);
        fence_mbar_init();
        s_bad = 0;
        if (c == 0) s_clock = p.st.g[G_CLOCK];
    }
    for (int i = tid; i < NL * MOE_KMAX; i += DEC_THREADS) prev[i] = -1;
    __syncthreads();

    unsigned epoch = 0;
    int use = 0;                      // (token, layer) index; barrier parity = use & 1
    bool pend_wt = false, pend_tbl = false, pend_gu = false, pend_dn = false;
    uint32_t wt_par = 0, tbl_par = 0;
    // Speculative copy issue (the cache prior off): warp 0 issues the gate/up
    // copies for the top-k of the logits, then computes the exact selection
    // while they land; a rank whose id differs makes it wait for those copies
    // and issue the right ones on the MB_FX barriers (fixed), parity fx_par.
    const bool spec = p.spec != 0 && !(p.delta > 0.0f);
    bool fixed = false;
    uint32_t fx_par = 0;

    // ---- prologue: router rows + table of layer 0, partials of (0, 0) --------
    if (tid == 0) {
        mbar_arrive_expect_tx(&mb[MB_WT], (uint32_t)(rows * E * 4));
        bulk_g2s(wt, p.layers[0].router_t + (size_t)h0 * E, (uint32_t)(rows * E * 4), &mb[MB_WT]);
        mbar_arrive_expect_tx(&mb[MB_TBL], (uint32_t)(E * 4));
        bulk_g2s(tbl, p.layers[0].table, (uint32_t)(E * 4), &mb[MB_TBL]);
    }
    pend_wt = pend_tbl = true;
    for (int i = tid; i < rows; i += DEC_THREADS) rown[i] = __ldg(p.h_in + h0 + i);
    if (!mbar_wait(&mb[MB_WT], 0, p.wait_ns)) {
        if (tid == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
    }
    pend_wt = false;
    wt_par = 1;
    __syncthreads();
    add_router_partials(p.acc, wt, rown, rows, E);   // step 0: buffer 0

    for (int t = 0; t < p.n_tok; ++t) {
        for (int L = 0; L < NL; ++L, ++use) {
            const LayerDesc ld = p.layers[L];
            const uint32_t par = (uint32_t)(use & 1);
#define PROF(ph) \
            if (p.prof && tid == ((ph) == 8 ? 32 : 0)) \
                p.prof[(((size_t)t * NL + L) * DEC_PHASES + (ph)) * G + c] = gtimer();
            PROF(0)

            // ---- A: partials and residual rows of (t, L) complete ---------------
            if (!grid_sync(p, epoch, &s_flag)) goto abort;
            PROF(1)

            // ---- 1. residual, the step's router totals, x = r * inv_rms ------------
            // Every CTA reads the full residual (one float4 per thread) and the
            // E + 1 fixed-point totals (one line each), and zeroes its share of
            // the other buffer: read during the previous step, next added to
            // after barrier B of this one.
            {
                // [E] logit totals (before * inv), in the down staging buffer: free
                // until this layer's down copies, which are issued after the
                // selection (the gate/up buffer may already be filling)
                float *tot = reinterpret_cast<float *>(dn);
                const long long *A = p.acc + (size_t)(use & 1) * (E + 1) * ACC_LINE;
                const float *src = L == 0 ? p.h_in + (size_t)t * H : p.resid;
                float4 xv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                const bool has_x = tid * 4 < H;
                if (has_x)
                    xv = L == 0 ? __ldg(reinterpret_cast<const float4 *>(src + tid * 4))
                                : __ldcg(reinterpret_cast<const float4 *>(src + tid * 4));
                const long long q = tid <= E ? __ldcg(A + (size_t)tid * ACC_LINE) : 0ll;
                if (tid == 0) {
                    long long *Z = p.acc + (size_t)((use + 1) & 1) * (E + 1) * ACC_LINE;
                    for (int e = c; e <= E; e += G) __stcg(Z + (size_t)e * ACC_LINE, 0ll);
                }
                if (has_x) *reinterpret_cast<float4 *>(xf + tid * 4) = xv;
                if (tid < E) tot[tid] = __fmul_rn(__ll2float_rn(q), FX_LOGIT_INV);
                if (tid == E) s_sumsq = __fmul_rn(__ll2float_rn(q), FX_SUMSQ_INV);
                __syncthreads();
                PROF(2)
                const float S = s_sumsq;
                const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(S, (float)H), p.rms_eps)));
                bool tbl_ok = true;
                if (pend_tbl) {
                    tbl_ok = mbar_wait(&mb[MB_TBL], tbl_par, p.wait_ns);
                    if (!tbl_ok && tid == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); s_bad = 1; }
                    pend_tbl = false;
                    tbl_par ^= 1;
                }
                const bool has_next = L + 1 < NL || t + 1 < p.n_tok;
                const int nl = L + 1 < NL ? L + 1 : 0;

                // warp 0: the exact selection (logits, softmax, prior, top-k, weights)
                // into s_ids / s_w / s_slot; returns true when a predicted id
                // (sp_id of rank `lane`, when sp_on) differs
                auto select_exact = [&](int sp_id, bool sp_on) -> bool {
                    int id_r;
                    float w_r;
                    // with a prediction (prior off), first the check that it is the
                    // selection; the full top-k only where it is not
                    const bool checked = sp_on && select_warp_check<E / 32>(tot, inv, K, lane, sp_id, id_r, w_r,
                                                                            s_ids, s_w);
                    if (!checked)
                        select_warp<E / 32>(tot, inv, tbl, ld.ns, p.delta, p.delta > 0.0f, K, lane, id_r, w_r,
                                            s_ids, s_w);
                    if (lane < K) {
                        const bool okid = id_r >= 0 && id_r < E;
                        s_ids[lane] = id_r;
                        prev[(size_t)L * MOE_KMAX + lane] = id_r;
                        s_w[lane] = w_r;
                        s_slot[lane] = okid ? tbl[id_r] : ld.ns;
                        if (!okid) { atomicOr(p.err, MOE_DEV_ERR_INDEX); s_bad = 1; }
                    }
                    if (KX > K && lane == K) {   // the shared expert: always on, weight 1, own buffer
                        s_ids[K] = E;
                        s_w[K] = 1.0f;
                        s_slot[K] = -1;
                    }
                    const bool missed = lane < K && (id_r < 0 || id_r >= E || tbl[id_r] == ld.ns);
                    const unsigned miss = __ballot_sync(MOE_FULL, missed);
                    if (lane == 0) s_any_miss = miss != 0;
                    const bool wrong = sp_on && __ballot_sync(MOE_FULL, lane < K && sp_id != id_r) != 0u;
                    __syncwarp();
                    return wrong;
                };
                // one warp of CTA 0: moe_obs_cb for the routed ids, and the debug dumps
                auto observe_ids = [&]() {
                    if (p.observe) observe_decode(p.st, L, s_ids, s_slot, K, ld.ns, &s_clock, lane);
                    if (p.dbg_ids && lane < K) {
                        p.dbg_ids[((size_t)t * NL + L) * K + lane] = s_ids[lane];
                        p.dbg_w[((size_t)t * NL + L) * K + lane] = s_w[lane];
                    }
                };
                // warp 0: once the gate/up pieces (barriers gmb, parity gpar) have
                // landed, which gives them the copy engine and HBM first, the down
                // rows of every rank, the next router rows and the next table
                auto issue_rest = [&](uint64_t *gmb, uint32_t gpar) {
                    __syncwarp();
                    if (lane < nch) mbar_wait(&gmb[lane], gpar, p.wait_ns);
                    __syncwarp();
                    if (lane >= 8 && lane < 8 + KX) {
                        const int kk = lane - 8;
                        const int slot = s_slot[kk];
                        fence_proxy_async();
                        if (rows > 0 && slot != ld.ns) {
                            const uint8_t *base = slot < 0 ? ld.sdown : ld.down + (size_t)slot * p.down_bytes;
                            const uintptr_t a0 = reinterpret_cast<uintptr_t>(base + (size_t)h0 * drow);
                            const uintptr_t a1 = reinterpret_cast<uintptr_t>(base + (size_t)h1 * drow);
                            const uintptr_t s0 = a0 & ~uintptr_t(15), s1 = (a1 + 15) & ~uintptr_t(15);
                            mbar_arrive_expect_tx(&mb[MB_DN + kk], (uint32_t)(s1 - s0));
                            bulk_g2s(dn + (size_t)kk * p.dn_stride, reinterpret_cast<const void *>(s0),
                                     (uint32_t)(s1 - s0), &mb[MB_DN + kk]);
                        } else {
                            mbar_arrive_expect_tx(&mb[MB_DN + kk], 0);
                        }
                    }
                    if (lane == 30 && has_next) {
                        fence_proxy_async();
                        mbar_arrive_expect_tx(&mb[MB_WT], (uint32_t)(rows * E * 4));
                        bulk_g2s(wt, p.layers[nl].router_t + (size_t)h0 * E, (uint32_t)(rows * E * 4),
                                 &mb[MB_WT]);
                    }
                    if (lane == 31 && has_next) {
                        fence_proxy_async();
                        mbar_arrive_expect_tx(&mb[MB_TBL], (uint32_t)(E * 4));
                        bulk_g2s(tbl, p.layers[nl].table, (uint32_t)(E * 4), &mb[MB_TBL]);
                    }
                };
                // warps 1..15: gate/up GEMV + SiLU*mul of this CTA's pieces (barriers
                // gmb, parity gpar), two rows per iteration; activations to L2
                auto gate_up_rows = [&](uint64_t *gmb, uint32_t gpar) {
                    const int units = (H / MOE_QK) * 4;
                    const int W = DEC_WARPS - 1, wi = warp - 1;
                    ActQ4 a;
                    if (lane < units) load_act_q4(a, xq, xd, xs, lane >> 2, lane & 3);
                    int waited = 0;
                    bool fail = false;
                    for (int rA = r0 + wi; rA < r1 && !fail; rA += 2 * W) {
                        const int rB = rA + W;
                        const bool hasB = rB < r1;
                        const int lA = rA - r0, lB = rB - r0;
                        int qA = 0, qB = 0;
                        while (qA + 1 < nch && lA >= ch_off[qA + 1]) ++qA;
                        while (hasB && qB + 1 < nch && lB >= ch_off[qB + 1]) ++qB;
                        if (!(waited & (1 << qA))) {
                            if (!mbar_wait(&gmb[qA], gpar, p.wait_ns)) { fail = true; break; }
                            waited |= 1 << qA;
                        }
                        if (hasB && !(waited & (1 << qB))) {
                            if (!mbar_wait(&gmb[qB], gpar, p.wait_ns)) { fail = true; break; }
                            waited |= 1 << qB;
                        }
                        float gA = 0.0f, uA = 0.0f, gB = 0.0f, uB = 0.0f;
                        if (lane < units) {
                            const int so = (lane >> 2) * MOE_Q4K_BYTES, pp = lane & 3;
                            gA = q4k_unit_dot(gate_sm + (size_t)lA * gurow + so, pp, a);
                            uA = q4k_unit_dot(up_sm + (size_t)lA * gurow + so, pp, a);
                            if (hasB) {
                                gB = q4k_unit_dot(gate_sm + (size_t)lB * gurow + so, pp, a);
                                uB = q4k_unit_dot(up_sm + (size_t)lB * gurow + so, pp, a);
                            }
                        }
                        // lanes 0-7: gate A, 8-15: up A, 16-23: gate B, 24-31: up B
                        const float sum = warp_sum4_t(gA, uA, gB, uB, lane);
                        const float up = __shfl_down_sync(MOE_FULL, sum, 8);
                        if (lane == 0)
                            __stcg(p.act + (size_t)ch_k[qA] * I + ch_i0[qA] + (lA - ch_off[qA]), silu_mul(sum, up));
                        if (lane == 16 && hasB)
                            __stcg(p.act + (size_t)ch_k[qB] * I + ch_i0[qB] + (lB - ch_off[qB]), silu_mul(sum, up));
                    }
                    if (fail && lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
                };

                // ---- 2. prediction (cache prior off): warp 0 takes the top-k of the
                //      logits and requests those experts' gate/up pieces; warps 1..15
                //      quantise x = r * inv to Q8_1 meanwhile ----------------------------
                int sp_id = -1;   // warp 0: the predicted id of rank `lane`
                bool sp_on = false, go = false;
                fixed = false;
                if (spec) {
                    if (warp == 0) {
                        const bool ok = __all_sync(MOE_FULL, tbl_ok);
                        bool resident = false;
                        if (ok) {
                            sp_id = spec_topk_warp<E / 32>(tot, inv, K, lane);
                            // tests of the re-issue path: a wrong rank-0 prediction in
                            // every other (token, layer)
                            if (p.spec == 2 && (use & 1) && lane == 0) sp_id = (sp_id + 1) % E;
                            int sp_slot = lane < K ? tbl[sp_id] : ld.ns;
                            if ((unsigned)sp_slot > (unsigned)ld.ns) sp_slot = ld.ns;
                            const int rk = lane < nch ? ch_k[lane] : 0;
                            const int sl = __shfl_sync(MOE_FULL, sp_slot, rk);
                            if (lane < nch)
                                issue_gu_piece(ld, rk < K ? sl : -1, lane, ch_i0, ch_n, ch_off, gurow,
                                               p.gate_bytes, gate_sm, up_sm, &mb[MB_GU + lane]);
                            resident = __ballot_sync(MOE_FULL, lane < K && sp_slot == ld.ns) == 0u;
                        }
                        if (lane == 0) { s_sp = ok ? 1 : 0; s_go = resident ? 1 : 0; }
                    } else {
                        q8_scale_quantize_cta(xf, inv, H / 32, xq, xd, xs, tid - 32, DEC_THREADS - 32);
                    }
                    __syncthreads();
                    sp_on = s_sp != 0;
                    go = sp_on && s_go != 0;
                    pend_gu = sp_on;
                }

                if (go) {
                    // ---- 3a. run ahead: warps 1..15 compute the predicted pieces while
                    //      warp 0 makes the exact selection and requests the down rows.
                    //      A wrong prediction is found before any activation is signalled:
                    //      the right pieces are then requested and computed again. --------
                    if (warp == 0) {
                        const bool wrong = select_exact(sp_id, true);
                        PROF(6)
                        if (c == 0) observe_ids();
                        const bool bad = s_bad != 0;
                        if (!bad) issue_rest(&mb[MB_GU], par);
                        if (lane == 0) { s_fix = wrong ? 1 : 0; s_rest = bad ? 0 : 1; }
                        PROF(7)
                    } else {
                        gate_up_rows(&mb[MB_GU], par);
                    }
                    __syncthreads();
                    pend_dn = s_rest != 0;
                    pend_wt = pend_tbl = pend_dn && has_next;
                    if (s_bad) {
                        if (tid == 0) atomicExch(p.abort_flag, 1);
                        goto abort;
                    }
                    if (s_fix) {
                        // the compute warps are done with the predicted pieces: the right
                        // ones go into the same buffers (missed experts from the host)
                        fixed = true;
                        if (warp == 0 && lane < nch)
                            issue_gu_piece(ld, s_slot[ch_k[lane]], lane, ch_i0, ch_n, ch_off, gurow, p.gate_bytes,
                                           gate_sm, up_sm, &mb[MB_FX + lane]);
                        if (s_any_miss)
                            host_miss_copies(ld.hgate, ld.hup, ld.hdown, ld.ns, p.gate_bytes, p.down_bytes,
                                             p.dn_stride, p.err, s_ids, s_slot, K, nch, ch_k, ch_i0, ch_n, ch_off,
                                             gate_sm, up_sm, dn, gurow, drow, h0, h1);
                        __syncthreads();
                    }
                    if (p.dbg_x && c == 0)
                        for (int i = tid; i < H; i += DEC_THREADS)
                            p.dbg_x[((size_t)t * NL + L) * H + i] = xf[i];
                } else {
                    // ---- 3b. the exact selection first (warp 0; warps 1..15 quantise x
                    //      unless the prediction did it), then the copies ---------------
                    if (warp == 0) {
                        const bool wrong = select_exact(sp_id, sp_on);
                        int fx = 0;
                        if (wrong) {
                            // wrong prediction, nothing computed yet: the predicted copies
                            // land first (the buffers are theirs until then), then the
                            // right ones go out
                            bool ok = lane < nch ? mbar_wait(&mb[MB_GU + lane], par, p.wait_ns) : true;
                            ok = __all_sync(MOE_FULL, ok);
                            if (!ok) {
                                if (lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); s_bad = 1; }
                            } else if (lane < nch) {
                                issue_gu_piece(ld, s_slot[ch_k[lane]], lane, ch_i0, ch_n, ch_off, gurow,
                                               p.gate_bytes, gate_sm, up_sm, &mb[MB_FX + lane]);
                            }
                            fx = ok ? 1 : 0;
                        }
                        if (lane == 0) s_fix = fx;
                    } else if (!spec) {
                        q8_scale_quantize_cta(xf, inv, H / 32, xq, xd, xs, tid - 32, DEC_THREADS - 32);
                    }
                    __syncthreads();
                    PROF(6)
                    fixed = s_fix != 0;
                    if (s_bad) {
                        if (tid == 0) atomicExch(p.abort_flag, 1);
                        goto abort;
                    }
                    if (p.dbg_x && c == 0)
                        for (int i = tid; i < H; i += DEC_THREADS)
                            p.dbg_x[((size_t)t * NL + L) * H + i] = xf[i];
                    if (c == 0 && warp == 1) observe_ids();
                    // warp 0 issues this layer's copies (+ next router rows / table); the
                    // issue blocks at roughly the data rate, so the other warps compute
                    // the gate/up rows meanwhile
                    if (warp == 0) {
                        if (!sp_on && lane < nch)
                            issue_gu_piece(ld, s_slot[ch_k[lane]], lane, ch_i0, ch_n, ch_off, gurow, p.gate_bytes,
                                           gate_sm, up_sm, &mb[MB_GU + lane]);
                        issue_rest(&mb[fixed ? MB_FX : MB_GU], fixed ? fx_par : par);
                    }
                    pend_wt = pend_tbl = has_next;
                    pend_gu = pend_dn = true;
                    // missed experts: zero-copy reads of the registered host weights
                    if (s_any_miss) {
                        host_miss_copies(ld.hgate, ld.hup, ld.hdown, ld.ns, p.gate_bytes, p.down_bytes,
                                         p.dn_stride, p.err, s_ids, s_slot, K, nch, ch_k, ch_i0, ch_n, ch_off,
                                         gate_sm, up_sm, dn, gurow, drow, h0, h1);
                        __syncthreads();
                    }
                    PROF(7)
                }
                // the pieces of the exact selection (after a run ahead: only when the
                // prediction was wrong)
                if (warp > 0 && (!go || fixed)) gate_up_rows(&mb[fixed ? MB_FX : MB_GU], fixed ? fx_par : par);
            }
            PROF(8)

            // ---- B: this CTA's gate/up rows are done: signal the ranks it produced
            //      (release; after the zeroing of the other router buffer, so that
            //      a CTA that has seen every rank's signal may add into it) --------
            if (tid == 0) s_fail = 0;
            __syncthreads();
            if (tid == 0)
                for (int q = 0; q < nch; ++q) red_release_add(p.ready + ch_k[q] * READY_STRIDE, 1u);
            PROF(9)
            pend_gu = false;
            if (fixed) fx_par ^= 1;
            // warp 15 puts the gate/up matrices of the previous token's experts
            // of the next step's layer into L2
            if (warp == DEC_WARPS - 1 && (L + 1 < NL || t + 1 < p.n_tok)) {
                // the next layer's table was queued with this layer's copies
                const int nl = L + 1 < NL ? L + 1 : 0;
                if (mbar_wait(&mb[MB_TBL], tbl_par, p.wait_ns))
                    prefetch_next_l2(p.layers[nl], prev + (size_t)nl * MOE_KMAX, tbl, K, KX, E,
                                     p.gate_bytes, c, G, lane);
            }

            // ---- 5/6. per rank k, a group of one or two warps: wait until every CTA
            //      producing rank k's activations has signalled, quantise them
            //      (Q8_1), then the down GEMV rows of rank k -- one lane per half
            //      super-block, 8-lane row groups.  Ranks whose producers finish
            //      early are done while the others still run; no grid barrier. ----
            {
                int kk = 0;
                while ((kk + 1) * DEC_WARPS / KX <= warp) ++kk;
                const int w0 = kk * DEC_WARPS / KX, nw = (kk + 1) * DEC_WARPS / KX - w0, gw = warp - w0;
                const unsigned gthreads = (unsigned)nw * 32u;
                if (gw == 0 && lane == 0) {
                    // p.starve = r + 1 (a test of the watchdog): rank r's first wait
                    // targets one signal more than its producers give
                    const unsigned target = (unsigned)(use + 1) * (unsigned)p.n_prod[kk] +
                                            (use == 0 && p.starve == kk + 1 ? 1u : 0u);
                    bool ok = true;
                    if (ld_acquire_u32(p.ready + kk * READY_STRIDE) < target) {
                        const uint64_t t0 = gtimer();
                        while (ld_acquire_u32(p.ready + kk * READY_STRIDE) < target) {
                            if (ld_relaxed_i32(p.abort_flag)) { ok = false; break; }
                            if (gtimer() - t0 > p.wait_ns) {
                                atomicOr(p.err, MOE_DEV_ERR_TIMEOUT);
                                atomicExch(p.abort_flag, 1);
                                ok = false;
                                break;
                            }
                        }
                    }
                    if (!ok) s_fail = 1;
                }
                if (nw > 1) asm volatile("bar.sync %0, %1;" ::"r"(1 + kk), "r"(gthreads) : "memory");
                else __syncwarp();
                // rank kk's activations -> Q8_1 (padded layout for the Q6_K rows)
                q8_quantize_cta16(p.act + (size_t)kk * I, I / 32,
                                  aq + (size_t)kk * (Q6_T ? I + I / 8 : I), ad + (size_t)kk * (I / 32),
                                  as_ + (size_t)kk * (I / 32),
                                  ac + (size_t)kk * (Q6_T ? ACT_C_STRIDE(I / 32) : I / 16),
                                  gw * 32 + lane, (int)gthreads, Q6_T ? I / 32 : 0);
                if (nw > 1) asm volatile("bar.sync %0, %1;" ::"r"(1 + kk), "r"(gthreads) : "memory");
                else __syncwarp();
                if (rows > 0) {
                    // Q6_K: a row is gs half-block units on consecutive lanes, 32 / gs
                    // rows per warp pass (5 with n_ff = 768)
                    const int gs = Q6_T ? (I / MOE_QK) * 2 : 8;
                    const int rpi = 32 / gs;
                    const int rr = lane / gs, u = lane - rr * gs;   // row in the pass, unit
                    const int nrg = Q6_T ? (rows + rpi - 1) / rpi : rows;
                    const int sl = s_slot[kk];
                    const uint8_t *base = sl < 0 ? ld.sdown
                        : sl != ld.ns ? ld.down + (size_t)sl * p.down_bytes
                                      : ld.hdown + (size_t)s_ids[kk] * p.down_bytes;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(base + (size_t)h0 * drow);
                    const uint8_t *rws = dn + (size_t)kk * p.dn_stride + (int)(a0 & 15);
                    const bool dn_ok = __all_sync(MOE_FULL, mbar_wait(&mb[MB_DN + kk], par, p.wait_ns));
                    if (!dn_ok && lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); s_fail = 1; }
                    for (int rg = gw; rg < nrg && dn_ok; rg += nw) {
                        if constexpr (Q6_T) {
                            const bool on = rr < rpi;
                            const int sb = u >> 1, hh = u & 1;
                            const int i = rg * rpi + rr;
                            ActHalfU a;
                            float v = 0.0f;
                            if (on) {
                                load_act_half_up(a, aq + (size_t)kk * (I + I / 8), ad + (size_t)kk * (I / 32),
                                                 ac + (size_t)kk * ACT_C_STRIDE(I / 32), sb, hh);
                                if (i < rows)
                                    v = q6k_half_dot_u(rws + (size_t)i * drow + sb * MOE_Q6K_BYTES, hh, a);
                            }
                            v = groupn_sum(v, u, gs);
                            if (on && u == 0 && i < rows) ys[kk * p.dn_rows_max + i] = v;
                        } else {
                            const int units = (I / MOE_QK) * 4;
                            const bool on = lane < units;
                            float v = 0.0f;
                            if (on) {
                                ActQ4 a;
                                load_act_q4(a, aq + (size_t)kk * I, ad + (size_t)kk * (I / 32),
                                            as_ + (size_t)kk * (I / 32), lane >> 2, lane & 3);
                                v = q4k_unit_dot(rws + (size_t)rg * drow + (lane >> 2) * MOE_Q4K_BYTES, lane & 3, a);
                            }
                            v = warp_sum(v);
                            if (lane == 0) ys[kk * p.dn_rows_max + rg] = v;
                        }
                    }
                }
            }
            PROF(10)
            __syncthreads();
            pend_dn = false;
            if (s_fail) {
                if (tid == 0) atomicExch(p.abort_flag, 1);
                goto abort;
            }
            const bool last = L == NL - 1;
            for (int i = tid; i < rows; i += DEC_THREADS) {
                float y = 0.0f;
                for (int kk = 0; kk < KX; ++kk) y = __fmaf_rn(s_w[kk], ys[kk * p.dn_rows_max + i], y);
                const float rn = __fadd_rn(rown[i], y);
                if (last) {
                    p.out[(size_t)t * H + h0 + i] = rn;
                    if (t + 1 < p.n_tok) rown[i] = __ldg(p.h_in + (size_t)(t + 1) * H + h0 + i);
                } else {
                    rown[i] = rn;
                    __stcg(p.resid + h0 + i, rn);
                }
                if (p.dbg_y) p.dbg_y[((size_t)t * NL + L) * H + h0 + i] = y;
            }
            PROF(11)
            // partials of the next (token, layer) over this CTA's rows
            if (pend_wt) {
                if (!mbar_wait(&mb[MB_WT], wt_par, p.wait_ns)) {
                    if (tid == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
                }
                __syncthreads();
                pend_wt = false;
                wt_par ^= 1;
                add_router_partials(p.acc + (size_t)((use + 1) & 1) * (E + 1) * ACC_LINE, wt, rown, rows, E);
            }
#undef PROF
        }
    }
    if (c == 0 && tid == 0) p.st.g[G_CLOCK] = s_clock;
    return;

abort:
    // bounded drain of this CTA's copies still in flight, then leave
    {
        const uint32_t par = (uint32_t)(use & 1);
        if (tid == 0) {
            if (pend_wt) mbar_wait(&mb[MB_WT], wt_par, p.wait_ns);
            if (pend_tbl) mbar_wait(&mb[MB_TBL], tbl_par, p.wait_ns);
            if (pend_gu) {
                for (int q = 0; q < nch; ++q) mbar_wait(&mb[MB_GU + q], par, p.wait_ns);
                if (fixed)
                    for (int q = 0; q < nch; ++q) mbar_wait(&mb[MB_FX + q], fx_par, p.wait_ns);
            }
            if (pend_dn)
                for (int kk = 0; kk < KX; ++kk) mbar_wait(&mb[MB_DN + kk], par, p.wait_ns);
            if (c == 0) p.st.g[G_CLOCK] = s_clock;
        }
        __syncthreads();
    }
}

static inline int align16(int v) { return (v + 15) & ~15; }

int decode_smem_layout(DecodeParams &p, int grid) {
    const int H = p.n_embd, I = p.n_ff, K = p.kx, E = p.n_expert;   // K: experts per token incl. shared
    const int gurow = (H / MOE_QK) * MOE_Q4K_BYTES;
    const int drow = (I / MOE_QK) * (p.down_type == MOE_QT_Q6K ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    (void)grid;
    int off = align16(N_MB * 8);
    p.off_xf = off; off = align16(off + H * 4);
    p.off_xq = off; off = align16(off + H);
    p.off_xd = off; off = align16(off + (H / 32) * 4);
    p.off_xs = off; off = align16(off + (H / 32) * 4);
    p.off_aq = off; off = align16(off + K * (I + I / 8));   // padded (load_act_half_up)
    p.off_ad = off; off = align16(off + K * (I / 32) * 4);
    p.off_as = off; off = align16(off + K * (I / 32) * 4);
    p.off_ac = off; off = align16(off + K * ACT_C_STRIDE(I / 32) * 4);
    p.off_rt = off; off = align16(off + p.dn_rows_max * E * 4);
    p.off_tbl = off; off = align16(off + E * 4);
    p.off_rown = off; off = align16(off + p.dn_rows_max * 4);
    p.off_gu = off; off = align16(off + 2 * p.gu_rows_max * gurow + 16);
    p.dn_stride = align16(p.dn_rows_max * drow + 32) + 16;
    p.off_dn = off; off = align16(off + K * p.dn_stride);
    p.off_ys = off; off = align16(off + K * p.dn_rows_max * 4);
    p.off_prev = off; off = align16(off + p.n_layers * MOE_KMAX * 4);
    p.smem_bytes = off;
    return off;
}

// the template instance for (n_expert, down type), or null
static const void *decode_kernel(int n_expert, int down_type) {
    const bool q6 = down_type == MOE_QT_Q6K;
    switch (n_expert) {
        case 32:  return q6 ? (const void *)k_decode<32, true> : (const void *)k_decode<32, false>;
        case 64:  return q6 ? (const void *)k_decode<64, true> : (const void *)k_decode<64, false>;
        case 128: return q6 ? (const void *)k_decode<128, true> : (const void *)k_decode<128, false>;
        case 256: return q6 ? (const void *)k_decode<256, true> : (const void *)k_decode<256, false>;
        default:  return nullptr;
    }
}

cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t s) {
    const void *fn = decode_kernel(p.n_expert, p.down_type);
    if (!fn) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem_bytes);
    if (e != cudaSuccess) return e;
    DecodeParams pp = p;
    void *args[] = {&pp};
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(DEC_THREADS), args, (size_t)p.smem_bytes, s);
}

int decode_max_grid(int smem_bytes, int device, int n_expert, int down_type) {
    const void *fn = decode_kernel(n_expert, down_type);
    if (!fn) return 0;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
        return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, DEC_THREADS, (size_t)smem_bytes) !=
        cudaSuccess)
        return 0;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return per_sm >= 1 ? sms : 0;
}

}  // namespace moe
