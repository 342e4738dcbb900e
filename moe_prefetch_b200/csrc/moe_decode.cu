// moe_decode.cu -- persistent batch-1 decode over the whole MoE stack.
//
// One cooperative launch, one CTA per SM, 16 warps.  For each token and
// layer every CTA:
//   1. reads the residual (L2), RMS-normalises it into shared memory;
//   2. computes its share of the router logits from router rows that were
//      bulk-copied into shared memory during the previous layer;
//   -- grid barrier (logits complete) --
//   3. selects top-k redundantly (canonical order -> every CTA gets the same
//      ids), resolves slots through the device table, and issues ONE bulk
//      copy (cp.async.bulk, TMA, no multicast) per contiguous piece of its
//      static share of the layer's expert bytes: gate/up rows of the
//      (expert, row) range it owns and the down rows of its output rows for
//      all k experts, plus the next layer's router rows;
//   4. computes gate/up GEMVs (Q4_K x Q8_1, dp4a) with SiLU*mul as each
//      piece lands, writes the activations to L2;
//   -- grid barrier (activations complete) --
//   5. re-quantises the k activation vectors (Q8_1) in shared memory;
//   6. computes the down GEMV rows (Q6_K x Q8_1) for all k experts, combines
//      them with the routing weights, adds the residual;
//   -- grid barrier (residual complete) at the start of the next layer --
// Every wait (grid barrier, mbarrier) is bounded by %globaltimer; on expiry
// the kernel raises an error bit and an abort flag, waits (bounded) for its
// own copies in flight, and returns.
#include "moe_kernels.h"

#include <algorithm>

namespace moe {

#define DEC_THREADS 512
#define DEC_WARPS (DEC_THREADS / 32)
#define MB_RT 0
#define MB_GU 1    // 4 barriers: gate/up pieces
#define MB_DN 5    // MOE_KMAX barriers: down pieces
#define N_MB (MB_DN + MOE_KMAX)

__device__ __forceinline__ bool grid_sync(const DecodeParams &p, unsigned &epoch, int *s_flag) {
    epoch += 1;
    const unsigned target = epoch * gridDim.x;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(p.bar, 1u);
        int ok = 1;
        if (ld_acquire_u32(p.bar) < target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire_u32(p.bar) < target) {
                if (ld_relaxed_i32(p.abort_flag)) { ok = 0; break; }
                if (gtimer() - t0 > MOE_TIMEOUT_NS) {
                    atomicOr(p.err, MOE_DEV_ERR_TIMEOUT);
                    atomicExch(p.abort_flag, 1);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        *s_flag = ok;
    }
    __syncthreads();
    return *s_flag != 0;
}

__device__ __forceinline__ void copy_host16(uint8_t *dst, const uint8_t *src, int bytes) {
    for (int off = threadIdx.x * 16; off < bytes; off += DEC_THREADS * 16)
        *reinterpret_cast<uint4 *>(dst + off) = *reinterpret_cast<const uint4 *>(src + off);
}

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
    float *rt = reinterpret_cast<float *>(sm + p.off_rt);
    uint8_t *gu = sm + p.off_gu;
    uint8_t *dn = sm + p.off_dn;
    float *ys = reinterpret_cast<float *>(sm + p.off_ys);

    __shared__ float s_lg[256];
    __shared__ int32_t s_ids[MOE_KMAX];
    __shared__ float s_w[MOE_KMAX];
    __shared__ int32_t s_slot[MOE_KMAX];
    __shared__ float s_red[DEC_WARPS];
    __shared__ int s_flag;
    __shared__ int s_bad;

    const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = p.n_expert, K = p.k, H = p.n_embd, I = p.n_ff, NL = p.n_layers;
    const int gurow = (H / MOE_QK) * MOE_Q4K_BYTES;
    const bool q6 = p.down_type == MOE_QT_Q6K;
    const int drow = (I / MOE_QK) * (q6 ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    const int r0 = p.gu_r0[c], r1 = p.gu_r1[c];
    const int h0 = p.dn_h0[c], h1 = p.dn_h1[c];
    const int rt_n = c < E ? (E - 1 - c) / G + 1 : 0;
    uint8_t *gate_sm = gu;
    uint8_t *up_sm = gu + (size_t)p.gu_rows_max * gurow;

    // static gate/up pieces of this CTA: [r0, r1) of the flattened (k, row)
    int ch_k[4], ch_i0[4], ch_n[4], ch_off[4];
    int nch = 0;
    for (int r = r0; r < r1 && nch < 4;) {
        const int kk = r / I, i0 = r % I;
        const int n = min(I - i0, r1 - r);
        ch_k[nch] = kk; ch_i0[nch] = i0; ch_n[nch] = n; ch_off[nch] = r - r0;
        ++nch;
        r += n;
    }

    if (tid == 0) {
        for (int i = 0; i < N_MB; ++i) mbar_init(&mb[i], 1);
        fence_mbar_init();
        s_bad = 0;
    }
    __syncthreads();

    unsigned epoch = 0;
    bool issued_rt = false;
    int use = 0;   // (token, layer) counter: each barrier completes once per use

    // router rows for (token 0, layer 0)
    if (tid == 0 && rt_n > 0) {
        mbar_arrive_expect_tx(&mb[MB_RT], (uint32_t)(rt_n * H * 4));
        for (int j = 0; j < rt_n; ++j)
            bulk_g2s(rt + (size_t)j * H, p.layers[0].router_w + (size_t)(c + G * j) * H,
                     (uint32_t)(H * 4), &mb[MB_RT]);
    }
    issued_rt = rt_n > 0;
    bool issued_gu = false, issued_dn = false;

    for (int t = 0; t < p.n_tok; ++t) {
        for (int L = 0; L < NL; ++L, ++use) {
            const LayerDesc ld = p.layers[L];
            const uint32_t par = (uint32_t)(use & 1);

            // ---- 1. x = RMSNorm(residual) ----------------------------------
            if (L > 0 && !grid_sync(p, epoch, &s_flag)) goto abort;
            {
                const float *src = L == 0 ? p.h_in + (size_t)t * H : p.resid;
                float ss = 0.0f;
                for (int i = tid * 4; i < H; i += DEC_THREADS * 4) {
                    const float4 v = L == 0 ? __ldg(reinterpret_cast<const float4 *>(src + i))
                                            : __ldcg(reinterpret_cast<const float4 *>(src + i));
                    *reinterpret_cast<float4 *>(xf + i) = v;
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
                ss = warp_sum(ss);
                if (lane == 0) s_red[warp] = ss;
                __syncthreads();
                if (warp == 0) {
                    float v = lane < DEC_WARPS ? s_red[lane] : 0.0f;
                    v = warp_sum(v);
                    if (lane == 0) s_red[0] = rsqrtf(v / (float)H + p.rms_eps);
                }
                __syncthreads();
                const float inv = s_red[0];
                for (int i = tid; i < H; i += DEC_THREADS) xf[i] *= inv;
                __syncthreads();
                if (p.dbg_x && c == 0)
                    for (int i = tid; i < H; i += DEC_THREADS)
                        p.dbg_x[((size_t)t * NL + L) * H + i] = xf[i];
            }

            // ---- 2. router logits of this CTA; x -> Q8_1 ------------------
            if (issued_rt) {
                if (!mbar_wait(&mb[MB_RT], par)) {
                    if (lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
                } else {
                    for (int j = warp; j < rt_n; j += DEC_WARPS) {
                        const float v = router_dot_warp(rt + (size_t)j * H, xf, H, lane);
                        if (lane == 0) __stcg(p.logits + c + G * j, v);
                    }
                }
            }
            for (int b = warp; b < H / 32; b += DEC_WARPS)
                q8_block_warp(xf[32 * b + lane], lane, xq + 32 * b, xd + b, xs + b);
            if (!grid_sync(p, epoch, &s_flag)) goto abort;
            issued_rt = false;

            // ---- 3. select, resolve, issue this layer's copies ------------
            for (int e = tid; e < E; e += DEC_THREADS) s_lg[e] = __ldcg(p.logits + e);
            __syncthreads();
            if (warp == 0)
                router_select_warp(s_lg, E, ld.table, ld.ns, p.delta, p.delta > 0.0f, K, s_ids, s_w,
                                   lane);
            __syncthreads();
            if (tid < K) {
                const int id = s_ids[tid];
                if (id < 0 || id >= E) {
                    atomicOr(p.err, MOE_DEV_ERR_INDEX);
                    s_bad = 1;
                    s_slot[tid] = ld.ns;
                } else {
                    s_slot[tid] = ld.table[id];
                }
            }
            __syncthreads();
            if (s_bad) {
                if (tid == 0) atomicExch(p.abort_flag, 1);
                goto abort;
            }
            if (c == 0 && tid == 0) {
                if (p.observe) observe_layer(p.st, L, s_ids, K);
                if (p.dbg_ids)
                    for (int i = 0; i < K; ++i) {
                        p.dbg_ids[((size_t)t * NL + L) * K + i] = s_ids[i];
                        p.dbg_w[((size_t)t * NL + L) * K + i] = s_w[i];
                    }
            }
            {
                // next (token, layer) router rows, into the buffer read above
                const bool has_next = L + 1 < NL || t + 1 < p.n_tok;
                const int nl = L + 1 < NL ? L + 1 : 0;
                if (tid == 0) {
                    fence_proxy_async();
                    if (has_next && rt_n > 0) {
                        mbar_arrive_expect_tx(&mb[MB_RT], (uint32_t)(rt_n * H * 4));
                        for (int j = 0; j < rt_n; ++j)
                            bulk_g2s(rt + (size_t)j * H,
                                     p.layers[nl].router_w + (size_t)(c + G * j) * H,
                                     (uint32_t)(H * 4), &mb[MB_RT]);
                    }
                    for (int q = 0; q < nch; ++q) {
                        const int kk = ch_k[q];
                        const int slot = s_slot[kk];
                        const uint32_t bytes = (uint32_t)(ch_n[q] * gurow);
                        if (slot != ld.ns) {
                            const size_t off = (size_t)slot * p.gate_bytes + (size_t)ch_i0[q] * gurow;
                            mbar_arrive_expect_tx(&mb[MB_GU + q], 2 * bytes);
                            bulk_g2s(gate_sm + (size_t)ch_off[q] * gurow, ld.gate + off, bytes, &mb[MB_GU + q]);
                            bulk_g2s(up_sm + (size_t)ch_off[q] * gurow, ld.up + off, bytes, &mb[MB_GU + q]);
                        } else {
                            mbar_arrive_expect_tx(&mb[MB_GU + q], 0);
                        }
                    }
                    for (int kk = 0; kk < K; ++kk) {
                        const int slot = s_slot[kk];
                        if (h1 > h0 && slot != ld.ns) {
                            const uint8_t *base = ld.down + (size_t)slot * p.down_bytes;
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
                }
                issued_rt = has_next && rt_n > 0;
                issued_gu = true;
                issued_dn = true;
                // missed experts: zero-copy reads of the registered host weights
                for (int q = 0; q < nch; ++q) {
                    const int kk = ch_k[q];
                    if (s_slot[kk] == ld.ns) {
                        const int id = s_ids[kk];
                        const size_t off = (size_t)id * p.gate_bytes + (size_t)ch_i0[q] * gurow;
                        if (ld.hgate && ld.hup) {
                            copy_host16(gate_sm + (size_t)ch_off[q] * gurow, ld.hgate + off, ch_n[q] * gurow);
                            copy_host16(up_sm + (size_t)ch_off[q] * gurow, ld.hup + off, ch_n[q] * gurow);
                        } else if (tid == 0) {
                            atomicOr(p.err, MOE_DEV_ERR_INDEX);
                        }
                    }
                }
                for (int kk = 0; kk < K; ++kk) {
                    if (h1 > h0 && s_slot[kk] == ld.ns) {
                        if (ld.hdown) {
                            const uint8_t *base = ld.hdown + (size_t)s_ids[kk] * p.down_bytes;
                            const uintptr_t a0 = reinterpret_cast<uintptr_t>(base + (size_t)h0 * drow);
                            const uintptr_t a1 = reinterpret_cast<uintptr_t>(base + (size_t)h1 * drow);
                            const uintptr_t s0 = a0 & ~uintptr_t(15), s1 = (a1 + 15) & ~uintptr_t(15);
                            copy_host16(dn + (size_t)kk * p.dn_stride, reinterpret_cast<const uint8_t *>(s0),
                                        (int)(s1 - s0));
                        } else if (tid == 0) {
                            atomicOr(p.err, MOE_DEV_ERR_INDEX);
                        }
                    }
                }
                __syncthreads();
            }

            // ---- 4. gate/up GEMV + SiLU*mul ----------------------------------
            {
                const int units = (H / MOE_QK) * 4;
                ActQ4 a;
                if (lane < units) load_act_q4(a, xq, xd, xs, lane >> 2, lane & 3);
                int waited = 0;   // bit q: piece q waited by this warp
                bool fail = false;
                for (int r = r0 + warp; r < r1; r += DEC_WARPS) {
                    const int lr = r - r0;
                    int q = 0;
                    while (q + 1 < nch && lr >= ch_off[q + 1]) ++q;
                    if (!(waited & (1 << q))) {
                        if (!mbar_wait(&mb[MB_GU + q], par)) { fail = true; break; }
                        waited |= 1 << q;
                    }
                    const int kk = ch_k[q];
                    const int i = ch_i0[q] + (lr - ch_off[q]);
                    float g = 0.0f, u = 0.0f;
                    if (lane < units) {
                        const int sb = lane >> 2, pp = lane & 3;
                        g = q4k_unit_dot(gate_sm + (size_t)lr * gurow + sb * MOE_Q4K_BYTES, pp, a);
                        u = q4k_unit_dot(up_sm + (size_t)lr * gurow + sb * MOE_Q4K_BYTES, pp, a);
                    }
                    g = warp_sum(g);
                    u = warp_sum(u);
                    if (lane == 0) __stcg(p.act + (size_t)kk * I + i, silu_mul(g, u));
                }
                if (fail && lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
            }
            if (!grid_sync(p, epoch, &s_flag)) goto abort;
            issued_gu = false;

            // ---- 5. activations -> Q8_1 -----------------------------------
            for (int b = warp; b < K * I / 32; b += DEC_WARPS)
                q8_block_warp(__ldcg(p.act + 32 * b + lane), lane, aq + 32 * b, ad + b, as_ + b);
            __syncthreads();

            // ---- 6. down GEMV, weighted combine, residual ------------------
            if (h1 > h0) {
                const int wpk = DEC_WARPS / K;   // warps per expert (>= 1)
                if (warp < K * wpk) {
                    const int kk = warp / wpk, sub = warp % wpk;
                    const uint8_t *base = ld.down + (size_t)s_slot[kk] * p.down_bytes;
                    if (s_slot[kk] == ld.ns) base = ld.hdown + (size_t)s_ids[kk] * p.down_bytes;
                    const uintptr_t a0 = reinterpret_cast<uintptr_t>(base + (size_t)h0 * drow);
                    const int lead = (int)(a0 & 15);
                    const uint8_t *rows = dn + (size_t)kk * p.dn_stride + lead;
                    if (!mbar_wait(&mb[MB_DN + kk], par)) {
                        if (lane == 0) { atomicOr(p.err, MOE_DEV_ERR_TIMEOUT); atomicExch(p.abort_flag, 1); }
                    } else if (q6) {
                        const int units = (I / MOE_QK) * 8;
                        ActQ6 a;
                        const bool act_on = lane < units;
                        if (act_on)
                            load_act_q6(a, aq + (size_t)kk * I, ad + (size_t)kk * (I / 32), lane >> 3,
                                        (lane >> 2) & 1, lane & 3);
                        for (int h = h0 + sub; h < h1; h += wpk) {
                            float v = 0.0f;
                            if (act_on)
                                v = q6k_unit_dot(rows + (size_t)(h - h0) * drow + (lane >> 3) * MOE_Q6K_BYTES,
                                                 (lane >> 2) & 1, lane & 3, a);
                            v = warp_sum(v);
                            if (lane == 0) ys[kk * p.dn_rows_max + (h - h0)] = v;
                        }
                    } else {
                        const int units = (I / MOE_QK) * 4;
                        ActQ4 a;
                        const bool act_on = lane < units;
                        if (act_on)
                            load_act_q4(a, aq + (size_t)kk * I, ad + (size_t)kk * (I / 32),
                                        as_ + (size_t)kk * (I / 32), lane >> 2, lane & 3);
                        for (int h = h0 + sub; h < h1; h += wpk) {
                            float v = 0.0f;
                            if (act_on)
                                v = q4k_unit_dot(rows + (size_t)(h - h0) * drow + (lane >> 2) * MOE_Q4K_BYTES,
                                                 lane & 3, a);
                            v = warp_sum(v);
                            if (lane == 0) ys[kk * p.dn_rows_max + (h - h0)] = v;
                        }
                    }
                }
            }
            __syncthreads();
            issued_dn = false;
            for (int h = h0 + tid; h < h1; h += DEC_THREADS) {
                float y = 0.0f;
                for (int kk = 0; kk < K; ++kk) y = __fmaf_rn(s_w[kk], ys[kk * p.dn_rows_max + (h - h0)], y);
                const float rin = L == 0 ? __ldg(p.h_in + (size_t)t * H + h) : p.resid[h];
                const float rn = __fadd_rn(rin, y);
                __stcg(p.resid + h, rn);
                if (L == NL - 1) p.out[(size_t)t * H + h] = rn;
                if (p.dbg_y) p.dbg_y[((size_t)t * NL + L) * H + h] = y;
            }
            if (ld_relaxed_i32(p.abort_flag)) goto abort;
        }
    }
    return;

abort:
    // bounded drain of this CTA's copies still in flight, then leave
    {
        const uint32_t par = (uint32_t)(use & 1);
        if (tid == 0) {
            if (issued_rt) mbar_wait(&mb[MB_RT], par);
            if (issued_gu)
                for (int q = 0; q < nch; ++q) mbar_wait(&mb[MB_GU + q], par);
            if (issued_dn)
                for (int kk = 0; kk < K; ++kk) mbar_wait(&mb[MB_DN + kk], par);
        }
        __syncthreads();
    }
}

static inline int align16(int v) { return (v + 15) & ~15; }

int decode_smem_layout(DecodeParams &p, int grid) {
    const int H = p.n_embd, I = p.n_ff, K = p.k, E = p.n_expert;
    const int gurow = (H / MOE_QK) * MOE_Q4K_BYTES;
    const int drow = (I / MOE_QK) * (p.down_type == MOE_QT_Q6K ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    int off = align16(N_MB * 8);
    p.off_xf = off; off = align16(off + H * 4);
    p.off_xq = off; off = align16(off + H);
    p.off_xd = off; off = align16(off + (H / 32) * 4);
    p.off_xs = off; off = align16(off + (H / 32) * 4);
    p.off_aq = off; off = align16(off + K * I);
    p.off_ad = off; off = align16(off + K * (I / 32) * 4);
    p.off_as = off; off = align16(off + K * (I / 32) * 4);
    p.rt_rows = (E + grid - 1) / grid;
    p.off_rt = off; off = align16(off + p.rt_rows * H * 4);
    p.off_gu = off; off = align16(off + 2 * p.gu_rows_max * gurow + 16);
    p.dn_stride = align16(p.dn_rows_max * drow + 32) + 16;
    p.off_dn = off; off = align16(off + K * p.dn_stride);
    p.off_ys = off; off = align16(off + K * p.dn_rows_max * 4);
    p.smem_bytes = off;
    return off;
}

cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         p.smem_bytes);
    if (e != cudaSuccess) return e;
    DecodeParams pp = p;
    void *args[] = {&pp};
    return cudaLaunchCooperativeKernel((const void *)k_decode, dim3(grid), dim3(DEC_THREADS), args,
                                       (size_t)p.smem_bytes, s);
}

int decode_max_grid(int smem_bytes, int device) {
    if (cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) !=
        cudaSuccess)
        return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode, DEC_THREADS,
                                                      (size_t)smem_bytes) != cudaSuccess)
        return 0;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return per_sm >= 1 ? sms : 0;
}

}  // namespace moe
