// moe_batched.cu -- the MoE layer for n_tok > 1 with tokens grouped by expert.
//
// The per-pair kernels (k_gate_up / k_down) read an expert's rows once per
// (token, expert) pair.  With a batch, many tokens share an expert, so here
// the routed pairs are first grouped by expert (k_group), and every CTA then
// reads its expert rows once for all of that expert's pairs in its tile:
//
//   k_group           pairs -> per-expert counts, offsets, stable positions,
//                     and the tile list (expert, token tile)
//   k_quant_rows      token rows -> Q8_1, once
//   k_gate_up_grouped gate/up GEMV (Q4_K x Q8_1) + SiLU*mul per pair, the
//                     activations quantised to Q8_1 per 32-row block
//   k_down_grouped    down GEMV per pair -> unweighted rows ypair[pos][h]
//   k_combine         y[t] = sum_r w[t][r] * ypair[pos(t, r)] in rank order
//
// Per pair, the activation and the down rows use exactly the unit mapping and
// reduction order of the per-pair kernels, and the combine adds in the same
// rank order.  The layer output is therefore bit-identical to the per-pair
// path, while the weights cross DRAM once per (expert, CTA) instead of once per
// pair.
#include "moe_kernels.h"

#include <algorithm>

namespace moe {

#define GROUP_THREADS 1024
#define GROUP_MAX_BUCKETS 264   // 256 routed experts + the shared one, rounded up

// One CTA, after `wait` when it has flags (the ids may come from peers).
// Pair p = t * k + r (token t, rank r) goes to bucket ids[p] / div
// (div 1: its expert; E / world: the rank owning the expert).  Positions are
// stable: the pairs of a bucket keep pair order.  Writes cnt[E], off[E + 1],
// pair_pos[P] (-1 for an id out of range, flagged in *err, and for the
// empty-slot id -1, skipped silently), pos_pair[P], and
// tiles[0 .. n_tiles) = (bucket << 16) | token-tile for tiles of `tile` pairs.
__global__ void __launch_bounds__(GROUP_THREADS) k_group(const int32_t *__restrict__ ids, int P,
                                                         int n_expert, int div, int tile, int32_t *cnt,
                                                         int32_t *off, int32_t *pair_pos,
                                                         int32_t *pos_pair, int32_t *tiles,
                                                         int32_t *n_tiles, int *err, FlagWait wait) {
    if (wait.flags) cta_wait_flags(wait.flags, wait.world, wait.epoch, wait.wait_ns, err);
    __shared__ int s_cnt[GROUP_MAX_BUCKETS], s_off[GROUP_MAX_BUCKETS + 1], s_base[GROUP_MAX_BUCKETS];
    // per warp and bucket: the warp's count in the chunk (low 16 bits), after
    // the scan the exclusive prefix over the chunk's warps (high 16 bits)
    __shared__ int s_wc[GROUP_THREADS / 32][GROUP_MAX_BUCKETS];
    __shared__ int s_bold[GROUP_MAX_BUCKETS];   // a bucket's base before the chunk
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < n_expert; e += GROUP_THREADS) { s_cnt[e] = 0; s_base[e] = 0; }
    for (int i = tid; i < (GROUP_THREADS / 32) * GROUP_MAX_BUCKETS; i += GROUP_THREADS)
        (&s_wc[0][0])[i] = 0;
    __syncthreads();
    for (int p0 = tid; p0 < P; p0 += 8 * GROUP_THREADS) {   // 8 loads in flight per thread
        int ev[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int p = p0 + j * GROUP_THREADS;
            ev[j] = p < P ? ids[p] : -1;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = ev[j];
            if (e >= 0 && e < n_expert * div) atomicAdd(&s_cnt[div == 1 ? e : e / div], 1);
            else if (e >= 0 || e < -1) atomicOr(err, MOE_DEV_ERR_INDEX);   // -1: an empty slot, skipped
        }
    }
    __syncthreads();
    if (warp == 0) {
        // lane l owns buckets [l*per, (l+1)*per): local sums of pairs and
        // tiles, an exclusive scan across lanes, then offsets and tile entries
        const int per = (n_expert + 31) / 32;
        int cs = 0, ts = 0;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < n_expert) { cs += s_cnt[e]; ts += (s_cnt[e] + tile - 1) / tile; }
        }
        int ci = cs, ti = ts;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int cu = __shfl_up_sync(MOE_FULL, ci, o), tu = __shfl_up_sync(MOE_FULL, ti, o);
            if (lane >= o) { ci += cu; ti += tu; }
        }
        int acc = ci - cs, nt = ti - ts;
        for (int i = 0; i < per; ++i) {
            const int e = lane * per + i;
            if (e < n_expert) {
                s_off[e] = acc;
                acc += s_cnt[e];
                for (int t0 = 0; t0 < s_cnt[e]; t0 += tile) tiles[nt++] = (e << 16) | (t0 / tile);
            }
        }
        if (lane == 31) {
            s_off[n_expert] = acc;
            *n_tiles = nt;
        }
    }
    __syncthreads();
    for (int e = tid; e <= n_expert; e += GROUP_THREADS) {
        off[e] = s_off[e];
        if (e < n_expert) cnt[e] = s_cnt[e];
    }
    const unsigned lt = (1u << lane) - 1u;
    // chunks of GROUP_THREADS pairs: per-warp counts per bucket, then one
    // thread per bucket turns them into the exclusive prefix over warps
    // (counts cleared for the next chunk) and advances the bucket's base
    for (int c0 = 0; c0 < P; c0 += GROUP_THREADS) {
        const int p = c0 + tid;
        int e = p < P ? ids[p] : -1;
        e = e < 0 || e >= n_expert * div ? -1 : div == 1 ? e : e / div;
        const unsigned mask = __match_any_sync(MOE_FULL, e);
        if (e >= 0 && lane == __ffs(mask) - 1) s_wc[warp][e] = __popc(mask);
        __syncthreads();
        for (int q = tid; q < n_expert; q += GROUP_THREADS) {
            int rel = 0;
#pragma unroll 8
            for (int w = 0; w < GROUP_THREADS / 32; ++w) {
                const int v = s_wc[w][q] & 0xFFFF;
                s_wc[w][q] = rel << 16;
                rel += v;
            }
            s_bold[q] = s_base[q];
            s_base[q] += rel;
        }
        __syncthreads();
        if (e >= 0) {
            const int pos = s_off[e] + s_bold[e] + (s_wc[warp][e] >> 16) + __popc(mask & lt);
            pair_pos[p] = pos;
            pos_pair[pos] = p;
        } else if (p < P) {
            pair_pos[p] = -1;
        }
    }
}

#define GU2_ROWS 64    // gate/up rows per CTA: two Q8_1 blocks of every pair's activations
#define DN2_ROWS 64    // down rows per CTA for Q4_K down weights: 8 per warp

// Down rows per CTA for Q6_K down weights: two warp passes of 32 / gs rows,
// gs = 2 n_ff / 256 lanes per row (80 rows at n_ff = 768, 128 at 512).
static inline int dn2_rows_q6(int n_ff) { return 8 * 2 * (32 / (2 * (n_ff / MOE_QK))); }

// x [n_rows][n_embd] -> Q8_1 (xq, d, s per 32-block), with the quantiser of
// k_gate_up, once per row.  grid n_rows; block 256.
__global__ void __launch_bounds__(256) k_quant_rows(const float *__restrict__ x, int n_embd,
                                                    int8_t *__restrict__ xq, float *__restrict__ xd,
                                                    float *__restrict__ xs) {
    const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nblk = n_embd / 32;
    // up to 8 blocks per warp: every load issued before the first block's arithmetic
    for (int b0 = warp; b0 < nblk; b0 += 8 * nw) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int b = b0 + j * nw;
            v[j] = b < nblk ? x[(size_t)t * n_embd + 32 * b + lane] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int b = b0 + j * nw;
            if (b < nblk)
                q8_block_warp(v[j], lane, xq + (size_t)t * n_embd + 32 * b, xd + (size_t)t * nblk + b,
                              xs + (size_t)t * nblk + b);
        }
    }
}

// Sum of each of 16 values over the 32 lanes, with every lane pair (l, l ^ o)
// combined at o = 16, 8, 4, 2, 1 exactly as warp_sum combines them, so each
// sum is bit-identical to warp_sum of that value.  Values are halved at each
// level: lane l ends with the sum of value l >> 1.
__device__ __forceinline__ float warp_sum16(float (&v)[16], int lane) {
    float a[8], b[4], c[2];
    const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float keep = u16 ? v[8 + i] : v[i], send = u16 ? v[i] : v[8 + i];
        a[i] = keep + __shfl_xor_sync(MOE_FULL, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float keep = u8 ? a[4 + i] : a[i], send = u8 ? a[i] : a[4 + i];
        b[i] = keep + __shfl_xor_sync(MOE_FULL, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float keep = u4 ? b[2 + i] : b[i], send = u4 ? b[i] : b[2 + i];
        c[i] = keep + __shfl_xor_sync(MOE_FULL, send, 4);
    }
    const float keep = u2 ? c[1] : c[0], send = u2 ? c[0] : c[1];
    float d = keep + __shfl_xor_sync(MOE_FULL, send, 2);
    return d + __shfl_xor_sync(MOE_FULL, d, 1);
}

// Padded shared-memory layouts of the tile's Q8_1 rows.  A lane reads one
// contiguous unit of a row (Q4_K: 64 int8, Q6_K: 128 int8) with 16-byte
// loads.  Units are stored at a 16-byte-padded stride (80 and 144 bytes), so
// the 8 lanes of a load phase hit disjoint banks.
#define PAD_U64 80     // stride of a 64-int8 unit
#define PAD_U128 144   // stride of a 128-int8 unit

// Copy rows[j] (j < np) of a Q8_1 buffer (values q [.][n], d/s [.][n/32])
// into shared memory: values unit-padded (`unit` int8 per unit, `stride`
// bytes apart), d and s dense [j][n/32].
__device__ __forceinline__ void stage_q8_padded(int8_t *q_s, float *d_s, float *s_s, const int8_t *q,
                                                const float *d, const float *sg, const int *rows,
                                                int np, int n, int unit, int stride) {
    const int c16 = n / 16, cpu = unit / 16, nb = n / 32;
    const int rowb = (n / unit) * stride;
    for (int i = threadIdx.x; i < np * c16; i += blockDim.x) {
        const int j = i / c16, c = i % c16;
        *reinterpret_cast<int4 *>(q_s + (size_t)j * rowb + (c / cpu) * stride + (c % cpu) * 16) =
            reinterpret_cast<const int4 *>(q + (size_t)rows[j] * n)[c];
    }
    for (int i = threadIdx.x; i < np * nb; i += blockDim.x) {
        const int j = i / nb, c = i % nb;
        d_s[j * nb + c] = d[(size_t)rows[j] * nb + c];
        if (s_s) s_s[j * nb + c] = sg[(size_t)rows[j] * nb + c];
    }
}

// Gate/up for the pairs of one tile over GU2_ROWS rows.  grid (n_ff / GU2_ROWS, max
// tiles); block 256.  The CTA stages the tile's Q8_1 token rows in shared
// memory; the gate and up rows are read by the lanes from the expert's
// memory.  Each warp takes GU2_ROWS / 8 rows:
// - every lane decodes its unit of the row once;
// - for every pair, the per-pair kernel's unit dots;
// - one transposed reduction of all 2 x np sums (warp_sum's pairing).
// Every activation is therefore bit-identical to k_gate_up's.  Each 32
// activations of a pair form one Q8_1 block, quantised as k_down does, into
// aq/ad/as [pos][...].
__global__ void __launch_bounds__(256, 2) k_gate_up_grouped(
    ExpertSrc src, const int8_t *__restrict__ xq, const float *__restrict__ xd,
    const float *__restrict__ xs, const int32_t *__restrict__ off, const int32_t *__restrict__ cnt,
    const int32_t *__restrict__ pos_pair, const int32_t *__restrict__ tiles,
    const int32_t *__restrict__ n_tiles, int k, int n_embd, int n_ff, int8_t *__restrict__ aq,
    float *__restrict__ ad, float *__restrict__ as, int *err) {
    extern __shared__ __align__(128) uint8_t smg[];
    __shared__ float act_s[GROUP_TILE][GU2_ROWS];
    __shared__ int s_tok[GROUP_TILE];
    if ((int)blockIdx.y >= *n_tiles) return;
    const int tl = tiles[blockIdx.y], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GROUP_TILE;
    const int np = min(GROUP_TILE, cnt[e] - tt * GROUP_TILE);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint8_t *gbase = expert_ptr(src, 0, e);
    const uint8_t *ubase = expert_ptr(src, 1, e);
    if (!gbase || !ubase) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    if (threadIdx.x < np) s_tok[threadIdx.x] = pos_pair[pos0 + threadIdx.x] / k;
    const size_t rb = (size_t)(n_embd / MOE_QK) * MOE_Q4K_BYTES;
    const int i0 = blockIdx.x * GU2_ROWS;
    const int nblk = n_embd / 32;
    const int xrow = (n_embd / 64) * PAD_U64;                                    // padded row bytes
    int8_t *xq_s = reinterpret_cast<int8_t *>(smg);                              // [8][xrow]
    float *xd_s = reinterpret_cast<float *>(xq_s + (size_t)GROUP_TILE * xrow);   // [8][nblk]
    float *xs_s = xd_s + GROUP_TILE * nblk;
    const int units = (n_embd / MOE_QK) * 4;   // n_embd == 2048: one unit per lane
    const bool on = lane < units;
    const int sb = lane >> 2, pp = lane & 3;
    // a lane reads its unit of each row straight from the expert's memory
    // (device slot, or registered host memory for a missed expert): every
    // weight byte is used by one lane once, so nothing is staged; the next
    // row's loads are in flight while a row is computed
    const uint8_t *grow = gbase + (size_t)i0 * rb + sb * MOE_Q4K_BYTES;
    const uint8_t *urow = ubase + (size_t)i0 * rb + sb * MOE_Q4K_BYTES;
    Q4Unit wg, wu;
    if (on && warp < GU2_ROWS) {
        q4k_unit_load(grow + (size_t)warp * rb, pp, wg);
        q4k_unit_load(urow + (size_t)warp * rb, pp, wu);
    }
    __syncthreads();   // s_tok
    stage_q8_padded(xq_s, xd_s, xs_s, xq, xd, xs, s_tok, np, n_embd, 64, PAD_U64);
    __syncthreads();
    for (int r = warp; r < GU2_ROWS; r += nw) {
        Q4UnitDec dg, du;
        if (on) {
            q4k_unit_decode(wg, pp, dg);
            q4k_unit_decode(wu, pp, du);
            if (r + nw < GU2_ROWS) {
                q4k_unit_load(grow + (size_t)(r + nw) * rb, pp, wg);
                q4k_unit_load(urow + (size_t)(r + nw) * rb, pp, wu);
            }
        }
        if (np <= 2) {
            // the common decode case: the four sums of at most two pairs by
            // warp_sum4_t (bit-identical to warp_sum16's)
            float g0 = 0.0f, u0 = 0.0f, g1 = 0.0f, u1 = 0.0f;
            if (on) {
                ActQ4 a;
                load_act_q4_unit(a, xq_s + lane * PAD_U64, xd_s, xs_s, 2 * lane);
                g0 += q4k_dec_compute(dg, a);
                u0 += q4k_dec_compute(du, a);
                if (np == 2) {
                    load_act_q4_unit(a, xq_s + (size_t)xrow + lane * PAD_U64, xd_s + nblk, xs_s + nblk,
                                     2 * lane);
                    g1 += q4k_dec_compute(dg, a);
                    u1 += q4k_dec_compute(du, a);
                }
            }
            const float sum = warp_sum4_t(g0, u0, g1, u1, lane);   // lanes 0-7 g0, 8-15 u0, 16-23 g1, 24-31 u1
            const float other = __shfl_down_sync(MOE_FULL, sum, 8);
            if (lane == 0) act_s[0][r] = silu_mul(sum, other);
            if (lane == 16 && np == 2) act_s[1][r] = silu_mul(sum, other);
        } else if (np <= 4) {
            // three or four pairs: the eight sums by warp_sum8_t (bit-identical)
            float v[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float g = 0.0f, up = 0.0f;
                if (on && j < np) {
                    ActQ4 a;
                    load_act_q4_unit(a, xq_s + (size_t)j * xrow + lane * PAD_U64, xd_s + j * nblk,
                                     xs_s + j * nblk, 2 * lane);
                    g += q4k_dec_compute(dg, a);
                    up += q4k_dec_compute(du, a);
                }
                v[j] = g;
                v[4 + j] = up;
            }
            const float sum = warp_sum8_t(v, lane);            // lane l: value l >> 2
            const float other = __shfl_down_sync(MOE_FULL, sum, 16);   // lane l < 16: value 4 + (l >> 2)
            if (lane < 16 && !(lane & 3) && (lane >> 2) < np)
                act_s[lane >> 2][r] = silu_mul(sum, other);
        } else {
            float v[16];
#pragma unroll
            for (int j = 0; j < GROUP_TILE; ++j) {
                float g = 0.0f, up = 0.0f;
                if (on && j < np) {
                    ActQ4 a;
                    load_act_q4_unit(a, xq_s + (size_t)j * xrow + lane * PAD_U64, xd_s + j * nblk,
                                     xs_s + j * nblk, 2 * lane);
                    g += q4k_dec_compute(dg, a);
                    up += q4k_dec_compute(du, a);
                }
                v[j] = g;
                v[GROUP_TILE + j] = up;
            }
            const float sum = warp_sum16(v, lane);      // lane l: value l >> 1
            const float other = __shfl_down_sync(MOE_FULL, sum, 16);   // lane l < 16: value 8 + (l >> 1)
            if (lane < 16 && !(lane & 1) && (lane >> 1) < np)
                act_s[lane >> 1][r] = silu_mul(sum, other);
        }
    }
    __syncthreads();
    const int ablk = n_ff / 32;
    for (int jb = warp; jb < np * (GU2_ROWS / 32); jb += nw) {   // (pair, 32-row block)
        const int j = jb / (GU2_ROWS / 32), b = jb % (GU2_ROWS / 32);
        const size_t pos = (size_t)(pos0 + j);
        q8_block_warp(act_s[j][32 * b + lane], lane, aq + pos * n_ff + i0 + 32 * b,
                      ad + pos * ablk + i0 / 32 + b, as + pos * ablk + i0 / 32 + b);
    }
}

// Down rows for the pairs of one tile, unweighted: ypair[pos][h], or with
// ydirect (one pair per row, nothing to combine) ydirect[pos_pair[pos]][h].  grid
// (n_embd / 64, max tiles); block 256.  The CTA stages its 64 rows and the
// tile's Q8_1 activations in shared memory; warp w takes rows 8w .. 8w + 7.
// Each lane decodes its half block (Q6_K; 8-lane row groups) or unit (Q4_K)
// once per row and dots it with every pair's activations: the per-pair
// kernel's arithmetic and reduction, bit for bit.
__global__ void __launch_bounds__(256, 3) k_down_grouped(
    ExpertSrc src, const int8_t *__restrict__ aq, const float *__restrict__ ad,
    const float *__restrict__ as, const int32_t *__restrict__ off, const int32_t *__restrict__ cnt,
    const int32_t *__restrict__ tiles, const int32_t *__restrict__ n_tiles, int n_embd, int n_ff,
    int down_type, int dn_rows, float *__restrict__ ypair, const int32_t *__restrict__ pos_pair,
    float *__restrict__ ydirect, int *err) {
    extern __shared__ __align__(128) uint8_t smg[];
    __shared__ int s_pos[GROUP_TILE];
    __shared__ int s_row[GROUP_TILE];   // output row: the position in ypair, or the pair in ydirect
    __shared__ __align__(8) uint64_t bar;
    if ((int)blockIdx.y >= *n_tiles) return;
    const int tl = tiles[blockIdx.y], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GROUP_TILE;
    const int np = min(GROUP_TILE, cnt[e] - tt * GROUP_TILE);
    const uint8_t *dbase = expert_ptr(src, 2, e);
    if (!dbase) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    if (threadIdx.x < np) {
        s_pos[threadIdx.x] = pos0 + threadIdx.x;
        s_row[threadIdx.x] = ydirect ? pos_pair[pos0 + threadIdx.x] : pos0 + threadIdx.x;
    }
    float *const out = ydirect ? ydirect : ypair;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = n_ff / MOE_QK, ablk = n_ff / 32;
    const bool q6 = down_type == MOE_QT_Q6K;
    const size_t rb = (size_t)nb * (q6 ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
    const int h0 = blockIdx.x * dn_rows;
    const int rows = min(dn_rows, n_embd - h0);           // the last CTA may have fewer
    const uint32_t bytes = (uint32_t)(rows * rb);         // rows a multiple of 8: bytes of 16
    const int unit = q6 ? 128 : 64, stride = q6 ? PAD_U128 : PAD_U64;
    const int arow = (n_ff / unit) * stride;                                      // padded row bytes
    int8_t *aq_s = reinterpret_cast<int8_t *>(smg + (((uint32_t)(dn_rows * rb) + 15) & ~15u));   // [8][arow]
    float *ad_s = reinterpret_cast<float *>(aq_s + (size_t)GROUP_TILE * arow);   // [8][ablk]
    float *as_s = ad_s + GROUP_TILE * ablk;
    const bool dev = expert_on_device(src, e);
    if (dev && threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar, bytes);
        bulk_g2s(smg, dbase + h0 * rb, bytes, &bar);
    }
    __syncthreads();
    stage_q8_padded(aq_s, ad_s, q6 ? nullptr : as_s, aq, ad, as, s_pos, np, n_ff, unit, stride);
    if (!dev)
        for (uint32_t o = threadIdx.x * 16; o < bytes; o += blockDim.x * 16)
            *reinterpret_cast<uint4 *>(smg + o) = *reinterpret_cast<const uint4 *>(dbase + h0 * rb + o);
    const bool ok = !dev || mbar_wait(&bar, 0);
    if (__syncthreads_or(!ok)) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_TIMEOUT);
        return;
    }
    const int wrows = dn_rows / 8;              // rows per warp
    const int rw = warp * wrows;                // first local row of this warp
    if (q6) {
        // a row is gs = 2 nb half-block units on consecutive lanes, 32 / gs rows
        // per pass; groupn_sum forms group8_sum's value (8-lane groups with
        // the lanes past the units at 0), so the rows match the per-pair kernel
        const int gs = nb * 2, rpp = 32 / gs;
        const int rr = lane / gs, u = lane - rr * gs;
        const int sb = u >> 1, hh = u & 1;
        for (int p0 = 0; p0 < wrows; p0 += rpp) {
            const int rl = p0 + rr, r = rw + rl;
            const bool live = rr < rpp && rl < wrows && r < rows;
            Q6HalfDec w;
            if (live) {
                Q6Half raw;
                q6k_half_load(smg + r * rb + sb * MOE_Q6K_BYTES, hh, raw);
                q6k_half_decode(raw, w);
            }
            for (int j = 0; j < np; ++j) {
                float v = 0.0f;
                if (live) {
                    ActHalf a;
                    load_act_half_at(a, aq_s + (size_t)j * arow + u * PAD_U128, ad_s + j * ablk + 4 * u);
                    v = q6k_dec_compute(w, a);
                }
                v = groupn_sum(v, u, gs);
                if (live && u == 0) out[(size_t)s_row[j] * n_embd + h0 + r] = v;
            }
        }
    } else {
        const int units = nb * 4;
        const bool on = lane < units;
        for (int rr = 0; rr < wrows && rw + rr < rows; ++rr) {
            const int r = rw + rr;
            Q4UnitDec w;
            if (on) {
                Q4Unit raw;
                q4k_unit_load(smg + r * rb + (lane >> 2) * MOE_Q4K_BYTES, lane & 3, raw);
                q4k_unit_decode(raw, lane & 3, w);
            }
            for (int j = 0; j < np; ++j) {
                float v = 0.0f;
                if (on) {
                    ActQ4 a;
                    load_act_q4_unit(a, aq_s + (size_t)j * arow + lane * PAD_U64, ad_s + j * ablk,
                                     as_s + j * ablk, 2 * lane);
                    v = q4k_dec_compute(w, a);
                }
                v = warp_sum(v);
                if (lane == 0) out[(size_t)s_row[j] * n_embd + h0 + r] = v;
            }
        }
    }
}

// y[t][h] = sum over ranks r in order of w[t][r] * ypair[pair_pos[t*k + r]][h]
// (an fma chain from 0, then + resid): the per-pair kernel's combine.  With
// w == null (k == 1) the row is copied unweighted.  Every CTA first does
// `wait` when it has flags (the rows may come from peers).  grid
// (ceil(n_embd / 256), n_tok); block 256.
__global__ void __launch_bounds__(256) k_combine(const float *__restrict__ ypair,
                                                 const int32_t *__restrict__ pair_pos,
                                                 const float *__restrict__ w, int k, int n_embd,
                                                 const float *__restrict__ resid,
                                                 float *__restrict__ y, FlagWait wait, int *err) {
    if (wait.flags) cta_wait_flags(wait.flags, wait.world, wait.epoch, wait.wait_ns, err);
    const int t = blockIdx.y, h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= n_embd) return;
    if (!w) {   // unweighted (k == 1): the row itself, for an expert-parallel owner
        const int pos = pair_pos[t];
        y[(size_t)t * n_embd + h] = pos >= 0 ? ypair[(size_t)pos * n_embd + h] : 0.0f;
        return;
    }
    float acc = 0.0f;
    for (int r = 0; r < k; ++r) {
        const int pos = pair_pos[(size_t)t * k + r];
        const float v = pos >= 0 ? ypair[(size_t)pos * n_embd + h] : 0.0f;
        acc = __fmaf_rn(w[(size_t)t * k + r], v, acc);
    }
    if (resid) acc = __fadd_rn(acc, resid[(size_t)t * n_embd + h]);
    y[(size_t)t * n_embd + h] = acc;
}

// ids_x/w_x [n_tok][k + 1] = the k routed pairs of each token, then the
// shared expert (id n_expert) with weight 1.
__global__ void k_append_shared(const int32_t *__restrict__ ids, const float *__restrict__ w,
                                int n_tok, int k, int n_expert, int32_t *__restrict__ ids_x,
                                float *__restrict__ w_x) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_tok * (k + 1)) return;
    const int t = i / (k + 1), r = i % (k + 1);
    ids_x[i] = r < k ? ids[t * k + r] : n_expert;
    w_x[i] = r < k ? w[t * k + r] : 1.0f;
}

cudaError_t launch_append_shared(const int32_t *ids, const float *w, int n_tok, int k, int n_expert,
                                 int32_t *ids_x, float *w_x, cudaStream_t s) {
    const int n = n_tok * (k + 1);
    k_append_shared<<<(n + 255) / 256, 256, 0, s>>>(ids, w, n_tok, k, n_expert, ids_x, w_x);
    return cudaGetLastError();
}

int group_max_tiles(int n_expert, int P, int tile) { return n_expert + (P + tile - 1) / tile; }

cudaError_t launch_group(const int32_t *ids, int P, int n_expert, int tile, const GroupBufs &g,
                         int *err, cudaStream_t s, int div, const FlagWait *wait) {
    if (n_expert > GROUP_MAX_BUCKETS || tile > 0xFFFF || div < 1 || (wait && wait->world > GROUP_THREADS))
        return cudaErrorInvalidValue;
    k_group<<<1, GROUP_THREADS, 0, s>>>(ids, P, n_expert, div, tile, g.cnt, g.off, g.pair_pos,
                                        g.pos_pair, g.tiles, g.n_tiles, err, wait ? *wait : FlagWait{});
    return cudaGetLastError();
}

size_t grouped_scratch_bytes(int P, int n_embd, int n_ff) {
    // Q8_1 token rows, then Q8_1 activations: int8 values + d + s per 32
    const size_t xq = (size_t)P * n_embd + 2 * sizeof(float) * (size_t)P * (n_embd / 32);
    const size_t aq = (size_t)P * n_ff + 2 * sizeof(float) * (size_t)P * (n_ff / 32);
    return ((xq + 255) & ~(size_t)255) + aq;
}

cudaError_t launch_experts_grouped(const ExpertSrc &src, const float *x, const GroupBufs &g,
                                   int n_tok, int k, int n_embd, int n_ff, int down_type,
                                   const float *w, void *scratch, float *ypair, const float *resid,
                                   float *y, int *err, cudaStream_t s) {
    if (n_embd != 2048 || n_ff % GU2_ROWS || n_embd % DN2_ROWS) return cudaErrorInvalidValue;
    const bool q6d = down_type == MOE_QT_Q6K;
    const int dn_rows = q6d ? dn2_rows_q6(n_ff) : DN2_ROWS;   // a multiple of 8 rows per CTA
    const int P = n_tok * k;
    const int maxt = group_max_tiles(src.n_expert + 1, P, GROUP_TILE);
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    int8_t *xq = reinterpret_cast<int8_t *>(sc);
    float *xd = reinterpret_cast<float *>(sc + (size_t)n_tok * n_embd);
    float *xs = xd + (size_t)n_tok * (n_embd / 32);
    const size_t xbytes = (size_t)P * n_embd + 2 * sizeof(float) * (size_t)P * (n_embd / 32);
    int8_t *aq = reinterpret_cast<int8_t *>(sc + ((xbytes + 255) & ~(size_t)255));
    float *ad = reinterpret_cast<float *>(aq + (size_t)P * n_ff);
    float *as = ad + (size_t)P * (n_ff / 32);
    k_quant_rows<<<n_tok, 256, 0, s>>>(x, n_embd, xq, xd, xs);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const bool q6 = down_type == MOE_QT_Q6K;
    const size_t sm1 = (size_t)GROUP_TILE * (n_embd / 64) * PAD_U64 +
                       2 * sizeof(float) * GROUP_TILE * (n_embd / 32);
    const size_t sm2 = (((size_t)dn_rows * (n_ff / MOE_QK) * (q6 ? MOE_Q6K_BYTES : MOE_Q4K_BYTES) + 15) &
                        ~(size_t)15) +
                       (size_t)GROUP_TILE * (q6 ? (n_ff / 128) * PAD_U128 : (n_ff / 64) * PAD_U64) +
                       2 * sizeof(float) * GROUP_TILE * (n_ff / 32);
    if ((e = cudaFuncSetAttribute(k_gate_up_grouped, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sm1)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(k_down_grouped, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sm2)) != cudaSuccess)
        return e;
    k_gate_up_grouped<<<dim3(n_ff / GU2_ROWS, maxt), 256, sm1, s>>>(
        src, xq, xd, xs, g.off, g.cnt, g.pos_pair, g.tiles, g.n_tiles, k, n_embd, n_ff, aq, ad, as, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // one pair per row and no weights: the down rows go straight to y (a
    // combine would only copy them; rows of empty slots are left as they are)
    const bool direct = k == 1 && !w && !resid;
    k_down_grouped<<<dim3((n_embd + dn_rows - 1) / dn_rows, maxt), 256, sm2, s>>>(
        src, aq, ad, as, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, down_type, dn_rows, ypair, g.pos_pair,
        direct ? y : nullptr, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return direct ? cudaSuccess : launch_combine(ypair, g.pair_pos, w, n_tok, k, n_embd, resid, y, s);
}

cudaError_t launch_combine(const float *ypair, const int32_t *pair_pos, const float *w, int n_tok,
                           int k, int n_embd, const float *resid, float *y, cudaStream_t s,
                           const FlagWait *wait, int *err) {
    if (wait && (wait->world > 256 || !err)) return cudaErrorInvalidValue;
    k_combine<<<dim3((n_embd + 255) / 256, n_tok), 256, 0, s>>>(ypair, pair_pos, w, k, n_embd, resid, y,
                                                                wait ? *wait : FlagWait{}, err);
    return cudaGetLastError();
}

}  // namespace moe
