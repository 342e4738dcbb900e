// moe_batched.cu -- the MoE layer for n_tok > 1 with tokens grouped by expert.
//
// The per-pair kernels (k_gate_up / k_down) read an expert's rows once per
// (token, expert) pair.  With a batch, many tokens share an expert, so here
// the routed pairs are first grouped by expert (k_group), and every CTA then
// reads its expert rows once for all of that expert's pairs in its tile:
//
//   k_group           pairs -> per-expert counts, offsets, stable positions,
//                     and the tile list (expert, token tile)
//   k_gate_up_grouped gate/up GEMV (Q4_K x Q8_1) + SiLU*mul per pair
//   k_down_grouped    down GEMV per pair -> unweighted rows ypair[pos][h]
//   k_combine         y[t] = sum_r w[t][r] * ypair[pos(t, r)] in rank order
//
// Per pair, the activation and the down rows use exactly the unit mapping and
// reduction order of the per-pair kernels, and the combine adds in the same
// rank order.  The layer output is therefore bit-identical to the per-pair
// path, while the weights cross DRAM once per (expert, CTA) instead of once per
// pair.
#include "moe_kernels.h"

namespace moe {

#define GROUP_THREADS 1024
#define GROUP_MAX_BUCKETS 264   // 256 routed experts + the shared one, rounded up

// One CTA.  Pair p = t * k + r (token t, rank r).  Positions are stable: the
// pairs of an expert keep pair order.  Writes cnt[E], off[E + 1],
// pair_pos[P] (-1 for an id out of range, flagged in *err), pos_pair[P], and
// tiles[0 .. n_tiles) = (expert << 16) | token-tile for tiles of `tile` pairs.
__global__ void __launch_bounds__(GROUP_THREADS) k_group(const int32_t *__restrict__ ids, int P,
                                                         int n_expert, int tile, int32_t *cnt,
                                                         int32_t *off, int32_t *pair_pos,
                                                         int32_t *pos_pair, int32_t *tiles,
                                                         int32_t *n_tiles, int *err) {
    __shared__ int s_cnt[GROUP_MAX_BUCKETS], s_off[GROUP_MAX_BUCKETS + 1], s_base[GROUP_MAX_BUCKETS];
    __shared__ int s_wc[GROUP_THREADS / 32][GROUP_MAX_BUCKETS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < n_expert; e += GROUP_THREADS) { s_cnt[e] = 0; s_base[e] = 0; }
    __syncthreads();
    for (int p = tid; p < P; p += GROUP_THREADS) {
        const int e = ids[p];
        if (e >= 0 && e < n_expert) atomicAdd(&s_cnt[e], 1);
        else atomicOr(err, MOE_DEV_ERR_INDEX);
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0, nt = 0;
        for (int e = 0; e < n_expert; ++e) {
            s_off[e] = acc;
            acc += s_cnt[e];
            for (int t0 = 0; t0 < s_cnt[e]; t0 += tile) tiles[nt++] = (e << 16) | (t0 / tile);
        }
        s_off[n_expert] = acc;
        *n_tiles = nt;
    }
    __syncthreads();
    for (int e = tid; e <= n_expert; e += GROUP_THREADS) {
        off[e] = s_off[e];
        if (e < n_expert) cnt[e] = s_cnt[e];
    }
    const unsigned lt = (1u << lane) - 1u;
    for (int c0 = 0; c0 < P; c0 += GROUP_THREADS) {
        for (int i = tid; i < (GROUP_THREADS / 32) * n_expert; i += GROUP_THREADS)
            s_wc[i / n_expert][i % n_expert] = 0;
        __syncthreads();
        const int p = c0 + tid;
        int e = p < P ? ids[p] : -1;
        if (e >= n_expert) e = -1;
        const unsigned mask = __match_any_sync(MOE_FULL, e);
        if (e >= 0 && lane == __ffs(mask) - 1) s_wc[warp][e] = __popc(mask);
        __syncthreads();
        if (e >= 0) {
            int rank = s_base[e] + __popc(mask & lt);
            for (int w = 0; w < warp; ++w) rank += s_wc[w][e];
            const int pos = s_off[e] + rank;
            pair_pos[p] = pos;
            pos_pair[pos] = p;
        } else if (p < P) {
            pair_pos[p] = -1;
        }
        __syncthreads();
        for (int q = tid; q < n_expert; q += GROUP_THREADS) {
            int sum = 0;
            for (int w = 0; w < GROUP_THREADS / 32; ++w) sum += s_wc[w][q];
            s_base[q] += sum;
        }
        __syncthreads();
    }
}

// Gate/up for the pairs of one tile.  grid (ceil(n_ff / GU_ROWS), max tiles);
// block 256.  Each pair's token is quantised to Q8_1 in shared memory (the
// same quantiser as k_gate_up); every row is dotted with every pair's
// activations, lane per unit, then warp_sum: the per-pair kernel's order.
__global__ void __launch_bounds__(256) k_gate_up_grouped(ExpertSrc src, const float *__restrict__ x,
                                                         const int32_t *__restrict__ off,
                                                         const int32_t *__restrict__ cnt,
                                                         const int32_t *__restrict__ pos_pair,
                                                         const int32_t *__restrict__ tiles,
                                                         const int32_t *__restrict__ n_tiles,
                                                         int k, int n_embd, int n_ff,
                                                         float *__restrict__ act, int *err) {
    extern __shared__ __align__(16) uint8_t smg[];
    if ((int)blockIdx.y >= *n_tiles) return;
    const int tl = tiles[blockIdx.y], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GROUP_TILE;
    const int np = min(GROUP_TILE, cnt[e] - tt * GROUP_TILE);
    const int nblk = n_embd / 32;
    int8_t *xq = reinterpret_cast<int8_t *>(smg);                           // [np][n_embd]
    float *xd = reinterpret_cast<float *>(smg + (size_t)GROUP_TILE * n_embd); // [np][nblk]
    float *xs = xd + GROUP_TILE * nblk;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int b = warp; b < np * nblk; b += nw) {
        const int j = b / nblk, bb = b % nblk;
        const int t = pos_pair[pos0 + j] / k;
        q8_block_warp(x[(size_t)t * n_embd + 32 * bb + lane], lane, xq + (size_t)j * n_embd + 32 * bb,
                      xd + j * nblk + bb, xs + j * nblk + bb);
    }
    __syncthreads();
    const uint8_t *gbase = expert_ptr(src, 0, e);
    const uint8_t *ubase = expert_ptr(src, 1, e);
    if (!gbase || !ubase) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    const int nb = n_embd / MOE_QK;
    const size_t rb = (size_t)nb * MOE_Q4K_BYTES;
    const int units = nb * 4;
    const int i0 = blockIdx.x * GU_ROWS;
    for (int r = warp; r < GU_ROWS; r += nw) {
        const int i = i0 + r;
        if (i >= n_ff) break;
        for (int j = 0; j < np; ++j) {
            const int8_t *q = xq + (size_t)j * n_embd;
            float g = 0.0f, up = 0.0f;
            for (int uu = lane; uu < units; uu += 32) {
                ActQ4 aa;
                load_act_q4(aa, q, xd + j * nblk, xs + j * nblk, uu >> 2, uu & 3);
                g += q4k_unit_dot(gbase + i * rb + (uu >> 2) * MOE_Q4K_BYTES, uu & 3, aa);
                up += q4k_unit_dot(ubase + i * rb + (uu >> 2) * MOE_Q4K_BYTES, uu & 3, aa);
            }
            g = warp_sum(g);
            up = warp_sum(up);
            if (lane == 0) act[(size_t)(pos0 + j) * n_ff + i] = silu_mul(g, up);
        }
    }
}

// Down rows for the pairs of one tile, unweighted: ypair[pos][h].  grid
// (ceil(n_embd / DN_ROWS), max tiles); block 256; warp j takes pair j with
// the per-pair kernel's lane mapping (Q6_K: 8-lane groups over half blocks).
__global__ void __launch_bounds__(256) k_down_grouped(ExpertSrc src, const float *__restrict__ act,
                                                      const int32_t *__restrict__ off,
                                                      const int32_t *__restrict__ cnt,
                                                      const int32_t *__restrict__ tiles,
                                                      const int32_t *__restrict__ n_tiles,
                                                      int n_embd, int n_ff, int down_type,
                                                      float *__restrict__ ypair, int *err) {
    extern __shared__ __align__(16) uint8_t smg[];
    if ((int)blockIdx.y >= *n_tiles) return;
    const int tl = tiles[blockIdx.y], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GROUP_TILE;
    const int np = min(GROUP_TILE, cnt[e] - tt * GROUP_TILE);
    const int nblk = n_ff / 32;
    int8_t *aq = reinterpret_cast<int8_t *>(smg);                            // [np][n_ff]
    float *ad = reinterpret_cast<float *>(smg + (size_t)GROUP_TILE * n_ff);  // [np][nblk]
    float *as = ad + GROUP_TILE * nblk;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int b = warp; b < np * nblk; b += nw) {
        const int j = b / nblk, bb = b % nblk;
        q8_block_warp(act[(size_t)(pos0 + j) * n_ff + 32 * bb + lane], lane,
                      aq + (size_t)j * n_ff + 32 * bb, ad + j * nblk + bb, as + j * nblk + bb);
    }
    __syncthreads();
    const uint8_t *dbase = expert_ptr(src, 2, e);
    if (!dbase) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    const int h0 = blockIdx.x * DN_ROWS;
    const int nb = n_ff / MOE_QK;
    for (int j = warp; j < np; j += nw) {
        const int8_t *q = aq + (size_t)j * n_ff;
        const float *dq = ad + j * nblk;
        const float *sq = as + j * nblk;
        float *yrow = ypair + (size_t)(pos0 + j) * n_embd;
        if (down_type == MOE_QT_Q6K) {
            const size_t rb = (size_t)nb * MOE_Q6K_BYTES;
            const int grp = lane >> 3, u = lane & 7;
            const bool on = u < nb * 2;
            const int sb = u >> 1, hh = u & 1;
            ActHalf a;
            if (on) load_act_half(a, q, dq, sb, hh);
            for (int r0w = 0; r0w < DN_ROWS; r0w += 4) {
                const int r = r0w + grp, h = h0 + r;
                float v = 0.0f;
                if (on && h < n_embd) v = q6k_half_dot(dbase + h * rb + sb * MOE_Q6K_BYTES, hh, a);
                v = group8_sum(v);
                if (u == 0 && h < n_embd) yrow[h] = v;
            }
        } else {
            const size_t rb = (size_t)nb * MOE_Q4K_BYTES;
            const int units = nb * 4;
            const bool active = lane < units;
            ActQ4 a;
            if (active) load_act_q4(a, q, dq, sq, lane >> 2, lane & 3);
            for (int r = 0; r < DN_ROWS; ++r) {
                const int h = h0 + r;
                float v = 0.0f;
                if (active && h < n_embd)
                    v = q4k_unit_dot(dbase + h * rb + (lane >> 2) * MOE_Q4K_BYTES, lane & 3, a);
                v = warp_sum(v);
                if (lane == 0 && h < n_embd) yrow[h] = v;
            }
        }
    }
}

// y[t][h] = sum over ranks r in order of w[t][r] * ypair[pair_pos[t*k + r]][h]
// (an fma chain from 0, then + resid): the per-pair kernel's combine.  With
// w == null (k == 1) the row is copied unweighted.  grid (ceil(n_embd / 256),
// n_tok); block 256.
__global__ void __launch_bounds__(256) k_combine(const float *__restrict__ ypair,
                                                 const int32_t *__restrict__ pair_pos,
                                                 const float *__restrict__ w, int k, int n_embd,
                                                 const float *__restrict__ resid,
                                                 float *__restrict__ y) {
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
                         int *err, cudaStream_t s) {
    if (n_expert > GROUP_MAX_BUCKETS || tile > 0xFFFF) return cudaErrorInvalidValue;
    k_group<<<1, GROUP_THREADS, 0, s>>>(ids, P, n_expert, tile, g.cnt, g.off, g.pair_pos,
                                        g.pos_pair, g.tiles, g.n_tiles, err);
    return cudaGetLastError();
}

cudaError_t launch_experts_grouped(const ExpertSrc &src, const float *x, const GroupBufs &g,
                                   int n_tok, int k, int n_embd, int n_ff, int down_type,
                                   const float *w, float *act, float *ypair, const float *resid,
                                   float *y, int *err, cudaStream_t s) {
    const int P = n_tok * k;
    const int maxt = group_max_tiles(src.n_expert + 1, P, GROUP_TILE);
    const size_t sm1 = (size_t)GROUP_TILE * n_embd + 2 * sizeof(float) * GROUP_TILE * (n_embd / 32);
    cudaError_t e;
    if (sm1 > 48 * 1024) {
        e = cudaFuncSetAttribute(k_gate_up_grouped, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
        if (e != cudaSuccess) return e;
    }
    k_gate_up_grouped<<<dim3((n_ff + GU_ROWS - 1) / GU_ROWS, maxt), 256, sm1, s>>>(
        src, x, g.off, g.cnt, g.pos_pair, g.tiles, g.n_tiles, k, n_embd, n_ff, act, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t sm2 = (size_t)GROUP_TILE * n_ff + 2 * sizeof(float) * GROUP_TILE * (n_ff / 32);
    if (sm2 > 48 * 1024) {
        e = cudaFuncSetAttribute(k_down_grouped, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
        if (e != cudaSuccess) return e;
    }
    k_down_grouped<<<dim3((n_embd + DN_ROWS - 1) / DN_ROWS, maxt), 256, sm2, s>>>(
        src, act, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, down_type, ypair, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return launch_combine(ypair, g.pair_pos, w, n_tok, k, n_embd, resid, y, s);
}

cudaError_t launch_combine(const float *ypair, const int32_t *pair_pos, const float *w, int n_tok,
                           int k, int n_embd, const float *resid, float *y, cudaStream_t s) {
    k_combine<<<dim3((n_embd + 255) / 256, n_tok), 256, 0, s>>>(ypair, pair_pos, w, k, n_embd,
                                                                resid, y);
    return cudaGetLastError();
}

}  // namespace moe
