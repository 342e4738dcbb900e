// moe_kernels.cu -- stand-alone kernels of libmoeb200.so:
//   weight quantisation (Q4_K / Q6_K, bit-identical to the oracle) and the
//   synthetic-weight generator; the fused router; the gate/up GEMV with fused
//   SiLU*mul; the down GEMV with the fused weighted top-k combine; the device
//   slot table (observation and the cache step).
// The persistent multi-layer decode kernel lives in moe_decode.cu.
#include "moe_kernels.h"

#include <cooperative_groups.h>

#include <algorithm>

namespace moe {

// ===========================================================================
// quantisation (our own quantiser; same fp32 operation sequence as
// or_quantize_q4_K / or_quantize_q6_K in the oracle)
// ===========================================================================

__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

__device__ void quantize_q4k_block(const float *xb, uint8_t *yb) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = xb[32 * j], mx = xb[32 * j];
        for (int l = 1; l < 32; ++l) {
            const float v = xb[32 * j + l];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        if (mn > 0.0f) mn = 0.0f;
        scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        minv[j] = -mn;
        if (scale[j] > max_scale) max_scale = scale[j];
        if (minv[j] > max_min) max_min = minv[j];
    }
    const __half dh = __float2half_rn(__fdiv_rn(max_scale, 63.0f));
    const __half mh = __float2half_rn(__fdiv_rn(max_min, 63.0f));
    const float dd = __half2float(dh), dm = __half2float(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = dd > 0.0f ? clampi((int)roundf(__fdiv_rn(scale[j], dd)), 0, 63) : 0;
        m[j] = dm > 0.0f ? clampi((int)roundf(__fdiv_rn(minv[j], dm)), 0, 63) : 0;
    }
    const unsigned short dbits = __half_as_ushort(dh), mbits = __half_as_ushort(mh);
    yb[0] = (uint8_t)(dbits & 0xFF);
    yb[1] = (uint8_t)(dbits >> 8);
    yb[2] = (uint8_t)(mbits & 0xFF);
    yb[3] = (uint8_t)(mbits >> 8);
    for (int j = 0; j < 4; ++j) {
        yb[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        yb[8 + j] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        yb[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    for (int p = 0; p < 4; ++p) {
        const float es0 = __fmul_rn(dd, (float)sc[2 * p]), em0 = __fmul_rn(dm, (float)m[2 * p]);
        const float es1 = __fmul_rn(dd, (float)sc[2 * p + 1]), em1 = __fmul_rn(dm, (float)m[2 * p + 1]);
        for (int l = 0; l < 32; ++l) {
            const int q0 = es0 > 0.0f
                ? clampi((int)roundf(__fdiv_rn(__fadd_rn(xb[64 * p + l], em0), es0)), 0, 15) : 0;
            const int q1 = es1 > 0.0f
                ? clampi((int)roundf(__fdiv_rn(__fadd_rn(xb[64 * p + 32 + l], em1), es1)), 0, 15) : 0;
            yb[16 + 32 * p + l] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

__device__ void quantize_q6k_block(const float *xb, uint8_t *yb) {
    float gscale[16];
    float max_scale = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float amax = 0.0f;
        for (int l = 0; l < 16; ++l) {
            const float a = fabsf(xb[16 * g + l]);
            if (a > amax) amax = a;
        }
        gscale[g] = __fdiv_rn(amax, 31.0f);
        if (gscale[g] > max_scale) max_scale = gscale[g];
    }
    const __half dh = __float2half_rn(__fdiv_rn(max_scale, 127.0f));
    const float dd = __half2float(dh);
    int sc[16];
    for (int g = 0; g < 16; ++g) {
        sc[g] = dd > 0.0f ? clampi((int)roundf(__fdiv_rn(gscale[g], dd)), -128, 127) : 0;
        yb[192 + g] = (uint8_t)(int8_t)sc[g];
    }
    for (int h = 0; h < 2; ++h) {
        for (int l = 0; l < 32; ++l) {
            int q[4];
            for (int mm = 0; mm < 4; ++mm) {
                const int e = 128 * h + 32 * mm + l;
                const float es = __fmul_rn(dd, (float)sc[e >> 4]);
                const int v = es != 0.0f ? clampi((int)roundf(__fdiv_rn(xb[e], es)), -32, 31) : 0;
                q[mm] = v + 32;
            }
            yb[64 * h + l] = (uint8_t)((q[0] & 0xF) | ((q[2] & 0xF) << 4));
            yb[64 * h + l + 32] = (uint8_t)((q[1] & 0xF) | ((q[3] & 0xF) << 4));
            yb[128 + 32 * h + l] = (uint8_t)((q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) |
                                             ((q[3] >> 4) << 6));
        }
    }
    const unsigned short dbits = __half_as_ushort(dh);
    yb[208] = (uint8_t)(dbits & 0xFF);
    yb[209] = (uint8_t)(dbits >> 8);
}

__global__ void k_quantize(const float *__restrict__ x, uint8_t *__restrict__ y, int64_t nb,
                           int qtype) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    if (qtype == MOE_QT_Q4K) quantize_q4k_block(x + b * MOE_QK, y + b * MOE_Q4K_BYTES);
    else quantize_q6k_block(x + b * MOE_QK, y + b * MOE_Q6K_BYTES);
}

// splitmix64 finaliser (S. Vigna's public-domain generator) as a counter hash
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Synthetic N(0, sigma^2) weights straight into quantised blocks: element i of
// block b takes the Box-Muller normal of hash(seed, b*256 + i).  No fp32 copy
// of the weights ever exists in HBM.
__global__ void k_synth_weights(uint8_t *__restrict__ y, int64_t nb, int qtype, uint64_t seed,
                                float sigma) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    float xb[MOE_QK];
    const uint64_t base = mix64(seed) ^ (uint64_t)b * 0x100000001B3ull;
    for (int i = 0; i < MOE_QK; i += 2) {
        const uint64_t h = mix64(base + (uint64_t)i);
        const float u1 = ((float)(h >> 40) + 1.0f) * 0x1.0p-24f;
        const float u2 = (float)(h & 0xFFFFFFull) * 0x1.0p-24f;
        const float r = sqrtf(-2.0f * logf(u1)) * sigma;
        float sn, cs;
        sincospif(2.0f * u2, &sn, &cs);
        xb[i] = r * cs;
        xb[i + 1] = r * sn;
    }
    if (qtype == MOE_QT_Q4K) quantize_q4k_block(xb, y + b * MOE_Q4K_BYTES);
    else quantize_q6k_block(xb, y + b * MOE_Q6K_BYTES);
}

// Synthetic fp32 N(0, sigma^2) (router weights, inputs), same hash.
__global__ void k_synth_f32(float *__restrict__ y, int64_t n, uint64_t seed, float sigma) {
    const int64_t i2 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (i2 >= n) return;
    const uint64_t h = mix64(mix64(seed) + (uint64_t)i2);
    const float u1 = ((float)(h >> 40) + 1.0f) * 0x1.0p-24f;
    const float u2 = (float)(h & 0xFFFFFFull) * 0x1.0p-24f;
    const float r = sqrtf(-2.0f * logf(u1)) * sigma;
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    y[i2] = r * cs;
    if (i2 + 1 < n) y[i2 + 1] = r * sn;
}

// ===========================================================================
// fused router: one CTA per token, one warp per logit, warp 0 selects
// ===========================================================================

__global__ void __launch_bounds__(512) k_router(const float *__restrict__ W,
                                                const float *__restrict__ x, int n_expert,
                                                int n_embd, const int32_t *__restrict__ table,
                                                int ns, float delta, int use_prior, int k,
                                                int32_t *__restrict__ ids, float *__restrict__ w,
                                                float *__restrict__ logits_out,
                                                SlotState st, int observe_layer_idx,
                                                const int32_t *__restrict__ pub) {
    extern __shared__ __align__(16) float sm[];
    float *xs = sm;                   // [n_embd]
    float *lg = sm + n_embd;          // [n_expert]
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < n_embd; i += blockDim.x) xs[i] = x[(size_t)t * n_embd + i];
    __syncthreads();
    for (int e = warp; e < n_expert; e += nw) {
        const float v = router_dot_warp(W + (size_t)e * n_embd, xs, n_embd, lane);
        if (lane == 0) {
            lg[e] = v;
            if (logits_out) logits_out[(size_t)t * n_expert + e] = v;
        }
    }
    __syncthreads();
    if (warp == 0) {
        __shared__ int32_t sids[MOE_KMAX];
        __shared__ float sw[MOE_KMAX];
        router_select_warp(lg, n_expert, table, ns, delta, use_prior != 0, k, sids, sw, lane, pub);
        __syncwarp();
        if (lane < k) {
            ids[(size_t)t * k + lane] = sids[lane];
            w[(size_t)t * k + lane] = sw[lane];
        }
        if (observe_layer_idx >= 0 && lane == 0) observe_layer(st, observe_layer_idx, sids, k);
    }
}

// Router for any number of tokens, one cluster of RB_CL CTAs per TOK tokens
// (the cache prior and the observation apply to single tokens only, and the
// caller passes them only then).  CTA r of a cluster
// computes the logits of experts [r E / RB_CL, (r + 1) E / RB_CL) for the
// cluster's tokens: warp w takes two of them at a time, holds its lanes'
// slice of both router rows in registers (n_embd == 2048: 16 float4 per lane
// each) and runs the four fma chains of router_dot_warp for every token, so
// every logit is computed in router_dot_warp's order, bit-identical to
// k_router.  After a cluster barrier, CTA r gathers token r's E logits from
// the cluster's shared memory and selects for it (router_select_warp).  Each
// CTA reads only its 1/RB_CL of the router, instead of all of it.
// Two shapes: TOK = 8 tokens per cluster with 8 warps per CTA for large
// batches (the router rows are reused over more tokens), and TOK = 4 with
// 16 warps, one router row each, for small ones (twice the clusters, and a
// warp's serial chain of row load and dots is a quarter as long).
#define RB_TOK 8
#define RB_TOK_SMALL 4
#define RB_SMALL_MAX 64   // batches up to this many tokens take TOK = 4
#define RB_CL 8

__device__ __forceinline__ float router_chain_dot(const float4 (&wv)[16], const float *xt, int lane) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
        const float4 xv = *reinterpret_cast<const float4 *>(xt + 128 * kk + 4 * lane);
        a0 = __fmaf_rn(wv[kk].x, xv.x, a0);
        a1 = __fmaf_rn(wv[kk].y, xv.y, a1);
        a2 = __fmaf_rn(wv[kk].z, xv.z, a2);
        a3 = __fmaf_rn(wv[kk].w, xv.w, a3);
    }
    float v = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(MOE_FULL, v, off));
    return v;
}

// grid RB_CL x ceil(n_tok / TOK) (cluster dims RB_CL); block NT;
// dynamic shared memory: the cluster's token rows [TOK][2048].
template <int TOK, int NT>
__global__ void __cluster_dims__(RB_CL, 1, 1) __launch_bounds__(NT)
    k_router_batch(const float *__restrict__ W, const float *__restrict__ x, int n_tok,
                   int n_expert, int k, int32_t *__restrict__ ids, float *__restrict__ w,
                   const int32_t *__restrict__ table, int ns, float delta, int use_prior,
                   SlotState st, int observe_layer_idx, const int32_t *__restrict__ pub) {
    namespace cg = cooperative_groups;
    static_assert(TOK % 2 == 0 && (TOK * 512) % NT == 0, "k_router_batch shape");
    extern __shared__ __align__(16) float xs[];          // [TOK][2048]
    __shared__ float lg[TOK][256 / RB_CL];               // this CTA's experts' logits
    __shared__ float lgf[256];                           // one token's logits, all experts
    __shared__ int32_t sids[MOE_KMAX];
    __shared__ float sw[MOE_KMAX];
    cg::cluster_group cl = cg::this_cluster();
    const int r = (int)cl.block_rank();
    const int t0 = (blockIdx.x / RB_CL) * TOK;
    const int nt = min(TOK, n_tok - t0);
    const int epc = n_expert / RB_CL, e0 = r * epc;     // this CTA's experts
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    {   // the token rows: every load issued before the first store
        constexpr int PER = TOK * 512 / NT;
        const float4 *xg = reinterpret_cast<const float4 *>(x + (size_t)t0 * 2048);
        float4 v[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = threadIdx.x + NT * j;
            v[j] = i < nt * 512 ? __ldg(xg + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) reinterpret_cast<float4 *>(xs)[threadIdx.x + NT * j] = v[j];
    }
    __syncthreads();
    for (int j = warp; j < epc; j += nw) {
        // one router row per pass, two tokens per step (eight fma chains)
        const float *Wr = W + (size_t)(e0 + j) * 2048;
        float4 wr[16];
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) wr[kk] = __ldg(reinterpret_cast<const float4 *>(Wr + 128 * kk + 4 * lane));
        for (int t = 0; t < nt; t += 2) {
            const int t2 = t + 1 < nt ? t + 1 : t;
            const float va = router_chain_dot(wr, xs + t * 2048, lane);
            const float vb = router_chain_dot(wr, xs + t2 * 2048, lane);
            if (lane == 0) {
                lg[t][j] = va;
                if (t + 1 < nt) lg[t + 1][j] = vb;
            }
        }
    }
    cl.sync();   // every CTA's logits are in its shared memory
    if (r < nt && warp == 0) {
        for (int e = lane; e < n_expert; e += 32) {
            const float *src = cl.map_shared_rank(&lg[r][0], e / epc);
            lgf[e] = src[e % epc];
        }
        __syncwarp();
        // select_warp with inv = 1: router_select_warp's result (prior
        // included), in registers (no indexed local arrays)
        int id_r = -1;
        float w_r = 0.0f;
        const bool pri = use_prior != 0;
        switch (n_expert) {
            case 32: select_warp<1>(lgf, 1.0f, table, ns, delta, pri, k, lane, id_r, w_r, sids, sw, pub); break;
            case 64: select_warp<2>(lgf, 1.0f, table, ns, delta, pri, k, lane, id_r, w_r, sids, sw, pub); break;
            case 128: select_warp<4>(lgf, 1.0f, table, ns, delta, pri, k, lane, id_r, w_r, sids, sw, pub); break;
            default: select_warp<8>(lgf, 1.0f, table, ns, delta, pri, k, lane, id_r, w_r, sids, sw, pub); break;
        }
        if (lane < k) {
            ids[(size_t)(t0 + r) * k + lane] = id_r;
            w[(size_t)(t0 + r) * k + lane] = w_r;
        }
        // a single token's layer is observed by one thread (moe_obs_cb)
        if (observe_layer_idx >= 0 && lane == 0) observe_layer(st, observe_layer_idx, sids, k);
    }
    cl.sync();   // no CTA leaves while another still reads its logits
}

// ===========================================================================
// gate/up GEMV with fused SiLU*mul (stand-alone; direct global loads)
// grid: (ceil(n_ff / GU_ROWS), n_tok * k); block 256 (8 warps)
// ===========================================================================

__global__ void __launch_bounds__(256) k_gate_up(ExpertSrc src, const float *__restrict__ x,
                                                 const int32_t *__restrict__ ids, int k,
                                                 int n_embd, int n_ff,
                                                 float *__restrict__ act, int *err) {
    __shared__ __align__(16) int8_t xq[4096];
    __shared__ float xd[128], xsum[128];
    const int tk = blockIdx.y, t = tk / k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *xt = x + (size_t)t * n_embd;
    for (int b = warp; b < n_embd / 32; b += nw)
        q8_block_warp(xt[32 * b + lane], lane, xq + 32 * b, xd + b, xsum + b);
    __syncthreads();
    const int id = ids[tk];
    const uint8_t *gbase = expert_ptr(src, 0, id);
    const uint8_t *ubase = expert_ptr(src, 1, id);
    if (!gbase || !ubase) {
        if (threadIdx.x == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    const int nb = n_embd / MOE_QK;           // super-blocks per row
    const size_t rb = (size_t)nb * MOE_Q4K_BYTES;
    const int units = nb * 4;   // n_embd == 2048 gives exactly one unit per lane
    const int u = lane;
    const bool active = u < units;
    ActQ4 a;
    if (active) load_act_q4(a, xq, xd, xsum, u >> 2, u & 3);
    const int i0 = blockIdx.x * GU_ROWS;
    for (int r = warp; r < GU_ROWS; r += nw) {
        const int i = i0 + r;
        if (i >= n_ff) break;
        float g = 0.0f, up = 0.0f;
        for (int uu = u; uu < units; uu += 32) {
            ActQ4 aa = a;
            if (uu != u) load_act_q4(aa, xq, xd, xsum, uu >> 2, uu & 3);
            g += q4k_unit_dot(gbase + i * rb + (uu >> 2) * MOE_Q4K_BYTES, uu & 3, aa);
            up += q4k_unit_dot(ubase + i * rb + (uu >> 2) * MOE_Q4K_BYTES, uu & 3, aa);
        }
        g = warp_sum(g);
        up = warp_sum(up);
        if (lane == 0) act[(size_t)tk * n_ff + i] = silu_mul(g, up);
    }
}

// ===========================================================================
// down GEMV with fused weighted combine (stand-alone; direct global loads)
// grid: (ceil(n_embd / DN_ROWS), n_tok); block 256
// ===========================================================================

__global__ void __launch_bounds__(256) k_down(ExpertSrc src, const float *__restrict__ act,
                                              const int32_t *__restrict__ ids,
                                              const float *__restrict__ wts, int k, int n_embd,
                                              int n_ff, int down_type,
                                              const float *__restrict__ resid,
                                              float *__restrict__ y, int *err) {
    extern __shared__ __align__(16) uint8_t smd[];
    int8_t *aq = reinterpret_cast<int8_t *>(smd);                       // [k][n_ff]
    float *ad = reinterpret_cast<float *>(smd + (size_t)k * n_ff);      // [k][n_ff/32]
    float *as = ad + (size_t)k * (n_ff / 32);                           // [k][n_ff/32]
    float *ys = as + (size_t)k * (n_ff / 32);                           // [k][DN_ROWS]
    const int t = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float *at = act + (size_t)t * k * n_ff;
    for (int b = warp; b < k * (n_ff / 32); b += nw)
        q8_block_warp(at[32 * b + lane], lane, aq + 32 * b, ad + b, as + b);
    __syncthreads();
    const int h0 = blockIdx.x * DN_ROWS;
    const int nb = n_ff / MOE_QK;
    for (int kk = warp; kk < k; kk += nw) {
        const int id = ids[(size_t)t * k + kk];
        const uint8_t *dbase = expert_ptr(src, 2, id);
        if (!dbase) {
            if (lane == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
            for (int r = 0; r < DN_ROWS; ++r) if (lane == 0) ys[kk * DN_ROWS + r] = 0.0f;
            continue;
        }
        const int8_t *q = aq + (size_t)kk * n_ff;
        const float *dq = ad + (size_t)kk * (n_ff / 32);
        const float *sq = as + (size_t)kk * (n_ff / 32);
        if (down_type == MOE_QT_Q6K) {
            // one lane per half super-block, 8-lane row groups: the same unit
            // mapping and reduction order as the persistent decode kernel
            const size_t rb = (size_t)nb * MOE_Q6K_BYTES;
            const int grp = lane >> 3, u = lane & 7;
            const bool on = u < nb * 2;
            const int sb = u >> 1, hh = u & 1;
            ActHalf a;
            if (on) load_act_half(a, q, dq, sb, hh);
            for (int r0w = 0; r0w < DN_ROWS; r0w += 4) {
                const int r = r0w + grp, h = h0 + r;
                float v = 0.0f;
                if (on && h < n_embd && dbase)
                    v = q6k_half_dot(dbase + h * rb + sb * MOE_Q6K_BYTES, hh, a);
                v = group8_sum(v);
                if (u == 0) ys[kk * DN_ROWS + r] = v;
            }
        } else {
            const size_t rb = (size_t)nb * MOE_Q4K_BYTES;
            const int units = nb * 4;
            const int u = lane;
            ActQ4 a;
            const bool active = u < units;
            if (active) load_act_q4(a, q, dq, sq, u >> 2, u & 3);
            for (int r = 0; r < DN_ROWS; ++r) {
                const int h = h0 + r;
                float v = 0.0f;
                if (active && h < n_embd && dbase)
                    v = q4k_unit_dot(dbase + h * rb + (u >> 2) * MOE_Q4K_BYTES, u & 3, a);
                v = warp_sum(v);
                if (lane == 0) ys[kk * DN_ROWS + r] = v;
            }
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < DN_ROWS; r += blockDim.x) {
        const int h = h0 + r;
        if (h >= n_embd) continue;
        float acc = 0.0f;
        for (int kk = 0; kk < k; ++kk) acc = __fmaf_rn(wts[(size_t)t * k + kk], ys[kk * DN_ROWS + r], acc);
        if (resid) acc = __fadd_rn(acc, resid[(size_t)t * n_embd + h]);
        y[(size_t)t * n_embd + h] = acc;
    }
}

// ===========================================================================
// slot table: observation of externally computed ids, and the cache step
// ===========================================================================

__global__ void k_transpose(const float *__restrict__ in, float *__restrict__ out, int rows,
                            int cols) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = by + j, cc = bx + threadIdx.x;
        if (r < rows && cc < cols) tile[j][threadIdx.x] = in[(size_t)r * cols + cc];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = bx + j, cc = by + threadIdx.x;   // out is [cols][rows]
        if (r < cols && cc < rows) out[(size_t)r * rows + cc] = tile[threadIdx.x][j];
    }
}

__global__ void k_observe(SlotState st, int layer, const int32_t *__restrict__ ids, int n) {
    if (threadIdx.x == 0 && blockIdx.x == 0) observe_layer(st, layer, ids, n);
}

// The predictor's half of moe_obs_cb (patches/0006:367-397, 0007:294-321):
// speculative uploads of the predicted ids `top` for layer l (the layer after
// the observed one), with the heat gate when admission is by heat, at most
// predict_top of them, keeping max_inserts slots of the pool for demand.
// One thread.
__global__ void k_issue_spec(SlotState st, int l, const int32_t *__restrict__ top, int n_top) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const int E = st.n_expert, ns = st.ns[l];
    if (st.admit_mode == 1) {
        const int pool_target = pool_target_of(st);
        const int nv = st.n_free[l] > pool_target ? -1 : lru_resident_dev(st, l);
        const int32_t *tbl = st.table + (size_t)l * E;
        int32_t *adm = st.admitted + (size_t)l * E;
        int n = 0;
        for (int i = 0; i < n_top && n < E; ++i) {
            const int id = top[i];
            if (id >= 0 && id < E && tbl[id] == ns && admit_ok_dev(st, l, id, nv)) adm[n++] = id;
        }
        issue_uploads_dev(st, l, adm, n, st.predict_top, st.max_inserts, 1);
    } else {
        issue_uploads_dev(st, l, top, n_top, st.predict_top, st.max_inserts, 1);
    }
}

// evict_scores (patches/0006:402-426) for every layer with a model, one CTA
// per layer, thread j = expert j: moe_predictor::score
// (cpp/moe-predictor.cpp:165-223) with its inputs prev = the next layer's
// previous-token ids, cur = this layer's ids, below = the previous layer's
// ids, self_prev = this layer's previous-token ids.  Row adds per expert in
// block and id order; the mean and variance as sequential fp32 sums on one
// thread; no fused multiply-adds.  blockDim >= n_expert.
__global__ void __launch_bounds__(256) k_evict_scores(SlotState st) {
    __shared__ float s_out[256];
    __shared__ float s_mu, s_sd;
    const int l = blockIdx.x, j = threadIdx.x, E = st.n_expert, L = st.n_layers;
    const int m = st.ev_index[l];
    if (m < 0) return;
    const float *W = st.ev_w + (size_t)m * st.ev_feat * E;
    const int32_t *ids[4] = {l + 1 < L ? st.prev_ids + (size_t)(l + 1) * CUR_IDS : nullptr,
                             st.cur_ids + (size_t)l * CUR_IDS,
                             l > 0 ? st.cur_ids + (size_t)(l - 1) * CUR_IDS : nullptr,
                             st.prev_ids + (size_t)l * CUR_IDS};
    const int n[4] = {l + 1 < L ? st.n_prev[l + 1] : 0, st.n_cur[l], l > 0 ? st.n_cur[l - 1] : 0,
                      st.n_prev[l]};
    if (j < E) {
        float o = st.ev_bias[(size_t)m * E + j];
        for (int g = 0; g < 4; ++g) {
            const int off = st.ev_off[g];
            if (off < 0 || !ids[g]) continue;
            for (int i = 0; i < n[g]; ++i) {
                const int e = ids[g][i];
                if (e >= 0 && e < E) o = __fadd_rn(o, W[(size_t)(off + e) * E + j]);
            }
        }
        s_out[j] = o;
    }
    __syncthreads();
    if (j == 0) {
        float mu = 0.0f;
        for (int q = 0; q < E; ++q) mu = __fadd_rn(mu, s_out[q]);
        mu = __fdiv_rn(mu, (float)E);
        float var = 0.0f;
        for (int q = 0; q < E; ++q) {
            const float d = __fsub_rn(s_out[q], mu);
            var = __fadd_rn(var, __fmul_rn(d, d));
        }
        s_mu = mu;
        s_sd = __fadd_rn(__fsqrt_rn(__fdiv_rn(var, (float)E)), 1e-9f);
    }
    __syncthreads();
    if (j < E) s_out[j] = __fdiv_rn(__fsub_rn(s_out[j], s_mu), s_sd);
    __syncthreads();
    if (j == 0) {
        const float pw = st.ev_prior[m];
        if (pw != 0.0f && ids[0])
            for (int i = 0; i < n[0]; ++i) {
                const int e = ids[0][i];
                if (e >= 0 && e < E) s_out[e] = __fadd_rn(s_out[e], pw);
            }
    }
    __syncthreads();
    if (j < E) st.ev_scores[(size_t)l * E + j] = s_out[j];
}

// The victim choice of llama_moe_cache_step with a model: the lowest score,
// recency breaking ties (patches/0006:806-818, :871-889).
__device__ __forceinline__ bool evict_better(float sc, uint64_t lu, float best_score, uint64_t best) {
    return sc < best_score || (sc == best_score && lu < best);
}

// llama_moe_cache_step on the device (patches/0006:765-953, 0007:655-773
// admission / probation / heat decay, 0008:613-627 deterministic
// publication).  One CTA: thread 0 publishes (the clock order is global),
// then one thread per layer schedules (without early issue) or tops the free
// pool back up (with it; the jobs were issued when the layers were
// observed).  Scheduled jobs are also written to `host_jobs` (mapped pinned
// memory) as (layer, expert, slot, spec) for the uploader.
__global__ void __launch_bounds__(256) k_step(SlotState st, int32_t *host_jobs,
                                              int32_t *host_njobs) {
    __shared__ int s_dirty;
    const int L = st.n_layers, E = st.n_expert, MI = st.job_cap;
    if (threadIdx.x == 0) {
        s_dirty = 0;
        uint64_t clock = st.g[G_CLOCK];
        const uint64_t n_steps = st.g[G_STEPS];
        uint64_t published = 0;
        for (int l = 0; l < L; ++l) {
            const int nj = st.n_jobs[l];
            int32_t *jb = st.jobs + (size_t)l * MI * 4;
            // deterministic publication: (layer, slot) order
            for (int a = 1; a < nj; ++a) {
                int32_t tmp[4] = {jb[4 * a], jb[4 * a + 1], jb[4 * a + 2], jb[4 * a + 3]};
                int b = a - 1;
                while (b >= 0 && jb[4 * b + 1] > tmp[1]) {
                    for (int c = 0; c < 4; ++c) jb[4 * (b + 1) + c] = jb[4 * b + c];
                    --b;
                }
                for (int c = 0; c < 4; ++c) jb[4 * (b + 1) + c] = tmp[c];
            }
            const int so = st.slot_off[l];
            for (int a = 0; a < nj; ++a) {
                const int e = jb[4 * a], slot = jb[4 * a + 1], spec = jb[4 * a + 2];
                st.slot_expert[so + slot] = e;
                st.table[(size_t)l * E + e] = slot;
                if (spec && st.spec_probation) {
                    st.last_use[so + slot] = 1;
                    st.protect[so + slot] = n_steps + 1;
                } else {
                    st.last_use[so + slot] = ++clock;
                }
                st.in_flight[so + slot] = 0;
                s_dirty = 1;
                published++;
            }
            st.n_jobs[l] = 0;
        }
        st.g[G_CLOCK] = clock;
        st.g[G_COPIED] += published;
        st.g[G_PUBLISHED] += published;
        st.g[G_STEPS] = n_steps + 1;
        *host_njobs = 0;
    }
    __syncthreads();
    const uint64_t n_steps = st.g[G_STEPS];
    if (st.early_issue) {
        // top the free pool back up to its target: evict the least recently
        // used resident, unprotected slots not in flight (patches/0006:843-913)
        const int pool_target = pool_target_of(st);
        for (int l = threadIdx.x; l < L; l += blockDim.x) {
            st.n_pending[l] = 0;
            const int ns = st.ns[l], so = st.slot_off[l];
            int32_t *tbl = st.table + (size_t)l * E;
            int nf = st.n_free[l];
            bool dirty = false;
            const float *esc = st.have_evict && st.ev_index[l] >= 0 ? st.ev_scores + (size_t)l * E : nullptr;
            while (nf < pool_target) {
                int slot = -1;
                uint64_t best = ~0ull;
                float best_score = 3.4e38f;
                for (int q = 0; q < ns; ++q) {
                    if (st.in_flight[so + q] || st.slot_expert[so + q] < 0) continue;
                    if (st.protect[so + q] >= n_steps) continue;
                    if (esc) {
                        const float sc = esc[st.slot_expert[so + q]];
                        if (evict_better(sc, st.last_use[so + q], best_score, best)) {
                            best_score = sc; best = st.last_use[so + q]; slot = q;
                        }
                    } else if (st.last_use[so + q] < best) {
                        best = st.last_use[so + q]; slot = q;
                    }
                }
                if (slot < 0) break;
                tbl[st.slot_expert[so + slot]] = ns;
                st.slot_expert[so + slot] = -1;
                st.free_slots[so + nf++] = slot;
                dirty = true;
            }
            st.n_free[l] = nf;
            if (dirty) s_dirty = 1;
        }
    }
    for (int l = threadIdx.x; l < L && !st.early_issue; l += blockDim.x) {
        const int np = st.n_pending[l];
        if (np == 0) continue;
        const int ns = st.ns[l], so = st.slot_off[l];
        int32_t *tbl = st.table + (size_t)l * E;
        const int32_t *pend = st.pending + (size_t)l * E;
        int budget = st.max_inserts;
        int nj = 0;
        uint64_t ok_n = 0, den_n = 0;
        bool dirty = false;
        const float *esc = st.have_evict && st.ev_index[l] >= 0 ? st.ev_scores + (size_t)l * E : nullptr;
        for (int it = np - 1; it >= 0 && budget > 0; --it) {
            const int id = pend[it];
            if (tbl[id] != ns) {
                --budget;
                continue;
            }
            int slot = -1;
            uint64_t best = ~0ull;
            float best_score = 3.4e38f;
            for (int s = 0; s < ns; ++s) {
                if (st.in_flight[so + s]) continue;
                if (st.slot_expert[so + s] < 0) { slot = s; break; }
                if (st.protect[so + s] >= n_steps) continue;
                if (esc) {
                    const float sc = esc[st.slot_expert[so + s]];
                    if (evict_better(sc, st.last_use[so + s], best_score, best)) {
                        best_score = sc; best = st.last_use[so + s]; slot = s;
                    }
                } else if (st.last_use[so + s] < best) {
                    best = st.last_use[so + s]; slot = s;
                }
            }
            if (slot < 0) break;
            const int victim = st.slot_expert[so + slot];
            // admit_ok (patches/0007:414-429)
            bool ok = true;
            if (st.admit_mode != 0 && victim >= 0) {
                if (st.admit_mode == 1) {
                    const float *ht = st.heat + (size_t)l * E;
                    ok = ht[id] > __fadd_rn(__fmul_rn(ht[victim], 1.25f), st.admit_floor);
                } else if (st.admit_mode == 2) {
                    const uint64_t mp = st.miss_prev[(size_t)l * E + id];
                    const uint64_t ml = st.miss_last[(size_t)l * E + id];
                    ok = mp != ~0ull && ml - mp < (uint64_t)st.admit_window;
                }
                if (ok) ok_n++; else den_n++;
            }
            if (!ok) continue;
            --budget;
            if (victim >= 0) {
                tbl[victim] = ns;
                st.slot_expert[so + slot] = -1;
                dirty = true;
            }
            st.in_flight[so + slot] = 1;
            int32_t *jb = st.jobs + ((size_t)l * MI + nj) * 4;
            jb[0] = id; jb[1] = slot; jb[2] = 0; jb[3] = 0;
            nj++;
        }
        st.n_jobs[l] = nj;
        st.n_pending[l] = 0;
        if (nj) atomicAdd((unsigned long long *)&st.g[G_SCHEDULED], (unsigned long long)nj);
        if (ok_n) atomicAdd((unsigned long long *)&st.g[G_ADMIT_OK], (unsigned long long)ok_n);
        if (den_n) atomicAdd((unsigned long long *)&st.g[G_ADMIT_DENIED], (unsigned long long)den_n);
        if (dirty) s_dirty = 1;
    }
    __syncthreads();
    // the token is over: its ids become the previous token's, after every
    // eviction decision of the step (patches/0006:914-922)
    if (st.have_evict)
        for (int l = threadIdx.x; l < L; l += blockDim.x) {
            const int nc = st.n_cur[l];
            for (int i = 0; i < nc; ++i) st.prev_ids[(size_t)l * CUR_IDS + i] = st.cur_ids[(size_t)l * CUR_IDS + i];
            st.n_prev[l] = nc;
        }
    if (st.admit_mode == 1 && st.admit_half > 0 && n_steps % (uint64_t)st.admit_half == 0) {
        for (int i = threadIdx.x; i < L * E; i += blockDim.x) st.heat[i] = __fmul_rn(st.heat[i], 0.5f);
    }
    if (threadIdx.x == 0) {
        if (s_dirty && st.batch_tables) st.g[G_FLUSHES] += 1;
        int n = 0;
        for (int l = 0; l < L; ++l) {
            for (int a = 0; a < st.n_jobs[l]; ++a) {
                const int32_t *jb = st.jobs + ((size_t)l * MI + a) * 4;
                host_jobs[4 * n + 0] = l;
                host_jobs[4 * n + 1] = jb[0];
                host_jobs[4 * n + 2] = jb[1];
                host_jobs[4 * n + 3] = jb[2];
                n++;
            }
        }
        __threadfence_system();
        *host_njobs = n;
    }
}

// ===========================================================================
// host-side launchers
// ===========================================================================

cudaError_t launch_quantize(const float *x, void *y, int64_t n, int qtype, cudaStream_t s) {
    const int64_t nb = n / MOE_QK;
    if (nb == 0) return cudaSuccess;
    k_quantize<<<(unsigned)((nb + 127) / 128), 128, 0, s>>>(x, (uint8_t *)y, nb, qtype);
    return cudaGetLastError();
}

cudaError_t launch_synth_weights(void *y, int64_t nb, int qtype, uint64_t seed, float sigma,
                                 cudaStream_t s) {
    if (nb == 0) return cudaSuccess;
    k_synth_weights<<<(unsigned)((nb + 127) / 128), 128, 0, s>>>((uint8_t *)y, nb, qtype, seed, sigma);
    return cudaGetLastError();
}

cudaError_t launch_synth_f32(float *y, int64_t n, uint64_t seed, float sigma, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int64_t nt = (n + 1) / 2;
    k_synth_f32<<<(unsigned)((nt + 255) / 256), 256, 0, s>>>(y, n, seed, sigma);
    return cudaGetLastError();
}

cudaError_t launch_router(const float *W, const float *x, int n_tok, int n_expert, int n_embd,
                          const int32_t *table, int ns, float delta, int use_prior, int k,
                          int32_t *ids, float *w, float *logits, const SlotState *st,
                          int observe_layer_idx, const int32_t *pub, cudaStream_t s) {
    if (n_embd == 2048 && !logits && (n_tok == 1 || (!use_prior && observe_layer_idx < 0))) {
        // one cluster of RB_CL CTAs per TOK tokens
        const bool small = n_tok <= RB_SMALL_MAX;
        const int tok = small ? RB_TOK_SMALL : RB_TOK;
        const size_t sm = sizeof(float) * (size_t)tok * 2048;
        const void *fn = small ? (const void *)k_router_batch<RB_TOK_SMALL, 512>
                               : (const void *)k_router_batch<RB_TOK, 256>;
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return e;
        const int groups = (n_tok + tok - 1) / tok;
        SlotState dummy_st{};
        const SlotState sst = st ? *st : dummy_st;
        const int obs = st ? observe_layer_idx : -1;
        if (small)
            k_router_batch<RB_TOK_SMALL, 512><<<groups * RB_CL, 512, sm, s>>>(
                W, x, n_tok, n_expert, k, ids, w, table, ns, delta, use_prior, sst, obs, pub);
        else
            k_router_batch<RB_TOK, 256><<<groups * RB_CL, 256, sm, s>>>(
                W, x, n_tok, n_expert, k, ids, w, table, ns, delta, use_prior, sst, obs, pub);
        return cudaGetLastError();
    }
    const size_t smem = sizeof(float) * ((size_t)n_embd + n_expert);
    SlotState dummy{};
    const int threads = n_expert >= 512 ? 512 : (n_expert < 32 ? 32 : n_expert);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_router, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
    }
    k_router<<<n_tok, threads, smem, s>>>(W, x, n_expert, n_embd, table, ns, delta, use_prior, k,
                                          ids, w, logits, st ? *st : dummy,
                                          st ? observe_layer_idx : -1, pub);
    return cudaGetLastError();
}

cudaError_t launch_experts(const ExpertSrc &src, const float *x, const int32_t *ids,
                           const float *w, int n_tok, int k, int n_embd, int n_ff, int down_type,
                           float *act, const float *resid, float *y, int *err, cudaStream_t s) {
    dim3 g1((n_ff + GU_ROWS - 1) / GU_ROWS, n_tok * k);
    k_gate_up<<<g1, 256, 0, s>>>(src, x, ids, k, n_embd, n_ff, act, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = (size_t)k * n_ff + 2 * sizeof(float) * (size_t)k * (n_ff / 32) +
                        sizeof(float) * (size_t)k * DN_ROWS + 16;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    dim3 g2((n_embd + DN_ROWS - 1) / DN_ROWS, n_tok);
    k_down<<<g2, 256, smem, s>>>(src, act, ids, w, k, n_embd, n_ff, down_type, resid, y, err);
    return cudaGetLastError();
}

cudaError_t launch_transpose(const float *in, float *out, int rows, int cols, cudaStream_t s) {
    dim3 grid((cols + 31) / 32, (rows + 31) / 32);
    k_transpose<<<grid, dim3(32, 8), 0, s>>>(in, out, rows, cols);
    return cudaGetLastError();
}

cudaError_t launch_observe(const SlotState &st, int layer, const int32_t *ids, int n,
                           cudaStream_t s) {
    k_observe<<<1, 32, 0, s>>>(st, layer, ids, n);
    return cudaGetLastError();
}

cudaError_t launch_step(const SlotState &st, int32_t *host_jobs, int32_t *host_njobs,
                        cudaStream_t s) {
    if (st.have_evict) {
        k_evict_scores<<<st.n_layers, 256, 0, s>>>(st);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    k_step<<<1, 256, 0, s>>>(st, host_jobs, host_njobs);
    return cudaGetLastError();
}

cudaError_t launch_issue_spec(const SlotState &st, int layer, const int32_t *top, int n_top,
                              cudaStream_t s) {
    k_issue_spec<<<1, 32, 0, s>>>(st, layer, top, n_top);
    return cudaGetLastError();
}

// ---- just-in-time streaming: the lookahead (patches/0010:383-474) ----------

#define AHEAD_WARPS 8

// scores[t][e] = router row e of layer layer0 + t (t < n_targets) dotted with
// the observed layer's input x, in router_dot_warp's order (the canonical
// router arithmetic: a score is the logit that router would give x).
// grid (n_expert / AHEAD_WARPS, n_targets); block AHEAD_WARPS warps.
__global__ void __launch_bounds__(AHEAD_WARPS * 32) k_ahead_scores(const float *__restrict__ routers,
                                                                   const float *__restrict__ x, int layer0,
                                                                   int n_expert, int n_embd,
                                                                   float *__restrict__ scores) {
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int e = blockIdx.x * AHEAD_WARPS + (threadIdx.x >> 5);
    if (e >= n_expert) return;
    const float *w = routers + ((size_t)(layer0 + t) * n_expert + e) * n_embd;
    const float v = router_dot_warp(w, x, n_embd, lane);
    if (lane == 0) scores[(size_t)t * n_expert + e] = v;
}

// One CTA of 32 * n_targets threads: warp t takes the topk best scores of
// target t (score descending, ties to the lower id) and keeps those its
// layer's table says are not resident, in that order (out[t][...], count
// n_out[t]: k_moe_ahead_post, patches/0010:407-474).  Then one thread claims
// slots for them from the free pools (issue_uploads with spec 2 = streamed),
// at most per_layer streamed jobs per layer and token, keeping max_inserts
// slots for demand (stream_take, patches/0010:1477-1520); the claims are
// listed for the host's mover.
__global__ void k_ahead_claim(SlotState st, const float *__restrict__ scores, int layer0, int n_targets,
                              int k, int per_layer, int32_t *__restrict__ out, int32_t *__restrict__ n_out) {
    __shared__ int32_t s_ids[2][16];
    __shared__ int s_n[2];
    const int t = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int E = st.n_expert;
    if (t < n_targets) {
        const int l = layer0 + t, ns = st.ns[l];
        const int32_t *tbl = st.table + (size_t)l * E;
        const float *sc = scores + (size_t)t * E;
        uint32_t taken = 0;       // bit j: this lane's expert lane + 32 j is picked
        int n = 0;
        for (int r = 0; r < k; ++r) {
            float best = 0.0f;
            int bi = -1;
            for (int j = 0, e = lane; e < E; ++j, e += 32)
                if (!(taken & (1u << j)) && (bi < 0 || sc[e] > best)) { best = sc[e]; bi = e; }
            for (int off = 16; off >= 1; off >>= 1) {
                const float ob = __shfl_xor_sync(MOE_FULL, best, off);
                const int oi = __shfl_xor_sync(MOE_FULL, bi, off);
                if (oi >= 0 && (bi < 0 || ob > best || (ob == best && oi < bi))) { best = ob; bi = oi; }
            }
            if (bi < 0) break;
            if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
            if (tbl[bi] == ns) {
                if (lane == 0) s_ids[t][n] = bi;
                ++n;
            }
        }
        if (lane == 0) {
            s_n[t] = n;
            n_out[t] = n;
            for (int i = 0; i < n; ++i) out[t * 16 + i] = s_ids[t][i];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0)
        for (int tt = 0; tt < n_targets; ++tt) {
            const int l = layer0 + tt;
            const int32_t *jb = st.jobs + (size_t)l * st.job_cap * 4;
            int streamed = 0;
            for (int a = 0; a < st.n_jobs[l]; ++a) streamed += jb[4 * a + 2] == 2;
            if (streamed < per_layer)
                issue_uploads_dev(st, l, s_ids[tt], s_n[tt], per_layer - streamed, st.max_inserts, 2);
        }
}

// Streamed jobs the mover gave up on (late, or their layer read its table
// first): each (layer, expert, slot) leaves its layer's job list and the
// slot goes back to the free pool (its partial copy is never published).
// One thread.
__global__ void k_stream_cancel(SlotState st, const int32_t *__restrict__ jobs, int n) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int q = 0; q < n; ++q) {
        const int l = jobs[3 * q], e = jobs[3 * q + 1], slot = jobs[3 * q + 2];
        if (l < 0 || l >= st.n_layers) continue;
        int32_t *jb = st.jobs + (size_t)l * st.job_cap * 4;
        const int nj = st.n_jobs[l];
        for (int a = 0; a < nj; ++a) {
            if (jb[4 * a] != e || jb[4 * a + 1] != slot) continue;
            for (int c = 0; c < 4; ++c) jb[4 * a + c] = jb[4 * (nj - 1) + c];
            st.n_jobs[l] = nj - 1;
            const int so = st.slot_off[l];
            st.in_flight[so + slot] = 0;
            st.free_slots[so + st.n_free[l]] = slot;
            st.n_free[l] += 1;
            st.g[G_SCHEDULED] -= 1;
            st.g[G_UPLOADS] -= 1;
            break;
        }
    }
}

cudaError_t launch_ahead(const SlotState &st, const float *routers, const float *x, int layer0,
                         int n_targets, int n_embd, int k, int per_layer, float *scores, int32_t *out,
                         int32_t *n_out, cudaStream_t s) {
    if (n_targets < 1 || n_targets > 2 || k < 1 || k > 16 || per_layer < 1) return cudaErrorInvalidValue;
    const int E = st.n_expert;
    k_ahead_scores<<<dim3((E + AHEAD_WARPS - 1) / AHEAD_WARPS, n_targets), AHEAD_WARPS * 32, 0, s>>>(
        routers, x, layer0, E, n_embd, scores);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    k_ahead_claim<<<1, 64, 0, s>>>(st, scores, layer0, n_targets, k, per_layer, out, n_out);
    return cudaGetLastError();
}

cudaError_t launch_stream_cancel(const SlotState &st, const int32_t *jobs, int n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    k_stream_cancel<<<1, 32, 0, s>>>(st, jobs, n);
    return cudaGetLastError();
}

}  // namespace moe
