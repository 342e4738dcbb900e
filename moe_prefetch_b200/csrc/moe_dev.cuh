// moe_dev.cuh -- device helpers shared by every kernel of libmoeb200.so:
// exact fp32 math (exp, SiLU), the canonical router reduction, Q4_K / Q6_K x
// Q8_1 integer dots, activation quantisation, bulk-copy / mbarrier / timer
// wrappers, and the slot-table observation (moe_obs_cb) on the device.
//
// Exactness contract: every fp32 operation whose result reaches an expert id
// (router dot, softmax, prior add, top-k, renormalisation) is written with
// explicit round-to-nearest intrinsics (__fmaf_rn, __fadd_rn, __fmul_rn,
// __fdiv_rn), so nvcc cannot contract or reorder them, and the CPU oracle
// (oracle/moe_oracle.c) performs the same operations in the same order.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#define MOE_FULL 0xffffffffu
#define MOE_QK 256
#define MOE_Q4K_BYTES 144
#define MOE_Q6K_BYTES 210
#define MOE_QT_Q4K 12
#define MOE_QT_Q6K 14
#define MOE_KMAX 16              // max experts per token (incl. shared)
#define MOE_TIMEOUT_NS 2000000000ull   // 2 s: every device wait gives up after this

// device error bits (moe_api maps them to MOE_ERR_*)
#define MOE_DEV_ERR_TIMEOUT 1
#define MOE_DEV_ERR_INDEX   2

namespace moe {

// ---------------------------------------------------------------------------
// exact fp32 math
// ---------------------------------------------------------------------------

// exp(x) by Cody-Waite reduction x = n ln2 + r (ln2 split in a head with 12
// trailing zero bits and a tail) and the degree-7 Taylor polynomial of e^r in
// Horner form, then 2^n through the exponent field.  The same sequence of
// correctly rounded fp32 operations as or_expf() in the oracle.
__device__ __forceinline__ float expf_exact(float x) {
    if (x < -80.0f) return 0.0f;
    if (x > 80.0f) x = 80.0f;
    const float t = __fmul_rn(x, 0x1.715476p+0f);
    const float n = rintf(t);
    float r = __fmaf_rn(-n, 0x1.62e000p-1f, x);
    r = __fmaf_rn(-n, 0x1.0bfbe8p-15f, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

// SiLU(g) * u = g / (1 + e^-g) * u
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float e = expf_exact(-g);
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

// ---------------------------------------------------------------------------
// canonical router: one warp per logit
// ---------------------------------------------------------------------------

// Lane l owns columns 128*kk + 4*l + c, keeps four fma chains (c = 0..3) over
// kk, folds them as (a0+a1)+(a2+a3), then an xor butterfly 16,8,4,2,1.
// Every lane returns the same value.  w and x may be shared or global.
__device__ __forceinline__ float router_dot_warp(const float *__restrict__ w,
                                                 const float *__restrict__ x, int n_embd,
                                                 int lane) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 16
    for (int kk = 0; kk < n_embd / 128; ++kk) {
        const int j = 128 * kk + 4 * lane;
        const float4 wv = *reinterpret_cast<const float4 *>(w + j);
        const float4 xv = *reinterpret_cast<const float4 *>(x + j);
        a0 = __fmaf_rn(wv.x, xv.x, a0);
        a1 = __fmaf_rn(wv.y, xv.y, a1);
        a2 = __fmaf_rn(wv.z, xv.z, a2);
        a3 = __fmaf_rn(wv.w, xv.w, a3);
    }
    float v = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(MOE_FULL, v, off));
    return v;
}

// The cache prior's residency test: expert e is resident as published at
// the last token boundary.  With `pub` (the layer's slot -> expert map, set
// only when a slot is published) a table word that a streamed copy wrote
// within the token does not count, so routing never depends on when a copy
// lands (the reference's prior tensor moves only at publication,
// patches/0007:328-346).  Without it, table[e] != ns.
__device__ __forceinline__ bool prior_resident(const int32_t *table, int ns, const int32_t *pub, int e) {
    const int s = table[e];
    return s != ns && (pub == nullptr || pub[s] == e);
}

// Softmax over n_expert logits, + delta on resident experts (prior_resident)
// when use_prior, top-k by selection value (ties to the lower id), weights
// from the unbiased probabilities renormalised over the k.  One warp; lane l
// holds experts l, l+32, ...  ids/w written by lane 0 (any memory).
__device__ __forceinline__ void router_select_warp(const float *logits, int n_expert,
                                                   const int32_t *table, int ns, float delta,
                                                   bool use_prior, int k, int32_t *ids_out,
                                                   float *w_out, int lane,
                                                   const int32_t *pub = nullptr) {
    const int m = n_expert >> 5;   // <= 8
    float lg[8], ex[8], p[8], sel[8];
    bool taken[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        lg[i] = i < m ? logits[lane + 32 * i] : -INFINITY;
        taken[i] = false;
    }
    float mx = lg[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
        if (i < m) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(MOE_FULL, mx, off));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < m) {
            ex[i] = expf_exact(__fsub_rn(lg[i], mx));
            s = i == 0 ? ex[0] : __fadd_rn(s, ex[i]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(MOE_FULL, s, off));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < m) {
            p[i] = __fdiv_rn(ex[i], s);
            const int e = lane + 32 * i;
            const bool res = use_prior && table != nullptr && prior_resident(table, ns, pub, e);
            sel[i] = res ? __fadd_rn(p[i], delta) : p[i];
        } else {
            p[i] = 0.0f;
            sel[i] = -INFINITY;
            taken[i] = true;
        }
    }
    float psel[MOE_KMAX];
    int isel[MOE_KMAX];
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        float bp = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            if (!taken[i] && (sel[i] > bv || (sel[i] == bv && e < bi))) {
                bv = sel[i];
                bi = e;
                bp = p[i];
            }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const float ov = __shfl_xor_sync(MOE_FULL, bv, off);
            const int oi = __shfl_xor_sync(MOE_FULL, bi, off);
            const float op = __shfl_xor_sync(MOE_FULL, bp, off);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
                bp = op;
            }
        }
        if ((bi & 31) == lane) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i == (bi >> 5)) taken[i] = true;
        }
        isel[r] = bi;
        psel[r] = bp;
    }
    float ws = psel[0];
    for (int r = 1; r < k; ++r) ws = __fadd_rn(ws, psel[r]);
    if (lane == 0) {
        for (int r = 0; r < k; ++r) {
            ids_out[r] = isel[r];
            w_out[r] = __fdiv_rn(psel[r], ws);
        }
    }
}

// The softmax half of router_select_warp, run by one warp: probabilities and
// selection values (p + delta on resident experts) into shared memory, in the
// same canonical order.
__device__ __forceinline__ void router_softmax_warp(const float *logits, int n_expert,
                                                    const int32_t *table, int ns, float delta,
                                                    bool use_prior, float *s_p, float *s_sel,
                                                    int lane, uint64_t *s_key = nullptr) {
    const int m = n_expert >> 5;
    float lg[8], ex[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) lg[i] = i < m ? logits[lane + 32 * i] : -INFINITY;
    float mx = lg[0];
#pragma unroll
    for (int i = 1; i < 8; ++i)
        if (i < m) mx = fmaxf(mx, lg[i]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(MOE_FULL, mx, off));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < m) {
            ex[i] = expf_exact(__fsub_rn(lg[i], mx));
            s = i == 0 ? ex[0] : __fadd_rn(s, ex[i]);
        }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(MOE_FULL, s, off));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < m) {
            const int e = lane + 32 * i;
            const float p = __fdiv_rn(ex[i], s);
            const bool res = use_prior && table != nullptr && table[e] != ns;
            const float sv = res ? __fadd_rn(p, delta) : p;
            s_p[e] = p;
            s_sel[e] = sv;
            if (s_key) s_key[e] = ((uint64_t)__float_as_uint(sv) << 32) | (uint64_t)(~(uint32_t)e);
        }
    }
}

// Fixed-point partial sums of the fused decode router.  A CTA's partial
// logit is clamped to [-2^20, 2^20] and rounded to the nearest multiple of
// 2^-32 (ties to even), its partial sum of squares clamped to 2^36 and rounded
// to a multiple of 2^-16; the int64 totals (at most 256 terms, no overflow)
// do not depend on the order of the additions, and each total becomes a float
// with one rounding.  or_router_fused restates this.
#define FX_LOGIT_SCALE 4294967296.0f            // 2^32
#define FX_LOGIT_INV 2.3283064365386963e-10f    // 2^-32
#define FX_SUMSQ_SCALE 65536.0f                 // 2^16
#define FX_SUMSQ_INV 1.52587890625e-05f         // 2^-16

__device__ __forceinline__ long long fx_logit(float v) {
    return __float2ll_rn(__fmul_rn(fminf(fmaxf(v, -1048576.0f), 1048576.0f), FX_LOGIT_SCALE));
}

__device__ __forceinline__ long long fx_sumsq(float v) {
    return __float2ll_rn(__fmul_rn(fminf(v, 68719476736.0f), FX_SUMSQ_SCALE));
}

// Compare-exchange of two (key high, key low, p) entries so that entry i holds
// the larger key: the sorting step of select_warp.
__device__ __forceinline__ void sel_cx(uint32_t &hi_a, uint32_t &lo_a, float &p_a, uint32_t &hi_b,
                                       uint32_t &lo_b, float &p_b) {
    const bool sw = hi_b > hi_a || (hi_b == hi_a && lo_b > lo_a);
    const uint32_t th = sw ? hi_b : hi_a, tl = sw ? lo_b : lo_a;
    const float tp = sw ? p_b : p_a;
    hi_b = sw ? hi_a : hi_b;
    lo_b = sw ? lo_a : lo_b;
    p_b = sw ? p_a : p_b;
    hi_a = th;
    lo_a = tl;
    p_a = tp;
}

// The whole selection of one token in one warp: the logits tot[e] * inv, the
// softmax and cache prior of router_softmax_warp, top-k in the total order of
// topk_key_block (selection bits, then ~id), and the weights p / sum(p) with
// the sum formed in rank order.  The same operations in the same order as
// those three steps, so the same bits.
//
// Top-k: every lane sorts its M keys once (descending); each round then
// takes the largest list head in the warp with two reductions (high word,
// then low word among the lanes holding that high word), and the lane that
// holds it pops its head.  Ids are unique, so exactly one lane wins a round.
// The winner writes rank r's id and p to s_id[r] / s_p[r] (shared, MOE_KMAX
// each).  Lane r < k returns rank r's id and weight.  M experts per lane
// (n_expert = 32 * M), M = 1, 2, 4 or 8.
template <int M>
__device__ __forceinline__ void select_warp(const float *tot, float inv, const int32_t *table,
                                            int ns, float delta, bool use_prior, int k, int lane,
                                            int &id_r, float &w_r, int32_t *s_id, float *s_p,
                                            const int32_t *pub = nullptr) {
    static_assert(M == 1 || M == 2 || M == 4 || M == 8, "select_warp: 32 to 256 experts");
    float lg[M], ex[M], pr[M];
    uint32_t kh[M], kl[M];
#pragma unroll
    for (int i = 0; i < M; ++i) lg[i] = __fmul_rn(tot[lane + 32 * i], inv);
    float mx = lg[0];
#pragma unroll
    for (int i = 1; i < M; ++i) mx = fmaxf(mx, lg[i]);
    // warp max through a signed integer image that orders like the floats
    // (negative values: low 31 bits flipped); the max of the values, as the
    // fmaxf butterfly gives it (a max of +-0 subtracts to the same exponent)
    int oi = __float_as_int(mx);
    oi = oi >= 0 ? oi : oi ^ 0x7FFFFFFF;
    oi = __reduce_max_sync(MOE_FULL, oi);
    mx = __int_as_float(oi >= 0 ? oi : oi ^ 0x7FFFFFFF);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        ex[i] = expf_exact(__fsub_rn(lg[i], mx));
        s = i == 0 ? ex[0] : __fadd_rn(s, ex[i]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(MOE_FULL, s, off));
#pragma unroll
    for (int i = 0; i < M; ++i) {
        const int e = lane + 32 * i;
        pr[i] = __fdiv_rn(ex[i], s);
        const bool res = use_prior && table != nullptr && prior_resident(table, ns, pub, e);
        const float sv = res ? __fadd_rn(pr[i], delta) : pr[i];
        kh[i] = __float_as_uint(sv);
        kl[i] = ~(uint32_t)e;
    }
    // sort the lane's M entries, largest first (Batcher's odd-even merge sort)
    if (M == 2) {
        sel_cx(kh[0], kl[0], pr[0], kh[1], kl[1], pr[1]);
    } else if (M == 4) {
        sel_cx(kh[0], kl[0], pr[0], kh[1], kl[1], pr[1]);
        sel_cx(kh[2], kl[2], pr[2], kh[3], kl[3], pr[3]);
        sel_cx(kh[0], kl[0], pr[0], kh[2], kl[2], pr[2]);
        sel_cx(kh[1], kl[1], pr[1], kh[3], kl[3], pr[3]);
        sel_cx(kh[1], kl[1], pr[1], kh[2], kl[2], pr[2]);
    } else if (M == 8) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) sel_cx(kh[i], kl[i], pr[i], kh[i + 1], kl[i + 1], pr[i + 1]);
#pragma unroll
        for (int i = 0; i < 8; i += 4) {
            sel_cx(kh[i], kl[i], pr[i], kh[i + 2], kl[i + 2], pr[i + 2]);
            sel_cx(kh[i + 1], kl[i + 1], pr[i + 1], kh[i + 3], kl[i + 3], pr[i + 3]);
            sel_cx(kh[i + 1], kl[i + 1], pr[i + 1], kh[i + 2], kl[i + 2], pr[i + 2]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sel_cx(kh[i], kl[i], pr[i], kh[i + 4], kl[i + 4], pr[i + 4]);
        sel_cx(kh[2], kl[2], pr[2], kh[4], kl[4], pr[4]);
        sel_cx(kh[3], kl[3], pr[3], kh[5], kl[5], pr[5]);
        sel_cx(kh[1], kl[1], pr[1], kh[2], kl[2], pr[2]);
        sel_cx(kh[3], kl[3], pr[3], kh[4], kl[4], pr[4]);
        sel_cx(kh[5], kl[5], pr[5], kh[6], kl[6], pr[6]);
    }
    // (0, 0) is below every real key (~id > 0): an exhausted list never wins
    for (int r = 0; r < k; ++r) {
        const uint32_t mh = __reduce_max_sync(MOE_FULL, kh[0]);
        const uint32_t ml = __reduce_max_sync(MOE_FULL, kh[0] == mh ? kl[0] : 0u);
        if (kh[0] == mh && kl[0] == ml) {
            s_id[r] = (int32_t)(~ml);
            s_p[r] = pr[0];
#pragma unroll
            for (int i = 0; i + 1 < M; ++i) {
                kh[i] = kh[i + 1];
                kl[i] = kl[i + 1];
                pr[i] = pr[i + 1];
            }
            kh[M - 1] = 0u;
            kl[M - 1] = 0u;
        }
    }
    __syncwarp();
    float ws = s_p[0];
    for (int r = 1; r < k; ++r) ws = __fadd_rn(ws, s_p[r]);
    id_r = lane < k ? s_id[lane] : -1;
    w_r = lane < k ? __fdiv_rn(s_p[lane], ws) : 0.0f;
    __syncwarp();
}

// The ids that select_warp is expected to return when the cache prior is off,
// without the softmax: top-k of the logits tot[e] * inv in the order (logit
// descending, id ascending).  exp and the division by the common sum keep
// that order except where they round two logits to one probability, so the
// result is a prediction that the caller checks against select_warp's ids.
// Returns the id of rank `lane` for lane < k, else -1.
template <int M>
__device__ __forceinline__ int spec_topk_warp(const float *tot, float inv, int k, int lane) {
    uint32_t kh[M], kl[M];
    float pd[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
        const uint32_t u = __float_as_uint(__fmul_rn(tot[lane + 32 * i], inv));
        kh[i] = (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // orders like the floats
        kl[i] = ~(uint32_t)(lane + 32 * i);
        pd[i] = 0.0f;
    }
    if (M == 2) {
        sel_cx(kh[0], kl[0], pd[0], kh[1], kl[1], pd[1]);
    } else if (M == 4) {
        sel_cx(kh[0], kl[0], pd[0], kh[1], kl[1], pd[1]);
        sel_cx(kh[2], kl[2], pd[2], kh[3], kl[3], pd[3]);
        sel_cx(kh[0], kl[0], pd[0], kh[2], kl[2], pd[2]);
        sel_cx(kh[1], kl[1], pd[1], kh[3], kl[3], pd[3]);
        sel_cx(kh[1], kl[1], pd[1], kh[2], kl[2], pd[2]);
    } else if (M == 8) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) sel_cx(kh[i], kl[i], pd[i], kh[i + 1], kl[i + 1], pd[i + 1]);
#pragma unroll
        for (int i = 0; i < 8; i += 4) {
            sel_cx(kh[i], kl[i], pd[i], kh[i + 2], kl[i + 2], pd[i + 2]);
            sel_cx(kh[i + 1], kl[i + 1], pd[i + 1], kh[i + 3], kl[i + 3], pd[i + 3]);
            sel_cx(kh[i + 1], kl[i + 1], pd[i + 1], kh[i + 2], kl[i + 2], pd[i + 2]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sel_cx(kh[i], kl[i], pd[i], kh[i + 4], kl[i + 4], pd[i + 4]);
        sel_cx(kh[2], kl[2], pd[2], kh[4], kl[4], pd[4]);
        sel_cx(kh[3], kl[3], pd[3], kh[5], kl[5], pd[5]);
        sel_cx(kh[1], kl[1], pd[1], kh[2], kl[2], pd[2]);
        sel_cx(kh[3], kl[3], pd[3], kh[4], kl[4], pd[4]);
        sel_cx(kh[5], kl[5], pd[5], kh[6], kl[6], pd[6]);
    }
    int out = -1;
    for (int r = 0; r < k; ++r) {
        const uint32_t mh = __reduce_max_sync(MOE_FULL, kh[0]);
        const uint32_t ml = __reduce_max_sync(MOE_FULL, kh[0] == mh ? kl[0] : 0u);
        if (lane == r) out = (int)(~ml);
        if (kh[0] == mh && kl[0] == ml) {
#pragma unroll
            for (int i = 0; i + 1 < M; ++i) {
                kh[i] = kh[i + 1];
                kl[i] = kl[i + 1];
            }
            kh[M - 1] = 0u;
            kl[M - 1] = 0u;
        }
    }
    return out;
}

// select_warp for the cache prior off, given a prediction of its ids (sp_id of
// rank `lane` for lane < k, distinct, in [0, 32 M)): the same logits, softmax
// and probabilities, bit for bit, but instead of the sort and the k rounds of
// arg-max, a check that the predicted order is the selection order.  It is
// when the predicted probabilities are strictly decreasing by rank and the
// last is strictly above every other expert's: then the k largest in the
// order (probability descending, id ascending) are the predicted ids, in the
// predicted order, whatever the ties elsewhere.  On success the outputs are
// select_warp's (s_id / s_p, id_r / w_r with the same rank-order sum) and
// true is returned; otherwise false and nothing is written, and the caller
// runs select_warp.
template <int M>
__device__ __forceinline__ bool select_warp_check(const float *tot, float inv, int k, int lane, int sp_id,
                                                  int &id_r, float &w_r, int32_t *s_id, float *s_p) {
    float lg[M], ex[M], pr[M];
#pragma unroll
    for (int i = 0; i < M; ++i) lg[i] = __fmul_rn(tot[lane + 32 * i], inv);
    float mx = lg[0];
#pragma unroll
    for (int i = 1; i < M; ++i) mx = fmaxf(mx, lg[i]);
    int oi = __float_as_int(mx);
    oi = oi >= 0 ? oi : oi ^ 0x7FFFFFFF;
    oi = __reduce_max_sync(MOE_FULL, oi);
    mx = __int_as_float(oi >= 0 ? oi : oi ^ 0x7FFFFFFF);
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        ex[i] = expf_exact(__fsub_rn(lg[i], mx));
        s = i == 0 ? ex[0] : __fadd_rn(s, ex[i]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(MOE_FULL, s, off));
#pragma unroll
    for (int i = 0; i < M; ++i) pr[i] = __fdiv_rn(ex[i], s);
    // the predicted experts among this lane's (id lane + 32 i), and the
    // probability of predicted rank `lane`
    const int src = sp_id & 31, idx = sp_id >> 5;
    bool mine[M];
    float p_r = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        mine[i] = false;
        const float v = __shfl_sync(MOE_FULL, pr[i], src);
        if (idx == i) p_r = v;
    }
    for (int r = 0; r < k; ++r) {
        const int id = __shfl_sync(MOE_FULL, sp_id, r);
#pragma unroll
        for (int i = 0; i < M; ++i) mine[i] |= id == lane + 32 * i;
    }
    // probabilities are >= 0: their bits order like unsigned integers
    uint32_t rest = 0u;
#pragma unroll
    for (int i = 0; i < M; ++i) rest = mine[i] ? rest : max(rest, __float_as_uint(pr[i]));
    rest = __reduce_max_sync(MOE_FULL, rest);
    const float p_next = __shfl_down_sync(MOE_FULL, p_r, 1);
    const bool ok = lane >= k || (lane + 1 < k ? p_r > p_next : __float_as_uint(p_r) > rest);
    if (!__all_sync(MOE_FULL, ok)) return false;
    if (lane < k) {
        s_id[lane] = sp_id;
        s_p[lane] = p_r;
    }
    __syncwarp();
    float ws = s_p[0];
    for (int r = 1; r < k; ++r) ws = __fadd_rn(ws, s_p[r]);
    id_r = lane < k ? sp_id : -1;
    w_r = lane < k ? __fdiv_rn(p_r, ws) : 0.0f;
    __syncwarp();
    return true;
}

// Top-k by rank, all threads of the CTA: rank(e) = #experts before e in the
// order (selection value descending, id ascending); the k experts with rank < k
// land at position rank.  The same total order as k rounds of arg-max with
// ties to the lower id, so the same ids in the same order.  Needs a
// __syncthreads() before (s_sel / s_p complete) and after (outputs).
__device__ __forceinline__ void topk_rank_block(const float *s_sel, const float *s_p,
                                                int n_expert, int k, int32_t *ids_out,
                                                float *psel_out, int tid, int nthreads) {
    const int parts = nthreads / n_expert;   // 2 (256 experts) or 4 (128): a power of 2
    const int e = tid / parts, part = tid % parts;
    const int span = n_expert / parts;
    int cnt = 0;
    float v = 0.0f;
    if (e < n_expert) {
        v = s_sel[e];
        for (int j = part * span; j < (part + 1) * span; ++j) {
            const float u = s_sel[j];
            cnt += (u > v || (u == v && j < e)) ? 1 : 0;
        }
    }
    for (int off = 1; off < parts; off <<= 1) cnt += __shfl_xor_sync(MOE_FULL, cnt, off);
    if (e < n_expert && part == 0 && cnt < k) {
        ids_out[cnt] = e;
        psel_out[cnt] = s_p[e];
    }
}

// ---------------------------------------------------------------------------
// activation quantisation (Q8_1 blocks of 32, fp32 d and s)
// ---------------------------------------------------------------------------

// All threads of the CTA quantise n_blocks blocks of 32 values, 4 threads per
// block (8 values each): same d, q and s as q8_block_warp / the oracle (amax
// and the integer sum do not depend on the order).  src is read with
// ld.global.cg when from_global (data written by other CTAs), else from
// shared memory.  n_blocks * 4 must be a multiple of 32.
__device__ __forceinline__ void q8_quantize_cta(const float *src, bool from_global, int n_blocks,
                                                int8_t *q, float *d, float *s, int tid,
                                                int nthreads) {
    const int lane = tid & 31;
    for (int base = tid - lane; base < n_blocks * 4; base += nthreads) {
        const int b4 = base + lane;
        const int blk = b4 >> 2, part = b4 & 3;
        const bool valid = b4 < n_blocks * 4;
        float v[8];
        if (valid) {
            const float4 *p = reinterpret_cast<const float4 *>(src + 32 * blk + 8 * part);
            const float4 a = from_global ? __ldcg(p) : p[0];
            const float4 c = from_global ? __ldcg(p + 1) : p[1];
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, 2));
        const float db = __fdiv_rn(amax, 127.0f);
        const float id = amax > 0.0f ? __fdiv_rn(1.0f, db) : 0.0f;
        int qi[8];
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qi[i] = (int)roundf(__fmul_rn(v[i], id));
            sum += qi[i];
        }
        sum += __shfl_xor_sync(MOE_FULL, sum, 1);
        sum += __shfl_xor_sync(MOE_FULL, sum, 2);
        if (valid) {
            const uint32_t lo = (uint32_t)(qi[0] & 0xFF) | ((uint32_t)(qi[1] & 0xFF) << 8) |
                                ((uint32_t)(qi[2] & 0xFF) << 16) | ((uint32_t)(qi[3] & 0xFF) << 24);
            const uint32_t hi = (uint32_t)(qi[4] & 0xFF) | ((uint32_t)(qi[5] & 0xFF) << 8) |
                                ((uint32_t)(qi[6] & 0xFF) << 16) | ((uint32_t)(qi[7] & 0xFF) << 24);
            *reinterpret_cast<uint2 *>(q + 32 * blk + 8 * part) = make_uint2(lo, hi);
            if (part == 0) {
                d[blk] = db;
                s[blk] = __fmul_rn(db, (float)sum);
            }
        }
    }
}

// q8_quantize_cta of x = xf * inv for x in shared memory, each thread scaling
// the 8 values it quantises (__fmul_rn, written back to xf) -- the same bits
// as scaling the whole vector first.
__device__ __forceinline__ void q8_scale_quantize_cta(float *xf, float inv, int n_blocks, int8_t *q,
                                                      float *d, float *s, int tid, int nthreads) {
    const int lane = tid & 31;
    for (int base = tid - lane; base < n_blocks * 4; base += nthreads) {
        const int b4 = base + lane;
        const int blk = b4 >> 2, part = b4 & 3;
        const bool valid = b4 < n_blocks * 4;
        float v[8];
        if (valid) {
            float4 *p = reinterpret_cast<float4 *>(xf + 32 * blk + 8 * part);
            float4 a = p[0], c = p[1];
            a.x = __fmul_rn(a.x, inv); a.y = __fmul_rn(a.y, inv);
            a.z = __fmul_rn(a.z, inv); a.w = __fmul_rn(a.w, inv);
            c.x = __fmul_rn(c.x, inv); c.y = __fmul_rn(c.y, inv);
            c.z = __fmul_rn(c.z, inv); c.w = __fmul_rn(c.w, inv);
            p[0] = a;
            p[1] = c;
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, 2));
        const float db = __fdiv_rn(amax, 127.0f);
        const float id = amax > 0.0f ? __fdiv_rn(1.0f, db) : 0.0f;
        int qi[8];
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qi[i] = (int)roundf(__fmul_rn(v[i], id));
            sum += qi[i];
        }
        sum += __shfl_xor_sync(MOE_FULL, sum, 1);
        sum += __shfl_xor_sync(MOE_FULL, sum, 2);
        if (valid) {
            const uint32_t lo = (uint32_t)(qi[0] & 0xFF) | ((uint32_t)(qi[1] & 0xFF) << 8) |
                                ((uint32_t)(qi[2] & 0xFF) << 16) | ((uint32_t)(qi[3] & 0xFF) << 24);
            const uint32_t hi = (uint32_t)(qi[4] & 0xFF) | ((uint32_t)(qi[5] & 0xFF) << 8) |
                                ((uint32_t)(qi[6] & 0xFF) << 16) | ((uint32_t)(qi[7] & 0xFF) << 24);
            *reinterpret_cast<uint2 *>(q + 32 * blk + 8 * part) = make_uint2(lo, hi);
            if (part == 0) {
                d[blk] = db;
                s[blk] = __fmul_rn(db, (float)sum);
            }
        }
    }
}

// Padded activation layout of the decode kernel's down rows: 16 bytes after
// every 128 int8 of q, and per expert ACT_C_STRIDE(bpe) group offsets with 4
// ints after every 32, so that the six half super-blocks a row group reads
// fall in different shared-memory banks.  bpe: Q8_1 blocks per expert.
#define ACT_C_STRIDE(bpe) (2 * (bpe) + (bpe) / 4)

// All threads quantise n_blocks blocks read from global memory that other
// CTAs wrote (ld.global.cg), two threads per block (16 values each), every
// load issued before the arithmetic: the same d, q and s as q8_quantize_cta.
// With bpe > 0, q and c16 are written in the padded layout above.
// Also c16[2 * blk + half] = -32 * (sum of the 16 q of that half): the start
// value that turns a dot of unsigned 6-bit values with q into a dot of
// (value - 32) with q (dp4a_us).
__device__ __forceinline__ void q8_quantize_cta16(const float *src, int n_blocks, int8_t *q,
                                                  float *d, float *s, int *c16, int tid,
                                                  int nthreads, int bpe = 0) {
    const int lane = tid & 31;
    for (int base = tid - lane; base < n_blocks * 2; base += nthreads) {
        const int t2 = base + lane;
        const int blk = t2 >> 1, part = t2 & 1;
        const bool valid = t2 < n_blocks * 2;
        float4 v4[4];
        if (valid) {
            const float4 *p = reinterpret_cast<const float4 *>(src + 32 * blk + 16 * part);
#pragma unroll
            for (int j = 0; j < 4; ++j) v4[j] = __ldcg(p + j);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) v4[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        float v[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[4 * j] = v4[j].x; v[4 * j + 1] = v4[j].y; v[4 * j + 2] = v4[j].z; v[4 * j + 3] = v4[j].w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, 1));
        const float db = __fdiv_rn(amax, 127.0f);
        const float id = amax > 0.0f ? __fdiv_rn(1.0f, db) : 0.0f;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        int sum16 = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int qi = (int)roundf(__fmul_rn(v[i], id));
            sum16 += qi;
            w[i >> 2] |= (uint32_t)(qi & 0xFF) << (8 * (i & 3));
        }
        const int sum = sum16 + __shfl_xor_sync(MOE_FULL, sum16, 1);
        if (valid) {
            const int e = 32 * blk + 16 * part;
            int ci = 2 * blk + part;
            if (bpe > 0) {   // padded layout (load_act_half_up): bpe blocks per expert
                const int kk = blk / bpe, lci = ci - 2 * kk * bpe;
                ci = kk * ACT_C_STRIDE(bpe) + lci + 4 * (lci >> 5);
            }
            *reinterpret_cast<uint4 *>(q + (bpe > 0 ? e + 16 * (e >> 7) : e)) = make_uint4(w[0], w[1], w[2], w[3]);
            c16[ci] = -32 * sum16;
            if (part == 0) {
                d[blk] = db;
                s[blk] = __fmul_rn(db, (float)sum);
            }
        }
    }
}

// One warp quantises one block of 32 values: lane l takes element l.
// d = amax / 127, q = roundf(x * (1/d)), s = d * sum(q); as or_quantize_q8_1().
__device__ __forceinline__ void q8_block_warp(float v, int lane, int8_t *q, float *d,
                                              float *s) {
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(MOE_FULL, amax, off));
    const float db = __fdiv_rn(amax, 127.0f);
    const float id = amax > 0.0f ? __fdiv_rn(1.0f, db) : 0.0f;
    const int qi = (int)roundf(__fmul_rn(v, id));
    int sum = qi;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(MOE_FULL, sum, off);
    q[lane] = (int8_t)qi;
    if (lane == 0) {
        *d = db;
        *s = __fmul_rn(db, (float)sum);
    }
}

// ---------------------------------------------------------------------------
// Q4_K x Q8_1
// ---------------------------------------------------------------------------

// Activations of one lane's unit: super-block sb, sub-block pair p, i.e.
// 64 int8 values (sub-blocks 2p and 2p+1) and their d / s.
struct ActQ4 {
    int lo[8], hi[8];
    float d0, d1, s0, s1;
};

__device__ __forceinline__ void load_act_q4(ActQ4 &a, const int8_t *q, const float *d,
                                            const float *s, int sb, int p) {
    const int4 *ql = reinterpret_cast<const int4 *>(q + 256 * sb + 64 * p);
    const int4 v0 = ql[0], v1 = ql[1], v2 = ql[2], v3 = ql[3];
    a.lo[0] = v0.x; a.lo[1] = v0.y; a.lo[2] = v0.z; a.lo[3] = v0.w;
    a.lo[4] = v1.x; a.lo[5] = v1.y; a.lo[6] = v1.z; a.lo[7] = v1.w;
    a.hi[0] = v2.x; a.hi[1] = v2.y; a.hi[2] = v2.z; a.hi[3] = v2.w;
    a.hi[4] = v3.x; a.hi[5] = v3.y; a.hi[6] = v3.z; a.hi[7] = v3.w;
    const int b = 8 * sb + 2 * p;
    a.d0 = d[b]; a.d1 = d[b + 1];
    a.s0 = s[b]; a.s1 = s[b + 1];
}

// load_act_q4 from a unit-padded copy: the 64 int8 of the unit at `qu`
// (16-byte aligned) and its two Q8_1 blocks' d/s at d[b], s[b].
__device__ __forceinline__ void load_act_q4_unit(ActQ4 &a, const int8_t *qu, const float *d,
                                                 const float *s, int b) {
    const int4 *ql = reinterpret_cast<const int4 *>(qu);
    const int4 v0 = ql[0], v1 = ql[1], v2 = ql[2], v3 = ql[3];
    a.lo[0] = v0.x; a.lo[1] = v0.y; a.lo[2] = v0.z; a.lo[3] = v0.w;
    a.lo[4] = v1.x; a.lo[5] = v1.y; a.lo[6] = v1.z; a.lo[7] = v1.w;
    a.hi[0] = v2.x; a.hi[1] = v2.y; a.hi[2] = v2.z; a.hi[3] = v2.w;
    a.hi[4] = v3.x; a.hi[5] = v3.y; a.hi[6] = v3.z; a.hi[7] = v3.w;
    a.d0 = d[b]; a.d1 = d[b + 1];
    a.s0 = s[b]; a.s1 = s[b + 1];
}

__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFF; }

// 4-way byte dot: unsigned bytes of a times signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// 6-bit scale and min of sub-block j from the 12 scale bytes held in
// (w0: bytes 0-3, w1: 4-7, w2: 8-11)  (upstream get_scale_min_k4).
__device__ __forceinline__ void q4k_sm(uint32_t w0, uint32_t w1, uint32_t w2, int j, int &sc,
                                       int &m) {
    if (j < 4) {
        sc = byte_of(w0, j) & 63;
        m = byte_of(w1, j) & 63;
    } else {
        const int jj = j - 4;
        const int b8 = byte_of(w2, jj);
        sc = (b8 & 0xF) | ((byte_of(w0, jj) >> 6) << 4);
        m = (b8 >> 4) | ((byte_of(w1, jj) >> 6) << 4);
    }
}

// q4k_sm for the pair of sub-blocks 2p, 2p + 1 at once, the same integers:
// the four 6-bit scales (mins) of one half of the 12 bytes are formed in one
// word with byte-wise masks (j < 4: the low 6 bits of bytes j / j + 4;
// j >= 4: the low / high nibble of byte j + 4 below the top two bits of
// bytes j - 4 / j), then bytes 2(p & 1) and 2(p & 1) + 1 are picked.
__device__ __forceinline__ void q4k_sm_pair(uint32_t w0, uint32_t w1, uint32_t w2, int p, int &sc0,
                                            int &m0, int &sc1, int &m1) {
    const bool upper = p >= 2;
    const uint32_t S = upper ? ((w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u)) : (w0 & 0x3F3F3F3Fu);
    const uint32_t M = upper ? (((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u)) : (w1 & 0x3F3F3F3Fu);
    const uint32_t b = (uint32_t)(p & 1) * 2u;
    sc0 = (int)__byte_perm(S, 0u, 0x4440u | b);
    sc1 = (int)__byte_perm(S, 0u, 0x4440u | (b + 1u));
    m0 = (int)__byte_perm(M, 0u, 0x4440u | b);
    m1 = (int)__byte_perm(M, 0u, 0x4440u | (b + 1u));
}

// The float steps of one Q4_K unit from its integer sums (slo, shi: the two
// sub-blocks' dots with the activations; sc / m: their 6-bit scales and mins),
// with every rounding explicit so that no contraction choice of the compiler
// can change the bits:
//   acc = fma(sc1 * shi, d1, (sc0 * slo) * d0),  mm = fma(m1, s1, m0 * s0),
//   v   = fma(d, acc, -(dmin * mm)).
// Every GEMV path and the oracle's kernel-order rows use exactly this.
__device__ __forceinline__ float q4k_unit_float(int slo, int shi, int sc0, int m0, int sc1, int m1,
                                                float d, float dmin, const ActQ4 &a) {
    const float acc = __fmaf_rn((float)(sc1 * shi), a.d1, __fmul_rn((float)(sc0 * slo), a.d0));
    const float mm = __fmaf_rn((float)m1, a.s1, __fmul_rn((float)m0, a.s0));
    return __fmaf_rn(d, acc, -__fmul_rn(dmin, mm));
}

// The bytes of one unit of a Q4_K row: the block header (d, dmin, scales)
// and the 32 quant bytes of sub-block pair p.
struct Q4Unit {
    uint4 hdr, q0, q1;
};

__device__ __forceinline__ void q4k_unit_load(const uint8_t *blk, int p, Q4Unit &w) {
    w.hdr = *reinterpret_cast<const uint4 *>(blk);
    w.q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
    w.q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * p);
}

// The high nibbles are dotted in place (bytes 16 n, unsigned) and the sum,
// a multiple of 16, shifted down: the same integer as dotting n.
__device__ __forceinline__ float q4k_unit_compute(const Q4Unit &u, int p, const ActQ4 &a) {
    const uint32_t w[8] = {u.q0.x, u.q0.y, u.q0.z, u.q0.w, u.q1.x, u.q1.y, u.q1.z, u.q1.w};
    int slo = 0, shi16 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        slo = __dp4a((int)(w[i] & 0x0F0F0F0Fu), a.lo[i], slo);
        shi16 = dp4a_us(w[i] & 0xF0F0F0F0u, a.hi[i], shi16);
    }
    const int shi = shi16 >> 4;
    int sc0, m0, sc1, m1;
    q4k_sm_pair(u.hdr.y, u.hdr.z, u.hdr.w, p, sc0, m0, sc1, m1);
    const float d = h2f(u.hdr.x), dmin = h2f(u.hdr.x >> 16);
    return q4k_unit_float(slo, shi, sc0, m0, sc1, m1, d, dmin, a);
}

// int -> float without the conversion unit, exact for |v| <= 2^22: v added
// to the bits of 1.5 * 2^23 (a float whose ulp is 1 over [2^23, 2^24)),
// then 1.5 * 2^23 subtracted.  An integer add and a float add instead of an
// I2F, for the kernels in which conversions contend for the XU pipe.
__device__ __forceinline__ float i2f_small(int v) {
    return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

// A Q4_K unit decoded once for many activation rows: the nibble words, the
// integer scales and (as floats) the mins of its two sub-blocks, d and dmin.
struct Q4UnitDec {
    int lo[8], hi[8];
    int sc0, sc1;
    float m0, m1;
    float d, dmin;
};

__device__ __forceinline__ void q4k_unit_decode(const Q4Unit &u, int p, Q4UnitDec &o) {
    const uint32_t w[8] = {u.q0.x, u.q0.y, u.q0.z, u.q0.w, u.q1.x, u.q1.y, u.q1.z, u.q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        o.lo[i] = (int)(w[i] & 0x0F0F0F0Fu);
        o.hi[i] = (int)((w[i] >> 4) & 0x0F0F0F0Fu);
    }
    int m0, m1;
    q4k_sm_pair(u.hdr.y, u.hdr.z, u.hdr.w, p, o.sc0, m0, o.sc1, m1);
    o.m0 = (float)m0;
    o.m1 = (float)m1;
    o.d = h2f(u.hdr.x);
    o.dmin = h2f(u.hdr.x >> 16);
}

// q4k_unit_compute on a decoded unit: the same integer sums and the same
// float expression, bit for bit (sc * sum is at most 63 * 32 * 15 * 128 <
// 2^22, so i2f_small converts it exactly).
__device__ __forceinline__ float q4k_dec_compute(const Q4UnitDec &u, const ActQ4 &a) {
    int slo = 0, shi = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        slo = __dp4a(u.lo[i], a.lo[i], slo);
        shi = __dp4a(u.hi[i], a.hi[i], shi);
    }
    const float acc = __fmaf_rn(i2f_small(u.sc1 * shi), a.d1, __fmul_rn(i2f_small(u.sc0 * slo), a.d0));
    const float mm = __fmaf_rn(u.m1, a.s1, __fmul_rn(u.m0, a.s0));
    return __fmaf_rn(u.d, acc, -__fmul_rn(u.dmin, mm));
}

// Partial dot of one unit of a Q4_K row (16-byte aligned block pointer `blk`
// of super-block sb) with the unit's activations.  Loads are 128-bit.
__device__ __forceinline__ float q4k_unit_dot(const uint8_t *blk, int p, const ActQ4 &a) {
    Q4Unit u;
    q4k_unit_load(blk, p, u);
    return q4k_unit_compute(u, p, a);
}

// ---------------------------------------------------------------------------
// Q6_K x Q8_1, one lane per half super-block (128 elements)
// ---------------------------------------------------------------------------

// n consecutive 32-bit words starting at a 2-byte-aligned address, read as
// aligned words and realigned with funnel shifts; reads only words that hold
// requested bytes.  The aligned pointer is ptr minus the misalignment (not a
// masked integer), so that the compiler still sees a shared-memory pointer
// as one and emits shared loads.
template <int N>
__device__ __forceinline__ void ldw_a2(const uint8_t *ptr, uint32_t (&w)[N]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptr);
    const uint32_t *p = reinterpret_cast<const uint32_t *>(ptr - (a & 3));
    const uint32_t sh = (uint32_t)(a & 2) * 8u;
    uint32_t raw[N + 1];
#pragma unroll
    for (int i = 0; i < N; ++i) raw[i] = p[i];
    raw[N] = sh ? p[N] : 0u;
#pragma unroll
    for (int i = 0; i < N; ++i) w[i] = __funnelshift_r(raw[i], raw[i + 1], sh);
}

// Activations of a half super-block: 128 int8 (l = 0..31 for m = 0..3, as
// q[m][l/4]) and the d of the four Q8_1 blocks.
struct ActHalf {
    int q[4][8];
    float d[4];
};

__device__ __forceinline__ void load_act_half(ActHalf &a, const int8_t *q, const float *d, int sb,
                                              int h) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int e = 256 * sb + 128 * h + 32 * m;
        const int4 *qp = reinterpret_cast<const int4 *>(q + e);
        const int4 v0 = qp[0], v1 = qp[1];
        a.q[m][0] = v0.x; a.q[m][1] = v0.y; a.q[m][2] = v0.z; a.q[m][3] = v0.w;
        a.q[m][4] = v1.x; a.q[m][5] = v1.y; a.q[m][6] = v1.z; a.q[m][7] = v1.w;
        a.d[m] = d[e >> 5];
    }
}

// The bytes of half h of a Q6_K block, realigned into words: ql (low and
// high 32), qh, the 8 scales and d.
struct Q6Half {
    uint32_t lo[8], hi[8], qh[8], sc[2];
    float d;
};

// Load half h of the Q6_K block at `blk` (2-byte aligned).
__device__ __forceinline__ void q6k_half_load(const uint8_t *blk, int h, Q6Half &w) {
    ldw_a2<8>(blk + 64 * h, w.lo);          // ql[64h + l],      l = 0..31
    ldw_a2<8>(blk + 64 * h + 32, w.hi);     // ql[64h + 32 + l]
    ldw_a2<8>(blk + 128 + 32 * h, w.qh);    // qh[32h + l]
    ldw_a2<2>(blk + 192 + 8 * h, w.sc);     // scales[8h .. 8h+7]
    w.d = h2f(*reinterpret_cast<const uint16_t *>(blk + 208));
}

// Partial dot of a loaded Q6_K half with a half of Q8_1 activations: for
// each of its 8 scale groups (m, lower/upper 16 of l) an integer sum, scaled
// by the group scale and the Q8_1 d, accumulated in (m, group) order; times
// the block's d.
__device__ __forceinline__ float q6k_half_compute(const Q6Half &w, const ActHalf &a) {
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        int is0 = 0, is1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t src = (m & 1) ? w.hi[i] : w.lo[i];
            const uint32_t nib = (m >> 1) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu);
            const uint32_t hb = ((w.qh[i] >> (2 * m)) & 0x03030303u) << 4;
            const int v = (int)__vsub4(nib | hb, 0x20202020u);
            if (i < 4) is0 = __dp4a(v, a.q[m][i], is0);
            else is1 = __dp4a(v, a.q[m][i], is1);
        }
        const int g0 = 2 * m, g1 = 2 * m + 1;   // scale bytes within the 8 loaded
        const int s0 = (int)(int8_t)((w.sc[g0 >> 2] >> (8 * (g0 & 3))) & 0xFF);
        const int s1 = (int)(int8_t)((w.sc[g1 >> 2] >> (8 * (g1 & 3))) & 0xFF);
        acc = __fmaf_rn((float)(s0 * is0), a.d[m], acc);
        acc = __fmaf_rn((float)(s1 * is1), a.d[m], acc);
    }
    return __fmul_rn(w.d, acc);
}

// A Q6_K half decoded once for many activation rows: the signed 6-bit values
// (q - 32) as int8x4 words per quarter m, the 8 scales and d.
struct Q6HalfDec {
    int v[4][8];
    int sc[8];
    float d;
};

__device__ __forceinline__ void q6k_half_decode(const Q6Half &w, Q6HalfDec &o) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t src = (m & 1) ? w.hi[i] : w.lo[i];
            const uint32_t nib = (m >> 1) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu);
            const uint32_t hb = ((w.qh[i] >> (2 * m)) & 0x03030303u) << 4;
            o.v[m][i] = (int)__vsub4(nib | hb, 0x20202020u);
        }
    }
#pragma unroll
    for (int g = 0; g < 8; ++g) o.sc[g] = (int)(int8_t)((w.sc[g >> 2] >> (8 * (g & 3))) & 0xFF);
    o.d = w.d;
}

// q6k_half_compute on a decoded half: the same integer sums, scales and
// float accumulation order, bit for bit.
__device__ __forceinline__ float q6k_dec_compute(const Q6HalfDec &w, const ActHalf &a) {
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        int is0 = 0, is1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (i < 4) is0 = __dp4a(w.v[m][i], a.q[m][i], is0);
            else is1 = __dp4a(w.v[m][i], a.q[m][i], is1);
        }
        acc = __fmaf_rn((float)(w.sc[2 * m] * is0), a.d[m], acc);
        acc = __fmaf_rn((float)(w.sc[2 * m + 1] * is1), a.d[m], acc);
    }
    return __fmul_rn(w.d, acc);
}

// load_act_half from a half-padded copy: the 128 int8 of the half at `qh`
// (16-byte aligned) and the d of its four Q8_1 blocks at d[0..3].
__device__ __forceinline__ void load_act_half_at(ActHalf &a, const int8_t *qh, const float *d) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int4 *qp = reinterpret_cast<const int4 *>(qh + 32 * m);
        const int4 v0 = qp[0], v1 = qp[1];
        a.q[m][0] = v0.x; a.q[m][1] = v0.y; a.q[m][2] = v0.z; a.q[m][3] = v0.w;
        a.q[m][4] = v1.x; a.q[m][5] = v1.y; a.q[m][6] = v1.z; a.q[m][7] = v1.w;
        a.d[m] = d[m];
    }
}

// Partial dot of half h of the Q6_K block at `blk` (2-byte aligned) with a
// half of Q8_1 activations.
__device__ __forceinline__ float q6k_half_dot(const uint8_t *blk, int h, const ActHalf &a) {
    Q6Half w;
    q6k_half_load(blk, h, w);
    return q6k_half_compute(w, a);
}


// ActHalf plus, per scale group g (16 values), c[g] = -32 * (sum of its q):
// the start value of the group's integer sum in q6k_half_compute_u.
struct ActHalfU {
    int q[4][8];
    float d[4];
    int c[8];
};

__device__ __forceinline__ void load_act_half_u(ActHalfU &a, const int8_t *q, const float *d,
                                                const int *c16, int sb, int h) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int e = 256 * sb + 128 * h + 32 * m;
        const int4 *qp = reinterpret_cast<const int4 *>(q + e);
        const int4 v0 = qp[0], v1 = qp[1];
        a.q[m][0] = v0.x; a.q[m][1] = v0.y; a.q[m][2] = v0.z; a.q[m][3] = v0.w;
        a.q[m][4] = v1.x; a.q[m][5] = v1.y; a.q[m][6] = v1.z; a.q[m][7] = v1.w;
        a.d[m] = d[e >> 5];
        const int2 cc = *reinterpret_cast<const int2 *>(c16 + (e >> 4));
        a.c[2 * m] = cc.x;
        a.c[2 * m + 1] = cc.y;
    }
}

// load_act_half_u from the padded layout (q16_base and c16 of one expert).
__device__ __forceinline__ void load_act_half_up(ActHalfU &a, const int8_t *q, const float *d,
                                                 const int *c16, int sb, int h) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int e = 256 * sb + 128 * h + 32 * m;
        const int4 *qp = reinterpret_cast<const int4 *>(q + e + 16 * (e >> 7));
        const int4 v0 = qp[0], v1 = qp[1];
        a.q[m][0] = v0.x; a.q[m][1] = v0.y; a.q[m][2] = v0.z; a.q[m][3] = v0.w;
        a.q[m][4] = v1.x; a.q[m][5] = v1.y; a.q[m][6] = v1.z; a.q[m][7] = v1.w;
        a.d[m] = d[e >> 5];
        const int ci = e >> 4;
        const int2 cc = *reinterpret_cast<const int2 *>(c16 + ci + 4 * (ci >> 5));
        a.c[2 * m] = cc.x;
        a.c[2 * m + 1] = cc.y;
    }
}

// q6k_half_compute with the 6-bit values left unsigned: each group's integer
// sum starts at -32 * sum(q) and adds q_unsigned * q, which is the same
// integer as sum((q_unsigned - 32) * q); the float steps are unchanged, so
// the result is the same bits.
__device__ __forceinline__ float q6k_half_compute_u(const Q6Half &w, const ActHalfU &a) {
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        int is0 = a.c[2 * m], is1 = a.c[2 * m + 1];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t src = (m & 1) ? w.hi[i] : w.lo[i];
            const uint32_t nib = (m >> 1) ? (src >> 4) : src;
            const uint32_t hb = m == 0 ? (w.qh[i] << 4)
                              : m == 1 ? (w.qh[i] << 2)
                              : m == 2 ? w.qh[i] : (w.qh[i] >> 2);
            const uint32_t v = (nib & 0x0F0F0F0Fu) | (hb & 0x30303030u);
            if (i < 4) is0 = dp4a_us(v, a.q[m][i], is0);
            else is1 = dp4a_us(v, a.q[m][i], is1);
        }
        const int g0 = 2 * m, g1 = 2 * m + 1;
        const int s0 = (int)(int8_t)((w.sc[g0 >> 2] >> (8 * (g0 & 3))) & 0xFF);
        const int s1 = (int)(int8_t)((w.sc[g1 >> 2] >> (8 * (g1 & 3))) & 0xFF);
        acc = __fmaf_rn((float)(s0 * is0), a.d[m], acc);
        acc = __fmaf_rn((float)(s1 * is1), a.d[m], acc);
    }
    return __fmul_rn(w.d, acc);
}

__device__ __forceinline__ float q6k_half_dot_u(const uint8_t *blk, int h, const ActHalfU &a) {
    Q6Half w;
    q6k_half_load(blk, h, w);
    return q6k_half_compute_u(w, a);
}

// Sum over the 8 lanes of an aligned 8-lane group, butterfly 1, 2, 4 (fixed
// order; every lane of the group gets the same value).
__device__ __forceinline__ float group8_sum(float v) {
    v += __shfl_xor_sync(MOE_FULL, v, 1);
    v += __shfl_xor_sync(MOE_FULL, v, 2);
    v += __shfl_xor_sync(MOE_FULL, v, 4);
    return v;
}

// group8_sum's value for a group of gs = 2, 4, 6 or 8 consecutive lanes
// (unit u = 0 .. gs - 1) where group8_sum's lanes gs .. 7 would hold +0: the
// same tree ((v0 + v1) + (v2 + v3)) + ((v4 + v5) + (v6 + v7)), each absent
// pair taken as +0.  The result is valid in the group's lane u = 0, so that
// groups need not be aligned to 8 lanes.
__device__ __forceinline__ float groupn_sum(float v, int u, int gs) {
    const float a = v + __shfl_down_sync(MOE_FULL, v, 1);
    const float t2 = __shfl_down_sync(MOE_FULL, a, 2);
    const float b = a + (u + 2 < gs ? t2 : 0.0f);
    const float t4 = __shfl_down_sync(MOE_FULL, b, 4);
    return b + (u + 4 < gs ? t4 : 0.0f);
}

// Top-k by rank over 64-bit keys (selection bits << 32 | ~id: larger is
// better, ties to the lower id), thread (e, part) comparing against experts
// part, part + parts, ...; the same total order as topk_rank_block.
__device__ __forceinline__ void topk_key_block(const uint64_t *s_key, const float *s_p,
                                               int n_expert, int k, int32_t *ids_out,
                                               float *psel_out, int tid, int nthreads) {
    const int parts = nthreads / n_expert;
    const int e = tid / parts, part = tid - e * parts;
    int cnt = 0;
    const uint64_t ke = e < n_expert ? s_key[e] : 0ull;
    if (e < n_expert)
        for (int j = part; j < n_expert; j += parts) cnt += s_key[j] > ke ? 1 : 0;
    for (int off = 1; off < parts; off <<= 1) cnt += __shfl_xor_sync(MOE_FULL, cnt, off);
    if (e < n_expert && part == 0 && cnt < k) {
        ids_out[cnt] = e;
        psel_out[cnt] = s_p[e];
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(MOE_FULL, v, off);
    return v;
}

// Eight warp_sum's at once, bit for bit: lane l returns the sum of v[l >> 2].
// 9 shuffles instead of 40.
__device__ __forceinline__ float warp_sum8_t(const float (&v)[8], int lane) {
    const bool u16 = (lane & 16) != 0, u8 = (lane & 8) != 0, u4 = (lane & 4) != 0;
    float a[4], b[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = (u16 ? v[4 + i] : v[i]) + __shfl_xor_sync(MOE_FULL, u16 ? v[i] : v[4 + i], 16);
#pragma unroll
    for (int i = 0; i < 2; ++i) b[i] = (u8 ? a[2 + i] : a[i]) + __shfl_xor_sync(MOE_FULL, u8 ? a[i] : a[2 + i], 8);
    float c = (u4 ? b[1] : b[0]) + __shfl_xor_sync(MOE_FULL, u4 ? b[0] : b[1], 4);
    c += __shfl_xor_sync(MOE_FULL, c, 2);
    c += __shfl_xor_sync(MOE_FULL, c, 1);
    return c;
}

// Four warp_sum's at once, bit for bit: the same pairs at every level (xor
// 16, 8, 4, 2, 1; own value first), but each level exchanges only the sums a
// lane still needs.  Lanes 0-7 return the sum of a, 8-15 of b, 16-23 of c,
// 24-31 of d.  7 shuffles instead of 20.
__device__ __forceinline__ float warp_sum4_t(float a, float b, float c, float d, int lane) {
    const bool u16 = (lane & 16) != 0;
    float k0 = u16 ? c : a, k1 = u16 ? d : b;
    k0 += __shfl_xor_sync(MOE_FULL, u16 ? a : c, 16);
    k1 += __shfl_xor_sync(MOE_FULL, u16 ? b : d, 16);
    const bool u8 = (lane & 8) != 0;
    float k = u8 ? k1 : k0;
    k += __shfl_xor_sync(MOE_FULL, u8 ? k0 : k1, 8);
    k += __shfl_xor_sync(MOE_FULL, k, 4);
    k += __shfl_xor_sync(MOE_FULL, k, 2);
    k += __shfl_xor_sync(MOE_FULL, k, 1);
    return k;
}

// ---------------------------------------------------------------------------
// bulk copies, mbarriers, timers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// A plain arrival (no transaction bytes) on an mbarrier.
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One try_wait with a suspend-time hint of 1 ms: a waiting warp sleeps until
// the phase completes (the hardware wakes it) or the hint runs out, instead
// of polling and taking issue slots from the warps that produce the data.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Thread s < world of the CTA waits until flags[s] carries at least *epoch
// (acquire, system scope), bounded by wait_ns; then the whole CTA
// synchronises.  On expiry the timeout bit goes into *err.  Every thread of
// the CTA calls it.
__device__ __forceinline__ void cta_wait_flags(const unsigned long long *flags, int world,
                                               const unsigned long long *epoch, uint64_t wait_ns, int *err) {
    const int s = threadIdx.x;
    if (s < world) {
        const unsigned long long e = *epoch;
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + s) : "memory");
        if (v < e) {
            const uint64_t t0 = gtimer();
            for (;;) {
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + s) : "memory");
                if (v >= e) break;
                if (gtimer() - t0 > wait_ns) {
                    atomicOr(err, MOE_DEV_ERR_TIMEOUT);
                    break;
                }
                __nanosleep(200);
            }
        }
    }
    __syncthreads();
}

// Bounded wait: false after limit_ns (MOE_TIMEOUT_NS unless given).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          uint64_t limit_ns = MOE_TIMEOUT_NS) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_try_wait(bar, parity)) {
        if (gtimer() - t0 > limit_ns) return false;
    }
    return true;
}

// global -> shared bulk copy (TMA, no multicast); dst, src 16-byte aligned,
// bytes a multiple of 16; completion is counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Launch-order index of the CTA `ahead` SM counts after this one (x fastest),
// as (x, y) of the grid: with `ahead` CTAs per SM resident, the CTA likely
// to start next when this one ends.
__device__ __forceinline__ void next_wave_cta(int ahead, int &nx, int &ny) {
    uint32_t nsm;
    asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
    const int nxt = (int)(blockIdx.y * gridDim.x + blockIdx.x + (uint32_t)ahead * nsm);
    ny = nxt / (int)gridDim.x;
    nx = nxt % (int)gridDim.x;
}

// Hint: bring [src, src + bytes) into L2 (no completion, no destination);
// src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const unsigned *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_relaxed_i32(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// slot-table state on the device
// ---------------------------------------------------------------------------

// Flattened per-layer arrays.  Slot-indexed arrays use slot_off[layer].
struct SlotState {
    int n_layers, n_expert, max_inserts, admit_mode, admit_window, admit_half;
    float admit_floor, cache_prior;
    int spec_probation, batch_tables, freeze;
    const int32_t *ns;          // [L]
    const int32_t *slot_off;    // [L]
    int32_t *table;             // [L][E]   expert -> slot, ns = not resident
    int32_t *slot_expert;       // [sum ns]
    uint64_t *last_use;         // [sum ns]
    uint64_t *protect;          // [sum ns]
    uint8_t *in_flight;         // [sum ns]
    int32_t *pending;           // [L][E]
    int32_t *n_pending;         // [L]
    float *heat;                // [L][E] or null
    uint64_t *miss_last;        // [L][E] or null
    uint64_t *miss_prev;        // [L][E] or null
    uint32_t *use_count;        // [L][E] or null
    uint64_t *n_hit;            // [L]
    uint64_t *n_miss;           // [L]
    uint64_t *g;                // globals: see G_* below
    int32_t *jobs;              // [L][job_cap][4] (expert, slot, spec, -)
    int32_t *n_jobs;            // [L]
    int job_cap;                // jobs per layer: max_inserts (+ predict_top with early issue)
    // early issue (patches/0006:251-293, 0007:230-246): uploads start when a
    // layer is observed, into slots from a free pool that the step tops up
    int early_issue, predict_top, have_pred;
    int stream;                 // just-in-time streaming is on (jobs of spec 2)
    int stream_reserve;         // its extra free slots kept per layer
    int32_t *free_slots;        // [sum ns] each layer's free pool, a stack (top = last)
    int32_t *n_free;            // [L]
    int32_t *admitted;          // [L][E] scratch: the pending ids that passed admission
    int32_t *cur_ids;           // [L][CUR_IDS] ids each layer observed last (the predictor's next_prev)
    int32_t *n_cur;             // [L]
    int32_t *host_jobs;         // mapped host: (layer, expert, slot, spec) since the last step
    int32_t *host_njobs;        // mapped host: their count
    int host_cap;               // entries host_jobs holds
    // LLAMA_MOE_EVICTOR (patches/0006:402-426, :790-913): an MOEP model whose
    // per-layer score picks the victim instead of LRU
    int have_evict, ev_feat;
    int ev_off[4];              // row offsets of the prev, cur, below, self_prev blocks, -1 absent
    const int32_t *ev_index;    // [L] model slot or -1
    const float *ev_w;          // [n_model][ev_feat][E]
    const float *ev_bias;       // [n_model][E]
    const float *ev_prior;      // [n_model]
    float *ev_scores;           // [L][E] this step's scores
    int32_t *prev_ids;          // [L][CUR_IDS] cur_ids one token earlier
    int32_t *n_prev;            // [L]
};

// ids a layer keeps of its last observation, for the predictor
#define CUR_IDS 64

// Free slots a layer keeps at the step boundary (patches/0006:843-913,
// 0010 pool_target_of): the demand path's inserts, the predictor's guesses
// and the streaming reserve.
__host__ __device__ __forceinline__ int pool_target_of(const SlotState &st) {
    return st.freeze ? 0
                     : st.max_inserts + (st.have_pred ? st.predict_top : 0) + st.stream_reserve;
}

enum { G_CLOCK = 0, G_STEPS, G_UPLOADS, G_SCHEDULED, G_COPIED, G_PUBLISHED, G_ADMIT_OK,
       G_ADMIT_DENIED, G_FLUSHES, G_UPLOAD_BYTES,
       G_STREAM_IN_TIME,   // a streamed expert was routed and found resident by its layer
       G_STREAM_LATE,      // a streamed expert was routed before its table word landed
       G_COUNT };

// lru_resident (patches/0007:398-412): the resident expert of the least
// recently used slot not in flight, or -1.
__device__ __forceinline__ int lru_resident_dev(const SlotState &st, int l) {
    const int ns = st.ns[l], so = st.slot_off[l];
    int victim = -1;
    uint64_t best = ~0ull;
    for (int s = 0; s < ns; ++s) {
        if (st.in_flight[so + s] || st.slot_expert[so + s] < 0) continue;
        if (st.last_use[so + s] < best) {
            best = st.last_use[so + s];
            victim = st.slot_expert[so + s];
        }
    }
    return victim;
}

// admit_ok (patches/0007:414-429), counted; one thread.
__device__ __forceinline__ bool admit_ok_dev(const SlotState &st, int l, int id, int victim) {
    if (st.admit_mode == 0 || victim < 0) return true;
    const size_t E = (size_t)st.n_expert;
    bool ok = true;
    if (st.admit_mode == 1) {
        // heat is added to with atomics (from the lanes of the decode
        // kernel's observer): read it where those land
        const float *ht = st.heat + (size_t)l * E;
        ok = __ldcg(ht + id) > __fadd_rn(__fmul_rn(__ldcg(ht + victim), 1.25f), st.admit_floor);
    } else if (st.admit_mode == 2) {
        const uint64_t mp = st.miss_prev[(size_t)l * E + id], ml = st.miss_last[(size_t)l * E + id];
        ok = mp != ~0ull && ml - mp < (uint64_t)st.admit_window;
    }
    st.g[ok ? G_ADMIT_OK : G_ADMIT_DENIED] += 1;
    return ok;
}

// issue_uploads (patches/0006:251-293, 0007:230-246, 0008:498-500), one
// thread: up to `budget` of ids (not resident, not already a job of this
// layer) each take a slot from the layer's free pool while more than
// min_keep slots are free; the job goes to the layer's list and, for the
// uploader, to the mapped host list.
__device__ __forceinline__ int issue_uploads_dev(const SlotState &st, int l, const int32_t *ids, int n,
                                                 int budget, int min_keep, int spec) {
    if (st.freeze) return 0;
    const int E = st.n_expert, ns = st.ns[l], so = st.slot_off[l];
    const int32_t *tbl = st.table + (size_t)l * E;
    int32_t *jb = st.jobs + (size_t)l * st.job_cap * 4;
    int issued = 0;
    for (int i = 0; i < n && issued < budget; ++i) {
        const int id = ids[i];
        if (id < 0 || id >= E || tbl[id] != ns) continue;
        if (st.n_free[l] <= min_keep) break;
        const int nj = st.n_jobs[l];
        bool dup = false;
        for (int a = 0; a < nj; ++a)
            if (jb[4 * a] == id) { dup = true; break; }
        if (dup) continue;
        if (nj >= st.job_cap) break;   // not reached: the free pool bounds a layer's jobs
        volatile int32_t *hn = st.host_njobs;
        const int h = *hn;
        if (h >= st.host_cap) break;   // the host list is full until the step (streamed
                                       // jobs that were given back still hold entries)
        const int nf = st.n_free[l] - 1;
        const int slot = st.free_slots[so + nf];
        st.n_free[l] = nf;
        st.in_flight[so + slot] = 1;
        jb[4 * nj] = id; jb[4 * nj + 1] = slot; jb[4 * nj + 2] = spec; jb[4 * nj + 3] = 0;
        st.n_jobs[l] = nj + 1;
        st.g[G_UPLOADS] += 1;
        st.g[G_SCHEDULED] += 1;
        st.host_jobs[4 * h] = l; st.host_jobs[4 * h + 1] = id;
        st.host_jobs[4 * h + 2] = slot; st.host_jobs[4 * h + 3] = spec;
        __threadfence_system();
        *hn = h + 1;
        ++issued;
    }
    return issued;
}

// The early-issue half of moe_obs_cb (patches/0006:346-366, 0007:271-293),
// after a layer's misses are pending: the admitted pending ids take slots of
// the free pool now (budget max_inserts).  The admission of each pending id
// is decided against the slot the next top-up would free.  One thread.
__device__ __forceinline__ void early_issue_pending(const SlotState &st, int l) {
    const int E = st.n_expert, ns = st.ns[l];
    const int pool_target = pool_target_of(st);
    const int32_t *pend = st.pending + (size_t)l * E;
    const int np = st.n_pending[l];
    if (st.admit_mode == 0) {
        issue_uploads_dev(st, l, pend, np, st.max_inserts, 0, 0);
        return;
    }
    const int next_victim = st.n_free[l] > pool_target ? -1 : lru_resident_dev(st, l);
    const int32_t *tbl = st.table + (size_t)l * E;
    int32_t *adm = st.admitted + (size_t)l * E;
    int na = 0;
    for (int q = 0; q < np; ++q) {
        const int id = pend[q];
        if (tbl[id] == ns && admit_ok_dev(st, l, id, next_victim)) adm[na++] = id;
    }
    issue_uploads_dev(st, l, adm, na, st.max_inserts, 0, 0);
}

// moe_obs_cb for one single-token layer (patches/0006:295-400 with the
// 0007:247-270 window/heat bookkeeping and, with early issue, the uploads of
// the admitted misses).  One thread.
__device__ __forceinline__ void observe_layer(const SlotState &st, int layer,
                                              const int32_t *ids, int n) {
    const int E = st.n_expert;
    const int ns = st.ns[layer];
    const int so = st.slot_off[layer];
    int32_t *tbl = st.table + (size_t)layer * E;
    int32_t *pend = st.pending + (size_t)layer * E;
    const uint64_t n_steps = st.g[G_STEPS];
    uint64_t clock = st.g[G_CLOCK];
    for (int i = 0; i < n; ++i) {
        const int id = ids[i];
        if (id < 0 || id >= E) continue;
        if (st.heat) st.heat[(size_t)layer * E + id] += 1.0f;
        if (st.use_count) st.use_count[(size_t)layer * E + id] += 1u;
        const int slot = tbl[id];
        if (st.stream) {
            // was it streamed for this token? (a job of spec 2 still listed)
            const int32_t *jb = st.jobs + (size_t)layer * st.job_cap * 4;
            for (int a = 0; a < st.n_jobs[layer]; ++a)
                if (jb[4 * a] == id && jb[4 * a + 2] == 2) {
                    st.g[slot != ns ? G_STREAM_IN_TIME : G_STREAM_LATE] += 1;
                    break;
                }
        }
        if (slot != ns) {
            st.n_hit[layer] += 1;
            st.last_use[so + slot] = ++clock;
        } else {
            st.n_miss[layer] += 1;
            if (st.miss_last) {
                uint64_t *ml = st.miss_last + (size_t)layer * E;
                uint64_t *mp = st.miss_prev + (size_t)layer * E;
                if (ml[id] != n_steps) {
                    mp[id] = ml[id];
                    ml[id] = n_steps;
                }
            }
            const int np = st.n_pending[layer];
            bool dup = false;
            for (int q = 0; q < np; ++q)
                if (pend[q] == id) { dup = true; break; }
            if (!dup) {
                pend[np] = id;
                st.n_pending[layer] = np + 1;
            }
        }
    }
    st.g[G_CLOCK] = clock;
    if (st.early_issue) early_issue_pending(st, layer);
    if (st.cur_ids) {
        const int nc = n < CUR_IDS ? n : CUR_IDS;
        for (int i = 0; i < nc; ++i) st.cur_ids[(size_t)layer * CUR_IDS + i] = ids[i];
        st.n_cur[layer] = nc;
    }
}

}  // namespace moe
