/*
 * moe_oracle.c -- CPU restatement of the reference's MoE-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see moe_oracle.h).  Built with
 * -ffp-contract=off so that every fmaf() below is the only fused operation and
 * every other fp32 operation rounds on its own, exactly like the device code.
 */
#include "moe_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar helpers                                                            */
/* ------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* IEEE binary32 -> binary16, round to nearest even (the rounding
 * __float2half_rn performs). */
uint16_t or_f32_to_f16(float f) {
    const uint32_t x = f2u(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t mant = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
    }
    const int e = (int)exp - 127 + 15;
    if (e >= 31) {
        return (uint16_t)(sign | 0x7C00u);
    }
    if (e <= 0) {
        if (e < -10) {
            return (uint16_t)sign;
        }
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) {
            h++;
        }
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        h++;
    }
    return (uint16_t)h;
}

float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    if (exp == 0x1Fu) {
        return u2f(sign | 0x7F800000u | (mant << 13));
    }
    if (exp == 0) {
        if (mant == 0) {
            return u2f(sign);
        }
        /* subnormal half: normalise */
        int e = -1;
        do {
            e++;
            mant <<= 1;
        } while ((mant & 0x400u) == 0);
        mant &= 0x3FFu;
        exp = (uint32_t)(127 - 15 - e);
        return u2f(sign | (exp << 23) | (mant << 13));
    }
    return u2f(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

/* exp(x) by Cody-Waite argument reduction x = n ln2 + r, |r| <= ln2/2, with
 * ln2 split into a 12-bit-trimmed head (n * LN2_HI exact for |n| < 2^12) and
 * a tail, then the degree-7 Taylor polynomial of e^r in Horner form (truncation
 * error < 6e-9 relative on the reduced range), then scaling by 2^n through the
 * exponent field.  The device copy (moe_prefetch_b200/csrc/moe_dev.cuh) runs
 * the identical sequence of fp32 operations, so both give the same bits. */
#define OR_LOG2E  0x1.715476p+0f      /* 1/ln2 rounded to fp32          */
#define OR_LN2_HI 0x1.62e000p-1f      /* ln2 with the low 12 bits zero  */
#define OR_LN2_LO 0x1.0bfbe8p-15f     /* ln2 - LN2_HI rounded to fp32   */
float or_expf(float x) {
    if (x < -80.0f) {
        return 0.0f;
    }
    if (x > 80.0f) {
        x = 80.0f;
    }
    const float t = x * OR_LOG2E;
    const float n = rintf(t);
    float r = fmaf(-n, OR_LN2_HI, x);
    r = fmaf(-n, OR_LN2_LO, r);
    float p = 0x1.a01a02p-13f;            /* 1/7! */
    p = fmaf(p, r, 0x1.6c16c2p-10f);        /* 1/6! */
    p = fmaf(p, r, 0x1.111112p-7f);         /* 1/5! */
    p = fmaf(p, r, 0x1.555556p-5f);         /* 1/4! */
    p = fmaf(p, r, 0x1.555556p-3f);         /* 1/3! */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n;
    const float scale = u2f((uint32_t)(ni + 127) << 23);
    return p * scale;
}

static inline float or_silu_mul(float g, float u) {
    const float e = or_expf(-g);
    const float s = g / (1.0f + e);
    return s * u;
}

/* ------------------------------------------------------------------------ */
/* block codecs                                                              */
/* ------------------------------------------------------------------------ */

static inline int or_clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

/* 6-bit scale/min unpacking of the Q4_K header (upstream get_scale_min_k4) */
static inline void q4k_scale_min(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

void or_quantize_q4_K(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const float *xb = x + b * OR_QK_K;
        uint8_t *yb = y + b * OR_Q4K_BYTES;
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
            scale[j] = (mx - mn) / 15.0f;
            minv[j] = -mn;
            if (scale[j] > max_scale) max_scale = scale[j];
            if (minv[j] > max_min) max_min = minv[j];
        }
        const uint16_t dh = or_f32_to_f16(max_scale / 63.0f);
        const uint16_t mh = or_f32_to_f16(max_min / 63.0f);
        const float dd = or_f16_to_f32(dh), dm = or_f16_to_f32(mh);
        int sc[8], m[8];
        for (int j = 0; j < 8; ++j) {
            sc[j] = dd > 0.0f ? or_clampi((int)roundf(scale[j] / dd), 0, 63) : 0;
            m[j] = dm > 0.0f ? or_clampi((int)roundf(minv[j] / dm), 0, 63) : 0;
        }
        yb[0] = (uint8_t)(dh & 0xFF);
        yb[1] = (uint8_t)(dh >> 8);
        yb[2] = (uint8_t)(mh & 0xFF);
        yb[3] = (uint8_t)(mh >> 8);
        uint8_t *sc12 = yb + 4;
        for (int j = 0; j < 4; ++j) {
            sc12[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            sc12[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            sc12[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
        }
        uint8_t q[OR_QK_K];
        for (int j = 0; j < 8; ++j) {
            const float es = dd * (float)sc[j];
            const float em = dm * (float)m[j];
            for (int l = 0; l < 32; ++l) {
                q[32 * j + l] = es > 0.0f
                    ? (uint8_t)or_clampi((int)roundf((xb[32 * j + l] + em) / es), 0, 15)
                    : 0;
            }
        }
        uint8_t *qs = yb + 16;
        for (int p = 0; p < 4; ++p) {
            for (int l = 0; l < 32; ++l) {
                qs[32 * p + l] = (uint8_t)(q[64 * p + l] | (q[64 * p + 32 + l] << 4));
            }
        }
    }
}

void or_dequantize_q4_K(const uint8_t *y, float *x, int64_t n) {
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *yb = y + b * OR_Q4K_BYTES;
        const float d = or_f16_to_f32((uint16_t)(yb[0] | (yb[1] << 8)));
        const float dmin = or_f16_to_f32((uint16_t)(yb[2] | (yb[3] << 8)));
        const uint8_t *qs = yb + 16;
        float *xb = x + b * OR_QK_K;
        for (int p = 0; p < 4; ++p) {
            int sc, m;
            q4k_scale_min(2 * p, yb + 4, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            q4k_scale_min(2 * p + 1, yb + 4, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; ++l) {
                xb[64 * p + l] = d1 * (float)(qs[32 * p + l] & 0xF) - m1;
                xb[64 * p + 32 + l] = d2 * (float)(qs[32 * p + l] >> 4) - m2;
            }
        }
    }
}

void or_quantize_q6_K(const float *x, uint8_t *y, int64_t n) {
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const float *xb = x + b * OR_QK_K;
        uint8_t *yb = y + b * OR_Q6K_BYTES;
        float gscale[16];
        float max_scale = 0.0f;
        for (int g = 0; g < 16; ++g) {
            float amax = 0.0f;
            for (int l = 0; l < 16; ++l) {
                const float a = fabsf(xb[16 * g + l]);
                if (a > amax) amax = a;
            }
            gscale[g] = amax / 31.0f;
            if (gscale[g] > max_scale) max_scale = gscale[g];
        }
        const uint16_t dh = or_f32_to_f16(max_scale / 127.0f);
        const float dd = or_f16_to_f32(dh);
        int8_t sc[16];
        for (int g = 0; g < 16; ++g) {
            sc[g] = (int8_t)(dd > 0.0f ? or_clampi((int)roundf(gscale[g] / dd), -128, 127) : 0);
        }
        uint8_t q[OR_QK_K];
        for (int e = 0; e < OR_QK_K; ++e) {
            const float es = dd * (float)sc[e / 16];
            const int v = es != 0.0f ? or_clampi((int)roundf(xb[e] / es), -32, 31) : 0;
            q[e] = (uint8_t)(v + 32);
        }
        uint8_t *ql = yb, *qh = yb + 128;
        for (int h = 0; h < 2; ++h) {
            for (int l = 0; l < 32; ++l) {
                const uint8_t q1 = q[128 * h + l], q2 = q[128 * h + l + 32];
                const uint8_t q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
                ql[64 * h + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
                ql[64 * h + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
                qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
            }
        }
        memcpy(yb + 192, sc, 16);
        yb[208] = (uint8_t)(dh & 0xFF);
        yb[209] = (uint8_t)(dh >> 8);
    }
}

static inline int q6k_value(const uint8_t *yb, int e) {
    /* element e of a Q6_K block as a signed 6-bit value in [-32, 31] */
    const int h = e / 128, r = e % 128, m = r / 32, l = r % 32;
    const uint8_t *ql = yb + 64 * h, *qh = yb + 128 + 32 * h;
    const int lo = (m & 1) ? ql[l + 32] : ql[l];
    const int nib = (m >> 1) ? (lo >> 4) : (lo & 0xF);
    const int hi = (qh[l] >> (2 * m)) & 3;
    return (nib | (hi << 4)) - 32;
}

void or_dequantize_q6_K(const uint8_t *y, float *x, int64_t n) {
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *yb = y + b * OR_Q6K_BYTES;
        const float d = or_f16_to_f32((uint16_t)(yb[208] | (yb[209] << 8)));
        const int8_t *sc = (const int8_t *)(yb + 192);
        for (int e = 0; e < OR_QK_K; ++e) {
            x[b * OR_QK_K + e] = d * (float)sc[e / 16] * (float)q6k_value(yb, e);
        }
    }
}

void or_quantize_q8_1(const float *x, int8_t *q, float *d, float *s, int64_t n) {
    for (int64_t b = 0; b < n / 32; ++b) {
        float amax = 0.0f;
        for (int l = 0; l < 32; ++l) {
            const float a = fabsf(x[32 * b + l]);
            if (a > amax) amax = a;
        }
        const float db = amax / 127.0f;
        const float id = amax > 0.0f ? 1.0f / db : 0.0f;
        int sum = 0;
        for (int l = 0; l < 32; ++l) {
            const int v = (int)roundf(x[32 * b + l] * id);
            q[32 * b + l] = (int8_t)v;
            sum += v;
        }
        d[b] = db;
        s[b] = db * (float)sum;
    }
}

void or_q8_K_roundtrip(const float *x, float *out, int64_t n) {
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const float *xb = x + b * OR_QK_K;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < OR_QK_K; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                mx = xb[j];
            }
        }
        if (amax == 0.0f) {
            for (int j = 0; j < OR_QK_K; ++j) out[b * OR_QK_K + j] = 0.0f;
            continue;
        }
        const float iscale = -127.0f / mx;
        const float dq = 1.0f / iscale;
        for (int j = 0; j < OR_QK_K; ++j) {
            int v = (int)rintf(iscale * xb[j]);
            if (v > 127) v = 127;
            out[b * OR_QK_K + j] = dq * (float)v;
        }
    }
}

double or_dot_q4_K_q8_1(const uint8_t *row, const int8_t *q, const float *d,
                        const float *s, int64_t n) {
    double acc = 0.0;
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *yb = row + b * OR_Q4K_BYTES;
        const double dd = or_f16_to_f32((uint16_t)(yb[0] | (yb[1] << 8)));
        const double dm = or_f16_to_f32((uint16_t)(yb[2] | (yb[3] << 8)));
        const uint8_t *qs = yb + 16;
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4k_scale_min(j, yb + 4, &sc, &m);
            const int p = j / 2, hi = j & 1;
            int isum = 0;
            for (int l = 0; l < 32; ++l) {
                const int w = hi ? (qs[32 * p + l] >> 4) : (qs[32 * p + l] & 0xF);
                isum += w * q[b * OR_QK_K + 32 * j + l];
            }
            const int64_t qb = b * 8 + j;
            acc += dd * sc * (double)d[qb] * isum - dm * m * (double)s[qb];
        }
    }
    return acc;
}

double or_dot_q6_K_q8_1(const uint8_t *row, const int8_t *q, const float *d,
                        const float *s, int64_t n) {
    (void)s;
    double acc = 0.0;
    for (int64_t b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *yb = row + b * OR_Q6K_BYTES;
        const double dd = or_f16_to_f32((uint16_t)(yb[208] | (yb[209] << 8)));
        const int8_t *sc = (const int8_t *)(yb + 192);
        for (int g = 0; g < 16; ++g) {
            int isum = 0;
            for (int l = 0; l < 16; ++l) {
                const int e = 16 * g + l;
                isum += q6k_value(yb, e) * q[b * OR_QK_K + e];
            }
            acc += dd * sc[g] * (double)d[(b * OR_QK_K + 16 * g) / 32] * isum;
        }
    }
    return acc;
}

/* ------------------------------------------------------------------------ */
/* the GEMV kernels' fp32 order                                              */
/* ------------------------------------------------------------------------ */
/* These restate, operation for operation, the fp32 arithmetic of the GEMV
 * paths (per-pair, grouped and persistent decode kernels; their shared unit
 * helpers in moe_prefetch_b200/csrc/moe_dev.cuh): the integer sums of a unit
 * are exact, and every float rounding is written out with fmaf, so the row
 * values, and with them the SiLU*up activations and their Q8_1 blocks, are
 * the same bits.  The double versions above are the precision reference. */

/* One Q4_K unit: super-block yb, sub-block pair p (64 weights), with that
 * super-block's 256 activations qb and its 8 block d / s. */
static float q4k_unit_f32(const uint8_t *yb, int p, const int8_t *qb, const float *db,
                          const float *sb) {
    const uint8_t *qs = yb + 16 + 32 * p;
    int slo = 0, shi = 0;
    for (int l = 0; l < 32; ++l) {
        slo += (qs[l] & 0xF) * qb[64 * p + l];
        shi += (qs[l] >> 4) * qb[64 * p + 32 + l];
    }
    int sc0, m0, sc1, m1;
    q4k_scale_min(2 * p, yb + 4, &sc0, &m0);
    q4k_scale_min(2 * p + 1, yb + 4, &sc1, &m1);
    const float d = or_f16_to_f32((uint16_t)(yb[0] | (yb[1] << 8)));
    const float dmin = or_f16_to_f32((uint16_t)(yb[2] | (yb[3] << 8)));
    const float acc = fmaf((float)(sc1 * shi), db[2 * p + 1], (float)(sc0 * slo) * db[2 * p]);
    const float mm = fmaf((float)m1, sb[2 * p + 1], (float)m0 * sb[2 * p]);
    return fmaf(d, acc, -(dmin * mm));
}

/* The 32-lane xor butterfly (offsets 16, 8, 4, 2, 1, own value first) as lane
 * 0 sees it. */
static float lane_tree32(float *v) {
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < off; ++l) v[l] = v[l] + v[l + off];
    return v[0];
}

/* A Q4_K row: unit u = 4 b + p sits on lane u mod 32, each lane adds its
 * units to 0.0f in order, then the butterfly.  n % 256 == 0. */
float or_dot_q4_K_q8_1_f32(const uint8_t *row, const int8_t *q, const float *d,
                           const float *s, int64_t n) {
    float lane[32];
    for (int l = 0; l < 32; ++l) lane[l] = 0.0f;
    const int units = (int)(n / OR_QK_K) * 4;
    for (int u = 0; u < units; ++u) {
        const int b = u >> 2;
        lane[u & 31] = lane[u & 31] + q4k_unit_f32(row + (size_t)b * OR_Q4K_BYTES, u & 3,
                                                   q + (size_t)b * OR_QK_K, d + 8 * b, s + 8 * b);
    }
    return lane_tree32(lane);
}

/* Half h of a Q6_K super-block (128 weights) with its 128 activations qh and
 * their 4 block d: per quarter m the integer sums of the two 16-value scale
 * groups, accumulated as fma(scale * isum, d_m, acc) in (m, group) order,
 * times the block's d. */
static float q6k_half_f32(const uint8_t *yb, int h, const int8_t *qa, const float *dh) {
    const uint8_t *ql = yb + 64 * h, *qhb = yb + 128 + 32 * h;
    const int8_t *sc = (const int8_t *)(yb + 192 + 8 * h);
    float acc = 0.0f;
    for (int m = 0; m < 4; ++m) {
        int is[2] = {0, 0};
        for (int l = 0; l < 32; ++l) {
            const int lo = (ql[32 * (m & 1) + l] >> (4 * (m >> 1))) & 0xF;
            const int hb = (qhb[l] >> (2 * m)) & 3;
            is[l >> 4] += ((lo | (hb << 4)) - 32) * qa[32 * m + l];
        }
        acc = fmaf((float)(sc[2 * m] * is[0]), dh[m], acc);
        acc = fmaf((float)(sc[2 * m + 1] * is[1]), dh[m], acc);
    }
    const float d = or_f16_to_f32((uint16_t)(yb[208] | (yb[209] << 8)));
    return d * acc;
}

/* A Q6_K row: half-units u = 2 b + h on the lanes of a row group, summed by
 * the group tree ((v0+v1)+(v2+v3))+((v4+v5)+(v6+v7)), absent lanes +0.
 * n % 256 == 0, n <= 1024. */
float or_dot_q6_K_q8_1_f32(const uint8_t *row, const int8_t *q, const float *d,
                           const float *s, int64_t n) {
    (void)s;
    float v[8];
    for (int u = 0; u < 8; ++u) v[u] = 0.0f;
    const int units = (int)(n / OR_QK_K) * 2;
    for (int u = 0; u < units && u < 8; ++u) {
        const int b = u >> 1, h = u & 1;
        v[u] = q6k_half_f32(row + (size_t)b * OR_Q6K_BYTES, h, q + (size_t)b * OR_QK_K + 128 * h,
                            d + 8 * b + 4 * h);
    }
    return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

/* The kernels' combine: per output element an fp32 fma chain from 0 over the
 * pairs in rank order. */
void or_combine_f32(const float *w, const float *rows, int k, int n_embd, float *y) {
    for (int h = 0; h < n_embd; ++h) {
        float acc = 0.0f;
        for (int i = 0; i < k; ++i) acc = fmaf(w[i], rows[(size_t)i * n_embd + h], acc);
        y[h] = acc;
    }
}

/* ------------------------------------------------------------------------ */
/* router                                                                    */
/* ------------------------------------------------------------------------ */

/* Canonical order: 32 lanes; lane l owns columns 128*kk + 4*l + c; it keeps
 * four fma chains (c = 0..3) over kk, folds them as (a0+a1)+(a2+a3), and the
 * 32 lane sums are combined by an xor butterfly with offsets 16,8,4,2,1.  The
 * device router issues exactly this (one warp per logit). */
float or_router_dot(const float *w, const float *x, int n_embd) {
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int kk = 0; kk < n_embd / 128; ++kk) {
            const int j = 128 * kk + 4 * l;
            a0 = fmaf(w[j + 0], x[j + 0], a0);
            a1 = fmaf(w[j + 1], x[j + 1], a1);
            a2 = fmaf(w[j + 2], x[j + 2], a2);
            a3 = fmaf(w[j + 3], x[j + 3], a3);
        }
        lane[l] = (a0 + a1) + (a2 + a3);
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nl[32];
        for (int l = 0; l < 32; ++l) nl[l] = lane[l] + lane[l ^ off];
        memcpy(lane, nl, sizeof(lane));
    }
    return lane[0];
}

void or_router(const float *W, const float *x, int n_expert, int n_embd,
               const float *prior, int k, int32_t *ids, float *w,
               float *probs_out, float *logits_out) {
    float logits[256];
    for (int e = 0; e < n_expert; ++e) {
        logits[e] = or_router_dot(W + (size_t)e * n_embd, x, n_embd);
    }
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)n_expert);
    or_router_select(logits, n_expert, prior, k, ids, w, probs_out);
}

void or_router_fused(const float *Wt, const float *r, int n_expert, int n_embd,
                     const int32_t *h0, const int32_t *h1, int G, float eps,
                     const float *prior, int k, int32_t *ids, float *w, float *x_out,
                     float *logits_out) {
    float *P = (float *)malloc(sizeof(float) * (size_t)G * n_expert);
    float *S = (float *)malloc(sizeof(float) * (size_t)G);
    for (int c = 0; c < G; ++c) {
        for (int e = 0; e < n_expert; ++e) {
            float acc = 0.0f;
            for (int h = h0[c]; h < h1[c]; ++h) acc = fmaf(Wt[(size_t)h * n_expert + e], r[h], acc);
            P[(size_t)c * n_expert + e] = acc;
        }
        float s = 0.0f;
        for (int h = h0[c]; h < h1[c]; ++h) s = fmaf(r[h], r[h], s);
        S[c] = s;
    }
    /* fixed-point totals (the decode kernel's red.add accumulators); the
     * device converts with __float2ll_rn / __ll2float_rn, both round to
     * nearest even like llrintf and the int64 -> float cast here */
    float logits[256];
    for (int e = 0; e < n_expert; ++e) {
        long long tot = 0;
        for (int c = 0; c < G; ++c) {
            const float v = fminf(fmaxf(P[(size_t)c * n_expert + e], -1048576.0f), 1048576.0f);
            tot += llrintf(v * 4294967296.0f);
        }
        logits[e] = (float)tot * 2.3283064365386963e-10f;
    }
    long long stot = 0;
    for (int c = 0; c < G; ++c) stot += llrintf(fminf(S[c], 68719476736.0f) * 65536.0f);
    const float st = (float)stot * 1.52587890625e-05f;
    const float inv = 1.0f / sqrtf(st / (float)n_embd + eps);
    for (int e = 0; e < n_expert; ++e) logits[e] = logits[e] * inv;
    if (x_out) for (int h = 0; h < n_embd; ++h) x_out[h] = r[h] * inv;
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)n_expert);
    or_router_select(logits, n_expert, prior, k, ids, w, NULL);
    free(P);
    free(S);
}

void or_router_select(const float *logits, int n_expert, const float *prior, int k,
                      int32_t *ids, float *w, float *probs_out) {
    float ex[256], p[256], sel[256];
    float mx = logits[0];
    for (int e = 1; e < n_expert; ++e) {
        if (logits[e] > mx) mx = logits[e];
    }
    for (int e = 0; e < n_expert; ++e) {
        ex[e] = or_expf(logits[e] - mx);
    }
    /* lane l holds experts l, l+32, ... summed in that order, then butterfly */
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        /* a lane past n_expert (fewer than 32 experts) holds 0 */
        float sacc = l < n_expert ? ex[l] : 0.0f;
        for (int m = 1; l + 32 * m < n_expert; ++m) sacc = sacc + ex[l + 32 * m];
        lane[l] = sacc;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nl[32];
        for (int l = 0; l < 32; ++l) nl[l] = lane[l] + lane[l ^ off];
        memcpy(lane, nl, sizeof(lane));
    }
    const float sum = lane[0];
    for (int e = 0; e < n_expert; ++e) {
        p[e] = ex[e] / sum;
        sel[e] = prior ? p[e] + prior[e] : p[e];
    }
    uint8_t taken[256] = {0};
    for (int i = 0; i < k; ++i) {
        int best = -1;
        float bv = 0.0f;
        for (int e = 0; e < n_expert; ++e) {
            if (taken[e]) continue;
            if (best < 0 || sel[e] > bv) {   /* strict: ties keep the lower id */
                best = e;
                bv = sel[e];
            }
        }
        taken[best] = 1;
        ids[i] = best;
    }
    float ws = p[ids[0]];
    for (int i = 1; i < k; ++i) ws = ws + p[ids[i]];
    for (int i = 0; i < k; ++i) w[i] = p[ids[i]] / ws;
    if (probs_out) memcpy(probs_out, p, sizeof(float) * (size_t)n_expert);
}

/* ------------------------------------------------------------------------ */
/* expert rows / layer                                                       */
/* ------------------------------------------------------------------------ */

static inline size_t row_bytes(int type, int n) {
    return (size_t)(n / OR_QK_K) * (type == OR_QTYPE_Q6_K ? OR_Q6K_BYTES : OR_Q4K_BYTES);
}

void or_expert_row(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                   int down_type, int n_embd, int n_ff, const float *x,
                   float *out, float *act_out) {
    int8_t *xq = (int8_t *)malloc((size_t)n_embd);
    float *xd = (float *)malloc(sizeof(float) * (size_t)(n_embd / 32));
    float *xs = (float *)malloc(sizeof(float) * (size_t)(n_embd / 32));
    float *act = (float *)malloc(sizeof(float) * (size_t)n_ff);
    int8_t *aq = (int8_t *)malloc((size_t)n_ff);
    float *ad = (float *)malloc(sizeof(float) * (size_t)(n_ff / 32));
    float *as = (float *)malloc(sizeof(float) * (size_t)(n_ff / 32));
    or_quantize_q8_1(x, xq, xd, xs, n_embd);
    const size_t grb = row_bytes(OR_QTYPE_Q4_K, n_embd);
    for (int i = 0; i < n_ff; ++i) {
        const float g = or_dot_q4_K_q8_1_f32(gate + i * grb, xq, xd, xs, n_embd);
        const float u = or_dot_q4_K_q8_1_f32(up + i * grb, xq, xd, xs, n_embd);
        act[i] = or_silu_mul(g, u);
    }
    if (act_out) memcpy(act_out, act, sizeof(float) * (size_t)n_ff);
    or_quantize_q8_1(act, aq, ad, as, n_ff);
    const size_t drb = row_bytes(down_type, n_ff);
    for (int h = 0; h < n_embd; ++h) {
        out[h] = down_type == OR_QTYPE_Q6_K
            ? or_dot_q6_K_q8_1_f32(down + h * drb, aq, ad, as, n_ff)
            : or_dot_q4_K_q8_1_f32(down + h * drb, aq, ad, as, n_ff);
    }
    free(xq); free(xd); free(xs); free(act); free(aq); free(ad); free(as);
}

static void deq_row(int type, const uint8_t *row, float *out, int n) {
    if (type == OR_QTYPE_Q6_K) or_dequantize_q6_K(row, out, n);
    else or_dequantize_q4_K(row, out, n);
}

void or_expert_row_q8K(const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                       int down_type, int n_embd, int n_ff, const float *x,
                       float *out) {
    float *xr = (float *)malloc(sizeof(float) * (size_t)n_embd);
    float *wr = (float *)malloc(sizeof(float) * (size_t)(n_embd > n_ff ? n_embd : n_ff));
    float *act = (float *)malloc(sizeof(float) * (size_t)n_ff);
    float *ar = (float *)malloc(sizeof(float) * (size_t)n_ff);
    or_q8_K_roundtrip(x, xr, n_embd);
    const size_t grb = row_bytes(OR_QTYPE_Q4_K, n_embd);
    for (int i = 0; i < n_ff; ++i) {
        double g = 0.0, u = 0.0;
        deq_row(OR_QTYPE_Q4_K, gate + i * grb, wr, n_embd);
        for (int j = 0; j < n_embd; ++j) g += (double)wr[j] * xr[j];
        deq_row(OR_QTYPE_Q4_K, up + i * grb, wr, n_embd);
        for (int j = 0; j < n_embd; ++j) u += (double)wr[j] * xr[j];
        act[i] = or_silu_mul((float)g, (float)u);
    }
    or_q8_K_roundtrip(act, ar, n_ff);
    const size_t drb = row_bytes(down_type, n_ff);
    for (int h = 0; h < n_embd; ++h) {
        double acc = 0.0;
        deq_row(down_type, down + h * drb, wr, n_ff);
        for (int j = 0; j < n_ff; ++j) acc += (double)wr[j] * ar[j];
        out[h] = (float)acc;
    }
    free(xr); free(wr); free(act); free(ar);
}

typedef void (*or_row_fn)(const uint8_t *, const uint8_t *, const uint8_t *, int, int, int,
                          const float *, float *);

static void or_expert_row_q81(const uint8_t *g, const uint8_t *u, const uint8_t *d, int dt,
                              int ne, int nf, const float *x, float *out) {
    or_expert_row(g, u, d, dt, ne, nf, x, out, NULL);
}

static void or_layer_impl(or_row_fn fn, const float *x, int n_tok, int n_embd, int n_ff,
                          int n_expert, int k, const float *router_w, const float *prior,
                          const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                          int down_type, int32_t *ids_out, float *w_out, float *y_out,
                          int n_threads) {
    const size_t gexp = row_bytes(OR_QTYPE_Q4_K, n_embd) * (size_t)n_ff;
    const size_t dexp = row_bytes(down_type, n_ff) * (size_t)n_embd;
    for (int t = 0; t < n_tok; ++t) {
        or_router(router_w, x + (size_t)t * n_embd, n_expert, n_embd,
                  n_tok == 1 ? prior : NULL, k, ids_out + (size_t)t * k,
                  w_out + (size_t)t * k, NULL, NULL);
    }
    float *rows = (float *)malloc(sizeof(float) * (size_t)n_tok * k * n_embd);
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads > 0 ? n_threads : 1) schedule(dynamic, 1)
#endif
    for (int tk = 0; tk < n_tok * k; ++tk) {
        const int t = tk / k;
        const int32_t e = ids_out[tk];
        fn(gate + e * gexp, up + e * gexp, down + e * dexp, down_type, n_embd, n_ff,
           x + (size_t)t * n_embd, rows + (size_t)tk * n_embd);
    }
    (void)n_threads;
    for (int t = 0; t < n_tok; ++t) {
        if (fn == or_expert_row_q81) {   /* the GPU paths' combine */
            or_combine_f32(w_out + (size_t)t * k, rows + (size_t)t * k * n_embd, k, n_embd,
                           y_out + (size_t)t * n_embd);
            continue;
        }
        for (int h = 0; h < n_embd; ++h) {
            double acc = 0.0;
            for (int i = 0; i < k; ++i) {
                acc += (double)w_out[t * k + i] * rows[((size_t)t * k + i) * n_embd + h];
            }
            y_out[(size_t)t * n_embd + h] = (float)acc;
        }
    }
    free(rows);
}

void or_moe_experts(const float *x, int n_tok, int n_embd, int n_ff, int k,
                    const int32_t *ids, const float *w, const uint8_t *gate,
                    const uint8_t *up, const uint8_t *down, int down_type, float *y_out,
                    int n_threads) {
    const size_t gexp = row_bytes(OR_QTYPE_Q4_K, n_embd) * (size_t)n_ff;
    const size_t dexp = row_bytes(down_type, n_ff) * (size_t)n_embd;
    float *rows = (float *)malloc(sizeof(float) * (size_t)n_tok * k * n_embd);
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads > 0 ? n_threads : 1) schedule(dynamic, 1)
#endif
    for (int tk = 0; tk < n_tok * k; ++tk) {
        const int t = tk / k;
        const int32_t e = ids[tk];
        or_expert_row(gate + e * gexp, up + e * gexp, down + e * dexp, down_type, n_embd, n_ff,
                      x + (size_t)t * n_embd, rows + (size_t)tk * n_embd, NULL);
    }
    (void)n_threads;
    for (int t = 0; t < n_tok; ++t)
        or_combine_f32(w + (size_t)t * k, rows + (size_t)t * k * n_embd, k, n_embd,
                       y_out + (size_t)t * n_embd);
    free(rows);
}

/* The expert half with unquantised activations: the fp32-accumulated
 * reference of a GEMM path.  Weights are dequantised exactly (ggml block
 * layout, as or_dequantize_*), x is used as given, every dot accumulates in
 * double, act = silu(g) * u in double, and y = sum_i w_i * row_i in double.
 * Follows the op order of ggml_cpu_moe_rows (patches/0008:186-251: up, gate,
 * swiglu(gate, up), down) without its Q8_K activation rounding.  Each expert
 * that is routed to is dequantised once. */
void or_moe_experts_f32(const float *x, int n_tok, int n_embd, int n_ff, int n_expert, int k,
                        const int32_t *ids, const float *w, const uint8_t *gate,
                        const uint8_t *up, const uint8_t *down, int down_type, float *y_out,
                        int n_threads) {
    const size_t grb = row_bytes(OR_QTYPE_Q4_K, n_embd), drb = row_bytes(down_type, n_ff);
    const size_t gexp = grb * (size_t)n_ff, dexp = drb * (size_t)n_embd;
    double *rows = (double *)calloc((size_t)n_tok * k * n_embd, sizeof(double));
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads > 0 ? n_threads : 1) schedule(dynamic, 1)
#endif
    for (int e = 0; e < n_expert; ++e) {
        int used = 0;
        for (int tk = 0; tk < n_tok * k && !used; ++tk) used = ids[tk] == e;
        if (!used) continue;
        float *wg = (float *)malloc(sizeof(float) * (size_t)n_ff * n_embd);
        float *wu = (float *)malloc(sizeof(float) * (size_t)n_ff * n_embd);
        float *wd = (float *)malloc(sizeof(float) * (size_t)n_embd * n_ff);
        double *act = (double *)malloc(sizeof(double) * (size_t)n_ff);
        for (int i = 0; i < n_ff; ++i) {
            or_dequantize_q4_K(gate + e * gexp + i * grb, wg + (size_t)i * n_embd, n_embd);
            or_dequantize_q4_K(up + e * gexp + i * grb, wu + (size_t)i * n_embd, n_embd);
        }
        for (int h = 0; h < n_embd; ++h) deq_row(down_type, down + e * dexp + h * drb,
                                                 wd + (size_t)h * n_ff, n_ff);
        for (int tk = 0; tk < n_tok * k; ++tk) {
            if (ids[tk] != e) continue;
            const float *xt = x + (size_t)(tk / k) * n_embd;
            for (int i = 0; i < n_ff; ++i) {
                double g = 0.0, u = 0.0;
                const float *rg = wg + (size_t)i * n_embd, *ru = wu + (size_t)i * n_embd;
                for (int j = 0; j < n_embd; ++j) {
                    g += (double)rg[j] * xt[j];
                    u += (double)ru[j] * xt[j];
                }
                act[i] = g / (1.0 + exp(-g)) * u;
            }
            double *out = rows + (size_t)tk * n_embd;
            for (int h = 0; h < n_embd; ++h) {
                double acc = 0.0;
                const float *rd = wd + (size_t)h * n_ff;
                for (int i = 0; i < n_ff; ++i) acc += (double)rd[i] * act[i];
                out[h] = acc;
            }
        }
        free(wg); free(wu); free(wd); free(act);
    }
    for (int t = 0; t < n_tok; ++t)
        for (int h = 0; h < n_embd; ++h) {
            double acc = 0.0;
            for (int i = 0; i < k; ++i) acc += (double)w[t * k + i] * rows[((size_t)t * k + i) * n_embd + h];
            y_out[(size_t)t * n_embd + h] = (float)acc;
        }
    free(rows);
}

void or_moe_layer(const float *x, int n_tok, int n_embd, int n_ff, int n_expert,
                  int k, const float *router_w, const float *prior,
                  const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                  int down_type, int32_t *ids_out, float *w_out, float *y_out,
                  int n_threads) {
    or_layer_impl(or_expert_row_q81, x, n_tok, n_embd, n_ff, n_expert, k, router_w, prior,
                  gate, up, down, down_type, ids_out, w_out, y_out, n_threads);
}

void or_moe_layer_q8K(const float *x, int n_tok, int n_embd, int n_ff, int n_expert,
                      int k, const float *router_w, const float *prior,
                      const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                      int down_type, int32_t *ids_out, float *w_out, float *y_out,
                      int n_threads) {
    or_layer_impl(or_expert_row_q8K, x, n_tok, n_embd, n_ff, n_expert, k, router_w, prior,
                  gate, up, down, down_type, ids_out, w_out, y_out, n_threads);
}

/* ---- the timed CPU baseline: integer dots, Q8_K activations, ggml op order -- */

typedef struct {
    float d;
    int8_t q[OR_QK_K];
    int16_t bsums[16];
} or_q8K_block;

static void q8K_quantize(const float *x, or_q8K_block *y, int n) {
    for (int b = 0; b < n / OR_QK_K; ++b) {
        const float *xb = x + b * OR_QK_K;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < OR_QK_K; ++j) {
            const float a = fabsf(xb[j]);
            if (a > amax) { amax = a; mx = xb[j]; }
        }
        if (amax == 0.0f) {
            memset(&y[b], 0, sizeof(y[b]));
            continue;
        }
        const float iscale = -127.0f / mx;
        for (int j = 0; j < OR_QK_K; ++j) {
            int v = (int)rintf(iscale * xb[j]);
            y[b].q[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int l = 0; l < 16; ++l) s += y[b].q[16 * g + l];
            y[b].bsums[g] = (int16_t)s;
        }
        y[b].d = 1.0f / iscale;
    }
}

static float vec_dot_q4K_q8K(const uint8_t *row, const or_q8K_block *y, int n) {
    float sumf = 0.0f;
    for (int b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *xb = row + b * OR_Q4K_BYTES;
        const float d = y[b].d * or_f16_to_f32((uint16_t)(xb[0] | (xb[1] << 8)));
        const float dmin = y[b].d * or_f16_to_f32((uint16_t)(xb[2] | (xb[3] << 8)));
        const uint8_t *qs = xb + 16;
        const int8_t *q8 = y[b].q;
        int sumi = 0, summs = 0;
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            q4k_scale_min(j, xb + 4, &sc, &m);
            const int p = j / 2, sh = (j & 1) * 4;
            int isum = 0;
            for (int l = 0; l < 32; ++l) isum += ((qs[32 * p + l] >> sh) & 0xF) * q8[32 * j + l];
            sumi += sc * isum;
            summs += m * (y[b].bsums[2 * j] + y[b].bsums[2 * j + 1]);
        }
        sumf += d * (float)sumi - dmin * (float)summs;
    }
    return sumf;
}

static float vec_dot_q6K_q8K(const uint8_t *row, const or_q8K_block *y, int n) {
    float sumf = 0.0f;
    for (int b = 0; b < n / OR_QK_K; ++b) {
        const uint8_t *xb = row + b * OR_Q6K_BYTES;
        const float d = y[b].d * or_f16_to_f32((uint16_t)(xb[208] | (xb[209] << 8)));
        const int8_t *sc = (const int8_t *)(xb + 192);
        const int8_t *q8 = y[b].q;
        int sumi = 0;
        for (int h = 0; h < 2; ++h) {
            const uint8_t *ql = xb + 64 * h, *qh = xb + 128 + 32 * h;
            for (int m = 0; m < 4; ++m) {
                int i0 = 0, i1 = 0;
                for (int l = 0; l < 32; ++l) {
                    const int lo = (m & 1) ? ql[l + 32] : ql[l];
                    const int nib = (m >> 1) ? (lo >> 4) : (lo & 0xF);
                    const int v = (nib | (((qh[l] >> (2 * m)) & 3) << 4)) - 32;
                    if (l < 16) i0 += v * q8[128 * h + 32 * m + l];
                    else i1 += v * q8[128 * h + 32 * m + l];
                }
                sumi += sc[8 * h + 2 * m] * i0 + sc[8 * h + 2 * m + 1] * i1;
            }
        }
        sumf += d * (float)sumi;
    }
    return sumf;
}

void or_moe_layer_cpu_fast(const float *x, int n_embd, int n_ff, int n_expert, int k,
                           const float *router_w, const float *prior,
                           const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                           int down_type, int32_t *ids_out, float *w_out,
                           float *y_out, int n_threads) {
    const size_t grb = row_bytes(OR_QTYPE_Q4_K, n_embd);
    const size_t drb = row_bytes(down_type, n_ff);
    const size_t gexp = grb * (size_t)n_ff, dexp = drb * (size_t)n_embd;
    or_router(router_w, x, n_expert, n_embd, prior, k, ids_out, w_out, NULL, NULL);
    or_q8K_block *xq = (or_q8K_block *)malloc(sizeof(or_q8K_block) * (size_t)(n_embd / OR_QK_K));
    q8K_quantize(x, xq, n_embd);
    float *up_r = (float *)malloc(sizeof(float) * (size_t)k * n_ff);
    float *gate_r = (float *)malloc(sizeof(float) * (size_t)k * n_ff);
    float *act = (float *)malloc(sizeof(float) * (size_t)k * n_ff);
    or_q8K_block *aq = (or_q8K_block *)malloc(sizeof(or_q8K_block) * (size_t)k * (n_ff / OR_QK_K));
    float *rows = (float *)malloc(sizeof(float) * (size_t)k * n_embd);
    const int nt = n_threads > 0 ? n_threads : 1;
    (void)nt;
    /* ggml_cpu_moe_rows order: up, gate, swiglu, down (patches/0008:232-250) */
#ifdef _OPENMP
#pragma omp parallel num_threads(nt)
#endif
    {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int r = 0; r < k * n_ff; ++r) {
            const int i = r / n_ff, row = r % n_ff;
            up_r[r] = vec_dot_q4K_q8K(up + ids_out[i] * gexp + row * grb, xq, n_embd);
        }
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int r = 0; r < k * n_ff; ++r) {
            const int i = r / n_ff, row = r % n_ff;
            gate_r[r] = vec_dot_q4K_q8K(gate + ids_out[i] * gexp + row * grb, xq, n_embd);
        }
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int r = 0; r < k * n_ff; ++r) {
            act[r] = or_silu_mul(gate_r[r], up_r[r]);
        }
#ifdef _OPENMP
#pragma omp single
#endif
        for (int i = 0; i < k; ++i) q8K_quantize(act + i * n_ff, aq + i * (n_ff / OR_QK_K), n_ff);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int r = 0; r < k * n_embd; ++r) {
            const int i = r / n_embd, h = r % n_embd;
            const uint8_t *drow = down + ids_out[i] * dexp + h * drb;
            rows[r] = down_type == OR_QTYPE_Q6_K
                ? vec_dot_q6K_q8K(drow, aq + i * (n_ff / OR_QK_K), n_ff)
                : vec_dot_q4K_q8K(drow, aq + i * (n_ff / OR_QK_K), n_ff);
        }
    }
    for (int h = 0; h < n_embd; ++h) {
        float acc = 0.0f;
        for (int i = 0; i < k; ++i) acc += w_out[i] * rows[i * n_embd + h];
        y_out[h] = acc;
    }
    free(xq); free(up_r); free(gate_r); free(act); free(aq); free(rows);
}

/* ------------------------------------------------------------------------ */
/* slot-table state machine                                                  */
/* ------------------------------------------------------------------------ */

typedef struct { int32_t layer, expert, slot, spec; } or_job;

typedef struct {
    int32_t ns;
    int32_t *slot_expert, *expert_slot;
    uint64_t *last_use, *protect;
    uint8_t *in_flight;
    int32_t *free_slots;
    int32_t n_free;
    int32_t *pending;
    int32_t n_pending;
    int32_t *cur_ids;
    int32_t n_cur;
    int32_t *prev_ids;     /* cur_ids one token earlier (the evictor's features) */
    int32_t n_prev;
    uint64_t n_hit, n_miss;
    float *heat;
    uint64_t *miss_last, *miss_prev;
    uint32_t *use_count;
    int32_t *tbl;          /* what the device table holds */
    float *prior;          /* what the device prior holds */
    int32_t *tbl_mirror;   /* batched mode: host mirror   */
    float *prior_mirror;
    int dirty;
} or_layer;

/* LLAMA_MOE_EVICTOR: an MOEP model scoring which resident expert is wanted
 * again soon (patches/0006:521-537 load, :402-426 evict_scores) */
typedef struct {
    int32_t n_model, feat_dim;
    int32_t off[4];        /* prev, cur, below, self_prev: row offsets, -1 absent */
    int32_t *index_of;     /* [n_layers] model slot or -1 */
    float *w, *bias, *prior;
    float *scores;         /* [n_expert] scratch */
} or_evictor;

struct or_cache {
    or_cache_cfg cfg;
    or_layer *L;
    or_evictor *ev;
    uint64_t clock, n_steps, n_uploads, n_scheduled, n_copied, n_published;
    uint64_t n_admit_ok, n_admit_denied, n_table_flushes;
    or_job *todo;
    int n_todo, cap_todo;
    or_predict_fn pred;
    void *pred_ud;
};

#define OR_U64_MAX 0xFFFFFFFFFFFFFFFFull

or_cache *or_cache_create(const or_cache_cfg *cfg) {
    or_cache *c = (or_cache *)calloc(1, sizeof(or_cache));
    c->cfg = *cfg;
    c->cfg.slot_profile = NULL;
    if (c->cfg.max_inserts <= 0) c->cfg.max_inserts = 2;
    if (c->cfg.freeze) c->cfg.max_inserts = 0;
    const int E = cfg->n_expert;
    c->L = (or_layer *)calloc((size_t)cfg->n_layers, sizeof(or_layer));
    for (int l = 0; l < cfg->n_layers; ++l) {
        or_layer *L = &c->L[l];
        const int ns = cfg->slot_profile && cfg->slot_profile[l] > 0 ? cfg->slot_profile[l] : cfg->n_slots;
        L->ns = ns;
        L->slot_expert = (int32_t *)malloc(sizeof(int32_t) * (size_t)ns);
        L->expert_slot = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
        L->last_use = (uint64_t *)calloc((size_t)ns, sizeof(uint64_t));
        L->protect = (uint64_t *)calloc((size_t)ns, sizeof(uint64_t));
        L->in_flight = (uint8_t *)calloc((size_t)ns, 1);
        L->free_slots = (int32_t *)malloc(sizeof(int32_t) * (size_t)ns);
        L->pending = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
        L->cur_ids = (int32_t *)malloc(sizeof(int32_t) * 4096);
        L->prev_ids = (int32_t *)malloc(sizeof(int32_t) * 4096);
        L->tbl = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
        L->prior = (float *)calloc((size_t)E, sizeof(float));
        L->tbl_mirror = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
        L->prior_mirror = (float *)calloc((size_t)E, sizeof(float));
        for (int s = 0; s < ns; ++s) {
            L->slot_expert[s] = -1;
            L->free_slots[s] = ns - 1 - s;
        }
        L->n_free = ns;
        for (int e = 0; e < E; ++e) {
            L->expert_slot[e] = -1;
            L->tbl[e] = ns;
            L->tbl_mirror[e] = ns;
        }
        if (cfg->admit_mode == 1) L->heat = (float *)calloc((size_t)E, sizeof(float));
        if (cfg->admit_mode == 2) {
            L->miss_last = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)E);
            L->miss_prev = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)E);
            for (int e = 0; e < E; ++e) L->miss_last[e] = L->miss_prev[e] = OR_U64_MAX;
        }
        if (cfg->use_heat_counts) L->use_count = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
    }
    c->cap_todo = 1024;
    c->todo = (or_job *)malloc(sizeof(or_job) * (size_t)c->cap_todo);
    return c;
}

void or_cache_destroy(or_cache *c) {
    if (!c) return;
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        or_layer *L = &c->L[l];
        free(L->slot_expert); free(L->expert_slot); free(L->last_use); free(L->protect);
        free(L->in_flight); free(L->free_slots); free(L->pending); free(L->cur_ids); free(L->prev_ids);
        free(L->tbl); free(L->prior); free(L->tbl_mirror); free(L->prior_mirror);
        free(L->heat); free(L->miss_last); free(L->miss_prev); free(L->use_count);
    }
    free(c->L);
    free(c->todo);
    if (c->ev) {
        free(c->ev->index_of); free(c->ev->w); free(c->ev->bias); free(c->ev->prior); free(c->ev->scores);
        free(c->ev);
    }
    free(c);
}

/* moe_predictor::score (cpp/moe-predictor.cpp:165-223), the evictor's and the
 * predictor's score of one layer: the bias, plus the weight rows the ids of
 * each block select (block order prev, cur, below, self_prev; ids in order;
 * out-of-range ids skipped; a repeated id adds twice), z-scored with the mean
 * and variance as running fp32 sums, then the repeat prior on the prev ids.
 * No fused multiply-adds (-ffp-contract=off). */
void or_evict_score(const float *W, const float *bias, float prior, const int32_t off[4], int E,
                    const int32_t *prev, int n_prev, const int32_t *cur, int n_cur,
                    const int32_t *below, int n_below, const int32_t *self_prev, int n_self_prev,
                    float *out) {
    const int32_t *ids[4] = {prev, cur, below, self_prev};
    const int n[4] = {n_prev, n_cur, n_below, n_self_prev};
    for (int j = 0; j < E; ++j) out[j] = bias[j];
    for (int g = 0; g < 4; ++g) {
        if (off[g] < 0 || !ids[g]) continue;
        for (int i = 0; i < n[g]; ++i) {
            const int32_t e = ids[g][i];
            if (e < 0 || e >= E) continue;
            const float *row = W + (size_t)(off[g] + e) * (size_t)E;
            for (int j = 0; j < E; ++j) out[j] += row[j];
        }
    }
    float mu = 0.0f;
    for (int j = 0; j < E; ++j) mu += out[j];
    mu /= (float)E;
    float var = 0.0f;
    for (int j = 0; j < E; ++j) {
        const float d = out[j] - mu;
        var += d * d;
    }
    const float sd = sqrtf(var / (float)E) + 1e-9f;
    for (int j = 0; j < E; ++j) out[j] = (out[j] - mu) / sd;
    if (prior != 0.0f && prev)
        for (int i = 0; i < n_prev; ++i) {
            const int32_t e = prev[i];
            if (e >= 0 && e < E) out[e] += prior;
        }
}

int or_cache_set_evictor(or_cache *c, int n_model, const int32_t *layer_of, int feat_dim,
                         const int32_t off[4], const float *w, const float *bias, const float *prior) {
    const int E = c->cfg.n_expert;
    if (n_model <= 0 || feat_dim <= 0) return -1;
    for (int g = 0; g < 4; ++g)
        if (off[g] >= 0 && off[g] + E > feat_dim) return -1;
    or_evictor *ev = (or_evictor *)calloc(1, sizeof(or_evictor));
    ev->n_model = n_model;
    ev->feat_dim = feat_dim;
    for (int g = 0; g < 4; ++g) ev->off[g] = off[g];
    ev->index_of = (int32_t *)malloc(sizeof(int32_t) * (size_t)c->cfg.n_layers);
    for (int l = 0; l < c->cfg.n_layers; ++l) ev->index_of[l] = -1;
    for (int m = 0; m < n_model; ++m)
        if (layer_of[m] >= 0 && layer_of[m] < c->cfg.n_layers) ev->index_of[layer_of[m]] = m;
    const size_t nw = (size_t)n_model * (size_t)feat_dim * (size_t)E;
    ev->w = (float *)malloc(sizeof(float) * nw);
    memcpy(ev->w, w, sizeof(float) * nw);
    ev->bias = (float *)malloc(sizeof(float) * (size_t)n_model * (size_t)E);
    memcpy(ev->bias, bias, sizeof(float) * (size_t)n_model * (size_t)E);
    ev->prior = (float *)malloc(sizeof(float) * (size_t)n_model);
    memcpy(ev->prior, prior, sizeof(float) * (size_t)n_model);
    ev->scores = (float *)malloc(sizeof(float) * (size_t)E);
    c->ev = ev;
    return 0;
}

/* evict_scores (patches/0006:402-426) for layer li: false when the layer has
 * no model.  Inputs: prev = the next layer's previous-token ids, cur = this
 * layer's ids, below = the previous layer's ids, self_prev = this layer's
 * previous-token ids. */
static int evict_scores(or_cache *c, int li) {
    or_evictor *ev = c->ev;
    if (!ev || ev->index_of[li] < 0) return 0;
    const int E = c->cfg.n_expert, m = ev->index_of[li];
    const or_layer *L = &c->L[li];
    const or_layer *A = li + 1 < c->cfg.n_layers ? &c->L[li + 1] : NULL;
    const or_layer *B = li > 0 ? &c->L[li - 1] : NULL;
    or_evict_score(ev->w + (size_t)m * ev->feat_dim * E, ev->bias + (size_t)m * E, ev->prior[m], ev->off, E,
                   A ? A->prev_ids : NULL, A ? A->n_prev : 0, L->cur_ids, L->n_cur,
                   B ? B->cur_ids : NULL, B ? B->n_cur : 0, L->prev_ids, L->n_prev, ev->scores);
    return 1;
}

void or_cache_set_predictor(or_cache *c, or_predict_fn fn, void *ud) {
    c->pred = fn;
    c->pred_ud = ud;
}

/* set_table_entry (patches/0007:326-348): the prior entry moves with it */
static void set_table_entry(or_cache *c, or_layer *L, int32_t expert, int32_t v) {
    const float p = v == L->ns ? 0.0f : c->cfg.cache_prior;
    if (c->cfg.batch_tables) {
        L->tbl_mirror[expert] = v;
        L->prior_mirror[expert] = p;
        L->dirty = 1;
        return;
    }
    L->tbl[expert] = v;
    L->prior[expert] = p;
}

/* flush_tables (patches/0007:350-396) */
static void flush_tables(or_cache *c) {
    if (!c->cfg.batch_tables) return;
    int any = 0;
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        or_layer *L = &c->L[l];
        if (!L->dirty) continue;
        memcpy(L->tbl, L->tbl_mirror, sizeof(int32_t) * (size_t)c->cfg.n_expert);
        memcpy(L->prior, L->prior_mirror, sizeof(float) * (size_t)c->cfg.n_expert);
        L->dirty = 0;
        any = 1;
    }
    if (any) c->n_table_flushes++;
}

/* lru_resident (patches/0007:398-412) */
static int32_t lru_resident(const or_layer *L) {
    int32_t victim = -1;
    uint64_t best = OR_U64_MAX;
    for (int s = 0; s < L->ns; ++s) {
        if (L->in_flight[s] || L->slot_expert[s] < 0) continue;
        if (L->last_use[s] < best) {
            best = L->last_use[s];
            victim = L->slot_expert[s];
        }
    }
    return victim;
}

/* admit_ok (patches/0007:414-429) */
static int admit_ok(or_cache *c, const or_layer *L, int32_t id, int32_t victim) {
    if (c->cfg.admit_mode == 0 || victim < 0) return 1;
    int ok = 1;
    if (c->cfg.admit_mode == 1) {
        const float bar = L->heat[victim] * 1.25f;
        ok = L->heat[id] > bar + c->cfg.admit_floor;
    } else if (c->cfg.admit_mode == 2) {
        ok = L->miss_prev[id] != OR_U64_MAX &&
             L->miss_last[id] - L->miss_prev[id] < (uint64_t)c->cfg.admit_window;
    }
    if (ok) c->n_admit_ok++; else c->n_admit_denied++;
    return ok;
}

static void push_job(or_cache *c, int32_t layer, int32_t expert, int32_t slot, int32_t spec) {
    if (c->n_todo == c->cap_todo) {
        c->cap_todo *= 2;
        c->todo = (or_job *)realloc(c->todo, sizeof(or_job) * (size_t)c->cap_todo);
    }
    or_job j = {layer, expert, slot, spec};
    c->todo[c->n_todo++] = j;
}

/* issue_uploads (patches/0006:251-293, 0007:230-246, 0008:498-500) */
static int issue_uploads(or_cache *c, int li, const int32_t *ids, int n, int budget,
                         int min_keep, int spec) {
    if (c->cfg.freeze) return 0;
    or_layer *L = &c->L[li];
    int issued = 0;
    for (int i = 0; i < n && issued < budget; ++i) {
        const int32_t id = ids[i];
        if (id < 0 || id >= c->cfg.n_expert) continue;
        if (L->expert_slot[id] >= 0) continue;
        if (L->n_free <= min_keep) break;
        int dup = 0;
        for (int t = 0; t < c->n_todo; ++t) {
            if (c->todo[t].layer == li && c->todo[t].expert == id) { dup = 1; break; }
        }
        if (dup) continue;
        const int32_t slot = L->free_slots[--L->n_free];
        L->in_flight[slot] = 1;
        push_job(c, li, id, slot, spec);
        c->n_uploads++;
        c->n_scheduled++;
        issued++;
    }
    return issued;
}

void or_cache_observe(or_cache *c, int layer, const int32_t *ids, int n_tok, int n_ids,
                      int force) {
    if (n_tok != 1 && !force) return;
    or_layer *L = &c->L[layer];
    const int E = c->cfg.n_expert;
    int32_t observed[4096];
    int n_obs = 0;
    for (int t = 0; t < n_tok; ++t) {
        for (int i = 0; i < n_ids; ++i) {
            const int32_t id = ids[t * n_ids + i];
            if (id < 0 || id >= E) continue;
            if (n_obs < 4096) observed[n_obs++] = id;
            if (L->heat) L->heat[id] += 1.0f;
            if (L->use_count) L->use_count[id]++;
            const int32_t slot = L->expert_slot[id];
            if (slot >= 0) {
                L->n_hit++;
                L->last_use[slot] = ++c->clock;
            } else {
                L->n_miss++;
                if (L->miss_last && L->miss_last[id] != c->n_steps) {
                    L->miss_prev[id] = L->miss_last[id];
                    L->miss_last[id] = c->n_steps;
                }
                int dup = 0;
                for (int p = 0; p < L->n_pending; ++p) {
                    if (L->pending[p] == id) { dup = 1; break; }
                }
                if (!dup) L->pending[L->n_pending++] = id;
            }
        }
    }
    if (c->cfg.early_issue) {
        const int have_pred = c->cfg.have_pred && c->pred;
        const int32_t pool_target = c->cfg.freeze ? 0
            : c->cfg.max_inserts + (have_pred ? c->cfg.predict_top : 0);
        const int32_t next_victim = c->cfg.admit_mode == 0 ? -1
            : (L->n_free > pool_target ? -1 : lru_resident(L));
        if (c->cfg.admit_mode == 0) {
            issue_uploads(c, layer, L->pending, L->n_pending, c->cfg.max_inserts, 0, 0);
        } else {
            int32_t admitted[512];
            int na = 0;
            for (int p = 0; p < L->n_pending; ++p) {
                const int32_t id = L->pending[p];
                if (L->expert_slot[id] < 0 && admit_ok(c, L, id, next_victim)) admitted[na++] = id;
            }
            issue_uploads(c, layer, admitted, na, c->cfg.max_inserts, 0, 0);
        }
        if (have_pred && layer + 1 < c->cfg.n_layers) {
            or_layer *N = &c->L[layer + 1];
            int32_t top[64];
            int kk = c->cfg.predict_top < 64 ? c->cfg.predict_top : 64;
            int n_top = c->pred(c->pred_ud, layer, observed, n_obs, N->cur_ids, N->n_cur, top, kk);
            if (n_top < 0) n_top = 0;
            int n_issue = n_top;
            if (c->cfg.admit_mode == 1) {
                const int32_t nv = N->n_free > pool_target ? -1 : lru_resident(N);
                n_issue = 0;
                for (int i = 0; i < n_top; ++i) {
                    const int32_t id = top[i];
                    if (id >= 0 && id < E && N->expert_slot[id] < 0 && admit_ok(c, N, id, nv)) {
                        top[n_issue++] = id;
                    }
                }
            }
            issue_uploads(c, layer + 1, top, n_issue, c->cfg.predict_top, c->cfg.max_inserts, 1);
        }
    }
    memcpy(L->cur_ids, observed, sizeof(int32_t) * (size_t)n_obs);
    L->n_cur = n_obs;
}

static int job_cmp(const void *a, const void *b) {
    const or_job *x = (const or_job *)a, *y = (const or_job *)b;
    if (x->layer != y->layer) return x->layer < y->layer ? -1 : 1;
    return x->slot < y->slot ? -1 : x->slot > y->slot ? 1 : 0;
}

void or_cache_step(or_cache *c) {
    /* deterministic publication (patches/0008:613-627): every scheduled copy
     * is complete; publish in (layer, slot) order */
    or_job *done = c->todo;
    const int n_done = c->n_todo;
    c->n_copied += (uint64_t)n_done;
    qsort(done, (size_t)n_done, sizeof(or_job), job_cmp);
    for (int i = 0; i < n_done; ++i) {
        const or_job *j = &done[i];
        or_layer *L = &c->L[j->layer];
        L->slot_expert[j->slot] = j->expert;
        L->expert_slot[j->expert] = j->slot;
        if (j->spec && c->cfg.spec_probation) {
            L->last_use[j->slot] = 1;
            L->protect[j->slot] = c->n_steps + 1;
        } else {
            L->last_use[j->slot] = ++c->clock;
        }
        L->in_flight[j->slot] = 0;
        set_table_entry(c, L, j->expert, j->slot);
        c->n_published++;
    }
    c->n_todo = 0;
    c->n_steps++;

    for (int li = 0; li < c->cfg.n_layers; ++li) {
        or_layer *L = &c->L[li];
        if (!c->cfg.early_issue) {
            if (L->n_pending == 0) continue;
            int budget = c->cfg.max_inserts;
            /* the evictor on this path too (patches/0006:790-830, 0007:680-700):
             * victim = an empty slot, else the lowest score (recency breaking
             * ties), else LRU */
            const int use_model = evict_scores(c, li);
            const float *esc = use_model ? c->ev->scores : NULL;
            for (int it = L->n_pending - 1; it >= 0 && budget > 0; --it) {
                const int32_t id = L->pending[it];
                if (L->expert_slot[id] >= 0) {
                    --budget;
                    continue;
                }
                int32_t slot = -1;
                uint64_t best = OR_U64_MAX;
                float best_score = 3.4e38f;
                for (int s = 0; s < L->ns; ++s) {
                    if (L->in_flight[s]) continue;
                    if (L->slot_expert[s] < 0) { slot = s; break; }
                    if (L->protect[s] >= c->n_steps) continue;
                    if (use_model) {
                        const float sc = esc[L->slot_expert[s]];
                        if (sc < best_score || (sc == best_score && L->last_use[s] < best)) {
                            best_score = sc; best = L->last_use[s]; slot = s;
                        }
                    } else if (L->last_use[s] < best) {
                        best = L->last_use[s]; slot = s;
                    }
                }
                if (slot < 0) break;
                const int32_t victim = L->slot_expert[slot];
                if (!admit_ok(c, L, id, victim)) continue;
                --budget;
                if (victim >= 0) {
                    L->expert_slot[victim] = -1;
                    L->slot_expert[slot] = -1;
                    set_table_entry(c, L, victim, L->ns);
                }
                L->in_flight[slot] = 1;
                push_job(c, li, id, slot, 0);
                c->n_scheduled++;
            }
            L->n_pending = 0;
            continue;
        }
        /* early-issue path: top the free pool back up (patches/0006:843-913) */
        L->n_pending = 0;
        const int have_pred = c->cfg.have_pred && c->pred;
        const int32_t pool_target = c->cfg.freeze ? 0
            : c->cfg.max_inserts + (have_pred ? c->cfg.predict_top : 0);
        const int use_model = evict_scores(c, li);
        const float *esc = use_model ? c->ev->scores : NULL;
        while (L->n_free < pool_target) {
            int32_t slot = -1;
            uint64_t best = OR_U64_MAX;
            float best_score = 3.4e38f;
            for (int s = 0; s < L->ns; ++s) {
                if (L->in_flight[s] || L->slot_expert[s] < 0) continue;
                if (L->protect[s] >= c->n_steps) continue;
                if (use_model) {
                    /* lowest predicted chance of being wanted again; recency
                     * breaks ties (patches/0006:871-889) */
                    const float sc = esc[L->slot_expert[s]];
                    if (sc < best_score || (sc == best_score && L->last_use[s] < best)) {
                        best_score = sc; best = L->last_use[s]; slot = s;
                    }
                } else if (L->last_use[s] < best) {
                    best = L->last_use[s]; slot = s;
                }
            }
            if (slot < 0) break;
            const int32_t victim = L->slot_expert[slot];
            L->expert_slot[victim] = -1;
            L->slot_expert[slot] = -1;
            set_table_entry(c, L, victim, L->ns);
            L->free_slots[L->n_free++] = slot;
        }
    }
    /* the token is over: its ids become the previous token's, after every
     * eviction decision of the step (patches/0006:914-922) */
    if (c->ev)
        for (int li = 0; li < c->cfg.n_layers; ++li) {
            or_layer *L = &c->L[li];
            memcpy(L->prev_ids, L->cur_ids, sizeof(int32_t) * (size_t)L->n_cur);
            L->n_prev = L->n_cur;
        }
    /* heat decay (patches/0007:736-744) */
    if (c->cfg.admit_mode == 1 && c->cfg.admit_half > 0 &&
        c->n_steps % (uint64_t)c->cfg.admit_half == 0) {
        for (int li = 0; li < c->cfg.n_layers; ++li) {
            for (int e = 0; e < c->cfg.n_expert; ++e) c->L[li].heat[e] *= 0.5f;
        }
    }
    flush_tables(c);
}

int32_t or_cache_n_slots(const or_cache *c, int layer) { return c->L[layer].ns; }

void or_cache_tables(const or_cache *c, int layer, int32_t *expert_slot, int32_t *slot_expert,
                     uint64_t *last_use, uint8_t *in_flight, uint64_t *protect) {
    const or_layer *L = &c->L[layer];
    if (expert_slot) memcpy(expert_slot, L->expert_slot, sizeof(int32_t) * (size_t)c->cfg.n_expert);
    if (slot_expert) memcpy(slot_expert, L->slot_expert, sizeof(int32_t) * (size_t)L->ns);
    if (last_use) memcpy(last_use, L->last_use, sizeof(uint64_t) * (size_t)L->ns);
    if (in_flight) memcpy(in_flight, L->in_flight, (size_t)L->ns);
    if (protect) memcpy(protect, L->protect, sizeof(uint64_t) * (size_t)L->ns);
}

void or_cache_dev_table(const or_cache *c, int layer, int32_t *table, float *prior) {
    const or_layer *L = &c->L[layer];
    if (table) memcpy(table, L->tbl, sizeof(int32_t) * (size_t)c->cfg.n_expert);
    if (prior) memcpy(prior, L->prior, sizeof(float) * (size_t)c->cfg.n_expert);
}

void or_cache_stats(const or_cache *c, uint64_t *out) {
    uint64_t h = 0, m = 0;
    for (int l = 0; l < c->cfg.n_layers; ++l) { h += c->L[l].n_hit; m += c->L[l].n_miss; }
    out[OR_ST_STEPS] = c->n_steps;
    out[OR_ST_CLOCK] = c->clock;
    out[OR_ST_HITS] = h;
    out[OR_ST_MISSES] = m;
    out[OR_ST_UPLOADS] = c->n_uploads;
    out[OR_ST_SCHEDULED] = c->n_scheduled;
    out[OR_ST_COPIED] = c->n_copied;
    out[OR_ST_PUBLISHED] = c->n_published;
    out[OR_ST_ADMIT_OK] = c->n_admit_ok;
    out[OR_ST_ADMIT_DENIED] = c->n_admit_denied;
    out[OR_ST_TABLE_FLUSHES] = c->n_table_flushes;
}

int or_cache_jobs(const or_cache *c, int32_t *out, int max) {
    int n = c->n_todo < max ? c->n_todo : max;
    for (int i = 0; i < n; ++i) {
        out[4 * i + 0] = c->todo[i].layer;
        out[4 * i + 1] = c->todo[i].expert;
        out[4 * i + 2] = c->todo[i].slot;
        out[4 * i + 3] = c->todo[i].spec;
    }
    return c->n_todo;
}

void or_cache_gate_state(const or_cache *c, int layer, float *heat, uint64_t *miss_last,
                         uint64_t *miss_prev, uint32_t *use_count) {
    const or_layer *L = &c->L[layer];
    const size_t E = (size_t)c->cfg.n_expert;
    if (heat && L->heat) memcpy(heat, L->heat, sizeof(float) * E);
    if (miss_last && L->miss_last) memcpy(miss_last, L->miss_last, sizeof(uint64_t) * E);
    if (miss_prev && L->miss_prev) memcpy(miss_prev, L->miss_prev, sizeof(uint64_t) * E);
    if (use_count && L->use_count) memcpy(use_count, L->use_count, sizeof(uint32_t) * E);
}

/* ---- map record text (patches/0008:417-489) ---------------------------------- */

typedef struct { char *buf; int cap; int len; } or_sbuf;

static void sb_printf(or_sbuf *sb, const char *fmt, long long a, long long b, long long c, int n) {
    char tmp[128];
    int k;
    if (n == 1) k = snprintf(tmp, sizeof(tmp), fmt, a);
    else if (n == 2) k = snprintf(tmp, sizeof(tmp), fmt, a, b);
    else k = snprintf(tmp, sizeof(tmp), fmt, a, b, c);
    if (sb->buf && sb->len + k < sb->cap) memcpy(sb->buf + sb->len, tmp, (size_t)k);
    sb->len += k;
}

int or_cache_map_header(const or_cache *c, char *buf, int cap) {
    or_sbuf sb = {buf, cap, 0};
    sb_printf(&sb, "moe-map 1 %lld\n", c->cfg.n_layers, 0, 0, 1);
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        sb_printf(&sb, "layer %lld %lld %lld\n", l, c->L[l].ns, c->cfg.n_expert, 3);
    }
    if (buf && sb.len < cap) buf[sb.len] = 0;
    return sb.len;
}

int or_cache_map_frame(const or_cache *c, char *buf, int cap) {
    or_sbuf sb = {buf, cap, 0};
    sb_printf(&sb, "step %lld\n", (long long)c->n_steps, 0, 0, 1);
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        const or_layer *L = &c->L[l];
        int32_t pub[4096];
        for (int s = 0; s < L->ns; ++s) pub[s] = -1;
        for (int e = 0; e < c->cfg.n_expert; ++e) {
            if (L->expert_slot[e] >= 0) pub[L->expert_slot[e]] = e;
        }
        sb_printf(&sb, "map %lld", l, 0, 0, 1);
        for (int s = 0; s < L->ns; ++s) sb_printf(&sb, " %lld", pub[s], 0, 0, 1);
        sb_printf(&sb, "\n", 0, 0, 0, 1);
    }
    if (buf && sb.len < cap) buf[sb.len] = 0;
    return sb.len;
}

/* ---- heat file (patches/0007:431-485, 567-618) ---------------------------------- */

int or_cache_save_heat(const or_cache *c, const char *path) {
    char tmp[4096];
    snprintf(tmp, sizeof(tmp), "%s.tmp", path);
    FILE *f = fopen(tmp, "w");
    if (!f) return 0;
    fprintf(f, "moe-heat 1 %d %d\n", c->cfg.n_layers, c->cfg.n_expert);
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        const or_layer *L = &c->L[l];
        if (!L->use_count) continue;
        for (int e = 0; e < c->cfg.n_expert; ++e) {
            if (L->use_count[e]) fprintf(f, "%d %d %u\n", l, e, L->use_count[e]);
        }
    }
    const int ok = fclose(f) == 0;
    return ok && rename(tmp, path) == 0;
}

int64_t or_cache_load_heat(or_cache *c, const char *path) {
    FILE *f = fopen(path, "r");
    if (!f) return 0;
    int ver = 0, nl = 0, ne = 0;
    if (fscanf(f, "moe-heat %d %d %d", &ver, &nl, &ne) != 3 || ver != 1 ||
        nl != c->cfg.n_layers || ne != c->cfg.n_expert) {
        fclose(f);
        return -1;
    }
    int il = 0, e = 0;
    unsigned cnt = 0;
    int64_t n = 0;
    while (fscanf(f, "%d %d %u", &il, &e, &cnt) == 3) {
        if (il < 0 || il >= c->cfg.n_layers) continue;
        or_layer *L = &c->L[il];
        if (!L->use_count || e < 0 || e >= c->cfg.n_expert) continue;
        L->use_count[e] = cnt / 2;
        n++;
    }
    fclose(f);
    return n;
}

int64_t or_cache_warm_start(or_cache *c) {
    const int have_pred = c->cfg.have_pred && c->pred;
    const int32_t reserve = c->cfg.early_issue
        ? c->cfg.max_inserts + (have_pred ? c->cfg.predict_top : 0) : 0;
    int64_t placed = 0;
    const int E = c->cfg.n_expert;
    int32_t *order = (int32_t *)malloc(sizeof(int32_t) * (size_t)E);
    for (int li = 0; li < c->cfg.n_layers; ++li) {
        or_layer *L = &c->L[li];
        if (!L->use_count) continue;
        /* stable sort by use_count descending (insertion sort keeps stability) */
        for (int e = 0; e < E; ++e) order[e] = e;
        for (int i = 1; i < E; ++i) {
            const int32_t v = order[i];
            int j = i - 1;
            while (j >= 0 && L->use_count[order[j]] < L->use_count[v]) {
                order[j + 1] = order[j];
                --j;
            }
            order[j + 1] = v;
        }
        const int32_t fill = L->ns - reserve > 0 ? L->ns - reserve : 0;
        int32_t slot = 0;
        for (int kk = 0; kk < E && slot < fill; ++kk) {
            const int32_t e = order[kk];
            if (L->use_count[e] == 0) break;
            L->slot_expert[slot] = e;
            L->expert_slot[e] = slot;
            L->last_use[slot] = (uint64_t)(fill - slot);
            set_table_entry(c, L, e, slot);
            ++slot;
            ++placed;
        }
        if ((uint64_t)fill > c->clock) c->clock = (uint64_t)fill;
        L->n_free = 0;
        for (int32_t f = L->ns - 1; f >= slot; --f) L->free_slots[L->n_free++] = f;
    }
    free(order);
    flush_tables(c);
    return placed;
}

/* ---- byte-priced greedy slot allocation (experiments/p7_slot_allocation.py:144-185) */

double or_greedy_allocate_bytes(const double *miss8, const int32_t *grid, int n_grid,
                                int n_layers, int uniform_cap,
                                const int32_t *frozen, int n_frozen,
                                const double *expert_bytes, int32_t *cap,
                                double *budget_out) {
    double known_sum = 0.0;
    int n_known = 0;
    for (int L = 0; L < n_layers; ++L) {
        if (expert_bytes[L] != 0.0) { known_sum += expert_bytes[L]; n_known++; }
    }
    const double mean_b = n_known ? known_sum / n_known : 0.0;
    double *cost = (double *)malloc(sizeof(double) * (size_t)n_layers);
    int *idx = (int *)calloc((size_t)n_layers, sizeof(int));
    int *is_frozen = (int *)calloc((size_t)n_layers, sizeof(int));
    int *active = (int *)calloc((size_t)n_layers, sizeof(int));
    double *key = (double *)calloc((size_t)n_layers, sizeof(double));
    for (int L = 0; L < n_layers; ++L) cost[L] = expert_bytes[L] != 0.0 ? expert_bytes[L] : mean_b;
    for (int i = 0; i < n_frozen; ++i) if (frozen[i] >= 0 && frozen[i] < n_layers) is_frozen[frozen[i]] = 1;
    double budget = 0.0;
    for (int L = 0; L < n_layers; ++L) budget += uniform_cap * cost[L];
    for (int L = 0; L < n_layers; ++L) cap[L] = is_frozen[L] ? uniform_cap : grid[0];
    double used0 = 0.0;
    for (int L = 0; L < n_layers; ++L) used0 += cap[L] * cost[L];
    double remaining = budget - used0;
#define OR_STEP(L, vout, cout) do {                                                  \
        if (is_frozen[L] || idx[L] + 1 >= n_grid) { vout = -1.0; cout = 0.0; break; } \
        const int i_ = idx[L];                                                        \
        const int ds_ = grid[i_ + 1] - grid[i_];                                      \
        const double dm_ = miss8[(size_t)i_ * n_layers + L] - miss8[(size_t)(i_ + 1) * n_layers + L]; \
        vout = dm_ / (ds_ * cost[L]);                                                 \
        cout = ds_ * cost[L];                                                         \
    } while (0)
    for (int L = 0; L < n_layers; ++L) {
        double v, cc;
        OR_STEP(L, v, cc);
        (void)cc;
        if (v > 0) { active[L] = 1; key[L] = v; }
    }
    for (;;) {
        int pick = -1;
        for (int L = 0; L < n_layers; ++L) {
            if (!active[L]) continue;
            if (pick < 0 || key[L] > key[pick]) pick = L;   /* ties: lowest L */
        }
        if (pick < 0) break;
        active[pick] = 0;
        double v, cc;
        OR_STEP(pick, v, cc);
        if (v <= 0 || cc > remaining) continue;
        idx[pick] += 1;
        cap[pick] = grid[idx[pick]];
        remaining -= cc;
        OR_STEP(pick, v, cc);
        if (v > 0) { active[pick] = 1; key[pick] = v; }
    }
#undef OR_STEP
    double used = 0.0;
    for (int L = 0; L < n_layers; ++L) used += cap[L] * cost[L];
    if (budget_out) *budget_out = budget;
    free(cost); free(idx); free(is_frozen); free(active); free(key);
    return used;
}
