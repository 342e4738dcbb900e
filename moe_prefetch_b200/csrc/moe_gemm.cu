// moe_gemm.cu -- grouped expert GEMM on the 5th-generation tensor cores, for
// batches whose per-expert token counts make the expert FFN a dense
// contraction (prefill chunks, large decode batches).
//
// The routed pairs are grouped by expert (k_group, tiles of GM_NT pairs).
// Then:
//   k_gather_x16    the tile's token rows -> fp16, written in the canonical
//                   K-major no-swizzle tcgen05 operand layout, one contiguous
//                   block per 64-wide K stage;
//   k_gemm_gate_up  CTA = (128 rows of gate and up, one token tile):
//                   - Q4_K rows are loaded (vector loads, one stage ahead in
//                     registers), dequantised to fp16 in shared memory;
//                   - the token tile arrives by bulk copy (TMA, no
//                     multicast);
//                   - one thread issues tcgen05.mma (M = 128, N = pairs
//                     rounded to 16, K = 16, fp32 accumulators in TMEM);
//                   - the epilogue reads TMEM (tcgen05.ld) and forms
//                     SiLU(g)*u.  It writes the activations as fp16,
//                     directly in the down GEMM's operand layout;
//   k_gemm_down     CTA = (128 rows of down, one token tile): Q6_K rows
//                   dequantised the same way, activations by bulk copy,
//                   tcgen05.mma, unweighted rows to ypair[pos][h];
//   k_combine       the weighted sum over ranks, in rank order.
//
// Numerics: weights and activations are rounded to fp16 once, and products
// accumulate in fp32.  The reference for this path is exact weights times
// unquantised activations with fp64 accumulation.  The GEMV kernels'
// Q8_1 activations are a different rounding, so the two paths agree only
// within tolerance.
#include "moe_kernels.h"

#include <cuda_fp16.h>

namespace moe {

#define GM_ROWS 128        // weight rows per CTA (MMA M)
#define GM_THREADS 256
#define GM_KS_GU 64        // K per gate/up stage (one Q4_K 64-element group)
#define GM_KS_DN 128       // K per down stage (one Q6_K half block)
#define DN_THREADS 512     // down GEMM: 4 threads per row, one quarter each

// ---- tcgen05 / TMEM wrappers ------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, one CTA.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// 16 consecutive fp32 columns of the calling warp's 32 TMEM lanes (lane =
// thread), waited for.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored contiguously; `lbo` = bytes between adjacent core
// matrices along K, `sbo` = bytes between adjacent 8-row groups; version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D, M x N.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ void st_shared_v4(void *p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}

// Exact small integer -> float (0 <= q < 2^23).
__device__ __forceinline__ float u2f(uint32_t q) {
    return __int_as_float(0x4B000000 | q) - 8388608.0f;
}

// Byte j of x as an exact float minus `bias`: the byte placed into the low
// mantissa of 2^23 (0x4B0000xx) by one byte permute, then one subtraction
// (exact for small integers), i.e. the same value as u2f(byte) - (bias - 2^23).
__device__ __forceinline__ float byte_f(uint32_t x, int j, float bias) {
    return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650u | (uint32_t)j)) - bias;
}

// ---- operand tiles --------------------------------------------------------
// Canonical no-swizzle K-major tile of R rows x KS columns (fp16): element
// (r, k) at byte ((k / 8) * R + r) * 16 + (k % 8) * 2, i.e. LBO = 16 R,
// SBO = 128.  A token tile has R = GM_NT rows.

// x [n_tok][n_embd] fp32 -> xt[tile][stage][k / 8][n][8] fp16 for every
// tile of the grouping (rows past the tile's pairs are zero).  grid (max
// tiles, n_embd / GX_COLS): CTA (i, cb) writes columns [cb GX_COLS,
// (cb + 1) GX_COLS) of tile i; the tile's token indices are read once into
// shared memory, and each thread's chunks are loaded before any is stored.
#define GX_COLS 256
__global__ void __launch_bounds__(256) k_gather_x16(const float *__restrict__ x,
                                                    const int32_t *__restrict__ off,
                                                    const int32_t *__restrict__ cnt,
                                                    const int32_t *__restrict__ pos_pair,
                                                    const int32_t *__restrict__ tiles,
                                                    const int32_t *__restrict__ n_tiles, int k,
                                                    int n_embd, __half *__restrict__ xt) {
    __shared__ int s_tok[GM_NT];
    const int i = blockIdx.x;
    if (i >= *n_tiles) return;
    const int tl = tiles[i], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GM_NT;
    const int np = min(GM_NT, cnt[e] - tt * GM_NT);
    if (threadIdx.x < GM_NT) s_tok[threadIdx.x] = threadIdx.x < np ? pos_pair[pos0 + threadIdx.x] / k : -1;
    __syncthreads();
    __half *dst = xt + (size_t)i * n_embd * GM_NT;
    constexpr int PER = (GX_COLS / 8) * GM_NT / 256;   // chunks per thread
    const int c0 = blockIdx.y * (GX_COLS / 8) * GM_NT;   // first chunk: (k/8, n) with k/8 = blockIdx.y * 32
    float4 va[PER], vb[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int c = c0 + threadIdx.x + 256 * j;
        const int n = c % GM_NT, kc = c / GM_NT;
        const int t = s_tok[n];
        va[j] = vb[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t >= 0) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)t * n_embd + 8 * kc);
            va[j] = src[0];
            vb[j] = src[1];
        }
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int c = c0 + threadIdx.x + 256 * j;
        *reinterpret_cast<uint4 *>(dst + (size_t)c * 8) =
            make_uint4(pack_h2(va[j].x, va[j].y), pack_h2(va[j].z, va[j].w), pack_h2(vb[j].x, vb[j].y),
                       pack_h2(vb[j].z, vb[j].w));
    }
}

// Dequantise one 64-element group g of a Q4_K super-block (header `hdr`,
// quants q0/q1 = the group's 32 bytes) into row m of a canonical 128-row
// tile at `A` (LBO 2048): w = d*sc*q - dmin*m in fp32, rounded to fp16 once.
__device__ __forceinline__ void deq_q4k_group(const uint4 &hdr, const uint4 &q0, const uint4 &q1,
                                              int g, uint8_t *A, int m) {
    int sc0, mn0, sc1, mn1;
    q4k_sm_pair(hdr.y, hdr.z, hdr.w, g, sc0, mn0, sc1, mn1);
    const float d = h2f(hdr.x & 0xFFFFu), dmin = h2f(hdr.x >> 16);
    const float d1 = d * (float)sc0, m1 = dmin * (float)mn0;
    const float d2 = d * (float)sc1, m2 = dmin * (float)mn1;
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint8_t *row = A + (m >> 3) * 128 + (m & 7) * 16;
#pragma unroll
    for (int c = 0; c < 4; ++c) {   // bytes 8c .. 8c+7 -> elements 8c.. (low), 32+8c.. (high)
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const uint32_t v = w[2 * c + b];
            const uint32_t L = v & 0x0F0F0F0Fu, Hh = (v >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                lo[2 * b + j] = pack_h2(fmaf(d1, byte_f(L, 2 * j, 8388608.0f), -m1),
                                        fmaf(d1, byte_f(L, 2 * j + 1, 8388608.0f), -m1));
                hi[2 * b + j] = pack_h2(fmaf(d2, byte_f(Hh, 2 * j, 8388608.0f), -m2),
                                        fmaf(d2, byte_f(Hh, 2 * j + 1, 8388608.0f), -m2));
            }
        }
        st_shared_v4(row + c * 2048, lo[0], lo[1], lo[2], lo[3]);
        st_shared_v4(row + (4 + c) * 2048, hi[0], hi[1], hi[2], hi[3]);
    }
}

struct GuRaw {
    uint4 hdr, q0, q1;
};

__device__ __forceinline__ GuRaw load_gu_raw(const uint8_t *row, int s) {
    const uint8_t *blk = row + (s >> 2) * MOE_Q4K_BYTES;
    GuRaw r;
    r.hdr = __ldg(reinterpret_cast<const uint4 *>(blk));
    r.q0 = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * (s & 3)));
    r.q1 = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * (s & 3)));
    return r;
}

// Shared memory of k_gemm_gate_up: A[2 stages][gate, up][128 x 64 fp16]
// (16 KB each), B[3][64 x 64 fp16] (8 KB each), barriers, TMEM address.
#define GU_A_BYTES (GM_ROWS * GM_KS_GU * 2)
#define GU_B_BYTES (GM_NT * GM_KS_GU * 2)
#define GU_SMEM (4 * GU_A_BYTES + 3 * GU_B_BYTES + 128)

// Warp roles: warps 0-7 (GM_THREADS) dequantise, thread (mat, m) row m of
// gate (mat 0) or up (mat 1); warp 8 issues the token-tile copies and, on
// one thread, the MMAs.  A stage's A buffer is handed over by a_full[b] (one
// arrival per dequantising warp, after each thread's proxy fence) and given
// back by the MMAs' commit to mma_done[b]; there is no CTA-wide barrier per
// stage, so a warp can run a stage ahead of another within the two buffers.
#define GU_THREADS (GM_THREADS + 32)
__global__ void __launch_bounds__(GU_THREADS, 2) k_gemm_gate_up(
    ExpertSrc src, const __half *__restrict__ xt, const int32_t *__restrict__ off,
    const int32_t *__restrict__ cnt, const int32_t *__restrict__ tiles,
    const int32_t *__restrict__ n_tiles, int n_embd, int n_ff, __half *__restrict__ at, int *err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int i = blockIdx.y;
    if (i >= *n_tiles) return;
    uint8_t *sA = sm;                                   // [stage][mat] 16 KB
    uint8_t *sB = sm + 4 * GU_A_BYTES;                  // [3] 8 KB
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(sB + 3 * GU_B_BYTES);   // [2]
    uint64_t *b_full = mma_done + 2;                                           // [3]
    uint64_t *a_full = b_full + 3;                                             // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(a_full + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tl = tiles[i], e = tl >> 16, tt = tl & 0xFFFF;
    const int np = min(GM_NT, cnt[e] - tt * GM_NT);
    const int N = (np + 15) & ~15;
    const int r0 = blockIdx.x * GM_ROWS;
    const int S = n_embd / GM_KS_GU;
    const uint8_t *gbase = expert_ptr(src, 0, e);
    const uint8_t *ubase = expert_ptr(src, 1, e);
    if (!gbase || !ubase) {
        if (tid == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    if (tid == 0) {
        for (int q = 0; q < 2; ++q) mbar_init(&mma_done[q], 1);
        for (int q = 0; q < 3; ++q) mbar_init(&b_full[q], 1);
        for (int q = 0; q < 2; ++q) mbar_init(&a_full[q], GM_THREADS / 32);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;               // gate accumulator: columns 0..63, up: 64..127
    const __half *xtile = xt + (size_t)i * n_embd * GM_NT;
    bool ok = true;
    if (warp == GM_THREADS / 32) {
        // ---- copy + MMA warp ----
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(GM_ROWS, N);
            mbar_arrive_expect_tx(&b_full[0], GU_B_BYTES);
            bulk_g2s(sB, xtile, GU_B_BYTES, &b_full[0]);
            for (int s = 0; s < S; ++s) {
                const int b = s & 1;
                if (s + 1 < S) {
                    // B buffer (s+1) % 3 was last read by the MMAs of stage s-2
                    if (s >= 2 && !mbar_wait(&mma_done[b], ((s - 2) >> 1) & 1)) ok = false;
                    const int nb = (s + 1) % 3;
                    fence_proxy_async();
                    mbar_arrive_expect_tx(&b_full[nb], GU_B_BYTES);
                    bulk_g2s(sB + nb * GU_B_BYTES, xtile + (size_t)(s + 1) * GM_NT * GM_KS_GU, GU_B_BYTES,
                             &b_full[nb]);
                }
                const bool ready = mbar_wait(&a_full[b], (s >> 1) & 1) && mbar_wait(&b_full[s % 3], (s / 3) & 1);
                tc_fence_after();
                if (ready) {
                    const uint32_t aG = smem_u32(sA + (2 * b) * GU_A_BYTES);
                    const uint32_t aU = smem_u32(sA + (2 * b + 1) * GU_A_BYTES);
                    const uint32_t bB = smem_u32(sB + (s % 3) * GU_B_BYTES);
#pragma unroll
                    for (int j = 0; j < GM_KS_GU / 16; ++j) {
                        const uint64_t db = smem_desc(bB + j * 2 * (GM_NT * 16), GM_NT * 16, 128);
                        tc_mma(tmem, smem_desc(aG + j * 2 * (GM_ROWS * 16), GM_ROWS * 16, 128), db,
                               idesc, (s | j) != 0);
                        tc_mma(tmem + 64, smem_desc(aU + j * 2 * (GM_ROWS * 16), GM_ROWS * 16, 128), db,
                               idesc, (s | j) != 0);
                    }
                } else {
                    ok = false;
                }
                tc_commit(&mma_done[b]);
            }
        }
        __syncwarp();
    } else {
        // ---- dequantising warps ----
        const int mat = tid >> 7, m = tid & 127;
        const size_t rb = (size_t)(n_embd / MOE_QK) * MOE_Q4K_BYTES;
        const uint8_t *row = (mat ? ubase : gbase) + (size_t)(r0 + m) * rb;
        GuRaw nxt = load_gu_raw(row, 0);
        for (int s = 0; s < S; ++s) {
            const GuRaw cur = nxt;
            if (s + 1 < S) nxt = load_gu_raw(row, s + 1);
            const int b = s & 1;
            if (s >= 2 && !mbar_wait(&mma_done[b], ((s - 2) >> 1) & 1)) ok = false;
            deq_q4k_group(cur.hdr, cur.q0, cur.q1, s & 3, sA + (2 * b + mat) * GU_A_BYTES, m);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
        }
    }
    if (!mbar_wait(&mma_done[(S - 1) & 1], ((S - 1) >> 1) & 1)) ok = false;
    tc_fence_after();
    if (warp < 4) {
        // epilogue: row m = 32 warp + lane; act = silu(g) * u -> the down GEMM's
        // operand tile: at[tile][stage r0/128][k/8 = m/8][n][m % 8]
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16);
        const int mm = warp * 32 + lane;
        __half *dst = at + ((size_t)i * n_ff + r0) * GM_NT + (size_t)(mm >> 3) * GM_NT * 8 + (mm & 7);
        for (int c0 = 0; c0 < N; c0 += 16) {
            float g[16], u[16];
            tmem_ld16(ta + c0, g);
            tmem_ld16(ta + 64 + c0, u);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int n = c0 + j;
                if (n < np) dst[(size_t)n * 8] = __float2half_rn(silu_mul(g[j], u[j]));
            }
        }
    }
    if (!ok) atomicOr(err, MOE_DEV_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 128);
}

// Quarter q (32 elements, l = 0..31) of a Q6_K half block -> row m of a
// canonical 128-row tile at `A` (LBO 2048): w = d * sc * (q6 - 32) in fp32,
// rounded to fp16 once.  src: the 8 ql words of the quarter (low half of the
// half block for even q, high for odd), qh: the half's 8 qh words.
__device__ __forceinline__ void deq_q6k_quarter(const uint32_t (&src)[8], const uint32_t (&qh)[8],
                                                const uint32_t (&sc)[2], float d, int q, uint8_t *A,
                                                int m) {
    uint8_t *row = A + (m >> 3) * 128 + (m & 7) * 16;
    const int ns = 4 * (q >> 1), hs = 2 * q;
#pragma unroll
    for (int c = 0; c < 4; ++c) {                      // l = 8c .. 8c+7
        const int g = (c >> 1) + 2 * q;                // scale byte (l / 16) + 2q
        const uint32_t scw = (g >> 2) ? sc[1] : sc[0];   // a select, not an indexed (local) array
        const float ws = d * (float)(int8_t)((scw >> (8 * (g & 3))) & 0xFFu);
        uint32_t o[4];
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const int i = 2 * c + wi;
            const uint32_t v6 = ((src[i] >> ns) & 0x0F0F0F0Fu) | (((qh[i] >> hs) & 0x03030303u) << 4);
            o[2 * wi] = pack_h2(ws * byte_f(v6, 0, 8388640.0f), ws * byte_f(v6, 1, 8388640.0f));
            o[2 * wi + 1] = pack_h2(ws * byte_f(v6, 2, 8388640.0f), ws * byte_f(v6, 3, 8388640.0f));
        }
        st_shared_v4(row + (4 * q + c) * 2048, o[0], o[1], o[2], o[3]);
    }
}

// Shared memory of k_gemm_down: the CTA's 128 Q6_K rows (one bulk copy, the
// rows being contiguous), A[2][128 x 128 fp16] (32 KB each), B[3][64 x 128
// fp16] (16 KB each), barriers, TMEM address.
#define DN_A_BYTES (GM_ROWS * GM_KS_DN * 2)
#define DN_B_BYTES (GM_NT * GM_KS_DN * 2)
static inline int dn_rows_bytes(int n_ff) { return ((GM_ROWS * (n_ff / MOE_QK) * MOE_Q6K_BYTES) + 127) & ~127; }
static inline int dn_smem(int n_ff) { return dn_rows_bytes(n_ff) + 2 * DN_A_BYTES + 3 * DN_B_BYTES + 128; }

// Warp roles as in k_gemm_gate_up: warps 0-15 (DN_THREADS) dequantise, four
// threads per row; warp 16 issues the token-tile copies and the MMAs.
#define DN_ALL_THREADS (DN_THREADS + 32)
__global__ void __launch_bounds__(DN_ALL_THREADS, 1) k_gemm_down(
    ExpertSrc src, const __half *__restrict__ at, const int32_t *__restrict__ off,
    const int32_t *__restrict__ cnt, const int32_t *__restrict__ tiles,
    const int32_t *__restrict__ n_tiles, int n_embd, int n_ff, float *__restrict__ ypair,
    int *err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int i = blockIdx.y;
    if (i >= *n_tiles) return;
    const size_t rb = (size_t)(n_ff / MOE_QK) * MOE_Q6K_BYTES;   // bytes per row
    const int rows_bytes = (GM_ROWS * (int)rb + 127) & ~127;
    uint8_t *sA = sm;                                   // [2] 32 KB
    uint8_t *sB = sm + 2 * DN_A_BYTES;                  // [3] 16 KB
    uint8_t *sR = sB + 3 * DN_B_BYTES;                  // the CTA's rows
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(sR + rows_bytes);       // [2]
    uint64_t *b_full = mma_done + 2;                                           // [3]
    uint64_t *r_full = b_full + 3;                                             // [1]
    uint64_t *a_full = r_full + 1;                                             // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(a_full + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tl = tiles[i], e = tl >> 16, tt = tl & 0xFFFF;
    const int pos0 = off[e] + tt * GM_NT;
    const int np = min(GM_NT, cnt[e] - tt * GM_NT);
    const int N = (np + 15) & ~15;
    const int r0 = blockIdx.x * GM_ROWS;
    const int S = n_ff / GM_KS_DN;
    const uint8_t *dbase = expert_ptr(src, 2, e);
    if (!dbase) {
        if (tid == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
        return;
    }
    if (tid == 0) {
        for (int q = 0; q < 2; ++q) mbar_init(&mma_done[q], 1);
        for (int q = 0; q < 3; ++q) mbar_init(&b_full[q], 1);
        mbar_init(r_full, 1);
        for (int q = 0; q < 2; ++q) mbar_init(&a_full[q], DN_THREADS / 32);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const __half *atile = at + (size_t)i * n_ff * GM_NT;
    // the CTA's 128 rows are contiguous: one bulk copy from device memory;
    // an expert in host memory (a miss) is copied by the threads
    const uint8_t *rows_g = dbase + (size_t)r0 * rb;
    const bool dev = expert_on_device(src, e);
    if (dev) {
        if (tid == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(r_full, (uint32_t)(GM_ROWS * rb));
            bulk_g2s(sR, rows_g, (uint32_t)(GM_ROWS * rb), r_full);
        }
    } else {
        for (int o = tid * 16; o < GM_ROWS * (int)rb; o += DN_ALL_THREADS * 16)
            *reinterpret_cast<uint4 *>(sR + o) = *reinterpret_cast<const uint4 *>(rows_g + o);
        __syncthreads();
    }
    // the CTA that will most likely take this SM next (one CTA per SM, launch
    // order x fastest): its rows into L2 now, so that its copy lands sooner
    if (tid == 32) {
        int nx, ny;
        next_wave_cta(1, nx, ny);
        if (ny < *n_tiles) {
            const int en = tiles[ny] >> 16;
            const uint8_t *dn = expert_on_device(src, en) ? expert_ptr(src, 2, en) : nullptr;
            if (dn) prefetch_l2(dn + (size_t)nx * GM_ROWS * rb, (uint32_t)(GM_ROWS * rb));
        }
    }
    bool ok = true;
    if (warp == DN_THREADS / 32) {
        // ---- copy + MMA warp ----
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(GM_ROWS, N);
            mbar_arrive_expect_tx(&b_full[0], DN_B_BYTES);
            bulk_g2s(sB, atile, DN_B_BYTES, &b_full[0]);
            for (int s = 0; s < S; ++s) {
                const int b = s & 1;
                if (s + 1 < S) {
                    // B buffer (s+1) % 3 was last read by the MMAs of stage s-2
                    if (s >= 2 && !mbar_wait(&mma_done[b], ((s - 2) >> 1) & 1)) ok = false;
                    const int nb = (s + 1) % 3;
                    mbar_arrive_expect_tx(&b_full[nb], DN_B_BYTES);
                    bulk_g2s(sB + nb * DN_B_BYTES, atile + (size_t)(s + 1) * GM_NT * GM_KS_DN, DN_B_BYTES,
                             &b_full[nb]);
                }
                const bool ready = mbar_wait(&a_full[b], (s >> 1) & 1) && mbar_wait(&b_full[s % 3], (s / 3) & 1);
                tc_fence_after();
                if (ready) {
                    const uint32_t aA = smem_u32(sA + b * DN_A_BYTES);
                    const uint32_t bB = smem_u32(sB + (s % 3) * DN_B_BYTES);
#pragma unroll
                    for (int j = 0; j < GM_KS_DN / 16; ++j)
                        tc_mma(tmem, smem_desc(aA + j * 2 * (GM_ROWS * 16), GM_ROWS * 16, 128),
                               smem_desc(bB + j * 2 * (GM_NT * 16), GM_NT * 16, 128), idesc,
                               (s | j) != 0);
                } else {
                    ok = false;
                }
                tc_commit(&mma_done[b]);
            }
        }
        __syncwarp();
    } else {
        // ---- dequantising warps ----
        const int qtr = tid >> 7, m = tid & 127;
        const uint8_t *row = sR + (size_t)m * rb;
        if (dev && !mbar_wait(r_full, 0)) ok = false;
        for (int s = 0; s < S; ++s) {
            const uint8_t *blk = row + (s >> 1) * MOE_Q6K_BYTES;
            const int h = s & 1;
            uint32_t src[8], qh[8], sc[2];
            ldw_a2<8>(blk + 64 * h + 32 * (qtr & 1), src);
            ldw_a2<8>(blk + 128 + 32 * h, qh);
            ldw_a2<2>(blk + 192 + 8 * h, sc);
            const float d = h2f(*reinterpret_cast<const uint16_t *>(blk + 208));
            const int b = s & 1;
            if (s >= 2 && !mbar_wait(&mma_done[b], ((s - 2) >> 1) & 1)) ok = false;
            deq_q6k_quarter(src, qh, sc, d, qtr, sA + b * DN_A_BYTES, m);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[b]);
        }
    }
    if (!mbar_wait(&mma_done[(S - 1) & 1], ((S - 1) >> 1) & 1)) ok = false;
    tc_fence_after();
    if (warp < 4) {
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16);
        const int hrow = r0 + warp * 32 + lane;
        for (int c0 = 0; c0 < N; c0 += 16) {
            float v[16];
            tmem_ld16(ta + c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int n = c0 + j;
                if (n < np) ypair[(size_t)(pos0 + n) * n_embd + hrow] = v[j];
            }
        }
    }
    if (!ok) atomicOr(err, MOE_DEV_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 64);
}

size_t gemm_scratch_halves(int n_expert, int P, int n_embd, int n_ff) {
    const size_t tiles = (size_t)group_max_tiles(n_expert, P, GM_NT);
    return tiles * GM_NT * ((size_t)n_embd + n_ff);
}

cudaError_t launch_experts_gemm(const ExpertSrc &src, const float *x, const GroupBufs &g,
                                int n_tok, int k, int n_embd, int n_ff, int down_type,
                                const float *w, void *scratch_v, float *ypair, const float *resid,
                                float *y, int *err, cudaStream_t s) {
    __half *scratch = static_cast<__half *>(scratch_v);
    if (down_type != MOE_QT_Q6K || n_ff % GM_KS_DN || n_embd % GM_ROWS || n_ff % GM_ROWS ||
        n_embd % GX_COLS || dn_smem(n_ff) > 227 * 1024)
        return cudaErrorInvalidValue;
    const int P = n_tok * k;
    const int maxt = group_max_tiles(src.n_expert + 1, P, GM_NT);
    __half *xt = scratch;
    __half *at = scratch + (size_t)maxt * GM_NT * n_embd;
    cudaError_t e;
    k_gather_x16<<<dim3(maxt, n_embd / GX_COLS), 256, 0, s>>>(x, g.off, g.cnt, g.pos_pair, g.tiles, g.n_tiles,
                                                               k, n_embd, xt);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_gemm_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  GU_SMEM)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(k_gemm_down, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  dn_smem(n_ff))) != cudaSuccess)
        return e;
    k_gemm_gate_up<<<dim3(n_ff / GM_ROWS, maxt), GU_THREADS, GU_SMEM, s>>>(
        src, xt, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, at, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_gemm_down<<<dim3(n_embd / GM_ROWS, maxt), DN_ALL_THREADS, dn_smem(n_ff), s>>>(
        src, at, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, ypair, err);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return launch_combine(ypair, g.pair_pos, w, n_tok, k, n_embd, resid, y, s);
}

}  // namespace moe
