// moe_gemm.cu -- grouped expert GEMM on the 5th-generation tensor cores, for
// batches whose per-expert token counts make the expert FFN a dense
// contraction (prefill chunks, large decode batches).
//
// The routed pairs are grouped by expert (k_group, tiles of GM_NT pairs).
// Then:
//   k_gather_x16    the tile's token rows -> fp16, written in the canonical
//                   K-major no-swizzle tcgen05 operand layout, one contiguous
//                   block per 64-wide K stage, and the sub-block sums of the
//                   rows (the gate/up min term's operand);
//   k_gemm_gate_up  persistent, one CTA per SM over (128 rows of gate and
//                   up, one token tile) items:
//                   - the Q4_K super-blocks of the rows arrive by 2-D TMA;
//                   - the weights go to the tensor cores as the exact
//                     integers sc * q in fp16, written to TMEM (tcgen05.st)
//                     as the MMA's A operand; the token tile by bulk copy;
//                   - two threads issue tcgen05.mma (gate, up; M = 128, N =
//                     pairs rounded to 16, K = 16) into fp32 accumulators,
//                     one per super-block, double-buffered in TMEM, with the
//                     min term folded into each;
//                   - epilogue warps scale each super-block's accumulator by
//                     its d while the next fills, and form SiLU(g) * u as
//                     fp16, directly in the down GEMM's operand layout;
//   k_gemm_down     persistent, one CTA per SM over (128 rows of down, one
//                   token tile) items: Q6_K rows by bulk copy, dequantised to
//                   fp16 into TMEM as the MMA's A operand, activations by
//                   bulk copy, tcgen05.mma, unweighted rows to ypair[pos][h]
//                   (or, one pair per row, straight to the output row);
//   k_combine       the weighted sum over ranks, in rank order.
//
// Numerics: activations are rounded to fp16 once, and products accumulate in
// fp32.  Gate/up weights are not rounded (their min term's two factors are
// carried as fp16 hi + lo); a down weight is its fp16 scale d * sc times the
// exact integer q6 - 32, rounded to fp16 (two roundings).  The
// reference for this path is exact weights times unquantised activations
// with fp64 accumulation.  The GEMV kernels' Q8_1 activations are a
// different rounding, so the two paths agree only within tolerance.
#include "moe_kernels.h"

#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

namespace moe {

#define GM_ROWS 128        // weight rows per CTA (MMA M)
#define GM_THREADS 256
#define GM_KS_GU 64        // K per gate/up stage (one Q4_K 64-element group)
#define GM_KS_DN 128       // K per down stage (one Q6_K half block)
#define DN_THREADS 512     // down GEMM: 4 threads per row, one quarter each

// tensor maps of the gate and up slot slabs and of the shared expert's
struct alignas(64) GuMaps {
    CUtensorMap g, u, sg, su;
};

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

// ---- operand tiles --------------------------------------------------------
// Canonical no-swizzle K-major tile of R rows x KS columns (fp16): element
// (r, k) at byte ((k / 8) * R + r) * 16 + (k % 8) * 2, i.e. LBO = 16 R,
// SBO = 128.  A token tile has R = GM_NT rows.

// x [n_tok][n_embd] fp32 -> xt[tile][stage][k / 8][n][8] fp16 for every
// tile of the grouping (rows past the tile's pairs are zero), and the gate/up
// GEMM's min-term operand xm[tile][super-block][k / 8][n][8] fp16: for
// sub-block j of the super-block (32 columns), k = 3j, 3j+1, 3j+2 hold
// hi(xs), lo(xs), hi(xs) of xs = the sum of the sub-block's fp16-rounded
// x values (fp32, chunks of 8 summed in order, then the four chunks in
// order); k >= 24 zero.  grid (max tiles, n_embd / GX_COLS): CTA (i, cb)
// writes columns [cb GX_COLS, (cb + 1) GX_COLS) = super-block cb of tile i;
// the tile's token indices are read once into shared memory, and each
// thread's chunks are loaded before any is stored.
#define GX_COLS 256
__global__ void __launch_bounds__(256) k_gather_x16(const float *__restrict__ x,
                                                    const int32_t *__restrict__ off,
                                                    const int32_t *__restrict__ cnt,
                                                    const int32_t *__restrict__ pos_pair,
                                                    const int32_t *__restrict__ tiles,
                                                    const int32_t *__restrict__ n_tiles, int k,
                                                    int n_embd, __half *__restrict__ xt,
                                                    __half *__restrict__ xm) {
    __shared__ int s_tok[GM_NT];
    __shared__ float s_part[4][8][GM_NT];   // [chunk of the sub-block][sub-block][token]
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
    // thread t holds token n = t % 64 and, in chunk j, columns 8 (t / 64 + 4 j)
    // .. +7 of the super-block: chunk t / 64 of sub-block j
    static_assert(PER == 8 && GX_COLS == 256 && GM_NT == 64, "one sub-block per chunk index");
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int c = c0 + threadIdx.x + 256 * j;
        const uint4 h = make_uint4(pack_h2(va[j].x, va[j].y), pack_h2(va[j].z, va[j].w),
                                   pack_h2(vb[j].x, vb[j].y), pack_h2(vb[j].z, vb[j].w));
        *reinterpret_cast<uint4 *>(dst + (size_t)c * 8) = h;
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const __half2 v = *reinterpret_cast<const __half2 *>(&hw[q]);
            sum = __fadd_rn(sum, __low2float(v));
            sum = __fadd_rn(sum, __high2float(v));
        }
        s_part[threadIdx.x / GM_NT][j][threadIdx.x % GM_NT] = sum;
    }
    __syncthreads();
    __half *mdst = xm + ((size_t)i * (n_embd / GX_COLS) + blockIdx.y) * 32 * GM_NT;
    for (int q = threadIdx.x; q < 8 * GM_NT; q += 256) {
        const int j = q / GM_NT, n = q % GM_NT;
        const float xs = __fadd_rn(__fadd_rn(__fadd_rn(s_part[0][j][n], s_part[1][j][n]), s_part[2][j][n]),
                                   s_part[3][j][n]);
        const __half hi = __float2half_rn(xs);
        const __half lo = __float2half_rn(__fsub_rn(xs, __half2float(hi)));
        const __half v3[3] = {hi, lo, hi};
#pragma unroll
        for (int u = 0; u < 3; ++u) {
            const int kk = 3 * j + u;
            mdst[((kk >> 3) * GM_NT + n) * 8 + (kk & 7)] = v3[u];
        }
        if (j == 7)   // k = 24 .. 31: zero
#pragma unroll
            for (int kk = 24; kk < 32; ++kk) mdst[((kk >> 3) * GM_NT + n) * 8 + (kk & 7)] = __float2half_rn(0.0f);
    }
}

// ---- gate/up: exact integer weights on the tensor cores ----------------------
// A Q4_K weight is w = d * sc_j * q - dmin * m_j (q 4-bit, sc_j / m_j the
// 6-bit scale and min of its 32-element sub-block j, d / dmin the fp16 pair
// of its 256-element super-block).  The MMA's A operand is sc_j * q (an
// integer <= 945, exact in fp16), so per super-block sb and token n
//   D_sb[m][n] = sum_k (sc q)[m][k] x~[n][k]          (fp32 accumulators)
// and the min term is one more contraction over the super-block's eight
// sub-blocks into the same accumulator,
//   D_sb[m][n] += sum_j (-(dmin / d) m_j)[m] * xs_j[n],   xs_j = sum of sub-block j of x~,
// with both factors split into fp16 hi + lo (three products per sub-block,
// hi*hi + hi*lo + lo*hi), so that y[m][n] = sum_sb d_sb[m] D_sb[m][n].  x~
// is x rounded to fp16 once; no weight is rounded.  D is double-buffered in
// TMEM by super-block: the epilogue warps scale and add one while the MMAs
// fill the other.

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b),
                        *reinterpret_cast<const __half2 *>(&c));
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// 32 consecutive 32-bit TMEM columns of the calling thread's lane, then
// waited for (the writes are complete when it returns).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::
            "r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, one CTA: A is M rows on
// the TMEM lanes, K packed two fp16 per 32-bit column (K-major).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Group g (elements 64g .. 64g+63) of the Q4_K super-block at `blk` (144
// bytes, shared or global memory) -> row m of the A operand in TMEM (the
// calling thread's lane, 32 columns from `a_taddr`, two fp16 per column in
// K order): sc * q as exact fp16, q taken as the fp16 value 1024 + q
// (byte q under exponent byte 0x64) and one fused (1024 + q) sc - 1024 sc.
// On g == 0 also the row's min columns of the whole super-block, folded
// into the same accumulator (sub-block j: k = 3j, 3j+1 -> hi(-(dmin / d)
// m_j), 3j+2 -> lo; k >= 24 zero; shared-memory tile `Am`, KS 32, no
// swizzle) and the scale d of that accumulator, returned in *dout (1 when
// d == 0, whose main operand is then zero).
__device__ __forceinline__ void deq2_q4k(const uint8_t *blk, int g, uint32_t a_taddr, int m, uint8_t *Am,
                                         float *dout) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * g);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * g);
    int sc0, mn0, sc1, mn1;
    q4k_sm_pair(hdr.y, hdr.z, hdr.w, g, sc0, mn0, sc1, mn1);
    // d == 0: the super-block's weights are -dmin m alone; the main operand
    // is then zero and the min term is scaled by 1 instead of d
    if ((hdr.x & 0x7FFFu) == 0) sc0 = sc1 = 0;
    const uint32_t s0 = h2_bits(__half2half2(__int2half_rn(sc0)));
    const uint32_t s1 = h2_bits(__half2half2(__int2half_rn(sc1)));
    const uint32_t n0 = h2_bits(__half2half2(__int2half_rn(-1024 * sc0)));
    const uint32_t n1 = h2_bits(__half2half2(__int2half_rn(-1024 * sc1)));
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    uint32_t a[32];   // column k / 2: low nibbles -> elements 0..31, high -> 32..63
#pragma unroll
    for (int c = 0; c < 8; ++c) {   // word c: bytes 4c .. 4c+3
        const uint32_t v = w[c];
        const uint32_t L = v & 0x0F0F0F0Fu, Hh = (v >> 4) & 0x0F0F0F0Fu;
        a[2 * c] = hfma2_u(__byte_perm(L, 0x64646464u, 0x4140u), s0, n0);
        a[2 * c + 1] = hfma2_u(__byte_perm(L, 0x64646464u, 0x4342u), s0, n0);
        a[16 + 2 * c] = hfma2_u(__byte_perm(Hh, 0x64646464u, 0x4140u), s1, n1);
        a[16 + 2 * c + 1] = hfma2_u(__byte_perm(Hh, 0x64646464u, 0x4342u), s1, n1);
    }
    tmem_st32(a_taddr, a);
    if (Am) {
        const float d = h2f(hdr.x & 0xFFFFu);
        const float d_eff = (hdr.x & 0x7FFFu) == 0 ? 1.0f : d;
        const float ratio = __fdiv_rn(h2f(hdr.x >> 16), d_eff);   // dmin / d
        *dout = d_eff;
        uint32_t h[16];   // 32 halves, two per word
#pragma unroll
        for (int i = 0; i < 16; ++i) h[i] = 0;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            int a0, m0, a1, m1;
            q4k_sm_pair(hdr.y, hdr.z, hdr.w, p, a0, m0, a1, m1);
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int j = 2 * p + t;
                const float v = -__fmul_rn(ratio, (float)(t ? m1 : m0));
                const __half vh = __float2half_rn(v);
                const __half vl = __float2half_rn(v - __half2float(vh));
                const uint32_t bh = (uint32_t)__half_as_ushort(vh), bl = (uint32_t)__half_as_ushort(vl);
                const int k = 3 * j;   // halves k, k+1 = hi, k+2 = lo
                const uint32_t vals[3] = {bh, bh, bl};
#pragma unroll
                for (int u = 0; u < 3; ++u) {
                    const int kk = k + u;
                    h[kk >> 1] |= vals[u] << (16 * (kk & 1));
                }
            }
        }
        uint8_t *arow = Am + (m >> 3) * 128 + (m & 7) * 16;
#pragma unroll
        for (int c = 0; c < 4; ++c) st_shared_v4(arow + c * 2048, h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
    }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared memory of k_gemm_gate_up (bytes): raw super-blocks [2 buf][gate, up]
// (128 rows x 144 B, by TMA), the epilogue's 32 KB exchange area, min tiles
// [gate, up] 128 x 32 fp16, B [GU_NB] 64 x 64 fp16 (a ring), the min-term B
// [2 buf] 64 x 32 fp16, d [4 super-blocks][gate, up][128] fp32, barriers,
// TMEM address.  The A operand of the main term lives in TMEM (written by
// the dequantising threads with tcgen05.st), so that the weights, once
// dequantised, cross shared memory neither on the way in nor on the way to
// the tensor cores.  A stage is K = 128 (two Q4_K groups, eight MMAs per
// matrix per barrier round trip).  TMEM columns: D [2 super-block
// parity][gate, up] x 64 at 0..255, A [2 stage parity][gate, up] x 64 at
// 256..511.
#define GU_RAW_BYTES (GM_ROWS * MOE_Q4K_BYTES)     // 18432
#define GU_X_BYTES (GM_ROWS * GM_NT * 4)           // 32768
#define GU_AM_BYTES (GM_ROWS * 32 * 2)             // 8192
#define GU_KS 128                                  // K per stage
#define GU_B_BYTES (GM_NT * GU_KS * 2)             // 16384
#define GU_BM_BYTES (GM_NT * 32 * 2)               // 4096
#define GU_NB 4
#define GU_OFF_X (4 * GU_RAW_BYTES)
#define GU_OFF_AM (GU_OFF_X + GU_X_BYTES)
#define GU_OFF_B (GU_OFF_AM + 2 * GU_AM_BYTES)
#define GU_OFF_BM (GU_OFF_B + GU_NB * GU_B_BYTES)
#define GU_OFF_D (GU_OFF_BM + 2 * GU_BM_BYTES)
#define GU_OFF_BAR (GU_OFF_D + 4 * 2 * GM_ROWS * 4)
#define GU_SMEM (GU_OFF_BAR + 512)   // 32 barriers (256 bytes) + the TMEM address
static_assert((4 + 4 + 4 + 4 + 2 * GU_NB + 2 + 2) * 8 + 4 <= 512, "gate/up barrier area");
#define GU_DQ_THREADS GM_THREADS                    // 8 dequantising warps
#define GU_THREADS (GU_DQ_THREADS + 3 * 32 + 256)   // + copy warp, 2 MMA warps, 8 epilogue warps

// One work item of the persistent gate/up kernel: 128 rows (row block rbk)
// of one expert tile.
struct GuItem {
    int i, e, np, N, r0, yrow;
    bool dev, shared_e, ok;
    const uint8_t *gbase, *ubase;
};

// The first GU_ITEMS items of a CTA are resolved once, at the start (as in
// the down kernel), so that no role starts an item with a chain of
// dependent global loads.
#define GU_ITEMS 32

__device__ __forceinline__ bool gu_item(const ExpertSrc &src, const int32_t *tiles, const int32_t *cnt, int w,
                                        int RB, int n_ff, GuItem &it) {
    it.i = w / RB;
    it.r0 = (w % RB) * GM_ROWS;
    const int tl = tiles[it.i], tt = tl & 0xFFFF;
    it.e = tl >> 16;
    it.np = min(GM_NT, cnt[it.e] - tt * GM_NT);
    it.N = (it.np + 15) & ~15;
    it.gbase = expert_ptr(src, 0, it.e);
    it.ubase = expert_ptr(src, 1, it.e);
    it.shared_e = it.e == src.n_expert;
    it.dev = expert_on_device(src, it.e);
    it.yrow = (it.shared_e ? 0 : (it.dev ? src.table[it.e] : 0) * n_ff) + it.r0;
    it.ok = it.gbase && it.ubase;
    return it.ok;
}

// Persistent: CTA c takes work items c, c + gridDim.x, ... (item w = row
// block w % (n_ff / 128) of tile w / (n_ff / 128)).  Every role walks the
// same items; the barrier phases run on counters global over the items
// (stage, super-block, raw super-block), so that the copies and MMAs of the
// next item start while the epilogue of this one finishes.
// Warp roles (gate and up run as two pipelines that share the token tiles):
//   warps 0-7   dequantise: thread (mat, m) row m of gate (mat 0, warps 0-3)
//               or up (mat 1, warps 4-7) into that matrix's A columns in
//               TMEM; a stage's A goes to the matrix's MMA warp through
//               a_full[mat] (one arrival per warp) and comes back through the
//               MMAs' commit (mma_done[mat]); a raw super-block is released
//               through raw_free after its last group;
//   warp 8      lane 0 issues the raw super-block TMAs (2 buffers) and the
//               token-tile copies (a ring of GU_NB stages, a slot reused once
//               both matrices' MMAs of it are done: b_free);
//   warps 9, 10 lane 0 issues the MMAs of gate / up: one issuing thread per
//               matrix, the issue itself (tens of ns per instruction and per
//               barrier operation) bounding a 128 x 64 x 64 stage;
//   warps 11-18 epilogue: warp w holds row 32 (w % 4) + lane of one matrix
//               and adds d_sb * D_sb into registers after each super-block
//               (d_full -> d_free), then forms SiLU(g) * u.
__global__ void __launch_bounds__(GU_THREADS, 1) k_gemm_gate_up(
    ExpertSrc src, const __grid_constant__ GuMaps maps, const __half *__restrict__ xt,
    const __half *__restrict__ xm, const int32_t *__restrict__ off, const int32_t *__restrict__ cnt,
    const int32_t *__restrict__ tiles, const int32_t *__restrict__ n_tiles, int n_embd, int n_ff,
    __half *__restrict__ at, int *err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int RB = n_ff / GM_ROWS;
    const int n_items = *n_tiles * RB;
    if ((int)blockIdx.x >= n_items) return;
    uint8_t *sRaw = sm;                                 // [buf][mat]
    uint8_t *sX = sm + GU_OFF_X;                        // the epilogue's exchange
    uint8_t *sAm = sm + GU_OFF_AM;                      // [mat]
    uint8_t *sB = sm + GU_OFF_B;                        // [GU_NB]
    uint8_t *sBm = sm + GU_OFF_BM;                      // [buf]
    float *sD = reinterpret_cast<float *>(sm + GU_OFF_D);   // [sb & 3][mat][128]
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(sm + GU_OFF_BAR);   // [mat][2]
    uint64_t *a_full = mma_done + 4;     // [mat][2]
    uint64_t *d_full = a_full + 4;       // [mat][2]
    uint64_t *d_free = d_full + 4;       // [mat][2]
    uint64_t *b_full = d_free + 4;       // [GU_NB]
    uint64_t *b_free = b_full + GU_NB;   // [GU_NB]
    uint64_t *raw_full = b_free + GU_NB; // [2]
    uint64_t *raw_free = raw_full + 2;   // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(raw_free + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = n_embd / GU_KS, NSB = S / 2;   // two stages per super-block
    const size_t rb = (size_t)(n_embd / MOE_QK) * MOE_Q4K_BYTES;   // bytes per row
    if (tid == 0) {
        for (int q = 0; q < 4; ++q) {
            mbar_init(&mma_done[q], 1);
            mbar_init(&a_full[q], GU_DQ_THREADS / 64);
            mbar_init(&d_full[q], 1);
            mbar_init(&d_free[q], 4);
        }
        for (int q = 0; q < GU_NB; ++q) {
            mbar_init(&b_full[q], 1);
            mbar_init(&b_free[q], 2);
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&raw_full[q], 1);
            mbar_init(&raw_free[q], GU_DQ_THREADS / 32);
        }
        fence_mbar_init();
    }
    __shared__ GuItem s_items[GU_ITEMS];
    const int G = gridDim.x;
    if (tid < GU_ITEMS && (int)blockIdx.x + tid * G < n_items)
        gu_item(src, tiles, cnt, blockIdx.x + tid * G, RB, n_ff, s_items[tid]);
    if (warp == 0) tmem_alloc(tslot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    bool ok = true;
    const int W_COPY = GU_DQ_THREADS / 32, W_MMA = W_COPY + 1, W_EPI = W_MMA + 2;
    // item k of this CTA (w = blockIdx.x + k G)
    auto item = [&](int k) {
        GuItem it;
        if (k < GU_ITEMS) it = s_items[k];
        else gu_item(src, tiles, cnt, blockIdx.x + k * G, RB, n_ff, it);
        return it;
    };
    if (warp == W_COPY) {
        // ---- copy warp: raw super-blocks and the token-tile ring ----
        if (lane == 0) {
            int gs = 0, rseq = 0;
            for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
                const GuItem it = item(k);
                if (!it.ok) continue;
                const CUtensorMap *mg = it.shared_e ? &maps.sg : &maps.g;
                const CUtensorMap *mu = it.shared_e ? &maps.su : &maps.u;
                const __half *xtile = xt + (size_t)it.i * n_embd * GM_NT;
                const __half *mtile = xm + (size_t)it.i * (n_embd / 8) * GM_NT;   // [sb][32 x 64]
                for (int sb = 0; sb < NSB; ++sb) {
                    if (it.dev) {
                        // raw buffer rseq & 1, last read by raw super-block rseq - 2
                        const int bf = rseq & 1;
                        if (rseq >= 2 && !mbar_wait(&raw_free[bf], ((rseq - 2) >> 1) & 1)) ok = false;
                        mbar_arrive_expect_tx(&raw_full[bf], 2 * GU_RAW_BYTES);
                        tma_load_2d(sRaw + (2 * bf) * GU_RAW_BYTES, mg, sb * MOE_Q4K_BYTES, it.yrow, &raw_full[bf]);
                        tma_load_2d(sRaw + (2 * bf + 1) * GU_RAW_BYTES, mu, sb * MOE_Q4K_BYTES, it.yrow,
                                    &raw_full[bf]);
                        ++rseq;
                    }
                    for (int h = 0; h < 2; ++h, ++gs) {
                        // ring slot gs % NB, last read by the MMAs of stage gs - NB
                        // (the min-term buffer of a first stage, by stage gs - 4)
                        const int nb = gs % GU_NB;
                        if (gs >= GU_NB && !mbar_wait(&b_free[nb], ((gs / GU_NB) - 1) & 1)) ok = false;
                        const int s = 2 * sb + h;
                        fence_proxy_async();
                        mbar_arrive_expect_tx(&b_full[nb], GU_B_BYTES + (h == 0 ? GU_BM_BYTES : 0));
                        // two 64-wide blocks of the gathered tile, contiguous
                        bulk_g2s(sB + nb * GU_B_BYTES, xtile + (size_t)s * GM_NT * GU_KS, GU_B_BYTES,
                                 &b_full[nb]);
                        if (h == 0)
                            bulk_g2s(sBm + ((gs >> 1) & 1) * GU_BM_BYTES, mtile + (size_t)sb * 32 * GM_NT,
                                     GU_BM_BYTES, &b_full[nb]);
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == W_MMA || warp == W_MMA + 1) {
        // ---- MMA warps: one matrix each ----
        const int mat = warp - W_MMA;
        if (lane == 0) {
            int gs = 0;
            for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
                const GuItem it = item(k);
                if (!it.ok) continue;
                const uint32_t idesc = idesc_f16(GM_ROWS, it.N);
                for (int s = 0; s < S; ++s, ++gs) {
                    const int gsb = gs >> 1, g = s & 1, b = gsb & 1;
                    // D[b] was last used by super-block gsb - 2: wait for its epilogue
                    if (g == 0 && gsb >= 2 && !mbar_wait(&d_free[mat * 2 + b], ((gsb - 2) >> 1) & 1)) ok = false;
                    const bool ready = mbar_wait(&a_full[mat * 2 + (gs & 1)], (gs >> 1) & 1) &&
                                       mbar_wait(&b_full[gs % GU_NB], (gs / GU_NB) & 1);
                    tc_fence_after();
                    if (ready) {
                        const uint32_t aA = tmem + 256 + (uint32_t)((2 * (gs & 1) + mat) * 64);
                        const uint32_t bB = smem_u32(sB + (gs % GU_NB) * GU_B_BYTES);
                        const uint32_t dD = tmem + (uint32_t)((2 * b + mat) * 64);
#pragma unroll
                        for (int j = 0; j < GU_KS / 16; ++j)   // K step j: block j / 4 of the two 64-wide ones
                            tc_mma_ts(dD, aA + 8 * j,
                                      smem_desc(bB + (j >> 2) * GM_NT * GM_KS_GU * 2 + (j & 3) * 2 * (GM_NT * 16),
                                                GM_NT * 16, 128),
                                      idesc, (g | j) != 0);
                        if (g == 0) {   // the folded min term of the super-block: K = 32
                            const uint32_t mA = smem_u32(sAm + mat * GU_AM_BYTES);
                            const uint32_t bM = smem_u32(sBm + b * GU_BM_BYTES);
#pragma unroll
                            for (int j = 0; j < 2; ++j)
                                tc_mma(dD, smem_desc(mA + j * 2 * (GM_ROWS * 16), GM_ROWS * 16, 128),
                                       smem_desc(bM + j * 2 * (GM_NT * 16), GM_NT * 16, 128), idesc, 1);
                        }
                    } else {
                        ok = false;
                    }
                    tc_commit(&mma_done[mat * 2 + (gs & 1)]);
                    tc_commit(&b_free[gs % GU_NB]);
                    if (g == 1) tc_commit(&d_full[mat * 2 + b]);
                }
            }
        }
        __syncwarp();
    } else if (warp < W_COPY) {
        // ---- dequantising warps ----
        const int mat = tid >> 7, m = tid & 127;
        int gs = 0, rseq = 0;
        for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
            const GuItem it = item(k);
            if (!it.ok) {
                if (tid == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
                continue;
            }
            const uint8_t *hrow = (mat ? it.ubase : it.gbase) + (size_t)(it.r0 + m) * rb;   // a miss: host memory
            for (int s = 0; s < S; ++s, ++gs) {
                const int gsb = gs >> 1, sb = s >> 1, g = s & 1, bf = rseq & 1;
                if (it.dev && g == 0 && !mbar_wait(&raw_full[bf], (rseq >> 1) & 1)) ok = false;
                if (gs >= 2 && !mbar_wait(&mma_done[mat * 2 + (gs & 1)], ((gs - 2) >> 1) & 1)) ok = false;
                // this thread's TMEM lane (row m), A columns of (stage parity, mat)
                const uint32_t A = tmem + ((uint32_t)((warp & 3) * 32) << 16) + 256 +
                                   (uint32_t)((2 * (gs & 1) + mat) * 64);
                // one min tile per matrix: the MMAs of stage gs - 2 (its last
                // reader) are done when the wait above returns
                uint8_t *Am = g == 0 ? sAm + mat * GU_AM_BYTES : nullptr;
                float *dd = &sD[((gsb & 3) * 2 + mat) * GM_ROWS + m];
                // groups 2g, 2g + 1 of the super-block; each call reads its raw
                // block in a known address space (shared loads on the hot path)
                for (int h = 0; h < 2; ++h) {
                    if (it.dev)
                        deq2_q4k(sRaw + (2 * bf + mat) * GU_RAW_BYTES + m * MOE_Q4K_BYTES, 2 * g + h, A + 32 * h, m,
                                 h == 0 ? Am : nullptr, dd);
                    else
                        deq2_q4k(hrow + (size_t)sb * MOE_Q4K_BYTES, 2 * g + h, A + 32 * h, m, h == 0 ? Am : nullptr,
                                 dd);
                }
                if (g == 0) fence_proxy_async();   // the min tile, read by the tensor cores
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[mat * 2 + (gs & 1)]);
                    if (it.dev && g == 1) mbar_arrive(&raw_free[bf]);
                }
                if (it.dev && g == 1) ++rseq;
            }
        }
    } else {
        // ---- epilogue warps ----
        const int ew = warp - W_EPI;
        const int mat = ew >> 2, quad = warp & 3, m = quad * 32 + lane;
        const uint32_t lanes = (uint32_t)(quad * 32) << 16;
        float *xch = reinterpret_cast<float *>(sX);   // [64][128]
        int gsb = 0;
        for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
            const GuItem it = item(k);
            if (!it.ok) continue;
            float R[64];
#pragma unroll
            for (int n = 0; n < 64; ++n) R[n] = 0.0f;
            for (int sb = 0; sb < NSB; ++sb, ++gsb) {
                const int b = gsb & 1;
                if (!mbar_wait(&d_full[mat * 2 + b], (gsb >> 1) & 1)) ok = false;
                tc_fence_after();
                const float d = sD[((gsb & 3) * 2 + mat) * GM_ROWS + m];
                const uint32_t ta = tmem + lanes + (uint32_t)((2 * b + mat) * 64);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (c * 16 < it.N) {
                        float v[16];
                        tmem_ld16(ta + c * 16, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) R[c * 16 + j] = fmaf(d, v[j], R[c * 16 + j]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_free[mat * 2 + b]);
            }
            // up -> shared memory, then the gate warps form SiLU(g) * u in the
            // down GEMM's operand layout: at[tile][stage r0/128][k/8 = m/8][n][m % 8]
            if (mat == 1)
#pragma unroll
                for (int n = 0; n < 64; ++n) xch[n * GM_ROWS + m] = R[n];
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (mat == 0) {
                __half *dst = at + ((size_t)it.i * n_ff + it.r0) * GM_NT + (size_t)(m >> 3) * GM_NT * 8 + (m & 7);
#pragma unroll
                for (int n = 0; n < 64; ++n)
                    if (n < it.np) dst[(size_t)n * 8] = __float2half_rn(silu_mul(R[n], xch[n * GM_ROWS + m]));
            }
            asm volatile("bar.sync 1, 256;" ::: "memory");   // xch is free for the next item
        }
    }
    if (!ok) atomicOr(err, MOE_DEV_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

// 16 consecutive 32-bit TMEM columns of the calling thread's lane, then
// waited for.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Quarter q (32 elements, l = 0..31) of a Q6_K half block -> 16 words of
// packed fp16 in K order (word c: elements 2c, 2c + 1): w = ws * (q6 - 32),
// with ws = d * sc rounded to fp16 once per 16 elements, and the product of
// ws and the exact integer q6 - 32 rounded once.  Per pair of weights: a
// byte permute places q6 in the mantissa of 1024 (0x64xx), a packed
// subtraction of 1056 leaves q6 - 32 exactly, and a packed multiplication
// applies ws.  src: the 8 ql words of the quarter (low half of the half
// block for even q, high for odd), qh: the half's 8 qh words.
__device__ __forceinline__ void deq_q6k_quarter(const uint32_t (&src)[8], const uint32_t (&qh)[8],
                                                const uint32_t (&sc)[2], float d, int q, uint32_t (&o)[16]) {
    const int ns = 4 * (q >> 1), hs = 2 * q;
    const __half2 bias = __float2half2_rn(1056.0f);
#pragma unroll
    for (int c = 0; c < 4; ++c) {                      // l = 8c .. 8c+7
        const int g = (c >> 1) + 2 * q;                // scale byte (l / 16) + 2q
        const uint32_t scw = (g >> 2) ? sc[1] : sc[0];   // a select, not an indexed (local) array
        const __half2 ws = __float2half2_rn(d * (float)(int8_t)((scw >> (8 * (g & 3))) & 0xFFu));
#pragma unroll
        for (int wi = 0; wi < 2; ++wi) {
            const int i = 2 * c + wi;
            const uint32_t v6 = ((src[i] >> ns) & 0x0F0F0F0Fu) | (((qh[i] >> hs) & 0x03030303u) << 4);
            const uint32_t lo = __byte_perm(v6, 0x64646464u, 0x4140u), hi = __byte_perm(v6, 0x64646464u, 0x4342u);
            o[4 * c + 2 * wi] = h2_bits(__hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&lo), bias), ws));
            o[4 * c + 2 * wi + 1] = h2_bits(__hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&hi), bias), ws));
        }
    }
}

// Shared memory of k_gemm_down (bytes): the 128 Q6_K rows of two items [2]
// (one bulk copy each, the rows being contiguous), the token-tile ring
// B [DN_NB] 64 x 128 fp16, barriers, TMEM address.  The A operand lives in
// TMEM, written by the dequantising threads (tcgen05.st).  TMEM columns: D
// [item parity] x 64 at 0..127, A [stage parity] x 64 (K = 128 as fp16
// pairs) at 128..255.
#define DN_B_BYTES (GM_NT * GM_KS_DN * 2)
#define DN_NB 3
__host__ __device__ static inline int dn_rows_bytes(int n_ff) {
    return ((GM_ROWS * (n_ff / MOE_QK) * MOE_Q6K_BYTES) + 127) & ~127;
}
static inline int dn_smem(int n_ff) { return 2 * dn_rows_bytes(n_ff) + DN_NB * DN_B_BYTES + 256; }
#define DN_EPI 4                                           // epilogue warps
#define DN_ALL_THREADS (DN_THREADS + 2 * 32 + DN_EPI * 32)  // + copy warp, MMA warp, epilogue warps

// One work item of the persistent down kernel: 128 rows (row block r0 /
// 128) of one expert tile.
struct DnItem {
    const uint8_t *rows;   // the item's first row (device slot, or host memory for a miss); null: none
    int i, np, N, pos0, r0, dev;
};

__device__ __forceinline__ DnItem dn_item(const ExpertSrc &src, const int32_t *off, const int32_t *tiles,
                                          const int32_t *cnt, int w, int RB, size_t rb) {
    DnItem it;
    it.i = w / RB;
    it.r0 = (w % RB) * GM_ROWS;
    const int tl = tiles[it.i], e = tl >> 16, tt = tl & 0xFFFF;
    it.pos0 = off[e] + tt * GM_NT;
    it.np = min(GM_NT, cnt[e] - tt * GM_NT);
    it.N = (it.np + 15) & ~15;
    const uint8_t *base = expert_ptr(src, 2, e);
    it.dev = expert_on_device(src, e);
    it.rows = base ? base + (size_t)it.r0 * rb : nullptr;
    return it;
}

// The first DN_ITEMS items of a CTA are resolved once, at the start, by as
// many threads; later ones (very large batches) by each role as it gets to
// them.  Every role thus starts an item without a chain of dependent global
// loads.
#define DN_ITEMS 64

// Persistent: CTA c takes work items c, c + gridDim.x, ... (item w = row
// block w % (n_embd / 128) of tile w / (n_embd / 128)).  Every role walks
// the same items; the barrier phases run on counters global over the items
// (stage, item), so that the next item's rows arrive while this one is
// dequantised, and its MMAs run while this one's accumulator is written out.
// Warp roles:
//   warps 0-15  dequantise, four threads per row, one quarter (32 of the
//               stage's K = 128) each, into the A columns of the stage's
//               parity in TMEM (a_full: one arrival per warp); the A
//               columns come back through the MMAs' commit (mma_done), the
//               item's rows through raw_free after its last stage;
//   warp 16     lane 0 issues the item's row copy (2 buffers; for a miss
//               only an arrival, the rows being read from host memory) and
//               the token-tile copies (a ring of DN_NB, freed by b_free);
//   warp 17     lane 0 issues the MMAs (M = 128, N = pairs rounded to 16, K
//               = 16; eight per stage) into the item's accumulator (D
//               double-buffered by item: d_full -> d_free);
//   warps 18-21 epilogue: the accumulator's rows to ypair[pos][h], unweighted.
__global__ void __launch_bounds__(DN_ALL_THREADS, 1) k_gemm_down(
    ExpertSrc src, const __half *__restrict__ at, const int32_t *__restrict__ off,
    const int32_t *__restrict__ cnt, const int32_t *__restrict__ tiles,
    const int32_t *__restrict__ n_tiles, int n_embd, int n_ff, float *__restrict__ ypair,
    const int32_t *__restrict__ pos_pair, float *__restrict__ ydirect, int *err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const int RB = n_embd / GM_ROWS;
    const int n_items = *n_tiles * RB;
    if ((int)blockIdx.x >= n_items) return;
    const size_t rb = (size_t)(n_ff / MOE_QK) * MOE_Q6K_BYTES;   // bytes per row
    const int rows_bytes = dn_rows_bytes(n_ff);
    uint8_t *sR = sm;                                    // [2] the items' rows
    uint8_t *sB = sm + 2 * rows_bytes;                   // [DN_NB]
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(sB + DN_NB * DN_B_BYTES);   // [2]
    uint64_t *raw_free = raw_full + 2;    // [2]
    uint64_t *a_full = raw_free + 2;      // [2]
    uint64_t *mma_done = a_full + 2;      // [2]
    uint64_t *b_full = mma_done + 2;      // [DN_NB]
    uint64_t *b_free = b_full + DN_NB;    // [DN_NB]
    uint64_t *d_full = b_free + DN_NB;    // [2]
    uint64_t *d_free = d_full + 2;        // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(d_free + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = n_ff / GM_KS_DN;
    if (tid == 0) {
        for (int q = 0; q < 2; ++q) {
            mbar_init(&raw_full[q], 1);
            mbar_init(&raw_free[q], DN_THREADS / 32);
            mbar_init(&a_full[q], DN_THREADS / 32);
            mbar_init(&mma_done[q], 1);
            mbar_init(&d_full[q], 1);
            mbar_init(&d_free[q], DN_EPI);
        }
        for (int q = 0; q < DN_NB; ++q) {
            mbar_init(&b_full[q], 1);
            mbar_init(&b_free[q], 1);
        }
        fence_mbar_init();
    }
    __shared__ DnItem s_items[DN_ITEMS];
    const int G = gridDim.x;
    if (tid < DN_ITEMS && (int)blockIdx.x + tid * G < n_items)
        s_items[tid] = dn_item(src, off, tiles, cnt, blockIdx.x + tid * G, RB, rb);
    if (warp == 0) tmem_alloc(tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    bool ok = true;
    const int W_COPY = DN_THREADS / 32, W_MMA = W_COPY + 1;   // then the epilogue warps
    // item k of this CTA (w = blockIdx.x + k G)
    auto item = [&](int k) {
        return k < DN_ITEMS ? s_items[k] : dn_item(src, off, tiles, cnt, blockIdx.x + k * G, RB, rb);
    };
    if (warp == W_COPY) {
        // ---- copy warp: the items' rows and the token-tile ring ----
        if (lane == 0) {
            int gi = 0, gs = 0;
            for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
                const DnItem it = item(k);
                if (!it.rows) continue;
                const int bf = gi & 1;
                // rows buffer gi & 1, last read by item gi - 2
                if (gi >= 2 && !mbar_wait(&raw_free[bf], ((gi - 2) >> 1) & 1)) ok = false;
                if (it.dev) {
                    mbar_arrive_expect_tx(&raw_full[bf], (uint32_t)(GM_ROWS * rb));
                    bulk_g2s(sR + bf * rows_bytes, it.rows, (uint32_t)(GM_ROWS * rb), &raw_full[bf]);
                } else {
                    mbar_arrive(&raw_full[bf]);
                }
                ++gi;
                const __half *atile = at + (size_t)it.i * n_ff * GM_NT;
                for (int s = 0; s < S; ++s, ++gs) {
                    const int nb = gs % DN_NB;
                    // ring slot gs % DN_NB, last read by the MMAs of stage gs - DN_NB
                    if (gs >= DN_NB && !mbar_wait(&b_free[nb], ((gs / DN_NB) - 1) & 1)) ok = false;
                    mbar_arrive_expect_tx(&b_full[nb], DN_B_BYTES);
                    bulk_g2s(sB + nb * DN_B_BYTES, atile + (size_t)s * GM_NT * GM_KS_DN, DN_B_BYTES, &b_full[nb]);
                }
            }
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        // ---- MMA warp ----
        if (lane == 0) {
            int gi = 0, gs = 0;
            for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
                const DnItem it = item(k);
                if (!it.rows) continue;
                const uint32_t idesc = idesc_f16(GM_ROWS, it.N);
                const int db = gi & 1;
                // D[db] was last used by item gi - 2: wait for its epilogue
                if (gi >= 2 && !mbar_wait(&d_free[db], ((gi - 2) >> 1) & 1)) ok = false;
                const uint32_t dD = tmem + (uint32_t)(db * 64);
                for (int s = 0; s < S; ++s, ++gs) {
                    const bool ready = mbar_wait(&a_full[gs & 1], (gs >> 1) & 1) &&
                                       mbar_wait(&b_full[gs % DN_NB], (gs / DN_NB) & 1);
                    tc_fence_after();
                    if (ready) {
                        const uint32_t aA = tmem + 128 + (uint32_t)((gs & 1) * 64);
                        const uint32_t bB = smem_u32(sB + (gs % DN_NB) * DN_B_BYTES);
#pragma unroll
                        for (int j = 0; j < GM_KS_DN / 16; ++j)
                            tc_mma_ts(dD, aA + 8 * j, smem_desc(bB + j * 2 * (GM_NT * 16), GM_NT * 16, 128), idesc,
                                      (s | j) != 0);
                    } else {
                        ok = false;
                    }
                    tc_commit(&mma_done[gs & 1]);
                    tc_commit(&b_free[gs % DN_NB]);
                }
                tc_commit(&d_full[db]);
                ++gi;
            }
        }
        __syncwarp();
    } else if (warp < W_COPY) {
        // ---- dequantising warps ----
        const int qtr = tid >> 7, m = tid & 127;
        int gi = 0, gs = 0;
        for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
            const DnItem it = item(k);
            if (!it.rows) {
                if (tid == 0) atomicOr(err, MOE_DEV_ERR_INDEX);
                continue;
            }
            const int bf = gi & 1;
            if (!mbar_wait(&raw_full[bf], (gi >> 1) & 1)) ok = false;
            // the item's row m: its copy in shared memory, or host memory for a miss
            const uint8_t *row = it.dev ? sR + bf * rows_bytes + (size_t)m * rb : it.rows + (size_t)m * rb;
            for (int s = 0; s < S; ++s, ++gs) {
                const uint8_t *blk = row + (s >> 1) * MOE_Q6K_BYTES;
                const int h = s & 1;
                uint32_t src8[8], qh[8], sc[2];
                ldw_a2<8>(blk + 64 * h + 32 * (qtr & 1), src8);
                ldw_a2<8>(blk + 128 + 32 * h, qh);
                ldw_a2<2>(blk + 192 + 8 * h, sc);
                const float d = h2f(*reinterpret_cast<const uint16_t *>(blk + 208));
                uint32_t o[16];
                deq_q6k_quarter(src8, qh, sc, d, qtr, o);
                // A columns of stage parity gs & 1, last read by the MMAs of stage gs - 2
                if (gs >= 2 && !mbar_wait(&mma_done[gs & 1], ((gs - 2) >> 1) & 1)) ok = false;
                tc_fence_after();
                tmem_st16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + 128 + (uint32_t)((gs & 1) * 64 + 16 * qtr), o);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[gs & 1]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_free[bf]);
            ++gi;
        }
    } else {
        // ---- epilogue warps ----
        const int quad = warp & 3;
        const uint32_t lanes = (uint32_t)(quad * 32) << 16;
        int gi = 0;
        for (int k = 0; (int)blockIdx.x + k * G < n_items; ++k) {
            const DnItem it = item(k);
            if (!it.rows) continue;
            const int db = gi & 1;
            if (!mbar_wait(&d_full[db], (gi >> 1) & 1)) ok = false;
            tc_fence_after();
            const int hrow = it.r0 + quad * 32 + lane;
            for (int c0 = 0; c0 < it.N; c0 += 16) {
                float v[16];
                tmem_ld16(tmem + lanes + (uint32_t)(db * 64 + c0), v);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int n = c0 + j;
                    if (n < it.np) {
                        const int pos = it.pos0 + n;
                        if (ydirect) ydirect[(size_t)pos_pair[pos] * n_embd + hrow] = v[j];
                        else ypair[(size_t)pos * n_embd + hrow] = v[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[db]);
            ++gi;
        }
    }
    if (!ok) atomicOr(err, MOE_DEV_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

size_t gemm_scratch_halves(int n_expert, int P, int n_embd, int n_ff) {
    const size_t tiles = (size_t)group_max_tiles(n_expert, P, GM_NT);
    // xt [tiles][n_embd][GM_NT], at [tiles][n_ff][GM_NT], xm [tiles][n_embd / 8][GM_NT]
    return tiles * GM_NT * ((size_t)n_embd + n_ff + n_embd / 8);
}

// The gate / up tensor maps: a 2-D view of a slab's rows (row bytes wide,
// rows tall), boxes of one super-block (144 bytes) x 128 rows.
typedef CUresult (*encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                    CUtensorMapFloatOOBfill);

static encode_tiled_fn encode_fn() {
    static encode_tiled_fn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<encode_tiled_fn>(p);
    }
    return fn;
}

static bool rows_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t row_bytes) {
    std::memset(m, 0, sizeof(*m));
    if (!base) return true;   // unused (no shared expert)
    encode_tiled_fn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {row_bytes, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {MOE_Q4K_BYTES, GM_ROWS};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
    __half *xm = at + (size_t)maxt * GM_NT * n_ff;
    const uint64_t rb = (uint64_t)(n_embd / MOE_QK) * MOE_Q4K_BYTES;
    GuMaps maps;
    if (!rows_map(&maps.g, src.gate, (uint64_t)(src.ns + 1) * n_ff, rb) ||
        !rows_map(&maps.u, src.up, (uint64_t)(src.ns + 1) * n_ff, rb) ||
        !rows_map(&maps.sg, src.sgate, (uint64_t)n_ff, rb) || !rows_map(&maps.su, src.sup, (uint64_t)n_ff, rb))
        return cudaErrorNotSupported;
    cudaError_t e;
    k_gather_x16<<<dim3(maxt, n_embd / GX_COLS), 256, 0, s>>>(x, g.off, g.cnt, g.pos_pair, g.tiles, g.n_tiles,
                                                               k, n_embd, xt, xm);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(k_gemm_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  GU_SMEM)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(k_gemm_down, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  dn_smem(n_ff))) != cudaSuccess)
        return e;
    {   // persistent: one CTA per SM (its TMEM and shared memory take an SM)
        int dev = 0, sms = 0;
        if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        const int items = maxt * (n_ff / GM_ROWS);
        k_gemm_gate_up<<<dim3(std::max(1, std::min(sms, items))), GU_THREADS, GU_SMEM, s>>>(
            src, maps, xt, xm, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, at, err);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // one pair per row and no weights: the down rows go straight to y (a
    // combine would only copy them; rows of empty slots are left as they are)
    const bool direct = k == 1 && !w && !resid;
    {   // persistent as well
        int dev = 0, sms = 0;
        if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        const int items = maxt * (n_embd / GM_ROWS);
        k_gemm_down<<<dim3(std::max(1, std::min(sms, items))), DN_ALL_THREADS, dn_smem(n_ff), s>>>(
            src, at, g.off, g.cnt, g.tiles, g.n_tiles, n_embd, n_ff, ypair, g.pos_pair, direct ? y : nullptr,
            err);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return direct ? cudaSuccess : launch_combine(ypair, g.pair_pos, w, n_tok, k, n_embd, resid, y, s);
}

}  // namespace moe
