// moe_ep.cu -- expert-parallel dispatch for batched decode and prefill.
//
// Rank g of `world` owns experts [g * E / world, (g + 1) * E / world) of every
// layer.  A rank routes its own (home) tokens, then sends each routed pair to
// the rank that owns the expert.  The send list is in rank order and, within
// a rank, in pair order (a stable grouping).  Each pair sends the token's
// row and the expert id.  The owners run the expert half on the rows they
// receive.  The unweighted rows come back in the same order, and the home
// rank combines them in rank order.  The exchange itself is NCCL all-to-all
// over NVLink, driven by the host (moe_prefetch_b200/ep.py).
#include "moe_kernels.h"

namespace moe {

// Send slot of the pair at grouped position q: q itself (compact), or, with
// `capacity` slots per rank, rank d's block at d * capacity + (q - off[d]),
// d = ids[p] / (n_expert / world) the rank owning the pair's expert.  The
// pair's expert id and its token's row go to that slot, and pair_pos is
// rewritten to the slot.  The pairs grouped are off[world].
__global__ void __launch_bounds__(256) k_ep_gather(const float *__restrict__ x,
                                                   const int32_t *__restrict__ ids,
                                                   const int32_t *__restrict__ pos_pair,
                                                   const int32_t *__restrict__ off, int world, int n_expert,
                                                   int k, int n_embd, int capacity,
                                                   int32_t *__restrict__ pair_pos,
                                                   int32_t *__restrict__ send_ids,
                                                   float *__restrict__ send_x) {
    const int q = blockIdx.x;
    if (q >= off[world]) return;
    const int p = pos_pair[q];
    int slot = q;
    if (capacity > 0) {
        const int d = ids[p] / (n_expert / world);
        slot = d * capacity + (q - off[d]);
    }
    if (threadIdx.x == 0) {
        send_ids[slot] = ids[p];
        if (capacity > 0) pair_pos[p] = slot;
    }
    const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)(p / k) * n_embd);
    float4 *dst = reinterpret_cast<float4 *>(send_x + (size_t)slot * n_embd);
    for (int i = threadIdx.x; i < n_embd / 4; i += blockDim.x) dst[i] = src[i];
}

__global__ void k_fill_i32(int32_t *p, int n, int v) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

cudaError_t launch_ep_pack(const int32_t *ids, const float *x, int n_tok, int k, int n_expert,
                           int n_embd, int world, int capacity, const GroupBufs &g, int32_t *send_ids,
                           float *send_x, int *err, cudaStream_t s) {
    const int P = n_tok * k;
    if (world < 1 || world > 256 || n_expert % world || capacity < 0) return cudaErrorInvalidValue;
    if (capacity > 0) {   // every slot starts empty
        const int n = world * capacity;
        k_fill_i32<<<(n + 255) / 256, 256, 0, s>>>(send_ids, n, -1);
    }
    // pairs bucketed by owning rank: expert id / (n_expert / world)
    cudaError_t e = launch_group(ids, P, world, 0x7FFF, g, err, s, n_expert / world);
    if (e != cudaSuccess) return e;
    k_ep_gather<<<P, 256, 0, s>>>(x, ids, g.pos_pair, g.off, world, n_expert, k, n_embd, capacity, g.pair_pos,
                                  send_ids, send_x);
    return cudaGetLastError();
}

// ===========================================================================
// The exchange over peer memory.  Every rank owns a mailbox in its device
// memory, mapped into the other ranks with CUDA IPC (plain loads and stores
// over NVLink; no multicast, no bulk copies from peer memory).  One layer:
//
//   source s (after route + pack, compact send order):
//     k_ep_push_rows   block d of its send list -> rank d's mailbox:
//                      ids[s][0 .. cap) (-1 past the count) and x[s][j];
//                      its last CTA: epoch += 1; on rank d: meta[s] =
//                      (count, offset), then flag_fwd[s] = epoch (release,
//                      system scope)
//   owner d:
//     expert rows      on its mailbox's world * cap slots (id -1: empty),
//                      their grouping kernel first waiting (bounded) until
//                      every flag_fwd[s] carries the epoch
//     k_ep_push_rows   (return) y rows of source s -> rank s's ret_y at
//                      offset + j; its last CTA: on rank s: flag_ret[d] = epoch
//   home s:
//     the combine of ret_y, each CTA first waiting until every flag_ret[d]
//     carries the epoch
//
// A source writes rank d's mailbox for the next layer only after its own
// combine, which waited for every owner's return rows, which each owner
// sends after its expert rows have read the mailbox: one mailbox suffices.
// Every rank runs the same sequence of exchanges, so the epochs agree.
// ===========================================================================

#define EP_RPC 4   // rows per CTA of the copy kernels

__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Send counts and offsets of blocks d (forward: the compact send list's
// exclusive scan) or the meta a source wrote (return), clamped to the slots.
__device__ __forceinline__ void ep_block(const EpMail &m, int d, const int32_t *send_count,
                                         const int32_t *meta, int &cnt, int &off) {
    if (send_count) {
        off = 0;
        for (int q = 0; q < d; ++q) off += send_count[q];
        cnt = send_count[d];
    } else {
        cnt = meta[2 * d];
        off = meta[2 * d + 1];
    }
    cnt = min(max(cnt, 0), m.cap);
    off = min(max(off, 0), m.cap - cnt);
}

// grid (ceil(cap / EP_RPC), world); block 256.  Forward (send_count != null):
// rows off + j of src -> rank d's x[me][j], and ids[me][j] (-1 past the
// count).  Return (send_count null): rows (d * cap + j) of src -> rank d's
// ret_y[off + j], (count, off) from this rank's meta[d].  A thread loads all
// of its float4s before it stores any (a load after a store would wait for
// the store's round trip over NVLink).  Every CTA ends with a system-scope
// fence and counts itself done; the last one raises the flags (ep_signal),
// so that the flags follow every row.
__device__ void ep_signal(const EpMail &m, uint8_t *const *peer, const int32_t *send_count,
                          unsigned long long *epoch);

__global__ void __launch_bounds__(256) k_ep_push_rows(EpMail m, uint8_t *const *peer,
                                                      const int32_t *__restrict__ send_count,
                                                      const int32_t *__restrict__ send_ids,
                                                      const float *__restrict__ src, unsigned long long *epoch,
                                                      unsigned int *done) {
    __shared__ bool s_last;
    const int d = blockIdx.y;
    const int32_t *meta = reinterpret_cast<const int32_t *>(peer[m.rank] + m.off_meta);
    int cnt, off;
    ep_block(m, d, send_count, meta, cnt, off);
    uint8_t *dst = peer[d];
    const int j0 = blockIdx.x * EP_RPC;
    const int n4 = m.n_embd / 4;
    float *out;
    const float *in;
    if (send_count) {
        int32_t *pids = reinterpret_cast<int32_t *>(dst + m.off_ids) + (size_t)m.rank * m.cap;
        for (int j = j0 + (int)threadIdx.x; j < min(j0 + EP_RPC, m.cap); j += blockDim.x)
            pids[j] = j < cnt ? send_ids[off + j] : -1;
        out = reinterpret_cast<float *>(dst + m.off_x) + (size_t)m.rank * m.cap * m.n_embd;
        in = src + (size_t)off * m.n_embd;
    } else {
        out = reinterpret_cast<float *>(dst + m.off_rety) + (size_t)off * m.n_embd;
        in = src + (size_t)d * m.cap * m.n_embd;
    }
    const int j1 = min(j0 + EP_RPC, cnt);
    const int total = max(j1 - j0, 0) * n4;   // float4s of the CTA's rows
    constexpr int PER = 8;                     // float4s in flight per thread
    for (int i0 = threadIdx.x; i0 < total; i0 += PER * blockDim.x) {
        float4 v[PER];
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int i = i0 + u * blockDim.x;
            if (i < total) {
                const int j = j0 + i / n4, c = i - (i / n4) * n4;
                v[u] = __ldcg(reinterpret_cast<const float4 *>(in + (size_t)j * m.n_embd) + c);
            }
        }
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int i = i0 + u * blockDim.x;
            if (i < total) {
                const int j = j0 + i / n4, c = i - (i / n4) * n4;
                reinterpret_cast<float4 *>(out + (size_t)j * m.n_embd)[c] = v[u];
            }
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int n = gridDim.x * gridDim.y;
        s_last = atomicAdd(done, 1u) == n - 1;
        if (s_last) *done = 0;   // for the next launch (every CTA has counted)
    }
    __syncthreads();
    if (s_last) {
        __threadfence_system();   // every CTA's rows (their fences preceded their counts) before the flags
        ep_signal(m, peer, send_count, epoch);
    }
}

// The last CTA of k_ep_push_rows.  Forward (send_count != null): thread 0
// first advances the epoch; then thread d < world writes (count, offset) of
// block d into rank d's meta[me] and the epoch into its flag_fwd[me].
// Return: the epoch into rank d's flag_ret[me].  The stores before a flag
// are the same thread's, or the other CTAs' rows, whose system-scope fences
// came before their counts.
__device__ void ep_signal(const EpMail &m, uint8_t *const *peer, const int32_t *send_count,
                          unsigned long long *epoch) {
    __shared__ unsigned long long s_e;
    if (threadIdx.x == 0) s_e = send_count ? ++*epoch : *epoch;
    __syncthreads();
    const int d = threadIdx.x;
    if (d >= m.world) return;
    uint8_t *dst = peer[d];
    if (send_count) {
        int cnt, off;
        ep_block(m, d, send_count, nullptr, cnt, off);
        int32_t *meta = reinterpret_cast<int32_t *>(dst + m.off_meta) + 2 * m.rank;
        meta[0] = cnt;
        meta[1] = off;
        st_release_sys_u64(reinterpret_cast<unsigned long long *>(dst + m.off_fflag) + m.rank, s_e);
    } else {
        st_release_sys_u64(reinterpret_cast<unsigned long long *>(dst + m.off_rflag) + m.rank, s_e);
    }
}

cudaError_t launch_ep_push(const EpMail &m, uint8_t *const *peer, const int32_t *send_count,
                           const int32_t *send_ids, const float *src, unsigned long long *epoch,
                           unsigned int *done, cudaStream_t s) {
    if (m.world > 256) return cudaErrorInvalidValue;   // one signalling thread per rank
    k_ep_push_rows<<<dim3((m.cap + EP_RPC - 1) / EP_RPC, m.world), 256, 0, s>>>(m, peer, send_count, send_ids,
                                                                                 src, epoch, done);
    return cudaGetLastError();
}

}  // namespace moe
