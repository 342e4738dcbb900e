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

// dest[p] = the rank owning expert ids[p] (-1 for an id out of range).
__global__ void k_ep_dest(const int32_t *__restrict__ ids, int P, int n_expert, int world,
                          int32_t *__restrict__ dest) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    const int e = ids[p];
    dest[p] = (e >= 0 && e < n_expert) ? e / (n_expert / world) : -1;
}

// Send slot of the pair at grouped position q: q itself (compact), or, with
// `capacity` slots per rank, rank d's block at d * capacity + (q - off[d]).
// The pair's expert id and its token's row go to that slot, and pair_pos is
// rewritten to the slot.
__global__ void __launch_bounds__(256) k_ep_gather(const float *__restrict__ x,
                                                   const int32_t *__restrict__ ids,
                                                   const int32_t *__restrict__ pos_pair,
                                                   const int32_t *__restrict__ dest,
                                                   const int32_t *__restrict__ off,
                                                   const int32_t *__restrict__ n_valid, int k,
                                                   int n_embd, int capacity,
                                                   int32_t *__restrict__ pair_pos,
                                                   int32_t *__restrict__ send_ids,
                                                   float *__restrict__ send_x) {
    const int q = blockIdx.x;
    if (q >= *n_valid) return;
    const int p = pos_pair[q];
    int slot = q;
    if (capacity > 0) {
        const int d = dest[p];
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

// Pairs that reached a send slot: off[world] of the rank grouping.
__global__ void k_ep_count(const int32_t *__restrict__ off, int world, int32_t *__restrict__ n) {
    *n = off[world];
}

cudaError_t launch_ep_pack(const int32_t *ids, const float *x, int n_tok, int k, int n_expert,
                           int n_embd, int world, int capacity, int32_t *dest, const GroupBufs &g,
                           int32_t *send_ids, float *send_x, int *err, cudaStream_t s) {
    const int P = n_tok * k;
    if (world < 1 || world > 256 || n_expert % world || capacity < 0) return cudaErrorInvalidValue;
    if (capacity > 0) {   // every slot starts empty
        const int n = world * capacity;
        k_fill_i32<<<(n + 255) / 256, 256, 0, s>>>(send_ids, n, -1);
    }
    k_ep_dest<<<(P + 255) / 256, 256, 0, s>>>(ids, P, n_expert, world, dest);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if ((e = launch_group(dest, P, world, 0x7FFF, g, err, s)) != cudaSuccess) return e;
    k_ep_count<<<1, 1, 0, s>>>(g.off, world, g.n_tiles);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_ep_gather<<<P, 256, 0, s>>>(x, ids, g.pos_pair, dest, g.off, g.n_tiles, k, n_embd, capacity,
                                  g.pair_pos, send_ids, send_x);
    return cudaGetLastError();
}

}  // namespace moe
