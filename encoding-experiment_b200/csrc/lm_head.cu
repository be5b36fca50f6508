// lm_head.cu — top-k of a logits vector by signed value, the selection step of
// VectorIndex::lm_head_knn_backend (crates/larql-vindex/src/index/walk.rs:549-583): after the Q4_0 x Q8
// matvec of the lm head (walk.rs:562-565, q4_dot.c:169-199 on the device), the reference collects
// (token id, logit) pairs, keeps the k largest logits with select_nth_unstable_by and sorts them descending
// (walk.rs:566-577).  Here: logits descending, equal logits by lower token id (the reference's order of exact
// ties is unspecified), NaN logits (on which the reference's partial_cmp().unwrap() panics) below -inf.
//
// Two launches, both reading the logits once:
//   1. logit_topk_partial_kernel: every warp walks a contiguous range of the logits 32 at a time and keeps a
//      warp-sorted list of 32 entries, one per lane (lane 0 best; its first k are the range's top k).  A batch
//      of 32 candidates costs one ballot against the list's k-th entry.  When one or two candidates beat it they
//      are inserted one by one (a ballot for the insertion point, a shuffle-up of the tail); when more do, the
//      batch is bitonic-sorted across the lanes and merged with the list (max of the list and the reversed
//      batch, then five bitonic steps), which keeps the first batches and dense stretches cheap.  One CTA of 8
//      warps per SM (warp ranges a multiple of 128 values); the CTA's 8 warp lists are merged pairwise in three
//      rounds through shared memory and the CTA writes its first k entries.
//   2. logit_topk_final_kernel: one CTA of 32 warps does the same over the CTAs' lists (five merge rounds) and
//      writes the first k entries as (token id, logit) pairs, the logit read back from the vector.
// An entry is a 64-bit key: the logit's order-preserving u32 image in the high half, the bit-inverted token id
// in the low half, so one unsigned compare orders by logit and then by lower id; 0 is an empty slot.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

namespace {

constexpr int kTkWarps1 = 8;  // stage 1: warps per CTA (one CTA per SM spreads the shuffle work)
constexpr int kTkWarps = 32;  // stage 2: one CTA of 1024 threads
constexpr unsigned kFull = 0xffffffffu;

// Order-preserving image of a float (larger value -> larger key); -0 ranks as +0 (they compare equal); every
// NaN -> 0, below -inf (0x007FFFFF).
__device__ __forceinline__ uint32_t logit_order(float v) {
    const uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
    if (v != v) return 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint64_t logit_entry(float v, uint32_t id) {
    return (static_cast<uint64_t>(logit_order(v)) << 32) | static_cast<uint32_t>(~id);
}

__device__ __forceinline__ uint64_t umax64(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

// Sorts one entry per lane descending across the warp (lane 0 largest): bitonic network, 15 exchange steps.
__device__ __forceinline__ uint64_t warp_sort_desc(uint64_t v, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint64_t o = __shfl_xor_sync(kFull, v, stride);
            const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0 || size == 32);
            v = keep_max ? umax64(v, o) : umin64(v, o);
        }
    }
    return v;
}

// The 32 largest of a descending list and a bitonic sequence c (e.g. another descending list reversed): the
// lane-wise max is bitonic and holds them; five exchange steps sort it descending.
__device__ __forceinline__ uint64_t warp_bitonic_clean(uint64_t v, int lane) {
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) {
        const uint64_t o = __shfl_xor_sync(kFull, v, stride);
        v = (lane & stride) == 0 ? umax64(v, o) : umin64(v, o);
    }
    return v;
}

// Merges the CTA's NW warp lists (lists[w] = warp w's, descending) pairwise in log2(NW) rounds; list 0 ends up
// with the 32 largest entries of all.  Every thread of the CTA calls it.
template <int NW>
__device__ __forceinline__ void cta_merge_lists(uint64_t (&lists)[NW][32], int w, int lane) {
#pragma unroll 1
    for (int half = NW / 2; half >= 1; half >>= 1) {
        uint64_t merged = 0;
        if (w < half) merged = warp_bitonic_clean(umax64(lists[w][lane], lists[w + half][31 - lane]), lane);
        __syncthreads();
        if (w < half) lists[w][lane] = merged;
        __syncthreads();
    }
}

// Offers one candidate per lane to the warp-sorted list `list` (lane i holds the i-th best entry; the first k
// lanes are the answer, the rest are real entries kept for merging).  Entries are distinct (token ids are),
// except empty slots (0), which never win.
__device__ __forceinline__ void warp_offer(uint64_t& list, uint64_t cand, int k, int lane) {
    uint64_t thr = __shfl_sync(kFull, list, k - 1);
    unsigned m = __ballot_sync(kFull, cand > thr);
    if (__popc(m) > 2) {  // dense batch: sort it and merge
        const uint64_t c = warp_sort_desc(cand > thr ? cand : 0ull, lane);
        list = warp_bitonic_clean(umax64(list, __shfl_sync(kFull, c, 31 - lane)), lane);
        return;
    }
    while (m) {
        const int src = __ffs(m) - 1;
        m &= m - 1;
        const uint64_t v = __shfl_sync(kFull, cand, src);
        if (v <= thr) continue;  // v and thr are the same in every lane
        const int pos = __popc(__ballot_sync(kFull, list > v));  // the list is descending: a prefix beats v
        const uint64_t up = __shfl_up_sync(kFull, list, 1);
        if (lane > pos) list = up;
        else if (lane == pos) list = v;
        thr = __shfl_sync(kFull, list, k - 1);
    }
}

__global__ void __launch_bounds__(32 * kTkWarps1) logit_topk_partial_kernel(const float* __restrict__ logits, int n,
                                                                             int k, int per_warp,
                                                                             uint64_t* __restrict__ part) {
    __shared__ uint64_t lists[kTkWarps1][32];
    pdl_launch_dependents();
    pdl_wait();  // the logits and `part` belong to the kernels before this one until they finish
    const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
    const long long b0 = (static_cast<long long>(blockIdx.x) * kTkWarps1 + wl) * per_warp;
    const long long b1 = min(b0 + per_warp, static_cast<long long>(n));  // b1 <= b0: a surplus warp, empty list
    uint64_t list = 0;
    // four batches of 32 loads in flight before they are offered
    for (long long base = b0; base < b1; base += 128) {
        uint64_t c[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const long long i = base + 32 * u + lane;
            c[u] = i < b1 ? logit_entry(__ldg(logits + i), static_cast<uint32_t>(i)) : 0ull;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) warp_offer(list, c[u], k, lane);
    }
    lists[wl][lane] = list;
    __syncthreads();
    cta_merge_lists<kTkWarps1>(lists, wl, lane);
    if (wl == 0 && lane < k) part[static_cast<size_t>(blockIdx.x) * k + lane] = lists[0][lane];
}

__global__ void __launch_bounds__(32 * kTkWarps) logit_topk_final_kernel(const uint64_t* __restrict__ part,
                                                                               int nparts, int k,
                                                                               const float* __restrict__ logits,
                                                                               uint32_t* __restrict__ out_id,
                                                                               float* __restrict__ out_logit) {
    __shared__ uint64_t lists[kTkWarps][32];
    pdl_launch_dependents();
    pdl_wait();  // `part`, the logits and the outputs belong to the kernels before this one until they finish
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int per = (nparts + kTkWarps - 1) / kTkWarps;
    const int b0 = w * per, b1 = min(b0 + per, nparts);
    uint64_t list = 0;
    for (int base = b0; base < b1; base += 32) {
        const int i = base + lane;
        warp_offer(list, i < b1 ? part[i] : 0ull, k, lane);
    }
    lists[w][lane] = list;
    __syncthreads();
    cta_merge_lists<kTkWarps>(lists, w, lane);
    if (w != 0) return;
    list = lists[0][lane];
    if (lane < k) {
        const uint32_t id = ~static_cast<uint32_t>(list);
        out_id[lane] = id;
        out_logit[lane] = logits[id];  // the logit itself (a -0 or a NaN keeps its bits)
    }
}

}  // namespace

// Entries of partial lists the two launches exchange (the caller's scratch holds this many uint64).
// Values per stage-1 warp: the logits spread over one CTA of 8 warps per SM, a multiple of 128.
static long long logit_topk_per_warp(int n, int num_sms) {
    const long long warps = static_cast<long long>(num_sms) * kTkWarps1;
    const long long per = (n + warps - 1) / warps;
    return (per + 127) / 128 * 128;
}

size_t logit_topk_scratch_entries(int n, int k, int num_sms) {
    if (n <= 0 || k <= 0) return 0;
    const long long per = logit_topk_per_warp(n, num_sms);
    const long long nblocks = (n + per * kTkWarps1 - 1) / (per * kTkWarps1);
    return static_cast<size_t>(nblocks) * k;
}

cudaError_t launch_logit_topk(const float* logits, int n, int k, int num_sms, uint64_t* scratch, uint32_t* out_id,
                              float* out_logit, cudaStream_t stream) {
    if (n <= 0 || k < 1 || k > 32 || k > n || num_sms < 1) return cudaErrorInvalidValue;
    const long long per = logit_topk_per_warp(n, num_sms);
    const int blocks = static_cast<int>((n + per * kTkWarps1 - 1) / (per * kTkWarps1));
    cudaError_t e = launch_pdl(logit_topk_partial_kernel, dim3(blocks), dim3(32 * kTkWarps1), 0, stream, logits, n, k,
                               static_cast<int>(per), scratch);
    note_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = launch_pdl(logit_topk_final_kernel, dim3(1), dim3(32 * kTkWarps), 0, stream, static_cast<const uint64_t*>(scratch),
                   blocks * k, k, logits, out_id, out_logit);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace larql
