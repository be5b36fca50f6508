// lm_head.cu — top-k of a logits vector by signed value, the selection step of
// VectorIndex::lm_head_knn_backend (crates/larql-vindex/src/index/walk.rs:549-583): after the Q4_0 x Q8
// matvec of the lm head (walk.rs:562-565, q4_dot.c:169-199 on the device), the reference collects
// (token id, logit) pairs, keeps the k largest logits with select_nth_unstable_by and sorts them descending
// (walk.rs:566-577).  Here: logits descending, equal logits by lower token id (the reference's order of exact
// ties is unspecified), NaN logits (on which the reference's partial_cmp().unwrap() panics) below -inf.
//
// Two launches, both reading the logits once:
//   1. logit_topk_partial_kernel: every warp walks a contiguous range of the logits 32 at a time and keeps its
//      best k in a warp-sorted list, one entry per lane (lane 0 best).  A batch of 32 candidates costs one
//      ballot against the list's k-th entry; the rare candidates that beat it are inserted one by one (a
//      ballot for the insertion point and a shuffle-up of the tail).  Each warp writes its k entries.
//   2. logit_topk_final_kernel: one CTA of 32 warps does the same over the partial lists, then warp 0 merges
//      the 32 warp lists and writes (token id, logit) pairs, the logit read back from the vector.
// An entry is a 64-bit key: the logit's order-preserving u32 image in the high half, the bit-inverted token id
// in the low half, so one unsigned compare orders by logit and then by lower id; 0 is an empty slot.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

namespace {

constexpr int kTkThreads = 256;    // stage 1: 8 warps per CTA
constexpr int kTkFinalWarps = 32;  // stage 2: one CTA of 1024 threads
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

// Offers one candidate per lane to the warp-sorted list `list` (lane i holds the i-th best entry; only the
// first k lanes matter).  Entries are distinct (token ids are), except empty slots, which never win.
__device__ __forceinline__ void warp_offer(uint64_t& list, uint64_t cand, int k, int lane) {
    uint64_t thr = __shfl_sync(kFull, list, k - 1);
    unsigned m = __ballot_sync(kFull, cand > thr);
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

__global__ void __launch_bounds__(kTkThreads) logit_topk_partial_kernel(const float* __restrict__ logits, int n,
                                                                         int k, int per_warp,
                                                                         uint64_t* __restrict__ part) {
    const int lane = threadIdx.x & 31;
    const int w = blockIdx.x * (kTkThreads / 32) + (threadIdx.x >> 5);
    const long long b0 = static_cast<long long>(w) * per_warp;
    if (b0 >= n) return;  // surplus warps of the last CTA: no range, no list slot
    const long long b1 = min(b0 + per_warp, static_cast<long long>(n));
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
    if (lane < k) part[static_cast<size_t>(w) * k + lane] = list;
}

__global__ void __launch_bounds__(32 * kTkFinalWarps) logit_topk_final_kernel(const uint64_t* __restrict__ part,
                                                                               int nparts, int k,
                                                                               const float* __restrict__ logits,
                                                                               uint32_t* __restrict__ out_id,
                                                                               float* __restrict__ out_logit) {
    __shared__ uint64_t lists[kTkFinalWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int per = (nparts + kTkFinalWarps - 1) / kTkFinalWarps;
    const int b0 = w * per, b1 = min(b0 + per, nparts);
    uint64_t list = 0;
    for (int base = b0; base < b1; base += 32) {
        const int i = base + lane;
        warp_offer(list, i < b1 ? part[i] : 0ull, k, lane);
    }
    lists[w][lane] = lane < k ? list : 0ull;
    __syncthreads();
    if (w != 0) return;
    list = lists[0][lane];
    for (int j = 1; j < kTkFinalWarps; ++j) warp_offer(list, lists[j][lane], k, lane);
    if (lane < k) {
        const uint32_t id = ~static_cast<uint32_t>(list);
        out_id[lane] = id;
        out_logit[lane] = logits[id];  // the logit itself (a -0 or a NaN keeps its bits)
    }
}

}  // namespace

// Entries of partial lists the two launches exchange (the caller's scratch holds this many uint64).
size_t logit_topk_scratch_entries(int n, int k, int num_sms) {
    if (n <= 0 || k <= 0) return 0;
    const long long warps = static_cast<long long>(num_sms) * (kTkThreads / 32);
    long long per = (n + warps - 1) / warps;
    per = (per + 127) / 128 * 128;
    const long long nw = (n + per - 1) / per;
    return static_cast<size_t>(nw) * k;
}

cudaError_t launch_logit_topk(const float* logits, int n, int k, int num_sms, uint64_t* scratch, uint32_t* out_id,
                              float* out_logit, cudaStream_t stream) {
    if (n <= 0 || k < 1 || k > 32 || k > n || num_sms < 1) return cudaErrorInvalidValue;
    const long long warps = static_cast<long long>(num_sms) * (kTkThreads / 32);
    long long per = (n + warps - 1) / warps;
    per = (per + 127) / 128 * 128;
    const int nw = static_cast<int>((n + per - 1) / per);
    const int wpb = kTkThreads / 32;
    const int blocks = (nw + wpb - 1) / wpb;
    logit_topk_partial_kernel<<<blocks, kTkThreads, 0, stream>>>(logits, n, k, static_cast<int>(per), scratch);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    logit_topk_final_kernel<<<1, 32 * kTkFinalWarps, 0, stream>>>(scratch, nw * k, k, logits, out_id, out_logit);
    note_launch();
    return cudaGetLastError();
}

}  // namespace larql
