// p2p_reduce.cu — one-shot all-reduce of a small f32 vector across the GPUs of one node over NVLink /
// NVSwitch peer memory, for the tensor-parallel decode's two reductions per layer (a 16 KB vector:
// NCCL's per-call latency, ~18 us here, dominates at that size).
//
// Every rank owns a receive area in its own memory, mapped into every other rank's address space
// (CUDA IPC): two parity buffers of [world][max_n] floats and [2][world] flag words.  One call:
//   1. rank r stores its vector into slot r of every peer's buffer (plain stores over NVLink);
//   2. after a system-scope fence it release-stores the call's epoch into flag r of every peer;
//   3. it waits (bounded) until every peer's flag in its own area holds the same epoch;
//   4. it sums the world vectors in rank order (its own from the source) into the output.
// Every rank adds the same values in the same order, so all ranks hold identical bits.  The epoch
// is a counter in device memory advanced by the kernel itself, so a captured CUDA graph replays
// correctly; the parity of the epoch picks the buffer, which keeps a rank that runs one call ahead
// from overwriting data a peer is still reading (it cannot run two ahead: it waits for that peer's
// flag of the next call).
#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kP2pThreads = 1024;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One CTA.  areas[p]: rank p's receive area as mapped here (areas[rank] = this rank's own);
// an area = [2][world][max_n] floats followed by [2][world] ints of flags.
__global__ void __launch_bounds__(kP2pThreads, 1)
    p2p_allreduce_kernel(const P2pAreas areas, int rank, int world, int max_n, int n, const float* __restrict__ src,
                         float* __restrict__ dst, int* __restrict__ epoch_ctr, int* status) {
    __shared__ int epoch_s;
    __shared__ int ok_s;
    const int t = threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();
    if (t == 0) {
        epoch_s = *epoch_ctr + 1;
        *epoch_ctr = epoch_s;
        ok_s = 1;
    }
    __syncthreads();
    const int e = epoch_s, par = e & 1;
    const size_t slot_floats = static_cast<size_t>(max_n);
    auto data = [&](int p, int q) {  // rank p's area: buffer `par`, slot q
        return reinterpret_cast<float*>(areas.base[p]) + (static_cast<size_t>(par) * world + q) * slot_floats;
    };
    auto flags = [&](int p) {
        return reinterpret_cast<int*>(reinterpret_cast<float*>(areas.base[p]) + 2 * static_cast<size_t>(world) * slot_floats);
    };
    // 1. push this rank's vector into every peer's slot `rank`
    const int n4 = n / 4;
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        float4* d4 = reinterpret_cast<float4*>(data(p, rank));
        const float4* s4 = reinterpret_cast<const float4*>(src);
        for (int i = t; i < n4; i += kP2pThreads) d4[i] = s4[i];
        for (int i = 4 * n4 + t; i < n; i += kP2pThreads) data(p, rank)[i] = src[i];
    }
    __threadfence_system();
    __syncthreads();
    // 2. publish: flag `rank` of every peer, buffer `par`
    if (t < world && t != rank) st_release_sys(flags(t) + par * world + rank, e);
    // 3. wait for every peer's data in this rank's own area
    if (t < world && t != rank) {
        const int* f = flags(rank) + par * world + t;
        bool got = ld_acquire_sys(f) == e;
        if (!got) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 1; !got; ++i) {
                got = ld_acquire_sys(f) == e;
                if (!got && (i & 63u) == 0) {
                    if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                        set_status(status, LARQL_ERR_TIMEOUT, 90);
                        break;
                    }
                    __nanosleep(100);
                }
            }
        }
        if (!got) atomicExch(&ok_s, 0);
    }
    __syncthreads();
    if (!ok_s) return;
    // 4. sum in rank order
    for (int i = t; i < n; i += kP2pThreads) {
        float s = 0.f;
        for (int p = 0; p < world; ++p) s += (p == rank) ? src[i] : __ldcv(data(rank, p) + i);
        dst[i] = s;
    }
}

size_t p2p_area_bytes(int world, int max_n) {
    return (2 * static_cast<size_t>(world) * max_n) * sizeof(float) + 2 * static_cast<size_t>(world) * sizeof(int);
}

cudaError_t launch_p2p_allreduce(const P2pAreas& areas, int rank, int world, int max_n, int n, const float* src,
                                 float* dst, int* epoch_ctr, int* status, cudaStream_t stream) {
    if (world < 2 || world > kP2pMaxRanks || rank < 0 || rank >= world || n < 1 || n > max_n)
        return cudaErrorInvalidValue;
    cudaError_t e = launch_pdl(p2p_allreduce_kernel, dim3(1), dim3(kP2pThreads), 0, stream, areas, rank, world,
                               max_n, n, src, dst, epoch_ctr, status);
    note_launch();
    return e;
}

}  // namespace larql
