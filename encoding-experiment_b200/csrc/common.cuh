// common.cuh — shared device helpers for the sm_100a kernels: status words,
// bounded waits, mbarrier / bulk-copy PTX wrappers, f16 decode.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/larql_cuda.h"

namespace larql {

// Host-side count of the kernel launches this library has enqueued (every
// launch site calls note_launch(); larql_cuda_launch_count() reads it).
inline std::atomic<unsigned long long>& launch_counter() {
    static std::atomic<unsigned long long> c{0};
    return c;
}
inline void note_launch() { launch_counter().fetch_add(1, std::memory_order_relaxed); }

// One bit per device, set once a per-device set-up step (a kernel attribute) has
// been done there.  The bits are atomic, so host threads making their first
// launches at the same time do not race on them; both may run the step, which is
// idempotent.  Devices 64 and up are never marked (the step just runs each time).
class DeviceFlags {
  public:
    bool test(int dev) const {
        return dev >= 0 && dev < 64 && ((bits_.load(std::memory_order_acquire) >> dev) & 1ull);
    }
    void set(int dev) {
        if (dev >= 0 && dev < 64) bits_.fetch_or(1ull << dev, std::memory_order_release);
    }

  private:
    std::atomic<uint64_t> bits_{0};
};

// Runs `setup` (returning cudaError_t) once per current device, marking `flags` on success.
template <class F>
inline cudaError_t once_per_device(DeviceFlags& flags, F&& setup) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (flags.test(dev)) return cudaSuccess;
    const cudaError_t e = setup();
    if (e == cudaSuccess) flags.set(dev);
    return e;
}

constexpr int kSmemLimit = 232448;  // 227 KB of opt-in dynamic shared memory per block on sm_100

// Device-side status word: kernels record the first error they hit here and
// return; the host reads it after synchronising (larql_cuda_sync()).
// Codes are LARQL_ERR_* values; the low 16 bits of the word hold the code,
// the high bits a kernel-specific site id for diagnostics.
__device__ __forceinline__ void set_status(int* status, int code, int site) {
    if (status) atomicCAS(status, 0, (site << 16) | code);
}

// Budget for every spin-wait on an mbarrier: a kernel that has not seen its
// barrier complete after this many nanoseconds records LARQL_ERR_TIMEOUT and
// stops waiting (the copies of a matvec finish in microseconds).
constexpr uint64_t kWaitBudgetNs = 200ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the warp is parked until the phase
// completes (or the hint elapses) instead of spinning on the shared-memory
// pipe that producers and consumers need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (after recording
// LARQL_ERR_TIMEOUT at `site`) if the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, 1000000u)) return true;
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, LARQL_ERR_TIMEOUT, site);
            return false;
        }
    }
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait that polls without suspending (for pipelines whose stages hand
// over every few hundred cycles, where a suspended thread wakes up too late).
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* status, int site) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, LARQL_ERR_TIMEOUT, site);
            return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load of the box at element coordinates (x, y) of `map` into
// this CTA's shared memory, completing on `bar`.  x * element size must be a
// multiple of 16 bytes; dst 128-byte aligned.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// L2 prefetch of the box at (x, y) of `map` (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait until the previous kernel's results are visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with programmatic stream serialization (the kernel calls pdl_wait
// before it reads what earlier kernels wrote, and writes nothing before it).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate across the participating threads.
__device__ __forceinline__ bool named_bar_red_or(int id, int nthreads, bool pred) {
    uint32_t out;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " setp.ne.u32 q, %1, 0;\n"
        " bar.red.or.pred p, %2, %3, q;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
        : "memory");
    return out != 0;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}

// Exact small unsigned int -> float (v < 2^23) without the I2F pipe.
__device__ __forceinline__ float u2f_small(uint32_t v) {
    return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

__device__ __forceinline__ float h2f_lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
__device__ __forceinline__ float h2f_hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

}  // namespace larql
