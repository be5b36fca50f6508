// prefill_tc.cu — batched prefill dequant-GEMM on tcgen05 tensor cores:
// Y[tokens][N] = X[tokens][K] . W[N][K]^T with W in LARQL Q4_K, plus the fused
// SwiGLU form act = silu(X . Wg^T) * (X . Wu^T).
//
// Reference: the prefill FFN of ComputeBackend::prefill_q4 (crates/larql-compute/
// src/backend.rs:143-152), i.e. per token the Q4_K matvec of q4k_matvec.rs:31-87
// for gate / up / down and silu_gate_up (crates/larql-inference/src/ffn/mod.rs:87-94).
//
//  * A operand: 128 weight rows per tile, dequantized w = d*sc_j*q - dmin*mn_j
//    (times a per-matrix power of two that keeps every value inside the f16
//    range) to f16 by eight transform warps, written in the 128-byte swizzle
//    layout of a K-major UMMA operand (64 K values per row of 128 bytes).  The
//    transform reads the weight from its prefill panels, built once per weight
//    by q4k_prefill_pack_kernel: per 128-row tile and super-block, the f16 pairs
//    (d*sc_j, -dmin*mn_j) and the nibbles stored word-major across the 128 rows,
//    so every load of a transform warp covers consecutive addresses.
//  * B operand: the tokens' activations as f16 with a per-token power of two,
//    prepared once per call, streamed by TMA (SWIZZLE_128B) in a 3-stage ring.
//  * One thread issues tcgen05.mma.kind::f16 (M128 x N x K16, f32 accumulate in
//    TMEM); in the SwiGLU form the gate and up tiles of the same rows use two
//    accumulators and the epilogue writes silu(g) * u directly.
//  * Epilogue warps read TMEM (lane = weight row, column = token) and write f32
//    rows of Y / act, coalesced across lanes.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kPfXformWarps = 8;  // transform warps (two threads per weight row)
constexpr int kPfDepth = 3;       // K blocks of weight words loaded ahead per transform thread
constexpr int kPfThreads = 32 * (2 + kPfXformWarps + 4);  // producer, MMA issuer, transform, 4 epilogue
constexpr int kPfM = 128;        // weight rows per tile (MMA M, TMEM lanes)
constexpr int kPfKB = 64;        // K per block (one 128-byte swizzle row)
constexpr int kPfMaxStages = 6;  // B (activation) ring depth bound (plan field nst)
constexpr int kPfMaxABuf = 4;    // A (dequantized weight) ring depth bound (plan field nab)
constexpr int kPfATile = kPfM * kPfKB * 2;  // 16 KB per weight per buffer
constexpr int kPfPanel = 8 * kPfM * 4 + 8 * kPfM * 16;  // 20 KB per (row tile, super-block) panel

__device__ __forceinline__ uint64_t pf_sw128_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;          // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;  // SBO: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;          // version
    d |= static_cast<uint64_t>(2) << 61;          // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void pf_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void pf_tmem_ld8(uint32_t ta, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
}

// ───────────────────────── per-call preparation ─────────────────────────

// One block per token row r < rows (padding rows zero): xh[r][:] = f16(x * 2^-e)
// in the permuted K order below, xs[r] = 2^e with |x * 2^-e| < 2^14 (NaN scale
// for a non-finite row).  K is a multiple of 256; a 16-byte aligned row is read
// as float4 pairs and written as one 16-byte group of 8 halves.
__global__ void prefill_x_prep_kernel(const float* __restrict__ x, int M, int K, int rows, __half* __restrict__ xh,
                                      float* __restrict__ xs) {
    const int r = blockIdx.x;
    __shared__ float red[32];
    __shared__ int bad_s;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) bad_s = 0;
    const float* row = x + static_cast<size_t>(r) * K;
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
    const int ng = K / 8;  // groups of 8 values
    float amax = 0.f;
    bool bad = false;
    if (r < M) {
        if (vec) {
            const float4* row4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
            for (int g = threadIdx.x; g < ng; g += blockDim.x) {
                const float4 a = row4[2 * g], b = row4[2 * g + 1];
                const float m = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                                      fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
                amax = fmaxf(amax, m);
                bad |= !(isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w) && isfinite(b.x) &&
                         isfinite(b.y) && isfinite(b.z) && isfinite(b.w));
            }
        } else {
            for (int k = threadIdx.x; k < K; k += blockDim.x) {
                const float v = row[k];
                amax = fmaxf(amax, fabsf(v));
                bad |= !isfinite(v);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    if (bad) bad_s = 1;
    __syncthreads();
    if (threadIdx.x < 32) {
        float a = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (threadIdx.x == 0) red[0] = a;
    }
    __syncthreads();
    const int ex = static_cast<int>((__float_as_uint(red[0]) >> 23) & 0xFFu) - 126;
    const int e = min(100, max(-100, ex - 14));
    const float down = __int_as_float((127 - e) << 23);
    const bool zero = !(r < M && !bad_s);
    // K order inside every group of 8 values: 0 4 1 5 2 6 3 7 (the order the weight
    // transform unpacks nibbles in; the GEMM sums over K, so both sides just agree)
    uint4* out4 = reinterpret_cast<uint4*>(xh + static_cast<size_t>(r) * K);
    if (vec || zero) {
        const float4* row4 = reinterpret_cast<const float4*>(row);
#pragma unroll 4
        for (int g = threadIdx.x; g < ng; g += blockDim.x) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (!zero) {
                a = row4[2 * g];
                b = row4[2 * g + 1];
            }
            const __half2 h0 = __halves2half2(__float2half_rn(a.x * down), __float2half_rn(b.x * down));
            const __half2 h1 = __halves2half2(__float2half_rn(a.y * down), __float2half_rn(b.y * down));
            const __half2 h2 = __halves2half2(__float2half_rn(a.z * down), __float2half_rn(b.z * down));
            const __half2 h3 = __halves2half2(__float2half_rn(a.w * down), __float2half_rn(b.w * down));
            out4[g] = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                 *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
        }
    } else {
        __half* out = xh + static_cast<size_t>(r) * K;
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const int src = (k & ~7) + ((k & 1) ? 4 : 0) + ((k & 7) >> 1);
            out[k] = __float2half_rn(row[src] * down);
        }
    }
    if (threadIdx.x == 0) xs[r] = r >= M ? 0.f : (bad_s ? __int_as_float(0x7fc00000) : __int_as_float((127 + e) << 23));
}

// Per-matrix exponent e with |w| < 2^14 * 2^e for every dequantized Q4_K value
// (|w| <= 63*15*|d| + 15*|dmin| per super-block): out = max over super-blocks.
__global__ void q4k_abs_bound_kernel(const uint8_t* __restrict__ w, size_t nsb, unsigned int* __restrict__ out) {
    float m = 0.f;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nsb;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t h = *reinterpret_cast<const uint32_t*>(w + i * 148);
        const float d = fabsf(h2f_lo(h)), dm = fabsf(h2f_hi(h));
        const float b = 945.f * d + 15.f * dm;
        if (b == b) m = fmaxf(m, b);  // NaN headers do not set the scale
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // non-negative floats order as uints
}

// Prefill panels: one thread per (row, super-block).  Panel (rt, sb) holds, for the
// rows rt*128 + r (zero past N):
//   bytes [0, 4096):      u32 [8 j][128 r] = half2(f16(d*ws * sc_j), -f16(dmin*ws * mn_j))
//   bytes [4096, 20480):  16 bytes [8 j][128 r] = the nibbles of sub-block j
// with the Q4_K field decode of q4k_matvec.rs:31-87 (6-bit scales in bytes 4..11,
// 4-bit mins in bytes 16..19, low nibble for j < 4, 16 nibble bytes per sub-block from byte 20).
__global__ void q4k_prefill_pack_kernel(const uint8_t* __restrict__ w, int N, int K, float ws,
                                        uint8_t* __restrict__ out) {
    const int nsb = K / 256;
    const size_t total = static_cast<size_t>((N + kPfM - 1) / kPfM) * kPfM * nsb;
    for (size_t idx = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(idx & (kPfM - 1));
        const size_t rest = idx >> 7;
        const int sb = static_cast<int>(rest % nsb);
        const size_t rt = rest / nsb;
        const size_t row = rt * kPfM + r;
        uint8_t* panel = out + (rt * nsb + sb) * kPfPanel;
        uint32_t* scw = reinterpret_cast<uint32_t*>(panel);
        uint4* nib = reinterpret_cast<uint4*>(panel + 8 * kPfM * 4);
        if (row < static_cast<size_t>(N)) {
            const uint8_t* b = w + row * (static_cast<size_t>(nsb) * 148) + static_cast<size_t>(sb) * 148;
            const uint32_t hdr = *reinterpret_cast<const uint32_t*>(b);
            const uint32_t s0 = *reinterpret_cast<const uint32_t*>(b + 4), s1 = *reinterpret_cast<const uint32_t*>(b + 8);
            const uint32_t mw = *reinterpret_cast<const uint32_t*>(b + 16);
            const float d = h2f_lo(hdr) * ws, dm = h2f_hi(hdr) * ws;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t sc = (((j < 4) ? s0 : s1) >> (8 * (j & 3))) & 0x3Fu;
                const uint32_t mn = (mw >> (8 * (j & 3) + 4 * (j >> 2))) & 0xFu;
                const __half2 v = __halves2half2(__float2half_rn(d * static_cast<float>(sc)),
                                                 __hneg(__float2half_rn(dm * static_cast<float>(mn))));
                scw[j * kPfM + r] = *reinterpret_cast<const uint32_t*>(&v);
                const uint32_t* q = reinterpret_cast<const uint32_t*>(b + 20 + 16 * j);
                nib[j * kPfM + r] = make_uint4(q[0], q[1], q[2], q[3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                scw[j * kPfM + r] = 0u;
                nib[j * kPfM + r] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    }
}

// ───────────────────────── the GEMM ─────────────────────────

// Stream-K schedule: the (tile, K block) units, tile-major, are split into
// gridDim.x equal contiguous ranges, one per CTA.  A CTA walks its range as
// segments of one tile each.  The segment holding K block 0 of a tile owns it.
// A tile's later parts belong to the next CTAs, which compute them at the start
// of their ranges and leave raw f32 partial sums in their workspace slot.  The
// owner reaches the tile at the end of its own range; it streams those slots
// into its (by then idle) operand rings with bulk copies, adds them in CTA order
// (a fixed order: results do not depend on timing) and writes the output.  A CTA
// has at most one non-owning segment (its first) and at most one owning segment
// with contributors (its last).
__device__ __forceinline__ long long pf_unit(const PrefillPlan& p, int c) {
    return static_cast<long long>(p.nitems) * p.nkb * c / p.grid;
}

__device__ __forceinline__ int pf_ld_acquire(const int* ptr) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
    return v;
}

__device__ __forceinline__ void pf_st_release(int* ptr, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Bounded wait for *flag == 1.
__device__ __forceinline__ bool pf_wait_flag(const int* flag, int* status, int site) {
    if (pf_ld_acquire(flag) == 1) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (pf_ld_acquire(flag) == 1) return true;
        if ((i & 63u) == 0) {
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                set_status(status, LARQL_ERR_TIMEOUT, site);
                return false;
            }
            __nanosleep(64);
        }
    }
}

// Ring position: slot index and the parity of its current use.
struct PfRing {
    int slot = 0, n = 0;
    uint32_t phase = 0;
    __device__ __forceinline__ void next(int size) {
        if (++slot == size) {
            slot = 0;
            phase ^= 1u;
        }
        ++n;
    }
};

constexpr int kPfFixTok = 16;                       // tokens per fixup piece
constexpr int kPfFixBytes = kPfFixTok * kPfM * 4;   // bytes per matrix per piece
constexpr int kPfFixBufs = 8;                       // fixup staging buffers (at most)

template <int FUSED>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t* __restrict__ w0,
                        const uint8_t* __restrict__ w1, float wscale0, float wscale1, const float* __restrict__ xs,
                        float* __restrict__ y, float* __restrict__ part, int* __restrict__ flags, const PrefillPlan p,
                        int* status) {
    constexpr int NW = FUSED ? 2 : 1;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int btile = p.NTOK * kPfKB * 2;  // activation bytes per stage
    const int nst = p.nst, nab = p.nab;
    uint8_t* abuf = smem;                            // [nab][NW][16 KB]
    uint8_t* bring = smem + nab * NW * kPfATile;     // [nst][btile]
    const int ring_bytes = nab * NW * kPfATile + nst * btile;
    uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + ring_bytes);
    uint64_t* bempty = bfull + nst;
    uint64_t* afull = bempty + nst;   // [nab] transform -> MMA (one arrive per transform warp)
    uint64_t* aempty = afull + nab;   // [nab] MMA commit -> transform
    uint64_t* dfull = aempty + nab;   // MMA commit -> epilogue
    uint64_t* dempty = dfull + 1;     // epilogue (4 warps) -> MMA
    uint64_t* fxfull = dempty + 1;    // [kPfFixBufs] fixup pieces landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fxfull + kPfFixBufs);
    volatile int* abortv = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < nst; ++i) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        for (int i = 0; i < nab; ++i) {
            mbar_init(&afull[i], kPfXformWarps);
            mbar_init(&aempty[i], 1);
        }
        mbar_init(dfull, 1);
        mbar_init(dempty, 4);
        for (int i = 0; i < kPfFixBufs; ++i) mbar_init(&fxfull[i], 1);
        *abortv = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int nkb = p.nkb;
    const long long ubeg = pf_unit(p, blockIdx.x), uend = pf_unit(p, blockIdx.x + 1);
    // segment of this CTA starting at unit u: tile, K blocks [kb0, kb1)
#define PF_SEGMENT(u, tile, kb0, kb1)                                                   \
    const int tile = static_cast<int>((u) / nkb);                                      \
    const int kb0 = static_cast<int>((u) - static_cast<long long>(tile) * nkb);         \
    const int kb1 = static_cast<int>(min(static_cast<long long>(nkb), uend - static_cast<long long>(tile) * nkb))

    // Waits: the MMA issuer polls (its operands turn ready every few hundred cycles); every other role
    // waits with the suspending try_wait, leaving the issue slots to the warps doing work.
    if (warp == 0) {
        // ───── producer: activation tiles (written by the prep kernel before this one) ─────
        if (lane == 0) {
            pdl_wait();
            PfRing rb;
            bool ok = true;
            for (long long u = ubeg; u < uend && ok;) {
                PF_SEGMENT(u, tile, kb0, kb1);
                const int tt = tile % p.ntt;
                for (int kb = kb0; kb < kb1; ++kb, rb.next(nst)) {
                    if (*abortv || (rb.n >= nst && !mbar_wait(&bempty[rb.slot], rb.phase ^ 1u, status, 61))) {
                        ok = false;
                        *abortv = 1;
                        break;
                    }
                    uint8_t* dst = bring + rb.slot * btile;
                    mbar_arrive_expect_tx(&bfull[rb.slot], static_cast<uint32_t>(btile));
                    for (int h = 0; h < (p.NTOK + 255) / 256; ++h)
                        tma_load_2d(dst + h * 256 * 128, &xmap, kb * kPfKB, tt * p.NTOK + 256 * h, &bfull[rb.slot]);
                }
                u = static_cast<long long>(tile) * nkb + kb1;
            }
            // drain: every issued load has landed before the CTA may exit
            for (int j = max(0, rb.n - nst); j < rb.n; ++j)
                if (!mbar_wait(&bfull[j % nst], (j / nst) & 1, status, 62)) break;
        }
    } else if (warp == 1) {
        // ───── MMA issuer ─────
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(p.NTOK >> 3) << 17) |
                                   (static_cast<uint32_t>(kPfM >> 4) << 24);
            const uint64_t db0 = pf_sw128_desc(smem_u32(bring)), da0 = pf_sw128_desc(smem_u32(abuf));
            PfRing rb, ra;
            int it = 0;
            bool ok = true;
            for (long long u = ubeg; u < uend && ok; ++it) {
                PF_SEGMENT(u, tile, kb0, kb1);
                if (it >= 1 && !mbar_wait(dempty, (it - 1) & 1, status, 63)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (*abortv || !mbar_wait_spin(&bfull[rb.slot], rb.phase, status, 64) ||
                        !mbar_wait_spin(&afull[ra.slot], ra.phase, status, 65)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    // descriptor start addresses advance in 16-byte units
                    const uint64_t db = db0 + static_cast<uint64_t>((rb.slot * btile) >> 4);
#pragma unroll
                    for (int wsel = 0; wsel < NW; ++wsel) {
                        const uint64_t da = da0 + static_cast<uint64_t>(((ra.slot * NW + wsel) * kPfATile) >> 4);
                        const uint32_t dt = tmem + static_cast<uint32_t>(wsel * p.NTOK);
#pragma unroll
                        for (int kk = 0; kk < kPfKB / 16; ++kk) {
                            const uint64_t off = static_cast<uint64_t>(kk * 2);  // +32 bytes
                            const uint32_t acc = (kb != kb0) || (kk != 0);
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(dt),
                                "l"(da + off), "l"(db + off), "r"(idesc), "r"(acc)
                                : "memory");
                        }
                    }
                    pf_commit(&bempty[rb.slot]);
                    pf_commit(&aempty[ra.slot]);
                    rb.next(nst);
                    ra.next(nab);
                }
                if (ok) pf_commit(dfull);
                u = static_cast<long long>(tile) * nkb + kb1;
            }
            if (!ok) *abortv = 1;
        }
    } else if (warp < 2 + kPfXformWarps) {
        // ───── transform: two threads per weight row, one 32-value sub-block each ─────
        // The 5 panel words a sub-block needs (scale/min pair, 4 nibble words) are
        // loaded kPfDepth K blocks ahead into a register queue.
        const int t = tid - 64;  // 0..255
        const int rr = t & (kPfM - 1), half = t >> 7;
        const int nsb = p.K / 256;
        PfRing ra;
        bool ok = true;
        for (long long u = ubeg; u < uend && ok;) {
            PF_SEGMENT(u, tile, kb0, kb1);
            const int rt = tile / p.ntt;
            uint32_t qd[kPfDepth][NW][5];
            auto load = [&](int kb, uint32_t (&dst)[NW][5]) {
                const int sb = kb >> 2, j = 2 * (kb & 3) + half;
#pragma unroll
                for (int wsel = 0; wsel < NW; ++wsel) {
                    const uint8_t* pan =
                        (wsel ? w1 : w0) + (static_cast<size_t>(rt) * nsb + sb) * static_cast<size_t>(kPfPanel);
                    if (kb < kb1) {
                        dst[wsel][0] = __ldg(reinterpret_cast<const uint32_t*>(pan + (j * kPfM + rr) * 4));
                        const uint4 v = __ldg(reinterpret_cast<const uint4*>(pan + 8 * kPfM * 4 + (j * kPfM + rr) * 16));
                        dst[wsel][1] = v.x;
                        dst[wsel][2] = v.y;
                        dst[wsel][3] = v.z;
                        dst[wsel][4] = v.w;
                    } else {
#pragma unroll
                        for (int i = 0; i < 5; ++i) dst[wsel][i] = 0;
                    }
                }
            };
#pragma unroll
            for (int dq = 0; dq < kPfDepth; ++dq) load(kb0 + dq, qd[dq]);
            // unrolled by the queue depth: buffer uq is consumed, then refilled with the block
            // kPfDepth ahead, so no register waits on a load still in flight
            for (int kbs = kb0; kbs < kb1 && ok; kbs += kPfDepth) {
#pragma unroll
                for (int uq = 0; uq < kPfDepth; ++uq) {
                    const int kb = kbs + uq;
                    if (kb >= kb1 || !ok) break;
                    if (ra.n >= nab) {
                        const bool got = !*abortv && mbar_wait(&aempty[ra.slot], ra.phase ^ 1u, status, 66);
                        if (!__all_sync(0xffffffffu, got)) {
                            ok = false;
                            break;
                        }
                    }
#pragma unroll
                    for (int wsel = 0; wsel < NW; ++wsel) {
                        const uint32_t smw = qd[uq][wsel][0];
                        const __half2 smh = *reinterpret_cast<const __half2*>(&smw);
                        const __half2 sc = __low2half2(smh), nmn = __high2half2(smh);
                        const __half2 k1024 = __float2half2_rn(1024.f);
                        uint32_t packed[16];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            // nibble word i: elements 8i..8i+7 of the sub-block.  (w >> 4s) & 0x000F000F
                            // | 0x64006400 is the half2 (1024 + e[s], 1024 + e[s + 4]) of nibbles s, s+4.
                            const uint32_t wq = qd[uq][wsel][1 + i];
#pragma unroll
                            for (int s2 = 0; s2 < 4; ++s2) {
                                const uint32_t bits = ((wq >> (4 * s2)) & 0x000F000Fu) | 0x64006400u;
                                const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&bits), k1024);
                                const __half2 wv = __hfma2(sc, qv, nmn);
                                packed[4 * i + s2] = *reinterpret_cast<const uint32_t*>(&wv);
                            }
                        }
                        // 32 f16 = chunks 4h..4h+3 of the row's 8; chunk c of row rr goes to c ^ (rr & 7)
                        uint8_t* dst = abuf + (ra.slot * NW + wsel) * kPfATile + rr * 128;
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const int c = 4 * half + c4;
                            *reinterpret_cast<uint4*>(dst + ((c ^ (rr & 7)) * 16)) =
                                make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2], packed[4 * c4 + 3]);
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[ra.slot]);
                    load(kb + kPfDepth, qd[uq]);
                    ra.next(nab);
                }
            }
            u = static_cast<long long>(tile) * nkb + kb1;
        }
        if (!ok) *abortv = 1;
    } else {
        // ───── epilogue: lane = weight row, columns = tokens ─────
        pdl_wait();
        const int q = warp & 3;  // TMEM lanes 32q..32q+31
        const int r = q * 32 + lane;
        const size_t slot_floats = static_cast<size_t>(NW) * p.NTOK * kPfM;
        // 1 / wscale is an exact power of two: s * inv == s / wscale
        const float inv0 = 1.0f / wscale0, inv1 = 1.0f / wscale1;
        int it = 0;
        bool ok = true;
        for (long long u = ubeg; u < uend; ++it) {
            PF_SEGMENT(u, tile, kb0, kb1);
            u = static_cast<long long>(tile) * nkb + kb1;
            const int rt = tile / p.ntt, tt = tile % p.ntt;
            const int row = rt * kPfM + r;
            // one verdict for all four warps (the fixup below synchronises them on barrier 1)
            const bool got = ok && !*abortv && mbar_wait(dfull, it & 1, status, 67);
            ok = !named_bar_red_or(1, 128, !got);
            if (!ok) continue;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16);
            // the tile's token scales: lane l holds tokens 8l..8l+7 (scaled by 1 / wscale)
            float xr0[8], xr1[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int tok = tt * p.NTOK + 8 * lane + i;
                const float v = (8 * lane < p.NTOK && tok < p.M) ? xs[tok] : 0.f;
                xr0[i] = v * inv0;
                xr1[i] = v * inv1;
            }
            // final values of 8 tokens c*8.. of this row from accumulators a0 (and a1)
            auto emit = [&](int c, const float (&a0)[8], const float (&a1)[8]) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int tok = tt * p.NTOK + c * 8 + i;
                    const float s0 = __shfl_sync(0xffffffffu, xr0[i], c);
                    float out;
                    if (FUSED) {
                        const float s1 = __shfl_sync(0xffffffffu, xr1[i], c);
                        const float g = a0[i] * s0, uu = a1[i] * s1;
                        // silu(g) * u.  The approximate divide: with the correctly rounded reciprocal the
                        // epilogue took ~25 us per 256-token tile (measured), holding the accumulator the next
                        // tile's MMAs wait for; this form ~5 us
                        out = __fdividef(g, 1.0f + __expf(-g)) * uu;
                    } else {
                        out = a0[i] * s0;
                    }
                    if (tok < p.M && row < p.N) y[static_cast<size_t>(tok) * p.N + row] = out;
                }
            };
            const long long tile_end = static_cast<long long>(tile + 1) * nkb;
            if (kb0 != 0) {
                // not the owner: raw partial sums to this CTA's slot [NW][NTOK][128], then the flag
                float* slot = part + blockIdx.x * slot_floats + r;
#pragma unroll 1
                for (int c = 0; c < p.NTOK / 8; ++c) {
                    uint32_t v0[8], v1[8];
                    pf_tmem_ld8(ta + static_cast<uint32_t>(c * 8), v0);
                    if (FUSED) pf_tmem_ld8(ta + static_cast<uint32_t>(p.NTOK + c * 8), v1);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        slot[static_cast<size_t>(c * 8 + i) * kPfM] = __uint_as_float(v0[i]);
                        if (FUSED) slot[static_cast<size_t>(p.NTOK + c * 8 + i) * kPfM] = __uint_as_float(v1[i]);
                    }
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) pf_st_release(&flags[blockIdx.x * 4 + q], 1);
            } else if (uend >= tile_end) {
                // the whole tile is this CTA's
#pragma unroll 1
                for (int c = 0; c < p.NTOK / 8; ++c) {
                    uint32_t v0[8], v1[8];
                    pf_tmem_ld8(ta + static_cast<uint32_t>(c * 8), v0);
                    if (FUSED) pf_tmem_ld8(ta + static_cast<uint32_t>(p.NTOK + c * 8), v1);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    float a0[8], a1[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        a0[i] = __uint_as_float(v0[i]);
                        a1[i] = FUSED ? __uint_as_float(v1[i]) : 0.f;
                    }
                    emit(c, a0, a1);
                }
            } else {
                // owner with contributors (this CTA's last segment: every MMA has completed, so
                // the operand rings are free).  Contributor slots are streamed in pieces of
                // kPfFixTok tokens into ring buffers; piece j = (token group pc, contributor ci).
                int clast = blockIdx.x;
                while (clast + 1 < static_cast<int>(gridDim.x) && pf_unit(p, clast + 1) < tile_end) ++clast;
                const int ncon = clast - static_cast<int>(blockIdx.x);
                const int npc = p.NTOK / kPfFixTok, J = npc * ncon;
                const int piece_bytes = NW * kPfFixBytes;
                const int R = min(kPfFixBufs, ring_bytes / piece_bytes);
                const bool issuer = (q == 0 && lane == 0);
                auto issue = [&](int j) {
                    const int pc = j / ncon, cc = static_cast<int>(blockIdx.x) + 1 + j % ncon;
                    uint8_t* dst = smem + (j % R) * piece_bytes;
                    mbar_arrive_expect_tx(&fxfull[j % R], static_cast<uint32_t>(piece_bytes));
#pragma unroll
                    for (int w = 0; w < NW; ++w)
                        bulk_g2s(dst + w * kPfFixBytes,
                                 part + cc * slot_floats + static_cast<size_t>(w * p.NTOK + pc * kPfFixTok) * kPfM,
                                 kPfFixBytes, &fxfull[j % R]);
                };
                bool bad = false;
                if (issuer) {
                    for (int cc = blockIdx.x + 1; cc <= clast && !bad; ++cc)
                        for (int w = 0; w < 4 && !bad; ++w) bad = !pf_wait_flag(&flags[cc * 4 + w], status, 68);
                    if (!bad) {
                        // the slots were written through the generic proxy; the bulk copies read them
                        // through the async proxy
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        for (int cc = blockIdx.x + 1; cc <= clast; ++cc)
                            for (int w = 0; w < 4; ++w) flags[cc * 4 + w] = 0;  // consumed: ready for the next launch
                        for (int j = 0; j < min(R, J); ++j) issue(j);
                    }
                }
                ok = !named_bar_red_or(1, 128, bad) && ok;
                if (ok) {
                    const float* ring_f = reinterpret_cast<const float*>(smem);
#pragma unroll 1
                    for (int pc = 0; pc < npc && ok; ++pc) {
                        float s0[kPfFixTok], s1[kPfFixTok];
#pragma unroll
                        for (int t2 = 0; t2 < kPfFixTok; ++t2) s0[t2] = s1[t2] = 0.f;
#pragma unroll 1
                        for (int ci = 0; ci < ncon; ++ci) {
                            const int j = pc * ncon + ci, b = j % R;
                            const bool got = mbar_wait(&fxfull[b], (j / R) & 1, status, 69);
                            if (named_bar_red_or(1, 128, !got)) {
                                ok = false;
                                break;
                            }
                            const float* sp = ring_f + b * (piece_bytes / 4) + r;
#pragma unroll
                            for (int t2 = 0; t2 < kPfFixTok; ++t2) {
                                s0[t2] += sp[t2 * kPfM];
                                if (FUSED) s1[t2] += sp[kPfFixBytes / 4 + t2 * kPfM];
                            }
                            named_bar_sync(1, 128);  // buffer b is read by all four warps
                            if (issuer && j + R < J) {
                                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                                issue(j + R);
                            }
                        }
                        if (!ok) break;
#pragma unroll
                        for (int c2 = 0; c2 < kPfFixTok / 8; ++c2) {
                            const int c = pc * (kPfFixTok / 8) + c2;
                            uint32_t v0[8], v1[8];
                            pf_tmem_ld8(ta + static_cast<uint32_t>(c * 8), v0);
                            if (FUSED) pf_tmem_ld8(ta + static_cast<uint32_t>(p.NTOK + c * 8), v1);
                            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                            float a0[8], a1[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i) {
                                a0[i] = __uint_as_float(v0[i]) + s0[c2 * 8 + i];
                                a1[i] = FUSED ? __uint_as_float(v1[i]) + s1[c2 * 8 + i] : 0.f;
                            }
                            emit(c, a0, a1);
                        }
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty);
        }
        if (!ok) *abortv = 1;
    }
#undef PF_SEGMENT

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// ───────────────────────── host side ─────────────────────────

bool prefill_make_plan(int N, int K, int M, bool fused, int num_sms, PrefillPlan* out) {
    if (N < 1 || M < 1 || K < 256 || K % 256) return false;
    PrefillPlan p{};
    p.N = N;
    p.K = K;
    p.M = M;
    p.fused = fused ? 1 : 0;
    p.nrt = (N + kPfM - 1) / kPfM;
    p.nkb = K / kPfKB;
    // tokens per tile: 256 (the stream-K schedule keeps every SM busy whatever the tile count)
    p.NTOK = 256;
    if (M <= 128) p.NTOK = M <= 64 ? 64 : 128;
    p.ntt = (M + p.NTOK - 1) / p.NTOK;
    p.nitems = p.nrt * p.ntt;
    // stream-K grid: every SM, unless that would leave a CTA fewer than 4 K blocks
    const long long units = static_cast<long long>(p.nitems) * p.nkb;
    long long g = units / 4;
    if (g < p.nitems) g = p.nitems;
    if (g > num_sms) g = num_sms;
    p.grid = static_cast<int>(g);
    // ring depths: as many A buffers (up to 4) and activation stages (up to 6) as shared memory holds
    const int nw = fused ? 2 : 1;
    const int abytes = nw * kPfATile, bbytes = p.NTOK * kPfKB * 2, fixed = 512 + 1024;
    p.nab = 2;
    p.nst = 2;
    for (bool grew = true; grew;) {
        grew = false;
        if (p.nab < kPfMaxABuf && fixed + (p.nab + 1) * abytes + p.nst * bbytes <= kSmemLimit) {
            ++p.nab;
            grew = true;
        }
        if (p.nst < kPfMaxStages && fixed + p.nab * abytes + (p.nst + 1) * bbytes <= kSmemLimit) {
            ++p.nst;
            grew = true;
        }
    }
    p.smem = fixed + p.nab * abytes + p.nst * bbytes;
    *out = p;
    return p.smem <= kSmemLimit;
}

int prefill_tokens_padded(const PrefillPlan& p) { return p.ntt * p.NTOK; }

cudaError_t launch_q4k_abs_bound(const uint8_t* w, size_t nsb, unsigned int* out, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(unsigned int), stream);
    if (e != cudaSuccess) return e;
    const size_t b = (nsb + 255) / 256;
    q4k_abs_bound_kernel<<<static_cast<unsigned>(b < 2048 ? b : 2048), 256, 0, stream>>>(w, nsb, out);
    note_launch();
    return cudaGetLastError();
}

size_t q4k_prefill_panel_bytes(size_t N, size_t K) { return (N + kPfM - 1) / kPfM * (K / 256) * kPfPanel; }

cudaError_t launch_q4k_prefill_pack(const uint8_t* w, int N, int K, float wscale, uint8_t* out, cudaStream_t stream) {
    const size_t threads = static_cast<size_t>((N + kPfM - 1) / kPfM) * kPfM * (K / 256);
    const size_t b = (threads + 255) / 256;
    q4k_prefill_pack_kernel<<<static_cast<unsigned>(b < 8192 ? b : 8192), 256, 0, stream>>>(w, N, K, wscale, out);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_prefill_x_prep(const float* x, int M, int K, int rows, __half* xh, float* xs, cudaStream_t stream) {
    cudaError_t e = launch_pdl(prefill_x_prep_kernel, dim3(rows), dim3(256), 0, stream, x, M, K, rows, xh, xs);
    note_launch();
    return e;
}

int prefill_encode_xmap(void* encode_fn, const __half* xh, int rows, int K, int box_rows, CUtensorMap* map) {
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kPfKB), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<Fn>(encode_fn)(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(xh), dims,
                                                 strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

// Floats of the stream-K partial-sum workspace (one slot per CTA) of a plan.
size_t prefill_part_floats(const PrefillPlan& p) {
    return static_cast<size_t>(p.grid) * (p.fused ? 2 : 1) * p.NTOK * kPfM;
}

// y [M][N] f32 = the plain or SwiGLU GEMM; xmap over the prepared f16 activations
// (rows = prefill_tokens_padded, box 64 x min(256, NTOK)); wscale = 2^-e per weight;
// w0 / w1 the prefill panels; part = prefill_part_floats workspace, flags = 4 * grid
// ints, zero on entry and left zero.
cudaError_t launch_prefill_gemm(const CUtensorMap& xmap, const uint8_t* w0, const uint8_t* w1, float wscale0,
                                float wscale1, const float* xs, float* y, float* part, int* flags, const PrefillPlan& p,
                                int* status, cudaStream_t stream) {
    static DeviceFlags attr_done[2];
    const int f = p.fused ? 1 : 0;
    cudaError_t e = once_per_device(attr_done[f], [f] {
        return f ? cudaFuncSetAttribute(prefill_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit)
                 : cudaFuncSetAttribute(prefill_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    e = f ? launch_pdl(prefill_gemm_kernel<1>, dim3(p.grid), dim3(kPfThreads), p.smem, stream, xmap, w0, w1,
                                   wscale0, wscale1, xs, y, part, flags, p, status)
                      : launch_pdl(prefill_gemm_kernel<0>, dim3(p.grid), dim3(kPfThreads), p.smem, stream, xmap, w0, w1,
                                   wscale0, wscale1, xs, y, part, flags, p, status);
    note_launch();
    return e;
}

}  // namespace larql
