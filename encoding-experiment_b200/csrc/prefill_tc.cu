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
// for a non-finite row).
__global__ void prefill_x_prep_kernel(const float* __restrict__ x, int M, int K, int rows, __half* __restrict__ xh,
                                      float* __restrict__ xs) {
    const int r = blockIdx.x;
    __shared__ float red[32];
    __shared__ int bad_s;
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) bad_s = 0;
    float amax = 0.f;
    bool bad = false;
    if (r < M)
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const float v = x[static_cast<size_t>(r) * K + k];
            amax = fmaxf(amax, fabsf(v));
            bad |= !isfinite(v);
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
    // K order inside every group of 8 values: 0 4 1 5 2 6 3 7 (the order the weight
    // transform unpacks nibbles in; the GEMM sums over K, so both sides just agree)
    __half* out = xh + static_cast<size_t>(r) * K;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const int src = (k & ~7) + ((k & 1) ? 4 : 0) + ((k & 7) >> 1);
        out[k] = __float2half_rn((r < M && !bad_s) ? x[static_cast<size_t>(r) * K + src] * down : 0.f);
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

template <int FUSED>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t* __restrict__ w0,
                        const uint8_t* __restrict__ w1, float wscale0, float wscale1, const float* __restrict__ xs,
                        float* __restrict__ y, const PrefillPlan p, int* status) {
    constexpr int NW = FUSED ? 2 : 1;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int btile = p.NTOK * kPfKB * 2;  // activation bytes per stage
    const int kPfStages = p.nst, kPfABuf = p.nab;
    uint8_t* abuf = smem;                                  // [nab][NW][16 KB]
    uint8_t* bring = smem + kPfABuf * NW * kPfATile;       // [nst][btile]
    uint64_t* bfull = reinterpret_cast<uint64_t*>(bring + kPfStages * btile);
    uint64_t* bempty = bfull + kPfStages;
    uint64_t* afull = bempty + kPfStages;   // [nab] transform -> MMA (one arrive per transform warp)
    uint64_t* aempty = afull + kPfABuf;     // [nab] MMA commit -> transform
    uint64_t* dfull = aempty + kPfABuf;     // MMA commit -> epilogue
    uint64_t* dempty = dfull + 1;           // epilogue (4 warps) -> MMA
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 1);
    volatile int* abortv = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < kPfStages; ++i) {
            mbar_init(&bfull[i], 1);
            mbar_init(&bempty[i], 1);
        }
        for (int i = 0; i < kPfABuf; ++i) {
            mbar_init(&afull[i], kPfXformWarps);
            mbar_init(&aempty[i], 1);
        }
        mbar_init(dfull, 1);
        mbar_init(dempty, 4);
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

    if (warp == 0) {
        // ───── producer: activation tiles (written by the prep kernel before this one) ─────
        if (lane == 0) {
            pdl_wait();
            int k = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x) {
                const int tt = item % p.ntt;
                for (int kb = 0; kb < nkb; ++kb, ++k) {
                    const int st = k % kPfStages;
                    if (*abortv || (k >= kPfStages &&
                                    !mbar_wait_spin(&bempty[st], ((k / kPfStages) - 1) & 1, status, 61))) {
                        ok = false;
                        *abortv = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&bfull[st], static_cast<uint32_t>(btile));
                    for (int h = 0; h < p.NTOK / 256 + (p.NTOK % 256 ? 1 : 0); ++h) {
                        const int rows = min(256, p.NTOK - 256 * h);
                        (void)rows;
                        tma_load_2d(bring + st * btile + h * 256 * 128, &xmap, kb * kPfKB, tt * p.NTOK + 256 * h,
                                    &bfull[st]);
                    }
                }
            }
            for (int j = max(0, k - kPfStages); j < k; ++j)
                if (!mbar_wait_spin(&bfull[j % kPfStages], (j / kPfStages) & 1, status, 62)) break;
        }
    } else if (warp == 1) {
        // ───── MMA issuer ─────
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(p.NTOK >> 3) << 17) |
                                   (static_cast<uint32_t>(kPfM >> 4) << 24);
            int k = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x, ++it) {
                if (it >= 1 && !mbar_wait_spin(dempty, (it - 1) & 1, status, 63)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int kb = 0; kb < nkb; ++kb, ++k) {
                    const int st = k % kPfStages, ab = k % kPfABuf;
                    if (*abortv || !mbar_wait_spin(&bfull[st], (k / kPfStages) & 1, status, 64) ||
                        !mbar_wait_spin(&afull[ab], (k / kPfABuf) & 1, status, 65)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t db = pf_sw128_desc(smem_u32(bring + st * btile));
#pragma unroll
                    for (int wsel = 0; wsel < NW; ++wsel) {
                        const uint64_t da = pf_sw128_desc(smem_u32(abuf + (ab * NW + wsel) * kPfATile));
                        const uint32_t dt = tmem + static_cast<uint32_t>(wsel * p.NTOK);
#pragma unroll
                        for (int kk = 0; kk < kPfKB / 16; ++kk) {
                            const uint64_t off = static_cast<uint64_t>(kk * 2);  // +32 bytes
                            const uint32_t acc = (kb | kk) != 0;
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(dt),
                                "l"(da + off), "l"(db + off), "r"(idesc), "r"(acc)
                                : "memory");
                        }
                    }
                    pf_commit(&bempty[st]);
                    pf_commit(&aempty[ab]);
                }
                if (ok) pf_commit(dfull);
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
        int k = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x) {
            const int rt = item / p.ntt;
            uint32_t qd[kPfDepth][NW][5];
            auto load = [&](int kb, uint32_t (&dst)[NW][5]) {
                const int sb = kb >> 2, j = 2 * (kb & 3) + half;
#pragma unroll
                for (int wsel = 0; wsel < NW; ++wsel) {
                    const uint8_t* pan =
                        (wsel ? w1 : w0) + (static_cast<size_t>(rt) * nsb + sb) * static_cast<size_t>(kPfPanel);
                    if (kb < nkb) {
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
            for (int dq = 0; dq < kPfDepth; ++dq) load(dq, qd[dq]);
            // unrolled by the queue depth: buffer u is consumed, then refilled with the block
            // kPfDepth ahead, so no register waits on a load still in flight
            for (int kb0 = 0; kb0 < nkb && ok; kb0 += kPfDepth) {
#pragma unroll
                for (int u = 0; u < kPfDepth; ++u) {
                    const int kb = kb0 + u;
                    if (kb >= nkb || !ok) break;
                    const int ab = k % kPfABuf;
                    if (k >= kPfABuf) {
                        const bool got = !*abortv && mbar_wait_spin(&aempty[ab], ((k / kPfABuf) - 1) & 1, status, 66);
                        if (!__all_sync(0xffffffffu, got)) {
                            ok = false;
                            break;
                        }
                    }
#pragma unroll
                    for (int wsel = 0; wsel < NW; ++wsel) {
                        const uint32_t smw = qd[u][wsel][0];
                        const __half2 smh = *reinterpret_cast<const __half2*>(&smw);
                        const __half2 sc = __low2half2(smh), nmn = __high2half2(smh);
                        const __half2 k1024 = __float2half2_rn(1024.f);
                        uint32_t packed[16];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            // nibble word i: elements 8i..8i+7 of the sub-block.  (w >> 4s) & 0x000F000F
                            // | 0x64006400 is the half2 (1024 + e[s], 1024 + e[s + 4]) of nibbles s, s+4.
                            const uint32_t wq = qd[u][wsel][1 + i];
#pragma unroll
                            for (int s2 = 0; s2 < 4; ++s2) {
                                const uint32_t bits = ((wq >> (4 * s2)) & 0x000F000Fu) | 0x64006400u;
                                const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&bits), k1024);
                                const __half2 wv = __hfma2(sc, qv, nmn);
                                packed[4 * i + s2] = *reinterpret_cast<const uint32_t*>(&wv);
                            }
                        }
                        // 32 f16 = chunks 4h..4h+3 of the row's 8; chunk c of row rr goes to c ^ (rr & 7)
                        uint8_t* dst = abuf + (ab * NW + wsel) * kPfATile + rr * 128;
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            const int c = 4 * half + c4;
                            *reinterpret_cast<uint4*>(dst + ((c ^ (rr & 7)) * 16)) =
                                make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2], packed[4 * c4 + 3]);
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&afull[ab]);
                    load(kb + kPfDepth, qd[u]);
                    ++k;
                }
            }
        }
        if (!ok) *abortv = 1;
    } else {
        // ───── epilogue: lane = weight row, columns = tokens ─────
        pdl_wait();
        const int q = warp & 3;
        const int r = q * 32 + lane;
        int it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < p.nitems; item += gridDim.x, ++it) {
            const int rt = item / p.ntt, tt = item % p.ntt;
            const int row = rt * kPfM + r;
            if (ok) {
                const bool got = !*abortv && mbar_wait_spin(dfull, it & 1, status, 67);
                ok = __all_sync(0xffffffffu, got);
            }
            if (!ok) continue;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < p.NTOK / 8; ++c) {
                uint32_t v0[8], v1[8];
                pf_tmem_ld8(ta + static_cast<uint32_t>(c * 8), v0);
                if (FUSED) pf_tmem_ld8(ta + static_cast<uint32_t>(p.NTOK + c * 8), v1);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int tok = tt * p.NTOK + c * 8 + i;
                    if (tok < p.M && row < p.N) {
                        const float s = xs[tok];
                        float out;
                        if (FUSED) {
                            const float g = __uint_as_float(v0[i]) * (s / wscale0);
                            const float u = __uint_as_float(v1[i]) * (s / wscale1);
                            out = g * (1.0f / (1.0f + expf(-g))) * u;
                        } else {
                            out = __uint_as_float(v0[i]) * (s / wscale0);
                        }
                        y[static_cast<size_t>(tok) * p.N + row] = out;
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(dempty);
        }
        if (!ok) *abortv = 1;
    }

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
    // tokens per tile: 256 when that still gives every SM work, else 128
    p.NTOK = 256;
    if (p.nrt * ((M + 255) / 256) < num_sms && M > 128) p.NTOK = 128;
    if (M <= 128) p.NTOK = M <= 64 ? 64 : 128;
    p.ntt = (M + p.NTOK - 1) / p.NTOK;
    p.nitems = p.nrt * p.ntt;
    p.grid = p.nitems < num_sms ? p.nitems : num_sms;
    // ring depths: as many A buffers (up to 4) and activation stages (up to 6) as shared memory holds
    const int nw = fused ? 2 : 1;
    const int abytes = nw * kPfATile, bbytes = p.NTOK * kPfKB * 2, fixed = 256 + 1024;
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

// y [M][N] f32 = the plain or SwiGLU GEMM; xmap over the prepared f16 activations
// (rows = prefill_tokens_padded, box 64 x min(256, NTOK)); wscale = 2^-e per weight.
cudaError_t launch_prefill_gemm(const CUtensorMap& xmap, const uint8_t* w0, const uint8_t* w1, float wscale0,
                                float wscale1, const float* xs, float* y, const PrefillPlan& p, int* status,
                                cudaStream_t stream) {
    static uint64_t attr_mask[2] = {0, 0};
    int dev = 0;
    cudaGetDevice(&dev);
    const int f = p.fused ? 1 : 0;
    if (!((attr_mask[f] >> dev) & 1)) {
        cudaError_t e = f ? cudaFuncSetAttribute(prefill_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit)
                          : cudaFuncSetAttribute(prefill_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) return e;
        attr_mask[f] |= 1ull << dev;
    }
    cudaError_t e = f ? launch_pdl(prefill_gemm_kernel<1>, dim3(p.grid), dim3(kPfThreads), p.smem, stream, xmap, w0, w1,
                                   wscale0, wscale1, xs, y, p, status)
                      : launch_pdl(prefill_gemm_kernel<0>, dim3(p.grid), dim3(kPfThreads), p.smem, stream, xmap, w0, w1,
                                   wscale0, wscale1, xs, y, p, status);
    note_launch();
    return e;
}

}  // namespace larql
