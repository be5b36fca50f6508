// gate_tc.cu — vindex gate walk on tcgen05 tensor cores.
//
// Reference: crates/larql-vindex/src/index/gate.rs:108-134 (gate_knn: scores =
// G[N, D] . r, G f16 rows decoded by crates/larql-models/src/quant/half.rs:4-20,
// f32 products) and :307-316 (top_k_from_scores: top-K by |score|, sorted
// descending); gate_knn_batch / gate_scores_batch (:500-559) are the same
// scores for many residuals.
//
// One launch scores every (layer, query) pair of a batch against every gate
// row of every layer and keeps the top-K:
//
//  * Queries are the MMA's A operand (M = 128 queries per block, one query per
//    TMEM lane), split per query into two f16 planes: q * 2^-e = hi + lo with
//    |q * 2^-e| < 2^15 (22-23 significant bits, f32 grade).  Both planes
//    accumulate into the same f32 accumulator column.
//  * Gate rows are the B operand (N = 256 rows per tile).  They are f16 in HBM
//    and exact as MMA operands; half.rs decodes f16 subnormals to half their IEEE
//    value, so registration rewrites each subnormal to its half.rs value rounded
//    to the nearest f16 subnormal (error <= 2^-25 per element).
//  * A producer warp streams 64-wide K blocks (128-byte rows, TMA SWIZZLE_128B)
//    of both query planes and of the gate tile into a 3-stage ring; one thread
//    issues tcgen05.mma.kind::f16 (M128 N256 K16, 8 per block) into one of two
//    256-column TMEM buffers; 4 epilogue warps read their 32 lanes' 256 scores
//    per tile and keep a running top-16 per query in registers.
//  * Up to 64 queries ("packed"): the hi and lo planes share one 128-row A tile, rows 32 Q + i holding the hi
//    plane (i < 16) or the lo plane (i >= 16) of query 16 Q + (i & 15), so one MMA per K step instead of two;
//    each epilogue warp's 32 TMEM lanes then hold both halves of its 16 queries, added with one shuffle.
//  * Work item = (layer, part of the layer's tiles, query block), query block
//    fastest so the CTAs working on the same gate tiles at the same time share
//    them through L2.  A merge kernel takes the top-K of the parts' candidates.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kGateThreads = 192;             // warp 0 producer, 1 MMA issuer, 2-5 epilogue
constexpr int kGateM = 128;                   // queries per block (TMEM lanes)
constexpr int kGateN = 256;                   // gate rows per tile (accumulator columns)
constexpr int kGateKB = 64;                   // K per stage: one 128-byte swizzle row
constexpr int kGateKM = 16;                   // top-K capacity per (query, part)
constexpr int kGateStages = 3;
constexpr int kGateAPlane = kGateM * kGateKB * 2;           // 16 KB
constexpr int kGateBTile = kGateN * kGateKB * 2;            // 32 KB
constexpr int kGateStage = 2 * kGateAPlane + kGateBTile;    // 64 KB
constexpr int kGateTmemCols = 512;

// ───────────────────────── registration fixup ─────────────────────────
//
// half.rs:4-20 returns (mant / 1024) * 2^-15 for a subnormal, half its IEEE
// value.  When every finite |g| < 32768 the stored matrix becomes 2 * g
// exactly: normals get exponent + 1, subnormals keep their bits (which as IEEE
// are exactly 2x the half.rs value), and scores are halved (factor 0.5).
// Otherwise each subnormal is replaced by the IEEE f16 nearest its half.rs
// value (ties to even; error <= 2^-25) and the factor is 1.

__global__ void gate_max_exp_kernel(const uint16_t* __restrict__ g, size_t n, int* __restrict__ out) {
    int m = 0;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int e = (g[i] >> 10) & 0x1F;
        if (e != 31) m = max(m, e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out, m);
}

__global__ void gate_halfrs_fixup_kernel(uint16_t* __restrict__ g, size_t n, const int* __restrict__ max_exp) {
    const bool doubled = *max_exp <= 29;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint16_t h = g[i];
        const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x03FFu;
        if (doubled) {
            if (e != 0 && e != 31) g[i] = static_cast<uint16_t>(h + 0x0400u);
        } else if (e == 0 && m != 0) {
            const uint32_t half = (m >> 1) + ((m & 1u) & ((m >> 1) & 1u));  // round half to even
            g[i] = static_cast<uint16_t>((h & 0x8000u) | half);
        }
    }
}

// work: one int of device scratch (zeroed here); *factor_host receives the score factor.
cudaError_t launch_gate_halfrs_fixup(uint16_t* g, size_t n, int* work, float* factor_host, cudaStream_t stream) {
    *factor_host = 1.0f;
    if (n == 0) return cudaSuccess;
    const size_t b = (n + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(b < 4096 ? b : 4096);
    cudaError_t e = cudaMemsetAsync(work, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
    gate_max_exp_kernel<<<blocks, 256, 0, stream>>>(g, n, work);
    note_launch();
    gate_halfrs_fixup_kernel<<<blocks, 256, 0, stream>>>(g, n, work);
    note_launch();
    int mx = 0;
    e = cudaMemcpyAsync(&mx, work, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    *factor_host = mx <= 29 ? 0.5f : 1.0f;
    return cudaGetLastError();
}

// ───────────────────────── query planes ─────────────────────────

// One block per query row r < rows (rows = query blocks * 128): planes[0][r][:] = hi,
// planes[1][r][:] = lo, qscale[r] = 2^e (0 for padding rows, NaN if q has a
// non-finite value).  Packed (rows = 128, B <= 64): row r is the hi (r & 16 == 0) or lo
// plane of query 16 (r / 32) + (r & 15), all in planes[0].
__global__ void gate_query_prep_kernel(const float* __restrict__ q, int B, int D, int rows, float factor,
                                       __half* __restrict__ planes, float* __restrict__ qscale, int packed) {
    pdl_launch_dependents();
    pdl_wait();  // the queries and the plane buffers belong to the kernels before this one until they finish
    const int row = blockIdx.x;
    const int r = packed ? 16 * (row >> 5) + (row & 15) : row;  // the query
    __shared__ float red[32];
    __shared__ int nonfin;
    float amax = 0.f;
    bool bad = false;
    if (threadIdx.x == 0) nonfin = 0;
    if (r < B) {
        for (int k = threadIdx.x; k < D; k += blockDim.x) {
            const float v = q[static_cast<size_t>(r) * D + k];
            amax = fmaxf(amax, fabsf(v));
            bad |= !isfinite(v);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    if (bad) nonfin = 1;
    __syncthreads();
    if (threadIdx.x < 32) {
        float a = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (threadIdx.x == 0) red[0] = a;
    }
    __syncthreads();
    amax = red[0];
    // amax < 2^ex; scale so that |q * 2^-e| < 2^15 (f16 max 65504)
    const int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 126;
    const int e = min(100, max(-100, ex - 15));
    const float down = __int_as_float((127 - e) << 23);
    const bool want_hi = !packed || (row & 16) == 0, want_lo = !packed || (row & 16) != 0;
    __half* hi = planes + static_cast<size_t>(row) * D;
    __half* lo = planes + (packed ? static_cast<size_t>(row) : static_cast<size_t>(rows) + row) * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
        const float v = (r < B && !nonfin) ? q[static_cast<size_t>(r) * D + k] * down : 0.f;
        const __half h = __float2half_rn(v);
        if (want_hi) hi[k] = h;
        if (want_lo) lo[k] = __float2half_rn(v - __half2float(h));
    }
    if (threadIdx.x == 0 && want_hi)
        qscale[r] = r >= B ? 0.f : (nonfin ? __int_as_float(0x7fc00000) : __int_as_float((127 + e) << 23) * factor);
}

// ───────────────────────── tensor-core scores + top-K ─────────────────────────

// K-major operand in the 128-byte swizzle layout (8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1) << 16;           // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;   // SBO
    d |= static_cast<uint64_t>(1) << 46;           // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2) << 61;           // SWIZZLE_128B
    return d;
}

__device__ __forceinline__ void gate_umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Item -> (layer, part, query block); the part's tiles are [t0, t1).
__device__ __forceinline__ void gate_item(const GatePlan& p, int item, int& l, int& part, int& qb, int& t0,
                                          int& t1) {
    qb = item % p.QB;
    const int lp = item / p.QB;
    part = lp % p.P;
    l = lp / p.P;
    t0 = part * p.T / p.P;
    t1 = (part + 1) * p.T / p.P;
}

// Branchless insertion of (a = |s|, s, idx) into a register list sorted by
// |score| descending (KM entries).  Candidates arrive in increasing index order
// and need a strictly larger |score| to move up, so the lower index wins ties.
__device__ __forceinline__ void topk_insert(float (&kv)[kGateKM], float (&sv)[kGateKM], uint32_t (&iv)[kGateKM],
                                            float a, float s, uint32_t idx) {
#pragma unroll
    for (int i = kGateKM - 1; i > 0; --i) {
        const bool up = a > kv[i - 1];  // the entry above moves down into slot i
        const bool here = a > kv[i];    // a lands in slot i (if the entry above stays)
        kv[i] = up ? kv[i - 1] : (here ? a : kv[i]);
        sv[i] = up ? sv[i - 1] : (here ? s : sv[i]);
        iv[i] = up ? iv[i - 1] : (here ? idx : iv[i]);
    }
    const bool top = a > kv[0];
    kv[0] = top ? a : kv[0];
    sv[0] = top ? s : sv[0];
    iv[0] = top ? idx : iv[0];
}

__device__ __forceinline__ void tmem_ld8(uint32_t ta, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(ta));
}

__global__ void __launch_bounds__(kGateThreads, 1)
    gate_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap gmap,
                   const float* __restrict__ qscale, float* __restrict__ cand_s, uint32_t* __restrict__ cand_i,
                   const GatePlan p, int* status, float* __restrict__ scores) {
    pdl_launch_dependents();
    pdl_wait();  // the query planes and the candidate buffers belong to the kernels before this one until they finish
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzled tiles need 1024-byte aligned shared addresses
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGateStages * kGateStage);
    uint64_t* empty = full + kGateStages;
    uint64_t* tfull = empty + kGateStages;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abortv = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kGateStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 4);
        }
        *abortv = 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kGateTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    const int qrows = p.QB * kGateM;  // plane 1 starts at this row of the query-plane tensor

    if (warp == 0) {
        // ───── producer ─────
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            const uint32_t bytes = static_cast<uint32_t>((p.packed ? 1 : 2) * p.qbox * kGateKB * 2 + kGateBTile);
            for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x) {
                int l, part, qb, t0, t1;
                gate_item(p, item, l, part, qb, t0, t1);
                for (int t = t0; t < t1 && ok; ++t) {
                    for (int kb = 0; kb < p.nkb; ++kb, ++k) {
                        const int st = k % kGateStages;
                        if (*abortv || (k >= kGateStages &&
                                        !mbar_wait(&empty[st], ((k / kGateStages) - 1) & 1, status, 51))) {
                            ok = false;
                            *abortv = 1;
                            break;
                        }
                        uint8_t* sb = smem + st * kGateStage;
                        mbar_arrive_expect_tx(&full[st], bytes);
                        tma_load_2d(sb, &qmap, kb * kGateKB, qb * kGateM, &full[st]);
                        if (!p.packed)
                            tma_load_2d(sb + kGateAPlane, &qmap, kb * kGateKB, qrows + qb * kGateM, &full[st]);
                        tma_load_2d(sb + 2 * kGateAPlane, &gmap, kb * kGateKB, l * p.F + t * kGateN, &full[st]);
                    }
                }
            }
            // every issued copy lands before the CTA's shared memory goes away
            for (int j = max(0, k - kGateStages); j < k; ++j)
                if (!mbar_wait(&full[j % kGateStages], (j / kGateStages) & 1, status, 52)) break;
        }
    } else if (warp == 1) {
        // ───── MMA issuer (one thread) ─────
        if (lane == 0) {
            // f16 x f16 -> f32, A and B K-major, N = 256, M = 128
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(kGateN >> 3) << 17) |
                                   (static_cast<uint32_t>(kGateM >> 4) << 24);
            int k = 0, tc = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x) {
                int l, part, qb, t0, t1;
                gate_item(p, item, l, part, qb, t0, t1);
                for (int t = t0; t < t1 && ok; ++t, ++tc) {
                    const int buf = tc & 1;
                    if (tc >= 2 && !mbar_wait(&tempty[buf], ((tc >> 1) - 1) & 1, status, 53)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t dt = tmem + static_cast<uint32_t>(buf * kGateN);
                    for (int kb = 0; kb < p.nkb; ++kb, ++k) {
                        const int st = k % kGateStages;
                        if (*abortv || !mbar_wait(&full[st], (k / kGateStages) & 1, status, 54)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t sa = smem_u32(smem + st * kGateStage);
                        const uint64_t dhi = sw128_desc(sa), dlo = sw128_desc(sa + kGateAPlane);
                        const uint64_t dg = sw128_desc(sa + 2 * kGateAPlane);
#pragma unroll
                        for (int kk = 0; kk < kGateKB / 16; ++kk) {
                            // +32 bytes per 16-element K step inside the swizzle row (descriptor units of 16 B)
                            const uint64_t off = static_cast<uint64_t>(kk * 2);
                            const int npl = p.packed ? 1 : 2;
                            for (int pl = 0; pl < npl; ++pl) {
                                const uint32_t acc = (kb | kk | pl) != 0;
                                asm volatile(
                                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(dt),
                                    "l"((pl ? dlo : dhi) + off), "l"(dg + off), "r"(idesc), "r"(acc)
                                    : "memory");
                            }
                        }
                        gate_umma_commit(&empty[st]);
                    }
                    if (ok) gate_umma_commit(&tfull[buf]);
                }
            }
            if (!ok) *abortv = 1;
        }
    } else {
        // ───── epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31 (one query each) ─────
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int tc = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < p.nitems; item += gridDim.x) {
            int l, part, qb, t0, t1;
            gate_item(p, item, l, part, qb, t0, t1);
            // packed: lanes 0..15 own query 16 * quarter + lane (hi plane), lanes 16..31 hold its lo plane
            const int q = p.packed ? 16 * quarter + (lane & 15) : qb * kGateM + row;
            const bool own = !p.packed || lane < 16;
            const float scale = own && q < p.B ? qscale[q] : 0.f;
            float kv[kGateKM], sv[kGateKM];
            uint32_t iv[kGateKM];
#pragma unroll
            for (int i = 0; i < kGateKM; ++i) {
                kv[i] = -1.f;
                sv[i] = 0.f;
                iv[i] = 0xFFFFFFFFu;
            }
            for (int t = t0; t < t1; ++t, ++tc) {
                const int buf = tc & 1;
                if (ok) {
                    const bool got = !*abortv && mbar_wait(&tfull[buf], (tc >> 1) & 1, status, 55);
                    ok = __all_sync(0xffffffffu, got);
                }
                if (!ok) continue;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ta = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * kGateN);
#pragma unroll 1
                for (int c = 0; c < kGateN / 8; ++c) {
                    uint32_t v[8];
                    tmem_ld8(ta + static_cast<uint32_t>(c * 8), v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (p.packed) {  // warp-uniform: hi (lane i) + lo (lane i + 16)
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float h = __uint_as_float(v[i]);
                            v[i] = __float_as_uint(h + __shfl_down_sync(0xffffffffu, h, 16));
                        }
                    }
                    const int f0 = t * kGateN + c * 8;
                    const int nv = min(8, p.F - f0);  // rows past the layer end are skipped
                    if (scores) {
                        // scores mode (gate_scores_batch): every score of this query's row, [L][B][F]
                        if (own && q < p.B) {
                            float* dst = scores + (static_cast<size_t>(l) * p.B + q) * p.F + f0;
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                if (i < nv) dst[i] = __uint_as_float(v[i]) * scale;
                        }
                        continue;
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float s = __uint_as_float(v[i]) * scale;
                        if (own && fabsf(s) > kv[kGateKM - 1] && i < nv)
                            topk_insert(kv, sv, iv, fabsf(s), s, static_cast<uint32_t>(f0 + i));
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            if (ok && own && q < p.B && !scores) {
                const size_t base = ((static_cast<size_t>(l) * p.B + q) * p.P + part) * kGateKM;
#pragma unroll
                for (int i = 0; i < kGateKM; ++i) {
                    cand_s[base + i] = sv[i];
                    cand_i[base + i] = iv[i];
                }
            }
        }
        if (!ok) *abortv = 1;
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGateTmemCols));
}

// One warp per (layer, query): top-k of the parts' candidates by |score|
// descending, ties by ascending feature index.
__global__ void gate_merge_kernel(const float* __restrict__ cand_s, const uint32_t* __restrict__ cand_i, int L,
                                  int B, int P, int k, uint32_t* __restrict__ out_i, float* __restrict__ out_s) {
    pdl_launch_dependents();
    pdl_wait();  // the candidates belong to the kernel before this one until it finishes
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= L * B) return;
    const int n = P * kGateKM;  // <= 512
    const float* cs = cand_s + static_cast<size_t>(w) * n;
    const uint32_t* ci = cand_i + static_cast<size_t>(w) * n;
    constexpr int J = 16;
    uint32_t key[J], idx[J];
    float sc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        const bool v = e < n && ci[e] != 0xFFFFFFFFu;
        sc[j] = v ? cs[e] : 0.f;
        idx[j] = v ? ci[e] : 0xFFFFFFFFu;
        key[j] = v ? __float_as_uint(fabsf(sc[j])) + 1u : 0u;  // 0 = empty; |score| bits order like the values
    }
    uint32_t* oi = out_i + static_cast<size_t>(w) * k;
    float* os = out_s + static_cast<size_t>(w) * k;
    for (int r = 0; r < k; ++r) {
        uint32_t bk = 0, bi = 0xFFFFFFFFu;
        int bj = -1;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (key[j] > bk || (key[j] == bk && key[j] != 0 && idx[j] < bi)) {
                bk = key[j];
                bi = idx[j];
                bj = j;
            }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t mi = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xFFFFFFFFu);
        float ms = 0.f;
        const bool mine = mk != 0 && bk == mk && bi == mi;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (mine && j == bj) {
                ms = sc[j];
                key[j] = 0;
            }
        const unsigned who = __ballot_sync(0xffffffffu, mine);
        ms = __shfl_sync(0xffffffffu, ms, who ? __ffs(who) - 1 : 0);
        if (lane == 0) {
            oi[r] = mk ? mi : 0xFFFFFFFFu;
            os[r] = mk ? ms : 0.f;
        }
    }
}

cudaError_t launch_gate_merge(const float* cand_s, const uint32_t* cand_i, int L, int B, int P, int k,
                              uint32_t* out_i, float* out_s, cudaStream_t stream) {
    if (P < 1 || P * kGateKM > 512 || k < 1 || k > kGateKM) return cudaErrorInvalidValue;
    const int warps = L * B;
    const cudaError_t e = launch_pdl(gate_merge_kernel, dim3((warps + 7) / 8), dim3(256), 0, stream,
                                     static_cast<const float*>(cand_s), static_cast<const uint32_t*>(cand_i), L, B, P,
                                     k, out_i, out_s);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

// Merge of n_lists top-k lists per row (the candidates gathered from row shards):
// in [n_lists][rows][kin] (index 0xFFFFFFFF = empty), index + offsets[list]
// (offsets may be null), out [rows][kout] by |score| descending, ties by index.
__global__ void topk_merge_lists_kernel(const uint32_t* __restrict__ in_i, const float* __restrict__ in_s,
                                        int n_lists, int rows, int kin, const uint32_t* __restrict__ offsets,
                                        int kout, uint32_t* __restrict__ out_i, float* __restrict__ out_s) {
    pdl_launch_dependents();
    pdl_wait();  // the lists belong to the kernels before this one until they finish
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= rows) return;
    const int n = n_lists * kin;  // <= 512
    constexpr int J = 16;
    uint32_t key[J], idx[J];
    float sc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        const int li = e / kin, c = e - li * kin;
        const size_t at = (static_cast<size_t>(li) * rows + w) * kin + c;
        const bool v = e < n && in_i[at] != 0xFFFFFFFFu;
        sc[j] = v ? in_s[at] : 0.f;
        idx[j] = v ? in_i[at] + (offsets ? offsets[li] : 0u) : 0xFFFFFFFFu;
        key[j] = v ? __float_as_uint(fabsf(sc[j])) + 1u : 0u;
    }
    for (int r = 0; r < kout; ++r) {
        uint32_t bk = 0, bi = 0xFFFFFFFFu;
        int bj = -1;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (key[j] > bk || (key[j] == bk && key[j] != 0 && idx[j] < bi)) {
                bk = key[j];
                bi = idx[j];
                bj = j;
            }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t mi = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xFFFFFFFFu);
        float ms = 0.f;
        const bool mine = mk != 0 && bk == mk && bi == mi;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (mine && j == bj) {
                ms = sc[j];
                key[j] = 0;
            }
        const unsigned who = __ballot_sync(0xffffffffu, mine);
        ms = __shfl_sync(0xffffffffu, ms, who ? __ffs(who) - 1 : 0);
        if (lane == 0) {
            out_i[static_cast<size_t>(w) * kout + r] = mk ? mi : 0xFFFFFFFFu;
            out_s[static_cast<size_t>(w) * kout + r] = mk ? ms : 0.f;
        }
    }
}

cudaError_t launch_topk_merge_lists(const uint32_t* in_i, const float* in_s, int n_lists, int rows, int kin,
                                    const uint32_t* offsets, int kout, uint32_t* out_i, float* out_s,
                                    cudaStream_t stream) {
    if (rows <= 0 || kout <= 0) return cudaSuccess;
    if (n_lists < 1 || kin < 1 || n_lists * kin > 512) return cudaErrorInvalidValue;
    const cudaError_t e = launch_pdl(topk_merge_lists_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, in_i, in_s,
                                     n_lists, rows, kin, offsets, kout, out_i, out_s);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

// ───────────────────────── host side ─────────────────────────

bool gate_make_plan(int L, int F, int D, int B, int k, int num_sms, GatePlan* out) {
    if (L < 1 || F < 1 || B < 1 || k < 1 || k > kGateKM || D % kGateKB || D < kGateKB) return false;
    GatePlan p{};
    p.L = L;
    p.F = F;
    p.D = D;
    p.B = B;
    p.k = k;
    p.QB = (B + kGateM - 1) / kGateM;
    p.T = (F + kGateN - 1) / kGateN;
    p.nkb = D / kGateKB;
    p.qbox = B >= kGateM ? kGateM : ((B + 7) / 8) * 8;
    p.packed = B <= kGateM / 2 ? 1 : 0;
    if (p.packed) p.qbox = kGateM;  // one 128-row tile of interleaved hi / lo rows
    // parts per layer: about two items per SM, at most 32 parts (merge width) and one tile per part
    int parts = (2 * num_sms + L * p.QB - 1) / (L * p.QB);
    parts = parts < 1 ? 1 : parts;
    parts = parts > 32 ? 32 : parts;
    parts = parts > p.T ? p.T : parts;
    p.P = parts;
    p.nitems = L * p.P * p.QB;
    p.grid = p.nitems < num_sms ? p.nitems : num_sms;
    // stages, barriers (256 B), alignment slack
    p.smem = kGateStages * kGateStage + 256 + 1024;
    *out = p;
    return true;
}

size_t gate_scratch_bytes(const GatePlan& p) {
    const size_t rows = static_cast<size_t>(p.QB) * kGateM;
    const size_t planes = 2 * rows * p.D * sizeof(__half);
    const size_t qs = ((rows * sizeof(float)) + 255) & ~size_t(255);
    const size_t cand = static_cast<size_t>(p.L) * p.B * p.P * kGateKM;
    return ((planes + 255) & ~size_t(255)) + qs + cand * (sizeof(float) + sizeof(uint32_t)) + 256;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2-D f16 [rows][D] tensor, 64 x box_rows boxes in the 128-byte swizzle.
int gate_encode_map(void* encode_fn, const void* base, size_t rows, int D, int box_rows, CUtensorMap* map) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kGateKB), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<EncodeFn>(encode_fn)(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                                                       dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

// queries f32 [B][D] -> top-k (idx, score) per (layer, query): out [L][B][k].
// gates: the fixed-up f16 rows [L * F][D] behind gmap (box 64 x 256), scores times `factor`.
// scores != nullptr: the scores mode instead, scores [L][B][F] (gate_scores_batch), no top-k.
cudaError_t launch_gate_topk(void* encode_fn, const CUtensorMap& gmap, float factor, const float* queries,
                             const GatePlan& p, uint8_t* scratch, uint32_t* out_i, float* out_s, int* status,
                             cudaStream_t stream, float* scores) {
    const size_t rows = static_cast<size_t>(p.QB) * kGateM;
    __half* planes = reinterpret_cast<__half*>(scratch);
    const size_t planes_bytes = (2 * rows * p.D * sizeof(__half) + 255) & ~size_t(255);
    float* qscale = reinterpret_cast<float*>(scratch + planes_bytes);
    const size_t qs_bytes = ((rows * sizeof(float)) + 255) & ~size_t(255);
    const size_t ncand = static_cast<size_t>(p.L) * p.B * p.P * kGateKM;
    float* cand_s = reinterpret_cast<float*>(scratch + planes_bytes + qs_bytes);
    uint32_t* cand_i = reinterpret_cast<uint32_t*>(cand_s + ncand);

    cudaError_t e = launch_pdl(gate_query_prep_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, stream, queries,
                               p.B, p.D, static_cast<int>(rows), factor, planes, qscale, p.packed);
    note_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap qmap;
    if (gate_encode_map(encode_fn, planes, 2 * rows, p.D, p.qbox, &qmap) != 0) return cudaErrorInvalidValue;
    static DeviceFlags attr_done;
    const int smem = static_cast<int>(p.smem);
    e = once_per_device(attr_done, [smem] {
        return cudaFuncSetAttribute(gate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (e != cudaSuccess) return e;
    e = launch_pdl(gate_tc_kernel, dim3(p.grid), dim3(kGateThreads), p.smem, stream, qmap, gmap,
                   static_cast<const float*>(qscale), cand_s, cand_i, p, status, scores);
    note_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess || scores) return e;
    return launch_gate_merge(cand_s, cand_i, p.L, p.B, p.P, p.k, out_i, out_s, stream);
}

}  // namespace larql
