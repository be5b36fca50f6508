// q4k_tc.cu — Q4_K (LARQL 148-byte blocks) dequant-matvec on the 5th-generation
// tensor cores (tcgen05.mma kind::i8), batch 1..8.
//
// Math (crates/larql-compute/src/cpu/ops/q4k_matvec.rs:70-81): for row r and
// 32-value sub-block j of super-block s,
//   sum_k W[r,k] x[k] = d*sc_j * sum_k q_k x_k  -  dmin*mn_j * sum_k x_k .
// x is converted once per call (x_prep kernel) into exact integer digits per
// 32-value group g: x_k = 2^e_g * (a_k*65536 + b_k*256 + c_k), a,b,c int8,
// |x_k * 2^-e_g| <= 2^22 (f32 precision at the group maximum).  The digit
// planes form the MMA's B operand (N = 3 planes x batch, padded to 16 / 32),
// the unpacked nibbles q (u8 0..15) its A operand, so one M=128 x N x K=32
// integer MMA per sub-block produces the exact int32 sums sum q*a, q*b, q*c
// for 128 rows at once, each sub-block into its own TMEM accumulator.  The
// epilogue (one thread per row = TMEM lane) folds in d*sc_j*2^e_g and the
// mins term.
//
// Pipeline per CTA (persistent, one per SM; tiles of H <= 128 rows chosen so
// the tile count is a multiple of the SM count):
//   warp 8      producer: per chunk of 4 super-blocks (592 B per row, 16-byte
//               aligned) one 2-D TMA load of the H x 592 B weight box plus bulk
//               copies of the chunk's digit planes and group scales/sums,
//               double buffered.
//   warps 0-7   transform: per sub-block, 8 rows x 16 packed bytes per warp
//               instruction (conflict-free: 592 B row pitch = 20 banks mod 32)
//               -> u8 nibbles written as 8-byte pieces into an A slot in the
//               canonical K-major core-matrix layout; 8 A slots in a ring.
//   warp 9      TMEM allocation + MMA issue (one elected thread), commits to
//               mbarriers that free A slots and publish accumulators.
//   warps 0-3   epilogue: tcgen05.ld of each sub-block accumulator, scale,
//               accumulate y for the row in registers, store at tile end.
// Nibble K-order inside a 32-byte A row: for packed word i (elements 8i..8i+7)
// bytes [8i, 8i+4) hold the low nibbles (elements 8i, 8i+2, 8i+4, 8i+6) and
// [8i+4, 8i+8) the high nibbles (8i+1, ..., 8i+7); x_prep writes B with the
// same permutation.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kTcThreads = 672;       // warps 0-7 transform, 8-15 epilogue, 16 producer, 17-20 MMA issuers
constexpr int kTcASlotBytes = 128 * 32;
constexpr int kTcChunkSub = 32;       // sub-blocks per chunk (4 super-blocks)
constexpr int kTcChunkRowBytes = 592; // 4 * 148
constexpr int kTcTmemCols = 512;


// canonical K-major, no-swizzle: core matrix = 8 rows x 16 B; K-chunks of
// 16 B are 128 B apart (LBO), 8-row groups 256 B apart (SBO).
__host__ __device__ __forceinline__ int canon_off(int row, int kb) {
    return (kb >> 4) * 128 + (row >> 3) * 256 + (row & 7) * 16 + (kb & 15);
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(128 >> 4) << 16;  // LBO
    d |= static_cast<uint64_t>(256 >> 4) << 32;  // SBO
    d |= static_cast<uint64_t>(1) << 46;          // descriptor version (sm_100)
    return d;                                     // SWIZZLE_NONE, base offset 0
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}


// ───────────── x -> digit planes (B operand) + per-group scale and sum ─────────────
// One warp per (batch b, 32-value group g).  Output layouts:
//   planes: [group g][nmma rows x 32 B canonical tile], row n = 3b + z
//   xinfo : [chunk c][batch b][sub-block j (32)][2] floats (2^e, sum x)
__global__ void q4k_x_prep(const float* __restrict__ x, int K, int batch, int nmma, uint8_t* __restrict__ planes,
                           float* __restrict__ xinfo) {
    // the main kernel may start its prologue and weight loads while this runs
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int ngroups = K / 32;
    if (gw >= ngroups * batch) return;
    const int b = gw / ngroups, g = gw % ngroups;
    const float v = x[static_cast<size_t>(b) * K + g * 32 + lane];
    float amax = fabsf(v), sum = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    int ex = 0;
    frexpf(amax, &ex);
    int e = max(-126, min(127, ex - 22));
    const bool fin = isfinite(amax);
    int xi = fin ? __float2int_rn(v * ldexpf(1.0f, -e)) : 0;
    const int c = (xi << 24) >> 24;
    xi = (xi - c) >> 8;
    const int bb = (xi << 24) >> 24;
    const int a = (xi - bb) >> 8;
    // element lane -> K byte: word i = lane/8, t = (lane%8)/2, parity p = lane%2
    const int i = lane >> 3, t = (lane & 7) >> 1, p = lane & 1;
    const int kb = 8 * i + 4 * p + t;
    uint8_t* tile = planes + static_cast<size_t>(g) * nmma * 32;
    tile[canon_off(3 * b + 0, kb)] = static_cast<uint8_t>(a);
    tile[canon_off(3 * b + 1, kb)] = static_cast<uint8_t>(bb);
    tile[canon_off(3 * b + 2, kb)] = static_cast<uint8_t>(c);
    if (lane == 0) {
        const int chunk = g / kTcChunkSub, j = g % kTcChunkSub;
        float* xo = xinfo + ((static_cast<size_t>(chunk) * batch + b) * kTcChunkSub + j) * 2;
        xo[0] = fin ? ldexpf(1.0f, e) : __int_as_float(0x7fc00000);
        xo[1] = sum;
    }
}

template <int NMMA>
struct TcCfg {
    static constexpr int G = 4;                    // sub-blocks per MMA group (one barrier phase, one commit)
    static constexpr int NG = NMMA == 16 ? 4 : 2;  // groups in flight (A slots = D slots = NG * G)
    static constexpr int NS = NG * G;
};

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// tcgen05.ld of W consecutive 32-bit columns for this warp's 32 lanes.
template <int W>
__device__ __forceinline__ void tmem_ld(uint32_t ta, uint32_t* v) {
    if constexpr (W == 4) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                     : "r"(ta));
    } else if constexpr (W == 8) {
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                     : "r"(ta));
    } else if constexpr (W == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(ta));
    } else {
        static_assert(W == 24, "load width");
        tmem_ld<16>(ta, v);
        tmem_ld<8>(ta + 16u, v + 16);
    }
}

// LW = accumulator columns the epilogue reads per sub-block (>= 3 * batch).
template <int NMMA, int LW>
__global__ void __launch_bounds__(kTcThreads, 1)
    q4k_tc_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ planes,
                  const float* __restrict__ xinfo, float* __restrict__ y, TcPlan p, int* status) {
    using C = TcCfg<NMMA>;
    constexpr int BMAX = LW / 3;  // batch rows whose 3 planes fit the columns read
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* full = bars;                 // [2]  stage loaded (TMA + bulk)
    uint64_t* empty = full + 2;            // [2]  stage consumed (8 transform + 8 epilogue warps + NG issuer commits)
    uint64_t* a_full = empty + 2;          // [NG] group's 4 A slots written (4 transform warps)
    uint64_t* grp_done = a_full + C::NG;   // [NG] group's MMAs complete: A slots free, accumulators ready (commit)
    uint64_t* d_free = grp_done + C::NG;   // [NG] group's accumulators read (4 epilogue warps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_free + C::NG);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 2);
    float* ybuf = reinterpret_cast<float*>(smem + p.bar_off + 64 * 8);  // [128 rows][8] partials of epilogue half 1
    uint8_t* aring = smem + p.a_off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 16 + C::NG); }
        for (int i = 0; i < C::NG; ++i) { mbar_init(&a_full[i], 4); mbar_init(&grp_done[i], 1); mbar_init(&d_free[i], 4); }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 17) {  // TMEM allocation / release by the first issuer warp
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    volatile int* abortv = abort_flag;

    const int nch = p.nchunks;
    const int my_tiles = (p.ntiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const int total = my_tiles * nch;  // chunks this CTA processes

    if (warp == 16) {
        // ───── producer ─────
        if (lane == 0) {
            int k = 0;
            bool planes_ready = false;
            for (; k < total; ++k) {
                if (*abortv) break;
                const int st = k & 1;
                if (k >= 2 && !mbar_wait(&empty[st], ((k >> 1) - 1) & 1, status, 21)) { *abortv = 1; break; }
                const int tile = blockIdx.x + (k / nch) * gridDim.x;
                const int chunk = k % nch;
                uint8_t* sb = smem + st * p.stage_bytes;
                mbar_arrive_expect_tx(&full[st], p.H * kTcChunkRowBytes + p.b_bytes + p.xi_bytes);
                tma_load_2d(sb, &wmap, chunk * (kTcChunkRowBytes / 4), tile * p.H, &full[st]);
                if (!planes_ready) {  // x_prep (the preceding grid) must be complete before its outputs are read
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    planes_ready = true;
                }
                bulk_g2s(sb + p.w_region, planes + static_cast<size_t>(chunk) * p.b_bytes, p.b_bytes, &full[st]);
                bulk_g2s(sb + p.w_region + p.b_bytes, xinfo + static_cast<size_t>(chunk) * p.xi_bytes / 4,
                         p.xi_bytes, &full[st]);
            }
            for (int j = max(0, k - 2); j < k; ++j)
                if (!mbar_wait(&full[j & 1], (j >> 1) & 1, status, 22)) break;
        }
    } else if (warp >= 17) {
        // ───── MMA issuers: warp 17 + i issues the groups of ring slot i (one elected thread each) ─────
        // A single thread cannot issue tcgen05.mma fast enough for one M=128 x N x K=32 MMA per 2 KB of
        // weights at HBM speed, so each ring slot has its own issuer; a slot's groups stay in order.
        const int me = warp - 17;
        if (lane == 0 && me < C::NG) {
            const uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(NMMA >> 3) << 17) |
                                   (static_cast<uint32_t>(128 >> 4) << 24);
            const uint64_t da0 = umma_desc(smem_u32(aring)) + static_cast<uint64_t>(me * C::G * (kTcASlotBytes >> 4));
            const uint32_t dt0 = tmem + static_cast<uint32_t>(me * C::G * NMMA);
            constexpr int GPC = kTcChunkSub / C::G;  // groups per chunk (8)
            int last_u = -1;
            bool ok = true;
            for (int k = 0; k < total && ok; ++k) {
                const int st = k & 1;
                if (!mbar_wait(&full[st], (k >> 1) & 1, status, 23)) { ok = false; break; }
                const uint64_t db0 = umma_desc(smem_u32(smem + st * p.stage_bytes + p.w_region));
#pragma unroll 1
                for (int gq = me; gq < GPC; gq += C::NG) {
                    const int u = k * GPC + gq, c = u / C::NG;  // u & (NG - 1) == me
                    if (c >= 1 && !mbar_wait(&d_free[me], (c - 1) & 1, status, 24)) { ok = false; break; }
                    if (!mbar_wait(&a_full[me], c & 1, status, 25)) { ok = false; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    uint64_t da = da0;
                    uint64_t db = db0 + static_cast<uint64_t>(gq * C::G * (NMMA * 32 >> 4));
                    uint32_t dt = dt0;
#pragma unroll
                    for (int i = 0; i < C::G; ++i) {
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(dt),
                            "l"(da), "l"(db), "r"(idesc), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
                            : "memory");
                        da += kTcASlotBytes >> 4;
                        db += (NMMA * 32) >> 4;
                        dt += NMMA;
                    }
                    umma_commit(&grp_done[me]);
                    last_u = u;
                }
                if (ok) umma_commit(&empty[st]);
            }
            if (!ok) *abortv = 1;
            if (last_u >= 0) mbar_wait(&grp_done[me], (last_u / C::NG) & 1, status, 26);
        }
    } else if (warp < 8) {
        // ───── transform: warp w owns sub-blocks w, w+8, w+16, w+24 of every chunk, two per round ─────
        // All packed words of a round are loaded into registers before any A
        // store, so the shared-memory loads overlap instead of serialising
        // behind stores the compiler cannot prove disjoint.
        const int ngroups = (p.H + 7) >> 3;  // <= 12 (H <= 96)
        const int tr = lane & 7, tw = lane >> 3;  // row in 8-row group, packed word in sub-block
        bool ok = true;
        for (int k = 0; k < total; ++k) {
            const int st = k & 1;
            if (ok) ok = mbar_wait(&full[st], (k >> 1) & 1, status, 27);
            const uint8_t* sw = smem + st * p.stage_bytes + tr * kTcChunkRowBytes + 4 * tw;
            for (int r2 = 0; r2 < 2; ++r2) {
                const int subA = warp + 16 * r2, subB = subA + 8;
                const int gA = k * kTcChunkSub + subA, gB = gA + 8;
                const int uA = gA / C::G, uB = gB / C::G;  // their groups
                // packed words of both sub-blocks first (stage reads do not depend on ring slots)
                const uint8_t* srcA = sw + (subA >> 3) * 148 + 20 + 16 * (subA & 7);
                const uint8_t* srcB = sw + (subB >> 3) * 148 + 20 + 16 * (subB & 7);
                uint32_t wa[12], wb[12];
#pragma unroll
                for (int i = 0; i < 12; ++i) {
                    wa[i] = (ok && i < ngroups) ? lds32(srcA + i * 8 * kTcChunkRowBytes) : 0u;
                    wb[i] = (ok && i < ngroups) ? lds32(srcB + i * 8 * kTcChunkRowBytes) : 0u;
                }
                // then each sub-block: wait for its slot, store, publish (A before B: with two groups in
                // flight, B's slot is freed by the group A completes)
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int gg = half ? gB : gA, uu = half ? uB : uA;
                    if (ok && uu >= C::NG) ok = mbar_wait(&grp_done[uu & (C::NG - 1)], ((uu / C::NG) - 1) & 1, status, 28);
                    if (ok) {
                        uint8_t* dst = aring + (gg & (C::NS - 1)) * kTcASlotBytes + canon_off(tr, 8 * tw);
#pragma unroll
                        for (int i = 0; i < 12; ++i) {
                            const uint32_t w = half ? wb[i] : wa[i];
                            if (i < ngroups)
                                *reinterpret_cast<uint2*>(dst + i * 256) = make_uint2(w & 0x0F0F0F0Fu, (w >> 4) & 0x0F0F0F0Fu);
                        }
                        fence_proxy_async_smem();
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[uu & (C::NG - 1)]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            if (!ok) *abortv = 1;
            if (*abortv) break;
        }
    } else {
        // ───── epilogue: warps 8-15; quadrant q = warp % 4 (TMEM lanes), half h takes D groups of parity h ─────
        const int q = warp & 3, h = (warp - 8) >> 2;
        const int row = q * 32 + lane;
        const int batch = p.batch;
        float acc[BMAX];
#pragma unroll
        for (int b = 0; b < BMAX; ++b) acc[b] = 0.f;
        bool ok = true;
        for (int k = 0; k < total; ++k) {
            const int st = k & 1;
            const int tile = blockIdx.x + (k / nch) * gridDim.x;
            const int chunk = k % nch;
            if (ok) ok = mbar_wait(&full[st], (k >> 1) & 1, status, 29);
            const uint8_t* sw = smem + st * p.stage_bytes;
            const float* sxi = reinterpret_cast<const float*>(sw + p.w_region + p.b_bytes);
            const bool live = row < p.H;
            for (int s = 0; s < 4; ++s) {
                // this half's group of super-block s: sub-blocks 8s + 4h .. 8s + 4h + 3
                const int g0 = k * kTcChunkSub + s * 8 + 4 * h;
                const int u = g0 / C::G, ng = u & (C::NG - 1);
                uint32_t hd = 0, scw = 0, mnw = 0;
                if (live) {
                    const uint8_t* hp = sw + row * kTcChunkRowBytes + s * 148;
                    hd = lds32(hp); scw = lds32(hp + 4 + 4 * h); mnw = lds32(hp + 16);
                }
                if (ok) ok = mbar_wait(&grp_done[ng], (u / C::NG) & 1, status, 30);
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(ng * C::G * NMMA);
                const float d = h2f_lo(hd), dmin = h2f_hi(hd);
                // accumulator reads in passes of LPW sub-blocks per tcgen05.wait::ld (register budget)
                constexpr int LPW = LW > 16 ? 1 : (LW == 16 ? 2 : C::G);
#pragma unroll
                for (int i0 = 0; i0 < C::G; i0 += LPW) {
                    uint32_t v[LPW][LW];
#pragma unroll
                    for (int i = 0; i < LPW; ++i) tmem_ld<LW>(ta + static_cast<uint32_t>((i0 + i) * NMMA), v[i]);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (i0 + LPW == C::G) {
                        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&d_free[ng]);
                    }
                    if (ok && live) {
#pragma unroll
                        for (int i = 0; i < LPW; ++i) {
                            const int j = 4 * h + i0 + i, sub = s * 8 + j;
                            const float dsc = d * u2f_small((scw >> (8 * (i0 + i))) & 0x3Fu);
                            const float dmn = dmin * u2f_small((mnw >> (8 * (i0 + i) + 4 * h)) & 0xFu);
#pragma unroll
                            for (int b = 0; b < BMAX; ++b) {
                                if (b < batch) {
                                    const int isum =
                                        (static_cast<int>(v[i][3 * b]) * 256 + static_cast<int>(v[i][3 * b + 1])) * 256 +
                                        static_cast<int>(v[i][3 * b + 2]);
                                    const float2 xi = *reinterpret_cast<const float2*>(sxi + (b * kTcChunkSub + sub) * 2);
                                    acc[b] = fmaf(dsc * xi.x, static_cast<float>(isum), fmaf(-dmn, xi.y, acc[b]));
                                }
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            if (chunk == nch - 1) {
                // combine the two halves: half 1 parks its partials, half 0 adds and stores
                if (h == 1 && live) {
#pragma unroll
                    for (int b = 0; b < BMAX; ++b) ybuf[row * 8 + b] = acc[b];
                }
                named_bar_sync(2, 256);
                const int grow = tile * p.H + row;
                if (h == 0 && live && grow < p.N && ok) {
#pragma unroll
                    for (int b = 0; b < BMAX; ++b)
                        if (b < batch) y[static_cast<size_t>(b) * p.N + grow] = acc[b] + ybuf[row * 8 + b];
                }
                named_bar_sync(2, 256);
#pragma unroll
                for (int b = 0; b < BMAX; ++b) acc[b] = 0.f;
            }
            if (!ok) *abortv = 1;
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 17)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
}

// ───────────── host side ─────────────

bool q4k_tc_make_plan(int N, int K, int batch, int num_sms, TcPlan* out) {
    if (K % 1024 || batch < 1 || batch > 8 || N < 1) return false;
    TcPlan p{};
    p.N = N;
    p.K = K;
    p.batch = batch;
    p.nmma = 3 * batch <= 16 ? 16 : 32;
    p.phase_subs = 512 / p.nmma;
    p.nchunks = K / 1024;
    const int hmax = 96;
    // tiles = k * num_sms with the smallest k that keeps tiles <= hmax rows
    int k = (N + hmax * num_sms - 1) / (hmax * num_sms);
    int tiles = k * num_sms;
    p.H = (N + tiles - 1) / tiles;
    if (p.H < 8) p.H = 8 < N ? 8 : N;  // at least one 8-row group per tile
    p.ntiles = (N + p.H - 1) / p.H;
    p.grid = p.ntiles < num_sms ? p.ntiles : num_sms;
    p.w_region = hmax * kTcChunkRowBytes;                 // multiple of 16
    p.b_bytes = kTcChunkSub * p.nmma * 32;
    p.xi_bytes = batch * kTcChunkSub * 8;
    p.stage_bytes = (p.w_region + p.b_bytes + p.xi_bytes + 1023) & ~1023;
    const int na = p.nmma == 16 ? 16 : 8;  // A slots = TcCfg<nmma>::NS
    p.a_off = 2 * p.stage_bytes;
    p.bar_off = p.a_off + na * kTcASlotBytes;
    p.smem = p.bar_off + 64 * 8 + 128 * 8 * 4;  // barriers + epilogue half-1 partials
    if (p.smem > kSmemLimit) return false;
    *out = p;
    return true;
}

size_t q4k_tc_scratch_bytes(int K, int batch) {
    const int nmma = 3 * batch <= 16 ? 16 : 32;
    const size_t planes = static_cast<size_t>(K / 32) * nmma * 32;
    const size_t xinfo = static_cast<size_t>(K / 32) * batch * 8;
    return ((planes + 255) & ~size_t(255)) + xinfo;
}

// The weight's 2-D tensor map: rows of row_bytes as uint32, box = 148 words x H rows.
int q4k_tc_encode_map(void* encode_fn, const void* w, int N, int K, int H, CUtensorMap* map) {
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    const uint64_t row_bytes = static_cast<uint64_t>(K / 256) * 148;
    cuuint64_t dims[2] = {row_bytes / 4, static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcChunkRowBytes / 4), static_cast<cuuint32_t>(H)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<Fn>(encode_fn)(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(w), dims,
                                                 strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

cudaError_t launch_q4k_tc(const CUtensorMap& map, const float* x, float* y, const TcPlan& p, uint8_t* scratch,
                          int* status, cudaStream_t stream) {
    uint8_t* planes = scratch;
    const size_t planes_bytes = static_cast<size_t>(p.K / 32) * p.nmma * 32;
    float* xinfo = reinterpret_cast<float*>(scratch + ((planes_bytes + 255) & ~size_t(255)));
    const int groups = p.K / 32 * p.batch;
    q4k_x_prep<<<(groups + 7) / 8, 256, 0, stream>>>(x, p.K, p.batch, p.nmma, planes, xinfo);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    static DeviceFlags attr_done[4];
    const int which = p.nmma == 32 ? 3 : (p.batch <= 1 ? 0 : (p.batch <= 2 ? 1 : 2));
    const void* fn = which == 0   ? reinterpret_cast<const void*>(q4k_tc_kernel<16, 4>)
                     : which == 1 ? reinterpret_cast<const void*>(q4k_tc_kernel<16, 8>)
                     : which == 2 ? reinterpret_cast<const void*>(q4k_tc_kernel<16, 16>)
                                  : reinterpret_cast<const void*>(q4k_tc_kernel<32, 24>);
    e = once_per_device(attr_done[which],
                        [fn] { return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit); });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (which) {
        case 0: e = cudaLaunchKernelEx(&cfg, q4k_tc_kernel<16, 4>, map, (const uint8_t*)planes, (const float*)xinfo, y, p, status); break;
        case 1: e = cudaLaunchKernelEx(&cfg, q4k_tc_kernel<16, 8>, map, (const uint8_t*)planes, (const float*)xinfo, y, p, status); break;
        case 2: e = cudaLaunchKernelEx(&cfg, q4k_tc_kernel<16, 16>, map, (const uint8_t*)planes, (const float*)xinfo, y, p, status); break;
        default: e = cudaLaunchKernelEx(&cfg, q4k_tc_kernel<32, 24>, map, (const uint8_t*)planes, (const float*)xinfo, y, p, status); break;
    }
    if (e != cudaSuccess) return e;
    note_launch();
    return cudaGetLastError();
}

}  // namespace larql

// ───────────── matvec without any device allocation ─────────────
//
// For callers that must not allocate device memory at call time: code that
// runs under a fixed memory budget decided up front, inside a host allocator
// callback, or in a process whose device memory is reserved by another
// framework.  The tensor-core matvec needs per-call scratch for the digit
// planes of x and the per-group scales/sums; here it lives in this file-scope
// device array.  The array is reserved on a device when this file's device code
// is loaded there — with CUDA's default lazy module loading, at the first
// noalloc call (its cudaGetSymbolAddress) or the first tensor-core Q4_K launch
// on that device — and held until the process exits.  Callers therefore make
// their first call during set-up.

namespace larql {

int fail(int code, const char* fmt, ...);

constexpr int kNoAllocMaxCols = 16384;  // K limit: digit planes of 512 groups
constexpr int kNoAllocMaxBatch = 8;
constexpr size_t kNoAllocScratchBytes = 557056;  // q4k_tc_scratch_bytes(16384, 8)

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_status;

namespace {
struct NoAllocDevice {
    bool ready = false;
    uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int* status = nullptr;       // device address of g_noalloc_status
    int num_sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];
void* g_noalloc_encode = nullptr;
}  // namespace

}  // namespace larql

extern "C" LARQL_API int larql_cuda_q4k_matvec_noalloc(const uint8_t* w_dev, size_t nbytes, size_t rows,
                                                       size_t cols, const float* x_dev, size_t batch, float* y_dev,
                                                       void* stream) {
    using namespace larql;
    if (!w_dev || !x_dev || !y_dev) return fail(LARQL_ERR_INVALID_ARG, "noalloc matvec: null pointer");
    if (rows == 0 || rows > 0x7fffffff) return fail(LARQL_ERR_BAD_SHAPE, "noalloc matvec: rows=%zu", rows);
    if (cols == 0 || cols % 1024 || cols > static_cast<size_t>(kNoAllocMaxCols))
        return fail(LARQL_ERR_BAD_SHAPE, "noalloc matvec: cols=%zu must be a multiple of 1024 and at most %d", cols,
                    kNoAllocMaxCols);
    if (batch < 1 || batch > static_cast<size_t>(kNoAllocMaxBatch))
        return fail(LARQL_ERR_BAD_SHAPE, "noalloc matvec: batch=%zu must be 1..%d", batch, kNoAllocMaxBatch);
    if (nbytes < rows * (cols / 256) * 148)
        return fail(LARQL_ERR_BAD_SHAPE, "noalloc matvec: %zu weight bytes for a %zu x %zu Q4_K matrix", nbytes, rows,
                    cols);
    if (reinterpret_cast<uintptr_t>(w_dev) % 16 || reinterpret_cast<uintptr_t>(x_dev) % 16)
        return fail(LARQL_ERR_INVALID_ARG, "noalloc matvec: weights and x must be 16-byte aligned");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) return fail(LARQL_ERR_CUDA, "noalloc matvec: cudaGetDevice failed");
    NoAllocDevice* d = &g_noalloc_dev[dev];
    {
        // one-time set-up per device, with that device current
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!d->ready) {
            void* sp = nullptr;
            void* st = nullptr;
            e = cudaGetSymbolAddress(&sp, g_noalloc_scratch);
            if (e != cudaSuccess)
                return fail(LARQL_ERR_CUDA, "noalloc matvec: cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
            e = cudaGetSymbolAddress(&st, g_noalloc_status);
            if (e != cudaSuccess)
                return fail(LARQL_ERR_CUDA, "noalloc matvec: cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
            int sms = 0;
            e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess) return fail(LARQL_ERR_CUDA, "noalloc matvec: SM count: %s", cudaGetErrorString(e));
            if (!g_noalloc_encode) {
                cudaDriverEntryPointQueryResult q;
                void* fn = nullptr;
                if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
                    q != cudaDriverEntryPointSuccess)
                    return fail(LARQL_ERR_CUDA, "noalloc matvec: cuTensorMapEncodeTiled unavailable");
                g_noalloc_encode = fn;
            }
            d->scratch = static_cast<uint8_t*>(sp);
            d->status = static_cast<int*>(st);
            d->num_sms = sms;
            d->ready = true;
        }
    }
    TcPlan p;
    if (!q4k_tc_make_plan(static_cast<int>(rows), static_cast<int>(cols), static_cast<int>(batch), d->num_sms, &p))
        return fail(LARQL_ERR_UNSUPPORTED, "noalloc matvec: no tensor-core plan for %zu x %zu batch %zu", rows, cols,
                    batch);
    if (q4k_tc_scratch_bytes(static_cast<int>(cols), static_cast<int>(batch)) > kNoAllocScratchBytes)
        return fail(LARQL_ERR_BAD_SHAPE, "noalloc matvec: scratch for cols=%zu batch=%zu exceeds %zu bytes", cols,
                    batch, kNoAllocScratchBytes);
    CUtensorMap map;
    if (q4k_tc_encode_map(g_noalloc_encode, w_dev, static_cast<int>(rows), static_cast<int>(cols), p.H, &map) != 0)
        return fail(LARQL_ERR_CUDA, "noalloc matvec: tensor map encoding failed");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(d->status, 0, sizeof(int), s);
    if (e == cudaSuccess) e = launch_q4k_tc(map, x_dev, y_dev, p, d->scratch, d->status, s);
    if (e != cudaSuccess) return fail(LARQL_ERR_CUDA, "noalloc matvec: launch: %s", cudaGetErrorString(e));
    int st = 0;
    e = cudaMemcpyAsync(&st, d->status, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(LARQL_ERR_CUDA, "noalloc matvec: %s", cudaGetErrorString(e));
    if (st != 0) return fail(st & 0xFFFF, "noalloc matvec: device reported status %d at site %d", st & 0xFFFF, st >> 16);
    return LARQL_OK;
}
