// q4k_ts.cu — Q4_K (LARQL 148-byte blocks) matvec for batch 1..8 on the tcgen05 tensor cores, with the
// weight operand held in tensor memory (the "TS" form of tcgen05.mma: A from TMEM, B from shared memory).
//
// Math (crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87): for row r and super-block s with sub-blocks j,
//   sum_k W[r,k] x[k] = sum_s [ d_s * sum_j sum_{k in j} (sc_j q_k) x_k  -  dmin_s * sum_j mn_j S_j ],
// S_j = the sum of x over sub-block j.  sc_j q_k <= 63 * 15 is exact in f16.  The x of every
// (super-block, batch row) is scaled by a power of two into [-2^15, 2^15) and split into two f16 planes
// hi + lo (22 significant bits).  Per 128-row tile and super-block:
//   * 16 MMAs M128 x N16 x K16 (kind::f16, f32 accumulation in TMEM) with A = sc*q (the transform warps write
//     it to TMEM with tcgen05.st) and B = the planes (column 2b = hi of batch row b, 2b + 1 = lo) give
//     D_main[r, n] = sum_k (sc q) plane_n, spread over 2 accumulator groups that the epilogue adds;
//   * the transform warps form the mins term sum_j mn_j S_j on the CUDA cores (8 FMAs per row and batch row,
//     S_j in f32 from ts_x_prep);
//   * the epilogue (the same warps, one thread per row = TMEM lane) adds
//     2^e * d * (sum of D_main over the groups, hi + lo) - dmin * (mins term) into the row's sums.
// The per-(row, sub-block) scale is folded into A by the f16 transform (one HFMA2 per two values), so no
// accumulator is rescaled per sub-block: the work per weight value does not grow with the batch.
//
// A's K order inside each packed word (8 nibbles = 8 consecutive values of one sub-block): TMEM column
// 4 * word + t holds values t and t + 4 of the word (low / high half), i.e. K position p of a super-block is
// x index 8 * (p / 8) + (p % 8) / 2 + 4 * (p % 2); ts_x_prep writes B in that order.
//
// CTA roles (608 threads, one persistent CTA per SM):
//   warps 0-15 transform + epilogue.  Warp w owns TMEM lanes 32 * (w % 4) .. + 31 (one tile row per thread)
//              and quarter j = w / 4 of every super-block: sub-blocks 2j, 2j + 1 (A columns 32j .. 32j + 31)
//              and batch rows 2j, 2j + 1 in the epilogue; four warps per SM sub-partition hide the latencies of
//              the shared-memory loads and the tensor-memory stores and loads.
//   warp 16    producer: per stage one 2-D TMA box (128 rows x 592 B = 4 super-blocks) of W, plus one bulk
//              copy of the stage's B tiles, sub-block sums and powers of two; an L2 prefetch one box ahead.
//   warps 17-18 MMA issue, one elected thread each (group g = warp - 17: K steps g, g + 2, ..); warp 17 also
//              allocates the tensor memory.
// Super-block u of a CTA's sequence uses A slot u % 2 (TMEM columns 128 (u % 2) .. + 127) and D slot u % 2
// (columns 256 + 32 (u % 2) .. + 31); the transform of u + 2 and the MMAs of u + 2 wait (through the commit barrier
// of u + 1) until the MMAs of u have drained and the epilogue of u has read its accumulators, so two slots
// suffice.
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kTsXform = 16;                      // transform + epilogue warps (0 .. 15)
constexpr int kTsProducer = kTsXform;             // warp 16
// MMA issuer warps (17, 18), one accumulator group each (K steps g, g + 2, .. into group g).  One thread issues a
// tcgen05.mma M128 x N16 x K16 only every ~100 cycles (measured: 210 cycles with its loop overhead, 57 with
// compile-time TMEM operands; 2 / 4 / 8 issuing warps reach 105 / 53 / 28 cycles per MMA per SM), but in this
// kernel 4 and 8 issuers measured slower than 2 (each extra role on the SM slows the transform warps, which bound
// it), and compile-time operands changed nothing.
constexpr int kTsIssuers = 2;
constexpr int kTsIssuer0 = kTsXform + 1;
constexpr int kTsThreads = 32 * (kTsIssuer0 + kTsIssuers);
constexpr int kTsRows = 128;                        // tile rows (the MMA's M)
constexpr int kTsChunkBytes = 592;                  // one row of a box: 4 super-blocks
constexpr int kTsBox = kTsRows * kTsChunkBytes;     // 75776
constexpr int kTsBTile = 512;                       // one K16 x N16 f16 B tile
constexpr int kTsBSb = 16 * kTsBTile;               // the 16 K-step tiles of a super-block
constexpr int kTsSOff = 4 * kTsBSb;                 // f32 sub-block sums S[4 sb][8 batch][8 sub-blocks]
constexpr int kTsEOff = kTsSOff + 4 * 8 * 8 * 4;    // 2^e[4 sb][8 batch]
constexpr int kTsBChunk = kTsEOff + 4 * 8 * 4;      // 33920
constexpr int kTsStage = kTsBox + kTsBChunk;        // 109696 (multiple of 128)
constexpr int kTsStages = 2;
constexpr int kTsBarOff = kTsStages * kTsStage;
constexpr int kTsSmem = kTsBarOff + 256;
constexpr int kTsTmemCols = 512;
constexpr int kTsColA = 0;      // A slots: 128 columns each
constexpr int kTsChains = kTsIssuers;
constexpr int kTsColD = 256;    // D slots: kTsChains groups x 16 columns
constexpr int kTsDSlot = 16 * kTsChains;
static_assert(kTsColD + 2 * kTsDSlot <= kTsTmemCols, "tensor memory columns");
static_assert(kTsSmem <= kSmemLimit, "shared memory");
static_assert(kTsBox % 1024 == 0 && kTsStage % 128 == 0 && kTsBChunk % 16 == 0, "alignment");

// B tile element (n, k): canonical K-major, no swizzle: 16-byte core-matrix rows, K halves 128 B apart (LBO),
// 8-row groups of n 256 B apart (SBO).
__host__ __device__ constexpr int ts_b_off(int n, int k) {
    return (k >> 3) * 128 + (n >> 3) * 256 + (n & 7) * 16 + (k & 7) * 2;
}

__device__ __forceinline__ uint64_t ts_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>(128 >> 4) << 16;  // LBO: K direction
    d |= static_cast<uint64_t>(256 >> 4) << 32;  // SBO: N direction
    d |= static_cast<uint64_t>(1) << 46;          // descriptor version (sm_100)
    return d;                                     // SWIZZLE_NONE, base offset 0
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// ───────────── x -> B tiles (f16 hi / lo planes in the A K order), sub-block sums, powers of two ─────────────
// One block of 8 warps per super-block sb; warp b = batch row (rows >= batch write zeros).  Lane l takes
// x values 8l .. 8l + 7 of the super-block: packed word l, i.e. K positions 8l .. 8l + 7 = one 16-byte row of
// tile l / 2 (K half l % 2), rows n = 2b (hi) and 2b + 1 (lo).  Output per chunk of 4 super-blocks:
// [4][16 tiles][512 B], then S[4][8][8] f32 (the reference's grouping sum_k x_k per sub-block), then 2^e[4][8]
// (NaN where the super-block's x or one of its S is not finite).
__global__ void __launch_bounds__(256) ts_x_prep(const float* __restrict__ x, int K, int batch,
                                                 uint8_t* __restrict__ xb) {
    pdl_launch_dependents();
    const int sb = blockIdx.x, b = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = sb >> 2, s = sb & 3;
    uint8_t* cb = xb + static_cast<size_t>(chunk) * kTsBChunk;
    uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
    float scale = 0.f, sum = 0.f;
    if (b < batch) {
        const float4* xp = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * K + sb * 256 + 8 * lane);
        const float4 v0 = xp[0], v1 = xp[1];
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        float amax = 0.f;
        bool fin = true;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            amax = fmaxf(amax, fabsf(v[r]));
            sum += v[r];
            fin = fin && isfinite(v[r]);
        }
        // sub-block sums: lanes 4j .. 4j + 3 hold sub-block j
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        fin = __all_sync(0xffffffffu, fin && isfinite(sum));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int ex = 0;
        frexpf(amax, &ex);  // amax < 2^ex
        const int e = max(-126, min(127, ex - 15));
        if (fin) {
            uint32_t h[8], l[8];
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float t = ldexpf(v[r], -e);
                const __half th = __float2half_rn(t);
                h[r] = __half_as_ushort(th);
                l[r] = __half_as_ushort(__float2half_rn(t - __half2float(th)));
            }
            // 16-byte row: K position 2t + p holds value t + 4p
            hi = make_uint4(h[0] | (h[4] << 16), h[1] | (h[5] << 16), h[2] | (h[6] << 16), h[3] | (h[7] << 16));
            lo = make_uint4(l[0] | (l[4] << 16), l[1] | (l[5] << 16), l[2] | (l[6] << 16), l[3] | (l[7] << 16));
            scale = ldexpf(1.0f, e);
        } else {
            scale = __int_as_float(0x7fc00000);
            sum = 0.f;
        }
    }
    uint8_t* t = cb + s * kTsBSb + (lane >> 1) * kTsBTile;
    *reinterpret_cast<uint4*>(t + ts_b_off(2 * b, 8 * (lane & 1))) = hi;
    *reinterpret_cast<uint4*>(t + ts_b_off(2 * b + 1, 8 * (lane & 1))) = lo;
    if ((lane & 3) == 0) reinterpret_cast<float*>(cb + kTsSOff)[(s * 8 + b) * 8 + (lane >> 2)] = sum;
    if (lane == 0) reinterpret_cast<float*>(cb + kTsEOff)[s * 8 + b] = scale;
}

// ───────────── device pieces of the main kernel ─────────────

template <int NV>
__device__ __forceinline__ void lds_span(const uint8_t* p, uint32_t (&v)[4 * NV]) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const uint4 t = *reinterpret_cast<const uint4*>(p + 16 * i);
        v[4 * i] = t.x;
        v[4 * i + 1] = t.y;
        v[4 * i + 2] = t.z;
        v[4 * i + 3] = t.w;
    }
}

// tcgen05.st of 16 consecutive 32-bit columns for this warp's 32 lanes.
__device__ __forceinline__ void tmem_st16(uint32_t ta, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(ta),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_ld4(uint32_t ta, uint32_t (&v)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(ta));
}

__device__ __forceinline__ void ts_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// What the epilogue of a super-block needs from its transform.
struct TsCarry {
    float d, dmin;
    float e[2];   // 2^e of the planes of batch rows 2j, 2j + 1
    float mt[2];  // sum_j mn_j S_j of batch rows 2j, 2j + 1 (the mins term before dmin)
};

// Transform of super-block S (0..3 within the stage) for half H of row `rp` (the row's 592 bytes in the
// stage): A = sc*q of sub-blocks 4H .. 4H + 3 into TMEM columns ta .. ta + 63, the mins into tm .. tm + 7
// (half 0 only).
// Transform of super-block S (0..3 within the stage) for quarter j4 of row `rp` (the row's 592 bytes in the
// stage): A = sc*q of sub-blocks 2 j4, 2 j4 + 1 into TMEM columns ta + 32 j4 .. + 31, and the row's mins term
// sum_j mn_j S_j for batch rows 2 j4, 2 j4 + 1 (S: the super-block's [8 batch][8] sums in the stage).  The nibble
// span's alignment depends on S only, so its words sit at static indices.
template <int S>
__device__ __forceinline__ void ts_transform(const uint8_t* rp, const float* sS, int j4, int batch, uint32_t ta,
                                             TsCarry& c) {
    constexpr int HB = 148 * S;               // super-block header
    constexpr int HA = HB & ~15;
    constexpr int QB = HB + 20;               // packed nibbles; quarter j4 at + 32 j4
    constexpr int QA = QB & ~15;
    constexpr int NQ = (QB - QA + 32 + 15) / 16;
    uint32_t hv[8], qv[4 * NQ];
    lds_span<2>(rp + HA, hv);
    lds_span<NQ>(rp + QA + 32 * j4, qv);
    const uint32_t dd = hv[(HB - HA) / 4];
    // 6-bit scales of sub-blocks 2 j4 and 2 j4 + 1: bytes 4 + 2 j4 and 5 + 2 j4 of the block
    const uint32_t scw = (j4 < 2 ? hv[(HB + 4 - HA) / 4] : hv[(HB + 8 - HA) / 4]) & 0x3F3F3F3Fu;
    const uint32_t sel0 = 2u * static_cast<uint32_t>(j4 & 1);
    c.d = h2f_lo(dd);
    c.dmin = h2f_hi(dd);
    const __half2 k1024 = u2h(0x64006400u), kn1024 = u2h(0xE400E400u);  // 1024, -1024
    const __half2 k16th = u2h(0x2C002C00u), kn64 = u2h(0xD400D400u);    // 1/16, -64
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
        // (1024 + sc, 1024 + sc) -> sc, then the HFMA2 operands of the low (1024 + q) and high (1024 + 16 q)
        // nibble forms: (1024 + q) sc - 1024 sc = q sc and (1024 + 16 q) (sc / 16) - 64 sc = q sc, exact
        const uint32_t sel = 0x4040u | ((sel0 + jj) * 0x0101u);
        const __half2 sc2 = __hsub2(u2h(__byte_perm(scw, 0x64646464u, sel)), k1024);
        const __half2 olo = __hmul2(sc2, kn1024), shi = __hmul2(sc2, k16th), ohi = __hmul2(sc2, kn64);
        uint32_t out[16];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const uint32_t w = qv[(QB - QA) / 4 + 4 * jj + m];
            const uint32_t w8 = w >> 8;
            const uint32_t h0 = (w & 0x000F000Fu) | 0x64006400u, h1 = (w & 0x00F000F0u) | 0x64006400u;
            const uint32_t h2 = (w8 & 0x000F000Fu) | 0x64006400u, h3 = (w8 & 0x00F000F0u) | 0x64006400u;
            out[4 * m + 0] = h2u(__hfma2(u2h(h0), sc2, olo));
            out[4 * m + 1] = h2u(__hfma2(u2h(h1), shi, ohi));
            out[4 * m + 2] = h2u(__hfma2(u2h(h2), sc2, olo));
            out[4 * m + 3] = h2u(__hfma2(u2h(h3), shi, ohi));
        }
        tmem_st16(ta + static_cast<uint32_t>(32 * j4 + 16 * jj), out);
    }
    // mins: mn_j = low nibble of byte 16 + j (j < 4), mn_j+4 its high nibble
    const uint32_t mnw = hv[(HB + 16 - HA) / 4];
    float mn[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        mn[j] = u2f_small((mnw >> (8 * j)) & 0xFu);
        mn[j + 4] = u2f_small((mnw >> (8 * j + 4)) & 0xFu);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float m = 0.f;
        if (2 * j4 + i < batch) {
            const float4* sp = reinterpret_cast<const float4*>(sS + (2 * j4 + i) * 8);
            const float4 s0 = sp[0], s1 = sp[1];
            m = mn[0] * s0.x;
            m = fmaf(mn[1], s0.y, m);
            m = fmaf(mn[2], s0.z, m);
            m = fmaf(mn[3], s0.w, m);
            m = fmaf(mn[4], s1.x, m);
            m = fmaf(mn[5], s1.y, m);
            m = fmaf(mn[6], s1.z, m);
            m = fmaf(mn[7], s1.w, m);
        }
        c.mt[i] = m;
    }
}

__device__ __forceinline__ void ts_transform_s(int s, const uint8_t* rp, const float* sS, int j4, int batch,
                                               uint32_t ta, TsCarry& c) {
    switch (s) {
        case 0: ts_transform<0>(rp, sS, j4, batch, ta, c); break;
        case 1: ts_transform<1>(rp, sS, j4, batch, ta, c); break;
        case 2: ts_transform<2>(rp, sS, j4, batch, ta, c); break;
        default: ts_transform<3>(rp, sS, j4, batch, ta, c); break;
    }
}

// Item i of the CTA's sequence: tile and chunk range.
__device__ __forceinline__ void ts_item(const TsPlan& p, int item, int& tile, int& part, int& c0, int& c1) {
    part = item / p.ntiles;
    tile = item - part * p.ntiles;
    c0 = part * p.nchunks / p.nparts;
    c1 = (part + 1) * p.nchunks / p.nparts;
}

// MMA issue of accumulator group G: K steps G, G + kTsChains, .. of every super-block.
template <int G>
__device__ void ts_issue(uint8_t* smem, uint32_t tbase, uint64_t* full, uint64_t* a_full, uint64_t* mma_done,
                         uint64_t* empty, int U, volatile int* abortv, int* status) {
    constexpr int NS = 16 / kTsChains;  // K steps per group: G, G + kTsChains, ...
    static_assert(G < kTsChains, "group");
    // f16 x f16 -> f32, A and B K-major, N = 16, M = 128
    constexpr uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(16 >> 3) << 17) |
                               (static_cast<uint32_t>(kTsRows >> 4) << 24);
    const uint32_t sbase = smem_u32(smem) + kTsBox;
    bool ok = true;
    int u = 0;
    for (; u < U && ok; ++u) {
        const int k = u >> 2, s = u & 3, st = k & 1, slot = u & 1;
        if (s == 0 && !mbar_wait(&full[st], (k >> 1) & 1, status, 63)) { ok = false; break; }
        if (*abortv || !mbar_wait(&a_full[slot], (u >> 1) & 1, status, 64)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t ta = tbase + static_cast<uint32_t>(kTsColA + 128 * slot + 8 * G);
        const uint32_t td = tbase + static_cast<uint32_t>(kTsColD + kTsDSlot * slot + 16 * G);
        const uint64_t db = ts_desc(sbase + static_cast<uint32_t>(st * kTsStage + s * kTsBSb + G * kTsBTile));
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(td),
                "r"(ta + static_cast<uint32_t>(8 * kTsChains * i)),
                "l"(db + static_cast<uint64_t>(i * kTsChains * (kTsBTile >> 4))), "r"(idesc), "r"(i)
                : "memory");
        }
        ts_commit(&mma_done[slot]);
        if (s == 3) ts_commit(&empty[st]);
    }
    if (!ok) *abortv = 1;
    // the last commit lands before the CTA (and its TMEM) goes away
    if (u > 0) mbar_wait(&mma_done[(u - 1) & 1], ((u - 1) >> 1) & 1, status, 65);
}

__global__ void __launch_bounds__(kTsThreads, 1)
    q4k_ts_kernel(const __grid_constant__ CUtensorMap wmap, const uint8_t* __restrict__ xb, float* __restrict__ y,
                  float* __restrict__ partial, int* __restrict__ tickets, const TsPlan p, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTsBarOff);
    uint64_t* full = bars;           // [2] stage loaded
    uint64_t* empty = full + 2;      // [2] stage consumed: the transform warps + the issuers' commits
    uint64_t* a_full = empty + 2;    // [2] A slot written: the transform warps
    uint64_t* mma_done = a_full + 2; // [2] the super-block's MMAs complete (commit)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 2);
    volatile int* abortv = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (warp == kTsProducer && lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kTsXform + kTsIssuers);
            mbar_init(&a_full[i], kTsXform);
            mbar_init(&mma_done[i], kTsIssuers);
        }
        *abortv = 0;
        fence_barrier_init();
    }
    if (warp == kTsIssuer0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTsTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // the CTA's stages: (item, chunk) in order; items blockIdx.x, + gridDim.x, ...
    int total = 0;
    for (int it = blockIdx.x; it < p.nitems; it += gridDim.x) {
        int tile, part, c0, c1;
        ts_item(p, it, tile, part, c0, c1);
        total += c1 - c0;
    }
    const int U = 4 * total;  // super-blocks

    if (warp == kTsProducer) {
        // ───── producer ─────
        if (lane == 0) {
            int it = blockIdx.x, tile = 0, part = 0, c0 = 0, c1 = 0, c = 0;
            if (it < p.nitems) { ts_item(p, it, tile, part, c0, c1); c = c0; }
            int pit = it, ptile = tile, pc = c, pc1 = c1;  // L2 prefetch cursor, one box ahead
            bool planes_ready = false;
            int k = 0;
            for (; k < total; ++k) {
                if (*abortv) break;
                const int st = k & 1;
                if (k >= 2 && !mbar_wait(&empty[st], ((k >> 1) - 1) & 1, status, 61)) { *abortv = 1; break; }
                uint8_t* sb = smem + st * kTsStage;
                mbar_arrive_expect_tx(&full[st], kTsBox + kTsBChunk);
                tma_load_2d(sb, &wmap, c * (kTsChunkBytes / 4), tile * kTsRows, &full[st]);
                // prefetch the next box into L2
                if (++pc >= pc1) {
                    pit += gridDim.x;
                    if (pit < p.nitems) { int pp, q0; ts_item(p, pit, ptile, pp, q0, pc1); pc = q0; }
                }
                if (pit < p.nitems) tma_prefetch_2d(&wmap, pc * (kTsChunkBytes / 4), ptile * kTsRows);
                if (!planes_ready) {  // ts_x_prep (the preceding grid) must be complete before its output is read
                    pdl_wait();
                    planes_ready = true;
                }
                bulk_g2s(sb + kTsBox, xb + static_cast<size_t>(c) * kTsBChunk, kTsBChunk, &full[st]);
                if (++c >= c1) {
                    it += gridDim.x;
                    if (it < p.nitems) { ts_item(p, it, tile, part, c0, c1); c = c0; }
                }
            }
            for (int j = max(0, k - 2); j < k; ++j)
                if (!mbar_wait(&full[j & 1], (j >> 1) & 1, status, 62)) break;
        }
    } else if (warp >= kTsIssuer0) {
        // ───── MMA issuers: warp kTsIssuer0 + g issues K steps g and g + 8 of every super-block into group g ─────
        if (lane == 0) {
            static_assert(kTsIssuers == 2, "issuer dispatch");
            if (warp == kTsIssuer0) ts_issue<0>(smem, tmem, full, a_full, mma_done, empty, U, abortv, status);
            else ts_issue<1>(smem, tmem, full, a_full, mma_done, empty, U, abortv, status);
        }
    } else {
        // ───── transform + epilogue: warps 0-15 ─────
        const int q = warp & 3, j4 = warp >> 2;
        const int row = 32 * q + lane;  // tile row = TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
        const int batch = p.batch, N = p.N;
        float acc[2] = {0.f, 0.f};
        TsCarry ccur, cprev;  // the transform's super-block and the one the epilogue reads
        // epilogue cursor: the item whose super-blocks the epilogue is summing
        int eit = blockIdx.x, etile = 0, epart = 0, ec0 = 0, ec1 = 0, eleft = 0;
        if (eit < p.nitems) { ts_item(p, eit, etile, epart, ec0, ec1); eleft = 4 * (ec1 - ec0); }
        bool ok = true;

        auto epilogue = [&](int v) {
            const int slot = v & 1;
            // columns 4j .. 4j + 3 of every group: (hi, lo) of batch rows 2j, 2j + 1
            const uint32_t td = tmem + lane_base + static_cast<uint32_t>(kTsColD + kTsDSlot * slot + 4 * j4);
            const TsCarry& c = cprev;
            if (2 * j4 < batch) {
                uint32_t mv[kTsChains][4];
#pragma unroll
                for (int g = 0; g < kTsChains; ++g) tmem_ld4(td + static_cast<uint32_t>(16 * g), mv[g]);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    float m = 0.f;
#pragma unroll
                    for (int g = 0; g < kTsChains; ++g)
                        m += __uint_as_float(mv[g][2 * i]) + __uint_as_float(mv[g][2 * i + 1]);
                    acc[i] = fmaf(c.e[i] * c.d, m, fmaf(-c.dmin, c.mt[i], acc[i]));
                }
            }
            if (--eleft == 0) {
                // item complete: store this thread's rows and batch rows, or its part and the ticket
                const int grow = etile * kTsRows + row;
                if (p.nparts == 1) {
                    if (grow < N && ok) {
#pragma unroll
                        for (int i = 0; i < 2; ++i)
                            if (2 * j4 + i < batch) y[static_cast<size_t>(2 * j4 + i) * N + grow] = acc[i];
                    }
                } else if (2 * j4 < batch) {
                    if (grow < N) {
#pragma unroll
                        for (int i = 0; i < 2; ++i)
                            if (2 * j4 + i < batch)
                                partial[(static_cast<size_t>(epart) * batch + 2 * j4 + i) * N + grow] = acc[i];
                    }
                    __threadfence();
                    __syncwarp();
                    int last = 0;
                    if (lane == 0) {
                        int* tk = tickets + etile * kTsXform + warp;
                        last = atomicAdd(tk, 1) == p.nparts - 1;
                        if (last) *tk = 0;  // ready for the next launch
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last) {
                        __threadfence();
                        if (grow < N && ok) {
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                const int b = 2 * j4 + i;
                                if (b < batch) {
                                    float s = 0.f;
                                    for (int pp = 0; pp < p.nparts; ++pp)
                                        s += __ldcg(partial + (static_cast<size_t>(pp) * batch + b) * N + grow);
                                    y[static_cast<size_t>(b) * N + grow] = s;
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) acc[i] = 0.f;
                eit += gridDim.x;
                if (eit < p.nitems) { ts_item(p, eit, etile, epart, ec0, ec1); eleft = 4 * (ec1 - ec0); }
            }
        };

        int u = 0;
        for (; u < U; ++u) {
            const int k = u >> 2, s = u & 3, st = k & 1, slot = u & 1;
            if (s == 0 && ok) ok = mbar_wait(&full[st], (k >> 1) & 1, status, 66);
            if (!ok || *abortv) { ok = false; break; }
            const uint8_t* sb = smem + st * kTsStage;
            // this super-block's powers of two of the planes of batch rows 2j, 2j + 1
            const float2 ev = *reinterpret_cast<const float2*>(sb + kTsBox + kTsEOff + (s * 8 + 2 * j4) * 4);
            TsCarry& c = ccur;
            c.e[0] = ev.x;
            c.e[1] = ev.y;
            const float* sS = reinterpret_cast<const float*>(sb + kTsBox + kTsSOff) + s * 64;
            const uint8_t* rp = sb + row * kTsChunkBytes;
            const uint32_t ta = tmem + lane_base + static_cast<uint32_t>(kTsColA + 128 * slot);
            ts_transform_s(s, rp, sS, j4, batch, ta, c);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                if (s == 3) mbar_arrive(&empty[st]);  // this warp's reads of the stage are done
                mbar_arrive(&a_full[slot]);
            }
            if (u >= 1) {
                // the MMAs of u - 1 (and everything before) are complete: read its accumulators
                if (!mbar_wait(&mma_done[(u - 1) & 1], ((u - 1) >> 1) & 1, status, 67)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                epilogue(u - 1);
            }
            cprev = ccur;
        }
        if (ok && U > 0 && u == U) {
            if (mbar_wait(&mma_done[(U - 1) & 1], ((U - 1) >> 1) & 1, status, 68)) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                epilogue(U - 1);
            } else {
                ok = false;
            }
        }
        if (!ok) *abortv = 1;
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == kTsIssuer0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTsTmemCols));
}

// ───────────── host side ─────────────

// Split-K parts: the fewest parts that reach the smallest per-CTA chunk count.
bool q4k_ts_make_plan(int N, int K, int batch, int num_sms, TsPlan* out) {
    if (K % 1024 || batch < 1 || batch > 8 || N < 1 || num_sms < 1) return false;
    TsPlan p{};
    p.N = N;
    p.K = K;
    p.batch = batch;
    p.nchunks = K / 1024;
    p.ntiles = (N + kTsRows - 1) / kTsRows;
    int best = -1;
    for (int np = 1; np <= p.nchunks && np <= 16; ++np) {
        const long items = static_cast<long>(p.ntiles) * np;
        const long waves = (items + num_sms - 1) / num_sms;
        const long cost = waves * ((p.nchunks + np - 1) / np);
        if (best < 0 || cost < best) {
            best = static_cast<int>(cost);
            p.nparts = np;
        }
    }
    p.nitems = p.ntiles * p.nparts;
    p.grid = p.nitems < num_sms ? p.nitems : num_sms;
    p.smem = kTsSmem;
    *out = p;
    return true;
}

size_t q4k_ts_scratch_bytes(const TsPlan& p) {
    const size_t xb = static_cast<size_t>(p.nchunks) * kTsBChunk;
    const size_t part = p.nparts > 1 ? static_cast<size_t>(p.nparts) * p.batch * p.N * sizeof(float) : 0;
    return ((xb + 255) & ~size_t(255)) + part;
}

size_t q4k_ts_tickets(const TsPlan& p) { return static_cast<size_t>(p.ntiles) * kTsXform; }

cudaError_t launch_q4k_ts(const CUtensorMap& map, const float* x, float* y, const TsPlan& p, uint8_t* scratch,
                          int* tickets, int* status, cudaStream_t stream) {
    uint8_t* xb = scratch;
    const size_t xb_bytes = static_cast<size_t>(p.nchunks) * kTsBChunk;
    float* partial = reinterpret_cast<float*>(scratch + ((xb_bytes + 255) & ~size_t(255)));
    ts_x_prep<<<p.K / 256, 256, 0, stream>>>(x, p.K, p.batch, xb);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    static DeviceFlags attr_done;
    e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(q4k_ts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTsSmem);
    });
    if (e != cudaSuccess) return e;
    e = launch_pdl(q4k_ts_kernel, dim3(p.grid), dim3(kTsThreads), static_cast<size_t>(kTsSmem), stream, map,
                   static_cast<const uint8_t*>(xb), y, partial, tickets, p, status);
    if (e != cudaSuccess) return e;
    note_launch();
    return cudaGetLastError();
}

}  // namespace larql
