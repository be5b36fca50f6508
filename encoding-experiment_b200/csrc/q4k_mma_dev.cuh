// q4k_mma_dev.cuh — device pieces of the warp-MMA Q4_K matvec shared by q4k_mma.cu (the matvec
// kernel) and decode_persist.cu (the persistent decode kernel): chunk / box geometry of each format,
// the m16n8k32 MMA wrappers, the digit-plane split of x, the x-table build and the Q4_K super-block
// step.  The factorisation they implement is described at the top of q4k_mma.cu.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kMmaMaxWarps = 8;                       // consumer warps per CTA
constexpr int kMmaRowBytes = 592;                     // one 1024-value chunk of one Q4_K row
constexpr int kMmaRowBytesQ40 = 576;                  // one 1024-value chunk of one Q4_0 row (32 x 18 B)
constexpr int kMmaRowBytesQ80 = 1088;                 // one 1024-value chunk of one GGUF Q8_0 row (32 x 34 B)
constexpr int kMmaRowBytesQ6K = 1680;                 // one 2048-value chunk of one Q6_K row (8 x 210 B)
constexpr int kMmaRowBytesQ4KG = 576;                 // one 1024-value chunk of one GGUF-144 Q4_K row (4 x 144 B)

__host__ __device__ constexpr int mma_rb(int fmt) {
    return fmt == 5 || fmt == 6 ? kMmaRowBytesQ4KG
                    : fmt == 4 ? kMmaRowBytesQ6K
                    : (fmt == 2 ? kMmaRowBytesQ80 : (fmt ? kMmaRowBytesQ40 : kMmaRowBytes));  // fmt 3: Q4_0 bytes
}
// Shared-memory bytes of one box row.  The 576-byte chunks (Q4_0, GGUF-144 Q4_K) are read 592 bytes wide and
// the 1088-byte GGUF Q8_0 chunks 1104 bytes wide (16 bytes of the next chunk, or the zero fill past a row's
// end): at a 576- or 1088-byte stride the 8 rows of an MMA group start on only two bank offsets (both are odd
// multiples of 64), at 592 or 1104 on eight distinct 16-byte ones.
__host__ __device__ constexpr int mma_sb(int fmt) {
    return fmt == 1 || fmt == 3 || fmt == 5 || fmt == 6 ? kMmaRowBytes
                                                          : (fmt == 2 ? kMmaRowBytesQ80 + 16 : mma_rb(fmt));
}
// tensor-map element of each format (a box row is one chunk; at most 256 elements): u32, or u64 for Q8_0 / Q6_K
__host__ __device__ constexpr int mma_elem(int fmt) { return fmt == 2 || fmt == 4 ? 8 : 4; }
// 256-value super-blocks per chunk: 4 (1024 values), or 8 for Q6_K (1024 Q6_K values are 840 bytes, not a
// multiple of 16, so its chunks hold 2048)
__host__ __device__ constexpr int mma_sbc(int fmt) { return fmt == 4 ? 8 : 4; }
// bytes of one 256-value super-block of a row
__host__ __device__ constexpr int mma_sbb(int fmt) {
    return fmt == 5 || fmt == 6 ? 144 : fmt == 4 ? 210 : (fmt == 2 ? 272 : (fmt ? 144 : 148));
}
constexpr int kMmaPrefetch = 1;                       // L2 prefetch distance in boxes


__device__ __forceinline__ void mma_u8s8(uint32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// 2^e for -126 <= e <= 127, built from the exponent field.
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }

// Digit planes per batch row of x: three (x * 2^-e within 2^22: 22-23 significant bits).  Two planes (14-15 bits
// relative to the super-block's largest |x|) would save an n-tile at batch 3-4 and 6-8, but measured on the GPU
// they miss the 1e-3 |y|_inf bound where a row's sum cancels (errors near 3e-4 of the terms' scale); the code
// keeps NP general for that reason only.
__host__ __device__ constexpr int mma_planes(int) { return 3; }
__host__ __device__ constexpr int mma_ntiles(int B) { return (mma_planes(B) * B + 7) / 8; }

// Exponent e with |v * 2^-e| < 2^22 (three planes) or 2^14 (two) for every |v| <= amax (amax finite).
template <int NP>
__device__ __forceinline__ int plane_exponent(float amax) {
    const int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu) - 126;  // amax < 2^ex
    return max(-126, ex - (NP == 3 ? 22 : 14));
}

// m16n8k32 s8 x s8, C = 0.
__device__ __forceinline__ void mma_s8s8(uint32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Exact float of an int with |c| < 2^22 (1.5 * 2^23 + c in the mantissa, then the bias removed).
__device__ __forceinline__ float i2f_small(int c) { return __int_as_float(c + 0x4B400000) - 12582912.0f; }

// m16n8k32 u8 x s8 with a C input.
__device__ __forceinline__ void mma_u8s8_c(uint32_t (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1, int c0, int c1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%10,%11};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}

// Balanced base-256 digits, most significant first: |xi| <= 2^22 as xi = d[0] * 65536 + d[1] * 256 + d[2]
// (NP = 3), |xi| <= 2^14 as xi = d[0] * 256 + d[1] (NP = 2); every digit in [-128, 127].
template <int NP>
__device__ __forceinline__ void digits(int xi, int (&d)[3]) {
    d[2] = 0;
#pragma unroll
    for (int z = NP - 1; z > 0; --z) {
        d[z] = (xi << 24) >> 24;
        xi = (xi - d[z]) >> 8;
    }
    d[0] = xi;
}

// Builds the x tables of chunks [c0, c1) (consumer threads only):
//   xt[(s * NT + nt) * 32 + lane]   uint2  B fragment of sub-block s, n-tile nt
//   mt[(sb * NT + nt) * 32 + lane]  u32    B fragment of the sub-block sums
//   wt[(sb * NT + nt) * 4 + t]      float4 {2^e col 2t, 2^e col 2t+1, 2^em col 2t, 2^em col 2t+1}
//                                   times the plane weight 256^(2 - plane)
template <int B, int NT, int PRO, int FMT = 0>
__device__ void mma_build_tables(const float* __restrict__ x, int K, int c0, int c1, uint8_t* smem, const MmaPlan& p,
                                 int ctid, int cwarp, int lane, const MmaFuse& fz, const volatile float* rms_s) {
    uint2* xt = reinterpret_cast<uint2*>(smem + p.xt_off);
    uint8_t* mt = smem + p.mt_off;
    float* wt = reinterpret_cast<float*>(smem + p.wt_off);
    constexpr int SBC = mma_sbc(FMT);
    constexpr int NP = mma_planes(B);
    const int nsb = (c1 - c0) * SBC;
    const int ncons = 32 * p.NW;
    // zero what the build leaves unwritten: columns past NP * B, unused min lanes
    {
        uint4* z = reinterpret_cast<uint4*>(smem + (NP * B < 8 * NT ? p.xt_off : p.mt_off));
        const int n16 = (p.bar_off - (NP * B < 8 * NT ? p.xt_off : p.mt_off)) / 16;
        for (int i = ctid; i < n16; i += ncons) z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    named_bar_sync(1, ncons);
    const float rms = PRO == 1 ? *rms_s : 1.f;
    const int j = lane >> 2, t = lane & 3;
    // U super-blocks per warp at a time (every batch row), their steps interleaved so the
    // shuffle rounds and loads of one overlap those of the others
    constexpr int U = B == 1 ? 4 : (B == 2 ? 2 : 1);
    for (int sbl0 = cwarp; sbl0 < nsb; sbl0 += U * p.NW) {
        float4 f[U][B][2];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int sbl = sbl0 + u * p.NW;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                if (sbl < nsb) {
                    const size_t off = static_cast<size_t>(c0 * SBC + sbl) * 256 + lane * 8;
                    const float4* xp = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * K + off);
                    f[u][b][0] = __ldg(xp);
                    f[u][b][1] = __ldg(xp + 1);
                    if constexpr (PRO != 0) {  // B == 1: the norm weight or the up half at the same index
                        const float4* sp = reinterpret_cast<const float4*>(PRO == 1 ? fz.nw + off : x + K + off);
                        float4 m[2] = {__ldg(sp), __ldg(sp + 1)};
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            float* v4 = reinterpret_cast<float*>(&f[u][b][h]);
                            const float* m4 = reinterpret_cast<const float*>(&m[h]);
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                v4[i] = PRO == 1 ? v4[i] / rms * (fz.offset + m4[i])
                                                 : v4[i] * (1.0f / (1.0f + expf(-v4[i]))) * m4[i];
                        }
                    }
                } else {
                    f[u][b][0] = f[u][b][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        float amax[U][B], s[U][B];
        bool nonfin[U][B];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float v[8] = {f[u][b][0].x, f[u][b][0].y, f[u][b][0].z, f[u][b][0].w,
                                    f[u][b][1].x, f[u][b][1].y, f[u][b][1].z, f[u][b][1].w};
                amax[u][b] = 0.f;
                s[u][b] = 0.f;
                nonfin[u][b] = false;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    amax[u][b] = fmaxf(amax[u][b], fabsf(v[i]));
                    s[u][b] += v[i];
                    nonfin[u][b] |= !isfinite(v[i]);
                }
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int b = 0; b < B; ++b) amax[u][b] = fmaxf(amax[u][b], __shfl_xor_sync(0xffffffffu, amax[u][b], o));
        // 32-value sums of the 8 sub-blocks
#pragma unroll
        for (int o = 1; o < 4; o <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int b = 0; b < B; ++b) s[u][b] += __shfl_xor_sync(0xffffffffu, s[u][b], o);
        float am[U][B];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int b = 0; b < B; ++b) am[u][b] = fabsf(s[u][b]);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int b = 0; b < B; ++b) am[u][b] = fmaxf(am[u][b], __shfl_xor_sync(0xffffffffu, am[u][b], o));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int sbl = sbl0 + u * p.NW;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const bool fin = !__any_sync(0xffffffffu, nonfin[u][b]);
                if (sbl >= nsb) continue;  // warp-uniform
                const float v[8] = {f[u][b][0].x, f[u][b][0].y, f[u][b][0].z, f[u][b][0].w,
                                    f[u][b][1].x, f[u][b][1].y, f[u][b][1].z, f[u][b][1].w};
                const int e = plane_exponent<NP>(amax[u][b]);
                const float down = pow2i(-e);
                uint32_t pl[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
                int dsum[3] = {0, 0, 0};
#pragma unroll
                for (int k2 = 0; k2 < 8; ++k2) {
                    const int xi = fin ? __float2int_rn(v[k2] * down) : 0;
                    int dg[3];
                    digits<NP>(xi, dg);
                    const int par = k2 & 1, pos = 8 * (k2 >> 1);
#pragma unroll
                    for (int z = 0; z < NP; ++z) {
                        pl[z][par] |= (static_cast<uint32_t>(dg[z]) & 0xFFu) << pos;
                        dsum[z] += dg[z];
                    }
                }
#pragma unroll
                for (int z = 0; z < NP; ++z) {
                    const int col = NP * b + z, nt = col >> 3, g = col & 7;
                    xt[((sbl * 8 + j) * NT + nt) * 32 + g * 4 + t] = make_uint2(pl[z][0], pl[z][1]);
                }
                if constexpr (FMT == 1 || FMT == 3) {
                    // C input of the block's MMA: -8 * (the 32 digits' sum) per column (4 lanes per block)
                    int* ct = reinterpret_cast<int*>(mt);
#pragma unroll
                    for (int z = 0; z < NP; ++z) {
                        dsum[z] += __shfl_xor_sync(0xffffffffu, dsum[z], 1);
                        dsum[z] += __shfl_xor_sync(0xffffffffu, dsum[z], 2);
                        const int col = NP * b + z, nt = col >> 3;
                        if (t == 0) ct[((sbl * 8 + j) * NT + nt) * 8 + (col & 7)] = -8 * dsum[z];
                    }
                } else if constexpr (FMT == 4) {
                    // C inputs of the two MMAs of a 32-value group: -32 * (digit sum) per 16-value sub-block
                    // (lanes t = 0, 1 hold the first sub-block's elements, t = 2, 3 the second's)
                    int* ct = reinterpret_cast<int*>(mt);
#pragma unroll
                    for (int z = 0; z < NP; ++z) {
                        dsum[z] += __shfl_xor_sync(0xffffffffu, dsum[z], 1);
                        const int col = NP * b + z, nt = col >> 3;
                        if ((t & 1) == 0) ct[(((sbl * 8 + j) * 2 + (t >> 1)) * NT + nt) * 8 + (col & 7)] = -32 * dsum[z];
                    }
                }
                const bool finm = fin && isfinite(am[u][b]);
                const int em = plane_exponent<NP>(finm ? am[u][b] : 0.f);
                if ((FMT == 0 || FMT == 5 || FMT == 6) && t == 0) {
                    const int xi = finm ? __float2int_rn(s[u][b] * pow2i(-em)) : 0;
                    int dz[3];
                    digits<NP>(xi, dz);
#pragma unroll
                    for (int z = 0; z < NP; ++z) {
                        const int col = NP * b + z, nt = col >> 3, g = col & 7;
                        mt[(((sbl * NT + nt) * 32) + g * 4 + (j >> 2)) * 4 + (j & 3)] =
                            static_cast<uint8_t>(dz[z] & 0xFF);
                    }
                }
                if (lane == 0) {
                    const float qnan = __int_as_float(0x7fc00000);
#pragma unroll
                    for (int z = 0; z < NP; ++z) {
                        const int col = NP * b + z, nt = col >> 3, c8 = col & 7;
                        float* w4 = wt + ((sbl * NT + nt) * 4 + (c8 >> 1)) * 4;
                        w4[c8 & 1] = fin ? pow2i(e + 8 * (NP - 1 - z)) : qnan;
                        w4[2 + (c8 & 1)] = finm ? pow2i(em + 8 * (NP - 1 - z)) : qnan;
                    }
                }
            }
        }
    }
    named_bar_sync(1, ncons);
}

// One super-block of the warp's 16 rows: hdr points at row g's 148-byte block
// inside the stage (row g + 8 is 8 * 592 bytes further).
template <int NT>
__device__ __forceinline__ void mma_superblock(const uint8_t* hdr, const uint2* __restrict__ xs,
                                               const uint32_t* __restrict__ ms, const float4* __restrict__ ws,
                                               int lane, int t, float (&acc)[NT][4]) {
    constexpr int R8 = 8 * kMmaRowBytes;
    const uint32_t hg = lds32(hdr), hg8 = lds32(hdr + R8);
    const uint32_t s0g = lds32(hdr + 4) & 0x3F3F3F3Fu, s1g = lds32(hdr + 8) & 0x3F3F3F3Fu;
    const uint32_t s0g8 = lds32(hdr + R8 + 4) & 0x3F3F3F3Fu, s1g8 = lds32(hdr + R8 + 8) & 0x3F3F3F3Fu;
    const uint32_t mng = lds32(hdr + 16), mng8 = lds32(hdr + R8 + 16);
    int ai[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ai[nt][0] = ai[nt][1] = ai[nt][2] = ai[nt][3] = 0;
    const uint8_t* qp = hdr + 20 + 4 * t;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t wg = lds32(qp + 16 * j);
        const uint32_t wg8 = lds32(qp + R8 + 16 * j);
        const uint32_t a0 = wg & 0x0F0F0F0Fu, a2 = (wg >> 4) & 0x0F0F0F0Fu;
        const uint32_t a1 = wg8 & 0x0F0F0F0Fu, a3 = (wg8 >> 4) & 0x0F0F0F0Fu;
        const int scg = static_cast<int>(((j < 4 ? s0g : s1g) >> (8 * (j & 3))) & 0xFFu);
        const int scg8 = static_cast<int>(((j < 4 ? s0g8 : s1g8) >> (8 * (j & 3))) & 0xFFu);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 b = xs[(j * NT + nt) * 32 + lane];
            uint32_t c[4];
            mma_u8s8(c, a0, a1, a2, a3, b.x, b.y);
            ai[nt][0] += scg * static_cast<int>(c[0]);
            ai[nt][1] += scg * static_cast<int>(c[1]);
            ai[nt][2] += scg8 * static_cast<int>(c[2]);
            ai[nt][3] += scg8 * static_cast<int>(c[3]);
        }
    }
    const uint32_t mlo = t == 0 ? mng : (mng >> 4), mlo8 = t == 0 ? mng8 : (mng8 >> 4);
    const uint32_t am0 = t < 2 ? (mlo & 0x0F0F0F0Fu) : 0u, am1 = t < 2 ? (mlo8 & 0x0F0F0F0Fu) : 0u;
    const float dg = h2f_lo(hg), dmg = h2f_hi(hg), dg8 = h2f_lo(hg8), dmg8 = h2f_hi(hg8);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        uint32_t m[4];
        mma_u8s8(m, am0, am1, 0u, 0u, ms[nt * 32 + lane], 0u);
        const float4 w = ws[nt * 4 + t];
        acc[nt][0] = fmaf(dg * w.x, static_cast<float>(ai[nt][0]), acc[nt][0]);
        acc[nt][1] = fmaf(dg * w.y, static_cast<float>(ai[nt][1]), acc[nt][1]);
        acc[nt][2] = fmaf(dg8 * w.x, static_cast<float>(ai[nt][2]), acc[nt][2]);
        acc[nt][3] = fmaf(dg8 * w.y, static_cast<float>(ai[nt][3]), acc[nt][3]);
        acc[nt][0] = fmaf(-dmg * w.z, static_cast<float>(static_cast<int>(m[0])), acc[nt][0]);
        acc[nt][1] = fmaf(-dmg * w.w, static_cast<float>(static_cast<int>(m[1])), acc[nt][1]);
        acc[nt][2] = fmaf(-dmg8 * w.z, static_cast<float>(static_cast<int>(m[2])), acc[nt][2]);
        acc[nt][3] = fmaf(-dmg8 * w.w, static_cast<float>(static_cast<int>(m[3])), acc[nt][3]);
    }
}


}  // namespace larql
