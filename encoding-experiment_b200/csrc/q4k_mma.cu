// q4k_mma.cu — Q4_K (LARQL 148 B per 256 values) matvec for batch 1..8 on the
// warp-level int8 tensor-core MMA (mma.sync m16n8k32, u8 x s8 -> s32).
//
// Reference: crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87, per row
//     y[r] = sum_sb sum_j sum_i (d * sc_j * q - dmin * mn_j) * x
// with sc_j = byte(4 + j) & 0x3F, mn_j = nibble j of bytes 16..19 (j < 4 low,
// j >= 4 high), d / dmin IEEE f16 (q4k_matvec.rs:10-26).
//
// Factorisation (all inner products exact in int32):
//     y[r] = sum_sb [ d * sum_j sc_j * (q_j . X_j)  -  dmin * sum_j mn_j * S_j ]
// X: each batch row of x split per 256-value super-block into three int8
// "digit planes", x = 2^e * (p0 * 65536 + p1 * 256 + p2) with |x * 2^-e| <= 2^22
// (balanced base-256 digits: 22-23 significant bits, f32 grade).  S_j: the
// 32-value sums of x, split the same way with their own exponent.  Every plane
// of every batch row is one column of the MMA's B operand (3 columns per batch
// row, n-tiles of 8 columns), so a weight nibble is unpacked once per launch
// whatever the batch.
//
// Fragment mapping (m16n8k32: A 16x32 u8 row-major, B 32x8 s8 col-major,
// lane = 4 * g + t):
//   A rows g and g + 8 of the warp's 16 weight rows; the 32 k slots are one
//   sub-block, permuted so a nibble word unpacks with two LOP3s:
//     slots 4t..4t+3       <- low nibbles of word t  (elements 8t, 8t+2, 8t+4, 8t+6)
//     slots 16+4t..16+4t+3 <- high nibbles of word t (elements 8t+1, ..., 8t+7)
//   B holds the same permutation of the digit plane of column g.
//   C (int32, rows g / g + 8, columns 2t / 2t + 1) is multiplied by the row's
//   6-bit sc_j (one IMAD each) and summed over the super-block; |sum| < 2^25.
//   The mins take one more MMA per super-block: A = the 8 mins of the row in
//   k slots 0..7 (lane t = 0: sub-blocks 0-3, t = 1: 4-7), B = the planes of
//   the 8 sub-block sums.
//
// Work split: rows are cut into tiles of RT = 16 * NG rows (NG 16-row MMA
// groups); each group is worked by KS warps that take every KS-th super-block
// of a chunk and add their sums through shared memory in slice order.  K is
// cut into `nparts` parts across CTAs; a persistent CTA walks
// (part, tile) items part-major.  A producer warp streams 1024-value chunks
// (RT x 592 B boxes of a 2-D tensor map; 592 = 37 * 16, so every box starts
// on a 16-byte boundary) into an NS-stage mbarrier ring.  The x tables of the
// current part live in shared memory; the consumer warps rebuild them when the
// part changes.  With nparts > 1 each item writes a partial row block and the
// last CTA to finish a tile (atomic ticket) adds the parts in part order, so
// results do not depend on scheduling.
//
// Q4_0 (FMT 1; ggml dequantize_q4_0, crates/larql-models/src/quant/ggml.rs:92-110: w = d * (q - 8), d decoded
// by half.rs:4-20, subnormals at half value) on the same machinery: a 32-value block is one MMA k-step with the
// same nibble permutation as a Q4_K sub-block; its C input is -8 * (sum of the block's plane digits) per column,
// so C = sum (q - 8) * digit exactly; C is scaled by the row's f16 d per block and by the column's plane weight
// per 256 values.  1024 values of a row are 576 bytes (32 blocks), read as RT x 592 B boxes (see mma_sb).
//
// Q6_K (FMT 4; crates/larql-compute/src/cpu/ops/q6k_matvec.rs:31-87: w = d * sc * (q - 32), 16 int8 scales per
// 256 values) with chunks of 2048 values (1680 bytes, u64 boxes): a lane assembles the 6-bit values of its 8
// elements of a 32-value group from one ql word (low nibbles, split even / odd) and 16 qh bits (spread to the
// bytes' bits 4-5), in the tables' k order; the group takes two MMAs, one per 16-value sub-block (the lanes
// holding the other sub-block's elements pass zeros), each with C input -32 * (the sub-block's digit sums),
// and the int32 results are scaled by the sub-blocks' int8 scales before the super-block's f16 d.
//
// GGUF-144 Q4_K (FMT 5; crates/larql-models/src/quant/ggml.rs:228-273, the GGUF loader's dequantize_q4_k:
// w = d * sc_j * q - dmin * mn_j with 6-bit scales and mins packed as llama.cpp get_scale_min_k4 in bytes 4..15,
// sub-block j's 16 bytes at 16 + 16 j holding its elements 0..15 in the low nibbles and 16..31 in the high,
// d / dmin decoded by half.rs) uses the Q4_K tables unchanged: lane (g, t) loads the 8 bytes holding its
// elements 8t..8t+7 (bytes 8(t & 1).., low nibbles for t < 2, high for t >= 2) and two byte permutes split
// them into the even / odd slot order.  1024 values of a row are 576 bytes.
//
// FMT 3 is Q4_0 with the scale decoded as IEEE f16 (csrc/q4_dot.c:9-35), for x that the caller quantised to Q8
// and dequantised (ComputeBackend::q4_matvec_pair_batch).
//
// GGUF Q8_0 (FMT 2; ggml.rs:136-151: w = d * q, q int8) the same way with s8 x s8 MMAs: 8 weight bytes of a
// lane are split into even / odd elements by two byte permutes (the tables' k order); 1024 values of a row are
// 1088 bytes, u64 tensor-map elements (136 per chunk, box rows of 138: see mma_sb).
//
// Decode fusions (batch 1, q4k_mma_kernel<1, PRO, EPI>, the modes compile-time): the x tables can be built
// from RMSNorm(x) (rms from f64 sums of squares per 16 values left by the
// previous matvec's epilogue, summed in a fixed order by one warp of every CTA;
// x / rms * (offset + w) as residual.rs:17-35) or from silu(gate) * up
// (ffn/mod.rs:87-94), each CTA transforming only its K part; and the output can
// be added to y in place (the residual) with the f64 sums of squares of the new
// y per 16 rows written for the next matvec's norm.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "q4k_mma_dev.cuh"

namespace larql {

// ggml / half.rs f16 decode (crates/larql-models/src/quant/half.rs:4-20): IEEE, subnormals at half value.
__device__ __forceinline__ float h2f_halfrs(uint32_t h16) {
    const float v = __half2float(__ushort_as_half(static_cast<unsigned short>(h16)));
    return (h16 & 0x7C00u) == 0u ? v * 0.5f : v;
}

// One GGUF-144 Q4_K super-block of the warp's 16 rows (hdr: row g's 144-byte block inside the stage, 16-byte
// aligned; row g + 8 is 8 * 576 bytes further), on the Q4_K tables.
template <int NT, bool LLAMA = false>
__device__ __forceinline__ void mma_superblock_gguf(const uint8_t* hdr, const uint2* __restrict__ xs,
                                                    const uint32_t* __restrict__ ms, const float4* __restrict__ ws,
                                                    int lane, int t, float (&acc)[NT][4]) {
    constexpr int R8 = 8 * mma_sb(5);
    const uint32_t hg = lds32(hdr), hg8 = lds32(hdr + R8);
    // get_scale_min_k4 over bytes 4..15 (words w0 w1 w2): sc 0..3 = w0 & 63, mn 0..3 = w1 & 63,
    // sc 4..7 = (w2 & 15) | (w0 >> 6) << 4, mn 4..7 = (w2 >> 4) | (w1 >> 6) << 4, byte-wise
    const uint32_t w0 = lds32(hdr + 4), w1 = lds32(hdr + 8), w2 = lds32(hdr + 12);
    const uint32_t v0 = lds32(hdr + R8 + 4), v1 = lds32(hdr + R8 + 8), v2 = lds32(hdr + R8 + 12);
    const uint32_t s0g = w0 & 0x3F3F3F3Fu, s1g = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
    const uint32_t s0g8 = v0 & 0x3F3F3F3Fu, s1g8 = (v2 & 0x0F0F0F0Fu) | ((v0 >> 2) & 0x30303030u);
    int ai[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ai[nt][0] = ai[nt][1] = ai[nt][2] = ai[nt][3] = 0;
    // ggml.rs: sub-block j's 16 bytes at 16 + 16 j, elements 0..15 low nibbles, 16..31 high; llama.cpp (LLAMA):
    // sub-blocks 2c / 2c + 1 in the low / high nibbles of the 32 bytes at 16 + 32 c, element e at byte e.  Either
    // way lane t reads the 8 bytes holding its elements 8t..8t+7 and shifts their nibbles into place.
    const uint8_t* qp = LLAMA ? hdr + 16 + 8 * t : hdr + 16 + 8 * (t & 1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int off = LLAMA ? 32 * (j >> 1) : 16 * j;
        const int sh = LLAMA ? 4 * (j & 1) : 4 * (t >> 1);
        const uint2 wg = *reinterpret_cast<const uint2*>(qp + off);
        const uint2 wg8 = *reinterpret_cast<const uint2*>(qp + R8 + off);
        const uint32_t L = (wg.x >> sh) & 0x0F0F0F0Fu, H = (wg.y >> sh) & 0x0F0F0F0Fu;
        const uint32_t L8 = (wg8.x >> sh) & 0x0F0F0F0Fu, H8 = (wg8.y >> sh) & 0x0F0F0F0Fu;
        const uint32_t a0 = __byte_perm(L, H, 0x6420), a2 = __byte_perm(L, H, 0x7531);
        const uint32_t a1 = __byte_perm(L8, H8, 0x6420), a3 = __byte_perm(L8, H8, 0x7531);
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
    // the 8 mins of rows g / g + 8 in k slots 0..7: lane t = 0 sub-blocks 0-3, t = 1 sub-blocks 4-7
    const uint32_t m0 = t == 0 ? (w1 & 0x3F3F3F3Fu) : (((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u));
    const uint32_t m8 = t == 0 ? (v1 & 0x3F3F3F3Fu) : (((v2 >> 4) & 0x0F0F0F0Fu) | ((v1 >> 2) & 0x30303030u));
    const uint32_t am0 = t < 2 ? m0 : 0u, am1 = t < 2 ? m8 : 0u;
    // d / dmin: half.rs (ggml.rs) or IEEE (llama.cpp's and the Metal kernels' half)
    const float dg = LLAMA ? h2f_lo(hg) : h2f_halfrs(hg & 0xFFFFu), dmg = LLAMA ? h2f_hi(hg) : h2f_halfrs(hg >> 16);
    const float dg8 = LLAMA ? h2f_lo(hg8) : h2f_halfrs(hg8 & 0xFFFFu);
    const float dmg8 = LLAMA ? h2f_hi(hg8) : h2f_halfrs(hg8 >> 16);
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

// One 256-value group (8 Q4_0 blocks) of the warp's 16 rows: hdr points at row g's first block inside the stage
// (4-byte aligned; block j starts 18 j bytes further, so odd blocks start 2 bytes off a word).
template <int NT, bool IEEE = false>
__device__ __forceinline__ void q40_group(const uint8_t* hdr, const uint2* __restrict__ xs,
                                          const int* __restrict__ cs, const float4* __restrict__ ws, int lane, int t,
                                          float (&acc)[NT][4]) {
    constexpr int R8 = 8 * mma_sb(1);
    float part[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint8_t* bp = hdr + 18 * j;
        uint32_t wg, wg8, dw, dw8;
        if (j & 1) {  // block starts at 2 mod 4: d in the upper half of the word before it, nibbles aligned
            wg = lds32(bp + 2 + 4 * t);
            wg8 = lds32(bp + R8 + 2 + 4 * t);
            dw = lds32(bp - 2) >> 16;
            dw8 = lds32(bp + R8 - 2) >> 16;
        } else {      // aligned block: nibble word t straddles two words
            wg = __funnelshift_r(lds32(bp + 4 * t), lds32(bp + 4 * t + 4), 16);
            wg8 = __funnelshift_r(lds32(bp + R8 + 4 * t), lds32(bp + R8 + 4 * t + 4), 16);
            dw = lds32(bp) & 0xFFFFu;
            dw8 = lds32(bp + R8) & 0xFFFFu;
        }
        const uint32_t a0 = wg & 0x0F0F0F0Fu, a2 = (wg >> 4) & 0x0F0F0F0Fu;
        const uint32_t a1 = wg8 & 0x0F0F0F0Fu, a3 = (wg8 >> 4) & 0x0F0F0F0Fu;
        const float dg = IEEE ? h2f_lo(dw) : h2f_halfrs(dw), dg8 = IEEE ? h2f_lo(dw8) : h2f_halfrs(dw8);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 b = xs[(j * NT + nt) * 32 + lane];
            const int2 ci = *reinterpret_cast<const int2*>(cs + (j * NT + nt) * 8 + 2 * t);
            uint32_t c[4];
            mma_u8s8_c(c, a0, a1, a2, a3, b.x, b.y, ci.x, ci.y);
            part[nt][0] = fmaf(dg, i2f_small(static_cast<int>(c[0])), part[nt][0]);
            part[nt][1] = fmaf(dg, i2f_small(static_cast<int>(c[1])), part[nt][1]);
            part[nt][2] = fmaf(dg8, i2f_small(static_cast<int>(c[2])), part[nt][2]);
            part[nt][3] = fmaf(dg8, i2f_small(static_cast<int>(c[3])), part[nt][3]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float4 w = ws[nt * 4 + t];
        acc[nt][0] = fmaf(part[nt][0], w.x, acc[nt][0]);
        acc[nt][1] = fmaf(part[nt][1], w.y, acc[nt][1]);
        acc[nt][2] = fmaf(part[nt][2], w.x, acc[nt][2]);
        acc[nt][3] = fmaf(part[nt][3], w.y, acc[nt][3]);
    }
}

// One 256-value group (8 GGUF Q8_0 blocks of 34 B) of the warp's 16 rows; hdr is 16-byte aligned, block j
// starts 34 j bytes further (odd blocks 2 bytes off a word).
template <int NT>
__device__ __forceinline__ void q80_group(const uint8_t* hdr, const uint2* __restrict__ xs,
                                          const float4* __restrict__ ws, int lane, int t, float (&acc)[NT][4]) {
    constexpr int R8 = 8 * mma_sb(2);
    float part[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint8_t* bp = hdr + 34 * j;
        uint32_t lo, hi, lo8, hi8, dw, dw8;  // weight bytes 8t .. 8t+7 (at bp + 2 + 8t) of rows g, g + 8
        if (j & 1) {
            lo = lds32(bp + 2 + 8 * t);
            hi = lds32(bp + 6 + 8 * t);
            lo8 = lds32(bp + R8 + 2 + 8 * t);
            hi8 = lds32(bp + R8 + 6 + 8 * t);
            dw = lds32(bp - 2) >> 16;
            dw8 = lds32(bp + R8 - 2) >> 16;
        } else {
            const uint32_t w0 = lds32(bp + 8 * t), w1 = lds32(bp + 8 * t + 4), w2 = lds32(bp + 8 * t + 8);
            const uint32_t v0 = lds32(bp + R8 + 8 * t), v1 = lds32(bp + R8 + 8 * t + 4), v2 = lds32(bp + R8 + 8 * t + 8);
            lo = __funnelshift_r(w0, w1, 16);
            hi = __funnelshift_r(w1, w2, 16);
            lo8 = __funnelshift_r(v0, v1, 16);
            hi8 = __funnelshift_r(v1, v2, 16);
            dw = lds32(bp) & 0xFFFFu;
            dw8 = lds32(bp + R8) & 0xFFFFu;
        }
        const uint32_t a0 = __byte_perm(lo, hi, 0x6420), a2 = __byte_perm(lo, hi, 0x7531);
        const uint32_t a1 = __byte_perm(lo8, hi8, 0x6420), a3 = __byte_perm(lo8, hi8, 0x7531);
        const float dg = h2f_halfrs(dw), dg8 = h2f_halfrs(dw8);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 b = xs[(j * NT + nt) * 32 + lane];
            uint32_t c[4];
            mma_s8s8(c, a0, a1, a2, a3, b.x, b.y);
            part[nt][0] = fmaf(dg, i2f_small(static_cast<int>(c[0])), part[nt][0]);
            part[nt][1] = fmaf(dg, i2f_small(static_cast<int>(c[1])), part[nt][1]);
            part[nt][2] = fmaf(dg8, i2f_small(static_cast<int>(c[2])), part[nt][2]);
            part[nt][3] = fmaf(dg8, i2f_small(static_cast<int>(c[3])), part[nt][3]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float4 w = ws[nt * 4 + t];
        acc[nt][0] = fmaf(part[nt][0], w.x, acc[nt][0]);
        acc[nt][1] = fmaf(part[nt][1], w.y, acc[nt][1]);
        acc[nt][2] = fmaf(part[nt][2], w.x, acc[nt][2]);
        acc[nt][3] = fmaf(part[nt][3], w.y, acc[nt][3]);
    }
}

__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// 8 bits b0..b3 of pairs in a 16-bit value (pair k at bits 4k..4k+1) spread to bits 4-5 of byte k.
__device__ __forceinline__ uint32_t q6_hi_bytes(uint32_t pairs) {
    uint32_t y = (pairs | (pairs << 8)) & 0x00FF00FFu;
    y = (y | (y << 4)) & 0x0F0F0F0Fu;
    return y << 4;
}

// One Q6_K super-block (ql[128] | qh[64] | sc[16] | d, 210 B) of the warp's 16 rows: hdr points at row g's
// super-block in the stage; `odd`: it starts 2 bytes off a word (odd super-blocks of a 1680-byte chunk row).
template <int NT>
__device__ __forceinline__ void q6k_superblock(const uint8_t* hdr, bool odd, const uint2* __restrict__ xs,
                                               const int* __restrict__ cs, const float4* __restrict__ ws, int lane,
                                               int t, float (&acc)[NT][4]) {
    constexpr int R8 = 8 * kMmaRowBytesQ6K;
    int ai[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) ai[nt][0] = ai[nt][1] = ai[nt][2] = ai[nt][3] = 0;
    const bool first = t < 2;  // this lane's elements lie in the group's first 16-value sub-block
#pragma unroll 2
    for (int G = 0; G < 8; ++G) {
        const uint8_t* qp = hdr + 16 * G + 4 * t;
        uint32_t wg, wg8;
        if (odd) {
            wg = lds16(qp) | (lds16(qp + 2) << 16);
            wg8 = lds16(qp + R8) | (lds16(qp + R8 + 2) << 16);
        } else {
            wg = lds32(qp);
            wg8 = lds32(qp + R8);
        }
        const uint32_t hg = lds16(hdr + 128 + 8 * G + 2 * t), hg8 = lds16(hdr + R8 + 128 + 8 * G + 2 * t);
        const uint32_t ae = (wg & 0x0F0F0F0Fu) | q6_hi_bytes(hg & 0x3333u);
        const uint32_t ao = ((wg >> 4) & 0x0F0F0F0Fu) | q6_hi_bytes((hg >> 2) & 0x3333u);
        const uint32_t ae8 = (wg8 & 0x0F0F0F0Fu) | q6_hi_bytes(hg8 & 0x3333u);
        const uint32_t ao8 = ((wg8 >> 4) & 0x0F0F0F0Fu) | q6_hi_bytes((hg8 >> 2) & 0x3333u);
        const uint32_t scw = lds16(hdr + 192 + 2 * G), scw8 = lds16(hdr + R8 + 192 + 2 * G);
        const int sa = static_cast<int>(static_cast<int8_t>(scw & 0xFFu)), sb = static_cast<int>(static_cast<int8_t>(scw >> 8));
        const int sa8 = static_cast<int>(static_cast<int8_t>(scw8 & 0xFFu)), sb8 = static_cast<int>(static_cast<int8_t>(scw8 >> 8));
        const uint32_t z = 0u;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 b = xs[(G * NT + nt) * 32 + lane];
            const int2 c0 = *reinterpret_cast<const int2*>(cs + ((G * 2) * NT + nt) * 8 + 2 * t);
            const int2 c1 = *reinterpret_cast<const int2*>(cs + ((G * 2 + 1) * NT + nt) * 8 + 2 * t);
            uint32_t r0[4], r1[4];
            mma_u8s8_c(r0, first ? ae : z, first ? ae8 : z, first ? ao : z, first ? ao8 : z, b.x, b.y, c0.x, c0.y);
            mma_u8s8_c(r1, first ? z : ae, first ? z : ae8, first ? z : ao, first ? z : ao8, b.x, b.y, c1.x, c1.y);
            ai[nt][0] += sa * static_cast<int>(r0[0]) + sb * static_cast<int>(r1[0]);
            ai[nt][1] += sa * static_cast<int>(r0[1]) + sb * static_cast<int>(r1[1]);
            ai[nt][2] += sa8 * static_cast<int>(r0[2]) + sb8 * static_cast<int>(r1[2]);
            ai[nt][3] += sa8 * static_cast<int>(r0[3]) + sb8 * static_cast<int>(r1[3]);
        }
    }
    const float dg = h2f_lo(lds16(hdr + 208)), dg8 = h2f_lo(lds16(hdr + R8 + 208));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float4 w = ws[nt * 4 + t];
        acc[nt][0] = fmaf(dg * w.x, static_cast<float>(ai[nt][0]), acc[nt][0]);
        acc[nt][1] = fmaf(dg * w.y, static_cast<float>(ai[nt][1]), acc[nt][1]);
        acc[nt][2] = fmaf(dg8 * w.x, static_cast<float>(ai[nt][2]), acc[nt][2]);
        acc[nt][3] = fmaf(dg8 * w.y, static_cast<float>(ai[nt][3]), acc[nt][3]);
    }
}

template <int B, int PRO, int EPI, int FMT = 0>
__global__ void __launch_bounds__(32 * (kMmaMaxWarps + 1), 1)
    q4k_mma_kernel(const __grid_constant__ CUtensorMap wmap, const float* __restrict__ x, float* __restrict__ y,
                   float* __restrict__ partial, int* __restrict__ tickets, const MmaPlan p, int* status,
                   const MmaFuse fz) {
    constexpr int NT = mma_ntiles(B);
    constexpr int NP = mma_planes(B);
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* empty = full + p.NS;
    volatile int* flags = reinterpret_cast<volatile int*>(empty + p.NS);  // [0] abort, [1] last-CTA ticket, [2] rms
    volatile float* rms_s = reinterpret_cast<volatile float*>(flags + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ncons = 32 * p.NW;
    // the producer's first TMA would otherwise wait for the descriptor to be fetched
    if (warp == p.NW && lane == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
    pdl_launch_dependents();
    if (tid == 0) {
        for (int i = 0; i < p.NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], p.NW);
        }
        flags[0] = 0;
        flags[1] = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == p.NW) {  // producer warp: one elected lane issues the TMA boxes
        if (lane == 0) {
            // L2 prefetch cursor, p.PF boxes ahead of the shared-memory loads: the
            // ring holds only 2-4 boxes, the prefetches keep more DRAM reads in flight
            int pf_item = blockIdx.x, pf_c = 0, pf_c1 = 0;
            auto pf_next = [&]() {
                while (pf_item < p.nitems) {
                    const int part = pf_item / p.ntiles;
                    if (pf_c1 == 0) {
                        pf_c = part * p.nchunks / p.nparts;
                        pf_c1 = (part + 1) * p.nchunks / p.nparts;
                    }
                    if (pf_c < pf_c1) {
                        tma_prefetch_2d(&wmap, pf_c * (mma_rb(FMT) / mma_elem(FMT)), (pf_item - part * p.ntiles) * p.RT);
                        ++pf_c;
                        return;
                    }
                    pf_item += gridDim.x;
                    pf_c1 = 0;
                }
            };
            for (int i = 0; i < p.PF; ++i) pf_next();
            int k = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < p.nitems && ok; item += gridDim.x) {
                const int part = item / p.ntiles, tile = item - part * p.ntiles;
                const int c0 = part * p.nchunks / p.nparts, c1 = (part + 1) * p.nchunks / p.nparts;
                for (int c = c0; c < c1; ++c, ++k) {
                    pf_next();
                    const int st = k % p.NS;
                    if (k >= p.NS && !mbar_wait(&empty[st], ((k / p.NS) - 1) & 1, status, 41)) {
                        ok = false;
                        flags[0] = 1;
                        break;
                    }
                    if (flags[0]) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(p.stage_bytes));
                    tma_load_2d(smem + static_cast<size_t>(st) * p.stage_bytes, &wmap, c * (mma_rb(FMT) / mma_elem(FMT)),
                                tile * p.RT, &full[st]);
                }
            }
            // every issued box must land before the CTA's shared memory goes away
            for (int jj = max(0, k - p.NS); jj < k; ++jj)
                if (!mbar_wait(&full[jj % p.NS], (jj / p.NS) & 1, status, 42)) break;
        }
        return;
    }

    // x, y, the partials and the tickets belong to the kernels before this one until
    // they finish (programmatic dependent launch): the producer above streams
    // weights meanwhile; the consumers touch nothing else before this wait
    pdl_wait();
    if constexpr (PRO == 1) {
        if (warp == 0) {  // ordered by the first table build's barrier
            const int ncnt = (p.K + 15) / 16;
            double v = 0.0;
            for (int i = lane; i < ncnt; i += 32) v += __ldcg(fz.ss_in + i);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) *rms_s = static_cast<float>(sqrt(v / static_cast<double>(p.K) + static_cast<double>(fz.eps)));
        }
    }
    const int g = lane >> 2, t = lane & 3;
    const int rg = warp % p.NG, ks = warp / p.NG;  // row group, K slice (super-blocks ks, ks + KS, ...)
    const int row_in_tile = 16 * rg + g;
    float* red = reinterpret_cast<float*>(smem + p.red_off);  // [2][KS][B][RT] when KS > 1
    int rbuf = 0;
    // batch row of each of this thread's C columns (2t, 2t + 1 of every n-tile)
    int colb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        colb[nt][0] = (nt * 8 + 2 * t) / NP;
        colb[nt][1] = (nt * 8 + 2 * t + 1) / NP;
    }
    const uint2* xt = reinterpret_cast<const uint2*>(smem + p.xt_off);
    const uint32_t* mt = reinterpret_cast<const uint32_t*>(smem + p.mt_off);
    const float4* wt = reinterpret_cast<const float4*>(smem + p.wt_off);

    int cur_part = -1;
    int k = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < p.nitems; item += gridDim.x) {
        const int part = item / p.ntiles, tile = item - part * p.ntiles;
        const int c0 = part * p.nchunks / p.nparts, c1 = (part + 1) * p.nchunks / p.nparts;
        if (part != cur_part) {
            // uniform decision: every consumer warp reaches this barrier for the same item
            if (named_bar_red_or(1, ncons, !ok)) return;
            mma_build_tables<B, NT, PRO, FMT>(x, p.K, c0, c1, smem, p, tid, warp, lane, fz, rms_s);
            cur_part = part;
        }
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        for (int c = c0; c < c1; ++c, ++k) {
            const int st = k % p.NS;
            if (ok) {
                const bool got = !flags[0] && mbar_wait(&full[st], (k / p.NS) & 1, status, 43);
                ok = __all_sync(0xffffffffu, got);
                if (!ok && lane == 0) flags[0] = 1;
            }
            if (ok) {
                const uint8_t* wrow = smem + static_cast<size_t>(st) * p.stage_bytes + row_in_tile * mma_sb(FMT);
                const int sbl0 = (c - c0) * mma_sbc(FMT);
#pragma unroll 1
                for (int s4 = ks; s4 < mma_sbc(FMT); s4 += p.KS) {
                    const int sbl = sbl0 + s4;
                    if constexpr (FMT == 4)
                        q6k_superblock<NT>(wrow + s4 * 210, (s4 & 1) != 0, xt + sbl * 8 * NT * 32,
                                           reinterpret_cast<const int*>(mt) + sbl * 16 * NT * 8, wt + sbl * NT * 4,
                                           lane, t, acc);
                    else if constexpr (FMT == 2)
                        q80_group<NT>(wrow + s4 * 272, xt + sbl * 8 * NT * 32, wt + sbl * NT * 4, lane, t, acc);
                    else if constexpr (FMT == 5 || FMT == 6)
                        mma_superblock_gguf<NT, FMT == 6>(wrow + s4 * 144, xt + sbl * 8 * NT * 32, mt + sbl * NT * 32,
                                                wt + sbl * NT * 4, lane, t, acc);
                    else if constexpr (FMT == 1 || FMT == 3)
                        q40_group<NT, FMT == 3>(wrow + s4 * 144, xt + sbl * 8 * NT * 32,
                                      reinterpret_cast<const int*>(mt) + sbl * 8 * NT * 8, wt + sbl * NT * 4, lane, t,
                                      acc);
                    else
                        mma_superblock<NT>(wrow + s4 * 148, xt + sbl * 8 * NT * 32, mt + sbl * NT * 32,
                                           wt + sbl * NT * 4, lane, t, acc);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
        }
        const size_t N = static_cast<size_t>(p.N);
        float* dst = p.nparts == 1 ? y : partial + static_cast<size_t>(part) * B * N;
        if (ok) {
            const int rowg = tile * p.RT + row_in_tile;
            float* rw = red + ((rbuf * p.KS + ks) * B) * p.RT + row_in_tile;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                float sg = 0.f, sg8 = 0.f;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        sg += colb[nt][q] == b ? acc[nt][q] : 0.f;
                        sg8 += colb[nt][q] == b ? acc[nt][2 + q] : 0.f;
                    }
                }
                sg += __shfl_xor_sync(0xffffffffu, sg, 1);
                sg += __shfl_xor_sync(0xffffffffu, sg, 2);
                sg8 += __shfl_xor_sync(0xffffffffu, sg8, 1);
                sg8 += __shfl_xor_sync(0xffffffffu, sg8, 2);
                if (EPI && p.KS == 1 && p.nparts == 1) {  // warp-uniform; B == 1
                    double q = 0.0;
                    if (t == 0 && rowg < p.N) {
                        const float v = y[rowg] + sg;
                        y[rowg] = v;
                        q = static_cast<double>(v) * static_cast<double>(v);
                    }
                    if (t == 0 && rowg + 8 < p.N) {
                        const float v = y[rowg + 8] + sg8;
                        y[rowg + 8] = v;
                        q += static_cast<double>(v) * static_cast<double>(v);
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
                    const int grp = tile * p.NG + rg;
                    if (lane == 0 && 16 * grp < p.N) fz.ss_out[grp] = q;
                } else if (t == 0) {
                    if (p.KS == 1) {
                        if (rowg < p.N) dst[b * N + rowg] = sg;
                        if (rowg + 8 < p.N) dst[b * N + rowg + 8] = sg8;
                    } else {
                        rw[b * p.RT] = sg;
                        rw[b * p.RT + 8] = sg8;
                    }
                }
            }
        }
        if (p.KS > 1) {
            // the K slices of a row group add their sums in slice order (double-buffered, one barrier)
            if (named_bar_red_or(1, ncons, !ok)) return;
            if (ks == 0) {
                const float* rr = red + (rbuf * p.KS * B) * p.RT + 16 * rg;
                if (EPI && p.nparts == 1) {  // B == 1: lanes 0..15 hold the group's rows
                    const int row = tile * p.RT + 16 * rg + (lane & 15);
                    double q = 0.0;
                    if (lane < 16 && row < p.N) {
                        float s = 0.f;
                        for (int qq = 0; qq < p.KS; ++qq) s += rr[qq * p.RT + lane];
                        const float v = y[row] + s;
                        y[row] = v;
                        q = static_cast<double>(v) * static_cast<double>(v);
                    }
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
                    const int grp = tile * p.NG + rg;
                    if (lane == 0 && 16 * grp < p.N) fz.ss_out[grp] = q;
                } else {
                    for (int i = lane; i < 16 * B; i += 32) {
                        const int b = i >> 4, r = i & 15, row = tile * p.RT + 16 * rg + r;
                        float s = 0.f;
                        for (int q = 0; q < p.KS; ++q) s += rr[(q * B + b) * p.RT + r];
                        if (row < p.N) dst[b * N + row] = s;
                    }
                }
            }
            rbuf ^= 1;
        }
        if (p.nparts > 1) {
            __threadfence();
            if (named_bar_red_or(1, ncons, !ok)) return;
            if (tid == 0) {
                const int old = atomicAdd(&tickets[tile], 1);
                const int last = old == p.nparts - 1;
                if (last) tickets[tile] = 0;  // ready for the next launch
                flags[1] = last;
            }
            named_bar_sync(1, ncons);
            if (EPI && flags[1]) {  // B == 1; ncons >= RT, so thread r owns row r of the tile
                __threadfence();
                if (32 * warp < p.RT) {
                    const int row = tile * p.RT + tid;
                    double q = 0.0;
                    if (tid < p.RT && row < p.N) {
                        float s = 0.f;
                        for (int pp = 0; pp < p.nparts; ++pp) s += __ldcg(partial + static_cast<size_t>(pp) * N + row);
                        const float v = y[row] + s;
                        y[row] = v;
                        q = static_cast<double>(v) * static_cast<double>(v);
                    }
#pragma unroll
                    for (int o = 8; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
                    const int grp = tile * p.NG + 2 * warp + (lane >> 4);
                    if ((lane & 15) == 0 && 16 * (2 * warp + (lane >> 4)) < p.RT && 16 * grp < p.N) fz.ss_out[grp] = q;
                }
            } else if (flags[1]) {
                __threadfence();
                for (int i = tid; i < p.RT * B; i += ncons) {
                    const int b = i / p.RT, r = i - b * p.RT, row = tile * p.RT + r;
                    if (row < p.N) {
                        float s = 0.f;
                        for (int q = 0; q < p.nparts; ++q) s += __ldcg(partial + (static_cast<size_t>(q) * B + b) * N + row);
                        y[b * N + row] = s;
                    }
                }
            }
            named_bar_sync(1, ncons);
        }
    }
}

// Tables + stages for one (NG, KS, nparts) choice; false if it does not fit.
static bool mma_layout(MmaPlan& p, int num_sms) {
    p.NW = p.NG * p.KS;
    p.RT = 16 * p.NG;
    p.stage_bytes = p.RT * mma_sb(p.fmt);
    p.kpc = (p.nchunks + p.nparts - 1) / p.nparts;
    const int sbc = mma_sbc(p.fmt);
    const int xt_bytes = p.kpc * 8 * sbc * p.NT * 256;
    // Q4_K: B fragments of the sub-block sums per 256 values; Q4_0: C inputs, 8 ints per block and n-tile
    // Q4_K: B fragments of the sub-block sums; Q4_0: C inputs per block; Q6_K: C inputs per 16-value sub-block
    const int mt_bytes = p.fmt == 4 ? p.kpc * 16 * sbc * p.NT * 32
                                    : (p.fmt == 2 ? 0
                                                  : (p.fmt == 0 || p.fmt == 5 || p.fmt == 6 ? p.kpc * 4 * p.NT * 128
                                                                              : p.kpc * 32 * p.NT * 32));
    const int wt_bytes = p.kpc * sbc * p.NT * 64;
    const int red_bytes = p.KS > 1 ? 2 * p.KS * p.batch * p.RT * 4 : 0;
    const int fixed = xt_bytes + mt_bytes + wt_bytes + red_bytes + 2 * 8 * 8 + 16;
    if (p.NS <= 0) {
        p.NS = (kSmemLimit - fixed) / p.stage_bytes;
        if (p.NS > 8) p.NS = 8;
    }
    if (p.NS < 2) return false;
    p.xt_off = p.NS * p.stage_bytes;
    p.mt_off = p.xt_off + xt_bytes;
    p.wt_off = p.mt_off + mt_bytes;
    p.red_off = p.wt_off + wt_bytes;
    p.bar_off = p.red_off + red_bytes;
    p.smem = p.bar_off + 2 * p.NS * 8 + 16;
    if (p.smem > kSmemLimit) return false;
    p.ntiles = (p.N + p.RT - 1) / p.RT;
    p.nitems = p.ntiles * p.nparts;
    p.grid = p.nitems < num_sms ? p.nitems : num_sms;
    return true;
}

// Picks the tile shape (row groups x K slices, 4..8 warps), the K split across
// CTAs and the ring depth with a cost model (microseconds) fitted to measured
// B200 sweeps of every plan on the 4096..128256 x 4096..14336 x batch 1..8
// cells (rms error 12%):
//   fixed + max(streaming at 38 GB/s per busy SM, warp-instructions at an issue
//   efficiency falling with n-tiles and rising with warps) + x-table builds
//   + split-K tickets per wave + K-slice reductions per wave.
bool q4k_mma_make_plan(int N, int K, int batch, int num_sms, MmaPlan* out, const int* force, int fmt) {
    const int cv = 256 * mma_sbc(fmt);  // values per chunk
    if (N <= 0 || K <= 0 || K % cv || batch < 1 || batch > 8 || fmt < 0 || fmt > 6) return false;
    const int nchunks = K / cv;
    const double wbytes = static_cast<double>(N) * (K / 256) * mma_sbb(fmt);
    const int NT = mma_ntiles(batch);
    const double instr_sb = 150.0 + 95.0 * NT;  // warp-instructions per super-block per 16-row group
    const double eff_nt = 0.633 + (0.401 - 0.633) * (NT - 1) / 2.0;
    bool found = false;
    double best = 0;
    MmaPlan bp{};
    for (int ng = 1; ng <= 8; ++ng) {
        if (force[0] > 0 && ng != force[0]) continue;
        for (int ks = 1; ks <= 4; ks *= 2) {
            if (force[1] > 0 && ks != force[1]) continue;
            // the cost model was fitted on 4-, 6- and 8-warp tiles; other widths measured slower
            if (ng * ks > kMmaMaxWarps || (force[0] == 0 && force[1] == 0 && (ng * ks) % 2) ||
                (force[0] == 0 && ng * ks < 4))
                continue;
            for (int parts = 1; parts <= nchunks; ++parts) {
                if (force[3] > 0 && parts != force[3]) continue;
                MmaPlan p{};
                p.fmt = fmt;
                p.N = N;
                p.K = K;
                p.batch = batch;
                p.NT = NT;
                p.NG = ng;
                p.KS = ks;
                p.NS = force[2];
                p.PF = force[4] > 0 ? force[4] : kMmaPrefetch;
                p.nchunks = nchunks;
                p.nparts = parts;
                if (!mma_layout(p, num_sms)) continue;
                const int waves = (p.nitems + num_sms - 1) / num_sms;
                const double eff = eff_nt * std::pow(p.NW / 8.0, 0.62);
                const double item_instr = static_cast<double>(ng) * p.kpc * mma_sbc(fmt) * instr_sb;
                const double mem = wbytes / (p.grid * 38283.0);
                const double comp = waves * item_instr / (4 * 1900.0 * eff);
                double tus = 8.31 + std::max(mem, comp);
                tus += std::min(waves, parts) * 2.172 * p.kpc * (1 + batch / 4.0) / 4.0;
                if (parts > 1) tus += 2.243 * waves;
                if (ks > 1) tus += 0.242 * waves;
                if (!found || tus < best) {
                    found = true;
                    best = tus;
                    bp = p;
                }
            }
        }
    }
    // Batch 1, Q4_K, K <= 4096: where one wave of whole tiles (no split-K) covers at least half of the SMs, it
    // beats the model's pick.  An in-graph sweep of every plan on 1536 / 4096 / 6144 / 11008 / 14336 x 4096 found
    // the single wave with the most tiles (16-row groups x 4 K slices, or 8 warps of row groups and slices) 2-19 %
    // faster than plans with a ragged second wave or split-K parts, whose cost the model underrates for matrices
    // this small.  At K = 14336 the split-K plans stay faster (4096 x 14336: 12.2 us against 14.7 for one wave).
    if (found && batch == 1 && fmt == 0 && nchunks <= 4 && force[0] == 0 && force[1] == 0 && force[3] == 0) {
        MmaPlan wave{};
        for (int ng = 1; ng <= 8; ng *= 2) {
            MmaPlan p{};
            p.fmt = fmt;
            p.N = N;
            p.K = K;
            p.batch = batch;
            p.NT = NT;
            p.NG = ng;
            p.KS = std::min(4, kMmaMaxWarps / ng);
            p.NS = force[2];
            p.PF = force[4] > 0 ? force[4] : kMmaPrefetch;
            p.nchunks = nchunks;
            p.nparts = 1;
            if (!mma_layout(p, num_sms)) continue;
            if (p.ntiles > num_sms || 2 * p.ntiles < num_sms) continue;
            if (wave.N == 0 || p.ntiles > wave.ntiles) wave = p;
        }
        if (wave.N != 0) bp = wave;
    }
    if (found) *out = bp;
    return found;
}

int mma_chunk_bytes(int fmt) { return mma_rb(fmt); }

// 2-D map of a Q4_K, Q4_0 (u32 elements) or GGUF Q8_0 (u64) weight as [N rows][row bytes / element], boxes of
// H rows x one 1024-value chunk.
int mma_encode_map(void* encode_fn, const void* w, int N, int K, int fmt, int H, CUtensorMap* map) {
    using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    const uint64_t row_bytes = static_cast<uint64_t>(K / 256) * mma_sbb(fmt);
    if (row_bytes % 16) return -1;
    const uint64_t el = static_cast<uint64_t>(mma_elem(fmt));
    cuuint64_t dims[2] = {row_bytes / el, static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(mma_sb(fmt) / el), static_cast<cuuint32_t>(H)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = reinterpret_cast<Fn>(encode_fn)(map, el == 8 ? CU_TENSOR_MAP_DATA_TYPE_UINT64
                                                             : CU_TENSOR_MAP_DATA_TYPE_UINT32,
                                                 2, const_cast<void*>(w), dims,
                                                 strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : static_cast<int>(r);
}

size_t q4k_mma_partial_floats(const MmaPlan& p) {
    return p.nparts > 1 ? static_cast<size_t>(p.nparts) * p.batch * p.N : 0;
}

template <int B, int PRO = 0, int EPI = 0, int FMT = 0>
static cudaError_t launch_mma_b(const CUtensorMap& map, const float* x, float* y, float* partial, int* tickets,
                                const MmaPlan& p, int* status, cudaStream_t stream, const MmaFuse& fz = MmaFuse{}) {
    if (p.NW > kMmaMaxWarps) return cudaErrorInvalidValue;
    static DeviceFlags attr_done;
    cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(q4k_mma_kernel<B, PRO, EPI, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    e = launch_pdl(q4k_mma_kernel<B, PRO, EPI, FMT>, dim3(p.grid), dim3(32 * (p.NW + 1)), p.smem, stream, map, x, y,
                   partial, tickets, p, status, fz);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

// y[batch, N] = Q4_K W[N, K] . x[batch, K] through the tensor map of W with
// box height p.RT.  partial: q4k_mma_partial_floats(p) floats; tickets: p.ntiles
// zeroed ints (left zeroed by every complete launch).
cudaError_t launch_q4k_mma(const CUtensorMap& map, const float* x, float* y, float* partial, int* tickets,
                           const MmaPlan& p, int* status, cudaStream_t stream) {
    if (p.fmt == 4) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 4>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.fmt == 3) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 3>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.fmt == 2) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 2>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.fmt == 5) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 5>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.fmt == 6) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 6>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.fmt == 1) {
        switch (p.batch) {
            case 1: return launch_mma_b<1, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 2: return launch_mma_b<2, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 3: return launch_mma_b<3, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 4: return launch_mma_b<4, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 5: return launch_mma_b<5, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 6: return launch_mma_b<6, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 7: return launch_mma_b<7, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            case 8: return launch_mma_b<8, 0, 0, 1>(map, x, y, partial, tickets, p, status, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (p.batch) {
        case 1: return launch_mma_b<1>(map, x, y, partial, tickets, p, status, stream);
        case 2: return launch_mma_b<2>(map, x, y, partial, tickets, p, status, stream);
        case 3: return launch_mma_b<3>(map, x, y, partial, tickets, p, status, stream);
        case 4: return launch_mma_b<4>(map, x, y, partial, tickets, p, status, stream);
        case 5: return launch_mma_b<5>(map, x, y, partial, tickets, p, status, stream);
        case 6: return launch_mma_b<6>(map, x, y, partial, tickets, p, status, stream);
        case 7: return launch_mma_b<7>(map, x, y, partial, tickets, p, status, stream);
        case 8: return launch_mma_b<8>(map, x, y, partial, tickets, p, status, stream);
        default: return cudaErrorInvalidValue;
    }
}

// Batch 1 with the decode fusions of MmaFuse.  pro 2 reads x[0 .. 2K); epi 1 writes y in place and
// ceil(N / 16) sums of squares.
cudaError_t launch_q4k_mma_fused(const CUtensorMap& map, const float* x, float* y, float* partial, int* tickets,
                                 const MmaPlan& p, const MmaFuse& f, int* status, cudaStream_t stream) {
    if (p.batch != 1 || p.fmt != 0 || f.pro < 0 || f.pro > 2 || (f.pro == 1 && (!f.ss_in || !f.nw)) ||
        (f.epi && !f.ss_out))
        return cudaErrorInvalidValue;
    switch (f.pro * 2 + (f.epi ? 1 : 0)) {
        case 0: return launch_mma_b<1, 0, 0>(map, x, y, partial, tickets, p, status, stream, f);
        case 1: return launch_mma_b<1, 0, 1>(map, x, y, partial, tickets, p, status, stream, f);
        case 2: return launch_mma_b<1, 1, 0>(map, x, y, partial, tickets, p, status, stream, f);
        case 4: return launch_mma_b<1, 2, 0>(map, x, y, partial, tickets, p, status, stream, f);
        case 5: return launch_mma_b<1, 2, 1>(map, x, y, partial, tickets, p, status, stream, f);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace larql
