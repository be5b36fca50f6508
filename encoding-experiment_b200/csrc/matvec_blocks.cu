// matvec_blocks.cu — dequant-matvec for the 32-value block formats on CUDA cores:
//
//   Q4_0  18 B / 32: f16 d + 16 nibble bytes, w = d * (q - 8)
//         x as f32  (crates/larql-models/src/quant/ggml.rs:92-110 dequantize + dot; Metal q4_f32_matvec)
//         x as Q8   (crates/larql-compute/csrc/q4_dot.c:169-199 via ComputeBackend::q4_matvec, backend.rs:49)
//   Q8_0  GGUF 34 B / 32: f16 d + 32 int8 (crates/larql-models/src/quant/ggml.rs:136-151 dequantize + dot)
//   Q8    compute layout: int8 values [N*K] + f32 scale per 32 (crates/larql-compute/src/cpu/ops/q8_matvec.rs:36-57),
//         against Q8(x) (quantize_to_q8, q4_common.rs:28-44)
//   Q6_K  210 B / 256: ql[128] low nibbles (sequential pairs), qh[64] high 2 bits (value i at bits 2(i%4) of
//         byte i/4), 16 int8 scales per 16 values, f16 d; w = d * sc * (q - 32)
//         (crates/larql-compute/src/cpu/ops/q6k_matvec.rs:31-87); a thread owns a 64-value quarter of a
//         super-block instead of a block pair
//
// Same staging as the Q4_K kernel: a producer warp streams tiles of RT consecutive rows (one contiguous byte
// range, 16-byte aligned) into a shared-memory ring with 1-D bulk copies; each consumer thread owns one PAIR of
// 32-value blocks (64 values) of the row for the whole kernel, so its slice of x is prepared once in registers
// as int8 digit planes (f32 x: x = 2^e (a*65536 + b*256 + c) per 32-value group) or as the caller's Q8 values.
// Blocks 2p and 2p+1 of a row start at a 4-byte boundary; the first block's payload is 2 bytes off and is
// realigned with funnel shifts.  dp4a gives exact int32 sums per block.
//
// f16 block scales are decoded the way each reference path decodes them: q4_dot.c decodes IEEE exactly; the
// ggml dequantizers use larql-models half.rs, which returns HALF the IEEE value for subnormal f16
// (quant/half.rs:11-14).
#include "common.cuh"
#include "kernels.h"

namespace larql {

enum BlockFmt { kQ4_0 = 0, kQ8_0G = 1, kQ8C = 2, kQ6K = 3 };

// larql-models half.rs:4-20 semantics: IEEE for normals/zero/inf/NaN, subnormals at half value.
__device__ __forceinline__ float f16_half_rs(uint32_t h16) {
    const float v = __half2float(__ushort_as_half(static_cast<unsigned short>(h16)));
    return ((h16 & 0x7C00u) == 0u) ? v * 0.5f : v;
}
__device__ __forceinline__ float f16_ieee(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16)));
}

struct BlkPlan {
    int P;           // block pairs per row (K / 64)
    int m;           // row lanes
    int T, Tpad;     // consumer threads
    int RT;          // rows per tile
    int row_bytes;   // packed bytes per row
    int srow_bytes;  // scale bytes per row (Q8 compute layout), else 0
    int tile_bytes, stile_bytes;
    int nstage, ntiles, grid, red_off, bar_off, smem;
};

constexpr int kBlkThreads = 512;

// x preparation for one 32-value block: NPL digit planes as 8 words; for Q4 the words are split into
// even elements (words 0..3) and odd elements (words 4..7) to match the nibble low/high split.
template <int NPL, bool Q4>
__device__ __forceinline__ void prep_planes_f32(const float* v, uint32_t (&pl)[NPL][8], float& xs, int& xsum_int) {
    float amax = 0.f;
    bool fin = true;  // fmaxf skips NaN, so every value is tested
#pragma unroll
    for (int i = 0; i < 32; ++i) { amax = fmaxf(amax, fabsf(v[i])); fin = fin && isfinite(v[i]); }
    int ex = 0;
    frexpf(amax, &ex);
    const int e = max(-126, min(127, ex - 22));
    const float down = ldexpf(1.0f, -e);
    xs = fin ? ldexpf(1.0f, e) : __int_as_float(0x7fc00000);
    int s = 0;
#pragma unroll
    for (int z = 0; z < NPL; ++z)
#pragma unroll
        for (int w = 0; w < 8; ++w) pl[z][w] = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        int xi = fin ? __float2int_rn(v[i] * down) : 0;
        s += xi;
        // destination word/byte of element i
        int word, pos;
        if (Q4) { const int w8 = i >> 3, t = (i & 7) >> 1, par = i & 1; word = par * 4 + w8; pos = 8 * t; }
        else { word = i >> 2; pos = 8 * (i & 3); }
#pragma unroll
        for (int z = NPL - 1; z >= 1; --z) {
            const int dgt = (xi << 24) >> 24;
            pl[z][word] |= (static_cast<uint32_t>(dgt) & 0xFFu) << pos;
            xi = (xi - dgt) >> 8;
        }
        pl[0][word] |= (static_cast<uint32_t>(xi) & 0xFFu) << pos;
    }
    xsum_int = s;
}

template <bool Q4>
__device__ __forceinline__ void prep_planes_q8(const int8_t* q, uint32_t (&pl)[1][8], int& xsum_int) {
    int s = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) pl[0][w] = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int xi = q[i];
        s += xi;
        int word, pos;
        if (Q4) { const int w8 = i >> 3, t = (i & 7) >> 1, par = i & 1; word = par * 4 + w8; pos = 8 * t; }
        else { word = i >> 2; pos = 8 * (i & 3); }
        pl[0][word] |= (static_cast<uint32_t>(xi) & 0xFFu) << pos;
    }
    xsum_int = s;
}

// x for a 64-value quarter of a Q6_K super-block: three int8 digit planes (x = 2^e (a*65536 + b*256 + c), one
// exponent for the 64 values).  Per 16-value sub-block s the plane words are ordered
// [x0 x4 x8 x12] [x1 x5 x9 x13] [x2 x6 x10 x14] [x3 x7 x11 x15] (words 4s..4s+3 of pa for s < 2, of pb for s >= 2),
// the order in which one byte permute of two ql words and masks of one qh word give the 6-bit values.
// neg[s][z] = -32 * (sum of plane z's digits over sub-block s): the dot accumulators start there, so each
// sum is exactly  sum (q - 32) * digit.
__device__ __forceinline__ void prep_q6k(const float* xp, bool active, uint32_t (&pa)[3][8], uint32_t (&pb)[3][8],
                                         int (&neg)[4][3], float& xs) {
    const float4* x4 = reinterpret_cast<const float4*>(xp);
    float amax = 0.f;
    bool fin = true;  // fmaxf skips NaN, so every value is tested
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float4 f = active ? __ldg(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
        fin = fin && isfinite(f.x) && isfinite(f.y) && isfinite(f.z) && isfinite(f.w);
    }
    int ex = 0;
    frexpf(amax, &ex);
    const int e = max(-126, min(127, ex - 22));
    const float down = ldexpf(1.0f, -e);
    xs = fin ? ldexpf(1.0f, e) : __int_as_float(0x7fc00000);
#pragma unroll
    for (int z = 0; z < 3; ++z)
#pragma unroll
        for (int w = 0; w < 8; ++w) { pa[z][w] = 0u; pb[z][w] = 0u; }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        float v[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 f = active ? __ldg(x4 + 4 * s + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        int sum[3] = {0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            int xi = fin ? __float2int_rn(v[i] * down) : 0;
            const int word = (s & 1) * 4 + (i & 3), pos = 8 * (i >> 2);
            uint32_t(&pl)[3][8] = s < 2 ? pa : pb;
#pragma unroll
            for (int z = 2; z >= 1; --z) {
                const int dgt = (xi << 24) >> 24;
                pl[z][word] |= (static_cast<uint32_t>(dgt) & 0xFFu) << pos;
                sum[z] += dgt;
                xi = (xi - dgt) >> 8;
            }
            pl[0][word] |= (static_cast<uint32_t>(xi) & 0xFFu) << pos;
            sum[0] += xi;
        }
#pragma unroll
        for (int z = 0; z < 3; ++z) neg[s][z] = -32 * sum[z];
    }
}

// One 64-value quarter (chunk c of 4) of a Q6_K super-block starting at `bp` (2-byte aligned) against the
// prepared planes: d * sum_s sc_s * sum (q - 32) * x / 2^e, the digit sums exact in int32
// (|sum| <= 16 * 32 * 128 per sub-block, times |sc| <= 128, four sub-blocks).
__device__ __forceinline__ float q6k_quarter_dot(const uint8_t* bp, const uint8_t* smem_base, int c,
                                                 const uint32_t (&pa)[3][8], const uint32_t (&pb)[3][8],
                                                 const int (&neg)[4][3]) {
    const int mis = static_cast<int>((bp - smem_base) & 3);
    const uint8_t* a = bp - mis;
    const uint32_t sh = 8u * static_cast<uint32_t>(mis);
    uint32_t ql[9], qh[5];
#pragma unroll
    for (int i = 0; i < 9; ++i) ql[i] = lds32(a + 32 * c + 4 * i);
#pragma unroll
    for (int i = 0; i < 5; ++i) qh[i] = lds32(a + 128 + 16 * c + 4 * i);
    const uint32_t scw = __funnelshift_r(lds32(a + 192 + 4 * c), lds32(a + 196 + 4 * c), sh);
    const float d = f16_ieee((lds32(a + 208) >> sh) & 0xFFFFu);
    int A[3] = {0, 0, 0};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const uint32_t w0 = __funnelshift_r(ql[2 * s], ql[2 * s + 1], sh);
        const uint32_t w1 = __funnelshift_r(ql[2 * s + 1], ql[2 * s + 2], sh);
        const uint32_t Q = __funnelshift_r(qh[s], qh[s + 1], sh);
        const uint32_t tA = __byte_perm(w0, w1, 0x6420), tC = __byte_perm(w0, w1, 0x7531);
        uint32_t q[4];
        q[0] = (tA & 0x0F0F0F0Fu) | ((Q << 4) & 0x30303030u);
        q[1] = ((tA >> 4) & 0x0F0F0F0Fu) | ((Q << 2) & 0x30303030u);
        q[2] = (tC & 0x0F0F0F0Fu) | (Q & 0x30303030u);
        q[3] = ((tC >> 4) & 0x0F0F0F0Fu) | ((Q >> 2) & 0x30303030u);
        const int sc = static_cast<int>(static_cast<int8_t>((scw >> (8 * s)) & 0xFFu));
#pragma unroll
        for (int z = 0; z < 3; ++z) {
            int acc = neg[s][z];
#pragma unroll
            for (int t = 0; t < 4; ++t)
                acc = __dp4a(static_cast<int>(q[t]), static_cast<int>(s < 2 ? pa[z][4 * s + t] : pb[z][4 * (s - 2) + t]), acc);
            A[z] += sc * acc;
        }
    }
    float f = static_cast<float>(A[0]);
    f = fmaf(f, 256.0f, static_cast<float>(A[1]));
    f = fmaf(f, 256.0f, static_cast<float>(A[2]));
    return d * f;
}

// exact integer dot of one block against NPL planes; returns the planes combined (value / 2^e), in float
// (the Q8 weights' sums do not fit an int32 combination of three planes).
template <int NPL, bool Q4>
__device__ __forceinline__ float block_dot(const uint32_t* wq, const uint32_t (&pl)[NPL][8], int xsum_int) {
    int acc[NPL];
#pragma unroll
    for (int z = 0; z < NPL; ++z) acc[z] = 0;
    if (Q4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int L = static_cast<int>(wq[i] & 0x0F0F0F0Fu);
            const int H = static_cast<int>((wq[i] >> 4) & 0x0F0F0F0Fu);
#pragma unroll
            for (int z = 0; z < NPL; ++z) {
                acc[z] = __dp4a(L, static_cast<int>(pl[z][i]), acc[z]);
                acc[z] = __dp4a(H, static_cast<int>(pl[z][4 + i]), acc[z]);
            }
        }
        // (q - 8) . x = q . x - 8 * sum(x): the exact combination fits int32 (|.| <= 8 * 2^22 * 32)
        int isum = acc[0];
#pragma unroll
        for (int z = 1; z < NPL; ++z) isum = isum * 256 + acc[z];
        return static_cast<float>(isum - 8 * xsum_int);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int z = 0; z < NPL; ++z) acc[z] = __dp4a(static_cast<int>(wq[i]), static_cast<int>(pl[z][i]), acc[z]);
        float f = static_cast<float>(acc[0]);
#pragma unroll
        for (int z = 1; z < NPL; ++z) f = fmaf(f, 256.0f, static_cast<float>(acc[z]));
        return f;
    }
}

template <int FMT, int NPL, int RPT>
__global__ void __launch_bounds__(kBlkThreads, 1)
    blk_matvec_kernel(const uint8_t* __restrict__ W, const float* __restrict__ wscale, const float* __restrict__ x,
                      const int8_t* __restrict__ q8x, const float* __restrict__ q8s, float* __restrict__ y, int N,
                      int K, BlkPlan p, int* status) {
    constexpr bool Q4 = FMT == kQ4_0;
    extern __shared__ __align__(128) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* empty = full + p.nstage;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ncw = p.Tpad >> 5;
    const int stage_bytes = p.tile_bytes + p.stile_bytes;
    pdl_launch_dependents();

    if (tid == 0) {
        for (int i = 0; i < p.nstage; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], ncw); }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == ncw) {  // producer
        if (lane == 0) {
            int k = 0;
            for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
                const int st = k % p.nstage;
                if (k >= p.nstage && !mbar_wait(&empty[st], ((k / p.nstage) - 1) & 1, status, 41)) break;
                const int rows = min(p.RT, N - tile * p.RT);
                const uint32_t wb = (static_cast<uint32_t>(rows * p.row_bytes) + 15u) & ~15u;
                const uint32_t sbytes = p.srow_bytes ? ((static_cast<uint32_t>(rows * p.srow_bytes) + 15u) & ~15u) : 0u;
                mbar_arrive_expect_tx(&full[st], wb + sbytes);
                uint8_t* sb = smem + static_cast<size_t>(st) * stage_bytes;
                bulk_g2s(sb, W + static_cast<size_t>(tile) * p.RT * p.row_bytes, wb, &full[st]);
                if (sbytes)
                    bulk_g2s(sb + p.tile_bytes, reinterpret_cast<const uint8_t*>(wscale) +
                                                    static_cast<size_t>(tile) * p.RT * p.srow_bytes,
                             sbytes, &full[st]);
            }
            for (int j = max(0, k - p.nstage); j < k; ++j)
                if (!mbar_wait(&full[j % p.nstage], (j / p.nstage) & 1, status, 42)) break;
        }
        return;
    }

    // x / the Q8 activations and y belong to the kernels before this one until they finish (programmatic
    // dependent launch): the producer above streams the weights meanwhile
    pdl_wait();
    const bool active = tid < p.T;
    const int pr = active ? tid % p.P : 0;  // block pair index
    const int rl = active ? tid / p.P : 0;
    // x for the two blocks of the pair
    uint32_t pa[NPL][8], pb[NPL][8];
    float xsa = 0.f, xsb = 0.f;
    int xia = 0, xib = 0;
    int neg6[4][3];
    if constexpr (FMT == kQ6K) {
        prep_q6k(x + pr * 64, active, pa, pb, neg6, xsa);
    } else if constexpr (NPL == 3) {
        float v[32];
        const float4* xp = reinterpret_cast<const float4*>(x + pr * 64);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = active ? __ldg(xp + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        prep_planes_f32<NPL, Q4>(v, pa, xsa, xia);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = active ? __ldg(xp + 8 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        prep_planes_f32<NPL, Q4>(v, pb, xsb, xib);
    } else {
        int8_t q[32];
        const int4* qp = reinterpret_cast<const int4*>(q8x + pr * 64);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int4 v = active ? __ldg(qp + 2 * h + c) : make_int4(0, 0, 0, 0);
                const int vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) q[16 * c + i] = static_cast<int8_t>((vv[i >> 2] >> (8 * (i & 3))) & 0xFF);
            }
            if (h == 0) prep_planes_q8<Q4>(q, pa, xia);
            else prep_planes_q8<Q4>(q, pb, xib);
        }
        xsa = active ? q8s[2 * pr] : 0.f;
        xsb = active ? q8s[2 * pr + 1] : 0.f;
    }

    const int pair_off = FMT == kQ6K ? (pr >> 2) * 210 : pr * (Q4 ? 36 : (FMT == kQ8_0G ? 68 : 64));
    const int row_stride = p.m * p.row_bytes;
    int k = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
        const int st = k % p.nstage;
        const bool got = mbar_wait(&full[st], (k / p.nstage) & 1, status, 43);
        const uint8_t* sbase = smem + static_cast<size_t>(st) * stage_bytes;
        const uint8_t* base = sbase + rl * p.row_bytes + pair_off;
        float* redb = red + (k & 1) * p.RT * p.P + rl * p.P + pr;
        const int row0 = tile * p.RT;
        if (active && got) {
            float acc[RPT];
#pragma unroll
            for (int rr = 0; rr < RPT; ++rr) {
                const uint8_t* bp = base + rr * row_stride;
                if constexpr (FMT == kQ6K) {
                    acc[rr] = xsa * q6k_quarter_dot(bp, smem, pr & 3, pa, pb, neg6);
                } else {
                    float da, db;
                    uint32_t qa[8], qb[8];
                    if (FMT == kQ4_0) {
                        uint32_t w[9];
#pragma unroll
                        for (int i = 0; i < 9; ++i) w[i] = lds32(bp + 4 * i);
                        const uint32_t ha = w[0] & 0xFFFFu, hb = w[4] >> 16;
                        da = NPL == 3 ? f16_half_rs(ha) : f16_ieee(ha);
                        db = NPL == 3 ? f16_half_rs(hb) : f16_ieee(hb);
#pragma unroll
                        for (int i = 0; i < 4; ++i) { qa[i] = __funnelshift_r(w[i], w[i + 1], 16); qb[i] = w[5 + i]; }
                    } else if (FMT == kQ8_0G) {
                        uint32_t w[17];
#pragma unroll
                        for (int i = 0; i < 17; ++i) w[i] = lds32(bp + 4 * i);
                        da = f16_half_rs(w[0] & 0xFFFFu);
                        db = f16_half_rs(w[8] >> 16);
#pragma unroll
                        for (int i = 0; i < 8; ++i) { qa[i] = __funnelshift_r(w[i], w[i + 1], 16); qb[i] = w[9 + i]; }
                    } else {
                        const uint4 v0 = *reinterpret_cast<const uint4*>(bp), v1 = *reinterpret_cast<const uint4*>(bp + 16);
                        const uint4 v2 = *reinterpret_cast<const uint4*>(bp + 32), v3 = *reinterpret_cast<const uint4*>(bp + 48);
                        qa[0] = v0.x; qa[1] = v0.y; qa[2] = v0.z; qa[3] = v0.w; qa[4] = v1.x; qa[5] = v1.y; qa[6] = v1.z; qa[7] = v1.w;
                        qb[0] = v2.x; qb[1] = v2.y; qb[2] = v2.z; qb[3] = v2.w; qb[4] = v3.x; qb[5] = v3.y; qb[6] = v3.z; qb[7] = v3.w;
                        const float2 sc = *reinterpret_cast<const float2*>(sbase + p.tile_bytes +
                                                                             (rl + rr * p.m) * p.srow_bytes + pr * 8);
                        da = sc.x;
                        db = sc.y;
                    }
                    const float sa = block_dot<NPL, Q4>(qa, pa, xia);
                    const float sb = block_dot<NPL, Q4>(qb, pb, xib);
                    acc[rr] = fmaf(da * xsa, sa, (db * xsb) * sb);
                }
            }
#pragma unroll
            for (int rr = 0; rr < RPT; ++rr) redb[rr * p.m * p.P] = acc[rr];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (named_bar_red_or(1, p.Tpad, !got)) return;
        const float* redr = red + (k & 1) * p.RT * p.P;
        for (int rloc = warp; rloc < p.RT; rloc += ncw) {
            if (row0 + rloc >= N) break;
            const float* rp = redr + rloc * p.P;
            float sum = 0.f;
            for (int i = lane; i < p.P; i += 32) sum += rp[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) y[row0 + rloc] = sum;
        }
    }
}

static bool blk_make_plan(int fmt, int N, int K, int rpt, int num_sms, BlkPlan* out) {
    if (K % (fmt == kQ6K ? 256 : 64)) return false;
    BlkPlan p{};
    p.P = K / 64;
    const int maxc = kBlkThreads - 32;
    if (p.P > maxc) return false;
    p.row_bytes = fmt == kQ4_0 ? K / 32 * 18 : (fmt == kQ8_0G ? K / 32 * 34 : (fmt == kQ6K ? K / 256 * 210 : K));
    p.srow_bytes = fmt == kQ8C ? K / 32 * 4 : 0;
    p.m = maxc / p.P;
    // tiles must start 16-byte aligned: RT * row_bytes (and RT * srow_bytes) multiples of 16
    auto aligned = [&](int rt) {
        return (static_cast<long long>(rt) * p.row_bytes) % 16 == 0 &&
               (static_cast<long long>(rt) * p.srow_bytes) % 16 == 0;
    };
    while (p.m > 1 && !aligned(p.m * rpt)) --p.m;
    if (!aligned(p.m * rpt)) return false;
    p.T = p.m * p.P;
    p.Tpad = (p.T + 31) & ~31;
    p.RT = p.m * rpt;
    p.tile_bytes = (p.RT * p.row_bytes + 15) & ~15;
    p.stile_bytes = (p.RT * p.srow_bytes + 15) & ~15;
    const int redb = 2 * p.RT * p.P * 4;
    p.nstage = 4;
    while (p.nstage >= 2 && p.nstage * (p.tile_bytes + p.stile_bytes) + redb + 64 > kSmemLimit) --p.nstage;
    if (p.nstage < 2) return false;
    p.ntiles = (N + p.RT - 1) / p.RT;
    p.grid = p.ntiles < num_sms ? p.ntiles : num_sms;
    p.red_off = p.nstage * (p.tile_bytes + p.stile_bytes);
    p.bar_off = (p.red_off + redb + 15) & ~15;
    p.smem = p.bar_off + 2 * p.nstage * 8;
    *out = p;
    return true;
}

template <int FMT, int NPL, int RPT>
static cudaError_t launch_blk(const uint8_t* W, const float* wscale, const float* x, const int8_t* q8x,
                              const float* q8s, float* y, int N, int K, const BlkPlan& p, int* status,
                              cudaStream_t stream) {
    static DeviceFlags attr_done;
    const cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(blk_matvec_kernel<FMT, NPL, RPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    const cudaError_t le = launch_pdl(blk_matvec_kernel<FMT, NPL, RPT>, dim3(p.grid), dim3(p.Tpad + 32),
                                      static_cast<size_t>(p.smem), stream, W, wscale, x, q8x, q8s, y, N, K, p,
                                      status);
    note_launch();
    return le != cudaSuccess ? le : cudaGetLastError();
}

// One row-pass of a block format.  fmt: 0 Q4_0, 1 Q8_0 (GGUF 34 B), 2 Q8 compute layout, 3 Q6_K (f32 x only).
// x32 != nullptr: f32 activations (digit planes); else q8x/q8s: Q8 activations (int8 + f32 scale per 32).
// Returns cudaErrorInvalidValue when the shape is not supported (K % 64 != 0, Q6_K K % 256 != 0, or too large).
cudaError_t launch_block_matvec(int fmt, const uint8_t* W, const float* wscale, const float* x32, const int8_t* q8x,
                                const float* q8s, float* y, int N, int K, int num_sms, int* status,
                                cudaStream_t stream) {
    if (N <= 0) return cudaSuccess;
    const int rpts[] = {4, 2};
    for (int rpt : rpts) {
        BlkPlan p;
        if (!blk_make_plan(fmt, N, K, rpt, num_sms, &p)) continue;
        if (p.nstage < 3 && rpt > 2) continue;
        const bool f32 = x32 != nullptr;
#define LB(F, NP, R) launch_blk<F, NP, R>(W, wscale, x32, q8x, q8s, y, N, K, p, status, stream)
        if (fmt == kQ4_0) return f32 ? (rpt == 4 ? LB(kQ4_0, 3, 4) : LB(kQ4_0, 3, 2)) : (rpt == 4 ? LB(kQ4_0, 1, 4) : LB(kQ4_0, 1, 2));
        if (fmt == kQ8_0G) return f32 ? (rpt == 4 ? LB(kQ8_0G, 3, 4) : LB(kQ8_0G, 3, 2)) : cudaErrorInvalidValue;
        if (fmt == kQ8C) return f32 ? cudaErrorInvalidValue : (rpt == 4 ? LB(kQ8C, 1, 4) : LB(kQ8C, 1, 2));
        if (fmt == kQ6K) return f32 ? (rpt == 4 ? LB(kQ6K, 3, 4) : LB(kQ6K, 3, 2)) : cudaErrorInvalidValue;
#undef LB
        return cudaErrorInvalidValue;
    }
    return cudaErrorInvalidValue;
}

// ── device quantizer of activations: quantize_to_q8 (q4_common.rs:28-44), bit-identical ──
// One warp per 32-value block: amax, scale = amax / 127, q = clamp(round(x / scale)) with Rust semantics.
__global__ void quantize_to_q8_kernel(const float* __restrict__ x, size_t nblocks, int8_t* __restrict__ q,
                                      float* __restrict__ s) {
    pdl_launch_dependents();
    pdl_wait();  // x, q and s belong to the kernels before this one until they finish
    const size_t b = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= nblocks) return;
    const float v = x[b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = __fdiv_rn(amax, 127.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    float r = roundf(__fmul_rn(v, inv));
    if (r < -128.0f) r = -128.0f;
    if (r > 127.0f) r = 127.0f;
    int qi = 0;
    if (r == r) qi = static_cast<int>(r);  // NaN -> 0 (Rust `as i8`)
    q[b * 32 + lane] = static_cast<int8_t>(qi);
    if (lane == 0) s[b] = scale;
}

// x'[i] = q[i] * s[i / 32]: Q8 activations back to f32 (the product rounded once; |q| <= 127) so the f32-x
// tensor-core matvec can take them.
__global__ void dequant_q8_kernel(const int8_t* __restrict__ q, const float* __restrict__ s, size_t n,
                                  float* __restrict__ out) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(static_cast<float>(q[i]), s[i / 32]);
}

cudaError_t launch_dequant_q8(const int8_t* q, const float* s, size_t n, float* out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    dequant_q8_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(q, s, n, out);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize_to_q8(const float* x, size_t n, int8_t* q, float* s, cudaStream_t stream) {
    const size_t nb = n / 32;
    if (nb == 0) return cudaSuccess;
    const cudaError_t e = launch_pdl(quantize_to_q8_kernel, dim3(static_cast<unsigned>((nb + 7) / 8)), dim3(256), 0,
                                     stream, x, nb, q, s);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace larql
