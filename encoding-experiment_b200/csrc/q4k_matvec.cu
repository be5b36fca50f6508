// q4k_matvec.cu — Q4_K (LARQL 148-byte super-block) dequant-matvec for sm_100a.
//
// Computes y[b, r] = sum_k W[r, k] * x[b, k] where W is stored as LARQL Q4_K
// (crates/larql-compute/src/cpu/ops/q4_common.rs:96-170): per 256 values
//   [0..2) f16 d, [2..4) f16 dmin, [4..12) 6-bit scales sc_j, [16..20) 4-bit
//   mins mn_j, [20..148) nibbles q (byte i of sub-block j = elems 2i, 2i+1),
// and W[r, k] = d*sc_j*q - dmin*mn_j (crates/larql-compute/src/cpu/ops/q4k_matvec.rs:70-81).
//
// Design (HBM-bound; one pass over the packed bytes as stored):
//  * Rows are contiguous, so a tile of RT consecutive rows is one contiguous
//    byte range.  A producer warp streams tiles into a ring of shared-memory
//    stages with 1-D bulk copies (cp.async.bulk) completing on mbarriers; the
//    CTA is persistent (one per SM), so copies for the next tiles are in
//    flight while the current one is consumed.  RT is a multiple of 4, which
//    makes every tile start 16-byte aligned (4 * 148 = 592 = 37 * 16).
//  * Consumer thread t owns one 32-value sub-block position s = t % S of the
//    row (S = 8 * K/256 sub-blocks per row) for the whole kernel, and rows
//    t / S + m*i of every tile.  Its slice of x therefore never changes: it is
//    converted once, in the prologue, into three int8 digit planes
//    (x = 2^e * (a*65536 + b*256 + c), e per 256-block so |x*2^-e| <= 2^22,
//    i.e. 22-23 significant bits — f32 precision at the block maximum) and
//    kept in 24 registers.
//  * Per (row, sub-block): 4 nibble words -> 8 byte-lanes of q (two LOP3 +
//    one shift per word) and 6 dp4a per word give exact int32 sums
//    sum q*a, sum q*b, sum q*c; they combine exactly in int32
//    (|.| < 2.07e9), convert once, and fold in d*sc_j*2^e.  The mins term
//    is -dmin*mn_j * sum(x over the sub-block), with the sum precomputed.
//    ~1.9 issued instructions per nibble, under the ~3.2/nibble the SMs can
//    issue while HBM delivers one 148-byte block per 256 nibbles.
//  * Partial sums of a row (one per sub-block position) are reduced through
//    shared memory once per tile and written as y.
#include "common.cuh"
#include "kernels.h"

namespace larql {

struct Q4kPlan {
    int nsb;         // super-blocks per row (K / 256)
    int S;           // sub-blocks per row
    int m;           // rows processed concurrently (row lanes)
    int T;           // active consumer threads = m * S
    int Tpad;        // consumer threads rounded to a warp multiple
    int RPT;         // rows per thread per tile
    int RT;          // rows per tile = m * RPT (multiple of 4)
    int row_bytes;   // nsb * 148
    int tile_bytes;  // RT * row_bytes (multiple of 16)
    int nstage;      // shared-memory ring depth
    int ntiles;
    int grid;
    int red_off;     // byte offset of the reduction buffer
    int bar_off;     // byte offset of the mbarriers
    int smem;        // dynamic shared memory bytes
    int batch;       // batch handled by one launch (1 or 2)
};

constexpr int kQ4kMaxThreads = 576;  // consumers + producer warp


template <int B>
__global__ void __launch_bounds__(kQ4kMaxThreads, 1)
    q4k_matvec_kernel(const uint8_t* __restrict__ W, const float* __restrict__ x, float* __restrict__ y,
                      int N, int K, Q4kPlan p, int* status) {
    extern __shared__ __align__(128) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* empty = full + p.nstage;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int ncw = p.Tpad >> 5;  // consumer warps

    if (tid == 0) {
        for (int i = 0; i < p.nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], ncw);
        }
        fence_barrier_init();
    }
    __syncthreads();

    // ───────────── producer warp ─────────────
    if (warp == ncw) {
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
                const int st = k % p.nstage;
                if (k >= p.nstage) {
                    if (!mbar_wait(&empty[st], ((k / p.nstage) - 1) & 1, status, 1)) { ok = false; break; }
                }
                const int rows = min(p.RT, N - tile * p.RT);
                const uint32_t bytes = (static_cast<uint32_t>(rows * p.row_bytes) + 15u) & ~15u;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(smem + static_cast<size_t>(st) * p.tile_bytes,
                         W + static_cast<size_t>(tile) * p.RT * p.row_bytes, bytes, &full[st]);
            }
            // Do not leave copies in flight: wait (bounded) for the last fills.
            const int issued = k;
            for (int j = max(0, issued - p.nstage); j < issued; ++j)
                if (!mbar_wait(&full[j % p.nstage], (j / p.nstage) & 1, status, 2)) break;
            (void)ok;
        }
        return;
    }

    // ───────────── consumers ─────────────
    const bool active = tid < p.T;
    const int s = active ? tid % p.S : 0;
    const int rl = active ? tid / p.S : 0;
    const int sb = s >> 3, jj = s & 7;
    const int sc_sh = 8 * (jj & 3);
    const int mn_sh = 8 * (jj & 3) + 4 * (jj >> 2);
    const int sc_off = 4 + (jj & 4);

    // x slice -> digit planes (registers for the whole kernel).
    uint32_t xe[B][3][4], xo[B][3][4];
    float xsum[B], xscale[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float v[32];
        const float4* xp = reinterpret_cast<const float4*>(x + static_cast<size_t>(b) * K + sb * 256 + jj * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 f = active ? __ldg(xp + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        float amax = 0.f, sum = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) { amax = fmaxf(amax, fabsf(v[i])); sum += v[i]; }
        // the 8 sub-blocks of a super-block are 8 aligned consecutive lanes
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        int ex = 0;
        frexpf(amax, &ex);
        int e = ex - 22;
        e = max(-126, min(127, e));
        const float down = ldexpf(1.0f, -e);
        xscale[b] = isfinite(amax) ? ldexpf(1.0f, e) : __int_as_float(0x7fc00000);
        xsum[b] = sum;
        int q[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) q[i] = isfinite(amax) ? __float2int_rn(v[i] * down) : 0;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            uint32_t pa[2] = {0, 0}, pb[2] = {0, 0}, pc[2] = {0, 0};
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
                const int xi = q[8 * w + k2];
                const int c = (xi << 24) >> 24;
                const int r1 = (xi - c) >> 8;
                const int bb = (r1 << 24) >> 24;
                const int a = (r1 - bb) >> 8;
                const int par = k2 & 1, pos = 8 * (k2 >> 1);
                pa[par] |= (static_cast<uint32_t>(a) & 0xFFu) << pos;
                pb[par] |= (static_cast<uint32_t>(bb) & 0xFFu) << pos;
                pc[par] |= (static_cast<uint32_t>(c) & 0xFFu) << pos;
            }
            xe[b][0][w] = pa[0]; xo[b][0][w] = pa[1];
            xe[b][1][w] = pb[0]; xo[b][1][w] = pb[1];
            xe[b][2][w] = pc[0]; xo[b][2][w] = pc[1];
        }
    }

    const int red_stride = p.RT * p.S;  // floats per (buffer, batch)
    int k = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
        const int st = k % p.nstage;
        const int buf = k & 1;
        const bool got = mbar_wait(&full[st], (k / p.nstage) & 1, status, 3);
        const uint8_t* stage = smem + static_cast<size_t>(st) * p.tile_bytes;
        const int row0 = tile * p.RT;

        if (active && got) {
#pragma unroll 1
            for (int rr = 0; rr < p.RPT; ++rr) {
                const int rloc = rl + rr * p.m;
                float acc[B];
#pragma unroll
                for (int b = 0; b < B; ++b) acc[b] = 0.f;
                if (row0 + rloc < N) {
                    const uint8_t* bp = stage + rloc * p.row_bytes + sb * 148;
                    const uint32_t h = lds32(bp);
                    const float d = h2f_lo(h), dmin = h2f_hi(h);
                    const float scf = u2f_small((lds32(bp + sc_off) >> sc_sh) & 0x3Fu);
                    const float mnf = u2f_small((lds32(bp + 16) >> mn_sh) & 0xFu);
                    const uint8_t* qp = bp + 20 + 16 * jj;
                    uint32_t wq[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) wq[i] = lds32(qp + 4 * i);
                    const float dsc = d * scf, dmn = dmin * mnf;
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        int ia = 0, ib = 0, ic = 0;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int L = static_cast<int>(wq[i] & 0x0F0F0F0Fu);
                            const int H = static_cast<int>((wq[i] >> 4) & 0x0F0F0F0Fu);
                            ia = __dp4a(L, static_cast<int>(xe[b][0][i]), ia);
                            ia = __dp4a(H, static_cast<int>(xo[b][0][i]), ia);
                            ib = __dp4a(L, static_cast<int>(xe[b][1][i]), ib);
                            ib = __dp4a(H, static_cast<int>(xo[b][1][i]), ib);
                            ic = __dp4a(L, static_cast<int>(xe[b][2][i]), ic);
                            ic = __dp4a(H, static_cast<int>(xo[b][2][i]), ic);
                        }
                        const int isum = (ia * 256 + ib) * 256 + ic;
                        acc[b] = fmaf(dsc * xscale[b], static_cast<float>(isum), -dmn * xsum[b]);
                    }
                }
#pragma unroll
                for (int b = 0; b < B; ++b) red[(buf * B + b) * red_stride + rloc * p.S + s] = acc[b];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        // all consumers leave together if any wait ran out of budget
        if (named_bar_red_or(1, p.Tpad, !got)) return;

        // reduce: one warp per row (round-robin), lanes stride the S partials
        for (int rloc = warp; rloc < p.RT; rloc += ncw) {
            if (row0 + rloc >= N) break;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float* rp = red + (buf * B + b) * red_stride + rloc * p.S;
                float sum = 0.f;
                for (int i = lane; i < p.S; i += 32) sum += rp[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                if (lane == 0) y[static_cast<size_t>(b) * N + row0 + rloc] = sum;
            }
        }
    }
}

// ─────────────────────────────────────────────────────────────────────────
// v2: each consumer thread owns a PAIR of adjacent sub-blocks (j0 = 2*jp,
// j0 + 1) of one super-block, so the block header (d, dmin, the scale and min
// words) is read and decoded once per two 32-value items; RPT rows per tile
// are unrolled for instruction-level parallelism.  NSL is the number of int8
// digit planes of x (3: 22-23 significant bits per 32-value group, f32 grade;
// 2: 15 bits).
// ─────────────────────────────────────────────────────────────────────────
struct Q4kPlan2 {
    int nsb, S2, m, T, Tpad, RT, row_bytes, tile_bytes, nstage, ntiles, grid, red_off, bar_off, smem;
};

// GG = false: the LARQL layout's nibble order (byte i of a sub-block holds elements 2i, 2i+1): xe = even
// elements, xo = odd.  GG = true: the GGUF-144 order of ggml.rs dequantize_q4_k (byte i holds elements i and
// 16 + i): xe[w] = elements 4w..4w+3, xo[w] = elements 16+4w..16+4w+3.
template <int NSL, bool GG = false>
__device__ __forceinline__ void x_digit_planes(const float* v, uint32_t (&xe)[NSL][4], uint32_t (&xo)[NSL][4],
                                               float& xscale, float& xsum) {
    float amax = 0.f, sum = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { amax = fmaxf(amax, fabsf(v[i])); sum += v[i]; }
    int ex = 0;
    frexpf(amax, &ex);
    // |x * 2^-e| <= 2^22 (3 planes) or 2^14 (2 planes)
    int e = ex - (NSL == 3 ? 22 : 14);
    e = max(-126, min(127, e));
    const float down = ldexpf(1.0f, -e);
    const bool fin = isfinite(amax);
    xscale = fin ? ldexpf(1.0f, e) : __int_as_float(0x7fc00000);
    xsum = sum;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t pl[NSL][2];
#pragma unroll
        for (int z = 0; z < NSL; ++z) pl[z][0] = pl[z][1] = 0u;
#pragma unroll
        for (int k2 = 0; k2 < 8; ++k2) {
            const int el = GG ? (k2 < 4 ? 4 * w + k2 : 16 + 4 * w + (k2 - 4)) : 8 * w + k2;
            int xi = fin ? __float2int_rn(v[el] * down) : 0;
            const int par = GG ? (k2 >> 2) : (k2 & 1), pos = GG ? 8 * (k2 & 3) : 8 * (k2 >> 1);
            // balanced base-256 digits, least significant first
#pragma unroll
            for (int z = NSL - 1; z >= 1; --z) {
                const int dgt = (xi << 24) >> 24;
                pl[z][par] |= (static_cast<uint32_t>(dgt) & 0xFFu) << pos;
                xi = (xi - dgt) >> 8;
            }
            pl[0][par] |= (static_cast<uint32_t>(xi) & 0xFFu) << pos;
        }
#pragma unroll
        for (int z = 0; z < NSL; ++z) { xe[z][w] = pl[z][0]; xo[z][w] = pl[z][1]; }
    }
}

template <int NSL>
__device__ __forceinline__ int q4_dot_planes(const uint32_t* wq, const uint32_t (&xe)[NSL][4],
                                             const uint32_t (&xo)[NSL][4]) {
    int acc[NSL];
#pragma unroll
    for (int z = 0; z < NSL; ++z) acc[z] = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int L = static_cast<int>(wq[i] & 0x0F0F0F0Fu);
        const int H = static_cast<int>((wq[i] >> 4) & 0x0F0F0F0Fu);
#pragma unroll
        for (int z = 0; z < NSL; ++z) {
            acc[z] = __dp4a(L, static_cast<int>(xe[z][i]), acc[z]);
            acc[z] = __dp4a(H, static_cast<int>(xo[z][i]), acc[z]);
        }
    }
    int isum = acc[0];
#pragma unroll
    for (int z = 1; z < NSL; ++z) isum = isum * 256 + acc[z];
    return isum;
}

constexpr int kQ4kPairThreads = 512;  // 15 consumer warps + 1 producer warp (128 registers/thread)

// f16 decode of crates/larql-models/src/quant/half.rs:4-20 (subnormals at half value), which ggml.rs's
// dequantize_q4_k uses for d and dmin.
__device__ __forceinline__ float f16_halfrs_q4k(uint32_t h16) {
    const float v = __half2float(__ushort_as_half(static_cast<unsigned short>(h16)));
    return (h16 & 0x7C00u) == 0u ? v * 0.5f : v;
}

// GG = true: GGUF-144 super-blocks as crates/larql-models/src/quant/ggml.rs:228-273 (dequantize_q4_k) reads
// them: [0..2) f16 d, [2..4) f16 dmin, [4..16) 6-bit scales and mins packed as llama.cpp get_scale_min_k4,
// [16..144) nibbles, sub-block j at 16 j (its 16 low nibbles first, then the 16 high); d / dmin decoded as
// half.rs.
template <int NSL, int RPT, bool GG = false>
__global__ void __launch_bounds__(kQ4kPairThreads, 1)
    q4k_matvec_pair_kernel(const uint8_t* __restrict__ W, const float* __restrict__ x, float* __restrict__ y,
                           int N, Q4kPlan2 p, int* status) {
    constexpr int SBB = GG ? 144 : 148;
    extern __shared__ __align__(128) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem + p.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
    uint64_t* empty = full + p.nstage;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int ncw = p.Tpad >> 5;

    if (tid == 0) {
        for (int i = 0; i < p.nstage; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], ncw);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == ncw) {  // producer warp
        if (lane == 0) {
            int k = 0;
            for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
                const int st = k % p.nstage;
                if (k >= p.nstage && !mbar_wait(&empty[st], ((k / p.nstage) - 1) & 1, status, 11)) break;
                const int rows = min(p.RT, N - tile * p.RT);
                const uint32_t bytes = (static_cast<uint32_t>(rows * p.row_bytes) + 15u) & ~15u;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(smem + static_cast<size_t>(st) * p.tile_bytes,
                         W + static_cast<size_t>(tile) * p.RT * p.row_bytes, bytes, &full[st]);
            }
            for (int j = max(0, k - p.nstage); j < k; ++j)
                if (!mbar_wait(&full[j % p.nstage], (j / p.nstage) & 1, status, 12)) break;
        }
        return;
    }

    const bool active = tid < p.T;
    const int s2 = active ? tid % p.S2 : 0;
    const int rl = active ? tid / p.S2 : 0;
    const int sb = s2 >> 2, j0 = 2 * (s2 & 3);
    const int sc_off = 4 + (j0 & 4);
    const int sc_sh = 8 * (j0 & 3);
    const int mn_sh = 8 * (j0 & 3) + 4 * (j0 >> 2);
    const int hdr_off = sb * SBB;
    const int q_off = hdr_off + (GG ? 16 : 20) + 16 * j0;
    const int jb = j0 & 3;  // GGUF-144: byte of the pair's first sub-block within its scale word

    uint32_t xe0[NSL][4], xo0[NSL][4], xe1[NSL][4], xo1[NSL][4];
    float xs0, xs1, xm0, xm1;
    {
        float v[32];
        const float4* xp = reinterpret_cast<const float4*>(x + sb * 256 + j0 * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = active ? __ldg(xp + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        x_digit_planes<NSL, GG>(v, xe0, xo0, xs0, xm0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = active ? __ldg(xp + 8 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        x_digit_planes<NSL, GG>(v, xe1, xo1, xs1, xm1);
    }

    const int row_stride = p.m * p.row_bytes;  // bytes between a thread's consecutive rows
    int k = 0;
    for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++k) {
        const int st = k % p.nstage;
        const bool got = mbar_wait(&full[st], (k / p.nstage) & 1, status, 13);
        const uint8_t* base = smem + static_cast<size_t>(st) * p.tile_bytes + rl * p.row_bytes;
        float* redb = red + (k & 1) * p.RT * p.S2 + rl * p.S2 + s2;
        if (active && got) {
            float acc[RPT];
#pragma unroll
            for (int rr = 0; rr < RPT; ++rr) {
                const uint8_t* bp = base + rr * row_stride;
                const uint32_t h = lds32(bp + hdr_off);
                uint32_t wq[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) wq[i] = lds32(bp + q_off + 4 * i);
                float d, dmin;
                uint32_t sc0, sc1, mn0, mn1;
                if constexpr (GG) {
                    // get_scale_min_k4 over s = bytes 4..15 (words W0 = s[0..3], W1 = s[4..7], W2 = s[8..11]):
                    // j < 4: sc = s[j] & 63, mn = s[j + 4] & 63; j >= 4: sc = (s[j + 4] & 15) | (s[j - 4] >> 6) << 4,
                    // mn = (s[j + 4] >> 4) | (s[j] >> 6) << 4
                    const uint32_t w0 = lds32(bp + hdr_off + 4), w1 = lds32(bp + hdr_off + 8);
                    const uint32_t w2 = lds32(bp + hdr_off + 12);
                    const uint32_t b0a = (w0 >> (8 * jb)) & 0xFFu, b0b = (w0 >> (8 * jb + 8)) & 0xFFu;
                    const uint32_t b1a = (w1 >> (8 * jb)) & 0xFFu, b1b = (w1 >> (8 * jb + 8)) & 0xFFu;
                    if (j0 < 4) {
                        sc0 = b0a & 0x3Fu; sc1 = b0b & 0x3Fu;
                        mn0 = b1a & 0x3Fu; mn1 = b1b & 0x3Fu;
                    } else {
                        const uint32_t b2a = (w2 >> (8 * jb)) & 0xFFu, b2b = (w2 >> (8 * jb + 8)) & 0xFFu;
                        sc0 = (b2a & 0xFu) | ((b0a >> 6) << 4); sc1 = (b2b & 0xFu) | ((b0b >> 6) << 4);
                        mn0 = (b2a >> 4) | ((b1a >> 6) << 4);   mn1 = (b2b >> 4) | ((b1b >> 6) << 4);
                    }
                    d = f16_halfrs_q4k(h & 0xFFFFu);
                    dmin = f16_halfrs_q4k(h >> 16);
                } else {
                    const uint32_t scw = lds32(bp + hdr_off + sc_off);
                    const uint32_t mnw = lds32(bp + hdr_off + 16);
                    sc0 = (scw >> sc_sh) & 0x3Fu; sc1 = (scw >> (sc_sh + 8)) & 0x3Fu;
                    mn0 = (mnw >> mn_sh) & 0xFu;  mn1 = (mnw >> (mn_sh + 8)) & 0xFu;
                    d = h2f_lo(h);
                    dmin = h2f_hi(h);
                }
                const float c0 = d * u2f_small(sc0) * xs0;
                const float c1 = d * u2f_small(sc1) * xs1;
                const float m0 = dmin * u2f_small(mn0) * xm0;
                const float m1 = dmin * u2f_small(mn1) * xm1;
                const int i0 = q4_dot_planes<NSL>(wq, xe0, xo0);
                const int i1 = q4_dot_planes<NSL>(wq + 4, xe1, xo1);
                acc[rr] = fmaf(c0, static_cast<float>(i0), fmaf(c1, static_cast<float>(i1), -(m0 + m1)));
            }
#pragma unroll
            for (int rr = 0; rr < RPT; ++rr) redb[rr * p.m * p.S2] = acc[rr];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (named_bar_red_or(1, p.Tpad, !got)) return;

        const int row0 = tile * p.RT;
        const float* redr = red + (k & 1) * p.RT * p.S2;
        for (int rloc = warp; rloc < p.RT; rloc += ncw) {
            if (row0 + rloc >= N) break;
            const float* rp = redr + rloc * p.S2;
            float sum = 0.f;
            for (int i = lane; i < p.S2; i += 32) sum += rp[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) y[row0 + rloc] = sum;
        }
    }
}

// Plan for the pair kernel: RT = m * RPT rows per tile (multiple of 4).
static bool q4k_make_plan2(int N, int K, int rpt, int num_sms, Q4kPlan2* out, int sbb = 148) {
    Q4kPlan2 p{};
    p.nsb = K / 256;
    p.S2 = 4 * p.nsb;
    const int maxc = kQ4kPairThreads - 32;
    if (p.S2 > maxc) return false;
    p.m = maxc / p.S2;
    // RT = m * rpt must be a multiple of 4 (16-byte aligned tiles)
    while (p.m > 1 && (p.m * rpt) % 4) --p.m;
    p.T = p.m * p.S2;
    p.Tpad = (p.T + 31) & ~31;
    p.RT = p.m * rpt;
    if (p.RT % 4) return false;
    p.row_bytes = p.nsb * sbb;
    p.tile_bytes = p.RT * p.row_bytes;
    const int redb = 2 * p.RT * p.S2 * 4;
    p.nstage = 4;
    while (p.nstage >= 2 && p.nstage * p.tile_bytes + redb + 64 > kSmemLimit) --p.nstage;
    if (p.nstage < 2) return false;
    p.ntiles = (N + p.RT - 1) / p.RT;
    p.grid = p.ntiles < num_sms ? p.ntiles : num_sms;
    p.red_off = p.nstage * p.tile_bytes;
    p.bar_off = (p.red_off + redb + 15) & ~15;
    p.smem = p.bar_off + 2 * p.nstage * 8;
    *out = p;
    return true;
}

template <int NSL, int RPT, bool GG = false>
static cudaError_t launch_pair(const uint8_t* W, const float* x, float* y, int N, const Q4kPlan2& p, int* status,
                               cudaStream_t stream) {
    static DeviceFlags attr_done;
    const cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(q4k_matvec_pair_kernel<NSL, RPT, GG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    q4k_matvec_pair_kernel<NSL, RPT, GG><<<p.grid, p.Tpad + 32, p.smem, stream>>>(W, x, y, N, p, status);
    note_launch();
    return cudaGetLastError();
}

// Chooses rows-per-thread: the plan with the most consumer threads and at
// least 3 pipeline stages (ties: the smaller tile).
static bool launch_pair_b1(const uint8_t* W, const float* x, float* y, int N, int K, int nsl, int num_sms,
                           int* status, cudaStream_t stream, cudaError_t* err) {
    Q4kPlan2 best{};
    int best_rpt = 0;
    const int rpts[] = {4, 2};
    for (int rpt : rpts) {
        Q4kPlan2 p;
        if (!q4k_make_plan2(N, K, rpt, num_sms, &p) || p.nstage < 3) continue;
        if (!best_rpt || p.T > best.T || (p.T == best.T && p.tile_bytes < best.tile_bytes)) {
            best = p;
            best_rpt = rpt;
        }
    }
    if (!best_rpt) return false;
    if (nsl == 3) *err = best_rpt == 4 ? launch_pair<3, 4>(W, x, y, N, best, status, stream)
                                       : launch_pair<3, 2>(W, x, y, N, best, status, stream);
    else *err = best_rpt == 4 ? launch_pair<2, 4>(W, x, y, N, best, status, stream)
                              : launch_pair<2, 2>(W, x, y, N, best, status, stream);
    return true;
}

int g_q4k_planes = 3;  // digit planes of x used by the batch-1 kernel (2 or 3)

// GGUF-144 Q4_K (ggml.rs:228-273 dequantize_q4_k + f32 dot) on the pair kernel, one weight pass per batch row,
// x as three digit planes.  cudaErrorInvalidValue when K % 256 != 0 or K / 256 > 120 (no plan).
cudaError_t launch_q4k_gguf_matvec(const uint8_t* W, int N, int K, const float* x, int batch, float* y,
                                   int num_sms, int* status, cudaStream_t stream) {
    if (N <= 0 || batch <= 0) return cudaSuccess;
    if (K % 256) return cudaErrorInvalidValue;
    Q4kPlan2 best{};
    int best_rpt = 0;
    const int rpts[] = {4, 2};
    for (int rpt : rpts) {
        Q4kPlan2 p;
        if (!q4k_make_plan2(N, K, rpt, num_sms, &p, 144) || p.nstage < 3) continue;
        if (!best_rpt || p.T > best.T || (p.T == best.T && p.tile_bytes < best.tile_bytes)) {
            best = p;
            best_rpt = rpt;
        }
    }
    if (!best_rpt) return cudaErrorInvalidValue;
    for (int b = 0; b < batch; ++b) {
        const float* xb = x + static_cast<size_t>(b) * K;
        float* yb = y + static_cast<size_t>(b) * N;
        const cudaError_t e = best_rpt == 4 ? launch_pair<3, 4, true>(W, xb, yb, N, best, status, stream)
                                            : launch_pair<3, 2, true>(W, xb, yb, N, best, status, stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Fallback for shapes the tiled kernel does not take (K/256 > 68): one warp
// per row, plain loads, f32 dequant and FMA.  Same math, no staging.
__global__ void q4k_matvec_simple(const uint8_t* __restrict__ W, const float* __restrict__ x,
                                  float* __restrict__ y, int N, int K, int B) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    const int nsb = K / 256;
    const uint8_t* rp = W + static_cast<size_t>(row) * nsb * 148;
    for (int b = 0; b < B; ++b) {
        const float* xb = x + static_cast<size_t>(b) * K;
        float acc = 0.f;
        for (int s = lane; s < nsb * 8; s += 32) {
            const uint8_t* bp = rp + (s >> 3) * 148;
            const int j = s & 7;
            const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(bp[0] | (bp[1] << 8))));
            const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(bp[2] | (bp[3] << 8))));
            const float sc = d * static_cast<float>(bp[4 + j] & 0x3F);
            const float mn = dmin * static_cast<float>(j < 4 ? (bp[16 + j] & 0xF) : (bp[12 + j] >> 4));
            const uint8_t* qp = bp + 20 + 16 * j;
            const float* xp = xb + (s >> 3) * 256 + j * 32;
            for (int i = 0; i < 16; ++i) {
                acc = fmaf(sc * static_cast<float>(qp[i] & 0xF) - mn, xp[2 * i], acc);
                acc = fmaf(sc * static_cast<float>(qp[i] >> 4) - mn, xp[2 * i + 1], acc);
            }
        }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) y[static_cast<size_t>(b) * N + row] = acc;
    }
}

// Picks tile / stage sizes for the tiled kernel.  Returns false when the
// shape needs the fallback.
bool q4k_make_plan(int N, int K, int batch, int num_sms, Q4kPlan* out) {
    Q4kPlan p{};
    p.nsb = K / 256;
    p.S = 8 * p.nsb;
    if (p.S + 32 > kQ4kMaxThreads || p.S < 8) return false;
    p.m = p.S >= 512 ? 1 : 512 / p.S;
    p.T = p.m * p.S;
    p.Tpad = (p.T + 31) & ~31;
    if (p.Tpad + 32 > kQ4kMaxThreads) {
        p.m = (kQ4kMaxThreads - 32 - 31) / p.S;
        if (p.m < 1) return false;
        p.T = p.m * p.S;
        p.Tpad = (p.T + 31) & ~31;
    }
    p.row_bytes = p.nsb * 148;
    p.batch = batch;
    const int bars = 2 * 4 * 8;
    int best_rpt = -1, best_stage = 0;
    for (int rpt = 8; rpt >= 1; --rpt) {
        const int rt = p.m * rpt;
        if (rt % 4) continue;
        const int tile = rt * p.row_bytes;
        const int redb = 2 * batch * rt * p.S * 4;
        int ns = 4;
        while (ns >= 2 && ns * tile + redb + bars > kSmemLimit) --ns;
        if (ns < 2) continue;
        if (tile > 49152 && rpt > 1 && (p.m * (rpt - 1)) % 4 == 0) continue;  // prefer ~48 KB stages
        best_rpt = rpt;
        best_stage = ns;
        break;
    }
    if (best_rpt < 0) {
        for (int rpt = 1; rpt <= 8; ++rpt) {
            const int rt = p.m * rpt;
            if (rt % 4) continue;
            const int tile = rt * p.row_bytes;
            const int redb = 2 * batch * rt * p.S * 4;
            if (2 * tile + redb + bars <= kSmemLimit) { best_rpt = rpt; best_stage = 2; break; }
        }
    }
    if (best_rpt < 0) return false;
    p.RPT = best_rpt;
    p.RT = p.m * p.RPT;
    p.tile_bytes = p.RT * p.row_bytes;
    p.nstage = best_stage;
    p.ntiles = (N + p.RT - 1) / p.RT;
    p.grid = p.ntiles < num_sms ? p.ntiles : num_sms;
    p.red_off = p.nstage * p.tile_bytes;
    p.bar_off = p.red_off + 2 * batch * p.RT * p.S * 4;
    p.bar_off = (p.bar_off + 15) & ~15;
    p.smem = p.bar_off + 2 * p.nstage * 8;
    *out = p;
    return true;
}

template <int B>
static cudaError_t launch_tiled(const uint8_t* W, const float* x, float* y, int N, int K, const Q4kPlan& p,
                                int* status, cudaStream_t stream) {
    static DeviceFlags attr_done;
    const cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(q4k_matvec_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    q4k_matvec_kernel<B><<<p.grid, p.Tpad + 32, p.smem, stream>>>(W, x, y, N, K, p, status);
    note_launch();
    return cudaGetLastError();
}

// y[batch, N] = Q4_K W[N, K] . x[batch, K].  W must be 16-byte aligned and
// readable for 15 bytes past its end (registry buffers are padded); x must be
// 16-byte aligned.
cudaError_t launch_q4k_matvec(const uint8_t* W, int N, int K, const float* x, int batch, float* y,
                              int num_sms, int* status, cudaStream_t stream) {
    if (N <= 0 || batch <= 0) return cudaSuccess;
    if (batch == 1) {
        cudaError_t e = cudaSuccess;
        if (launch_pair_b1(W, x, y, N, K, g_q4k_planes, num_sms, status, stream, &e)) return e;
    }
    for (int b0 = 0; b0 < batch; b0 += 2) {
        const int nb = min(2, batch - b0);
        Q4kPlan p;
        cudaError_t e;
        const float* xb = x + static_cast<size_t>(b0) * K;
        float* yb = y + static_cast<size_t>(b0) * N;
        if (q4k_make_plan(N, K, nb, num_sms, &p)) {
            e = nb == 2 ? launch_tiled<2>(W, xb, yb, N, K, p, status, stream)
                        : launch_tiled<1>(W, xb, yb, N, K, p, status, stream);
        } else {
            const int wpb = 8;
            q4k_matvec_simple<<<(N + wpb - 1) / wpb, wpb * 32, 0, stream>>>(W, xb, yb, N, K, nb);
            note_launch();
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace larql
