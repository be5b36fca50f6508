// decode_persist.cu — one decode token through every layer in ONE persistent kernel launch.
//
// The per-layer pipeline of decode.cu + q4k_mma.cu (norm, Q|K|V matvec, attention, O matvec, residual + norm,
// gate|up matvec, SiLU, down matvec, residual) pays a launch, a TMA pipeline fill and a drain per kernel: eight
// kernels per layer, each matvec carrying ~4.5-5.5 us of fixed cost against 2-11 us of weight streaming.  Here one
// CTA per SM lives for the whole token:
//
//   * a producer warp streams the token's Q4_K weights — every layer's Q|K|V, O, gate|up and down row tiles this
//     CTA owns, in the order the consumers use them — through a ring of shared-memory stages with TMA.  Weights
//     do not depend on the activations, so the stream never waits for a phase to finish, only for a free stage:
//     while the consumers run attention or wait at a grid barrier the ring fills with the next matrices' tiles.
//   * eight consumer warps run the phases, separated by grid-wide barriers (an arrival counter in global memory,
//     every wait bounded by the status-word budget):
//       A  Q|K|V matvec of RMSNorm(x + the previous layer's down output), the new residual written;
//       B  attention partials: (KV head, 128-key range) items; RoPE, KV-cache append, f32 scores, f64 softmax sums;
//       C  attention combine: per (query head, 32 dimensions), the ranges in order;
//       D  O matvec of the attention output;
//       E  gate|up matvec of RMSNorm(x + O output), the new residual written;
//       F  down matvec of silu(gate) * up;
//     and after the last layer the final residual.  Six barriers per layer.
//
// Matvec arithmetic: the warp-MMA Q4_K factorisation of q4k_mma.cu (mma_superblock<1> on 32-row tiles of 2
// row groups x 4 K slices, 1024-value chunks).  K is split into `nparts` parts; each part's partial sums land in
// a per-part buffer and the reader of a projection adds the parts in part order (the split-K order of
// q4k_mma.cu).  RMSNorm's scale is applied after the product: the x tables of a norm-fused projection hold
// x * (offset + w), and its results are divided by rms — the tables are built from the whole residual, so the
// same pass yields the f64 sum of squares.
//
// References (the CPU pieces the decode layer composes; the reference's CPU backend has no decode_token,
// crates/larql-compute/src/backend.rs:115-124): rms_norm_eps crates/larql-inference/src/residual.rs:17-35,
// apply_rope crates/larql-inference/src/attention/rope.rs:22-55, GQA crates/larql-inference/src/attention/
// gqa.rs:29-110, silu_gate_up crates/larql-inference/src/ffn/mod.rs:87-94, Q4_K rows
// crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "q4k_mma_dev.cuh"

namespace larql {

constexpr int kPdW = 8;                           // consumer warps
constexpr int kPdCons = 32 * kPdW;                // consumer threads
constexpr int kPdThreads = kPdCons + 32;          // + the producer warp
constexpr int kPdNG = 2, kPdKS = 4;               // 16-row groups x K slices per tile
constexpr int kPdRT = 16 * kPdNG;                 // rows per tile
constexpr int kPdStage = kPdRT * kMmaRowBytes;    // one ring stage: 32 rows x one 1024-value chunk
constexpr int kPdKC = 128;                        // keys per attention item
constexpr int kPdHd = 128;                        // head dimension
constexpr int kPdMaxKpc = 8;                      // chunks per K part at most (x-table room)
constexpr int kPdMaxHidden = kPdMaxKpc * 1024;    // norm-fused projections take all of hidden in one part
// x tables of up to kPdMaxKpc chunks (B = 1, one n-tile): per chunk 8 KB of B fragments, 512 B of sum
// fragments, 256 B of plane weights; then the K-slice reduction area
constexpr int kPdXt = 0;
constexpr int kPdMt = kPdXt + kPdMaxKpc * 8192;
constexpr int kPdWt = kPdMt + kPdMaxKpc * 512;
constexpr int kPdRed = kPdWt + kPdMaxKpc * 256;
constexpr int kPdTabEnd = kPdRed + 2 * kPdKS * kPdRT * 4;
constexpr int kPdAux = 80 * 1024;                 // tables, or the attention's K / V staging and scores
constexpr int kPdMisc = 1024;
static_assert(kPdTabEnd <= kPdAux, "x tables exceed the aux region");
static_assert(2 * kPdKC * 256 + 8 * kPdHd * 4 * 2 + 2 * kPdHd * 4 + 8 * 4 + 8 * 8 <= kPdAux,
              "attention staging exceeds the aux region");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier over the consumer threads of every CTA: bar[0] counts arrivals over the whole launch (zeroed
// before it), so barrier number n of the launch is passed once bar[0] reaches n * gridDim.x; bar[2] is an abort
// flag.  `epoch` is thread 0's count of barriers passed.  The wait is bounded by the status-word budget.
__device__ bool pd_grid_sync(unsigned* bar, unsigned& epoch, int* status, int site, volatile int* cta_abort) {
    bool ok = true;
    named_bar_sync(1, kPdCons);
    if (threadIdx.x == 0) {
        ++epoch;
        const unsigned target = epoch * gridDim.x;
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const uint64_t t0 = globaltimer_ns();
        for (int spin = 0; ld_acquire_u32(bar) < target; ++spin) {
            if ((spin & 63) == 63) {
                if (ld_acquire_u32(bar + 2) != 0u) {
                    ok = false;
                    break;
                }
                if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                    set_status(status, LARQL_ERR_TIMEOUT, site);
                    atomicExch(bar + 2, 1u);
                    ok = false;
                    break;
                }
            }
        }
        __threadfence();
        if (!ok) *cta_abort = 1;
    }
    return !named_bar_red_or(1, kPdCons, !ok);
}

// One projection type (the same shape in every layer).
struct PdMat {
    int N, K, nchunks, nparts, ntiles, nitems;
};

struct PdParams {
    int L, H, I, nq, nkv, qkvd, qd;
    int pos, nch;      // token position, attention key ranges (ceil((pos + 1) / kPdKC))
    int NS, smem;      // ring stages, dynamic shared memory
    PdMat m[4];        // 0 Q|K|V [qkvd x H], 1 O [H x qd], 2 gate|up [2I x H], 3 down [H x I]
    double rope_base;
};

struct PdLayer {
    const float* norms;  // [2][H]
    __half* kc;          // [max_seq][nkv * 128]
    __half* vc;
    float offset, eps, scale;
};

struct PdBufs {
    float* x[2];       // x[0]: the caller's residual (in and out), x[1]: the alternate copy
    float* part[4];    // per projection: [nparts][N] partial sums
    float* att_acc;    // [nkv * nch][REPS * 128]
    float* att_m;      // [nkv * nch][REPS]
    double* att_l;     // [nkv * nch][REPS]
    float* attn;       // [qd]
    unsigned* bar;     // [4] grid barrier (zero before the launch)
};

__host__ __device__ inline int pd_part_c0(const PdMat& m, int part) { return part * m.nchunks / m.nparts; }

// Items [lo, hi) of a projection run on CTA b: a contiguous range, so the K part changes at most once.
__device__ __forceinline__ int pd_item_lo(const PdMat& m, int b) {
    return static_cast<int>(static_cast<long long>(b) * m.nitems / gridDim.x);
}

// Sum of a projection's K parts at indices i .. i + 3, in part order (the split-K order of q4k_mma.cu).
__device__ __forceinline__ float4 pd_sum_parts4(const float* part, int nparts, int N, int i) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int q = 0; q < nparts; ++q) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(part + static_cast<size_t>(q) * N + i));
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
    }
    return s;
}

// The producer's box sequence: every layer's projections, this CTA's items, their chunks.
struct PdCursor {
    int l, mi, item, ihi, c, c1;
    __device__ void start_mat(const PdParams& p) {
        for (; l < p.L; ++l, mi = 0) {
            for (; mi < 4; ++mi) {
                const PdMat& m = p.m[mi];
                item = pd_item_lo(m, blockIdx.x);
                ihi = pd_item_lo(m, blockIdx.x + 1);
                if (item < ihi) {
                    const int part = item / m.ntiles;
                    c = pd_part_c0(m, part);
                    c1 = pd_part_c0(m, part + 1);
                    return;
                }
            }
        }
    }
    __device__ bool valid(const PdParams& p) const { return l < p.L; }
    __device__ int tile(const PdParams& p) const { return item % p.m[mi].ntiles; }
    __device__ void next(const PdParams& p) {
        if (++c < c1) return;
        const PdMat& m = p.m[mi];
        if (++item < ihi) {
            const int part = item / m.ntiles;
            c = pd_part_c0(m, part);
            c1 = pd_part_c0(m, part + 1);
            return;
        }
        ++mi;
        if (mi == 4) {
            mi = 0;
            ++l;
        }
        start_mat(p);
    }
};

struct PdV8 {
    float4 a, b;
    double sq;  // norm sources: the sum of squares of the residual values behind a, b
};

// Where a projection's x comes from (one code path for all four projections keeps the table build and the MMA
// loop in the instruction cache from phase to phase).
struct PdSrc {
    int kind;          // 0: xin as given; 1: RMSNorm source; 2: silu(gate) * up
    const float* xin;  // kind 0: x; kind 1: the residual before the add
    const float* add;  // kind 1: parts to add to xin ([addp][H]); kind 2: gate|up parts ([addp][2I])
    int addp;
    float* xout;       // kind 1: where this CTA writes its slice of the new residual
    const float* nw;   // kind 1: norm weight
    float off;         // kind 1: norm offset
    int n;             // kind 1: H (part stride); kind 2: I
    int slo, shi;      // kind 1: this CTA's residual slice in float4 groups
};

// Values k0 .. k0 + 7 of a projection's x.  Kind 1 returns x * (offset + w) of the new residual x = xin + parts,
// writes the slice of x this CTA owns, and the sum of squares of x; kind 2 silu(gate) * up (ffn/mod.rs:87-94).
__device__ __forceinline__ PdV8 pd_load(const PdSrc& sr, int k0) {
    // every load of the first part (and of x and the norm weight) is issued before any of them is used
    PdV8 r;
    r.sq = 0.0;
    if (sr.kind == 2) {
        const int N2 = 2 * sr.n;
        const float4* g = reinterpret_cast<const float4*>(sr.add + k0);
        const float4* u = reinterpret_cast<const float4*>(sr.add + sr.n + k0);
        float4 g0 = __ldcg(g), g1 = __ldcg(g + 1), u0 = __ldcg(u), u1 = __ldcg(u + 1);
        for (int q = 1; q < sr.addp; ++q) {
            const size_t o4 = static_cast<size_t>(q) * N2 / 4;
            const float4 h0 = __ldcg(g + o4), h1 = __ldcg(g + o4 + 1), v0 = __ldcg(u + o4), v1 = __ldcg(u + o4 + 1);
            g0 = make_float4(g0.x + h0.x, g0.y + h0.y, g0.z + h0.z, g0.w + h0.w);
            g1 = make_float4(g1.x + h1.x, g1.y + h1.y, g1.z + h1.z, g1.w + h1.w);
            u0 = make_float4(u0.x + v0.x, u0.y + v0.y, u0.z + v0.z, u0.w + v0.w);
            u1 = make_float4(u1.x + v1.x, u1.y + v1.y, u1.z + v1.z, u1.w + v1.w);
        }
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = gv[i] * (1.0f / (1.0f + expf(-gv[i]))) * uv[i];
        r.a = make_float4(o[0], o[1], o[2], o[3]);
        r.b = make_float4(o[4], o[5], o[6], o[7]);
        return r;
    }
    float4 x0 = __ldcg(reinterpret_cast<const float4*>(sr.xin + k0));
    float4 x1 = __ldcg(reinterpret_cast<const float4*>(sr.xin + k0 + 4));
    if (sr.kind == 0) {
        r.a = x0;
        r.b = x1;
        return r;
    }
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(sr.nw + k0));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(sr.nw + k0 + 4));
    if (sr.addp) {
        const float4* pa = reinterpret_cast<const float4*>(sr.add + k0);
        float4 a0 = __ldcg(pa), a1 = __ldcg(pa + 1);
        for (int q = 1; q < sr.addp; ++q) {
            const size_t o4 = static_cast<size_t>(q) * sr.n / 4;
            const float4 h0 = __ldcg(pa + o4), h1 = __ldcg(pa + o4 + 1);
            a0 = make_float4(a0.x + h0.x, a0.y + h0.y, a0.z + h0.z, a0.w + h0.w);
            a1 = make_float4(a1.x + h1.x, a1.y + h1.y, a1.z + h1.z, a1.w + h1.w);
        }
        x0 = make_float4(x0.x + a0.x, x0.y + a0.y, x0.z + a0.z, x0.w + a0.w);
        x1 = make_float4(x1.x + a1.x, x1.y + a1.y, x1.z + a1.z, x1.w + a1.w);
        const int i4 = k0 >> 2;
        if (i4 >= sr.slo && i4 < sr.shi) reinterpret_cast<float4*>(sr.xout)[i4] = x0;
        if (i4 + 1 >= sr.slo && i4 + 1 < sr.shi) reinterpret_cast<float4*>(sr.xout)[i4 + 1] = x1;
    }
    const float off = sr.off;
    r.a = make_float4(x0.x * (off + w0.x), x0.y * (off + w0.y), x0.z * (off + w0.z), x0.w * (off + w0.w));
    r.b = make_float4(x1.x * (off + w1.x), x1.y * (off + w1.y), x1.z * (off + w1.z), x1.w * (off + w1.w));
    const float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    double q = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) q += static_cast<double>(xs[i]) * static_cast<double>(xs[i]);
    r.sq = q;
    return r;
}

// x tables of chunks [c0, c1) from the source's values (consumer threads); returns this thread's sum of the
// source's sq.  The layout and digit planes are those of mma_build_tables<1, 1, PRO, 0> (q4k_mma_dev.cuh).
__device__ __forceinline__ double pd_build_tables(uint8_t* aux, int c0, int c1, int ctid, int cwarp, int lane,
                                                  const PdSrc& src) {
    uint2* xt = reinterpret_cast<uint2*>(aux + kPdXt);
    uint8_t* mt = aux + kPdMt;
    float* wt = reinterpret_cast<float*>(aux + kPdWt);
    const int nsb = (c1 - c0) * 4;
    {
        uint4* z = reinterpret_cast<uint4*>(aux);
        for (int i = ctid; i < kPdRed / 16; i += kPdCons) z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    named_bar_sync(1, kPdCons);
    const int j = lane >> 2, t = lane & 3;
    constexpr int U = 2;
    double sq = 0.0;
#pragma unroll 1
    for (int sbl0 = cwarp; sbl0 < nsb; sbl0 += U * kPdW) {
        float v[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int sbl = sbl0 + u * kPdW;
            PdV8 r{make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f), 0.0};
            if (sbl < nsb) r = pd_load(src, (c0 * 4 + sbl) * 256 + lane * 8);
            sq += r.sq;
            v[u][0] = r.a.x;
            v[u][1] = r.a.y;
            v[u][2] = r.a.z;
            v[u][3] = r.a.w;
            v[u][4] = r.b.x;
            v[u][5] = r.b.y;
            v[u][6] = r.b.z;
            v[u][7] = r.b.w;
        }
        float amax[U], s[U];
        bool nonfin[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            amax[u] = 0.f;
            s[u] = 0.f;
            nonfin[u] = false;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                amax[u] = fmaxf(amax[u], fabsf(v[u][i]));
                s[u] += v[u][i];
                nonfin[u] |= !isfinite(v[u][i]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int u = 0; u < U; ++u) amax[u] = fmaxf(amax[u], __shfl_xor_sync(0xffffffffu, amax[u], o));
#pragma unroll
        for (int o = 1; o < 4; o <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
        float am[U];
#pragma unroll
        for (int u = 0; u < U; ++u) am[u] = fabsf(s[u]);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u) am[u] = fmaxf(am[u], __shfl_xor_sync(0xffffffffu, am[u], o));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int sbl = sbl0 + u * kPdW;
            const bool fin = !__any_sync(0xffffffffu, nonfin[u]);
            if (sbl >= nsb) continue;  // warp-uniform
            const int e = plane_exponent<3>(amax[u]);
            const float down = pow2i(-e);
            uint32_t pl[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
            for (int k2 = 0; k2 < 8; ++k2) {
                const int xi = fin ? __float2int_rn(v[u][k2] * down) : 0;
                int dg[3];
                digits<3>(xi, dg);
                const int par = k2 & 1, pos = 8 * (k2 >> 1);
#pragma unroll
                for (int z = 0; z < 3; ++z) pl[z][par] |= (static_cast<uint32_t>(dg[z]) & 0xFFu) << pos;
            }
#pragma unroll
            for (int z = 0; z < 3; ++z) xt[(sbl * 8 + j) * 32 + z * 4 + t] = make_uint2(pl[z][0], pl[z][1]);
            const bool finm = fin && isfinite(am[u]);
            const int em = plane_exponent<3>(finm ? am[u] : 0.f);
            if (t == 0) {
                const int xi = finm ? __float2int_rn(s[u] * pow2i(-em)) : 0;
                int dz[3];
                digits<3>(xi, dz);
#pragma unroll
                for (int z = 0; z < 3; ++z)
                    mt[((sbl * 32) + z * 4 + (j >> 2)) * 4 + (j & 3)] = static_cast<uint8_t>(dz[z] & 0xFF);
            }
            if (lane == 0) {
                const float qnan = __int_as_float(0x7fc00000);
#pragma unroll
                for (int z = 0; z < 3; ++z) {
                    float* w4 = wt + (sbl * 4 + (z >> 1)) * 4;
                    w4[z & 1] = fin ? pow2i(e + 8 * (2 - z)) : qnan;
                    w4[2 + (z & 1)] = finm ? pow2i(em + 8 * (2 - z)) : qnan;
                }
            }
        }
    }
    named_bar_sync(1, kPdCons);
    return sq;
}

// One projection: this CTA's (part, tile) items, chunks taken from the ring in the producer's order.  Tables are
// built with `load` whenever the part changes.  Results: part buffer [part][N].  norm_h > 0 (a single K part):
// the loader returned x * (offset + w) and the sums of squares of x, so every result is divided by
// rms = sqrt(sum / norm_h + eps) in f64 — RMSNorm's scale, applied after the product instead of before it.
__device__ __noinline__ bool pd_matvec(const PdMat m, uint8_t* smem, uint8_t* aux, uint64_t* full, uint64_t* empty,
                                       int NS, int* kp, float* dst, int ctid, int cwarp, int lane, int* status,
                                       volatile int* cta_abort, double* red, volatile float* rms_s, int norm_h,
                                       float eps, const PdSrc src) {
    int k = *kp;
    const int g = lane >> 2, t = lane & 3;
    const int rg = cwarp % kPdNG, ks = cwarp / kPdNG;
    const int row_in_tile = 16 * rg + g;
    const uint2* xt = reinterpret_cast<const uint2*>(aux + kPdXt);
    const uint32_t* mt = reinterpret_cast<const uint32_t*>(aux + kPdMt);
    const float4* wt = reinterpret_cast<const float4*>(aux + kPdWt);
    float* redk = reinterpret_cast<float*>(aux + kPdRed);
    int rbuf = 0;
    int cur_part = -1;
    float rms = 1.f;
    const int ihi = pd_item_lo(m, blockIdx.x + 1);
    for (int item = pd_item_lo(m, blockIdx.x); item < ihi; ++item) {
        const int part = item / m.ntiles, tile = item - part * m.ntiles;
        const int c0 = pd_part_c0(m, part), c1 = pd_part_c0(m, part + 1);
        if (part != cur_part) {
            double sq = pd_build_tables(aux, c0, c1, ctid, cwarp, lane, src);
            if (norm_h > 0) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (lane == 0) red[cwarp] = sq;
                named_bar_sync(1, kPdCons);
                if (ctid == 0) {
                    double tsum = 0.0;
                    for (int w = 0; w < kPdW; ++w) tsum += red[w];
                    *rms_s = static_cast<float>(sqrt(tsum / static_cast<double>(norm_h) + static_cast<double>(eps)));
                }
                named_bar_sync(1, kPdCons);
                rms = *rms_s;
            }
            cur_part = part;
        }
        float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
        bool ok = true;
        for (int c = c0; c < c1; ++c, ++k) {
            const int st = k % NS;
            if (ok) {
                const bool got = !*cta_abort && mbar_wait(&full[st], (k / NS) & 1, status, 61);
                ok = __all_sync(0xffffffffu, got);
            }
            if (ok) {
                const uint8_t* wrow = smem + static_cast<size_t>(st) * kPdStage + row_in_tile * kMmaRowBytes;
                const int sbl = (c - c0) * 4 + ks;
                mma_superblock<1>(wrow + ks * 148, xt + sbl * 8 * 32, mt + sbl * 32, wt + sbl * 4, lane, t, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
        }
        if (!ok && lane == 0) *cta_abort = 1;
        // this thread's two rows (g, g + 8): C columns 0..2 are the three planes of the one batch row
        float sg = 0.f, sg8 = 0.f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            if ((2 * t + q) / 3 == 0) {
                sg += acc[0][q];
                sg8 += acc[0][2 + q];
            }
        }
        sg += __shfl_xor_sync(0xffffffffu, sg, 1);
        sg += __shfl_xor_sync(0xffffffffu, sg, 2);
        sg8 += __shfl_xor_sync(0xffffffffu, sg8, 1);
        sg8 += __shfl_xor_sync(0xffffffffu, sg8, 2);
        float* rw = redk + (rbuf * kPdKS + ks) * kPdRT + row_in_tile;
        if (t == 0) {
            rw[0] = sg;
            rw[8] = sg8;
        }
        // the K slices of a row group add their sums in slice order
        if (named_bar_red_or(1, kPdCons, !ok || *cta_abort)) {
            *kp = k;
            return false;
        }
        if (ks == 0 && lane < 16) {
            const float* rr = redk + (rbuf * kPdKS) * kPdRT + 16 * rg + lane;
            float s = 0.f;
            for (int q = 0; q < kPdKS; ++q) s += rr[q * kPdRT];
            const int row = tile * kPdRT + 16 * rg + lane;
            if (row < m.N) dst[static_cast<size_t>(part) * m.N + row] = norm_h > 0 ? s / rms : s;
        }
        rbuf ^= 1;
    }
    *kp = k;
    return true;
}

// Attention partials of one layer: item = (KV head, range of kPdKC keys).  Follows decode_attention_kernel
// (decode.cu) for one sub-chunk: RoPE of the REPS query heads and the new key (cos / sin of the position from
// f64 angles), the new k / v appended to the f16 caches by the item holding key `pos`, f32 dots times the scale,
// exp(s - max) and its sum in f64, P . V summed over warps in warp order.
template <int REPS>
__device__ __noinline__ void pd_attention(const PdParams& p, const PdLayer& L, const PdBufs& b, uint8_t* aux,
                             const float* rope_c, const float* rope_s, int ctid, int cwarp, int lane) {
    uint8_t* ksm = aux;                                   // [kPdKC][256 B], chunk c of key j at c ^ (j & 7)
    uint8_t* vsm = aux + kPdKC * 256;                     // [kPdKC][256 B]
    float* qs = reinterpret_cast<float*>(aux + 2 * kPdKC * 256);  // [REPS][128]
    float* kn = qs + 8 * kPdHd;                           // [128]
    float* vn = kn + kPdHd;                               // [128]
    float* sc = vn + kPdHd;                               // [REPS][kPdKC]
    float* cm = sc + 8 * kPdKC;                           // [8]
    double* cl = reinterpret_cast<double*>(cm + 8);       // [8]
    const int G = static_cast<int>(gridDim.x);
    const int kvd = p.nkv * kPdHd;
    const int nkeys = p.pos + 1;
    const int nitems = p.nkv * p.nch;
    const float* qkv = b.part[0];
    const int np0 = p.m[0].nparts, N0 = p.m[0].N;
    for (int item = blockIdx.x; item < nitems; item += G) {
        const int kvh = item / p.nch, ch = item - kvh * p.nch;
        const int jb = ch * kPdKC, je = min(nkeys, jb + kPdKC), nks = je - jb;
        // the range's K / V rows, staged asynchronously; row `pos` (when in range) is staged too but never read:
        // this item uses the new key and value from registers and writes that row to the caches itself
        for (int i = ctid; i < nks * 16; i += kPdCons) {
            const int jj = i >> 4, c = i & 15;
            const size_t off = static_cast<size_t>(jb + jj) * kvd + kvh * kPdHd + c * 8;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ksm + jj * 256 + ((c ^ (jj & 7)) << 4))),
                         "l"(L.kc + off)
                         : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(vsm + jj * 256 + (c << 4))),
                         "l"(L.vc + off)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        // the projection values this item needs (REPS query heads, the new key and value), parts summed in order
        if (ctid < kPdHd) {
            float r[REPS + 2];
#pragma unroll
            for (int i = 0; i < REPS + 2; ++i) r[i] = 0.f;
            for (int q = 0; q < np0; ++q) {
                const float* src = qkv + static_cast<size_t>(q) * N0;
                float tv[REPS + 2];
#pragma unroll
                for (int h = 0; h < REPS; ++h) tv[h] = __ldcg(src + (kvh * REPS + h) * kPdHd + ctid);
                tv[REPS] = __ldcg(src + p.nq * kPdHd + kvh * kPdHd + ctid);
                tv[REPS + 1] = __ldcg(src + p.nq * kPdHd + kvd + kvh * kPdHd + ctid);
#pragma unroll
                for (int i = 0; i < REPS + 2; ++i) r[i] += tv[i];
            }
#pragma unroll
            for (int h = 0; h < REPS; ++h) qs[h * kPdHd + ctid] = r[h];
            kn[ctid] = r[REPS];
            vn[ctid] = r[REPS + 1];
        }
        named_bar_sync(1, kPdCons);
        // RoPE (split halves) of the query heads and the new key, in place
        if (ctid < kPdHd / 2) {
            const float c = rope_c[ctid], sn = rope_s[ctid];
#pragma unroll
            for (int h = 0; h < REPS; ++h) {
                const float x0 = qs[h * kPdHd + ctid], x1 = qs[h * kPdHd + ctid + kPdHd / 2];
                qs[h * kPdHd + ctid] = x0 * c - x1 * sn;
                qs[h * kPdHd + ctid + kPdHd / 2] = x0 * sn + x1 * c;
            }
            const float x0 = kn[ctid], x1 = kn[ctid + kPdHd / 2];
            kn[ctid] = x0 * c - x1 * sn;
            kn[ctid + kPdHd / 2] = x0 * sn + x1 * c;
        }
        named_bar_sync(1, kPdCons);
        if (p.pos >= jb && p.pos < je && ctid < kPdHd) {
            L.kc[static_cast<size_t>(p.pos) * kvd + kvh * kPdHd + ctid] = __float2half_rn(kn[ctid]);
            L.vc[static_cast<size_t>(p.pos) * kvd + kvh * kPdHd + ctid] = __float2half_rn(vn[ctid]);
        }
        float4 q4[REPS];
#pragma unroll
        for (int h = 0; h < REPS; ++h) q4[h] = *reinterpret_cast<const float4*>(&qs[h * kPdHd + 4 * lane]);
        const float4 kn4 = *reinterpret_cast<const float4*>(&kn[4 * lane]);
        const float4 vn4 = *reinterpret_cast<const float4*>(&vn[4 * lane]);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        named_bar_sync(1, kPdCons);
        // scores: warp w takes the groups of GK keys starting at GK*w, GK*(w+8), ...; lane holds dimensions
        // 4l..4l+3; the GK * REPS partial dots are reduce-scattered over the 32 lanes
        constexpr int GK = 32 / REPS;
        for (int g0 = cwarp * GK; g0 < nks; g0 += kPdW * GK) {
            float v[32];
#pragma unroll
            for (int kk = 0; kk < GK; ++kk) {
                const int jj = g0 + kk;
                float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (jj < nks) {
                    if (jb + jj == p.pos) {
                        k4 = kn4;
                    } else {
                        const uint2 raw = *reinterpret_cast<const uint2*>(
                            ksm + jj * 256 + (((lane >> 1) ^ (jj & 7)) << 4) + ((lane & 1) << 3));
                        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                        const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                        k4 = make_float4(a.x, a.y, b2.x, b2.y);
                    }
                }
#pragma unroll
                for (int h = 0; h < REPS; ++h) {
                    float pr = q4[h].x * k4.x;
                    pr = fmaf(q4[h].y, k4.y, pr);
                    pr = fmaf(q4[h].z, k4.z, pr);
                    pr = fmaf(q4[h].w, k4.w, pr);
                    v[kk * REPS + h] = pr;
                }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const bool up = (lane & o) != 0;
#pragma unroll
                for (int i = 0; i < o; ++i) {
                    const float send = up ? v[i] : v[i + o];
                    const float keep = up ? v[i + o] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            const int jj = g0 + lane / REPS;
            if (jj < nks) sc[(lane % REPS) * kPdKC + jj] = v[0] * L.scale;
        }
        named_bar_sync(1, kPdCons);
        // softmax over this range per head (warp h): exp(s - max) in f64 and its f64 sum
        for (int h = cwarp; h < REPS; h += kPdW) {
            float mx = -INFINITY;
            for (int jj = lane; jj < nks; jj += 32) mx = fmaxf(mx, sc[h * kPdKC + jj]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            double l = 0.0;
            for (int jj = lane; jj < nks; jj += 32) {
                const double e = exp(static_cast<double>(sc[h * kPdKC + jj] - mx));
                sc[h * kPdKC + jj] = static_cast<float>(e);
                l += e;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                cm[h] = mx;
                cl[h] = l;
            }
        }
        named_bar_sync(1, kPdCons);
        // P . V: warp w over keys w, w+8, ..., lane over dimensions 4l..4l+3
        float4 acc[REPS];
#pragma unroll
        for (int h = 0; h < REPS; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int jj = cwarp; jj < nks; jj += kPdW) {
            float4 v4;
            if (jb + jj == p.pos) {
                v4 = vn4;
            } else {
                const uint2 raw = *reinterpret_cast<const uint2*>(vsm + jj * 256 + 8 * lane);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                v4 = make_float4(a.x, a.y, b2.x, b2.y);
            }
#pragma unroll
            for (int h = 0; h < REPS; ++h) {
                const float pr = sc[h * kPdKC + jj];
                acc[h].x = fmaf(pr, v4.x, acc[h].x);
                acc[h].y = fmaf(pr, v4.y, acc[h].y);
                acc[h].z = fmaf(pr, v4.z, acc[h].z);
                acc[h].w = fmaf(pr, v4.w, acc[h].w);
            }
        }
        named_bar_sync(1, kPdCons);  // every warp is done with K (the reduction area)
        float* red = reinterpret_cast<float*>(ksm);  // [8 warps][REPS][128]
#pragma unroll
        for (int h = 0; h < REPS; ++h) *reinterpret_cast<float4*>(&red[(cwarp * REPS + h) * kPdHd + 4 * lane]) = acc[h];
        named_bar_sync(1, kPdCons);
        float* dst = b.att_acc + static_cast<size_t>(item) * REPS * kPdHd;
        for (int i = ctid; i < REPS * kPdHd; i += kPdCons) {
            const int h = i / kPdHd;
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kPdW; ++w) s += red[(w * REPS + h) * kPdHd + (i % kPdHd)];
            dst[i] = s;
        }
        if (ctid < REPS) {
            b.att_m[item * REPS + ctid] = cm[ctid];
            b.att_l[item * REPS + ctid] = cl[ctid];
        }
        named_bar_sync(1, kPdCons);  // shared memory is reused by the next item
    }
}

// Attention output per (query head, 32 dimensions), one warp each: the key ranges combined in range order with
// weights exp(m_r - M) (f64, as the reference's sum), normalised by the f64 total.  The ranges' statistics are
// spread over the lanes and every range's accumulator is loaded before the ordered sums.
template <int REPS>
__device__ __noinline__ void pd_attention_combine(const PdParams& p, const PdBufs& b, int cwarp, int lane) {
    const int units = p.nq * 4;
    for (int u = static_cast<int>(blockIdx.x) * kPdW + cwarp; u < units; u += static_cast<int>(gridDim.x) * kPdW) {
        const int head = u >> 2, kvh = head / REPS, hr = head % REPS, d = (u & 3) * 32 + lane;
        const int base = kvh * p.nch;
        float M = -INFINITY;
        for (int c = lane; c < p.nch; c += 32) M = fmaxf(M, __ldcg(b.att_m + (base + c) * REPS + hr));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        double Lsum = 0.0;
        float o = 0.f;
        for (int c0 = 0; c0 < p.nch; c0 += 32) {
            const int c = c0 + lane, cnt = min(32, p.nch - c0);
            float f = 0.f;
            double lf = 0.0;
            if (c < p.nch) {
                const float mc = __ldcg(b.att_m + (base + c) * REPS + hr);
                const double fd = mc == -INFINITY ? 0.0 : exp(static_cast<double>(mc - M));
                lf = __ldcg(b.att_l + (base + c) * REPS + hr) * fd;
                f = static_cast<float>(fd);
            }
            float av[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
                av[i] = i < cnt ? __ldcg(b.att_acc + (static_cast<size_t>(base + c0 + i) * REPS + hr) * kPdHd + d) : 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const double li = __shfl_sync(0xffffffffu, lf, i);
                const float fi = __shfl_sync(0xffffffffu, f, i);
                if (i < cnt) {
                    Lsum += li;
                    o = fmaf(av[i], fi, o);
                }
            }
        }
        b.attn[head * kPdHd + d] = o * static_cast<float>(1.0 / Lsum);
    }
}

template <int REPS>
__global__ void __launch_bounds__(kPdThreads, 1)
    decode_persist_kernel(const PdParams p, const PdLayer* __restrict__ lay, const CUtensorMap* __restrict__ maps,
                          const PdBufs b, int* status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int NS = p.NS;
    uint8_t* aux = smem + static_cast<size_t>(NS) * kPdStage;
    uint8_t* misc = aux + kPdAux;
    uint64_t* full = reinterpret_cast<uint64_t*>(misc);
    uint64_t* empty = full + NS;
    volatile int* cta_abort = reinterpret_cast<volatile int*>(empty + NS);
    volatile float* rms_s = reinterpret_cast<volatile float*>(cta_abort + 1);
    double* red = reinterpret_cast<double*>(misc + 2 * 8 * NS + 16);  // [kPdW]
    float* rope_c = reinterpret_cast<float*>(red + kPdW);              // [64]
    float* rope_s = rope_c + kPdHd / 2;                                // [64]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = static_cast<int>(gridDim.x);
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kPdW);
        }
        *cta_abort = 0;
        fence_barrier_init();
    }
    // RoPE angles of the position (rope.rs:22-55): f64 inverse frequencies and angles, cos / sin rounded to f32
    if (tid < kPdHd / 2) {
        const double inv = 1.0 / pow(p.rope_base, 2.0 * tid / static_cast<double>(kPdHd));
        double sd, cd;
        sincos(static_cast<double>(p.pos) * inv, &sd, &cd);
        rope_c[tid] = static_cast<float>(cd);
        rope_s[tid] = static_cast<float>(sd);
    }
    __syncthreads();

    if (warp == kPdW) {  // producer: one elected lane streams every projection's boxes in the consumers' order
        if (lane == 0) {
            // (an L2 prefetch cursor running 6 or 16 boxes beyond the ring measured slower: its traffic competes
            // with the attention and the partial sums for L2)
            PdCursor cur{0, 0, 0, 0, 0, 0};
            cur.start_mat(p);
            int k = 0;
            for (; cur.valid(p); cur.next(p), ++k) {
                const int st = k % NS;
                if (*cta_abort || (k >= NS && !mbar_wait(&empty[st], ((k / NS) - 1) & 1, status, 62))) {
                    *cta_abort = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(kPdStage));
                tma_load_2d(smem + static_cast<size_t>(st) * kPdStage, maps + cur.l * 4 + cur.mi,
                            cur.c * (kMmaRowBytes / 4), cur.tile(p) * kPdRT, &full[st]);
            }
            // every issued box lands before the CTA's shared memory goes away
            for (int jj = max(0, k - NS); jj < k; ++jj)
                if (!mbar_wait(&full[jj % NS], (jj / NS) & 1, status, 63)) break;
        }
        return;
    }

    const int ctid = tid, cwarp = warp;
    unsigned epoch = 0;
    int k = 0;
    int xr = 0;  // b.x[xr] holds the current residual
    const int H4 = p.H / 4;
    const int slo = static_cast<int>(static_cast<long long>(blockIdx.x) * H4 / G);  // this CTA's residual slice
    const int shi = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * H4 / G);
    auto norm_src = [&](const float* xin, const float* add, int addp, float* xout, const float* nw, float off) {
        PdSrc r{};
        r.kind = 1;
        r.xin = xin;
        r.add = add;
        r.addp = addp;
        r.xout = xout;
        r.nw = nw;
        r.off = off;
        r.n = p.H;
        r.slo = slo;
        r.shi = shi;
        return r;
    };
    // A CTA with no items of a norm-fused projection still writes its slice of the new residual.
    auto slice_only = [=](const PdMat& m, const float* xin, const float* add, int addp, float* xout) {
        if (addp == 0 || pd_item_lo(m, blockIdx.x) < pd_item_lo(m, blockIdx.x + 1)) return;
        for (int i4 = slo + ctid; i4 < shi; i4 += kPdCons) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(xin) + i4);
            const float4 a4 = pd_sum_parts4(add, addp, p.H, 4 * i4);
            reinterpret_cast<float4*>(xout)[i4] = make_float4(v.x + a4.x, v.y + a4.y, v.z + a4.z, v.w + a4.w);
        }
    };
    for (int l = 0; l < p.L; ++l) {
        const PdLayer& L = lay[l];
        // A: Q|K|V of RMSNorm(x + the previous layer's down output)
        {
            const int addp = l ? p.m[3].nparts : 0;
            if (!pd_matvec(p.m[0], smem, aux, full, empty, NS, &k, b.part[0], ctid, cwarp, lane, status, cta_abort,
                           red, rms_s, p.H, L.eps, norm_src(b.x[xr], b.part[3], addp, b.x[xr ^ 1], L.norms, L.offset)))
                return;
            slice_only(p.m[0], b.x[xr], b.part[3], addp, b.x[xr ^ 1]);
            if (l) xr ^= 1;
        }
        if (!pd_grid_sync(b.bar, epoch, status, 64, cta_abort)) return;
        // B: attention partials
        pd_attention<REPS>(p, L, b, aux, rope_c, rope_s, ctid, cwarp, lane);
        if (!pd_grid_sync(b.bar, epoch, status, 65, cta_abort)) return;
        // C: attention combine
        pd_attention_combine<REPS>(p, b, cwarp, lane);
        if (!pd_grid_sync(b.bar, epoch, status, 66, cta_abort)) return;
        // D: O projection of the attention output
        {
            PdSrc so{};
            so.kind = 0;
            so.xin = b.attn;
            if (!pd_matvec(p.m[1], smem, aux, full, empty, NS, &k, b.part[1], ctid, cwarp, lane, status, cta_abort,
                           red, rms_s, 0, 0.f, so))
                return;
        }
        if (!pd_grid_sync(b.bar, epoch, status, 67, cta_abort)) return;
        // E: gate|up of RMSNorm(x + O output)
        {
            const int addp = p.m[1].nparts;
            if (!pd_matvec(p.m[2], smem, aux, full, empty, NS, &k, b.part[2], ctid, cwarp, lane, status, cta_abort,
                           red, rms_s, p.H, L.eps,
                           norm_src(b.x[xr], b.part[1], addp, b.x[xr ^ 1], L.norms + p.H, L.offset)))
                return;
            slice_only(p.m[2], b.x[xr], b.part[1], addp, b.x[xr ^ 1]);
            xr ^= 1;
        }
        if (!pd_grid_sync(b.bar, epoch, status, 68, cta_abort)) return;
        // F: down projection of silu(gate) * up (ffn/mod.rs:87-94)
        {
            PdSrc sd{};
            sd.kind = 2;
            sd.add = b.part[2];
            sd.addp = p.m[2].nparts;
            sd.n = p.I;
            if (!pd_matvec(p.m[3], smem, aux, full, empty, NS, &k, b.part[3], ctid, cwarp, lane, status, cta_abort,
                           red, rms_s, 0, 0.f, sd))
                return;
        }
        if (!pd_grid_sync(b.bar, epoch, status, 69, cta_abort)) return;
    }
    // the last residual: x = x + down output, each CTA its slice, into the caller's buffer
    for (int i4 = slo + ctid; i4 < shi; i4 += kPdCons) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(b.x[xr]) + i4);
        const float4 a = pd_sum_parts4(b.part[3], p.m[3].nparts, p.H, 4 * i4);
        reinterpret_cast<float4*>(b.x[xr ^ 1])[i4] = make_float4(v.x + a.x, v.y + a.y, v.z + a.z, v.w + a.w);
    }
}

// ───────────────────────── host side ─────────────────────────

// single: one K part (the norm-fused projections, whose table build also yields the RMS of the whole residual)
static void pd_fill_mat(PdMat& m, int N, int K, int num_sms, bool single) {
    m.N = N;
    m.K = K;
    m.nchunks = K / 1024;
    m.ntiles = (N + kPdRT - 1) / kPdRT;
    // the fewest K parts whose tables fit, then more while the items do not cover the SMs
    int np = (m.nchunks + kPdMaxKpc - 1) / kPdMaxKpc;
    while (!single && np < m.nchunks && m.ntiles * np < num_sms) ++np;
    m.nparts = np;
    m.nitems = m.ntiles * np;
}

int decode_persist_plan(int L, int H, int I, int nq, int nkv, int pos, int num_sms, double rope_base,
                        DecodePersistPlan* out) {
    if (L < 1 || H <= 0 || I <= 0 || nkv < 1 || nq % nkv || pos < 0 || num_sms < 1) return -1;
    const int reps = nq / nkv;
    if (reps != 1 && reps != 2 && reps != 4 && reps != 8) return -1;
    const int qd = nq * kPdHd, qkvd = (nq + 2 * nkv) * kPdHd;
    if (H % 1024 || I % 1024 || qd % 1024 || H > kPdMaxHidden) return -1;
    PdParams p{};
    p.L = L;
    p.H = H;
    p.I = I;
    p.nq = nq;
    p.nkv = nkv;
    p.qd = qd;
    p.qkvd = qkvd;
    p.pos = pos;
    p.nch = (pos + 1 + kPdKC - 1) / kPdKC;
    pd_fill_mat(p.m[0], qkvd, H, num_sms, true);
    pd_fill_mat(p.m[1], H, qd, num_sms, false);
    pd_fill_mat(p.m[2], 2 * I, H, num_sms, true);
    pd_fill_mat(p.m[3], H, I, num_sms, false);
    p.NS = (kSmemLimit - kPdAux - kPdMisc) / kPdStage;
    if (p.NS > 8) p.NS = 8;
    if (p.NS < 2) return -1;
    p.smem = p.NS * kPdStage + kPdAux + kPdMisc;
    p.rope_base = rope_base;
    static_assert(sizeof(PdParams) <= sizeof(out->raw), "plan storage");
    memcpy(out->raw, &p, sizeof(p));
    out->reps = reps;
    out->grid = num_sms;
    out->smem = p.smem;
    for (int i = 0; i < 4; ++i) {
        out->N[i] = p.m[i].N;
        out->K[i] = p.m[i].K;
        out->nparts[i] = p.m[i].nparts;
    }
    out->att_items = nkv * p.nch;
    return 0;
}

int decode_persist_map(void* encode_fn, const void* w, int N, int K, CUtensorMap* map) {
    return mma_encode_map(encode_fn, w, N, K, 0, kPdRT, map);
}

// (every plan on a device has the same shared memory and grid, so a device that passed once passes for good)
template <int REPS>
static cudaError_t pd_attr(int smem, int grid) {
    static DeviceFlags resident_ok;
    int dev0 = 0;
    if (cudaGetDevice(&dev0) == cudaSuccess && resident_ok.test(dev0)) return cudaSuccess;
    static DeviceFlags attr_done;
    cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(decode_persist_kernel<REPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    int dev = 0, coop = 0, sms = 0, per_sm = 0;
    e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persist_kernel<REPS>, kPdThreads, smem);
    if (e != cudaSuccess) return e;
    if (!coop || static_cast<long long>(per_sm) * sms < grid) return cudaErrorCooperativeLaunchTooLarge;
    resident_ok.set(dev);
    return cudaSuccess;
}

// cudaSuccess when every CTA of the plan's grid can be resident at once (a cooperative launch is possible);
// cudaErrorCooperativeLaunchTooLarge when not.
cudaError_t decode_persist_check(const DecodePersistPlan& plan) {
    switch (plan.reps) {
        case 1: return pd_attr<1>(plan.smem, plan.grid);
        case 2: return pd_attr<2>(plan.smem, plan.grid);
        case 4: return pd_attr<4>(plan.smem, plan.grid);
        case 8: return pd_attr<8>(plan.smem, plan.grid);
        default: return cudaErrorInvalidValue;
    }
}

template <int REPS>
static cudaError_t launch_pd(const DecodePersistPlan& plan, const void* lay, const CUtensorMap* maps,
                             const DecodePersistBufs& bufs, int* status, cudaStream_t stream) {
    cudaError_t e = pd_attr<REPS>(plan.smem, plan.grid);
    if (e != cudaSuccess) return e;
    PdParams p;
    memcpy(&p, plan.raw, sizeof(p));
    PdBufs b{};
    b.x[0] = bufs.x;
    b.x[1] = bufs.xalt;
    for (int i = 0; i < 4; ++i) b.part[i] = bufs.part[i];
    b.att_acc = bufs.att_acc;
    b.att_m = bufs.att_m;
    b.att_l = bufs.att_l;
    b.attn = bufs.attn;
    b.bar = bufs.bar;
    e = cudaMemsetAsync(bufs.bar, 0, 4 * sizeof(unsigned), stream);
    if (e != cudaSuccess) return e;
    // cooperative: every CTA resident at once (the grid barriers need it), one per SM
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(kPdThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_persist_kernel<REPS>, p, static_cast<const PdLayer*>(lay), maps, b, status);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_decode_persist(const DecodePersistPlan& plan, const void* lay, const CUtensorMap* maps,
                                  const DecodePersistBufs& bufs, int* status, cudaStream_t stream) {
    switch (plan.reps) {
        case 1: return launch_pd<1>(plan, lay, maps, bufs, status, stream);
        case 2: return launch_pd<2>(plan, lay, maps, bufs, status, stream);
        case 4: return launch_pd<4>(plan, lay, maps, bufs, status, stream);
        case 8: return launch_pd<8>(plan, lay, maps, bufs, status, stream);
        default: return cudaErrorInvalidValue;
    }
}

size_t decode_persist_layer_bytes() { return sizeof(PdLayer); }

void decode_persist_layer_fill(void* dst, const float* norms, __half* kc, __half* vc, float offset, float eps,
                               float scale) {
    PdLayer l{};
    l.norms = norms;
    l.kc = kc;
    l.vc = vc;
    l.offset = offset;
    l.eps = eps;
    l.scale = scale;
    memcpy(dst, &l, sizeof(l));
}

}  // namespace larql
