// decode.cu — the non-matvec kernels of one Llama-style decode layer (one
// token): RMSNorm with the residual add fused in, RoPE + KV-cache append +
// grouped-query attention over the f16 cache, SiLU(gate) * up, and the final
// residual add.  The projections are Q4_K matvecs on fused weights (Q|K|V rows
// concatenated, gate|up rows concatenated) served by the matvec kernels.
//
// References (the CPU pieces the decode pipeline composes; the reference's CPU
// backend has no decode_token, crates/larql-compute/src/backend.rs:115-124):
//   rms_norm_eps     crates/larql-inference/src/residual.rs:17-35 (f64 sum of squares,
//                    out = x / rms * (offset + w))
//   apply_rope       crates/larql-inference/src/attention/rope.rs:22-55 (split-half,
//                    f64 inverse frequencies and angles, cos / sin rounded to f32)
//   gqa attention    crates/larql-inference/src/attention/gqa.rs:29-110 (f32 dots
//                    times an f32 scale, exp of (s - max) and its sum in f64)
//   silu_gate_up     crates/larql-inference/src/ffn/mod.rs:87-94
#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kAttnHd = 128;      // head dimension served
constexpr int kAttnChunk = 64;    // keys per CTA (flash-decoding split)

// x += add (if add); h = x / rms(x) * (offset + w), rms in f64 as the reference.
// One CTA of 1024 threads.  For n a multiple of 4 up to 8192 each thread keeps
// its (at most two) float4 groups in registers between the two passes; the norm
// weight, which no earlier kernel writes, is loaded before the dependency wait.
__global__ void __launch_bounds__(1024) decode_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                                              const float* __restrict__ w, float offset, float eps,
                                                              int n, float* __restrict__ h) {
    __shared__ double red[32];
    pdl_launch_dependents();
    const int t = threadIdx.x;
    const bool vec = (n % 4) == 0 && n <= 8 * 1024 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && (reinterpret_cast<uintptr_t>(h) & 15u) == 0 &&
                     (!add || (reinterpret_cast<uintptr_t>(add) & 15u) == 0);
    const int n4 = n / 4;
    float4 wv[2], xv[2];
    if (vec) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = t + u * 1024;
            wv[u] = i < n4 ? reinterpret_cast<const float4*>(w)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    pdl_wait();
    double sq = 0.0;
    if (vec) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = t + u * 1024;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n4) {
                v = reinterpret_cast<const float4*>(x)[i];
                if (add) {
                    const float4 a = reinterpret_cast<const float4*>(add)[i];
                    v.x += a.x;
                    v.y += a.y;
                    v.z += a.z;
                    v.w += a.w;
                    reinterpret_cast<float4*>(x)[i] = v;
                }
            }
            xv[u] = v;
            sq += static_cast<double>(v.x) * static_cast<double>(v.x);
            sq += static_cast<double>(v.y) * static_cast<double>(v.y);
            sq += static_cast<double>(v.z) * static_cast<double>(v.z);
            sq += static_cast<double>(v.w) * static_cast<double>(v.w);
        }
    } else {
        for (int i = t; i < n; i += blockDim.x) {
            float v = x[i];
            if (add) {
                v += add[i];
                x[i] = v;
            }
            sq += static_cast<double>(v) * static_cast<double>(v);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((t & 31) == 0) red[t >> 5] = sq;
    __syncthreads();
    if (t < 32) {
        double v = t < (blockDim.x >> 5) ? red[t] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (t == 0) red[0] = v;
    }
    __syncthreads();
    const float rms = static_cast<float>(sqrt(red[0] / static_cast<double>(n) + static_cast<double>(eps)));
    if (vec) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = t + u * 1024;
            if (i < n4) {
                float4 o;
                o.x = xv[u].x / rms * (offset + wv[u].x);
                o.y = xv[u].y / rms * (offset + wv[u].y);
                o.z = xv[u].z / rms * (offset + wv[u].z);
                o.w = xv[u].w / rms * (offset + wv[u].w);
                reinterpret_cast<float4*>(h)[i] = o;
            }
        }
    } else {
        for (int i = t; i < n; i += blockDim.x) h[i] = x[i] / rms * (offset + w[i]);
    }
}

// act[i] = silu(gate[i]) * up[i] with gu = [gate | up] (f32 sigmoid as ffn/mod.rs:87-94).
__global__ void decode_silu_mul_kernel(const float* __restrict__ gu, int inter, float* __restrict__ act) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < inter) {
        const float g = gu[i];
        act[i] = g * (1.0f / (1.0f + expf(-g))) * gu[inter + i];
    }
}

__global__ void decode_add_kernel(float* __restrict__ x, const float* __restrict__ d, int n) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += d[i];
}

// Attention for one token at position `pos` over keys 0..pos of one layer.
// Grid (n_kv heads, splits); CTA (kvh, s) takes keys [s*64, s*64+64) for the
// REPS query heads of KV head kvh.  qkv = [q (nq*128) | k (nkv*128) | v (nkv*128)]
// before RoPE.  The CTA's K and V rows are loaded into shared memory with every
// load issued up front (K rows padded to an odd number of words so that one
// thread per key reads its row without bank conflicts).  The CTA whose range
// holds key `pos` uses the new k / v from registers and appends them to the f16
// caches.  Partial (max, sum, unnormalised output) per split are combined, in
// split order, by the last CTA of each KV head (atomic ticket, reset for the
// next launch).
constexpr int kAttnKRow = kAttnHd + 2;  // halves per K row in shared memory (65 words: odd)

template <int REPS>
__global__ void __launch_bounds__(128)
    decode_attention_kernel(const float* __restrict__ qkv, int nq, int nkv, int pos, float scale, double rope_base,
                            __half* __restrict__ kc, __half* __restrict__ vc, float* __restrict__ part_o,
                            float* __restrict__ part_m, double* __restrict__ part_l, int* __restrict__ tickets,
                            float* __restrict__ out) {
    __shared__ float qs[REPS][kAttnHd];
    __shared__ float kn[kAttnHd], vn[kAttnHd];
    __shared__ __align__(16) __half ks[kAttnChunk][kAttnKRow];
    __shared__ __align__(16) __half vs[kAttnChunk][kAttnHd];
    __shared__ float sc[REPS][kAttnChunk];
    __shared__ float sm[REPS];
    __shared__ double sl[REPS];
    __shared__ int last;
    const int kvh = blockIdx.x, s = blockIdx.y, S = gridDim.y;
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
    pdl_launch_dependents();
    const int kvd = nkv * kAttnHd;
    const int j0 = s * kAttnChunk, j1 = min(pos + 1, j0 + kAttnChunk), nk = j1 - j0;

    // K / V rows of this split below `pos`, 16 bytes per load, all in flight before
    // the first use.  They are issued before the dependency wait: those rows were
    // written by this layer's attention for earlier tokens, and a kernel that far
    // back in the stream has completed (a token's kernels each wait for their
    // predecessor, and at most a few of them are resident at once).
    constexpr int kLoads = kAttnChunk * kAttnHd * 2 / 16 / 128;  // uint4 loads per thread per matrix
    uint4 kr[kLoads], vr[kLoads];
#pragma unroll
    for (int i = 0; i < kLoads; ++i) {
        const int idx = i * 128 + d, jj = idx >> 4, c = idx & 15;  // 16 uint4 per 128-dim row
        const int j = j0 + jj;
        if (jj < nk && j != pos) {
            const size_t off = static_cast<size_t>(j) * kvd + kvh * kAttnHd + c * 8;
            kr[i] = __ldcs(reinterpret_cast<const uint4*>(kc + off));
            vr[i] = __ldcs(reinterpret_cast<const uint4*>(vc + off));
        } else {
            kr[i] = vr[i] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    pdl_wait();

    // RoPE of this CTA's query heads and of the new key (rope.rs:22-55)
    if (d < kAttnHd / 2) {
        const double inv = 1.0 / pow(rope_base, 2.0 * d / static_cast<double>(kAttnHd));
        double sd, cd;
        sincos(static_cast<double>(pos) * inv, &sd, &cd);
        const float c = static_cast<float>(cd), sn = static_cast<float>(sd);
#pragma unroll
        for (int h = 0; h < REPS; ++h) {
            const float* qh = qkv + (kvh * REPS + h) * kAttnHd;
            const float x0 = qh[d], x1 = qh[d + kAttnHd / 2];
            qs[h][d] = x0 * c - x1 * sn;
            qs[h][d + kAttnHd / 2] = x0 * sn + x1 * c;
        }
        const float* kh = qkv + nq * kAttnHd + kvh * kAttnHd;
        const float x0 = kh[d], x1 = kh[d + kAttnHd / 2];
        kn[d] = x0 * c - x1 * sn;
        kn[d + kAttnHd / 2] = x0 * sn + x1 * c;
    }
    vn[d] = qkv[nq * kAttnHd + kvd + kvh * kAttnHd + d];
#pragma unroll
    for (int i = 0; i < kLoads; ++i) {
        const int idx = i * 128 + d, jj = idx >> 4, c = idx & 15;
        uint32_t* kw = reinterpret_cast<uint32_t*>(&ks[jj][c * 8]);  // 4-byte aligned (odd row stride)
        kw[0] = kr[i].x;
        kw[1] = kr[i].y;
        kw[2] = kr[i].z;
        kw[3] = kr[i].w;
        *reinterpret_cast<uint4*>(&vs[jj][c * 8]) = vr[i];
    }
    __syncthreads();
    const bool holds_new = pos >= j0 && pos < j1;
    if (holds_new) {
        kc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + d] = __float2half_rn(kn[d]);
        vc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + d] = __float2half_rn(vn[d]);
    }

    // scores: thread (key jj = d % 64, heads h = d / 64, d / 64 + 2, ...), f32 dots over 128 dims
    {
        const int jj = d & (kAttnChunk - 1);
        if (jj < nk) {
            const bool is_new = j0 + jj == pos;
            for (int h = d / kAttnChunk; h < REPS; h += 128 / kAttnChunk) {
                float p = 0.f;
                if (is_new) {
                    for (int t = 0; t < kAttnHd; ++t) p = fmaf(qs[h][t], kn[t], p);
                } else {
                    const __half2* kh2 = reinterpret_cast<const __half2*>(&ks[jj][0]);
#pragma unroll 16
                    for (int t = 0; t < kAttnHd / 2; ++t) {
                        const float2 kf = __half22float2(kh2[t]);
                        p = fmaf(qs[h][2 * t], kf.x, p);
                        p = fmaf(qs[h][2 * t + 1], kf.y, p);
                    }
                }
                sc[h][jj] = p * scale;
            }
        }
    }
    __syncthreads();
    // per head: max, exp(s - max) in f64 and its f64 sum (gqa.rs:29-110)
    for (int h = warp; h < REPS; h += 4) {
        float m = -INFINITY;
        for (int jj = lane; jj < nk; jj += 32) m = fmaxf(m, sc[h][jj]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        double l = 0.0;
        for (int jj = lane; jj < nk; jj += 32) {
            const double e = exp(static_cast<double>(sc[h][jj] - m));
            sc[h][jj] = static_cast<float>(e);
            l += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            sm[h] = m;
            sl[h] = l;
        }
    }
    __syncthreads();
    // unnormalised output of this split: thread d owns dimension d of every head
    float acc[REPS];
#pragma unroll
    for (int h = 0; h < REPS; ++h) acc[h] = 0.f;
    for (int jj = 0; jj < nk; ++jj) {
        const float v = j0 + jj == pos ? vn[d] : __half2float(vs[jj][d]);
#pragma unroll
        for (int h = 0; h < REPS; ++h) acc[h] = fmaf(sc[h][jj], v, acc[h]);
    }
    const size_t pb = (static_cast<size_t>(kvh) * S + s) * REPS;
#pragma unroll
    for (int h = 0; h < REPS; ++h) part_o[(pb + h) * kAttnHd + d] = acc[h];
    if (d < REPS) {
        part_m[pb + d] = sm[d];
        part_l[pb + d] = sl[d];
    }
    __threadfence();
    __syncthreads();
    if (d == 0) {
        const int t = atomicAdd(&tickets[kvh], 1);
        last = t == S - 1;
        if (last) tickets[kvh] = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // combine the S splits, one head at a time: thread q < S (in groups of 128) takes
    // split q for the maximum and the weights exp(m_q - M) (f64, as the reference's
    // sum); the f64 sum L is a fixed-shape tree; thread d sums part_o over q in split
    // order with the loads of 8 splits in flight
    __shared__ float fw[128];
    __shared__ double lsum[4];
    for (int h = 0; h < REPS; ++h) {
        float M = -INFINITY;
        for (int q = d; q < S; q += 128) M = fmaxf(M, __ldcg(part_m + (static_cast<size_t>(kvh) * S + q) * REPS + h));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) sc[0][warp] = M;  // sc is free now
        __syncthreads();
        M = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[0][2], sc[0][3]));
        double L = 0.0;
        float o = 0.f;
        for (int q0 = 0; q0 < S; q0 += 128) {
            const int q = q0 + d;
            double lq = 0.0;
            __syncthreads();  // fw of the previous group consumed
            if (q < S) {
                const size_t bq = (static_cast<size_t>(kvh) * S + q) * REPS + h;
                const double f = exp(static_cast<double>(__ldcg(part_m + bq) - M));
                lq = __ldcg(part_l + bq) * f;
                fw[d] = static_cast<float>(f);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) lq += __shfl_xor_sync(0xffffffffu, lq, off);
            if (lane == 0) lsum[warp] = lq;
            __syncthreads();
            L += (lsum[0] + lsum[1]) + (lsum[2] + lsum[3]);
            const int nq_ = min(128, S - q0);
            const float* po = part_o + ((static_cast<size_t>(kvh) * S + q0) * REPS + h) * kAttnHd + d;
            const size_t stride = static_cast<size_t>(REPS) * kAttnHd;
            int i = 0;
            for (; i + 8 <= nq_; i += 8) {
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(po + (i + u) * stride);
#pragma unroll
                for (int u = 0; u < 8; ++u) o = fmaf(v[u], fw[i + u], o);
            }
            for (; i < nq_; ++i) o = fmaf(__ldcg(po + i * stride), fw[i], o);
        }
        out[(kvh * REPS + h) * kAttnHd + d] = o * static_cast<float>(1.0 / L);
        __syncthreads();  // sc[0][*] and fw reused by the next head
    }
}

// ───────────────────────── host launchers ─────────────────────────

size_t decode_attn_scratch_bytes(int nkv, int reps, int max_seq) {
    const size_t S = (static_cast<size_t>(max_seq) + kAttnChunk - 1) / kAttnChunk;
    const size_t parts = static_cast<size_t>(nkv) * S * reps;
    return parts * kAttnHd * sizeof(float) + parts * sizeof(float) + parts * sizeof(double) + 1024;
}

cudaError_t launch_decode_rmsnorm(float* x, const float* add, const float* w, float offset, float eps, int n,
                                  float* h, cudaStream_t stream) {
    cudaError_t e = launch_pdl(decode_rmsnorm_kernel, dim3(1), dim3(1024), 0, stream, x, add, w, offset, eps, n, h);
    note_launch();
    return e;
}

cudaError_t launch_decode_silu_mul(const float* gu, int inter, float* act, cudaStream_t stream) {
    cudaError_t e = launch_pdl(decode_silu_mul_kernel, dim3((inter + 255) / 256), dim3(256), 0, stream, gu, inter, act);
    note_launch();
    return e;
}

cudaError_t launch_decode_add(float* x, const float* d, int n, cudaStream_t stream) {
    cudaError_t e = launch_pdl(decode_add_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, x, d, n);
    note_launch();
    return e;
}

// scratch: decode_attn_scratch_bytes(nkv, nq / nkv, >= pos + 1); tickets: nkv zeroed ints.
cudaError_t launch_decode_attention(const float* qkv, int nq, int nkv, int hd, int pos, float scale,
                                    double rope_base, __half* kc, __half* vc, uint8_t* scratch, int* tickets,
                                    float* out, cudaStream_t stream) {
    if (hd != kAttnHd || nkv < 1 || nq % nkv) return cudaErrorInvalidValue;
    const int reps = nq / nkv;
    const int S = (pos + 1 + kAttnChunk - 1) / kAttnChunk;
    const size_t parts = static_cast<size_t>(nkv) * S * reps;
    float* part_o = reinterpret_cast<float*>(scratch);
    float* part_m = part_o + parts * kAttnHd;
    double* part_l = reinterpret_cast<double*>(reinterpret_cast<uintptr_t>(part_m + parts + 1) & ~uintptr_t(7));
    const dim3 grid(nkv, S);
    cudaError_t e = cudaSuccess;
    switch (reps) {
        case 1: e = launch_pdl(decode_attention_kernel<1>, grid, dim3(kAttnHd), 0, stream, qkv, nq, nkv, pos, scale, rope_base, kc, vc, part_o, part_m, part_l, tickets, out); break;
        case 2: e = launch_pdl(decode_attention_kernel<2>, grid, dim3(kAttnHd), 0, stream, qkv, nq, nkv, pos, scale, rope_base, kc, vc, part_o, part_m, part_l, tickets, out); break;
        case 4: e = launch_pdl(decode_attention_kernel<4>, grid, dim3(kAttnHd), 0, stream, qkv, nq, nkv, pos, scale, rope_base, kc, vc, part_o, part_m, part_l, tickets, out); break;
        case 8: e = launch_pdl(decode_attention_kernel<8>, grid, dim3(kAttnHd), 0, stream, qkv, nq, nkv, pos, scale, rope_base, kc, vc, part_o, part_m, part_l, tickets, out); break;
        default: return cudaErrorInvalidValue;
    }
    note_launch();
    return e;
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, size_t n, __half* __restrict__ out) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[i] = __float2half_rn(in[i]);
}

cudaError_t launch_f32_to_f16(const float* in, size_t n, __half* out, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const size_t b = (n + 255) / 256;
    f32_to_f16_kernel<<<static_cast<unsigned>(b < 4096 ? b : 4096), 256, 0, stream>>>(in, n, out);
    note_launch();
    return cudaGetLastError();
}

}  // namespace larql
