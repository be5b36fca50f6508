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
constexpr int kAttnChunk = 128;   // keys per CTA (flash-decoding split)

// x += add (if add); h = x / rms(x) * (offset + w), rms in f64 as the reference.
__global__ void decode_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                      const float* __restrict__ w, float offset, float eps, int n,
                                      float* __restrict__ h) {
    __shared__ double red[32];
    pdl_launch_dependents();
    pdl_wait();
    double sq = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (add) {
            v += add[i];
            x[i] = v;
        }
        sq += static_cast<double>(v) * static_cast<double>(v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float rms = static_cast<float>(sqrt(red[0] / static_cast<double>(n) + static_cast<double>(eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) h[i] = x[i] / rms * (offset + w[i]);
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
// Grid (n_kv heads, splits); CTA (kvh, s) takes keys [s*128, s*128+128) for the
// REPS query heads of KV head kvh.  qkv = [q (nq*128) | k (nkv*128) | v (nkv*128)]
// before RoPE.  The CTA whose range holds key `pos` uses the new k / v from
// registers and appends them to the f16 caches.  Partial (max, sum, unnormalised
// output) per split are combined, in split order, by the last CTA of each KV
// head (atomic ticket, reset for the next launch).
template <int REPS>
__global__ void __launch_bounds__(128)
    decode_attention_kernel(const float* __restrict__ qkv, int nq, int nkv, int pos, float scale, double rope_base,
                            __half* __restrict__ kc, __half* __restrict__ vc, float* __restrict__ part_o,
                            float* __restrict__ part_m, double* __restrict__ part_l, int* __restrict__ tickets,
                            float* __restrict__ out) {
    __shared__ float qs[REPS][kAttnHd];
    __shared__ float kn[kAttnHd], vn[kAttnHd];
    __shared__ float sc[REPS][kAttnChunk];
    __shared__ float sm[REPS];
    __shared__ double sl[REPS];
    __shared__ int last;
    const int kvh = blockIdx.x, s = blockIdx.y, S = gridDim.y;
    const int d = threadIdx.x, warp = d >> 5, lane = d & 31;
    pdl_launch_dependents();
    pdl_wait();
    const int kvd = nkv * kAttnHd;
    const int j0 = s * kAttnChunk, j1 = min(pos + 1, j0 + kAttnChunk), nk = j1 - j0;

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
    __syncthreads();
    const bool holds_new = pos >= j0 && pos < j1;
    if (holds_new) {
        kc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + d] = __float2half_rn(kn[d]);
        vc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + d] = __float2half_rn(vn[d]);
    }

    // scores: a warp per key, 4 dims per lane
    for (int jj = warp; jj < nk; jj += 4) {
        const int j = j0 + jj;
        float k4[4];
        if (j == pos) {
#pragma unroll
            for (int t = 0; t < 4; ++t) k4[t] = kn[4 * lane + t];
        } else {
            const uint2 raw = *reinterpret_cast<const uint2*>(kc + static_cast<size_t>(j) * kvd + kvh * kAttnHd + 4 * lane);
            const __half2 a = *reinterpret_cast<const __half2*>(&raw.x), b = *reinterpret_cast<const __half2*>(&raw.y);
            k4[0] = __low2float(a);
            k4[1] = __high2float(a);
            k4[2] = __low2float(b);
            k4[3] = __high2float(b);
        }
#pragma unroll
        for (int h = 0; h < REPS; ++h) {
            float p = 0.f;
#pragma unroll
            for (int t = 0; t < 4; ++t) p = fmaf(qs[h][4 * lane + t], k4[t], p);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
            if (lane == 0) sc[h][jj] = p * scale;
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
        const int j = j0 + jj;
        const float v = j == pos ? vn[d] : __half2float(vc[static_cast<size_t>(j) * kvd + kvh * kAttnHd + d]);
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
#pragma unroll
    for (int h = 0; h < REPS; ++h) {
        float M = -INFINITY;
        for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(part_m + (static_cast<size_t>(kvh) * S + q) * REPS + h));
        double L = 0.0;
        float o = 0.f;
        for (int q = 0; q < S; ++q) {
            const size_t b = (static_cast<size_t>(kvh) * S + q) * REPS + h;
            const double f = exp(static_cast<double>(__ldcg(part_m + b) - M));
            L += __ldcg(part_l + b) * f;
            o = fmaf(__ldcg(part_o + b * kAttnHd + d), static_cast<float>(f), o);
        }
        out[(kvh * REPS + h) * kAttnHd + d] = o * static_cast<float>(1.0 / L);
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
