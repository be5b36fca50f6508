// quantize.cu — device-side weight quantizers, bit-identical to the
// reference's CPU quantizers so weights can be produced or converted on the
// GPU at load time.  All float steps use explicit round-to-nearest intrinsics
// (no contraction into FMA), f32::round semantics (roundf: half away from
// zero) and Rust's saturating `as u8` casts.
#include "common.cuh"
#include "kernels.h"

namespace larql {

// crates/larql-compute/src/cpu/ops/q4_common.rs:83-94 (truncating f32 -> f16).
__device__ __forceinline__ uint16_t f32_to_f16_trunc(float v) {
    const uint32_t bits = __float_as_uint(v);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int exp = static_cast<int>((bits >> 23) & 0xFF);
    const uint32_t mant = bits & 0x7FFFFFu;
    if (exp == 0) return static_cast<uint16_t>(sign);
    if (exp == 255) return static_cast<uint16_t>(sign | 0x7C00u | (mant >> 13));
    const int ne = exp - 127 + 15;
    if (ne >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
    if (ne <= 0) return static_cast<uint16_t>(sign);
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(ne) << 10) | (mant >> 13));
}

// Rust `f.round().clamp(lo, hi) as u8` (clamp keeps NaN; `as u8` maps NaN to 0).
__device__ __forceinline__ uint32_t round_clamp_u8(float v, float lo, float hi) {
    float r = roundf(v);
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    if (!(r > 0.0f)) return 0u;  // NaN or <= 0
    return static_cast<uint32_t>(r);
}

// LARQL Q4_K, 148 B per 256 values (q4_common.rs:104-170).  One warp per
// super-block; lane l holds values 8l..8l+7 (sub-block j = l / 4).
__global__ void quantize_q4_k_kernel(const float* __restrict__ data, uint8_t* __restrict__ out, size_t nsb) {
    const size_t sb = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (sb >= nsb) return;
    const float4* src = reinterpret_cast<const float4*>(data + sb * 256 + lane * 8);
    const float4 f0 = src[0], f1 = src[1];
    const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) { mn = fminf(mn, v[i]); mx = fmaxf(mx, v[i]); }
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float range = __fsub_rn(mx, mn);  // this lane's sub-block range
    float gmr = fmaxf(0.0f, range), gmin = mn;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        gmr = fmaxf(gmr, __shfl_xor_sync(0xffffffffu, gmr, o));
        gmin = fminf(gmin, __shfl_xor_sync(0xffffffffu, gmin, o));
    }
    const float d = gmr > 0.0f ? __fdiv_rn(gmr, 63.0f) : 0.0f;
    const float dmin = gmin < 0.0f ? __fdiv_rn(-gmin, 15.0f) : 0.0f;
    const uint32_t qs = d > 0.0f ? round_clamp_u8(__fdiv_rn(range, d), 0.0f, 63.0f) : 0u;
    const uint32_t qm = dmin > 0.0f ? round_clamp_u8(__fdiv_rn(-mn, dmin), 0.0f, 15.0f) : 0u;

    const float sc = __fmul_rn(d, static_cast<float>(qs));
    const float mnv = __fmul_rn(dmin, static_cast<float>(qm));
    const float inv = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = round_clamp_u8(__fmul_rn(__fadd_rn(v[2 * i], mnv), inv), 0.0f, 15.0f);
        const uint32_t hi = round_clamp_u8(__fmul_rn(__fadd_rn(v[2 * i + 1], mnv), inv), 0.0f, 15.0f);
        word |= (lo | (hi << 4)) << (8 * i);
    }
    uint8_t* ob = out + sb * 148;
    const int j = lane >> 2;
    *reinterpret_cast<uint32_t*>(ob + 20 + 16 * j + 4 * (lane & 3)) = word;

    // header: gather the 8 (scale, min) pairs from lanes 0, 4, ..., 28
    uint32_t sw0 = 0, sw1 = 0, mw = 0;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
        const uint32_t s = __shfl_sync(0xffffffffu, qs, jj * 4) & 0x3Fu;
        const uint32_t m = __shfl_sync(0xffffffffu, qm, jj * 4) & 0x0Fu;
        if (jj < 4) { sw0 |= s << (8 * jj); mw |= m << (8 * jj); }
        else { sw1 |= s << (8 * (jj - 4)); mw |= m << (8 * (jj - 4) + 4); }
    }
    uint32_t* hw = reinterpret_cast<uint32_t*>(ob);
    if (lane == 0) hw[0] = static_cast<uint32_t>(f32_to_f16_trunc(d)) | (static_cast<uint32_t>(f32_to_f16_trunc(dmin)) << 16);
    if (lane == 1) hw[1] = sw0;
    if (lane == 2) hw[2] = sw1;
    if (lane == 3) hw[3] = 0u;
    if (lane == 4) hw[4] = mw;
}

// Rust `(v).round() as i32` clamped to [lo, hi] (NaN -> 0 before the clamp).
__device__ __forceinline__ int round_as_i32_clamped(float v, int lo, int hi) {
    float r = roundf(v);
    if (!(r == r)) r = 0.0f;
    r = fminf(fmaxf(r, static_cast<float>(lo)), static_cast<float>(hi));
    return static_cast<int>(r);
}

// 32-value block formats, one warp per block, lane l holding value l:
//   FMT 0  Q4_0 (q4_common.rs:50-80; ggml.rs:310-337): f16 scale = amax/7 (truncating), nibble =
//          (round(v/scale) as i32 + 8).clamp(0, 15), byte j = elem 2j | elem 2j+1 << 4; 18 B.
//   FMT 1  GGUF Q8_0 (ggml.rs:342-363): f16 scale = amax/127 (half.rs:28-41, truncating),
//          int8 = round(v/scale).clamp(-128, 127); 34 B.
// amax folds |v| with f32::max from 0 (NaN values are skipped); inv = 1/scale or 0.
template <int FMT>
__global__ void quantize_block32_kernel(const float* __restrict__ data, uint8_t* __restrict__ out, size_t nb) {
    const size_t b = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (b >= nb) return;
    const float v = data[b * 32 + lane];
    float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = __fdiv_rn(amax, FMT == 0 ? 7.0f : 127.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    const float t = __fmul_rn(v, inv);
    constexpr int kBytes = FMT == 0 ? 18 : 34;
    uint8_t* ob = out + b * kBytes;
    if (lane == 0) {
        const uint16_t h = f32_to_f16_trunc(scale);
        ob[0] = static_cast<uint8_t>(h & 0xFF);
        ob[1] = static_cast<uint8_t>(h >> 8);
    }
    if (FMT == 0) {
        const int q = round_as_i32_clamped(t, -8, 7) + 8;
        const int qn = __shfl_down_sync(0xffffffffu, q, 1);
        if ((lane & 1) == 0) ob[2 + (lane >> 1)] = static_cast<uint8_t>(q | (qn << 4));
    } else {
        ob[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(round_as_i32_clamped(t, -128, 127)));
    }
}

// LARQL Q6_K, 210 B per 256 values (q4_common.rs:179-239).  One warp per super-block; lane l holds values
// 8l..8l+7 (sub-block l / 2).  d = amax / 32 (truncating f16 on store, the f32 d for quantizing); per 16 values
// sc = round(smax / d) as i8; q = round(v / (d * sc)) clamped to [-32, 31], stored biased by 32.
__global__ void quantize_q6_k_kernel(const float* __restrict__ data, uint8_t* __restrict__ out, size_t nsb) {
    const size_t sb = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (sb >= nsb) return;
    const float4* src = reinterpret_cast<const float4*>(data + sb * 256 + lane * 8);
    const float4 f0 = src[0], f1 = src[1];
    const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
    float smax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) smax = fmaxf(smax, fabsf(v[i]));
    smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 1));
    float amax = smax;
#pragma unroll
    for (int o = 2; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 32.0f);
    const int ss = round_as_i32_clamped(d > 0.0f ? __fdiv_rn(smax, d) : 0.0f, -128, 127);
    const float sc = __fmul_rn(d, static_cast<float>(ss));
    const float inv = fabsf(sc) > 1e-10f ? __fdiv_rn(1.0f, sc) : 0.0f;
    uint32_t q6[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q6[i] = static_cast<uint32_t>(round_as_i32_clamped(__fmul_rn(v[i], inv), -32, 31) + 32);
    uint8_t* ob = out + sb * 210;  // 2-byte aligned: byte stores
#pragma unroll
    for (int i = 0; i < 4; ++i) ob[4 * lane + i] = static_cast<uint8_t>((q6[2 * i] & 0x0F) | ((q6[2 * i + 1] & 0x0F) << 4));
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t b = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) b |= ((q6[4 * h + i] >> 4) & 0x03u) << (2 * i);
        ob[128 + 2 * lane + h] = static_cast<uint8_t>(b);
    }
    if ((lane & 1) == 0) ob[192 + (lane >> 1)] = static_cast<uint8_t>(static_cast<int8_t>(ss));
    if (lane == 0) {
        const uint16_t hd = f32_to_f16_trunc(d);
        ob[208] = static_cast<uint8_t>(hd & 0xFF);
        ob[209] = static_cast<uint8_t>(hd >> 8);
    }
}

cudaError_t launch_quantize_q6_k(const float* data, size_t n, uint8_t* out, cudaStream_t stream) {
    const size_t nsb = n / 256;
    if (nsb == 0) return cudaSuccess;
    const size_t blocks = (nsb + 7) / 8;
    quantize_q6_k_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(data, out, nsb);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize_block32(int fmt, const float* data, size_t n, uint8_t* out, cudaStream_t stream) {
    const size_t nb = n / 32;
    if (nb == 0) return cudaSuccess;
    const unsigned blocks = static_cast<unsigned>((nb + 7) / 8);
    if (fmt == 0)
        quantize_block32_kernel<0><<<blocks, 256, 0, stream>>>(data, out, nb);
    else
        quantize_block32_kernel<1><<<blocks, 256, 0, stream>>>(data, out, nb);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_quantize_q4_k(const float* data, size_t n, uint8_t* out, cudaStream_t stream) {
    const size_t nsb = n / 256;
    if (nsb == 0) return cudaSuccess;
    const int wpb = 8;
    const size_t blocks = (nsb + wpb - 1) / wpb;
    quantize_q4_k_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, stream>>>(data, out, nsb);
    note_launch();
    return cudaGetLastError();
}

}  // namespace larql
