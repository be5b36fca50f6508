// vecmat.cu — Q4_0 vector-matrix product out[hidden] = act[inter] @ Q4_0[inter, hidden]
// (ComputeBackend::q4_vecmat, crates/larql-compute/src/backend.rs:56-60; CPU reference
// crates/larql-compute/csrc/q4_dot.c:201-232, reached through cpu/ops/q4_vecmat.rs:8-17).
//
// The reference scatters every row into the output: per 32-value block, scale = f16(d) * act[row] and
// out[col] += (q - 8) * scale, skipping rows with -1e-10 < act < 1e-10 (their weights are never read, so a
// non-finite weight there does not reach the output).  The weight is row-major, so the reduction runs over
// rows: a CTA takes one group of 32 blocks (1024 columns) of a contiguous range of rows; lane l of each warp
// owns block l of the group for the whole kernel (32 f32 accumulators), so a warp reads one row's 576-byte
// slice per step, coalesced.  Weight loads do not wait for the activation (kVmUnroll rows of them are in
// flight per warp); a skipped row's loaded bytes are simply not used.  Nibbles become floats exactly through the
// 2^23 magic number (bits 0x4B000000 | q = 8388608 + q; minus 8388616 gives q - 8).  The 8 warps of a CTA
// are summed in warp order through shared memory; row ranges are summed in range order by a second kernel,
// so results do not depend on scheduling.
#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kVmThreads = 256;
constexpr int kVmWarps = kVmThreads / 32;
constexpr int kVmUnroll = 8;  // rows in flight per warp

// ALIGN4: row starts are 4-byte aligned (hidden % 64 == 0): a block's 18 bytes come from 5 aligned words
// (the last may reach 2 bytes into the next block or the allocation's slack) and funnel shifts; otherwise 9
// 2-byte loads.
template <bool ALIGN4>
__global__ void __launch_bounds__(kVmThreads)
    q4_vecmat_kernel(const float* __restrict__ act, const uint8_t* __restrict__ w, int inter, int hidden,
                     int ngroups, int rows_per_range, float* __restrict__ dst) {
    __shared__ float red[kVmWarps * 32 * 33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cg = blockIdx.x % ngroups, rg = blockIdx.x / ngroups;
    const int nb = hidden / 32;
    const int b = cg * 32 + lane;
    const bool col_ok = b < nb;
    const size_t bpr = static_cast<size_t>(nb) * 18;
    const int r0 = rg * rows_per_range, r1 = min(inter, r0 + rows_per_range);
    pdl_launch_dependents();

    float o[32];
#pragma unroll
    for (int v = 0; v < 32; ++v) o[v] = 0.f;

    for (int rb = r0 + warp; rb < r1; rb += kVmWarps * kVmUnroll) {
        // raw[u]: the block's 18 bytes as 5 words from its first byte (ALIGN4), or 9 half-words
        uint32_t raw[kVmUnroll][9];
        float a[kVmUnroll];
        bool live[kVmUnroll];
#pragma unroll
        for (int u = 0; u < kVmUnroll; ++u) {
            const int r = rb + u * kVmWarps;
            live[u] = r < r1 && col_ok;
            a[u] = r < r1 ? __ldg(act + r) : 0.f;
            const uint8_t* p = w + static_cast<size_t>(r) * bpr + b * 18;
            if constexpr (ALIGN4) {
                const uint32_t* q = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
#pragma unroll
                for (int i = 0; i < 5; ++i) raw[u][i] = live[u] ? __ldg(q + i) : 0u;
            } else {
                const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
                for (int i = 0; i < 9; ++i) raw[u][i] = live[u] ? __ldg(q + i) : 0u;
            }
        }
        const uint32_t sh = ALIGN4 ? 8u * ((static_cast<uint32_t>(b) * 18u) & 3u) : 0u;
#pragma unroll
        for (int u = 0; u < kVmUnroll; ++u) {
            if (!live[u] || (a[u] > -1e-10f && a[u] < 1e-10f)) continue;
            // d in bits 0..15 of word 0; quant bytes 2i, 2i+1 (values 4i .. 4i+3) in 16-bit piece i
            uint32_t d16, qw[4];  // qw[k]: quant bytes 4k .. 4k+3
            if constexpr (ALIGN4) {
                uint32_t t[5];
#pragma unroll
                for (int i = 0; i < 4; ++i) t[i] = __funnelshift_r(raw[u][i], raw[u][i + 1], sh);
                t[4] = raw[u][4] >> sh;
                d16 = t[0] & 0xFFFFu;
#pragma unroll
                for (int k = 0; k < 4; ++k) qw[k] = __funnelshift_r(t[k], t[k + 1], 16);
            } else {
                d16 = raw[u][0];
#pragma unroll
                for (int k = 0; k < 4; ++k) qw[k] = raw[u][1 + 2 * k] | (raw[u][2 + 2 * k] << 16);
            }
            const float scale = __fmul_rn(__half2float(__ushort_as_half(static_cast<unsigned short>(d16))), a[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const float f = __int_as_float(0x4B000000 | ((qw[k] >> (4 * n)) & 0xFu)) - 8388616.0f;
                    o[8 * k + n] = fmaf(f, scale, o[8 * k + n]);
                }
        }
    }

#pragma unroll
    for (int v = 0; v < 32; ++v) red[(warp * 32 + lane) * 33 + v] = o[v];
    __syncthreads();
    for (int c = threadIdx.x; c < 1024; c += kVmThreads) {
        const int l = c >> 5, v = c & 31;
        const int col = (cg * 32 + l) * 32 + v;
        if (col >= hidden) continue;
        float s = 0.f;
#pragma unroll
        for (int ww = 0; ww < kVmWarps; ++ww) s += red[(ww * 32 + l) * 33 + v];
        dst[static_cast<size_t>(rg) * hidden + col] = s;
    }
}

// out[col] = sum over row ranges, in range order.
__global__ void q4_vecmat_reduce_kernel(const float* __restrict__ part, int nranges, int hidden,
                                        float* __restrict__ out) {
    pdl_wait();
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= hidden) return;
    float s = 0.f;
    for (int g = 0; g < nranges; ++g) s += part[static_cast<size_t>(g) * hidden + col];
    out[col] = s;
}

VecmatPlan q4_vecmat_plan(int inter, int hidden, int num_sms) {
    VecmatPlan p{};
    p.ngroups = (hidden / 32 + 31) / 32;
    // about two CTAs per SM, each with at least 64 rows
    const int want = max(1, 2 * num_sms / p.ngroups);
    p.nranges = max(1, min(want, (inter + 63) / 64));
    p.rows_per_range = (inter + p.nranges - 1) / p.nranges;
    p.nranges = (inter + p.rows_per_range - 1) / p.rows_per_range;
    return p;
}

size_t q4_vecmat_part_floats(const VecmatPlan& p, int hidden) {
    return p.nranges > 1 ? static_cast<size_t>(p.nranges) * hidden : 0;
}

cudaError_t launch_q4_vecmat(const float* act, const uint8_t* w, int inter, int hidden, const VecmatPlan& p,
                             float* part, float* out, cudaStream_t stream) {
    if (hidden <= 0 || hidden % 32 || inter < 0) return cudaErrorInvalidValue;
    if (inter == 0) return cudaMemsetAsync(out, 0, static_cast<size_t>(hidden) * sizeof(float), stream);
    const bool split = p.nranges > 1;
    const bool align4 = hidden % 64 == 0 && (reinterpret_cast<uintptr_t>(w) & 3) == 0;
    if (align4)
        q4_vecmat_kernel<true><<<p.ngroups * p.nranges, kVmThreads, 0, stream>>>(act, w, inter, hidden, p.ngroups,
                                                                                 p.rows_per_range, split ? part : out);
    else
        q4_vecmat_kernel<false><<<p.ngroups * p.nranges, kVmThreads, 0, stream>>>(act, w, inter, hidden, p.ngroups,
                                                                                  p.rows_per_range, split ? part : out);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !split) return e;
    e = launch_pdl(q4_vecmat_reduce_kernel, dim3((hidden + 255) / 256), dim3(256), 0, stream,
                   static_cast<const float*>(part), p.nranges, hidden, out);
    note_launch();
    return e;
}

}  // namespace larql
