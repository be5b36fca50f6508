// vecmat.cu — Q4_0 vector-matrix product out[hidden] = act[inter] @ Q4_0[inter, hidden]
// (ComputeBackend::q4_vecmat, crates/larql-compute/src/backend.rs:56-60; CPU reference
// crates/larql-compute/csrc/q4_dot.c:201-232, reached through cpu/ops/q4_vecmat.rs:8-17).
//
// The reference scatters every row into the output: per 32-value block, scale = f16(d) * act[row] and
// out[col] += (q - 8) * scale, skipping rows with -1e-10 < act < 1e-10 (their weights are never read, so a
// non-finite weight there does not reach the output).  The weight is row-major, so the reduction runs over
// rows: a CTA takes one group of 32 blocks (1024 columns) of a contiguous range of rows; lane l of each warp
// owns block l of the group for the whole kernel (32 f32 accumulators), so a warp reads one row's 576-byte
// slice per step, coalesced.  Skipped rows are not loaded.  Nibbles become floats exactly through the
// 2^23 magic number (bits 0x4B000000 | q = 8388608 + q; minus 8388616 gives q - 8).  The 8 warps of a CTA
// are summed in warp order through shared memory; row ranges are summed in range order by a second kernel,
// so results do not depend on scheduling.
#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kVmThreads = 256;
constexpr int kVmWarps = kVmThreads / 32;
constexpr int kVmUnroll = 4;  // rows in flight per warp

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
        uint32_t h[kVmUnroll][9];
        float a[kVmUnroll];
        bool use[kVmUnroll];
#pragma unroll
        for (int u = 0; u < kVmUnroll; ++u) {
            const int r = rb + u * kVmWarps;
            a[u] = r < r1 ? __ldg(act + r) : 0.f;
            use[u] = r < r1 && !(a[u] > -1e-10f && a[u] < 1e-10f) && col_ok;
            const uint16_t* p = reinterpret_cast<const uint16_t*>(w + static_cast<size_t>(r) * bpr + b * 18);
#pragma unroll
            for (int i = 0; i < 9; ++i) h[u][i] = use[u] ? __ldg(p + i) : 0u;
        }
#pragma unroll
        for (int u = 0; u < kVmUnroll; ++u) {
            if (!use[u]) continue;
            const float scale = __fmul_rn(__half2float(__ushort_as_half(static_cast<unsigned short>(h[u][0]))), a[u]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t q = h[u][1 + i];  // bytes 2i, 2i+1 = values 4i .. 4i+3
#pragma unroll
                for (int n = 0; n < 4; ++n) {
                    const float f = __int_as_float(0x4B000000 | ((q >> (4 * n)) & 0xFu)) - 8388616.0f;
                    o[4 * i + n] = fmaf(f, scale, o[4 * i + n]);
                }
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
    q4_vecmat_kernel<<<p.ngroups * p.nranges, kVmThreads, 0, stream>>>(act, w, inter, hidden, p.ngroups,
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
