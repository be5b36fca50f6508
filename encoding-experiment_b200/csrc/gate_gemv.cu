// gate_gemv.cu — the vindex gate walk for small query batches (B <= 4) on CUDA cores.
//
// Reference: crates/larql-vindex/src/index/gate.rs:108-134 (gate_knn: f32 scores of the f16 gate rows,
// decoded by crates/larql-models/src/quant/half.rs:4-20, against the residual) and :307-316
// (top_k_from_scores: top-K by |score|, descending).
//
// With one to four queries the tensor-core walk (gate_tc.cu) fills a 128-query MMA tile for a handful of
// rows; here every gate byte is read once by an f32 dot instead.  A CTA takes a contiguous range of one
// layer's rows; a warp reads a whole 2*D-byte row per step (lane l: halves 8 l + 256 i, 16-byte loads, two
// rows in flight), converts to f32 and multiplies with the queries held in shared memory, then reduces over
// the lanes.  Scores (times the registration factor, the same matrix the tensor-core walk reads) go to shared
// memory; at the end one warp per query picks the range's top 16 by |score| (ties by lower index) into the
// candidate layout [layer][query][part][16] that gate_merge_kernel reduces to the top-k.
#include "common.cuh"
#include "kernels.h"

namespace larql {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvKM = 16;  // candidates per (layer, query, part), as the tensor-core walk

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, sizeof(h));
    return __half22float2(h);
}

template <int B>
__global__ void __launch_bounds__(kGvThreads)
    gate_gemv_kernel(const __half* __restrict__ g, const float* __restrict__ q, int F, int D, int P, int rows_pp,
                     float factor, float* __restrict__ cand_s, uint32_t* __restrict__ cand_i) {
    // q and the candidate buffers belong to the kernels before this one until they finish.  No early trigger of
    // the dependent launch: this grid runs in more than one wave, and the merge's CTAs taking residency before the
    // last wave is scheduled cost 14 % at batch 1 (measured)
    pdl_wait();
    extern __shared__ __align__(16) float gsm[];
    float* qs = gsm;                        // [B][D]
    float* sc = gsm + static_cast<size_t>(B) * D;  // [B][rows_pp]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int l = blockIdx.x / P, part = blockIdx.x - l * P;
    const int r0 = part * rows_pp, r1 = min(F, r0 + rows_pp);
    for (int i = threadIdx.x; i < B * D / 4; i += kGvThreads)
        reinterpret_cast<float4*>(qs)[i] = __ldg(reinterpret_cast<const float4*>(q) + i);
    __syncthreads();

    const int nstep = D / 256;  // 16-byte loads per lane per row
    const __half* layer = g + static_cast<size_t>(l) * F * D;
    for (int rb = r0 + warp; rb < r1; rb += 2 * kGvWarps) {
        const int rA = rb, rB = rb + kGvWarps;
        const bool hasB = rB < r1;
        const uint4* pa = reinterpret_cast<const uint4*>(layer + static_cast<size_t>(rA) * D) + lane;
        const uint4* pb = reinterpret_cast<const uint4*>(layer + static_cast<size_t>(hasB ? rB : rA) * D) + lane;
        float accA[B], accB[B];
#pragma unroll
        for (int b = 0; b < B; ++b) accA[b] = accB[b] = 0.f;
        for (int i0 = 0; i0 < nstep; i0 += 5) {
            uint4 wa[5], wb[5];
#pragma unroll
            for (int u = 0; u < 5; ++u) {
                const bool in = i0 + u < nstep;
                wa[u] = in ? __ldg(pa + 32 * (i0 + u)) : make_uint4(0u, 0u, 0u, 0u);
                wb[u] = in && hasB ? __ldg(pb + 32 * (i0 + u)) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 5; ++u) {
                if (i0 + u >= nstep) break;
                const int k0 = (i0 + u) * 256 + lane * 8;
                float ga[8], gb[8];
                const uint32_t wa4[4] = {wa[u].x, wa[u].y, wa[u].z, wa[u].w};
                const uint32_t wb4[4] = {wb[u].x, wb[u].y, wb[u].z, wb[u].w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    const float2 fa = half2_bits_to_float2(wa4[h]);
                    const float2 fb = half2_bits_to_float2(wb4[h]);
                    ga[2 * h] = fa.x;
                    ga[2 * h + 1] = fa.y;
                    gb[2 * h] = fb.x;
                    gb[2 * h + 1] = fb.y;
                }
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4 q0 = *reinterpret_cast<const float4*>(qs + static_cast<size_t>(b) * D + k0);
                    const float4 q1 = *reinterpret_cast<const float4*>(qs + static_cast<size_t>(b) * D + k0 + 4);
                    const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        accA[b] = fmaf(ga[e], qv[e], accA[b]);
                        accB[b] = fmaf(gb[e], qv[e], accB[b]);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                accA[b] += __shfl_xor_sync(0xffffffffu, accA[b], o);
                accB[b] += __shfl_xor_sync(0xffffffffu, accB[b], o);
            }
            if (lane == 0) {
                sc[static_cast<size_t>(b) * rows_pp + (rA - r0)] = accA[b] * factor;
                if (hasB) sc[static_cast<size_t>(b) * rows_pp + (rB - r0)] = accB[b] * factor;
            }
        }
    }
    __syncthreads();

    // top 16 of the range per query: 16 rounds of a warp arg-max over |score| (ties: lower index)
    const int n = r1 - r0;
    for (int b = warp; b < B; b += kGvWarps) {
        float* s = sc + static_cast<size_t>(b) * rows_pp;
        const size_t base = ((static_cast<size_t>(l) * B + b) * P + part) * kGvKM;
        for (int r = 0; r < kGvKM; ++r) {
            uint32_t bk = 0, bi = 0xFFFFFFFFu;  // key: |score| bits + 1 (0 = empty / taken)
            for (int i = lane; i < n; i += 32) {
                const float v = s[i];
                const uint32_t k = (v == v) ? __float_as_uint(fabsf(v)) + 1u : 0u;
                if (k > bk) {
                    bk = k;
                    bi = static_cast<uint32_t>(i);
                }
            }
            const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
            const uint32_t mi = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xFFFFFFFFu);
            float mv = 0.f;
            if (mk != 0 && lane == 0) {
                mv = s[mi];
                s[mi] = __int_as_float(0x7fc00000);  // taken
            }
            __syncwarp();
            if (lane == 0) {
                cand_s[base + r] = mk ? mv : 0.f;
                cand_i[base + r] = mk ? static_cast<uint32_t>(r0) + mi : 0xFFFFFFFFu;
            }
        }
    }
}

// The Q4_0 gate walk's selection step (gate.rs:714-731 gate_knn_q4 -> top_k_from_scores, :307-316): scores
// [B][L][F] (one Q4_0 x Q8 matvec per query over every layer's rows) -> the top 16 by |score| (ties: lower index)
// of each (layer, query, part) range, in the candidate layout gate_merge_kernel reduces.  One CTA per range:
// the range's scores are staged in shared memory and one warp takes 16 rounds of arg-max.
__global__ void __launch_bounds__(kGvThreads)
    gate_score_cand_kernel(const float* __restrict__ scores, int L, int F, int P, int rows_pp,
                           float* __restrict__ cand_s, uint32_t* __restrict__ cand_i) {
    pdl_wait();  // the scores belong to the kernel before this one until it finishes (no early trigger: several waves)
    extern __shared__ __align__(16) float cs_sm[];  // [rows_pp]
    const int l = blockIdx.x / P, part = blockIdx.x - l * P, b = blockIdx.y, B = gridDim.y;
    const int r0 = part * rows_pp, r1 = min(F, r0 + rows_pp), n = max(0, r1 - r0);
    const float* src = scores + (static_cast<size_t>(b) * L + l) * F + r0;
    for (int i = threadIdx.x; i < n; i += kGvThreads) cs_sm[i] = __ldg(src + i);
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const size_t base = ((static_cast<size_t>(l) * B + b) * P + part) * kGvKM;
    for (int r = 0; r < kGvKM; ++r) {
        uint32_t bk = 0, bi = 0xFFFFFFFFu;  // key: |score| bits + 1 (0 = empty / taken)
        for (int i = lane; i < n; i += 32) {
            const float v = cs_sm[i];
            const uint32_t k = (v == v) ? __float_as_uint(fabsf(v)) + 1u : 0u;
            if (k > bk) {
                bk = k;
                bi = static_cast<uint32_t>(i);
            }
        }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t mi = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xFFFFFFFFu);
        float mv = 0.f;
        if (mk != 0 && lane == 0) {
            mv = cs_sm[mi];
            cs_sm[mi] = __int_as_float(0x7fc00000);  // taken
        }
        __syncwarp();
        if (lane == 0) {
            cand_s[base + r] = mk ? mv : 0.f;
            cand_i[base + r] = mk ? static_cast<uint32_t>(r0) + mi : 0xFFFFFFFFu;
        }
    }
}

int gate_score_cand_parts(int L, int F, int B, int num_sms) {
    int parts = (4 * num_sms + L * B - 1) / (L * B);
    parts = parts < 1 ? 1 : (parts > 32 ? 32 : parts);
    return parts > F ? F : parts;
}

cudaError_t launch_gate_score_topk(const float* scores, int L, int F, int B, int k, int parts, float* cand_s,
                                   uint32_t* cand_i, uint32_t* out_i, float* out_s, cudaStream_t stream) {
    if (k < 1 || k > kGvKM || parts < 1 || parts > 32 || B < 1 || B > 65535 || L < 1 || F < 1)
        return cudaErrorInvalidValue;
    const int rows_pp = (F + parts - 1) / parts;
    const size_t smem = static_cast<size_t>(rows_pp) * sizeof(float);
    if (smem > static_cast<size_t>(kSmemLimit)) return cudaErrorInvalidValue;
    static DeviceFlags attr_done;
    cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(gate_score_cand_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    e = launch_pdl(gate_score_cand_kernel, dim3(L * parts, B), dim3(kGvThreads), smem, stream, scores, L, F, parts,
                   rows_pp, cand_s, cand_i);
    note_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_gate_merge(cand_s, cand_i, L, B, parts, k, out_i, out_s, stream);
}

bool gate_gemv_ok(int D, int B) { return B >= 1 && B <= 4 && D % 256 == 0 && D <= 8192; }

int gate_gemv_parts(int L, int F, int num_sms) {
    int parts = (2 * num_sms + L - 1) / L;
    parts = parts < 1 ? 1 : (parts > 32 ? 32 : parts);
    return parts > F ? F : parts;
}

template <int B>
static cudaError_t launch_gemv_b(const __half* g, const float* q, int L, int F, int D, int parts, int rows_pp,
                                 size_t smem, float factor, float* cand_s, uint32_t* cand_i, cudaStream_t stream) {
    static DeviceFlags attr_done;
    cudaError_t e = once_per_device(attr_done, [] {
        return cudaFuncSetAttribute(gate_gemv_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    });
    if (e != cudaSuccess) return e;
    e = launch_pdl(gate_gemv_kernel<B>, dim3(L * parts), dim3(kGvThreads), smem, stream, g, q, F, D, parts, rows_pp,
                   factor, cand_s, cand_i);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
}

// candidates: L * B * parts * 16 of (float, u32) in cand_s / cand_i; then the merge to the top-k.
cudaError_t launch_gate_gemv(const __half* g, float factor, const float* q, int L, int F, int D, int B, int k,
                             int parts, float* cand_s, uint32_t* cand_i, uint32_t* out_i, float* out_s,
                             cudaStream_t stream) {
    if (!gate_gemv_ok(D, B) || k < 1 || k > kGvKM || parts < 1 || parts > 32) return cudaErrorInvalidValue;
    const int rows_pp = (F + parts - 1) / parts;
    const size_t smem = (static_cast<size_t>(B) * D + static_cast<size_t>(B) * rows_pp) * sizeof(float);
    if (smem > static_cast<size_t>(kSmemLimit)) return cudaErrorInvalidValue;
    cudaError_t e;
    switch (B) {
        case 1: e = launch_gemv_b<1>(g, q, L, F, D, parts, rows_pp, smem, factor, cand_s, cand_i, stream); break;
        case 2: e = launch_gemv_b<2>(g, q, L, F, D, parts, rows_pp, smem, factor, cand_s, cand_i, stream); break;
        case 3: e = launch_gemv_b<3>(g, q, L, F, D, parts, rows_pp, smem, factor, cand_s, cand_i, stream); break;
        default: e = launch_gemv_b<4>(g, q, L, F, D, parts, rows_pp, smem, factor, cand_s, cand_i, stream); break;
    }
    if (e != cudaSuccess) return e;
    return launch_gate_merge(cand_s, cand_i, L, B, parts, k, out_i, out_s, stream);
}

}  // namespace larql
