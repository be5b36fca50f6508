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

// ss[g] = sum of x[16g .. 16g + 15]^2 in f64: the sums of squares the first norm-fused matvec of a token
// reads (later ones come from the residual epilogue of the matvec before them).
__global__ void decode_sumsq16_kernel(const float* __restrict__ x, int n, double* __restrict__ ss) {
    pdl_launch_dependents();
    pdl_wait();
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (16 * g >= n) return;
    double s = 0.0;
    for (int i = 16 * g; i < min(n, 16 * g + 16); ++i) s += static_cast<double>(x[i]) * static_cast<double>(x[i]);
    ss[g] = s;
}

cudaError_t launch_decode_sumsq16(const float* x, int n, double* ss, cudaStream_t stream) {
    const int ng = (n + 15) / 16;
    cudaError_t e = launch_pdl(decode_sumsq16_kernel, dim3((ng + 127) / 128), dim3(128), 0, stream, x, n, ss);
    note_launch();
    return e;
}

__global__ void decode_add_kernel(float* __restrict__ x, const float* __restrict__ d, int n) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += d[i];
}

// Attention for one token at position `pos` over keys 0..pos of one layer.
// One thread-block cluster of C CTAs per KV head (grid (n_kv heads, C)); CTA r of
// the cluster takes keys [r*kpc, (r+1)*kpc), kpc = ceil((pos+1) / C), for the REPS
// query heads of its KV head, in sub-chunks of up to 256 keys staged in shared
// memory by cp.async (K rows with their 16-byte chunks XOR-swizzled by key & 7,
// so one thread per key reads its row without bank conflicts).  Within a CTA the
// softmax is online (running max, f64 running sum, rescaled accumulators).  The
// CTAs then combine through distributed shared memory: CTA r finalises its share
// of the REPS * 128 outputs from every CTA's (max, sum, accumulator), in rank
// order.  qkv = [q (nq*128) | k (nkv*128) | v (nkv*128)] before RoPE; the CTA
// whose range holds key `pos` uses the new k / v in f32 and appends them to the
// f16 caches.
constexpr int kAtThreads = 256;
constexpr int kAtSub = 160;                              // keys per shared-memory sub-chunk (two CTAs per SM)
constexpr int kAtRow = kAttnHd * 2;                      // bytes per K / V row
constexpr int kAtSmem = 2 * kAtSub * kAtRow;             // dynamic shared memory: K then V

__device__ __forceinline__ uint32_t at_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t at_mapa(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
// Remote shared-memory loads, issued after a cluster barrier; not volatile, so the
// compiler may batch them.
__device__ __forceinline__ float at_ld_f32(uint32_t a) {
    float v;
    asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ double at_ld_f64(uint32_t a) {
    double v;
    asm("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void at_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void at_cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

template <int REPS>
__global__ void __launch_bounds__(kAtThreads)
    decode_attention_kernel(const float* __restrict__ qkv, int nq, int nkv, int pos, float scale, double rope_base,
                            __half* __restrict__ kc, __half* __restrict__ vc, float* __restrict__ out) {
    extern __shared__ __align__(1024) uint8_t at_smem[];
    uint8_t* ks = at_smem;                  // [kAtSub][256 B], 16-byte chunk c of key j at c ^ (j & 7)
    uint8_t* vs = at_smem + kAtSub * kAtRow;  // [kAtSub][256 B]
    __shared__ float qs[REPS][kAttnHd];
    __shared__ float kn[kAttnHd], vn[kAttnHd];
    __shared__ float sc[REPS][kAtSub];
    __shared__ float cm[REPS], corr[REPS];  // running max, rescale of the current sub-chunk
    __shared__ double cl[REPS];             // running f64 sum
    __shared__ float co[REPS][kAttnHd];     // this CTA's accumulators, read by the cluster
    const int kvh = blockIdx.x;
    const int C = static_cast<int>(gridDim.y);
    const int r = static_cast<int>(at_cluster_rank());
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    pdl_launch_dependents();
    const int kvd = nkv * kAttnHd;
    const int nkeys = pos + 1, kpc = (nkeys + C - 1) / C;
    const int jb = min(nkeys, r * kpc), je = min(nkeys, jb + kpc);

    // Rows below `pos` are issued before the dependency wait: they were written by
    // this layer's attention for earlier tokens, and a kernel that far back in the
    // stream has completed (a token's kernels each wait for their predecessor, and
    // at most a few of them are resident at once).
    auto stage = [&](int j0, int nks) {
        for (int i = t; i < nks * 16; i += kAtThreads) {
            const int jj = i >> 4, c = i & 15;
            const size_t off = static_cast<size_t>(j0 + jj) * kvd + kvh * kAttnHd + c * 8;
            at_cp16(ks + jj * kAtRow + ((c ^ (jj & 7)) << 4), kc + off);
            at_cp16(vs + jj * kAtRow + (c << 4), vc + off);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (jb < je) stage(jb, min(kAtSub, je - jb));
    // RoPE angles (rope.rs:22-55: f64 inverse frequencies and angles, cos / sin rounded to f32) depend only on
    // the position, so they are computed before the wait for the q / k projections
    float c = 0.f, sn = 0.f;
    if (t < kAttnHd / 2) {
        const double inv = 1.0 / pow(rope_base, 2.0 * t / static_cast<double>(kAttnHd));
        double sd, cd;
        sincos(static_cast<double>(pos) * inv, &sd, &cd);
        c = static_cast<float>(cd);
        sn = static_cast<float>(sd);
    }
    pdl_wait();

    // RoPE of this CTA's query heads and of the new key
    if (t < kAttnHd / 2) {
#pragma unroll
        for (int h = 0; h < REPS; ++h) {
            const float* qh = qkv + (kvh * REPS + h) * kAttnHd;
            const float x0 = qh[t], x1 = qh[t + kAttnHd / 2];
            qs[h][t] = x0 * c - x1 * sn;
            qs[h][t + kAttnHd / 2] = x0 * sn + x1 * c;
        }
        const float* kh = qkv + nq * kAttnHd + kvh * kAttnHd;
        const float x0 = kh[t], x1 = kh[t + kAttnHd / 2];
        kn[t] = x0 * c - x1 * sn;
        kn[t + kAttnHd / 2] = x0 * sn + x1 * c;
    }
    if (t < kAttnHd) vn[t] = qkv[nq * kAttnHd + kvd + kvh * kAttnHd + t];
    if (t < REPS) {
        cm[t] = -INFINITY;
        cl[t] = 0.0;
    }
    __syncthreads();
    if (pos >= jb && pos < je && t < kAttnHd) {
        kc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + t] = __float2half_rn(kn[t]);
        vc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + t] = __float2half_rn(vn[t]);
    }

    // q of every head for this lane's 4 dimensions, in registers
    float4 q4[REPS];
#pragma unroll
    for (int h = 0; h < REPS; ++h) q4[h] = *reinterpret_cast<const float4*>(&qs[h][4 * lane]);
    const float4 kn4 = *reinterpret_cast<const float4*>(&kn[4 * lane]);
    const float4 vn4 = *reinterpret_cast<const float4*>(&vn[4 * lane]);
    for (int i = t; i < REPS * kAttnHd; i += kAtThreads) reinterpret_cast<float*>(co)[i] = 0.f;
    float* red = reinterpret_cast<float*>(ks);  // [8 warps][REPS][128] partial outputs (K region, free by then)
    constexpr int G = 32 / REPS;                // keys per butterfly group (G * REPS = 32 values)
    for (int j0 = jb; j0 < je; j0 += kAtSub) {
        const int nks = min(kAtSub, je - j0);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        // scores: warp w takes the groups of G keys starting at G*w, G*(w+8), ...; lane holds dimensions 4l..4l+3.  For G keys
        // at a time the G * REPS partial dots are reduce-scattered over the 32 lanes (lane l ends
        // with key l / REPS, head l % REPS).
        for (int g0 = warp * G; g0 < nks; g0 += (kAtThreads / 32) * G) {
            float v[32];
#pragma unroll
            for (int kk = 0; kk < G; ++kk) {
                const int jj = g0 + kk;
                float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (jj < nks) {
                    if (j0 + jj == pos) {
                        k4 = kn4;
                    } else {
                        const uint2 raw = *reinterpret_cast<const uint2*>(
                            ks + jj * kAtRow + (((lane >> 1) ^ (jj & 7)) << 4) + ((lane & 1) << 3));
                        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                        const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                        k4 = make_float4(a.x, a.y, b2.x, b2.y);
                    }
                }
#pragma unroll
                for (int h = 0; h < REPS; ++h) {
                    float p = q4[h].x * k4.x;
                    p = fmaf(q4[h].y, k4.y, p);
                    p = fmaf(q4[h].z, k4.z, p);
                    p = fmaf(q4[h].w, k4.w, p);
                    v[kk * REPS + h] = p;
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
            if (jj < nks) sc[lane % REPS][jj] = v[0] * scale;
        }
        __syncthreads();
        // online softmax per head (warp h): exp(s - max) in f64 and its f64 sum (gqa.rs:29-110)
        for (int h = warp; h < REPS; h += kAtThreads / 32) {
            float m = -INFINITY;
            for (int jj = lane; jj < nks; jj += 32) m = fmaxf(m, sc[h][jj]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float mo = cm[h], mn = fmaxf(mo, m);
            double l = 0.0;
            for (int jj = lane; jj < nks; jj += 32) {
                const double e = exp(static_cast<double>(sc[h][jj] - mn));
                sc[h][jj] = static_cast<float>(e);
                l += e;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                const double f = mo == -INFINITY ? 0.0 : exp(static_cast<double>(mo - mn));
                cl[h] = cl[h] * f + l;
                cm[h] = mn;
                corr[h] = static_cast<float>(f);
            }
        }
        __syncthreads();
        // P . V: warp w over keys w, w+8, ..., lane over dimensions 4l..4l+3
        float4 acc[REPS];
#pragma unroll
        for (int h = 0; h < REPS; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int jj = warp; jj < nks; jj += kAtThreads / 32) {
            float4 v4;
            if (j0 + jj == pos) {
                v4 = vn4;
            } else {
                const uint2 raw = *reinterpret_cast<const uint2*>(vs + jj * kAtRow + 8 * lane);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                const float2 b2 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                v4 = make_float4(a.x, a.y, b2.x, b2.y);
            }
#pragma unroll
            for (int h = 0; h < REPS; ++h) {
                const float p = sc[h][jj];
                acc[h].x = fmaf(p, v4.x, acc[h].x);
                acc[h].y = fmaf(p, v4.y, acc[h].y);
                acc[h].z = fmaf(p, v4.z, acc[h].z);
                acc[h].w = fmaf(p, v4.w, acc[h].w);
            }
        }
        __syncthreads();  // every warp is done with K (the reduction area) and V
#pragma unroll
        for (int h = 0; h < REPS; ++h)
            *reinterpret_cast<float4*>(&red[(warp * REPS + h) * kAttnHd + 4 * lane]) = acc[h];
        __syncthreads();
        // running accumulators: co = co * corr + the warps' sums in warp order
        for (int i = t; i < REPS * kAttnHd; i += kAtThreads) {
            const int h = i / kAttnHd;
            float sum = 0.f;
#pragma unroll
            for (int w = 0; w < kAtThreads / 32; ++w) sum += red[(w * REPS + h) * kAttnHd + (i % kAttnHd)];
            reinterpret_cast<float*>(co)[i] = reinterpret_cast<float*>(co)[i] * corr[h] + sum;
        }
        if (j0 + kAtSub < je) {
            __syncthreads();  // the sub-chunk is consumed: stage the next one
            stage(j0 + kAtSub, min(kAtSub, je - j0 - kAtSub));
        }
    }
    // combine across the cluster: this CTA finalises outputs [r*np, (r+1)*np) of the
    // REPS * 128 (head, dimension) pairs, over the CTAs in rank order
    at_cluster_sync();
    // per (CTA q, head h): the weight f = exp(m_q - M_h) (f64, as the reference's sum) and l_q * f, computed
    // once here, then the sum L_h over the CTAs in rank order
    __shared__ float fw[16][REPS];
    __shared__ double lw[16][REPS];
    __shared__ float Mh[REPS];
    __shared__ float Linv[REPS];
    if (t < C * REPS) {
        const int q = t / REPS, h = t % REPS;
        fw[q][h] = at_ld_f32(at_mapa(&cm[h], q));
        lw[q][h] = at_ld_f64(at_mapa(&cl[h], q));
    }
    __syncthreads();
    if (t < REPS) {
        float M = -INFINITY;
        for (int q = 0; q < C; ++q) M = fmaxf(M, fw[q][t]);
        Mh[t] = M;
    }
    __syncthreads();
    if (t < C * REPS) {
        const int q = t / REPS, h = t % REPS;
        const double f = fw[q][h] == -INFINITY ? 0.0 : exp(static_cast<double>(fw[q][h] - Mh[h]));
        lw[q][h] *= f;
        fw[q][h] = static_cast<float>(f);
    }
    __syncthreads();
    if (t < REPS) {
        double L = 0.0;
        for (int q = 0; q < C; ++q) L += lw[q][t];
        Linv[t] = static_cast<float>(1.0 / L);
    }
    __syncthreads();
    // this CTA finalises outputs [r*np, (r+1)*np) of the REPS * 128 (head, dimension) pairs
    const int np = (REPS * kAttnHd + C - 1) / C;
    for (int pi = t; pi < np; pi += kAtThreads) {
        const int pr = r * np + pi;
        if (pr < REPS * kAttnHd) {
            const int h = pr / kAttnHd, dd = pr % kAttnHd;
            float oq[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) oq[q] = q < C ? at_ld_f32(at_mapa(&co[h][dd], q)) : 0.f;
            float o = 0.f;
#pragma unroll
            for (int q = 0; q < 16; ++q)
                if (q < C) o = fmaf(oq[q], fw[q][h], o);
            out[(kvh * REPS + h) * kAttnHd + dd] = o * Linv[h];
        }
    }
    at_cluster_sync();  // no CTA leaves while another reads its shared memory
}

// ───────────────────────── host launchers ─────────────────────────

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

// Cluster size of the attention kernel on this device: 16 CTAs per KV head where a
// cluster of 16 with this kernel's shared memory can be resident, else 8.
template <int REPS>
static int attention_cluster_size() {
    static std::atomic<int> cached[64];  // zero-initialised (static storage); 0 = not yet measured
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 8;
    if (const int c = cached[dev].load(std::memory_order_acquire)) return c;
    int c = 8;
    cudaFuncSetAttribute(decode_attention_kernel<REPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
    if (cudaFuncSetAttribute(decode_attention_kernel<REPS>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
        cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1, 16);
        cfg.blockDim = dim3(kAtThreads);
        cfg.dynamicSmemBytes = kAtSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 16;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, decode_attention_kernel<REPS>, &cfg) == cudaSuccess && n >= 1) c = 16;
    }
    cudaGetLastError();  // a refused query leaves no error behind
    cached[dev].store(c, std::memory_order_release);
    return c;
}

template <int REPS>
static cudaError_t launch_attention_reps(const float* qkv, int nq, int nkv, int pos, float scale, double rope_base,
                                         __half* kc, __half* vc, float* out, cudaStream_t stream) {
    const int C = attention_cluster_size<REPS>();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nkv, C);
    cfg.blockDim = dim3(kAtThreads);
    cfg.dynamicSmemBytes = kAtSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = C;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, decode_attention_kernel<REPS>, qkv, nq, nkv, pos, scale, rope_base, kc, vc, out);
}

// out [nq * 128] = attention of the token at `pos` (RoPE'd q against keys 0..pos), the
// new k / v appended to the caches.  No workspace: the splits combine in the cluster.
cudaError_t launch_decode_attention(const float* qkv, int nq, int nkv, int hd, int pos, float scale,
                                    double rope_base, __half* kc, __half* vc, float* out, cudaStream_t stream) {
    if (hd != kAttnHd || nkv < 1 || nq % nkv || pos < 0) return cudaErrorInvalidValue;
    cudaError_t e = cudaErrorInvalidValue;
    switch (nq / nkv) {
        case 1: e = launch_attention_reps<1>(qkv, nq, nkv, pos, scale, rope_base, kc, vc, out, stream); break;
        case 2: e = launch_attention_reps<2>(qkv, nq, nkv, pos, scale, rope_base, kc, vc, out, stream); break;
        case 4: e = launch_attention_reps<4>(qkv, nq, nkv, pos, scale, rope_base, kc, vc, out, stream); break;
        case 8: e = launch_attention_reps<8>(qkv, nq, nkv, pos, scale, rope_base, kc, vc, out, stream); break;
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
