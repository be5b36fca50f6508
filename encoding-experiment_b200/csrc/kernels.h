// kernels.h — plans and host launchers of the sm_100a kernels (C++; shared by
// the kernel translation units and the context in backend.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace larql {

// ── CUDA-core Q4_K matvec (q4k_matvec.cu) ──
cudaError_t launch_q4k_matvec(const uint8_t* W, int N, int K, const float* x, int batch, float* y, int num_sms,
                              int* status, cudaStream_t stream);
// GGUF-144 Q4_K x f32 (ggml.rs:228-273 dequantize_q4_k + dot), one weight pass per batch row (q4k_matvec.cu).
cudaError_t launch_q4k_gguf_matvec(const uint8_t* W, int N, int K, const float* x, int batch, float* y,
                                   int num_sms, int* status, cudaStream_t stream);
extern int g_q4k_planes;

// ── tcgen05 Q4_K matvec (q4k_tc.cu) ──
struct TcPlan {
    int N, K, nchunks, H, ntiles, grid, batch, nmma, phase_subs;
    int w_region, b_bytes, xi_bytes, stage_bytes, a_off, bar_off, smem;
};
bool q4k_tc_make_plan(int N, int K, int batch, int num_sms, TcPlan* out);
size_t q4k_tc_scratch_bytes(int K, int batch);
int q4k_tc_encode_map(void* encode_fn, const void* w, int N, int K, int H, CUtensorMap* map);
cudaError_t launch_q4k_tc(const CUtensorMap& map, const float* x, float* y, const TcPlan& p, uint8_t* scratch,
                          int* status, cudaStream_t stream);

// ── tcgen05 Q4_K matvec with sc*q in tensor memory (q4k_ts.cu) ──
struct TsPlan {
    int N, K, batch, nchunks, ntiles, nparts, nitems, grid, smem;
};
bool q4k_ts_make_plan(int N, int K, int batch, int num_sms, TsPlan* out);
size_t q4k_ts_scratch_bytes(const TsPlan& p);  // B tiles + split-K partials
size_t q4k_ts_tickets(const TsPlan& p);        // zeroed ints (left zeroed by every complete launch)
cudaError_t launch_q4k_ts(const CUtensorMap& map, const float* x, float* y, const TsPlan& p, uint8_t* scratch,
                          int* tickets, int* status, cudaStream_t stream);

// ── warp-MMA Q4_K matvec (q4k_mma.cu) ──
struct MmaPlan {
    int fmt;             // 0: Q4_K (148 B / 256), 1: Q4_0 (18 B / 32), 2: GGUF Q8_0 (34 B / 32); ggml dequantisation
                         // (half.rs f16 scales) for 1 and 2
    int N, K, batch, NT;
    int NG, KS, NW, RT;  // 16-row groups per tile, warps per group (K slices), consumer warps, rows per tile
    int NS, PF;          // ring stages, L2 prefetch distance (boxes)
    int nchunks, nparts, kpc;
    int ntiles, nitems, grid;
    int stage_bytes, xt_off, mt_off, wt_off, red_off, bar_off, smem;
};
// force: {groups, kslices, stages, parts, prefetch}, 0 = planner's choice
bool q4k_mma_make_plan(int N, int K, int batch, int num_sms, MmaPlan* out, const int* force, int fmt = 0);
int mma_chunk_bytes(int fmt);
int mma_encode_map(void* encode_fn, const void* w, int N, int K, int fmt, int H, CUtensorMap* map);
size_t q4k_mma_partial_floats(const MmaPlan& p);
cudaError_t launch_q4k_mma(const CUtensorMap& map, const float* x, float* y, float* partial, int* tickets,
                           const MmaPlan& p, int* status, cudaStream_t stream);
// Decode fusions of the batch-1 MMA matvec: a transform of x applied while the x tables are built, and a
// residual epilogue.
struct MmaFuse {
    int pro;              // 0: x as given; 1: RMSNorm of x (x / rms * (offset + nw), rms from ss_in);
                          // 2: SiLU: x' = silu(x[k]) * x[K + k] (x = [gate | up])
    const double* ss_in;  // pro 1: f64 sums of squares of x per 16 values, ceil(K / 16) of them
    const float* nw;      // pro 1: norm weight [K]
    float offset, eps;    // pro 1
    int epi;              // 1: y[r] += (W x')[r] in place, and ss_out[r / 16] = sum of the new y^2 per 16 rows
    double* ss_out;
};
cudaError_t launch_q4k_mma_fused(const CUtensorMap& map, const float* x, float* y, float* partial, int* tickets,
                                 const MmaPlan& p, const MmaFuse& f, int* status, cudaStream_t stream);

// ── block formats: Q4_0, Q8_0, Q8 compute layout, Q6_K (matvec_blocks.cu) ──
cudaError_t launch_block_matvec(int fmt, const uint8_t* W, const float* wscale, const float* x32, const int8_t* q8x,
                                const float* q8s, float* y, int N, int K, int num_sms, int* status,
                                cudaStream_t stream);
cudaError_t launch_quantize_to_q8(const float* x, size_t n, int8_t* q, float* s, cudaStream_t stream);
cudaError_t launch_dequant_q8(const int8_t* q, const float* s, size_t n, float* out, cudaStream_t stream);

// ── Q4_0 vector-matrix product (vecmat.cu) ──
struct VecmatPlan {
    int ngroups;         // column groups of 32 blocks (1024 columns)
    int nranges;         // contiguous row ranges (summed by a second kernel when > 1)
    int rows_per_range;
};
VecmatPlan q4_vecmat_plan(int inter, int hidden, int num_sms);
size_t q4_vecmat_part_floats(const VecmatPlan& p, int hidden);
cudaError_t launch_q4_vecmat(const float* act, const uint8_t* w, int inter, int hidden, const VecmatPlan& p,
                             float* part, float* out, cudaStream_t stream);

// ── vindex gate walk (gate_tc.cu) ──
struct GatePlan {
    int L, F, D, B;
    int QB, P, T;
    int nkb, qbox, k;
    int nitems, grid, smem;
    int packed;  // B <= 64: hi and lo planes of 16 queries in alternate 16-row blocks of one 128-row A tile
};
bool gate_make_plan(int L, int F, int D, int B, int k, int num_sms, GatePlan* out);
size_t gate_scratch_bytes(const GatePlan& p);
int gate_encode_map(void* encode_fn, const void* base, size_t rows, int D, int box_rows, CUtensorMap* map);
cudaError_t launch_gate_topk(void* encode_fn, const CUtensorMap& gmap, float factor, const float* queries,
                             const GatePlan& p, uint8_t* scratch, uint32_t* out_i, float* out_s, int* status,
                             cudaStream_t stream, float* scores = nullptr);
cudaError_t launch_gate_merge(const float* cand_s, const uint32_t* cand_i, int L, int B, int P, int k,
                              uint32_t* out_i, float* out_s, cudaStream_t stream);
// small query batches on CUDA cores (gate_gemv.cu)
bool gate_gemv_ok(int D, int B);
// Q4_0 gate walk selection: scores [B][L][F] -> top-k by |score| per (layer, query) (candidates of `parts` ranges,
// L * B * parts * 16 entries of cand_s / cand_i, then the merge).
int gate_score_cand_parts(int L, int F, int B, int num_sms);
cudaError_t launch_gate_score_topk(const float* scores, int L, int F, int B, int k, int parts, float* cand_s,
                                   uint32_t* cand_i, uint32_t* out_i, float* out_s, cudaStream_t stream);
int gate_gemv_parts(int L, int F, int num_sms);
cudaError_t launch_gate_gemv(const __half* g, float factor, const float* q, int L, int F, int D, int B, int k,
                             int parts, float* cand_s, uint32_t* cand_i, uint32_t* out_i, float* out_s,
                             cudaStream_t stream);
cudaError_t launch_topk_merge_lists(const uint32_t* in_i, const float* in_s, int n_lists, int rows, int kin,
                                    const uint32_t* offsets, int kout, uint32_t* out_i, float* out_s,
                                    cudaStream_t stream);
cudaError_t launch_gate_halfrs_fixup(uint16_t* g, size_t n, int* work, float* factor_host, cudaStream_t stream);

// ── logits top-k by signed value (lm_head.cu) ──
size_t logit_topk_scratch_entries(int n, int k, int num_sms);
cudaError_t launch_logit_topk(const float* logits, int n, int k, int num_sms, uint64_t* scratch, uint32_t* out_id,
                              float* out_logit, cudaStream_t stream);

// ── decode layer (decode.cu) ──
cudaError_t launch_decode_rmsnorm(float* x, const float* add, const float* w, float offset, float eps, int n,
                                  float* h, cudaStream_t stream);
cudaError_t launch_decode_silu_mul(const float* gu, int inter, float* act, cudaStream_t stream);
cudaError_t launch_decode_add(float* x, const float* d, int n, cudaStream_t stream);
cudaError_t launch_decode_sumsq16(const float* x, int n, double* ss, cudaStream_t stream);
cudaError_t launch_decode_attention(const float* qkv, int nq, int nkv, int hd, int pos, float scale,
                                    double rope_base, __half* kc, __half* vc, float* out, cudaStream_t stream);
cudaError_t launch_f32_to_f16(const float* in, size_t n, __half* out, cudaStream_t stream);

// ── persistent decode: one launch per token through every layer (decode_persist.cu) ──
struct DecodePersistPlan {
    alignas(8) unsigned char raw[256];  // the kernel's parameter block
    int reps, grid, smem, att_items;
    int N[4], K[4], nparts[4];          // Q|K|V, O, gate|up, down
};
struct DecodePersistBufs {
    float* x;        // the residual (in and out)
    float* xalt;     // [H] alternate residual
    float* part[4];  // per projection [nparts][N] partial sums
    float* att_acc;  // [att items][reps * 128]
    float* att_m;    // [att items][reps]
    double* att_l;   // [att items][reps]
    float* attn;     // [nq * 128]
    unsigned* bar;   // [4] grid barrier state (zeroed by the launcher)
};
// 0 when the shapes are served (hidden, inter and nq * 128 multiples of 1024, hidden <= 8192; 1, 2, 4 or 8 query
// heads per KV head, head dim 128).
int decode_persist_plan(int L, int H, int I, int nq, int nkv, int pos, int num_sms, double rope_base,
                        DecodePersistPlan* out);
int decode_persist_map(void* encode_fn, const void* w, int N, int K, CUtensorMap* map);
size_t decode_persist_layer_bytes();
void decode_persist_layer_fill(void* dst, const float* norms, __half* kc, __half* vc, float offset, float eps,
                               float scale);
// cudaSuccess when the plan's grid can be resident at once (cooperative launch), else
// cudaErrorCooperativeLaunchTooLarge
cudaError_t decode_persist_check(const DecodePersistPlan& plan);
cudaError_t launch_decode_persist(const DecodePersistPlan& plan, const void* layers_dev, const CUtensorMap* maps_dev,
                                  const DecodePersistBufs& bufs, int* status, cudaStream_t stream);

// ── prefill dequant-GEMM (prefill_tc.cu) ──
struct PrefillPlan {
    int N, K, M;   // weight rows, K, tokens
    int NTOK;      // tokens per tile (MMA N): 64, 128 or 256
    int fused;     // 1: gate/up SwiGLU (two weights), 0: plain
    int nrt, ntt;  // row tiles, token tiles
    int nitems, grid, nkb, smem;
    int nab, nst;  // dequantized-weight buffers, activation stages
};
bool prefill_make_plan(int N, int K, int M, bool fused, int num_sms, PrefillPlan* out);
int prefill_tokens_padded(const PrefillPlan& p);
cudaError_t launch_q4k_abs_bound(const uint8_t* w, size_t nsb, unsigned int* out, cudaStream_t stream);
size_t q4k_prefill_panel_bytes(size_t N, size_t K);
cudaError_t launch_q4k_prefill_pack(const uint8_t* w, int N, int K, float wscale, uint8_t* out, cudaStream_t stream);
cudaError_t launch_prefill_x_prep(const float* x, int M, int K, int rows, __half* xh, float* xs, cudaStream_t stream);
int prefill_encode_xmap(void* encode_fn, const __half* xh, int rows, int K, int box_rows, CUtensorMap* map);
size_t prefill_part_floats(const PrefillPlan& p);
cudaError_t launch_prefill_gemm(const CUtensorMap& xmap, const uint8_t* w0, const uint8_t* w1, float wscale0,
                                float wscale1, const float* xs, float* y, float* part, int* flags, const PrefillPlan& p,
                                int* status, cudaStream_t stream);

// ── one-shot all-reduce over peer memory (p2p_reduce.cu) ──
constexpr int kP2pMaxRanks = 8;
struct P2pAreas {
    void* base[kP2pMaxRanks];  // every rank's receive area as mapped in this process
};
size_t p2p_area_bytes(int world, int max_n);
cudaError_t launch_p2p_allreduce(const P2pAreas& areas, int rank, int world, int max_n, int n, const float* src,
                                 float* dst, int* epoch_ctr, int* status, cudaStream_t stream);

// ── quantizers (quantize.cu) ──
cudaError_t launch_quantize_q4_k(const float* data, size_t n, uint8_t* out, cudaStream_t stream);
cudaError_t launch_quantize_block32(int fmt, const float* data, size_t n, uint8_t* out, cudaStream_t stream);
cudaError_t launch_quantize_q6_k(const float* data, size_t n, uint8_t* out, cudaStream_t stream);

}  // namespace larql
