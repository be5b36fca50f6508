// backend.h — host-side context and weight registry (C++; not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/larql_cuda.h"

#include "kernels.h"

namespace larql {

struct Q4kRoute {
    enum { kMma, kTc, kDp4a, kTs } kind;
    MmaPlan mp;
    TcPlan tp;
    TsPlan sp;
    const CUtensorMap* map;
};

struct Weight {
    void* dev = nullptr;          // context-owned copy (padded)
    float* scales_dev = nullptr;  // LARQL_FMT_Q8_0 separate scales
    size_t nbytes = 0;
    int format = -1;
    size_t rows = 0, cols = 0;
    const void* key = nullptr;  // registering pointer (registry key)
    size_t key_len = 0;
    bool owned = false;
    // TMA tensor maps of the Q4_K tensor-core paths, one per tile height in use
    static constexpr int kMaps = 4;
    CUtensorMap tmap[kMaps];
    int tmap_h[kMaps] = {0, 0, 0, 0};
    int tmap_next = 0;
    CUtensorMap gmap;  // gate walk: f16 rows, 64 x 256 boxes, 128-byte swizzle
    bool gmap_ok = false;
    float gate_factor = 1.0f;  // scores of a LARQL_FMT_F16_HALFRS weight are multiplied by this
    float f16_scale = 0.f;     // Q4_K: power of two keeping every dequantized value inside f16 (0 = not yet known)
    uint8_t* pf_dev = nullptr;  // Q4_K: prefill panels (q4k_prefill_pack), built on first GEMM use
    MmaPlan blk_plans[8] = {};  // Q4_0 / Q8_0 / Q6_K: warp-MMA plan per batch (N 0 = not planned, -1 = not served)
    // Q4_K: the route per batch, planned on first use (the tensor map is looked up again on every use: the
    // map slots are reused round-robin)
    Q4kRoute q4k_route[8] = {};
    bool q4k_routed[8] = {};
};

struct Layer {
    uint64_t qkv = 0, o = 0, gu = 0, down = 0;  // weight handles (Q|K|V and gate|up fused)
    float* norms = nullptr;                     // [2][hidden]: input_norm, post_attn_norm
    size_t hidden = 0, inter = 0, nq = 0, nkv = 0, hd = 0;  // inter, nq, nkv: this rank's share when sharded
    float offset = 0.f, eps = 1e-5f, attn_scale = 1.f;
    size_t world = 1;  // > 1: one rank's head / FFN shard (O and down produce partial sums)
};

struct KvLayer {
    __half* k = nullptr;  // [max_seq][nkv * hd]
    __half* v = nullptr;
};


struct Ctx {
    int device = 0;
    int num_sms = 0;
    int l2_bytes = 0;
    char dev_name[256] = {0};
    cudaStream_t stream = nullptr;
    std::recursive_mutex mu;  // recursive: a reduction callback may call back into the context on the same thread
    std::unordered_map<uint64_t, Weight> weights;
    std::map<std::pair<uintptr_t, size_t>, uint64_t> by_ptr;
    uint64_t next_handle = 1;
    int* status_dev = nullptr;   // [0] device status word, [1..15] scratch ints
    int* status_host = nullptr;  // pinned
    float* x_dev = nullptr;
    size_t x_cap = 0;
    float* y_dev = nullptr;
    size_t y_cap = 0;
    uint8_t* scratch = nullptr;  // per-call operand staging of the tensor-core kernels
    size_t scratch_cap = 0;
    uint8_t* aux = nullptr;  // operands of composite calls whose kernels use `scratch` themselves
    size_t aux_cap = 0;
    void* encode_tiled = nullptr;  // cuTensorMapEncodeTiled (driver entry point)
    bool use_tc = true;           // tensor-core Q4_K path (LARQL_CUDA_Q4K_TC=0 disables)
    // Q4_K kernel family: 0 = warp-MMA (default), 1 = tcgen05 kind::i8 for batch >= 2, 2 = dp4a only,
    // 3 = tcgen05 with sc*q in tensor memory for every batch (LARQL_CUDA_Q4K_PATH=mma|tc|dp4a|ts);
    // LARQL_CUDA_MMA_CFG="groups,slices,stages,parts,prefetch" pins the MMA plan.
    int q4k_path = 0;
    // default path: batches from this size on the tensor-memory kernel (q4k_ts.cu) when K % 1024 == 0
    // (LARQL_CUDA_TS_MIN_BATCH)
    int ts_min_batch = 9;
    // decode fusions into the matvecs, bits: 1 SiLU, 2 norm + residual (LARQL_CUDA_DECODE_FUSE; off by default:
    // measured slower than the separate kernels on configs[2])
    int fuse_decode = 0;
    // persistent decode (decode_persist.cu): one launch per token through every layer
    // (LARQL_CUDA_DECODE_PERSIST=1; falls back to the per-kernel pipeline where the shapes are not served)
    int decode_persist = 0;
    struct PersistState {
        std::vector<uint64_t> handles;         // the layers the uploaded blocks and maps describe
        std::vector<unsigned char> lay_host;   // the uploaded per-layer blocks
        void* lay_dev = nullptr;
        CUtensorMap* maps_dev = nullptr;       // [layers][4] tensor maps with 32-row boxes
        uint8_t* ws = nullptr;                 // partial sums, attention partials, alternate residual, barrier
        size_t ws_cap = 0;
    } pd;
    int q6k_mma_min_batch = 2;  // Q6_K batches from this size on the warp-MMA kernel (LARQL_CUDA_Q6K_MMA_MIN_BATCH)
    // Q4_0 x f32 batches from this size on the warp-MMA kernel, smaller ones on the block kernel
    // (LARQL_CUDA_Q40_MMA_MIN_BATCH; batch 1 measured faster on the MMA kernel once its box rows were padded)
    int q40_mma_min_batch = 1;
    bool gate_gemv = true;  // gate walk of 1-4 queries on CUDA cores (LARQL_CUDA_GATE_GEMV=0: the tensor-core walk)
    int mma_force[5] = {0, 0, 0, 0, 0};  // groups, K slices, stages, parts, prefetch (0 = planner)
    int* tickets = nullptr;  // split-K tickets of the MMA path (kept zeroed)
    size_t tickets_cap = 0;
    // decode: registered layers, the f16 KV cache and the per-token workspace
    std::unordered_map<uint64_t, Layer> layers;
    std::vector<KvLayer> kv;
    size_t kv_max_seq = 0, kv_nkv = 0, kv_hd = 0, kv_len = 0;
    float* dws = nullptr;  // h | o | d | qkv | attn | gu | act | 2 x f64 sums of squares per 16 values
    size_t dws_cap = 0;
    // one-shot all-reduce over peer memory (tensor-parallel decode)
    int p2p_rank = -1, p2p_world = 0, p2p_max_n = 0;
    void* p2p_local = nullptr;   // this rank's receive area
    int* p2p_epoch = nullptr;    // call counter, advanced by the kernel
    P2pAreas p2p_areas{};        // every rank's area as mapped here (IPC)
    bool p2p_ready = false;
    // prefill GEMM stream-K: partial-sum slots and their flags ([num_sms][4], kept zeroed)
    float* pf_part = nullptr;
    size_t pf_part_cap = 0;
    int* pf_flags = nullptr;

    ~Ctx();
    int ensure_io(size_t x_floats, size_t y_floats);
    int finish();
    Weight* find(uint64_t h);
    int add_weight(const void* src, bool src_is_device, size_t nbytes, const float* scales, bool scales_device,
                   int format, size_t rows, size_t cols, uint64_t* handle);
    int weight_for(const void* host, size_t nbytes, int format, size_t rows, size_t cols, uint64_t* handle);
    int matvec_dev(Weight* w, const float* x, size_t batch, float* y, cudaStream_t s);
    bool fusable(Weight* w);
    int matvec_fused_dev(Weight* w, const float* x, float* y, const MmaFuse& f, cudaStream_t s);
    int matvec_host(Weight* w, const float* x, size_t batch, float* y);
    int q4_matvec_q8_dev(Weight* w, const int8_t* q8x, const float* q8s, float* y, cudaStream_t s);
    int logit_topk_dev(const float* logits, size_t n, size_t top_k, uint32_t* ids, float* vals, cudaStream_t s);
    int lm_head_knn_dev(Weight* w, const float* query, size_t top_k, uint32_t* ids, float* vals, cudaStream_t s);
    int q4_vecmat_dev(Weight* w, const float* act, float* out, cudaStream_t s);
    int q4_pair_batch_dev(Weight* g, Weight* u, const float* x, size_t seq, float* gout, float* uout,
                          cudaStream_t s);
    int gate_topk_dev(Weight* w, size_t n_layers, size_t n_feat, const float* q, size_t batch, size_t top_k,
                      uint32_t* out_i, float* out_s, cudaStream_t s, float* scores = nullptr);
    int gate_topk_q4_dev(Weight* w, size_t n_layers, size_t n_feat, const float* q, size_t batch, size_t top_k,
                         uint32_t* out_i, float* out_s, cudaStream_t s);
    int ensure_scratch(size_t bytes);
    int ensure_tickets(size_t n);
    int ensure_aux(size_t bytes);
    int add_weight_parts(const void* const* parts, const size_t* part_bytes, int nparts, bool src_is_device,
                         int format, size_t rows, size_t cols, uint64_t* handle);
    void release_handle(uint64_t h);
    int layer_register(const larql_cuda_layer_desc* d, size_t hidden, size_t inter, size_t nq, size_t nkv, size_t hd,
                       bool src_is_device, uint64_t* handle);
    int layer_register_shard(const larql_cuda_layer_desc* d, size_t hidden, size_t inter, size_t nq, size_t nkv,
                             size_t hd, size_t rank, size_t world, bool src_is_device, uint64_t* handle);
    int add_weight_cols(const void* src, bool src_is_device, size_t rows, size_t cols, size_t c0, size_t c1,
                        uint64_t* handle);
    int decode_sharded_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, float* red,
                           larql_cuda_reduce_fn fn, void* user, cudaStream_t s);
    int decode_workspace(const uint64_t* lh, size_t n, size_t pos, float** ws, double** ss = nullptr);
    int kv_init(size_t n_layers, size_t max_seq, size_t nkv, size_t hd);
    int decode_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, cudaStream_t s);
    int decode_persist_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, cudaStream_t s);
    int q4k_f16_scale(Weight* w, float* scale);
    int q4k_prefill_panels(Weight* w, float* scale, const uint8_t** panels);
    int ensure_prefill_ws(size_t part_floats);
    int gemm_q4k_dev(Weight* w, const float* x, size_t M, float* y, cudaStream_t s);
    int prefill_ffn_dev(Weight* wg, Weight* wu, Weight* wd, const float* x, size_t M, float* y, cudaStream_t s);
    const CUtensorMap* q4k_map(Weight* w, int H);
    int route_q4k(Weight* w, size_t batch, Q4kRoute* r);  // cached per weight and batch
    int plan_q4k(Weight* w, size_t batch, Q4kRoute* r);   // the routing decision itself
    const MmaPlan* blk_mma_plan(Weight* w, size_t batch);
    int describe_q4k(Weight* w, size_t batch, char* buf, size_t len);
};

int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
size_t format_bytes(int format, size_t rows, size_t cols);

}  // namespace larql

// The C ABI's opaque context: one Ctx per GPU.
struct larql_cuda_ctx {
    larql::Ctx impl;
};

// Entry-point prologue: null check, the context lock, the context's device current.
#define LARQL_CTX_GUARD(ctx)                                                           \
    if (!(ctx)) return larql::fail(LARQL_ERR_INVALID_ARG, "null context");             \
    std::lock_guard<std::recursive_mutex> _lk((ctx)->impl.mu);                         \
    {                                                                                  \
        cudaError_t _e = cudaSetDevice((ctx)->impl.device);                            \
        if (_e != cudaSuccess) return larql::cuda_fail(_e, "cudaSetDevice");           \
    }
