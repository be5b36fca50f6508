/*
 * larql_cuda.h — C ABI of the B200 (sm_100a) compute backend for LARQL's
 * quantized-matvec / gate-walk hot path.
 *
 * The entry points mirror the reference trait `ComputeBackend`
 * (crates/larql-compute/src/backend.rs:24-164, paths relative to the
 * larql-main workspace) so that a Rust `CudaBackend` can bind them with
 * `extern "C"` exactly as crates/larql-compute/src/cpu/ops/q4_common.rs:6-25
 * binds csrc/q4_dot.c today.  Plain pointers and sizes only.
 *
 * Conventions
 *  - Every function returns an int status (LARQL_OK == 0).  The reference
 *    returns Option::None for "unsupported"; a Rust wrapper maps any non-zero
 *    status to None and logs larql_cuda_last_error().
 *  - Functions without a `_dev` suffix take HOST pointers and are synchronous
 *    on return, like the trait (which returns an owned Vec<f32>).
 *  - `_dev` functions take DEVICE pointers and enqueue on `stream`
 *    (a cudaStream_t passed as void*, NULL = the context's stream); they
 *    return once the work is enqueued.
 *  - Weights are placed on the device once.  The by-pointer entry points
 *    (larql_cuda_q4k_matvec etc.) look the weight up in a registry keyed by
 *    (host pointer, byte length), uploading it on first use — the semantics of
 *    the Metal backend's buffer cache (crates/larql-compute/src/metal/buffers.rs:13-83).
 *    Handle-based entry points take a handle from larql_cuda_register_weight().
 *  - A context is bound to one device and is safe to share across host
 *    threads (calls are serialised per context).
 */
#ifndef LARQL_CUDA_H
#define LARQL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LARQL_API __attribute__((visibility("default")))
#else
#define LARQL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ── status codes ── */
#define LARQL_OK 0
#define LARQL_ERR_INVALID_ARG 1   /* null pointer, zero-sized where not allowed */
#define LARQL_ERR_BAD_SHAPE 2     /* hidden not a multiple of the block size, size mismatch */
#define LARQL_ERR_UNSUPPORTED 3   /* format/op not provided (reference: Option::None) */
#define LARQL_ERR_CUDA 4          /* CUDA runtime error */
#define LARQL_ERR_NCCL 5          /* NCCL error / NCCL unavailable */
#define LARQL_ERR_TIMEOUT 6       /* a bounded device-side wait ran out */
#define LARQL_ERR_OOM 7           /* device allocation failed */
#define LARQL_ERR_NOT_FOUND 8     /* unknown handle */

/* ── weight formats: crates/larql-compute/src/pipeline.rs:12-18 (QuantFormat) ── */
#define LARQL_FMT_Q4_0 0       /* 18 B / 32 values: f16 scale + 16 B nibbles */
#define LARQL_FMT_Q4_K 1       /* LARQL 148 B / 256 values (q4_common.rs:96-170) */
#define LARQL_FMT_Q4_KF 2      /* 160 B / 256 values, pre-baked f16 scales (not provided) */
#define LARQL_FMT_Q6_K 3       /* 210 B / 256 values (q4_common.rs:172-239) */
#define LARQL_FMT_Q8_0 4       /* compute layout: int8 values + separate f32 scale per 32 (QuantWeight.scales) */
#define LARQL_FMT_Q8_0_GGUF 5  /* GGUF 34 B / 32 values: f16 scale + 32 int8 (larql-models ggml.rs:136) */
#define LARQL_FMT_F16 6        /* f16 rows, IEEE decoding */
#define LARQL_FMT_F16_HALFRS 7 /* f16 rows decoded like crates/larql-models/src/quant/half.rs:4-20 (subnormals at
                                  half their IEEE value): the vindex gate vectors (gate.rs:86-94, 287, 762) */
#define LARQL_FMT_Q4_K_GGUF 8  /* GGUF 144 B / 256 values as crates/larql-models/src/quant/ggml.rs:228-273
                                  (dequantize_q4_k, the GGUF loader's decoder, gguf.rs:191) reads them */
#define LARQL_FMT_Q4_K_GGUF_LLAMA 9 /* GGUF 144 B / 256 values in llama.cpp's layout (quants in 32-byte chunks,
                                       sub-blocks 2c / 2c+1 in the low / high nibbles of chunk c; IEEE f16 d / dmin),
                                       as the reference's Metal q4kf kernels read them
                                       (crates/larql-compute/src/metal/shaders/q4kf_qkv_proj.rs:136-220) */

typedef struct larql_cuda_ctx larql_cuda_ctx;

/* ── version / errors ── */
/* Library version as major*10000 + minor*100 + patch. */
LARQL_API int larql_cuda_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to len). */
LARQL_API int larql_cuda_last_error(char* buf, size_t len);
/* Static description of a status code. */
LARQL_API const char* larql_cuda_status_string(int status);

/* ── context ── */
/* Replaces default_backend()'s backend construction (crates/larql-compute/src/lib.rs:68-84). */
LARQL_API int larql_cuda_create(int device, larql_cuda_ctx** out);
LARQL_API int larql_cuda_destroy(larql_cuda_ctx* ctx);
/* ComputeBackend::name (backend.rs:160) / device_info (backend.rs:163). */
LARQL_API int larql_cuda_name(larql_cuda_ctx* ctx, char* buf, size_t len);
LARQL_API int larql_cuda_device_info(larql_cuda_ctx* ctx, char* buf, size_t len);
/* ComputeBackend::has_q4 (backend.rs:155): writes 1. */
LARQL_API int larql_cuda_has_q4(larql_cuda_ctx* ctx, int* out);
/* The context's stream (cudaStream_t as void*). */
LARQL_API int larql_cuda_stream(larql_cuda_ctx* ctx, void** stream);
/* Waits for the context's stream, then reports (and clears) any error a
 * kernel recorded on the device (e.g. LARQL_ERR_TIMEOUT from a bounded wait). */
LARQL_API int larql_cuda_sync(larql_cuda_ctx* ctx);

/* ── weight registry: one-time placement (metal/buffers.rs:62-83 semantics) ── */
/* Uploads `nbytes` of `format` weights for a [rows, cols] matrix (cols = hidden =
 * K, rows = N output features).  `scales` is only used for LARQL_FMT_Q8_0
 * (rows*cols/32 f32, pipeline.rs:24 QuantWeight.scales).  Registering the same
 * (pointer, length) again returns the existing handle. */
LARQL_API int larql_cuda_register_weight(larql_cuda_ctx* ctx, const void* host_data, size_t nbytes,
                               const float* scales, int format, size_t rows, size_t cols,
                               uint64_t* handle);
/* Same, from device memory (copied into a context-owned, padded buffer). */
LARQL_API int larql_cuda_register_weight_device(larql_cuda_ctx* ctx, const void* dev_data, size_t nbytes,
                                      const float* dev_scales, int format, size_t rows,
                                      size_t cols, uint64_t* handle);
LARQL_API int larql_cuda_release_weight(larql_cuda_ctx* ctx, uint64_t handle);
/* Device pointer of a registered weight (read-only use). */
LARQL_API int larql_cuda_weight_device_ptr(larql_cuda_ctx* ctx, uint64_t handle, const void** dev_ptr);

/* ── trait mirrors (host pointers, synchronous) ── */
/* ComputeBackend::q4k_matvec (backend.rs:126-130); CPU reference
 * crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87.  out[num_rows]. */
LARQL_API int larql_cuda_q4k_matvec(larql_cuda_ctx* ctx, const uint8_t* q4k_data, size_t nbytes,
                          const float* x, size_t num_rows, size_t hidden, float* out);

/* ComputeBackend::q6k_matvec (backend.rs:133-137); CPU reference
 * crates/larql-compute/src/cpu/ops/q6k_matvec.rs:31-87 (210 B per 256 values, hidden % 256 == 0).
 * out[num_rows]. */
LARQL_API int larql_cuda_q6k_matvec(larql_cuda_ctx* ctx, const uint8_t* q6k_data, size_t nbytes,
                          const float* x, size_t num_rows, size_t hidden, float* out);

/* ComputeBackend::q4_matvec (backend.rs:49-53): scores[N] = Q4_0[N,K] @ Q8_x[K],
 * x pre-quantized by quantize_to_q8 (q4_common.rs:28-44: int8 + f32 scale per 32).
 * CPU reference crates/larql-compute/csrc/q4_dot.c:169-199 (q4_0_matvec_c). */
LARQL_API int larql_cuda_q4_matvec(larql_cuda_ctx* ctx, const uint8_t* q4_data, size_t nbytes, const int8_t* q8_x,
                         const float* q8_scales, size_t num_rows, size_t hidden, float* out);
LARQL_API int larql_cuda_q4_matvec_dev(larql_cuda_ctx* ctx, uint64_t handle, const int8_t* q8_x_dev,
                             const float* q8_scales_dev, float* y_dev, void* stream);

/* ComputeBackend::q4_vecmat (backend.rs:56-60): out[hidden] = activation[intermediate] @ Q4_0[intermediate, hidden];
 * rows with -1e-10 < activation < 1e-10 are skipped.  CPU reference crates/larql-compute/csrc/q4_dot.c:201-232
 * (q4_0_vecmat_c, via cpu/ops/q4_vecmat.rs:8-17).  hidden % 32 == 0. */
LARQL_API int larql_cuda_q4_vecmat(larql_cuda_ctx* ctx, const float* activation, const uint8_t* q4_data, size_t nbytes,
                         size_t intermediate, size_t hidden, float* out);
/* Device form: handle = a Q4_0 weight registered as intermediate rows x hidden cols; act_dev[rows], out_dev[cols]. */
LARQL_API int larql_cuda_q4_vecmat_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* act_dev, float* out_dev,
                             void* stream);

/* ComputeBackend::q4_matvec_pair_batch (backend.rs:64-69; Metal metal/ops/q4_batched.rs:19-80): for each of
 * seq_len positions, x_matrix[t] quantized by quantize_to_q8 (q4_common.rs:28-44), then the Q4_0 x Q8 matvec
 * (q4_dot.c:169-199) against gate and up.  gate_out / up_out: [seq_len][num_rows].  hidden % 64 == 0. */
LARQL_API int larql_cuda_q4_matvec_pair_batch(larql_cuda_ctx* ctx, const uint8_t* gate_q4, size_t gate_nbytes,
                                    const uint8_t* up_q4, size_t up_nbytes, const float* x_matrix, size_t seq_len,
                                    size_t num_rows, size_t hidden, float* gate_out, float* up_out);
LARQL_API int larql_cuda_q4_matvec_pair_batch_dev(larql_cuda_ctx* ctx, uint64_t gate, uint64_t up, const float* x_dev,
                                        size_t seq_len, float* gate_out_dev, float* up_out_dev, void* stream);

/* ── handle-based matvec, batch 1..8 ── */
/* y[b, r] = W[r, :] . x[b, :] for b < batch.  x is [batch, cols] f32, y is
 * [batch, rows] f32.  Formats and CPU references:
 *   LARQL_FMT_Q4_K       crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87
 *   LARQL_FMT_Q4_0       crates/larql-models/src/quant/ggml.rs:92-110 dequantize + f32 dot
 *   LARQL_FMT_Q8_0_GGUF  crates/larql-models/src/quant/ggml.rs:136-151 dequantize + f32 dot
 *   LARQL_FMT_Q8_0       crates/larql-compute/src/cpu/ops/q8_matvec.rs:36-57 against
 *                        quantize_to_q8(x) (q4_common.rs:28-44), quantized on the device
 *   LARQL_FMT_Q6_K       crates/larql-compute/src/cpu/ops/q6k_matvec.rs:31-87 (cols % 256 == 0)
 *   LARQL_FMT_Q4_K_GGUF  crates/larql-models/src/quant/ggml.rs:228-273 dequantize + f32 dot (cols % 256 == 0,
 *                        cols <= 30720)
 *   LARQL_FMT_Q4_K_GGUF_LLAMA  the Metal q4kf_proj kernel (shaders/q4kf_qkv_proj.rs:136-220): llama.cpp layout,
 *                        cols % 1024 == 0 */
LARQL_API int larql_cuda_matvec(larql_cuda_ctx* ctx, uint64_t handle, const float* x, size_t batch, float* y);
LARQL_API int larql_cuda_matvec_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* x_dev, size_t batch,
                          float* y_dev, void* stream);

/* ── device-side quantizers (bit-identical to the reference quantizers) ── */
/* crates/larql-compute/src/cpu/ops/q4_common.rs:28-44 (quantize_to_q8): n f32 (multiple of 32)
 * -> n int8 + n/32 f32 scales. */
LARQL_API int larql_cuda_quantize_to_q8_dev(larql_cuda_ctx* ctx, const float* x_dev, size_t n, int8_t* q8_dev,
                                  float* scales_dev, void* stream);
/* crates/larql-compute/src/cpu/ops/q4_common.rs:104-170 (quantize_q4_k, 148 B/256).
 * n = number of f32 values (multiple of 256); out receives n/256*148 bytes. */
LARQL_API int larql_cuda_quantize_q4_k_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n,
                                 uint8_t* out_dev, void* stream);
/* crates/larql-compute/src/cpu/ops/q4_common.rs:50-80 (quantize_q4_0, 18 B/32; identical to
 * crates/larql-models/src/quant/ggml.rs:310-337).  n multiple of 32; out receives n/32*18 bytes. */
LARQL_API int larql_cuda_quantize_q4_0_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n,
                                 uint8_t* out_dev, void* stream);
/* crates/larql-models/src/quant/ggml.rs:342-363 (quantize_q8_0, GGUF 34 B/32).  n multiple of 32;
 * out receives n/32*34 bytes. */
LARQL_API int larql_cuda_quantize_q8_0_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n,
                                 uint8_t* out_dev, void* stream);
/* crates/larql-compute/src/cpu/ops/q4_common.rs:179-239 (quantize_q6_k, 210 B/256).  n multiple of 256;
 * out receives n/256*210 bytes. */
LARQL_API int larql_cuda_quantize_q6_k_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n,
                                 uint8_t* out_dev, void* stream);

/* ── matvec without device allocation ──
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory while they run (a fixed budget reserved up front, or memory owned by
 * another framework): a Q4_K (LARQL 148 B) matvec on the tensor-core kernel
 * whose per-call scratch is a fixed array compiled into this library (544 KiB
 * on every device that loads it, held until the process exits), so the call
 * allocates nothing.  w_dev, x_dev, y_dev are device pointers as for
 * larql_cuda_matvec_dev; cols must be a multiple of 1024 and <= 16384,
 * batch 1..8; larger shapes return LARQL_ERR_BAD_SHAPE.  Every call is
 * synchronous: it waits for its stream and copies a status word back to the
 * host before it returns.  The first call on a device loads this part of the
 * library's device code there (under CUDA's default lazy module loading; at
 * context creation with CUDA_MODULE_LOADING=EAGER), which reserves the array on
 * that device, and looks up the array's device address: make it during set-up,
 * before any stream capture and before the caller's memory budget is fixed.
 * All calls on a device share the one array: calls that overlap on the GPU
 * race and must be serialised by the caller. */
LARQL_API int larql_cuda_q4k_matvec_noalloc(const uint8_t* w_dev, size_t nbytes, size_t rows, size_t cols,
                                            const float* x_dev, size_t batch, float* y_dev, void* stream);

/* ── vindex gate walk ── */

/* VectorIndex::gate_knn (crates/larql-vindex/src/index/gate.rs:108-134) + top_k_from_scores (:307-316) over
 * every layer of a vindex at once, for a batch of residuals (gate_knn_batch, :500-537, keeps the per-query
 * lists here instead of their union).  `gates`: n_layers x n_feat rows of `hidden` f16 values, layer-major as in
 * gate_vectors.bin (format/load.rs:19-87), decoded as half.rs does; `queries`: f32 [batch][hidden].
 * out_idx / out_score: [n_layers][batch][top_k], feature index within the layer and signed score, ordered by
 * |score| descending (ties: lower index first); rows past n_feat never appear.  top_k <= 16, hidden a multiple
 * of 64.  Host pointers; synchronous.  The gate matrix is registered on first use by (pointer, length). */
LARQL_API int larql_cuda_gate_topk_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes, size_t n_layers,
                                       size_t n_feat, size_t hidden, const float* queries, size_t batch,
                                       size_t top_k, uint32_t* out_idx, float* out_score);
/* Same on a registered LARQL_FMT_F16_HALFRS weight of n_layers * n_feat rows, device pointers, enqueued on
 * `stream` (NULL = the context's stream). */
LARQL_API int larql_cuda_gate_topk_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                                       const float* queries_dev, size_t batch, size_t top_k, uint32_t* out_idx_dev,
                                       float* out_score_dev, void* stream);

/* Merge of per-shard top-k lists (the gate rows of a layer split across GPUs, candidates all-gathered):
 * in [n_lists][rows][k_in] (index 0xFFFFFFFF = empty), each list's indices shifted by offsets_dev[list]
 * (NULL = no shift), out [rows][k_out] by |score| descending, ties by lower index.  n_lists * k_in <= 512.
 * Device pointers, enqueued on `stream`.  (gate.rs:307-316 applied to the union of the shards' lists.) */
LARQL_API int larql_cuda_topk_merge_dev(larql_cuda_ctx* ctx, const uint32_t* idx_in, const float* score_in,
                                        size_t n_lists, size_t rows, size_t k_in, const uint32_t* offsets_dev,
                                        size_t k_out, uint32_t* idx_out, float* score_out, void* stream);

/* gate_scores_batch (gate.rs:545-559, for n_layers stacked layers): every score, out_scores [n_layers][batch][n_feat]
 * f32 = queries . gate rows (f16 decoded as half.rs does).  Host pointers; synchronous.  Same registration and
 * shape rules as larql_cuda_gate_topk_f16 (hidden a multiple of 64). */
LARQL_API int larql_cuda_gate_scores_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes, size_t n_layers,
                                         size_t n_feat, size_t hidden, const float* queries, size_t batch,
                                         float* out_scores);
/* Same on a registered LARQL_FMT_F16_HALFRS weight of n_layers * n_feat rows, device pointers, enqueued on `stream`. */
LARQL_API int larql_cuda_gate_scores_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                                         const float* queries_dev, size_t batch, float* out_scores_dev, void* stream);
/* gate_knn_batch (gate.rs:500-537): the sorted union of the per-position top_k features (by |score|) of
 * x [seq_len][hidden] against one layer's n_feat gate rows.  out_idx holds up to seq_len * min(top_k, n_feat)
 * entries, *out_count the union's size.  top_k <= 16.  Host pointers; synchronous. */
LARQL_API int larql_cuda_gate_knn_batch_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes,
                                            size_t n_feat, size_t hidden, const float* x, size_t seq_len,
                                            size_t top_k, uint32_t* out_idx, size_t* out_count);

/* ── lm-head KNN ── */

/* VectorIndex::lm_head_knn_backend, its Q4 branch (crates/larql-vindex/src/index/walk.rs:549-583): the query
 * quantized by quantize_to_q8 (q4_common.rs:28-44), logits[vocab] = Q4_0 lm head [vocab][hidden] x Q8 query
 * (ComputeBackend::q4_matvec, q4_dot.c:169-199), then the min(top_k, vocab) largest logits by signed value,
 * descending (walk.rs:566-577; equal logits by lower token id, NaN logits below -inf).  top_k 1..32; top_k 0
 * (the reference then returns every logit sorted) or min(top_k, vocab) > 32 gives LARQL_ERR_UNSUPPORTED, the
 * caller's cue to take its f32 lm_head_knn path as it does when q4_matvec returns None.  hidden % 64 == 0.
 * Host pointers, synchronous; *out_count = entries written.  The lm head is registered on first use by
 * (pointer, length). */
LARQL_API int larql_cuda_lm_head_knn(larql_cuda_ctx* ctx, const uint8_t* q4_data, size_t nbytes, size_t vocab,
                                     size_t hidden, const float* query, size_t top_k, uint32_t* out_ids,
                                     float* out_logits, size_t* out_count);
/* Same on a registered Q4_0 weight (vocab rows x hidden cols): query_dev f32 [hidden], ids_dev / logits_dev
 * [min(top_k, vocab)], enqueued on `stream`. */
LARQL_API int larql_cuda_lm_head_knn_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* query_dev, size_t top_k,
                                         uint32_t* ids_dev, float* logits_dev, void* stream);
/* The selection step alone (walk.rs:566-577): the min(top_k, n) largest of n f32 logits on the device, same
 * order and limits as larql_cuda_lm_head_knn.  Device pointers, enqueued on `stream`. */
LARQL_API int larql_cuda_logit_topk_dev(larql_cuda_ctx* ctx, const float* logits_dev, size_t n, size_t top_k,
                                        uint32_t* ids_dev, float* logits_out_dev, void* stream);

/* ── decode (one token through Llama-style Q4_K layers with an f16 KV cache) ── */

/* The Llama / Q4_K subset of FullPipelineLayer (crates/larql-compute/src/pipeline.rs:60-110): RMSNorm
 * (norm_offset + weight), gated SiLU FFN, no post-norms.  Weights are LARQL Q4_K (148 B / 256 values) row-major
 * [rows][cols]: wq [nq*hd][hidden], wk / wv [nkv*hd][hidden], wo [hidden][nq*hd], gate / up [inter][hidden],
 * down [hidden][inter].  Norm weights are f32 [hidden]. */
typedef struct larql_cuda_layer_desc {
    const uint8_t* wq;
    const uint8_t* wk;
    const uint8_t* wv;
    const uint8_t* wo;
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    const float* input_norm;
    const float* post_attn_norm;
    float norm_offset; /* 0 for Llama */
    float eps;         /* RMSNorm epsilon */
    float attn_scale;  /* 1/sqrt(head_dim) for Llama */
} larql_cuda_layer_desc;

/* Places one layer on the device (Q|K|V and gate|up are stored fused).  src_is_device: the pointers in `d` are
 * device pointers.  head_dim must be 128, nq a multiple of nkv (<= 8 query heads per KV head), hidden and inter
 * multiples of 256. */
LARQL_API int larql_cuda_layer_register(larql_cuda_ctx* ctx, const larql_cuda_layer_desc* d, size_t hidden,
                                        size_t inter, size_t nq, size_t nkv, size_t head_dim, int src_is_device,
                                        uint64_t* handle);
LARQL_API int larql_cuda_layer_release(larql_cuda_ctx* ctx, uint64_t handle);
/* f16 KV cache of n_layers x max_seq x nkv x head_dim (K and V), zeroed, length 0 (has_kv_cache, backend.rs:99). */
LARQL_API int larql_cuda_kv_init(larql_cuda_ctx* ctx, size_t n_layers, size_t max_seq, size_t nkv, size_t head_dim);
/* populate_kv_layer (backend.rs:103-107): k / v [seq_len][nkv*head_dim] f32 (host), stored as f16 (nearest);
 * sets the cache length to seq_len. */
LARQL_API int larql_cuda_kv_populate(larql_cuda_ctx* ctx, size_t layer, const float* k, const float* v,
                                     size_t seq_len);
/* Same from device f16 data [seq_len][nkv*head_dim]. */
LARQL_API int larql_cuda_kv_populate_f16_dev(larql_cuda_ctx* ctx, size_t layer, const void* k, const void* v,
                                             size_t seq_len, void* stream);
/* reset_kv_cache (backend.rs:110): length 0.  kv_length: the current length. */
LARQL_API int larql_cuda_kv_reset(larql_cuda_ctx* ctx);
LARQL_API int larql_cuda_kv_set_length(larql_cuda_ctx* ctx, size_t len);
LARQL_API int larql_cuda_kv_length(larql_cuda_ctx* ctx, size_t* len);
/* Decode kernel selection for later decode_token calls (no counterpart in the reference, a switch of this
 * library): on != 0 runs a whole token as one persistent launch (every layer in one kernel, LARQL_CUDA_DECODE_PERSIST=1
 * sets it at context creation) where the layers allow it — same shapes in every layer, Q4_K projections, hidden,
 * inter and nq*128 multiples of 1024, hidden <= 8192 — and the per-kernel pipeline elsewhere; 0 (the default)
 * always runs the pipeline.  The first persistent call for a layer list uploads its tensor maps and must come
 * before any stream capture of it. */
LARQL_API int larql_cuda_decode_set_persistent(larql_cuda_ctx* ctx, int on);
/* Tensor-parallel decode (heads and FFN rows split over `world` ranks, one context per GPU; no counterpart in
 * the reference, whose decode runs on one device).  Registers rank `rank`'s share of the layer described by
 * `d` (full-size weights): the Q / K / V rows of query heads [rank*nq/world, ...) and KV heads
 * [rank*nkv/world, ...), the gate / up rows [rank*inter/world, ...), and the input-column slices of O (those
 * heads' dimensions) and down (those FFN rows).  Requires nkv % world == 0, (nq/world)*head_dim and inter/world
 * multiples of 256.  The rank's KV cache holds its nkv/world heads (larql_cuda_kv_init with that count). */
LARQL_API int larql_cuda_layer_register_shard(larql_cuda_ctx* ctx, const larql_cuda_layer_desc* d, size_t hidden,
                                              size_t inter, size_t nq, size_t nkv, size_t head_dim, size_t rank,
                                              size_t world, int src_is_device, uint64_t* handle);
/* Called twice per layer while a sharded token is enqueued: `buf` (device, n floats) holds this rank's partial
 * sum of the O (then the down) projection; the callee must replace it, on `stream`, by the sum over all ranks
 * (an all-reduce) and return 0 (non-zero aborts the token with LARQL_ERR_NCCL). */
typedef int (*larql_cuda_reduce_fn)(void* user, float* buf, size_t n, void* stream);
/* One token through sharded layers at position `pos` (x_dev [hidden] replicated on every rank, updated in
 * place); red_dev: a device buffer of >= hidden floats the reductions run on.  Enqueued on `stream`. */
LARQL_API int larql_cuda_decode_token_sharded_dev(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers,
                                                  float* x_dev, size_t pos, float rope_base, float* red_dev,
                                                  larql_cuda_reduce_fn reduce, void* user, void* stream);
/* One-shot all-reduce (sum) of up to max_n floats across the `world` GPUs of one node over NVLink / NVSwitch peer
 * memory, for the two reductions per layer of the sharded decode (no counterpart in the reference).  Each rank:
 * larql_cuda_p2p_init (allocates its receive area, returns a 64-byte CUDA IPC handle), exchanges the handles
 * (e.g. an all-gather over the process group), then larql_cuda_p2p_connect with all `world` handles in rank
 * order.  larql_cuda_p2p_allreduce_dev sums buf_dev in place on `stream` (capturable); every rank must make the
 * same sequence of calls; a peer that does not arrive within the wait budget gives LARQL_ERR_TIMEOUT at the
 * next larql_cuda_sync.  All ranks get identical bits (ranks summed in order). */
LARQL_API int larql_cuda_p2p_init(larql_cuda_ctx* ctx, size_t rank, size_t world, size_t max_n, void* ipc_handle);
LARQL_API int larql_cuda_p2p_connect(larql_cuda_ctx* ctx, const void* handles);
LARQL_API int larql_cuda_p2p_allreduce_dev(larql_cuda_ctx* ctx, float* buf_dev, size_t n, void* stream);
/* decode_token (backend.rs:115-124): x [hidden] (host) through layers[0..n) (layer i uses KV layer i) at position
 * = the cache length, which then grows by one; out [hidden] (host) = the residual after the last layer. */
LARQL_API int larql_cuda_decode_token(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers, const float* x,
                                      float rope_base, float* out);
/* Device form: x_dev [hidden] updated in place, position `pos` given explicitly, the cache length unchanged
 * (capturable in a CUDA graph).  Enqueued on `stream`. */
LARQL_API int larql_cuda_decode_token_dev(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers, float* x_dev,
                                          size_t pos, float rope_base, void* stream);

/* ── batched prefill (dequant-GEMM on tensor cores) ── */

/* Y[t][n] = W[n] . X[t] for t < n_tokens: the batched form of q4k_matvec (q4k_matvec.rs:31-87), W a registered
 * Q4_K weight [N][K], X [n_tokens][K] and Y [n_tokens][N] f32 device pointers.  Tiles of W are dequantized to f16
 * (times a per-matrix power of two) and X to f16 (times a per-token power of two); tcgen05 MMAs accumulate in f32.
 * K a multiple of 256.  Enqueued on `stream`. */
LARQL_API int larql_cuda_q4k_gemm_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* x_dev, size_t n_tokens,
                                      float* y_dev, void* stream);
/* The prefill FFN of prefill_q4 (backend.rs:143-152): y[t] = down . (silu(gate . x[t]) * (up . x[t]))
 * (silu_gate_up, crates/larql-inference/src/ffn/mod.rs:87-94) for t < n_tokens; gate / up [inter][hidden],
 * down [hidden][inter] registered Q4_K handles; x, y [n_tokens][hidden] f32 device pointers. */
LARQL_API int larql_cuda_prefill_ffn_dev(larql_cuda_ctx* ctx, uint64_t gate, uint64_t up, uint64_t down,
                                         const float* x_dev, size_t n_tokens, float* y_dev, void* stream);
/* The same FFN in the ownership form of ComputeBackend::prefill_q4 (backend.rs:143-152): the three Q4_K weights
 * as borrowed host slices (placed on the device once, found again by (pointer, length) like every host-pointer
 * entry), x [n_tokens][hidden] host f32 in, y [n_tokens][hidden] host f32 out; synchronous.  gate / up are
 * [inter][hidden], down [hidden][inter].  The attention half of prefill_q4 is not provided here. */
LARQL_API int larql_cuda_prefill_ffn(larql_cuda_ctx* ctx, const uint8_t* gate, size_t gate_bytes, const uint8_t* up,
                                     size_t up_bytes, const uint8_t* down, size_t down_bytes, size_t hidden,
                                     size_t inter, const float* x, size_t n_tokens, float* y);

/* VectorIndex::gate_knn_q4 / gate_knn_adaptive's Q4 branch (crates/larql-vindex/src/index/gate.rs:672-731): the
 * Q4_0 gate rows of every layer (gate_vectors_q4.bin, crates/larql-vindex/src/index/walk.rs:303-328: layers
 * contiguous, [n_layers * n_feat][hidden] Q4_0) scored against each query quantized by quantize_to_q8
 * (q4_common.rs:28-44) with q4_matvec (q4_dot.c:169-199), then top_k_from_scores (gate.rs:307-316: top-K by
 * |score|, here ties by lower index) per (layer, query).  hidden % 64 == 0, top_k <= 16; out
 * [n_layers][batch][top_k] layer-local indices.  Host buffers, synchronous; weight found by (pointer, length). */
LARQL_API int larql_cuda_gate_topk_q4(larql_cuda_ctx* ctx, const uint8_t* gates_q4, size_t nbytes, size_t n_layers,
                                      size_t n_feat, size_t hidden, const float* queries, size_t batch, size_t top_k,
                                      uint32_t* out_idx, float* out_score);
/* Same on a registered LARQL_FMT_Q4_0 weight of n_layers * n_feat rows, device buffers, enqueued on `stream`. */
LARQL_API int larql_cuda_gate_topk_q4_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                                          const float* queries_dev, size_t batch, size_t top_k, uint32_t* out_idx_dev,
                                          float* out_score_dev, void* stream);

/* ── vindex loader: a .vindex directory placed once on the GPU ──
 * A vindex directory as the reference writes it: index.json (crates/larql-vindex/src/config/types.rs
 * VindexConfig: num_layers, hidden_size, intermediate_size, dtype "f32" | "f16", layers[] with num_features and
 * the byte offset / length of each layer's gate rows), gate_vectors.bin (the rows), and optionally
 * interleaved_q4k.bin (per layer gate, up in Q4_K and down in Q4_K or Q6_K) and attn_weights_q4k.bin with
 * attn_weights_q4k_manifest.json (Q, K, V, O per layer in Q4_K or Q6_K). */
typedef struct larql_cuda_vindex larql_cuda_vindex;
typedef struct {
    size_t num_layers, hidden, intermediate, vocab;
    size_t features_max;      /* largest num_features of any layer */
    int gate_bits;            /* 16 (f16 rows, decoded as half.rs) or 32 (f32 rows) */
    int ffn_q4k;              /* interleaved_q4k.bin: 0 absent, 1 gate / up / down all Q4_K, 2 down in Q6_K */
    int attn_q4k;             /* 1: attn_weights_q4k.bin and its manifest present */
    int gate_q4;              /* 1: gate_vectors_q4.bin present (Q4_0 gate rows, walk.rs:303-328) */
    size_t shard_rank, shard_count;  /* open(): the row shard this handle holds (0, 1 when probed) */
    size_t shard_row0, shard_rows;   /* first gate row of every layer on this shard, rows per layer held */
} larql_cuda_vindex_info;

/* Reads and checks a vindex directory without a GPU (index.json, the file sizes the layers and manifests
 * name).  LARQL_ERR_INVALID_ARG with a message naming the file and field on malformed input. */
LARQL_API int larql_cuda_vindex_probe(const char* dir, larql_cuda_vindex_info* info);
/* VectorIndex::load_vindex (crates/larql-vindex/src/format/load.rs:19-87), with the one-time device placement
 * the Metal backend does by (pointer, length): rows [shard_rank * per, (shard_rank + 1) * per) of every layer's
 * gate vectors (per = ceil(features_max / shard_count)) are copied once to the context's GPU in the layout the
 * gate walk reads (f16 rows as stored; f32 rows as an f16 high / scaled-low pair), hidden padded with zeros to
 * a multiple of 64 and short layers with zero rows.  shard_count 1 holds every row. */
LARQL_API int larql_cuda_vindex_open(larql_cuda_ctx* ctx, const char* dir, size_t shard_rank, size_t shard_count,
                                     larql_cuda_vindex** out);
LARQL_API int larql_cuda_vindex_info_get(const larql_cuda_vindex* v, larql_cuda_vindex_info* info);
/* gate_knn (gate.rs:108-134, 307-316) of `batch` residuals [batch][hidden] against every layer held:
 * out [num_layers][batch][top_k], feature indices within the layer (shard_row0 added), slots past a layer's
 * rows 0xFFFFFFFF / 0.  top_k <= 16.  Synchronous, host buffers. */
LARQL_API int larql_cuda_vindex_gate_knn(larql_cuda_vindex* v, const float* queries, size_t batch, size_t top_k,
                                         uint32_t* out_idx, float* out_score);
/* gate_knn_q4 (gate.rs:714-731) over the Q4_0 gate rows of gate_vectors_q4.bin placed at open: each residual
 * quantized by quantize_to_q8, q4_matvec, top-K by |score|; same output convention as larql_cuda_vindex_gate_knn.
 * hidden % 64 == 0; LARQL_ERR_UNSUPPORTED when the vindex has no Q4_0 gates. */
LARQL_API int larql_cuda_vindex_gate_knn_q4(larql_cuda_vindex* v, const float* queries, size_t batch, size_t top_k,
                                            uint32_t* out_idx, float* out_score);
/* Same on device buffers, enqueued on `stream`: indices are shard-local (add shard_row0 when merging shards
 * with larql_cuda_topk_merge_dev); an index >= the layer's rows on this shard marks an empty slot. */
LARQL_API int larql_cuda_vindex_gate_knn_dev(larql_cuda_vindex* v, const float* queries_dev, size_t batch,
                                             size_t top_k, uint32_t* out_idx_dev, float* out_score_dev, void* stream);
/* The FFN of a layer from interleaved_q4k.bin as it is sliced for FullPipelineLayer (VectorIndex::
 * load_interleaved_q4k, crates/larql-vindex/src/index/walk.rs:225; resolve_ffn_weights,
 * crates/larql-inference/src/layer_graph/pipeline_layer.rs:121-134): registered weight handles of this shard's
 * rows of gate, up ([intermediate][hidden], Q4_K) and down ([hidden][intermediate], Q4_K or Q6_K, *down_format).
 * Placed on first request, released by larql_cuda_vindex_close. */
LARQL_API int larql_cuda_vindex_ffn(larql_cuda_vindex* v, size_t layer, uint64_t* gate, uint64_t* up,
                                    uint64_t* down, int* down_format);
/* Q, K, V, O of a layer from attn_weights_q4k.bin and its manifest (VectorIndex::load_attn_q4k /
 * attn_q4k_layer_data, walk.rs:402-445): handles of this shard's rows and their LARQL_FMT_* formats. */
LARQL_API int larql_cuda_vindex_attn(larql_cuda_vindex* v, size_t layer, uint64_t handles[4], int formats[4]);
/* Releases every device copy the vindex placed and unmaps its files. */
LARQL_API int larql_cuda_vindex_close(larql_cuda_vindex* v);

/* Diagnostic (no counterpart in the reference): a one-line description of the kernel(s) and launch plan
 * larql_cuda_matvec / _matvec_dev would use for `handle` at `batch` (e.g. "q4k_mma_kernel<1> groups=8 ..."). */
LARQL_API int larql_cuda_describe_matvec(larql_cuda_ctx* ctx, uint64_t handle, size_t batch, char* buf, size_t len);

/* Diagnostic (no counterpart in the reference): the number of kernel launches this library has enqueued in
 * this process, over all contexts.  Launches replayed from a captured CUDA graph are not counted again. */
LARQL_API int larql_cuda_launch_count(uint64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* LARQL_CUDA_H */
