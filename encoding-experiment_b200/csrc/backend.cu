// backend.cu — host side of the CUDA backend: context, weight registry,
// error reporting and the C ABI declared in include/larql_cuda.h.
//
// The registry gives the reference's "weights arrive by host pointer on every
// call" convention (crates/larql-compute/src/backend.rs:126-130) the Metal
// backend's caching semantics (crates/larql-compute/src/metal/buffers.rs:62-83):
// the first call with a given (pointer, length) uploads the bytes once into a
// context-owned device buffer, later calls reuse it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>

#include "../../include/larql_cuda.h"
#include "backend.h"
#include "common.cuh"
#include "kernels.h"

namespace larql {

static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? LARQL_ERR_OOM : LARQL_ERR_CUDA, "%s: %s (%s)", what,
                cudaGetErrorName(e), cudaGetErrorString(e));
}

size_t format_bytes(int format, size_t rows, size_t cols) {
    const size_t n = rows * cols;
    switch (format) {
        case LARQL_FMT_Q4_0: return n / 32 * 18;
        case LARQL_FMT_Q4_K: return n / 256 * 148;
        case LARQL_FMT_Q4_KF: return n / 256 * 160;
        case LARQL_FMT_Q4_K_GGUF:
        case LARQL_FMT_Q4_K_GGUF_LLAMA: return n / 256 * 144;
        case LARQL_FMT_Q6_K: return n / 256 * 210;
        case LARQL_FMT_Q8_0: return n;  // int8 values; scales separate
        case LARQL_FMT_Q8_0_GGUF: return n / 32 * 34;
        case LARQL_FMT_F16:
        case LARQL_FMT_F16_HALFRS: return n * 2;
        default: return 0;
    }
}

size_t format_block(int format) {
    switch (format) {
        case LARQL_FMT_Q4_0:
        case LARQL_FMT_Q8_0:
        case LARQL_FMT_Q8_0_GGUF: return 32;
        case LARQL_FMT_Q4_K:
        case LARQL_FMT_Q4_KF:
        case LARQL_FMT_Q4_K_GGUF:
        case LARQL_FMT_Q4_K_GGUF_LLAMA:
        case LARQL_FMT_Q6_K: return 256;
        case LARQL_FMT_F16:
        case LARQL_FMT_F16_HALFRS: return 1;
        default: return 0;
    }
}

// Device allocations carry 256 bytes of zeroed slack so 16-byte bulk copies
// that round a tail up never read past the allocation.
constexpr size_t kPad = 256;

Ctx::~Ctx() {
    cudaSetDevice(device);
    for (auto& kv : weights) {
        if (kv.second.owned) cudaFree(kv.second.dev);
        if (kv.second.scales_dev) cudaFree(kv.second.scales_dev);
        if (kv.second.pf_dev) cudaFree(kv.second.pf_dev);
    }
    if (x_dev) cudaFree(x_dev);
    if (y_dev) cudaFree(y_dev);
    if (scratch) cudaFree(scratch);
    if (aux) cudaFree(aux);
    if (tickets) cudaFree(tickets);
    for (auto& kv_l : kv) {
        if (kv_l.k) cudaFree(kv_l.k);
        if (kv_l.v) cudaFree(kv_l.v);
    }
    for (auto& l : layers)
        if (l.second.norms) cudaFree(l.second.norms);
    if (dws) cudaFree(dws);
    if (pd.lay_dev) cudaFree(pd.lay_dev);
    if (pd.maps_dev) cudaFree(pd.maps_dev);
    if (pd.ws) cudaFree(pd.ws);
    if (pf_part) cudaFree(pf_part);
    if (pf_flags) cudaFree(pf_flags);
    for (int p = 0; p < p2p_world; ++p)
        if (p != p2p_rank && p2p_areas.base[p]) cudaIpcCloseMemHandle(p2p_areas.base[p]);
    if (p2p_local) cudaFree(p2p_local);
    if (p2p_epoch) cudaFree(p2p_epoch);
    if (status_dev) cudaFree(status_dev);
    if (status_host) cudaFreeHost(status_host);
    if (stream) cudaStreamDestroy(stream);
}

int Ctx::ensure_io(size_t x_floats, size_t y_floats) {
    if (x_floats > x_cap) {
        if (x_dev) cudaFree(x_dev);
        x_dev = nullptr;
        cudaError_t e = cudaMalloc(&x_dev, x_floats * sizeof(float) + kPad);
        if (e != cudaSuccess) { x_cap = 0; return cuda_fail(e, "cudaMalloc(x)"); }
        x_cap = x_floats;
    }
    if (y_floats > y_cap) {
        if (y_dev) cudaFree(y_dev);
        y_dev = nullptr;
        cudaError_t e = cudaMalloc(&y_dev, y_floats * sizeof(float) + kPad);
        if (e != cudaSuccess) { y_cap = 0; return cuda_fail(e, "cudaMalloc(y)"); }
        y_cap = y_floats;
    }
    return LARQL_OK;
}

int Ctx::ensure_scratch(size_t bytes) {
    if (bytes <= scratch_cap) return LARQL_OK;
    cudaStreamSynchronize(stream);
    if (scratch) cudaFree(scratch);
    scratch = nullptr;
    scratch_cap = 0;
    cudaError_t e = cudaMalloc(&scratch, bytes + kPad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(scratch)");
    scratch_cap = bytes;
    return LARQL_OK;
}

const CUtensorMap* Ctx::q4k_map(Weight* w, int H) {
    for (int i = 0; i < Weight::kMaps; ++i)
        if (w->tmap_h[i] == H) return &w->tmap[i];
    if (!encode_tiled) return nullptr;
    const int slot = w->tmap_next;
    w->tmap_h[slot] = 0;
    const int fmt = w->format == LARQL_FMT_Q4_0 ? 1
                    : w->format == LARQL_FMT_Q4_K_GGUF ? 5
                    : w->format == LARQL_FMT_Q4_K_GGUF_LLAMA ? 6
                    : (w->format == LARQL_FMT_Q8_0_GGUF ? 2 : (w->format == LARQL_FMT_Q6_K ? 4 : 0));
    if (mma_encode_map(encode_tiled, w->dev, static_cast<int>(w->rows), static_cast<int>(w->cols), fmt, H,
                       &w->tmap[slot]) != 0)
        return nullptr;
    w->tmap_h[slot] = H;
    w->tmap_next = (slot + 1) % Weight::kMaps;
    return &w->tmap[slot];
}

int Ctx::ensure_aux(size_t bytes) {
    if (bytes <= aux_cap) return LARQL_OK;
    if (aux) cudaFree(aux);
    aux = nullptr;
    aux_cap = 0;
    cudaError_t e = cudaMalloc(&aux, bytes + kPad);
    if (e != cudaSuccess) return cuda_fail(e, "aux buffer");
    aux_cap = bytes;
    return LARQL_OK;
}

int Ctx::ensure_tickets(size_t n) {
    if (n <= tickets_cap) return LARQL_OK;
    if (tickets) cudaFree(tickets);
    tickets = nullptr;
    tickets_cap = 0;
    const size_t cap = n < 4096 ? 4096 : n;
    cudaError_t e = cudaMalloc(&tickets, cap * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(tickets, 0, cap * sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "split-K ticket buffer");
    tickets_cap = cap;
    return LARQL_OK;
}

// Reads (and clears) the device status word after the stream has drained.
int Ctx::finish() {
    cudaError_t e = cudaMemcpyAsync(status_host, status_dev, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e, "status copy");
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    const int st = *status_host;
    if (st != 0) {
        // a kernel that gave up may have left split-K tickets half counted
        if (tickets) cudaMemsetAsync(tickets, 0, tickets_cap * sizeof(int), stream);
        if (pf_flags) cudaMemsetAsync(pf_flags, 0, static_cast<size_t>(num_sms) * 4 * sizeof(int), stream);
        cudaMemsetAsync(status_dev, 0, sizeof(int), stream);
        cudaStreamSynchronize(stream);
        return fail(st & 0xFFFF, "device reported status %d at site %d", st & 0xFFFF, st >> 16);
    }
    return LARQL_OK;
}

Weight* Ctx::find(uint64_t h) {
    auto it = weights.find(h);
    return it == weights.end() ? nullptr : &it->second;
}

int Ctx::add_weight(const void* src, bool src_is_device, size_t nbytes, const float* scales, bool scales_device,
                    int format, size_t rows, size_t cols, uint64_t* handle) {
    if (!src || !handle || rows == 0 || cols == 0) return fail(LARQL_ERR_INVALID_ARG, "null weight or zero shape");
    const size_t blk = format_block(format);
    if (blk == 0) return fail(LARQL_ERR_UNSUPPORTED, "unknown weight format %d", format);
    if (cols % blk) return fail(LARQL_ERR_BAD_SHAPE, "cols=%zu is not a multiple of the %zu-value block", cols, blk);
    const size_t need = format_bytes(format, rows, cols);
    if (nbytes < need)
        return fail(LARQL_ERR_BAD_SHAPE, "weight has %zu bytes, a [%zu x %zu] matrix of format %d needs %zu", nbytes,
                    rows, cols, format, need);
    if (format == LARQL_FMT_Q8_0 && !scales) return fail(LARQL_ERR_INVALID_ARG, "Q8_0 compute layout needs scales");
    Weight w;
    w.format = format;
    w.rows = rows;
    w.cols = cols;
    w.nbytes = need;
    w.key = src;
    w.key_len = nbytes;
    cudaError_t e = cudaMalloc(&w.dev, need + kPad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight)");
    w.owned = true;
    e = cudaMemsetAsync(static_cast<uint8_t*>(w.dev) + need, 0, kPad, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w.dev, src, need, src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess && scales) {
        const size_t sb = rows * cols / 32 * sizeof(float);
        e = cudaMalloc(&w.scales_dev, sb + kPad);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(w.scales_dev, scales, sb,
                                scales_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
    }
    // half.rs decodes subnormals to half their IEEE value; store that value so IEEE consumers agree
    if (e == cudaSuccess && format == LARQL_FMT_F16_HALFRS)
        e = launch_gate_halfrs_fixup(static_cast<uint16_t*>(w.dev), rows * cols, status_dev + 1, &w.gate_factor,
                                     stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        cudaFree(w.dev);
        if (w.scales_dev) cudaFree(w.scales_dev);
        return cuda_fail(e, "weight upload");
    }
    const uint64_t h = next_handle++;
    weights.emplace(h, w);
    if (!src_is_device) by_ptr[{reinterpret_cast<uintptr_t>(src), nbytes}] = h;
    *handle = h;
    return LARQL_OK;
}

// A device weight whose rows are the concatenation of `parts` (same format and
// cols; not entered in the (pointer, length) registry).
int Ctx::add_weight_parts(const void* const* parts, const size_t* part_bytes, int nparts, bool src_is_device,
                          int format, size_t rows, size_t cols, uint64_t* handle) {
    const size_t need = format_bytes(format, rows, cols);
    size_t total = 0;
    for (int i = 0; i < nparts; ++i) total += part_bytes[i];
    if (total != need) return fail(LARQL_ERR_BAD_SHAPE, "fused weight has %zu bytes, needs %zu", total, need);
    Weight w;
    w.format = format;
    w.rows = rows;
    w.cols = cols;
    w.nbytes = need;
    cudaError_t e = cudaMalloc(&w.dev, need + kPad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(fused weight)");
    w.owned = true;
    e = cudaMemsetAsync(static_cast<uint8_t*>(w.dev) + need, 0, kPad, stream);
    size_t off = 0;
    for (int i = 0; i < nparts && e == cudaSuccess; ++i) {
        if (!parts[i]) e = cudaErrorInvalidValue;
        else
            e = cudaMemcpyAsync(static_cast<uint8_t*>(w.dev) + off, parts[i], part_bytes[i],
                                src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
        off += part_bytes[i];
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        cudaFree(w.dev);
        return e == cudaErrorInvalidValue ? fail(LARQL_ERR_INVALID_ARG, "null weight part") : cuda_fail(e, "weight upload");
    }
    const uint64_t h = next_handle++;
    weights.emplace(h, w);
    *handle = h;
    return LARQL_OK;
}

void Ctx::release_handle(uint64_t h) {
    auto it = weights.find(h);
    if (it == weights.end()) return;
    if (it->second.owned) cudaFree(it->second.dev);
    if (it->second.scales_dev) cudaFree(it->second.scales_dev);
    if (it->second.pf_dev) cudaFree(it->second.pf_dev);
    weights.erase(it);
}

// Q4_K input-column slice [c0, c1) (multiples of 256) of a rows x cols weight: whole blocks, one pitched copy.
int Ctx::add_weight_cols(const void* src, bool src_is_device, size_t rows, size_t cols, size_t c0, size_t c1,
                         uint64_t* handle) {
    if (!src) return fail(LARQL_ERR_INVALID_ARG, "null weight");
    if (c0 % 256 || c1 % 256 || c1 <= c0 || c1 > cols || cols % 256)
        return fail(LARQL_ERR_BAD_SHAPE, "column slice [%zu, %zu) of %zu", c0, c1, cols);
    const size_t sp = cols / 256 * 148, wp = (c1 - c0) / 256 * 148;
    Weight w;
    w.format = LARQL_FMT_Q4_K;
    w.rows = rows;
    w.cols = c1 - c0;
    w.nbytes = rows * wp;
    cudaError_t e = cudaMalloc(&w.dev, w.nbytes + kPad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight slice)");
    w.owned = true;
    e = cudaMemsetAsync(static_cast<uint8_t*>(w.dev) + w.nbytes, 0, kPad, stream);
    if (e == cudaSuccess)
        e = cudaMemcpy2DAsync(w.dev, wp, static_cast<const uint8_t*>(src) + c0 / 256 * 148, sp, wp, rows,
                              src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        cudaFree(w.dev);
        return cuda_fail(e, "weight slice upload");
    }
    const uint64_t h = next_handle++;
    weights.emplace(h, w);
    *handle = h;
    return LARQL_OK;
}

// One rank's share of a layer for tensor-parallel decode (heads and FFN rows split over `world`).
int Ctx::layer_register_shard(const larql_cuda_layer_desc* d, size_t hidden, size_t inter, size_t nq, size_t nkv,
                              size_t hd, size_t rank, size_t world, bool src_is_device, uint64_t* handle) {
    if (!d || !handle) return fail(LARQL_ERR_INVALID_ARG, "null layer description");
    if (world == 0 || rank >= world) return fail(LARQL_ERR_INVALID_ARG, "rank %zu of %zu", rank, world);
    if (hd != 128 || nkv == 0 || nq % nkv || nq / nkv > 8 || (nq / nkv) & (nq / nkv - 1))
        return fail(LARQL_ERR_UNSUPPORTED, "decode needs head_dim 128 and 1, 2, 4 or 8 query heads per KV head");
    if (nkv % world || hidden % 256 || hidden == 0 || inter % (256 * world) || inter == 0 ||
        (nq / world * hd) % 256)
        return fail(LARQL_ERR_BAD_SHAPE, "shard of %zu q / %zu kv heads, FFN %zu over %zu ranks", nq, nkv, inter, world);
    if (!d->input_norm || !d->post_attn_norm || !d->wq || !d->wk || !d->wv || !d->wo || !d->gate || !d->up ||
        !d->down)
        return fail(LARQL_ERR_INVALID_ARG, "null weight in the layer description");
    const size_t nq_l = nq / world, nkv_l = nkv / world, inter_l = inter / world;
    const size_t qd_l = nq_l * hd, kvd_l = nkv_l * hd, rb = hidden / 256 * 148;
    Layer L;
    L.hidden = hidden;
    L.inter = inter_l;
    L.nq = nq_l;
    L.nkv = nkv_l;
    L.hd = hd;
    L.offset = d->norm_offset;
    L.eps = d->eps;
    L.attn_scale = d->attn_scale;
    L.world = world;
    const void* qkv_p[3] = {d->wq + rank * qd_l * rb, d->wk + rank * kvd_l * rb, d->wv + rank * kvd_l * rb};
    const size_t qkv_b[3] = {qd_l * rb, kvd_l * rb, kvd_l * rb};
    int rc = add_weight_parts(qkv_p, qkv_b, 3, src_is_device, LARQL_FMT_Q4_K, qd_l + 2 * kvd_l, hidden, &L.qkv);
    if (!rc) rc = add_weight_cols(d->wo, src_is_device, hidden, nq * hd, rank * qd_l, (rank + 1) * qd_l, &L.o);
    const void* gu_p[2] = {d->gate + rank * inter_l * rb, d->up + rank * inter_l * rb};
    const size_t gu_b[2] = {inter_l * rb, inter_l * rb};
    if (!rc) rc = add_weight_parts(gu_p, gu_b, 2, src_is_device, LARQL_FMT_Q4_K, 2 * inter_l, hidden, &L.gu);
    if (!rc) rc = add_weight_cols(d->down, src_is_device, hidden, inter, rank * inter_l, (rank + 1) * inter_l, &L.down);
    if (!rc) {
        cudaError_t e = cudaMalloc(&L.norms, 2 * hidden * sizeof(float));
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(L.norms, d->input_norm, hidden * sizeof(float),
                                src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(L.norms + hidden, d->post_attn_norm, hidden * sizeof(float),
                                src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "norm upload");
    }
    if (rc) {
        for (uint64_t h : {L.qkv, L.o, L.gu, L.down}) release_handle(h);
        if (L.norms) cudaFree(L.norms);
        return rc;
    }
    const uint64_t h = next_handle++;
    layers.emplace(h, L);
    *handle = h;
    return LARQL_OK;
}

int Ctx::layer_register(const larql_cuda_layer_desc* d, size_t hidden, size_t inter, size_t nq, size_t nkv,
                        size_t hd, bool src_is_device, uint64_t* handle) {
    if (!d || !handle) return fail(LARQL_ERR_INVALID_ARG, "null layer description");
    if (hd != 128 || nkv == 0 || nq % nkv || nq / nkv > 8 || (nq / nkv) & (nq / nkv - 1))
        return fail(LARQL_ERR_UNSUPPORTED, "decode needs head_dim 128 and 1, 2, 4 or 8 query heads per KV head");
    if (hidden % 256 || inter % 256 || (nq * hd) % 256 || hidden == 0 || inter == 0)
        return fail(LARQL_ERR_BAD_SHAPE, "hidden, inter and nq*head_dim must be multiples of 256");
    if (!d->input_norm || !d->post_attn_norm) return fail(LARQL_ERR_INVALID_ARG, "null norm weights");
    const size_t qd = nq * hd, kvd = nkv * hd;
    Layer L;
    L.hidden = hidden;
    L.inter = inter;
    L.nq = nq;
    L.nkv = nkv;
    L.hd = hd;
    L.offset = d->norm_offset;
    L.eps = d->eps;
    L.attn_scale = d->attn_scale;
    const void* qkv_p[3] = {d->wq, d->wk, d->wv};
    const size_t qkv_b[3] = {format_bytes(LARQL_FMT_Q4_K, qd, hidden), format_bytes(LARQL_FMT_Q4_K, kvd, hidden),
                             format_bytes(LARQL_FMT_Q4_K, kvd, hidden)};
    int rc = add_weight_parts(qkv_p, qkv_b, 3, src_is_device, LARQL_FMT_Q4_K, qd + 2 * kvd, hidden, &L.qkv);
    const void* o_p[1] = {d->wo};
    const size_t o_b[1] = {format_bytes(LARQL_FMT_Q4_K, hidden, qd)};
    if (!rc) rc = add_weight_parts(o_p, o_b, 1, src_is_device, LARQL_FMT_Q4_K, hidden, qd, &L.o);
    const void* gu_p[2] = {d->gate, d->up};
    const size_t gu_b[2] = {format_bytes(LARQL_FMT_Q4_K, inter, hidden), format_bytes(LARQL_FMT_Q4_K, inter, hidden)};
    if (!rc) rc = add_weight_parts(gu_p, gu_b, 2, src_is_device, LARQL_FMT_Q4_K, 2 * inter, hidden, &L.gu);
    const void* d_p[1] = {d->down};
    const size_t d_b[1] = {format_bytes(LARQL_FMT_Q4_K, hidden, inter)};
    if (!rc) rc = add_weight_parts(d_p, d_b, 1, src_is_device, LARQL_FMT_Q4_K, hidden, inter, &L.down);
    if (!rc) {
        cudaError_t e = cudaMalloc(&L.norms, 2 * hidden * sizeof(float));
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(L.norms, d->input_norm, hidden * sizeof(float),
                                src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(L.norms + hidden, d->post_attn_norm, hidden * sizeof(float),
                                src_is_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "norm upload");
    }
    if (rc) {
        for (uint64_t h : {L.qkv, L.o, L.gu, L.down}) release_handle(h);
        if (L.norms) cudaFree(L.norms);
        return rc;
    }
    const uint64_t h = next_handle++;
    layers.emplace(h, L);
    *handle = h;
    return LARQL_OK;
}

int Ctx::kv_init(size_t n_layers, size_t max_seq, size_t nkv, size_t hd) {
    if (n_layers == 0 || max_seq == 0 || nkv == 0 || hd != 128)
        return fail(LARQL_ERR_BAD_SHAPE, "kv cache needs layers, max_seq, nkv > 0 and head_dim 128");
    for (auto& l : kv) {
        if (l.k) cudaFree(l.k);
        if (l.v) cudaFree(l.v);
    }
    kv.assign(n_layers, KvLayer{});
    const size_t bytes = max_seq * nkv * hd * sizeof(__half);
    for (auto& l : kv) {
        cudaError_t e = cudaMalloc(&l.k, bytes);
        if (e == cudaSuccess) e = cudaMalloc(&l.v, bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(l.k, 0, bytes, stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(l.v, 0, bytes, stream);
        if (e != cudaSuccess) return cuda_fail(e, "kv cache allocation");
    }
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "kv init");
    kv_max_seq = max_seq;
    kv_nkv = nkv;
    kv_hd = hd;
    kv_len = 0;
    return LARQL_OK;
}

// One token through layers lh[0..n) at position pos (layer i uses KV layer i); x updated in place.
// Checks the layers against the KV cache and grows the per-token workspace for the largest of them;
// ws[0..6] = h, o, dd, q|k|v, attn, gate|up, act.
int Ctx::decode_workspace(const uint64_t* lh, size_t n, size_t pos, float** ws, double** ss) {
    if (n > kv.size()) return fail(LARQL_ERR_BAD_SHAPE, "%zu layers but the kv cache has %zu", n, kv.size());
    if (pos >= kv_max_seq) return fail(LARQL_ERR_BAD_SHAPE, "position %zu past the kv cache (%zu)", pos, kv_max_seq);
    size_t hid = 0, inter = 0, qkvd = 0, qd = 0;
    for (size_t i = 0; i < n; ++i) {
        auto it = layers.find(lh[i]);
        if (it == layers.end()) return fail(LARQL_ERR_NOT_FOUND, "unknown layer handle");
        const Layer& L = it->second;
        if (L.nkv != kv_nkv || L.hd != kv_hd) return fail(LARQL_ERR_BAD_SHAPE, "layer heads do not match the kv cache");
        hid = std::max(hid, L.hidden);
        inter = std::max(inter, L.inter);
        qd = std::max(qd, L.nq * L.hd);
        qkvd = std::max(qkvd, (L.nq + 2 * L.nkv) * L.hd);
    }
    auto up16 = [](size_t v) { return (v + 15) & ~size_t(15); };
    const size_t ssf = up16((hid + 15) / 16 * 2);  // floats holding one array of f64 sums of squares
    const size_t need = up16(hid) * 3 + up16(qkvd) + up16(qd) + up16(2 * inter) + up16(inter) + 2 * ssf;
    if (need > dws_cap) {
        if (dws) cudaFree(dws);
        dws = nullptr;
        dws_cap = 0;
        cudaError_t e = cudaMalloc(&dws, need * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "decode workspace");
        dws_cap = need;
    }
    ws[0] = dws;
    ws[1] = ws[0] + up16(hid);
    ws[2] = ws[1] + up16(hid);
    ws[3] = ws[2] + up16(hid);
    ws[4] = ws[3] + up16(qkvd);
    ws[5] = ws[4] + up16(qd);
    ws[6] = ws[5] + up16(2 * inter);
    if (ss) {
        ss[0] = reinterpret_cast<double*>(ws[6] + up16(inter));
        ss[1] = reinterpret_cast<double*>(ws[6] + up16(inter) + ssf);
    }
    return LARQL_OK;
}

// A weight the batch-1 MMA matvec serves, hence one the decode fusions apply to.
bool Ctx::fusable(Weight* w) {
    if (!w || w->format != LARQL_FMT_Q4_K) return false;
    Q4kRoute r;
    return route_q4k(w, 1, &r) == LARQL_OK && r.kind == Q4kRoute::kMma;
}

int Ctx::matvec_fused_dev(Weight* w, const float* x, float* y, const MmaFuse& f, cudaStream_t s) {
    Q4kRoute r;
    int rc = route_q4k(w, 1, &r);
    if (rc) return rc;
    if (r.kind != Q4kRoute::kMma) return fail(LARQL_ERR_UNSUPPORTED, "fused matvec needs the MMA route");
    const size_t pf = q4k_mma_partial_floats(r.mp);
    rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
    if (!rc) rc = ensure_tickets(static_cast<size_t>(r.mp.ntiles));
    if (rc) return rc;
    cudaError_t e =
        launch_q4k_mma_fused(*r.map, x, y, reinterpret_cast<float*>(scratch), tickets, r.mp, f, status_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "fused matvec launch");
    return LARQL_OK;
}

// One token through every layer in one persistent launch (decode_persist.cu).  Returns -1 (nothing done) where
// the layers are not served: shapes that differ between layers, a sharded layer, a projection that is not Q4_K,
// sizes the kernel does not take, or a device where its grid cannot be resident at once; the caller then runs the
// per-kernel pipeline.  The per-layer blocks and tensor
// maps are uploaded when the layer list (or its KV cache) changes, which must happen outside stream capture.
int Ctx::decode_persist_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, cudaStream_t s) {
    const Layer& L0 = layers.find(lh[0])->second;
    for (size_t i = 0; i < n; ++i) {
        const Layer& L = layers.find(lh[i])->second;
        if (L.world != 1 || L.hidden != L0.hidden || L.inter != L0.inter || L.nq != L0.nq || L.nkv != L0.nkv ||
            L.hd != 128)
            return -1;
        for (uint64_t h : {L.qkv, L.o, L.gu, L.down}) {
            Weight* w = find(h);
            if (!w || w->format != LARQL_FMT_Q4_K) return -1;
        }
    }
    if (!encode_tiled) return -1;
    DecodePersistPlan plan;
    if (decode_persist_plan(static_cast<int>(n), static_cast<int>(L0.hidden), static_cast<int>(L0.inter),
                            static_cast<int>(L0.nq), static_cast<int>(L0.nkv), static_cast<int>(pos), num_sms,
                            static_cast<double>(rope_base), &plan))
        return -1;
    // a grid that cannot be resident at once (the device shared or partitioned) takes the pipeline instead
    {
        const cudaError_t ce = decode_persist_check(plan);
        if (ce == cudaErrorCooperativeLaunchTooLarge) return -1;
        if (ce != cudaSuccess) return cuda_fail(ce, "persistent decode occupancy");
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(s, &cs);
    if (e != cudaSuccess) return cuda_fail(e, "capture status");
    const bool capturing = cs != cudaStreamCaptureStatusNone;
    const size_t lb = decode_persist_layer_bytes();
    std::vector<unsigned char> lay(n * lb);
    for (size_t i = 0; i < n; ++i) {
        const Layer& L = layers.find(lh[i])->second;
        decode_persist_layer_fill(lay.data() + i * lb, L.norms, kv[i].k, kv[i].v, L.offset, L.eps, L.attn_scale);
    }
    if (pd.handles.size() != n || !std::equal(pd.handles.begin(), pd.handles.end(), lh) || pd.lay_host != lay) {
        if (capturing) return fail(LARQL_ERR_UNSUPPORTED, "run the persistent decode once before capturing it");
        std::vector<CUtensorMap> maps(4 * n);
        for (size_t i = 0; i < n; ++i) {
            const Layer& L = layers.find(lh[i])->second;
            const uint64_t hs[4] = {L.qkv, L.o, L.gu, L.down};
            for (int m = 0; m < 4; ++m) {
                Weight* w = find(hs[m]);
                if (decode_persist_map(encode_tiled, w->dev, static_cast<int>(w->rows), static_cast<int>(w->cols),
                                       &maps[4 * i + m]))
                    return fail(LARQL_ERR_CUDA, "tensor map of a decode weight");
            }
        }
        if (pd.lay_dev) cudaFree(pd.lay_dev);
        if (pd.maps_dev) cudaFree(pd.maps_dev);
        pd.lay_dev = nullptr;
        pd.maps_dev = nullptr;
        pd.handles.clear();
        pd.lay_host.clear();
        e = cudaMalloc(&pd.lay_dev, lay.size());
        if (e == cudaSuccess) e = cudaMalloc(&pd.maps_dev, maps.size() * sizeof(CUtensorMap));
        if (e == cudaSuccess) e = cudaMemcpy(pd.lay_dev, lay.data(), lay.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(pd.maps_dev, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "persistent decode set-up");
        pd.handles.assign(lh, lh + n);
        pd.lay_host = lay;
    }
    // workspace: alternate residual, the four projections' partial sums, attention partials for the longest
    // cache, attention output, barrier; every piece 256-byte aligned
    const size_t nch_max = (kv_max_seq + 127) / 128;
    const size_t att_items = L0.nkv * nch_max, reps = L0.nq / L0.nkv;
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    size_t off[10], cur = 0;
    const size_t sz[10] = {L0.hidden * 4,
                           static_cast<size_t>(plan.nparts[0]) * plan.N[0] * 4,
                           static_cast<size_t>(plan.nparts[1]) * plan.N[1] * 4,
                           static_cast<size_t>(plan.nparts[2]) * plan.N[2] * 4,
                           static_cast<size_t>(plan.nparts[3]) * plan.N[3] * 4,
                           att_items * reps * 128 * 4,
                           att_items * reps * 4,
                           att_items * reps * 8,
                           L0.nq * 128 * 4,
                           16};
    for (int i = 0; i < 10; ++i) {
        off[i] = cur;
        cur += up(sz[i]);
    }
    if (cur > pd.ws_cap) {
        if (capturing) return fail(LARQL_ERR_UNSUPPORTED, "run the persistent decode once before capturing it");
        if (pd.ws) cudaFree(pd.ws);
        pd.ws = nullptr;
        pd.ws_cap = 0;
        e = cudaMalloc(&pd.ws, cur);
        if (e != cudaSuccess) return cuda_fail(e, "persistent decode workspace");
        pd.ws_cap = cur;
    }
    DecodePersistBufs bufs{};
    bufs.x = x;
    bufs.xalt = reinterpret_cast<float*>(pd.ws + off[0]);
    for (int i = 0; i < 4; ++i) bufs.part[i] = reinterpret_cast<float*>(pd.ws + off[1 + i]);
    bufs.att_acc = reinterpret_cast<float*>(pd.ws + off[5]);
    bufs.att_m = reinterpret_cast<float*>(pd.ws + off[6]);
    bufs.att_l = reinterpret_cast<double*>(pd.ws + off[7]);
    bufs.attn = reinterpret_cast<float*>(pd.ws + off[8]);
    bufs.bar = reinterpret_cast<unsigned*>(pd.ws + off[9]);
    e = launch_decode_persist(plan, pd.lay_dev, pd.maps_dev, bufs, status_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "persistent decode launch");
    return LARQL_OK;
}

int Ctx::decode_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, cudaStream_t s) {
    if (n == 0) return LARQL_OK;
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail(LARQL_ERR_INVALID_ARG, "x must be 16-byte aligned");
    for (size_t i = 0; i < n; ++i) {
        auto it = layers.find(lh[i]);
        if (it != layers.end() && it->second.world > 1)
            return fail(LARQL_ERR_INVALID_ARG, "a sharded layer needs larql_cuda_decode_token_sharded_dev");
    }
    float* ws[7];
    double* ss[2];
    int rc0 = decode_workspace(lh, n, pos, ws, ss);
    if (rc0) return rc0;
    if (decode_persist) {
        const int rp = decode_persist_dev(lh, n, x, pos, rope_base, s);
        if (rp >= 0) return rp;
    }
    float *h = ws[0], *o = ws[1], *dd = ws[2], *qkv = ws[3], *attn = ws[4], *gu = ws[5], *act = ws[6];
    cudaError_t e = cudaSuccess;
    int rc = LARQL_OK;
    // Fusions (every projection on the batch-1 MMA matvec; bits of fuse_decode):
    //   2  norm: the O and down matvecs add their output to x in place and leave f64 sums of squares per
    //      16 values; the Q|K|V and gate|up matvecs normalise x from those while building their x tables
    //      (no RMSNorm kernels, no final residual add);
    //   1  SiLU: the down matvec builds its x tables from silu(gate) * up (no SiLU kernel).
    int fm = fuse_decode;
    for (size_t i = 0; i < n && fm; ++i) {
        const Layer& L = layers.find(lh[i])->second;
        if (!(fusable(find(L.qkv)) && fusable(find(L.o)) && fusable(find(L.gu)) && fusable(find(L.down)))) fm = 0;
    }
    const bool fn = (fm & 2) != 0, fs = (fm & 1) != 0;
    if (fn) e = launch_decode_sumsq16(x, static_cast<int>(layers.find(lh[0])->second.hidden), ss[0], s);
    for (size_t i = 0; i < n && !rc && e == cudaSuccess; ++i) {
        const Layer& L = layers.find(lh[i])->second;
        const int H = static_cast<int>(L.hidden);
        MmaFuse fq{};
        fq.pro = 1;
        fq.ss_in = ss[0];
        fq.nw = L.norms;
        fq.offset = L.offset;
        fq.eps = L.eps;
        if (fn) {
            rc = matvec_fused_dev(find(L.qkv), x, qkv, fq, s);
        } else {
            // residual of the previous layer's FFN added before this layer's input norm
            e = launch_decode_rmsnorm(x, i ? dd : nullptr, L.norms, L.offset, L.eps, H, h, s);
            if (e == cudaSuccess) rc = matvec_dev(find(L.qkv), h, 1, qkv, s);
        }
        if (!rc && e == cudaSuccess)
            e = launch_decode_attention(qkv, static_cast<int>(L.nq), static_cast<int>(L.nkv), static_cast<int>(L.hd),
                                        static_cast<int>(pos), L.attn_scale, static_cast<double>(rope_base), kv[i].k,
                                        kv[i].v, attn, s);
        if (fn) {
            MmaFuse fo{};
            fo.epi = 1;
            fo.ss_out = ss[1];
            if (!rc && e == cudaSuccess) rc = matvec_fused_dev(find(L.o), attn, x, fo, s);
            fq.ss_in = ss[1];
            fq.nw = L.norms + L.hidden;
            if (!rc && e == cudaSuccess) rc = matvec_fused_dev(find(L.gu), x, gu, fq, s);
        } else {
            if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.o), attn, 1, o, s);
            if (!rc && e == cudaSuccess) e = launch_decode_rmsnorm(x, o, L.norms + L.hidden, L.offset, L.eps, H, h, s);
            if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.gu), h, 1, gu, s);
        }
        if (fn || fs) {
            MmaFuse fd{};
            fd.pro = fs ? 2 : 0;
            fd.epi = fn ? 1 : 0;
            fd.ss_out = ss[0];
            if (!fs && !rc && e == cudaSuccess) e = launch_decode_silu_mul(gu, static_cast<int>(L.inter), act, s);
            if (!rc && e == cudaSuccess) rc = matvec_fused_dev(find(L.down), fs ? gu : act, fn ? x : dd, fd, s);
        } else {
            if (!rc && e == cudaSuccess) e = launch_decode_silu_mul(gu, static_cast<int>(L.inter), act, s);
            if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.down), act, 1, dd, s);
        }
    }
    if (!fn && !rc && e == cudaSuccess)
        e = launch_decode_add(x, dd, static_cast<int>(layers.find(lh[n - 1])->second.hidden), s);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    return LARQL_OK;
}

// One token through sharded layers: every rank computes its heads' attention and its FFN rows; the O and
// down projections leave partial sums in `red`, which `fn` all-reduces across ranks on the stream.
int Ctx::decode_sharded_dev(const uint64_t* lh, size_t n, float* x, size_t pos, float rope_base, float* red,
                            larql_cuda_reduce_fn fn, void* user, cudaStream_t s) {
    if (n == 0) return LARQL_OK;
    if (!fn || !red) return fail(LARQL_ERR_INVALID_ARG, "a sharded token needs a reduction buffer and callback");
    if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(red) % 16)
        return fail(LARQL_ERR_INVALID_ARG, "x and the reduction buffer must be 16-byte aligned");
    float* ws[7];
    int rc = decode_workspace(lh, n, pos, ws);
    if (rc) return rc;
    float *h = ws[0], *qkv = ws[3], *attn = ws[4], *gu = ws[5], *act = ws[6];
    cudaError_t e = cudaSuccess;
    size_t H = 0;
    for (size_t i = 0; i < n && !rc && e == cudaSuccess; ++i) {
        const Layer& L = layers.find(lh[i])->second;
        H = L.hidden;
        // the previous layer's all-reduced down projection is the residual added before this layer's norm
        e = launch_decode_rmsnorm(x, i ? red : nullptr, L.norms, L.offset, L.eps, static_cast<int>(H), h, s);
        if (e == cudaSuccess) rc = matvec_dev(find(L.qkv), h, 1, qkv, s);
        if (!rc && e == cudaSuccess)
            e = launch_decode_attention(qkv, static_cast<int>(L.nq), static_cast<int>(L.nkv), static_cast<int>(L.hd),
                                        static_cast<int>(pos), L.attn_scale, static_cast<double>(rope_base), kv[i].k,
                                        kv[i].v, attn, s);
        if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.o), attn, 1, red, s);
        if (!rc && e == cudaSuccess && fn(user, red, H, s) != 0)
            rc = fail(LARQL_ERR_NCCL, "reduction callback failed after the O projection of layer %zu", i);
        if (!rc && e == cudaSuccess) e = launch_decode_rmsnorm(x, red, L.norms + H, L.offset, L.eps, static_cast<int>(H), h, s);
        if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.gu), h, 1, gu, s);
        if (!rc && e == cudaSuccess) e = launch_decode_silu_mul(gu, static_cast<int>(L.inter), act, s);
        if (!rc && e == cudaSuccess) rc = matvec_dev(find(L.down), act, 1, red, s);
        if (!rc && e == cudaSuccess && fn(user, red, H, s) != 0)
            rc = fail(LARQL_ERR_NCCL, "reduction callback failed after the down projection of layer %zu", i);
    }
    if (!rc && e == cudaSuccess) e = launch_decode_add(x, red, static_cast<int>(H), s);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    return LARQL_OK;
}

// 2^-e with every dequantized value of the Q4_K weight below 2^14 after scaling
// (computed once from the super-block headers: |w| <= 945 |d| + 15 |dmin|).
int Ctx::q4k_f16_scale(Weight* w, float* scale) {
    if (w->f16_scale == 0.f) {
        unsigned int* work = reinterpret_cast<unsigned int*>(status_dev + 2);
        cudaError_t e = launch_q4k_abs_bound(static_cast<const uint8_t*>(w->dev), w->rows * w->cols / 256, work, stream);
        unsigned int bits = 0;
        if (e == cudaSuccess) e = cudaMemcpyAsync(&bits, work, sizeof(bits), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "weight bound");
        float bound;
        memcpy(&bound, &bits, sizeof(bound));
        int ex = 0;
        if (bound > 0.f && std::isfinite(bound)) ex = static_cast<int>((bits >> 23) & 0xFF) - 126;  // bound < 2^ex
        const int e2 = std::min(100, std::max(-100, ex - 14));
        w->f16_scale = std::ldexp(1.0f, -e2);
    }
    *scale = w->f16_scale;
    return LARQL_OK;
}

// The prefill panels of a Q4_K weight (q4k_prefill_pack: per 128-row tile and
// super-block, word-major f16 scale/min pairs and nibbles), built once.
int Ctx::q4k_prefill_panels(Weight* w, float* scale, const uint8_t** panels) {
    int rc = q4k_f16_scale(w, scale);
    if (rc) return rc;
    if (!w->pf_dev) {
        const size_t bytes = q4k_prefill_panel_bytes(w->rows, w->cols);
        cudaError_t e = cudaMalloc(&w->pf_dev, bytes);
        if (e != cudaSuccess) {
            w->pf_dev = nullptr;
            return cuda_fail(e, "prefill panel allocation");
        }
        e = launch_q4k_prefill_pack(static_cast<const uint8_t*>(w->dev), static_cast<int>(w->rows),
                                    static_cast<int>(w->cols), *scale, w->pf_dev, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) {
            cudaFree(w->pf_dev);
            w->pf_dev = nullptr;
            return cuda_fail(e, "prefill panel packing");
        }
    }
    *panels = w->pf_dev;
    return LARQL_OK;
}

// Stream-K workspace of the prefill GEMMs: part_floats partial sums and the
// [num_sms][4] slot flags (zeroed once; the kernels leave them zero).
int Ctx::ensure_prefill_ws(size_t part_floats) {
    if (!pf_flags) {
        cudaError_t e = cudaMalloc(&pf_flags, static_cast<size_t>(num_sms) * 4 * sizeof(int));
        if (e == cudaSuccess) e = cudaMemsetAsync(pf_flags, 0, static_cast<size_t>(num_sms) * 4 * sizeof(int), stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) {
            if (pf_flags) cudaFree(pf_flags);
            pf_flags = nullptr;
            return cuda_fail(e, "prefill flags");
        }
    }
    if (part_floats > pf_part_cap) {
        if (pf_part) cudaFree(pf_part);
        pf_part = nullptr;
        pf_part_cap = 0;
        cudaError_t e = cudaMalloc(&pf_part, part_floats * sizeof(float));
        if (e != cudaSuccess) {
            pf_part = nullptr;
            return cuda_fail(e, "prefill workspace");
        }
        pf_part_cap = part_floats;
    }
    return LARQL_OK;
}

// Y[t][n] = W[n] . X[t] for t < M (tcgen05, f16 dequantized tiles, f32 accumulate).
int Ctx::gemm_q4k_dev(Weight* w, const float* x, size_t M, float* y, cudaStream_t s) {
    if (w->format != LARQL_FMT_Q4_K) return fail(LARQL_ERR_UNSUPPORTED, "Q4_K GEMM needs a Q4_K weight");
    if (M == 0) return LARQL_OK;
    if (!encode_tiled) return fail(LARQL_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    PrefillPlan p;
    if (M > (1u << 20) || w->rows > 0x7fffffff || w->cols > 0x7fffffff ||
        !prefill_make_plan(static_cast<int>(w->rows), static_cast<int>(w->cols), static_cast<int>(M), false, num_sms, &p))
        return fail(LARQL_ERR_UNSUPPORTED, "Q4_K GEMM shape %zu x %zu x %zu not supported", w->rows, w->cols, M);
    float ws;
    const uint8_t* pw = nullptr;
    int rc = q4k_prefill_panels(w, &ws, &pw);
    if (!rc) rc = ensure_prefill_ws(prefill_part_floats(p));
    if (rc) return rc;
    const size_t rows = prefill_tokens_padded(p);
    const size_t xh_bytes = (rows * w->cols * 2 + 255) & ~size_t(255);
    rc = ensure_scratch(xh_bytes + rows * 4 + 256);
    if (rc) return rc;
    __half* xh = reinterpret_cast<__half*>(scratch);
    float* xs = reinterpret_cast<float*>(scratch + xh_bytes);
    cudaError_t e = launch_prefill_x_prep(x, static_cast<int>(M), static_cast<int>(w->cols), static_cast<int>(rows), xh, xs, s);
    CUtensorMap xmap;
    if (e == cudaSuccess && prefill_encode_xmap(encode_tiled, xh, static_cast<int>(rows), static_cast<int>(w->cols),
                                                std::min(256, p.NTOK), &xmap) != 0)
        return fail(LARQL_ERR_CUDA, "activation tensor map encoding failed");
    if (e == cudaSuccess)
        e = launch_prefill_gemm(xmap, pw, nullptr, ws, 1.f, xs, y, pf_part, pf_flags, p, status_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "Q4_K GEMM launch");
    return LARQL_OK;
}

// y = down . (silu(gate . x) * (up . x)) for M tokens: fused gate/up GEMM, then the down GEMM.
int Ctx::prefill_ffn_dev(Weight* wg, Weight* wu, Weight* wd, const float* x, size_t M, float* y, cudaStream_t s) {
    for (Weight* w : {wg, wu, wd})
        if (w->format != LARQL_FMT_Q4_K) return fail(LARQL_ERR_UNSUPPORTED, "prefill FFN needs Q4_K weights");
    const size_t H = wg->cols, I = wg->rows;
    if (wu->rows != I || wu->cols != H || wd->rows != H || wd->cols != I)
        return fail(LARQL_ERR_BAD_SHAPE, "gate/up [%zu x %zu] and down [%zu x %zu] do not chain", I, H, wd->rows, wd->cols);
    if (M == 0) return LARQL_OK;
    if (!encode_tiled) return fail(LARQL_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    PrefillPlan p1, p2;
    if (M > (1u << 20) || I > 0x7fffffff || H > 0x7fffffff ||
        !prefill_make_plan(static_cast<int>(I), static_cast<int>(H), static_cast<int>(M), true, num_sms, &p1) ||
        !prefill_make_plan(static_cast<int>(H), static_cast<int>(I), static_cast<int>(M), false, num_sms, &p2))
        return fail(LARQL_ERR_UNSUPPORTED, "prefill FFN shape not supported");
    float sg, su, sd;
    const uint8_t *pg = nullptr, *pu = nullptr, *pd = nullptr;
    int rc = q4k_prefill_panels(wg, &sg, &pg);
    if (!rc) rc = q4k_prefill_panels(wu, &su, &pu);
    if (!rc) rc = q4k_prefill_panels(wd, &sd, &pd);
    if (!rc) rc = ensure_prefill_ws(std::max(prefill_part_floats(p1), prefill_part_floats(p2)));
    if (rc) return rc;
    auto up256 = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t r1 = prefill_tokens_padded(p1), r2 = prefill_tokens_padded(p2);
    const size_t b_xh = up256(r1 * H * 2), b_xs = up256(r1 * 4), b_act = up256(M * I * 4), b_ah = up256(r2 * I * 2),
                 b_as = up256(r2 * 4);
    rc = ensure_scratch(b_xh + b_xs + b_act + b_ah + b_as);
    if (rc) return rc;
    __half* xh = reinterpret_cast<__half*>(scratch);
    float* xs = reinterpret_cast<float*>(scratch + b_xh);
    float* act = reinterpret_cast<float*>(scratch + b_xh + b_xs);
    __half* ah = reinterpret_cast<__half*>(scratch + b_xh + b_xs + b_act);
    float* as = reinterpret_cast<float*>(scratch + b_xh + b_xs + b_act + b_ah);
    CUtensorMap m1, m2;
    if (prefill_encode_xmap(encode_tiled, xh, static_cast<int>(r1), static_cast<int>(H), std::min(256, p1.NTOK), &m1) ||
        prefill_encode_xmap(encode_tiled, ah, static_cast<int>(r2), static_cast<int>(I), std::min(256, p2.NTOK), &m2))
        return fail(LARQL_ERR_CUDA, "activation tensor map encoding failed");
    cudaError_t e = launch_prefill_x_prep(x, static_cast<int>(M), static_cast<int>(H), static_cast<int>(r1), xh, xs, s);
    if (e == cudaSuccess)
        e = launch_prefill_gemm(m1, pg, pu, sg, su, xs, act, pf_part, pf_flags, p1, status_dev, s);
    if (e == cudaSuccess)
        e = launch_prefill_x_prep(act, static_cast<int>(M), static_cast<int>(I), static_cast<int>(r2), ah, as, s);
    if (e == cudaSuccess)
        e = launch_prefill_gemm(m2, pd, nullptr, sd, 1.f, as, y, pf_part, pf_flags, p2, status_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "prefill FFN launch");
    return LARQL_OK;
}

int Ctx::weight_for(const void* host, size_t nbytes, int format, size_t rows, size_t cols, uint64_t* handle) {
    auto it = by_ptr.find({reinterpret_cast<uintptr_t>(host), nbytes});
    if (it != by_ptr.end()) {
        Weight* w = find(it->second);
        if (w && w->format == format && w->rows == rows && w->cols == cols) {
            *handle = it->second;
            return LARQL_OK;
        }
    }
    return add_weight(host, false, nbytes, nullptr, false, format, rows, cols, handle);
}

// Which Q4_K kernel serves (w, batch): the warp-MMA kernel where K % 1024 == 0
// (default), the tcgen05 kernel for batch >= 2 when selected, else the CUDA-core
// dp4a kernels.  Encodes the tensor map the chosen kernel streams through.
// The warp-MMA plan of a Q4_0 or GGUF Q8_0 weight at this batch (f32 x), or null when the shape or the
// selected path leaves it to the per-row block kernel.  Batch 1 stays on the block kernel (measured faster: its
// per-block float scaling is cheaper than the MMA form's); from batch 2 one MMA pass beats a block pass per row.
// Plans are kept per weight and batch.
const MmaPlan* Ctx::blk_mma_plan(Weight* w, size_t batch) {
    const int fmt = w->format == LARQL_FMT_Q4_0 ? 1
                    : w->format == LARQL_FMT_Q4_K_GGUF ? 5
                    : w->format == LARQL_FMT_Q4_K_GGUF_LLAMA ? 6
                    : (w->format == LARQL_FMT_Q8_0_GGUF ? 2 : (w->format == LARQL_FMT_Q6_K ? 4 : -1));
    if (fmt < 0 || q4k_path != 0 || batch < 1 || batch > 8 || !encode_tiled) return nullptr;
    if (batch < (fmt == 4 ? q6k_mma_min_batch : (fmt == 5 || fmt == 6 ? 1 : (fmt == 1 ? q40_mma_min_batch : 2))))
        return nullptr;
    MmaPlan& mp = w->blk_plans[batch - 1];
    if (mp.N == 0 && !q4k_mma_make_plan(static_cast<int>(w->rows), static_cast<int>(w->cols), static_cast<int>(batch),
                                        num_sms, &mp, mma_force, fmt)) {
        mp.N = -1;
    }
    return mp.N > 0 ? &mp : nullptr;
}

int Ctx::route_q4k(Weight* w, size_t batch, Q4kRoute* r) {
    const int bi = static_cast<int>(batch) - 1;
    if (bi >= 0 && bi < 8 && w->q4k_routed[bi]) {
        *r = w->q4k_route[bi];
        const int H = r->kind == Q4kRoute::kMma ? r->mp.RT
                      : r->kind == Q4kRoute::kTc ? r->tp.H
                      : r->kind == Q4kRoute::kTs ? 128 : 0;
        r->map = H ? q4k_map(w, H) : nullptr;
        if (!H || r->map) return LARQL_OK;
    }
    const int rc = plan_q4k(w, batch, r);
    if (rc == LARQL_OK && bi >= 0 && bi < 8) {
        w->q4k_route[bi] = *r;
        w->q4k_routed[bi] = true;
    }
    return rc;
}

int Ctx::plan_q4k(Weight* w, size_t batch, Q4kRoute* r) {
    const int N = static_cast<int>(w->rows), K = static_cast<int>(w->cols), B = static_cast<int>(batch);
    r->kind = Q4kRoute::kDp4a;
    r->map = nullptr;
    if (K % 1024 == 0 && (q4k_path == 3 || (q4k_path == 0 && B >= ts_min_batch)) &&
        q4k_ts_make_plan(N, K, B, num_sms, &r->sp) && (r->map = q4k_map(w, 128))) {
        r->kind = Q4kRoute::kTs;
        return LARQL_OK;
    }
    if (q4k_path == 0 && K % 1024 == 0) {
        const bool pinned = mma_force[0] > 0 || mma_force[1] > 0 || mma_force[2] > 0 || mma_force[3] > 0 ||
                            mma_force[4] > 0;
        if (q4k_mma_make_plan(N, K, B, num_sms, &r->mp, mma_force)) {
            if ((r->map = q4k_map(w, r->mp.RT))) {
                r->kind = Q4kRoute::kMma;
                return LARQL_OK;
            }
        } else if (pinned) {
            return fail(LARQL_ERR_UNSUPPORTED, "pinned MMA plan (%d groups, %d slices, %d stages, %d parts) does not "
                        "fit %zu x %zu batch %zu", mma_force[0], mma_force[1], mma_force[2], mma_force[3], w->rows,
                        w->cols, batch);
        }
    }
    if (use_tc && q4k_path != 2 && batch >= 2 && q4k_tc_make_plan(N, K, B, num_sms, &r->tp) &&
        (r->map = q4k_map(w, r->tp.H)))
        r->kind = Q4kRoute::kTc;
    return LARQL_OK;
}

int Ctx::describe_q4k(Weight* w, size_t batch, char* buf, size_t len) {
    Q4kRoute r;
    int rc = route_q4k(w, batch, &r);
    if (rc) return rc;
    if (r.kind == Q4kRoute::kMma)
        snprintf(buf, len, "q4k_mma_kernel<%zu> groups=%d slices=%d rows/tile=%d parts=%d stages=%d prefetch=%d "
                 "grid=%d warps=%d", batch, r.mp.NG, r.mp.KS, r.mp.RT, r.mp.nparts, r.mp.NS, r.mp.PF, r.mp.grid,
                 r.mp.NW + 1);
    else if (r.kind == Q4kRoute::kTc)
        snprintf(buf, len, "q4k_x_prep + q4k_tc_kernel (tcgen05) batch=%zu tile_rows=%d grid=%d", batch, r.tp.H,
                 r.tp.grid);
    else if (r.kind == Q4kRoute::kTs)
        snprintf(buf, len, "ts_x_prep + q4k_ts_kernel (tcgen05, sc*q in TMEM) batch=%zu rows/tile=128 parts=%d "
                 "grid=%d", batch, r.sp.nparts, r.sp.grid);
    else
        snprintf(buf, len, "%s batch=%zu", batch == 1 ? "q4k_matvec_pair_kernel (dp4a)" : "q4k_matvec_kernel (dp4a)",
                 batch);
    return LARQL_OK;
}

int Ctx::matvec_dev(Weight* w, const float* x, size_t batch, float* y, cudaStream_t s) {
    if (batch == 0) return LARQL_OK;
    if (batch > 8) return fail(LARQL_ERR_BAD_SHAPE, "batch %zu > 8", batch);
    if (reinterpret_cast<uintptr_t>(x) % 16) return fail(LARQL_ERR_INVALID_ARG, "x must be 16-byte aligned");
    if (w->rows > 0x7fffffff || w->cols > 0x7fffffff) return fail(LARQL_ERR_BAD_SHAPE, "matrix too large");
    cudaError_t e;
    switch (w->format) {
        case LARQL_FMT_Q4_K: {
            Q4kRoute r;
            int rc = route_q4k(w, batch, &r);
            if (rc) return rc;
            if (r.kind == Q4kRoute::kMma) {
                const size_t pf = q4k_mma_partial_floats(r.mp);
                rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
                if (!rc) rc = ensure_tickets(static_cast<size_t>(r.mp.ntiles));
                if (rc) return rc;
                e = launch_q4k_mma(*r.map, x, y, reinterpret_cast<float*>(scratch), tickets, r.mp, status_dev, s);
            } else if (r.kind == Q4kRoute::kTc) {
                rc = ensure_scratch(q4k_tc_scratch_bytes(static_cast<int>(w->cols), static_cast<int>(batch)));
                if (rc) return rc;
                e = launch_q4k_tc(*r.map, x, y, r.tp, scratch, status_dev, s);
            } else if (r.kind == Q4kRoute::kTs) {
                rc = ensure_scratch(q4k_ts_scratch_bytes(r.sp));
                if (!rc) rc = ensure_tickets(q4k_ts_tickets(r.sp));
                if (rc) return rc;
                e = launch_q4k_ts(*r.map, x, y, r.sp, scratch, tickets, status_dev, s);
            } else {
                e = launch_q4k_matvec(static_cast<const uint8_t*>(w->dev), static_cast<int>(w->rows),
                                      static_cast<int>(w->cols), x, static_cast<int>(batch), y, num_sms, status_dev, s);
            }
            break;
        }
        case LARQL_FMT_Q4_0:
        case LARQL_FMT_Q8_0_GGUF: {
            // K % 1024 == 0 (Q4_0 from batch 1, GGUF Q8_0 from batch 2): the warp-MMA kernel, one weight pass for
            // the whole batch
            {
                const MmaPlan* mp = blk_mma_plan(w, batch);
                if (mp) {
                    const size_t pf = q4k_mma_partial_floats(*mp);
                    int rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
                    if (!rc) rc = ensure_tickets(static_cast<size_t>(mp->ntiles));
                    if (rc) return rc;
                    const CUtensorMap* map = q4k_map(w, mp->RT);
                    if (map) {
                        e = launch_q4k_mma(*map, x, y, reinterpret_cast<float*>(scratch), tickets, *mp, status_dev, s);
                        break;
                    }
                }
            }
            // otherwise (and GGUF Q8_0) one weight pass per batch row
            const int fmt = w->format == LARQL_FMT_Q4_0 ? 0 : 1;
            if (w->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "block matvec needs cols %% 64 == 0");
            e = cudaSuccess;
            for (size_t b = 0; b < batch && e == cudaSuccess; ++b)
                e = launch_block_matvec(fmt, static_cast<const uint8_t*>(w->dev), nullptr, x + b * w->cols, nullptr,
                                        nullptr, y + b * w->rows, static_cast<int>(w->rows), static_cast<int>(w->cols),
                                        num_sms, status_dev, s);
            break;
        }
        case LARQL_FMT_Q6_K: {
            // q6k_matvec.rs:31-87.  K % 2048 == 0 (and batch >= q6k_mma_min_batch): the warp-MMA kernel, one
            // weight pass for the whole batch
            if (const MmaPlan* mp = blk_mma_plan(w, batch)) {
                const size_t pf = q4k_mma_partial_floats(*mp);
                int rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
                if (!rc) rc = ensure_tickets(static_cast<size_t>(mp->ntiles));
                if (rc) return rc;
                if (const CUtensorMap* map = q4k_map(w, mp->RT)) {
                    e = launch_q4k_mma(*map, x, y, reinterpret_cast<float*>(scratch), tickets, *mp, status_dev, s);
                    break;
                }
            }
            // otherwise one weight pass per batch row on the block kernel
            if (w->cols % 256) return fail(LARQL_ERR_UNSUPPORTED, "Q6_K matvec needs cols %% 256 == 0");
            e = cudaSuccess;
            for (size_t b = 0; b < batch && e == cudaSuccess; ++b)
                e = launch_block_matvec(3, static_cast<const uint8_t*>(w->dev), nullptr, x + b * w->cols, nullptr,
                                        nullptr, y + b * w->rows, static_cast<int>(w->rows), static_cast<int>(w->cols),
                                        num_sms, status_dev, s);
            break;
        }
        case LARQL_FMT_Q4_K_GGUF: {
            // ggml.rs:228-273 (dequantize_q4_k, the GGUF loader's decoder) + f32 dot.  K % 1024 == 0: the warp-MMA
            // kernel on the Q4_K tables, one weight pass for the whole batch
            if (const MmaPlan* mp = blk_mma_plan(w, batch)) {
                const size_t pf = q4k_mma_partial_floats(*mp);
                int rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
                if (!rc) rc = ensure_tickets(static_cast<size_t>(mp->ntiles));
                if (rc) return rc;
                if (const CUtensorMap* map = q4k_map(w, mp->RT)) {
                    e = launch_q4k_mma(*map, x, y, reinterpret_cast<float*>(scratch), tickets, *mp, status_dev, s);
                    break;
                }
            }
            // otherwise the dp4a pair kernel, one weight pass per batch row
            if (w->cols % 256) return fail(LARQL_ERR_UNSUPPORTED, "GGUF Q4_K matvec needs cols %% 256 == 0");
            e = launch_q4k_gguf_matvec(static_cast<const uint8_t*>(w->dev), static_cast<int>(w->rows),
                                       static_cast<int>(w->cols), x, static_cast<int>(batch), y, num_sms, status_dev,
                                       s);
            break;
        }
        case LARQL_FMT_Q4_K_GGUF_LLAMA: {
            // GGUF-144 Q4_K in llama.cpp's layout, as the reference's Metal q4kf kernels read it
            // (crates/larql-compute/src/metal/shaders/q4kf_qkv_proj.rs): the warp-MMA kernel, K % 1024 == 0
            const MmaPlan* mp = blk_mma_plan(w, batch);
            if (!mp) return fail(LARQL_ERR_UNSUPPORTED, "llama.cpp-layout Q4_K matvec needs cols %% 1024 == 0");
            const size_t pf = q4k_mma_partial_floats(*mp);
            int rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
            if (!rc) rc = ensure_tickets(static_cast<size_t>(mp->ntiles));
            if (rc) return rc;
            const CUtensorMap* map = q4k_map(w, mp->RT);
            if (!map) return fail(LARQL_ERR_CUDA, "tensor map encoding failed");
            e = launch_q4k_mma(*map, x, y, reinterpret_cast<float*>(scratch), tickets, *mp, status_dev, s);
            break;
        }
        case LARQL_FMT_Q8_0: {
            // compute layout against Q8(x) (q8_matvec.rs:36-57): quantize x on the device, then int8 dot
            if (w->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "block matvec needs cols %% 64 == 0");
            const size_t qbytes = (w->cols + 255) & ~size_t(255);
            int rc = ensure_scratch(batch * (qbytes + w->cols / 32 * 4 + 256));
            if (rc) return rc;
            int8_t* q8 = reinterpret_cast<int8_t*>(scratch);
            float* q8s = reinterpret_cast<float*>(scratch + batch * qbytes);
            e = launch_quantize_to_q8(x, batch * w->cols, q8, q8s, s);
            for (size_t b = 0; b < batch && e == cudaSuccess; ++b)
                e = launch_block_matvec(2, static_cast<const uint8_t*>(w->dev), w->scales_dev, nullptr, q8 + b * qbytes,
                                        q8s + b * (w->cols / 32), y + b * w->rows, static_cast<int>(w->rows),
                                        static_cast<int>(w->cols), num_sms, status_dev, s);
            break;
        }
        default: return fail(LARQL_ERR_UNSUPPORTED, "matvec for weight format %d is not provided", w->format);
    }
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "shape %zu x %zu not supported for format %d",
                                                w->rows, w->cols, w->format);
    if (e != cudaSuccess) return cuda_fail(e, "matvec launch");
    return LARQL_OK;
}

int Ctx::q4_matvec_q8_dev(Weight* w, const int8_t* q8x, const float* q8s, float* y, cudaStream_t s) {
    if (w->format != LARQL_FMT_Q4_0) return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec needs a Q4_0 weight");
    if (w->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec needs hidden %% 64 == 0");
    if (reinterpret_cast<uintptr_t>(q8x) % 16) return fail(LARQL_ERR_INVALID_ARG, "q8_x must be 16-byte aligned");
    cudaError_t e = launch_block_matvec(0, static_cast<const uint8_t*>(w->dev), nullptr, nullptr, q8x, q8s, y,
                                        static_cast<int>(w->rows), static_cast<int>(w->cols), num_sms, status_dev, s);
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "shape not supported");
    if (e != cudaSuccess) return cuda_fail(e, "q4_matvec launch");
    return LARQL_OK;
}

// The k largest logits by signed value, descending, equal logits by lower id (walk.rs:566-577); k = min(top_k, n)
// entries.  top_k 0 (the reference then returns every logit sorted) or k > 32 is not provided.
int Ctx::logit_topk_dev(const float* logits, size_t n, size_t top_k, uint32_t* ids, float* vals, cudaStream_t s) {
    if (n == 0) return LARQL_OK;
    if (n > 0x7fffffff) return fail(LARQL_ERR_BAD_SHAPE, "logit top-k: n=%zu too large", n);
    const size_t k = top_k < n ? top_k : n;
    if (top_k == 0 || k > 32) return fail(LARQL_ERR_UNSUPPORTED, "logit top-k: top_k=%zu (1..32 provided)", top_k);
    const size_t ent = logit_topk_scratch_entries(static_cast<int>(n), static_cast<int>(k), num_sms);
    int rc = ensure_scratch(ent * sizeof(uint64_t));
    if (rc) return rc;
    cudaError_t e = launch_logit_topk(logits, static_cast<int>(n), static_cast<int>(k), num_sms,
                                      reinterpret_cast<uint64_t*>(scratch), ids, vals, s);
    if (e != cudaSuccess) return cuda_fail(e, "logit top-k launch");
    return LARQL_OK;
}

// VectorIndex::lm_head_knn_backend, Q4 branch (walk.rs:549-583): the query quantized by quantize_to_q8
// (q4_common.rs:28-44), logits = Q4_0 lm head x Q8 query (q4_dot.c:169-199), then logit_topk_dev.
int Ctx::lm_head_knn_dev(Weight* w, const float* query, size_t top_k, uint32_t* ids, float* vals, cudaStream_t s) {
    if (w->format != LARQL_FMT_Q4_0) return fail(LARQL_ERR_UNSUPPORTED, "lm_head_knn needs a Q4_0 lm head");
    if (w->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "lm_head_knn needs hidden %% 64 == 0");
    const size_t k = top_k < w->rows ? top_k : w->rows;
    if (top_k == 0 || k > 32) return fail(LARQL_ERR_UNSUPPORTED, "lm_head_knn: top_k=%zu (1..32 provided)", top_k);
    const size_t qb = (w->cols + 255) & ~size_t(255);
    const size_t sb = (w->cols / 32 * 4 + 255) & ~size_t(255);
    int rc = ensure_aux(qb + sb + w->rows * sizeof(float));
    if (rc) return rc;
    int8_t* q8 = reinterpret_cast<int8_t*>(aux);
    float* q8s = reinterpret_cast<float*>(aux + qb);
    float* logits = reinterpret_cast<float*>(aux + qb + sb);
    cudaError_t e = launch_quantize_to_q8(query, w->cols, q8, q8s, s);
    if (e != cudaSuccess) return cuda_fail(e, "quantize_to_q8 launch");
    rc = q4_matvec_q8_dev(w, q8, q8s, logits, s);
    if (rc) return rc;
    return logit_topk_dev(logits, w->rows, top_k, ids, vals, s);
}

// q4_vecmat (q4_dot.c:201-232): out[cols] = act[rows] @ W, W a Q4_0 weight of rows x cols.
int Ctx::q4_vecmat_dev(Weight* w, const float* act, float* out, cudaStream_t s) {
    if (w->format != LARQL_FMT_Q4_0) return fail(LARQL_ERR_UNSUPPORTED, "q4_vecmat needs a Q4_0 weight");
    if (w->rows > 0x7fffffff || w->cols > 0x7fffffff) return fail(LARQL_ERR_BAD_SHAPE, "matrix too large");
    const VecmatPlan p = q4_vecmat_plan(static_cast<int>(w->rows), static_cast<int>(w->cols), num_sms);
    const size_t pf = q4_vecmat_part_floats(p, static_cast<int>(w->cols));
    if (pf) {
        int rc = ensure_scratch(pf * sizeof(float));
        if (rc) return rc;
    }
    cudaError_t e = launch_q4_vecmat(act, static_cast<const uint8_t*>(w->dev), static_cast<int>(w->rows),
                                     static_cast<int>(w->cols), p, reinterpret_cast<float*>(scratch), out, s);
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "q4_vecmat shape not supported");
    if (e != cudaSuccess) return cuda_fail(e, "q4_vecmat launch");
    return LARQL_OK;
}

// q4_matvec_pair_batch (metal/ops/q4_batched.rs:19-80): every position's x quantized by quantize_to_q8
// (one launch over all positions: hidden % 32 == 0 keeps each position's blocks its own), then the Q4_0 x Q8
// matvec of q4_dot.c against gate and up for each position.
int Ctx::q4_pair_batch_dev(Weight* g, Weight* u, const float* x, size_t seq, float* gout, float* uout,
                           cudaStream_t s) {
    if (g->format != LARQL_FMT_Q4_0 || u->format != LARQL_FMT_Q4_0)
        return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec_pair_batch needs Q4_0 weights");
    if (g->rows != u->rows || g->cols != u->cols)
        return fail(LARQL_ERR_BAD_SHAPE, "gate %zu x %zu and up %zu x %zu differ", g->rows, g->cols, u->rows, u->cols);
    if (g->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec_pair_batch needs hidden %% 64 == 0");
    if (seq == 0) return LARQL_OK;
    const size_t hidden = g->cols, qbytes = seq * hidden;
    const size_t qoff = (qbytes + 255) & ~size_t(255);
    const size_t soff = qoff + ((seq * (hidden / 32) * sizeof(float) + 255) & ~size_t(255));
    // Q8 values, their scales and (for the tensor-core form) the dequantised f32 copy live in the aux buffer;
    // the matvec kernels use the scratch buffer for their split-K partial sums
    int rc = ensure_aux(soff + qbytes * sizeof(float));
    if (rc) return rc;
    int8_t* q8 = reinterpret_cast<int8_t*>(aux);
    float* q8s = reinterpret_cast<float*>(aux + qoff);
    cudaError_t e = launch_quantize_to_q8(x, seq * hidden, q8, q8s, s);
    if (e != cudaSuccess) return cuda_fail(e, "q4_matvec_pair_batch launch");
    // K % 1024 == 0 and two or more positions: the Q4_0 warp-MMA matvec (IEEE-decoded scales, as q4_dot.c) on
    // x' = q8 * scale, up to 8 positions per weight pass (one position: the block kernel, measured faster)
    MmaPlan mp8;
    if (seq >= 2 && q4k_path == 0 && hidden % 1024 == 0 && encode_tiled &&
        q4k_mma_make_plan(static_cast<int>(g->rows), static_cast<int>(hidden), 8, num_sms, &mp8, mma_force, 3)) {
        float* xf = reinterpret_cast<float*>(aux + soff);
        e = launch_dequant_q8(q8, q8s, seq * hidden, xf, s);
        for (size_t t0 = 0; t0 < seq && e == cudaSuccess; t0 += 8) {
            const int nb = static_cast<int>(std::min<size_t>(8, seq - t0));
            MmaPlan mp;
            if (!q4k_mma_make_plan(static_cast<int>(g->rows), static_cast<int>(hidden), nb, num_sms, &mp, mma_force,
                                   3))
                return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec_pair_batch: no plan for %d positions", nb);
            const size_t pf = q4k_mma_partial_floats(mp);
            rc = pf ? ensure_scratch(pf * sizeof(float)) : LARQL_OK;
            if (!rc) rc = ensure_tickets(static_cast<size_t>(mp.ntiles));
            if (rc) return rc;
            for (int wsel = 0; wsel < 2 && e == cudaSuccess; ++wsel) {
                Weight* w = wsel ? u : g;
                const CUtensorMap* map = q4k_map(w, mp.RT);
                if (!map) return fail(LARQL_ERR_CUDA, "tensor map encoding failed");
                e = launch_q4k_mma(*map, xf + t0 * hidden, (wsel ? uout : gout) + t0 * w->rows,
                                   reinterpret_cast<float*>(scratch), tickets, mp, status_dev, s);
            }
        }
        if (e != cudaSuccess) return cuda_fail(e, "q4_matvec_pair_batch launch");
        return LARQL_OK;
    }
    for (size_t t = 0; t < seq && e == cudaSuccess; ++t) {
        e = launch_block_matvec(0, static_cast<const uint8_t*>(g->dev), nullptr, nullptr, q8 + t * hidden,
                                q8s + t * (hidden / 32), gout + t * g->rows, static_cast<int>(g->rows),
                                static_cast<int>(hidden), num_sms, status_dev, s);
        if (e == cudaSuccess)
            e = launch_block_matvec(0, static_cast<const uint8_t*>(u->dev), nullptr, nullptr, q8 + t * hidden,
                                    q8s + t * (hidden / 32), uout + t * u->rows, static_cast<int>(u->rows),
                                    static_cast<int>(hidden), num_sms, status_dev, s);
    }
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "q4_matvec_pair_batch shape not supported");
    if (e != cudaSuccess) return cuda_fail(e, "q4_matvec_pair_batch launch");
    return LARQL_OK;
}

// Top-k per (layer, query), or with `scores` every score [L][B][F] instead (top_k unused).
int Ctx::gate_topk_dev(Weight* w, size_t n_layers, size_t n_feat, const float* q, size_t batch, size_t top_k,
                       uint32_t* out_i, float* out_s, cudaStream_t s, float* scores) {
    if (w->format != LARQL_FMT_F16_HALFRS && w->format != LARQL_FMT_F16)
        return fail(LARQL_ERR_UNSUPPORTED, "gate walk needs f16 rows (LARQL_FMT_F16_HALFRS or LARQL_FMT_F16), not "
                    "format %d", w->format);
    if (n_layers == 0 || n_feat == 0 || n_layers * n_feat != w->rows)
        return fail(LARQL_ERR_BAD_SHAPE, "n_layers %zu x n_feat %zu != %zu registered rows", n_layers, n_feat, w->rows);
    if (scores) top_k = 1;
    if (batch == 0 || top_k == 0) return LARQL_OK;
    if (batch > (1u << 20) || w->rows > 0x7fffffff || w->cols > 0x7fffffff)
        return fail(LARQL_ERR_BAD_SHAPE, "gate walk too large");
    if (reinterpret_cast<uintptr_t>(q) % 16) return fail(LARQL_ERR_INVALID_ARG, "queries must be 16-byte aligned");
    if (!scores && gate_gemv && top_k <= 16 && gate_gemv_ok(static_cast<int>(w->cols), static_cast<int>(batch)) &&
        reinterpret_cast<uintptr_t>(w->dev) % 16 == 0) {
        // one to four queries: CUDA-core dot products, every gate byte read once
        const int L = static_cast<int>(n_layers), F = static_cast<int>(n_feat);
        const int parts = gate_gemv_parts(L, F, num_sms);
        const size_t ncand = static_cast<size_t>(L) * batch * parts * 16;
        int rc = ensure_scratch(ncand * (sizeof(float) + sizeof(uint32_t)) + 256);
        if (rc) return rc;
        float* cs = reinterpret_cast<float*>(scratch);
        uint32_t* ci = reinterpret_cast<uint32_t*>(cs + ncand);
        cudaError_t e = launch_gate_gemv(static_cast<const __half*>(w->dev), w->gate_factor, q, L, F,
                                         static_cast<int>(w->cols), static_cast<int>(batch),
                                         static_cast<int>(top_k), parts, cs, ci, out_i, out_s, s);
        if (e != cudaSuccess) return cuda_fail(e, "gate walk (CUDA cores) launch");
        return LARQL_OK;
    }
    if (!encode_tiled) return fail(LARQL_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    GatePlan p;
    if (!gate_make_plan(static_cast<int>(n_layers), static_cast<int>(n_feat), static_cast<int>(w->cols),
                        static_cast<int>(batch), static_cast<int>(top_k), num_sms, &p))
        return fail(LARQL_ERR_UNSUPPORTED, "gate walk needs hidden %% 64 == 0 and top_k <= 16 (hidden %zu, top_k %zu)",
                    w->cols, top_k);
    if (!w->gmap_ok) {
        if (gate_encode_map(encode_tiled, w->dev, w->rows, static_cast<int>(w->cols), 256, &w->gmap) != 0)
            return fail(LARQL_ERR_CUDA, "gate tensor map encoding failed");
        w->gmap_ok = true;
    }
    int rc = ensure_scratch(gate_scratch_bytes(p));
    if (rc) return rc;
    cudaError_t e =
        launch_gate_topk(encode_tiled, w->gmap, w->gate_factor, q, p, scratch, out_i, out_s, status_dev, s, scores);
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "gate walk shape not supported");
    if (e != cudaSuccess) return cuda_fail(e, "gate walk launch");
    return LARQL_OK;
}

// VectorIndex::gate_knn_q4 (gate.rs:714-731) for every layer of a Q4_0 gate matrix [n_layers * n_feat][hidden]
// (gate_vectors_q4.bin, walk.rs:303-328) and every query: each query quantized by quantize_to_q8
// (q4_common.rs:28-44), one Q4_0 x Q8 matvec over all layers' rows (q4_dot.c:169-199), then the top-k by |score|
// of every (layer, query) (top_k_from_scores, gate.rs:307-316; ties by lower index).
int Ctx::gate_topk_q4_dev(Weight* w, size_t n_layers, size_t n_feat, const float* q, size_t batch, size_t top_k,
                          uint32_t* out_i, float* out_s, cudaStream_t s) {
    if (w->format != LARQL_FMT_Q4_0) return fail(LARQL_ERR_UNSUPPORTED, "Q4 gate walk needs a Q4_0 weight");
    if (n_layers == 0 || n_feat == 0 || n_layers * n_feat != w->rows)
        return fail(LARQL_ERR_BAD_SHAPE, "n_layers %zu x n_feat %zu != %zu registered rows", n_layers, n_feat, w->rows);
    if (batch == 0 || top_k == 0) return LARQL_OK;
    if (top_k > 16) return fail(LARQL_ERR_UNSUPPORTED, "Q4 gate walk: top_k %zu > 16", top_k);
    if (w->cols % 64) return fail(LARQL_ERR_UNSUPPORTED, "Q4 gate walk needs hidden %% 64 == 0");
    if (batch > 65535 || w->rows > 0x7fffffff) return fail(LARQL_ERR_BAD_SHAPE, "Q4 gate walk too large");
    if (reinterpret_cast<uintptr_t>(q) % 16) return fail(LARQL_ERR_INVALID_ARG, "queries must be 16-byte aligned");
    const int L = static_cast<int>(n_layers), F = static_cast<int>(n_feat), B = static_cast<int>(batch);
    const size_t H = w->cols;
    const size_t qb = (H + 255) & ~size_t(255), sb = (H / 32 * 4 + 255) & ~size_t(255);
    const size_t per_q = qb + sb + ((w->rows * sizeof(float) + 255) & ~size_t(255));
    int rc = ensure_aux(batch * per_q);
    if (rc) return rc;
    const int parts = gate_score_cand_parts(L, F, B, num_sms);
    const size_t ncand = static_cast<size_t>(L) * batch * parts * 16;
    rc = ensure_scratch(ncand * (sizeof(float) + sizeof(uint32_t)) + 256);
    if (rc) return rc;
    // aux: the scores [B][L][F] f32, then per query its Q8 values and scales (256-byte aligned)
    float* scores = reinterpret_cast<float*>(aux);
    int8_t* q8 = reinterpret_cast<int8_t*>(aux + ((batch * w->rows * sizeof(float) + 255) & ~size_t(255)));
    const size_t q8_stride = qb + sb;
    for (size_t b = 0; b < batch; ++b) {
        int8_t* qx = q8 + b * q8_stride;
        float* qs = reinterpret_cast<float*>(q8 + b * q8_stride + qb);
        cudaError_t e = launch_quantize_to_q8(q + b * H, H, qx, qs, s);
        if (e != cudaSuccess) return cuda_fail(e, "quantize_to_q8 launch");
        rc = q4_matvec_q8_dev(w, qx, qs, scores + b * w->rows, s);
        if (rc) return rc;
    }
    float* cs = reinterpret_cast<float*>(scratch);
    uint32_t* ci = reinterpret_cast<uint32_t*>(cs + ncand);
    cudaError_t e = launch_gate_score_topk(scores, L, F, B, static_cast<int>(top_k), parts, cs, ci, out_i, out_s, s);
    if (e == cudaErrorInvalidValue) return fail(LARQL_ERR_UNSUPPORTED, "Q4 gate walk shape not supported");
    if (e != cudaSuccess) return cuda_fail(e, "Q4 gate walk selection launch");
    return LARQL_OK;
}

int Ctx::matvec_host(Weight* w, const float* x, size_t batch, float* y) {
    if (!x || !y) return fail(LARQL_ERR_INVALID_ARG, "null x or y");
    int rc = ensure_io(batch * w->cols, batch * w->rows);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(x_dev, x, batch * w->cols * sizeof(float), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return cuda_fail(e, "x upload");
    rc = matvec_dev(w, x_dev, batch, y_dev, stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(y, y_dev, batch * w->rows * sizeof(float), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return cuda_fail(e, "y download");
    return finish();
}

}  // namespace larql

using larql::Ctx;
using larql::fail;
using larql::cuda_fail;

extern "C" {

int larql_cuda_version(void) { return 100; }

int larql_cuda_last_error(char* buf, size_t len) {
    if (!buf || len == 0) return LARQL_ERR_INVALID_ARG;
    snprintf(buf, len, "%s", larql::g_last_error.c_str());
    return LARQL_OK;
}

const char* larql_cuda_status_string(int status) {
    switch (status) {
        case LARQL_OK: return "ok";
        case LARQL_ERR_INVALID_ARG: return "invalid argument";
        case LARQL_ERR_BAD_SHAPE: return "bad shape";
        case LARQL_ERR_UNSUPPORTED: return "unsupported";
        case LARQL_ERR_CUDA: return "CUDA error";
        case LARQL_ERR_NCCL: return "NCCL error";
        case LARQL_ERR_TIMEOUT: return "device wait timed out";
        case LARQL_ERR_OOM: return "out of device memory";
        case LARQL_ERR_NOT_FOUND: return "unknown handle";
        default: return "unknown status";
    }
}

int larql_cuda_create(int device, larql_cuda_ctx** out) {
    if (!out) return fail(LARQL_ERR_INVALID_ARG, "null output");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(LARQL_ERR_INVALID_ARG, "device %d of %d", device, n);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10) return fail(LARQL_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                                      device, prop.major, prop.minor);
    // Digit planes of x in the batch-1 Q4_K kernel: 3 (default, 22-23 significant
    // bits per 32-value group) or 2 (15 bits, fewer dp4a).
    if (const char* ev = getenv("LARQL_CUDA_Q4K_PLANES")) {
        const int v = atoi(ev);
        if (v == 2 || v == 3) larql::g_q4k_planes = v;
    }
    auto* c = new larql_cuda_ctx();
    Ctx& x = c->impl;
    x.device = device;
    x.num_sms = prop.multiProcessorCount;
    x.l2_bytes = prop.l2CacheSize;
    snprintf(x.dev_name, sizeof(x.dev_name), "%s", prop.name);
    {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            x.encode_tiled = fn;
        if (const char* ev = getenv("LARQL_CUDA_Q4K_TC")) x.use_tc = atoi(ev) != 0;
        if (const char* ev = getenv("LARQL_CUDA_Q4K_PATH"))
            x.q4k_path = strcmp(ev, "tc") == 0 ? 1 : (strcmp(ev, "dp4a") == 0 ? 2 : (strcmp(ev, "ts") == 0 ? 3 : 0));
        if (const char* ev = getenv("LARQL_CUDA_TS_MIN_BATCH")) x.ts_min_batch = atoi(ev);
        if (const char* ev = getenv("LARQL_CUDA_DECODE_FUSE")) x.fuse_decode = atoi(ev) & 3;
        if (const char* ev = getenv("LARQL_CUDA_DECODE_PERSIST")) x.decode_persist = atoi(ev) != 0;
        if (const char* ev = getenv("LARQL_CUDA_GATE_GEMV")) x.gate_gemv = atoi(ev) != 0;
        if (const char* ev = getenv("LARQL_CUDA_Q6K_MMA_MIN_BATCH")) x.q6k_mma_min_batch = atoi(ev);
        if (const char* ev = getenv("LARQL_CUDA_Q40_MMA_MIN_BATCH")) x.q40_mma_min_batch = atoi(ev);
        if (const char* ev = getenv("LARQL_CUDA_MMA_CFG"))
            sscanf(ev, "%d,%d,%d,%d,%d", &x.mma_force[0], &x.mma_force[1], &x.mma_force[2], &x.mma_force[3], &x.mma_force[4]);
    }
    e = cudaStreamCreateWithFlags(&x.stream, cudaStreamNonBlocking);
    // status word + a few ints of device scratch for host-synchronous helpers (registration)
    if (e == cudaSuccess) e = cudaMalloc(&x.status_dev, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(x.status_dev, 0, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&x.status_host, sizeof(int));
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "context setup");
    }
    *out = c;
    return LARQL_OK;
}

int larql_cuda_destroy(larql_cuda_ctx* ctx) {
    if (!ctx) return LARQL_OK;
    delete ctx;
    return LARQL_OK;
}

int larql_cuda_name(larql_cuda_ctx* ctx, char* buf, size_t len) {
    if (!ctx || !buf || !len) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    snprintf(buf, len, "cuda (sm_100a, dp4a/bulk-copy Q4 kernels)");
    return LARQL_OK;
}

int larql_cuda_device_info(larql_cuda_ctx* ctx, char* buf, size_t len) {
    if (!ctx || !buf || !len) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    snprintf(buf, len, "%s (device %d, %d SMs, L2 %d MB)", ctx->impl.dev_name, ctx->impl.device, ctx->impl.num_sms,
             ctx->impl.l2_bytes >> 20);
    return LARQL_OK;
}

int larql_cuda_has_q4(larql_cuda_ctx* ctx, int* out) {
    if (!ctx || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    *out = 1;
    return LARQL_OK;
}

int larql_cuda_stream(larql_cuda_ctx* ctx, void** stream) {
    if (!ctx || !stream) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    *stream = ctx->impl.stream;
    return LARQL_OK;
}

int larql_cuda_sync(larql_cuda_ctx* ctx) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.finish();
}

int larql_cuda_register_weight(larql_cuda_ctx* ctx, const void* host_data, size_t nbytes, const float* scales,
                               int format, size_t rows, size_t cols, uint64_t* handle) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.add_weight(host_data, false, nbytes, scales, false, format, rows, cols, handle);
}

int larql_cuda_register_weight_device(larql_cuda_ctx* ctx, const void* dev_data, size_t nbytes,
                                      const float* dev_scales, int format, size_t rows, size_t cols,
                                      uint64_t* handle) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.add_weight(dev_data, true, nbytes, dev_scales, true, format, rows, cols, handle);
}

int larql_cuda_release_weight(larql_cuda_ctx* ctx, uint64_t handle) {
    LARQL_CTX_GUARD(ctx);
    auto it = ctx->impl.weights.find(handle);
    if (it == ctx->impl.weights.end()) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle %llu",
                                                   static_cast<unsigned long long>(handle));
    cudaStreamSynchronize(ctx->impl.stream);
    if (it->second.owned) cudaFree(it->second.dev);
    if (it->second.scales_dev) cudaFree(it->second.scales_dev);
    for (auto p = ctx->impl.by_ptr.begin(); p != ctx->impl.by_ptr.end();) {
        if (p->second == handle) p = ctx->impl.by_ptr.erase(p);
        else ++p;
    }
    ctx->impl.weights.erase(it);
    return LARQL_OK;
}

int larql_cuda_weight_device_ptr(larql_cuda_ctx* ctx, uint64_t handle, const void** dev_ptr) {
    LARQL_CTX_GUARD(ctx);
    if (!dev_ptr) return fail(LARQL_ERR_INVALID_ARG, "null output");
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    *dev_ptr = w->dev;
    return LARQL_OK;
}

int larql_cuda_q4k_matvec(larql_cuda_ctx* ctx, const uint8_t* q4k_data, size_t nbytes, const float* x,
                          size_t num_rows, size_t hidden, float* out) {
    LARQL_CTX_GUARD(ctx);
    if (!q4k_data || !x || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (num_rows == 0) return LARQL_OK;
    uint64_t h;
    int rc = ctx->impl.weight_for(q4k_data, nbytes, LARQL_FMT_Q4_K, num_rows, hidden, &h);
    if (rc) return rc;
    return ctx->impl.matvec_host(ctx->impl.find(h), x, 1, out);
}

int larql_cuda_q6k_matvec(larql_cuda_ctx* ctx, const uint8_t* q6k_data, size_t nbytes, const float* x,
                          size_t num_rows, size_t hidden, float* out) {
    LARQL_CTX_GUARD(ctx);
    if (!q6k_data || !x || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (num_rows == 0) return LARQL_OK;
    uint64_t h;
    int rc = ctx->impl.weight_for(q6k_data, nbytes, LARQL_FMT_Q6_K, num_rows, hidden, &h);
    if (rc) return rc;
    return ctx->impl.matvec_host(ctx->impl.find(h), x, 1, out);
}

int larql_cuda_q4_matvec(larql_cuda_ctx* ctx, const uint8_t* q4_data, size_t nbytes, const int8_t* q8_x,
                         const float* q8_scales, size_t num_rows, size_t hidden, float* out) {
    LARQL_CTX_GUARD(ctx);
    if (!q4_data || !q8_x || !q8_scales || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (num_rows == 0) return LARQL_OK;
    uint64_t h;
    int rc = ctx->impl.weight_for(q4_data, nbytes, LARQL_FMT_Q4_0, num_rows, hidden, &h);
    if (rc) return rc;
    Ctx& c = ctx->impl;
    // q8 values then scales in the context's x buffer (16-byte aligned pieces)
    const size_t qb = (hidden + 15) & ~size_t(15);
    rc = c.ensure_io((qb + hidden / 32 * 4) / 4 + 4, num_rows);
    if (rc) return rc;
    int8_t* dq = reinterpret_cast<int8_t*>(c.x_dev);
    float* ds = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(c.x_dev) + qb);
    cudaError_t e = cudaMemcpyAsync(dq, q8_x, hidden, cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ds, q8_scales, hidden / 32 * 4, cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "q8 upload");
    rc = c.q4_matvec_q8_dev(c.find(h), dq, ds, c.y_dev, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out, c.y_dev, num_rows * 4, cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "y download");
    return c.finish();
}

int larql_cuda_q4_vecmat(larql_cuda_ctx* ctx, const float* activation, const uint8_t* q4_data, size_t nbytes,
                         size_t intermediate, size_t hidden, float* out) {
    LARQL_CTX_GUARD(ctx);
    if (!activation || !q4_data || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (hidden == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    if (intermediate == 0) {
        memset(out, 0, hidden * sizeof(float));
        return LARQL_OK;
    }
    uint64_t h;
    int rc = c.weight_for(q4_data, nbytes, LARQL_FMT_Q4_0, intermediate, hidden, &h);
    if (rc) return rc;
    rc = c.ensure_io(intermediate, hidden);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, activation, intermediate * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "activation upload");
    rc = c.q4_vecmat_dev(c.find(h), c.x_dev, c.y_dev, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out, c.y_dev, hidden * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "out download");
    return c.finish();
}

int larql_cuda_q4_vecmat_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* act_dev, float* out_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!act_dev || !out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    return ctx->impl.q4_vecmat_dev(w, act_dev, out_dev, stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
}

int larql_cuda_q4_matvec_pair_batch(larql_cuda_ctx* ctx, const uint8_t* gate_q4, size_t gate_nbytes,
                                    const uint8_t* up_q4, size_t up_nbytes, const float* x_matrix, size_t seq_len,
                                    size_t num_rows, size_t hidden, float* gate_out, float* up_out) {
    LARQL_CTX_GUARD(ctx);
    if (!gate_q4 || !up_q4 || !x_matrix || !gate_out || !up_out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (seq_len == 0 || num_rows == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    uint64_t hg, hu;
    int rc = c.weight_for(gate_q4, gate_nbytes, LARQL_FMT_Q4_0, num_rows, hidden, &hg);
    if (!rc) rc = c.weight_for(up_q4, up_nbytes, LARQL_FMT_Q4_0, num_rows, hidden, &hu);
    if (rc) return rc;
    rc = c.ensure_io(seq_len * hidden, 2 * seq_len * num_rows);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, x_matrix, seq_len * hidden * sizeof(float), cudaMemcpyHostToDevice,
                                    c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "x upload");
    float* gy = c.y_dev;
    float* uy = c.y_dev + seq_len * num_rows;
    rc = c.q4_pair_batch_dev(c.find(hg), c.find(hu), c.x_dev, seq_len, gy, uy, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(gate_out, gy, seq_len * num_rows * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(up_out, uy, seq_len * num_rows * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "output download");
    return c.finish();
}

int larql_cuda_q4_matvec_pair_batch_dev(larql_cuda_ctx* ctx, uint64_t gate, uint64_t up, const float* x_dev,
                                        size_t seq_len, float* gate_out_dev, float* up_out_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* g = ctx->impl.find(gate);
    larql::Weight* u = ctx->impl.find(up);
    if (!g || !u) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!x_dev || !gate_out_dev || !up_out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    return ctx->impl.q4_pair_batch_dev(g, u, x_dev, seq_len, gate_out_dev, up_out_dev,
                                       stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
}

int larql_cuda_q4_matvec_dev(larql_cuda_ctx* ctx, uint64_t handle, const int8_t* q8_x_dev, const float* q8_scales_dev,
                             float* y_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!q8_x_dev || !q8_scales_dev || !y_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    return ctx->impl.q4_matvec_q8_dev(w, q8_x_dev, q8_scales_dev, y_dev,
                                      stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
}

int larql_cuda_logit_topk_dev(larql_cuda_ctx* ctx, const float* logits_dev, size_t n, size_t top_k,
                              uint32_t* ids_dev, float* logits_out_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!logits_dev || !ids_dev || !logits_out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    return ctx->impl.logit_topk_dev(logits_dev, n, top_k, ids_dev, logits_out_dev,
                                    stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
}

int larql_cuda_lm_head_knn_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* query_dev, size_t top_k,
                               uint32_t* ids_dev, float* logits_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!query_dev || !ids_dev || !logits_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    return ctx->impl.lm_head_knn_dev(w, query_dev, top_k, ids_dev, logits_dev,
                                     stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
}

int larql_cuda_lm_head_knn(larql_cuda_ctx* ctx, const uint8_t* q4_data, size_t nbytes, size_t vocab, size_t hidden,
                           const float* query, size_t top_k, uint32_t* out_ids, float* out_logits, size_t* out_count) {
    LARQL_CTX_GUARD(ctx);
    if (!q4_data || !query || !out_ids || !out_logits || !out_count) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    *out_count = 0;
    if (vocab == 0) return LARQL_OK;
    uint64_t h;
    int rc = ctx->impl.weight_for(q4_data, nbytes, LARQL_FMT_Q4_0, vocab, hidden, &h);
    if (rc) return rc;
    Ctx& c = ctx->impl;
    const size_t k = top_k < vocab ? top_k : vocab;
    rc = c.ensure_io(hidden, 64);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, query, hidden * 4, cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    uint32_t* ids = reinterpret_cast<uint32_t*>(c.y_dev);
    float* vals = c.y_dev + 32;
    rc = c.lm_head_knn_dev(c.find(h), c.x_dev, top_k, ids, vals, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out_ids, ids, k * 4, cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_logits, vals, k * 4, cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k download");
    rc = c.finish();
    if (rc == LARQL_OK) *out_count = k;
    return rc;
}

int larql_cuda_quantize_to_q8_dev(larql_cuda_ctx* ctx, const float* x_dev, size_t n, int8_t* q8_dev, float* scales_dev,
                                  void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!x_dev || !q8_dev || !scales_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n % 32) return fail(LARQL_ERR_BAD_SHAPE, "n=%zu is not a multiple of 32", n);
    cudaError_t e = larql::launch_quantize_to_q8(x_dev, n, q8_dev, scales_dev,
                                                 stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream);
    if (e != cudaSuccess) return cuda_fail(e, "quantize_to_q8 launch");
    return LARQL_OK;
}

int larql_cuda_matvec(larql_cuda_ctx* ctx, uint64_t handle, const float* x, size_t batch, float* y) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (batch == 0) return LARQL_OK;
    return ctx->impl.matvec_host(w, x, batch, y);
}

int larql_cuda_matvec_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* x_dev, size_t batch, float* y_dev,
                          void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!x_dev || !y_dev) return fail(LARQL_ERR_INVALID_ARG, "null x or y");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.matvec_dev(w, x_dev, batch, y_dev, s);
}

int larql_cuda_quantize_q4_k_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n, uint8_t* out_dev,
                                 void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!data_dev || !out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n % 256) return fail(LARQL_ERR_BAD_SHAPE, "n=%zu is not a multiple of 256", n);
    if (reinterpret_cast<uintptr_t>(data_dev) % 16 || reinterpret_cast<uintptr_t>(out_dev) % 4)
        return fail(LARQL_ERR_INVALID_ARG, "data must be 16-byte and out 4-byte aligned");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    cudaError_t e = larql::launch_quantize_q4_k(data_dev, n, out_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "quantize_q4_k launch");
    return LARQL_OK;
}

static int quantize_block32_dev(larql_cuda_ctx* ctx, int fmt, const float* data_dev, size_t n, uint8_t* out_dev,
                                void* stream) {
    if (!data_dev || !out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n % 32) return fail(LARQL_ERR_BAD_SHAPE, "n=%zu is not a multiple of 32", n);
    if (reinterpret_cast<uintptr_t>(data_dev) % 4) return fail(LARQL_ERR_INVALID_ARG, "data must be 4-byte aligned");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    cudaError_t e = larql::launch_quantize_block32(fmt, data_dev, n, out_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "block quantizer launch");
    return LARQL_OK;
}

int larql_cuda_quantize_q4_0_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n, uint8_t* out_dev,
                                 void* stream) {
    LARQL_CTX_GUARD(ctx);
    return quantize_block32_dev(ctx, 0, data_dev, n, out_dev, stream);
}

int larql_cuda_quantize_q8_0_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n, uint8_t* out_dev,
                                 void* stream) {
    LARQL_CTX_GUARD(ctx);
    return quantize_block32_dev(ctx, 1, data_dev, n, out_dev, stream);
}

int larql_cuda_quantize_q6_k_dev(larql_cuda_ctx* ctx, const float* data_dev, size_t n, uint8_t* out_dev,
                                 void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!data_dev || !out_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n % 256) return fail(LARQL_ERR_BAD_SHAPE, "n=%zu is not a multiple of 256", n);
    if (reinterpret_cast<uintptr_t>(data_dev) % 16) return fail(LARQL_ERR_INVALID_ARG, "data must be 16-byte aligned");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    cudaError_t e = larql::launch_quantize_q6_k(data_dev, n, out_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "quantize_q6_k launch");
    return LARQL_OK;
}

int larql_cuda_gate_topk_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                             const float* queries_dev, size_t batch, size_t top_k, uint32_t* out_idx_dev,
                             float* out_score_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!queries_dev || !out_idx_dev || !out_score_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.gate_topk_dev(w, n_layers, n_feat, queries_dev, batch, top_k, out_idx_dev, out_score_dev, s);
}

int larql_cuda_topk_merge_dev(larql_cuda_ctx* ctx, const uint32_t* idx_in, const float* score_in, size_t n_lists,
                              size_t rows, size_t k_in, const uint32_t* offsets_dev, size_t k_out, uint32_t* idx_out,
                              float* score_out, void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!idx_in || !score_in || !idx_out || !score_out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n_lists == 0 || k_in == 0 || n_lists * k_in > 512 || rows > 0x7fffffff || k_out > 512)
        return fail(LARQL_ERR_BAD_SHAPE, "merge of %zu lists x %zu (<= 512 candidates per row)", n_lists, k_in);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    cudaError_t e = larql::launch_topk_merge_lists(idx_in, score_in, static_cast<int>(n_lists), static_cast<int>(rows),
                                                   static_cast<int>(k_in), offsets_dev, static_cast<int>(k_out),
                                                   idx_out, score_out, s);
    if (e != cudaSuccess) return cuda_fail(e, "top-k merge launch");
    return LARQL_OK;
}

int larql_cuda_gate_topk_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes, size_t n_layers,
                             size_t n_feat, size_t hidden, const float* queries, size_t batch, size_t top_k,
                             uint32_t* out_idx, float* out_score) {
    LARQL_CTX_GUARD(ctx);
    if (!gates || !queries || !out_idx || !out_score) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (batch == 0 || top_k == 0 || n_layers == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    uint64_t h;
    int rc = c.weight_for(gates, nbytes, LARQL_FMT_F16_HALFRS, n_layers * n_feat, hidden, &h);
    if (rc) return rc;
    const size_t nout = n_layers * batch * top_k;
    // queries, then the outputs, in the context's io buffers
    rc = c.ensure_io(batch * hidden, 2 * nout);
    if (rc) return rc;
    uint32_t* di = reinterpret_cast<uint32_t*>(c.y_dev);
    float* ds = c.y_dev + nout;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, queries, batch * hidden * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    rc = c.gate_topk_dev(c.find(h), n_layers, n_feat, c.x_dev, batch, top_k, di, ds, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out_idx, di, nout * sizeof(uint32_t), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_score, ds, nout * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k download");
    return c.finish();
}

int larql_cuda_gate_topk_q4_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                                const float* queries_dev, size_t batch, size_t top_k, uint32_t* out_idx_dev,
                                float* out_score_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!queries_dev || !out_idx_dev || !out_score_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.gate_topk_q4_dev(w, n_layers, n_feat, queries_dev, batch, top_k, out_idx_dev, out_score_dev, s);
}

int larql_cuda_gate_topk_q4(larql_cuda_ctx* ctx, const uint8_t* gates_q4, size_t nbytes, size_t n_layers,
                            size_t n_feat, size_t hidden, const float* queries, size_t batch, size_t top_k,
                            uint32_t* out_idx, float* out_score) {
    LARQL_CTX_GUARD(ctx);
    if (!gates_q4 || !queries || !out_idx || !out_score) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (batch == 0 || top_k == 0 || n_layers == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    uint64_t h;
    int rc = c.weight_for(gates_q4, nbytes, LARQL_FMT_Q4_0, n_layers * n_feat, hidden, &h);
    if (rc) return rc;
    const size_t nout = n_layers * batch * top_k;
    rc = c.ensure_io(batch * hidden, 2 * nout);
    if (rc) return rc;
    uint32_t* di = reinterpret_cast<uint32_t*>(c.y_dev);
    float* ds = c.y_dev + nout;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, queries, batch * hidden * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    rc = c.gate_topk_q4_dev(c.find(h), n_layers, n_feat, c.x_dev, batch, top_k, di, ds, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out_idx, di, nout * sizeof(uint32_t), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_score, ds, nout * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k download");
    return c.finish();
}

int larql_cuda_gate_scores_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes, size_t n_layers,
                               size_t n_feat, size_t hidden, const float* queries, size_t batch, float* out_scores) {
    LARQL_CTX_GUARD(ctx);
    if (!gates || !queries || !out_scores) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (batch == 0 || n_layers == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    uint64_t h;
    int rc = c.weight_for(gates, nbytes, LARQL_FMT_F16_HALFRS, n_layers * n_feat, hidden, &h);
    if (rc) return rc;
    const size_t nout = n_layers * batch * n_feat;
    rc = c.ensure_io(batch * hidden, nout);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, queries, batch * hidden * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    rc = c.gate_topk_dev(c.find(h), n_layers, n_feat, c.x_dev, batch, 1, nullptr, nullptr, c.stream, c.y_dev);
    if (rc) return rc;
    e = cudaMemcpyAsync(out_scores, c.y_dev, nout * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "score download");
    return c.finish();
}

int larql_cuda_gate_scores_dev(larql_cuda_ctx* ctx, uint64_t handle, size_t n_layers, size_t n_feat,
                               const float* queries_dev, size_t batch, float* out_scores_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    larql::Weight* w = c.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!queries_dev || !out_scores_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    return c.gate_topk_dev(w, n_layers, n_feat, queries_dev, batch, 1, nullptr, nullptr, s, out_scores_dev);
}

int larql_cuda_gate_knn_batch_f16(larql_cuda_ctx* ctx, const uint16_t* gates, size_t nbytes, size_t n_feat,
                                  size_t hidden, const float* x, size_t seq_len, size_t top_k, uint32_t* out_idx,
                                  size_t* out_count) {
    LARQL_CTX_GUARD(ctx);
    if (!gates || !x || !out_idx || !out_count) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    *out_count = 0;
    if (seq_len == 0 || top_k == 0) return LARQL_OK;
    const size_t k = std::min(top_k, n_feat);
    // per-position top-k on the device (the context lock is already held: no nested ABI call)
    Ctx& c = ctx->impl;
    uint64_t h;
    int rc = c.weight_for(gates, nbytes, LARQL_FMT_F16_HALFRS, n_feat, hidden, &h);
    if (rc) return rc;
    const size_t nout = seq_len * top_k;
    rc = c.ensure_io(seq_len * hidden, 2 * nout);
    if (rc) return rc;
    uint32_t* di = reinterpret_cast<uint32_t*>(c.y_dev);
    cudaError_t e = cudaMemcpyAsync(c.x_dev, x, seq_len * hidden * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    rc = c.gate_topk_dev(c.find(h), 1, n_feat, c.x_dev, seq_len, top_k, di, c.y_dev + nout, c.stream);
    if (rc) return rc;
    std::vector<uint32_t> idx(nout);
    e = cudaMemcpyAsync(idx.data(), di, nout * sizeof(uint32_t), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k download");
    rc = c.finish();
    if (rc) return rc;
    // union of the per-position top-k (gate.rs:522-535 collects them into a BTreeSet): sorted, unique
    std::vector<uint32_t> u;
    u.reserve(seq_len * k);
    for (size_t s = 0; s < seq_len; ++s)
        for (size_t i = 0; i < k; ++i)
            if (idx[s * top_k + i] != 0xFFFFFFFFu) u.push_back(idx[s * top_k + i]);
    std::sort(u.begin(), u.end());
    u.erase(std::unique(u.begin(), u.end()), u.end());
    std::copy(u.begin(), u.end(), out_idx);
    *out_count = u.size();
    return LARQL_OK;
}

int larql_cuda_layer_register(larql_cuda_ctx* ctx, const larql_cuda_layer_desc* d, size_t hidden, size_t inter,
                              size_t nq, size_t nkv, size_t head_dim, int src_is_device, uint64_t* handle) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.layer_register(d, hidden, inter, nq, nkv, head_dim, src_is_device != 0, handle);
}

int larql_cuda_layer_register_shard(larql_cuda_ctx* ctx, const larql_cuda_layer_desc* d, size_t hidden, size_t inter,
                                    size_t nq, size_t nkv, size_t head_dim, size_t rank, size_t world,
                                    int src_is_device, uint64_t* handle) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.layer_register_shard(d, hidden, inter, nq, nkv, head_dim, rank, world, src_is_device != 0,
                                          handle);
}

int larql_cuda_decode_token_sharded_dev(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers, float* x_dev,
                                        size_t pos, float rope_base, float* red_dev, larql_cuda_reduce_fn reduce,
                                        void* user, void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!layers || !x_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    Ctx& c = ctx->impl;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    return c.decode_sharded_dev(layers, n_layers, x_dev, pos, rope_base, red_dev, reduce, user, s);
}

int larql_cuda_p2p_init(larql_cuda_ctx* ctx, size_t rank, size_t world, size_t max_n, void* ipc_handle) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (!ipc_handle) return fail(LARQL_ERR_INVALID_ARG, "null handle output");
    if (world < 2 || world > static_cast<size_t>(larql::kP2pMaxRanks) || rank >= world || max_n == 0 ||
        max_n % 4 || max_n > (1u << 24))
        return fail(LARQL_ERR_BAD_SHAPE, "peer all-reduce for rank %zu of %zu, %zu floats", rank, world, max_n);
    if (c.p2p_local) return fail(LARQL_ERR_INVALID_ARG, "peer all-reduce already initialised");
    const size_t bytes = larql::p2p_area_bytes(static_cast<int>(world), static_cast<int>(max_n));
    cudaError_t e = cudaMalloc(&c.p2p_local, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c.p2p_epoch, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c.p2p_local, 0, bytes);
    if (e == cudaSuccess) e = cudaMemset(c.p2p_epoch, 0, sizeof(int));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c.p2p_local);
    if (e != cudaSuccess) {
        if (c.p2p_local) cudaFree(c.p2p_local);
        if (c.p2p_epoch) cudaFree(c.p2p_epoch);
        c.p2p_local = nullptr;
        c.p2p_epoch = nullptr;
        return cuda_fail(e, "peer all-reduce area");
    }
    memcpy(ipc_handle, &h, sizeof(h));
    c.p2p_rank = static_cast<int>(rank);
    c.p2p_world = static_cast<int>(world);
    c.p2p_max_n = static_cast<int>(max_n);
    return LARQL_OK;
}

int larql_cuda_p2p_connect(larql_cuda_ctx* ctx, const void* handles) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (!handles) return fail(LARQL_ERR_INVALID_ARG, "null handles");
    if (!c.p2p_local) return fail(LARQL_ERR_INVALID_ARG, "larql_cuda_p2p_init first");
    if (c.p2p_ready) return LARQL_OK;
    for (int p = 0; p < c.p2p_world; ++p) {
        if (p == c.p2p_rank) {
            c.p2p_areas.base[p] = c.p2p_local;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + p * sizeof(cudaIpcMemHandle_t), sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < p; ++q)
                if (q != c.p2p_rank && c.p2p_areas.base[q]) cudaIpcCloseMemHandle(c.p2p_areas.base[q]);
            c.p2p_areas = larql::P2pAreas{};
            return cuda_fail(e, "opening a peer's all-reduce area");
        }
        c.p2p_areas.base[p] = ptr;
    }
    c.p2p_ready = true;
    return LARQL_OK;
}

int larql_cuda_p2p_allreduce_dev(larql_cuda_ctx* ctx, float* buf_dev, size_t n, void* stream) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (!c.p2p_ready) return fail(LARQL_ERR_INVALID_ARG, "peer all-reduce not connected");
    if (!buf_dev || reinterpret_cast<uintptr_t>(buf_dev) % 16) return fail(LARQL_ERR_INVALID_ARG, "buffer must be 16-byte aligned");
    if (n == 0) return LARQL_OK;
    if (n > static_cast<size_t>(c.p2p_max_n)) return fail(LARQL_ERR_BAD_SHAPE, "%zu floats > %d", n, c.p2p_max_n);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    cudaError_t e = larql::launch_p2p_allreduce(c.p2p_areas, c.p2p_rank, c.p2p_world, c.p2p_max_n, static_cast<int>(n),
                                                buf_dev, buf_dev, c.p2p_epoch, c.status_dev, s);
    if (e != cudaSuccess) return cuda_fail(e, "peer all-reduce launch");
    return LARQL_OK;
}

int larql_cuda_layer_release(larql_cuda_ctx* ctx, uint64_t handle) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    auto it = c.layers.find(handle);
    if (it == c.layers.end()) return fail(LARQL_ERR_NOT_FOUND, "unknown layer handle");
    cudaStreamSynchronize(c.stream);
    for (uint64_t h : {it->second.qkv, it->second.o, it->second.gu, it->second.down}) c.release_handle(h);
    if (it->second.norms) cudaFree(it->second.norms);
    c.layers.erase(it);
    return LARQL_OK;
}

int larql_cuda_kv_init(larql_cuda_ctx* ctx, size_t n_layers, size_t max_seq, size_t nkv, size_t head_dim) {
    LARQL_CTX_GUARD(ctx);
    return ctx->impl.kv_init(n_layers, max_seq, nkv, head_dim);
}

int larql_cuda_kv_populate(larql_cuda_ctx* ctx, size_t layer, const float* k, const float* v, size_t seq_len) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (layer >= c.kv.size()) return fail(LARQL_ERR_BAD_SHAPE, "kv layer %zu of %zu", layer, c.kv.size());
    if (seq_len > c.kv_max_seq) return fail(LARQL_ERR_BAD_SHAPE, "seq_len %zu > kv capacity %zu", seq_len, c.kv_max_seq);
    if (!k || !v) return fail(LARQL_ERR_INVALID_ARG, "null k / v");
    const size_t n = seq_len * c.kv_nkv * c.kv_hd;
    int rc = c.ensure_io(2 * n, 0);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, k, n * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c.x_dev + n, v, n * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e == cudaSuccess) e = larql::launch_f32_to_f16(c.x_dev, n, c.kv[layer].k, c.stream);
    if (e == cudaSuccess) e = larql::launch_f32_to_f16(c.x_dev + n, n, c.kv[layer].v, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "kv populate");
    c.kv_len = seq_len;
    return c.finish();
}

int larql_cuda_kv_populate_f16_dev(larql_cuda_ctx* ctx, size_t layer, const void* k, const void* v, size_t seq_len,
                                   void* stream) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (layer >= c.kv.size()) return fail(LARQL_ERR_BAD_SHAPE, "kv layer %zu of %zu", layer, c.kv.size());
    if (seq_len > c.kv_max_seq) return fail(LARQL_ERR_BAD_SHAPE, "seq_len %zu > kv capacity %zu", seq_len, c.kv_max_seq);
    if (!k || !v) return fail(LARQL_ERR_INVALID_ARG, "null k / v");
    const size_t bytes = seq_len * c.kv_nkv * c.kv_hd * sizeof(__half);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c.stream;
    cudaError_t e = cudaMemcpyAsync(c.kv[layer].k, k, bytes, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c.kv[layer].v, v, bytes, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e, "kv populate");
    c.kv_len = seq_len;
    return LARQL_OK;
}

int larql_cuda_kv_reset(larql_cuda_ctx* ctx) {
    LARQL_CTX_GUARD(ctx);
    ctx->impl.kv_len = 0;
    return LARQL_OK;
}

int larql_cuda_decode_set_persistent(larql_cuda_ctx* ctx, int on) {
    LARQL_CTX_GUARD(ctx);
    ctx->impl.decode_persist = on != 0;
    return LARQL_OK;
}

int larql_cuda_kv_set_length(larql_cuda_ctx* ctx, size_t len) {
    LARQL_CTX_GUARD(ctx);
    if (len > ctx->impl.kv_max_seq) return fail(LARQL_ERR_BAD_SHAPE, "length %zu > capacity", len);
    ctx->impl.kv_len = len;
    return LARQL_OK;
}

int larql_cuda_kv_length(larql_cuda_ctx* ctx, size_t* len) {
    LARQL_CTX_GUARD(ctx);
    if (!len) return fail(LARQL_ERR_INVALID_ARG, "null out");
    *len = ctx->impl.kv_len;
    return LARQL_OK;
}

int larql_cuda_decode_token(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers, const float* x,
                            float rope_base, float* out) {
    LARQL_CTX_GUARD(ctx);
    Ctx& c = ctx->impl;
    if (!layers || !x || !out) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n_layers == 0) return LARQL_OK;
    auto it = c.layers.find(layers[0]);
    if (it == c.layers.end()) return fail(LARQL_ERR_NOT_FOUND, "unknown layer handle");
    const size_t hidden = it->second.hidden;
    int rc = c.ensure_io(hidden, hidden);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, x, hidden * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "x upload");
    rc = c.decode_dev(layers, n_layers, c.x_dev, c.kv_len, rope_base, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out, c.x_dev, hidden * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "x download");
    rc = c.finish();
    if (!rc) c.kv_len += 1;
    return rc;
}

int larql_cuda_decode_token_dev(larql_cuda_ctx* ctx, const uint64_t* layers, size_t n_layers, float* x_dev,
                                size_t pos, float rope_base, void* stream) {
    LARQL_CTX_GUARD(ctx);
    if (!layers || !x_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.decode_dev(layers, n_layers, x_dev, pos, rope_base, s);
}

int larql_cuda_q4k_gemm_dev(larql_cuda_ctx* ctx, uint64_t handle, const float* x_dev, size_t n_tokens, float* y_dev,
                            void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!x_dev || !y_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.gemm_q4k_dev(w, x_dev, n_tokens, y_dev, s);
}

int larql_cuda_prefill_ffn_dev(larql_cuda_ctx* ctx, uint64_t gate, uint64_t up, uint64_t down, const float* x_dev,
                               size_t n_tokens, float* y_dev, void* stream) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* wg = ctx->impl.find(gate);
    larql::Weight* wu = ctx->impl.find(up);
    larql::Weight* wd = ctx->impl.find(down);
    if (!wg || !wu || !wd) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!x_dev || !y_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->impl.stream;
    return ctx->impl.prefill_ffn_dev(wg, wu, wd, x_dev, n_tokens, y_dev, s);
}

int larql_cuda_prefill_ffn(larql_cuda_ctx* ctx, const uint8_t* gate, size_t gate_bytes, const uint8_t* up,
                           size_t up_bytes, const uint8_t* down, size_t down_bytes, size_t hidden, size_t inter,
                           const float* x, size_t n_tokens, float* y) {
    LARQL_CTX_GUARD(ctx);
    if (!gate || !up || !down || !x || !y) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (n_tokens == 0) return LARQL_OK;
    Ctx& c = ctx->impl;
    uint64_t hg, hu, hd;
    int rc = c.weight_for(gate, gate_bytes, LARQL_FMT_Q4_K, inter, hidden, &hg);
    if (!rc) rc = c.weight_for(up, up_bytes, LARQL_FMT_Q4_K, inter, hidden, &hu);
    if (!rc) rc = c.weight_for(down, down_bytes, LARQL_FMT_Q4_K, hidden, inter, &hd);
    if (rc) return rc;
    const size_t n = n_tokens * hidden;
    rc = c.ensure_io(n, n);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, x, n * sizeof(float), cudaMemcpyHostToDevice, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "activation upload");
    rc = c.prefill_ffn_dev(c.find(hg), c.find(hu), c.find(hd), c.x_dev, n_tokens, c.y_dev, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(y, c.y_dev, n * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "output download");
    return c.finish();
}

int larql_cuda_describe_matvec(larql_cuda_ctx* ctx, uint64_t handle, size_t batch, char* buf, size_t len) {
    LARQL_CTX_GUARD(ctx);
    larql::Weight* w = ctx->impl.find(handle);
    if (!w) return fail(LARQL_ERR_NOT_FOUND, "unknown weight handle");
    if (!buf || len == 0) return fail(LARQL_ERR_INVALID_ARG, "null buffer");
    if (batch == 0 || batch > 8) return fail(LARQL_ERR_BAD_SHAPE, "batch %zu", batch);
    if (w->format == LARQL_FMT_Q4_K) return ctx->impl.describe_q4k(w, batch, buf, len);
    if (const larql::MmaPlan* mp = ctx->impl.blk_mma_plan(w, batch)) {
        snprintf(buf, len, "q4k_mma_kernel<%zu, %s> groups=%d slices=%d rows/tile=%d parts=%d stages=%d grid=%d "
                 "warps=%d", batch,
                 mp->fmt == 1 ? "Q4_0"
                 : (mp->fmt == 4 ? "Q6_K"
                                 : (mp->fmt == 5 ? "Q4_K_GGUF" : (mp->fmt == 6 ? "Q4_K_GGUF_LLAMA" : "Q8_0"))),
                 mp->NG,
                 mp->KS, mp->RT,
                 mp->nparts, mp->NS,
                 mp->grid, mp->NW + 1);
        return LARQL_OK;
    }
    const char* k = w->format == LARQL_FMT_Q4_0 ? "blk_matvec_kernel<Q4_0> (dp4a), one launch per batch row"
                    : w->format == LARQL_FMT_Q8_0_GGUF ? "blk_matvec_kernel<Q8_0> (dp4a), one launch per batch row"
                    : w->format == LARQL_FMT_Q8_0 ? "quantize_to_q8_kernel + blk_matvec_kernel<Q8 compute layout>"
                    : w->format == LARQL_FMT_Q6_K ? "blk_matvec_kernel<Q6_K> (dp4a), one launch per batch row"
                    : w->format == LARQL_FMT_Q4_K_GGUF ? "q4k_matvec_pair_kernel<GGUF-144> (dp4a), one launch per batch row"
                                                   : "not provided";
    snprintf(buf, len, "%s", k);
    return LARQL_OK;
}

int larql_cuda_launch_count(uint64_t* out) {
    if (!out) return fail(LARQL_ERR_INVALID_ARG, "null out");
    *out = larql::launch_counter().load(std::memory_order_relaxed);
    return LARQL_OK;
}

}  // extern "C"
