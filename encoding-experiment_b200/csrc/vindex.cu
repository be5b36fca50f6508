// vindex.cu — a .vindex directory read once and placed on the GPU (host C++ plus one query-layout kernel).
//
// Reference: crates/larql-vindex/src/format/load.rs:19-87 (VectorIndex::load_vindex: index.json, gate_vectors.bin
// mapped, per-layer slices from the layers[] byte offsets), crates/larql-vindex/src/config/types.rs (VindexConfig,
// VindexLayerInfo), crates/larql-vindex/src/config/dtype.rs (dtype "f32" | "f16", f32 when absent),
// crates/larql-vindex/src/index/walk.rs:225 (interleaved_q4k.bin) and :402-445 (attn_weights_q4k.bin and its
// manifest), crates/larql-inference/src/layer_graph/pipeline_layer.rs:121-134 (how the FFN file is sliced).
//
// Gate rows go to the device once, in the layout the gate walk (gate_tc.cu, gate_gemv.cu) reads: per layer a block
// of `per` rows (this shard's share of the largest layer, zero rows after a short layer's end) of Dp values, Dp
// the hidden size rounded up to 64 with zeros.  f16 rows are stored as they are and decoded as half.rs does
// (LARQL_FMT_F16_HALFRS).  f32 rows become an f16 pair [hi | lo * 2^12] (hi = f16(g), lo = g - hi; IEEE decoding,
// LARQL_FMT_F16) and each query the matching pair [q | q * 2^-12], so the walk's f32 scores see g to ~22 bits.
//
// The interleaved FFN file is read as the reference's writer lays it out (crates/larql-vindex/examples/
// build_q4k_weights.rs: per layer gate and up in Q4_K, then down in Q6_K) or, when its size says so, as the
// reader slices it (three equal Q4_K matrices per layer); both are recognised from the file size.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "backend.h"
#include "common.cuh"
#include "kernels.h"

namespace larql {

// ───────────── a small JSON reader (objects, arrays, strings, numbers, literals) ─────────────
namespace json {

struct Value {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;

    const Value* get(const char* key) const {
        if (kind != kObj) return nullptr;
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class Parser {
  public:
    Parser(const char* s, size_t n) : p_(s), end_(s + n) {}
    bool parse(Value* out, std::string* err) {
        ws();
        if (!value(out, 0)) {
            *err = err_.empty() ? "malformed JSON" : err_;
            return false;
        }
        ws();
        if (p_ != end_) {
            *err = "trailing characters after the JSON value";
            return false;
        }
        return true;
    }

  private:
    const char* p_;
    const char* end_;
    std::string err_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = strlen(w);
        if (static_cast<size_t>(end_ - p_) < n || memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    bool str(std::string* out) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            char c = *p_++;
            if (c == '\\') {
                if (p_ >= end_) return false;
                const char e = *p_++;
                switch (e) {
                    case '"': c = '"'; break;
                    case '\\': c = '\\'; break;
                    case '/': c = '/'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'n': c = '\n'; break;
                    case 'r': c = '\r'; break;
                    case 't': c = '\t'; break;
                    case 'u': {  // keys and values read here are ASCII; other code points are kept as '?'
                        if (end_ - p_ < 4) return false;
                        p_ += 4;
                        c = '?';
                        break;
                    }
                    default: return false;
                }
            }
            out->push_back(c);
        }
        if (p_ >= end_) return false;
        ++p_;
        return true;
    }
    bool value(Value* v, int depth) {
        if (depth > 64) {
            err_ = "JSON nested too deeply";
            return false;
        }
        ws();
        if (p_ >= end_) return false;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v->kind = Value::kObj;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            for (;;) {
                ws();
                std::string key;
                if (!str(&key)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                Value item;
                if (!value(&item, depth + 1)) return false;
                v->obj.emplace_back(std::move(key), std::move(item));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v->kind = Value::kArr;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            for (;;) {
                Value item;
                if (!value(&item, depth + 1)) return false;
                v->arr.push_back(std::move(item));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v->kind = Value::kStr;
            return str(&v->str);
        }
        if (lit("true")) {
            v->kind = Value::kBool;
            v->b = true;
            return true;
        }
        if (lit("false")) {
            v->kind = Value::kBool;
            return true;
        }
        if (lit("null")) {
            v->kind = Value::kNull;
            return true;
        }
        // number
        const char* s = p_;
        while (p_ < end_ && (isdigit(static_cast<unsigned char>(*p_)) || *p_ == '-' || *p_ == '+' || *p_ == '.' ||
                             *p_ == 'e' || *p_ == 'E'))
            ++p_;
        if (p_ == s) return false;
        const std::string t(s, p_);
        char* e = nullptr;
        v->num = strtod(t.c_str(), &e);
        if (!e || *e != '\0') return false;
        v->kind = Value::kNum;
        return true;
    }
};

}  // namespace json

namespace {

// a whole file read into memory (index.json, manifests)
bool read_text(const std::string& path, std::string* out) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return false;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out->append(buf, n);
    const bool ok = !ferror(f);
    fclose(f);
    return ok;
}

bool file_size(const std::string& path, size_t* out) {
    struct stat st;
    if (stat(path.c_str(), &st) != 0 || !S_ISREG(st.st_mode)) return false;
    *out = static_cast<size_t>(st.st_size);
    return true;
}

// A read-only mapping of a whole file.
struct Mapped {
    const uint8_t* data = nullptr;
    size_t size = 0;
    bool open(const std::string& path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) return false;
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            return false;
        }
        size = static_cast<size_t>(st.st_size);
        if (size == 0) {
            ::close(fd);
            return true;
        }
        void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (p == MAP_FAILED) {
            size = 0;
            return false;
        }
        data = static_cast<const uint8_t*>(p);
        return true;
    }
    ~Mapped() {
        if (data) munmap(const_cast<uint8_t*>(data), size);
    }
};

bool as_size(const json::Value* v, size_t* out) {
    if (!v || v->kind != json::Value::kNum || !(v->num >= 0) || v->num > 9.0e15 || v->num != std::floor(v->num))
        return false;
    *out = static_cast<size_t>(v->num);
    return true;
}

struct LayerInfo {
    size_t features = 0, offset = 0, length = 0;
};
struct AttnEntry {
    size_t offset = 0, length = 0, rows = 0, cols = 0;
    int format = LARQL_FMT_Q4_K;
};

// Everything index.json and the manifests say, checked against the file sizes.
struct Layout {
    std::string dir;
    size_t num_layers = 0, hidden = 0, inter = 0, vocab = 0, features_max = 0;
    int gate_bits = 32;
    std::vector<LayerInfo> layers;
    size_t head_dim = 0, nq = 0, nkv = 0;  // model_config, when present
    int ffn = 0;                           // 0 none, 1 three Q4_K matrices per layer, 2 down in Q6_K
    size_t ffn_q4k_bytes = 0, ffn_down_bytes = 0;
    int attn = 0;
    int gate_q4 = 0;  // gate_vectors_q4.bin present (Q4_0 rows of every layer, layers contiguous)
    std::vector<AttnEntry> attn_entries;
};

size_t q4k_bytes(size_t n) { return (n + 255) / 256 * 148; }
size_t q6k_bytes(size_t n) { return (n + 255) / 256 * 210; }

int probe(const char* dir, Layout* L) {
    if (!dir) return fail(LARQL_ERR_INVALID_ARG, "null vindex directory");
    L->dir = dir;
    std::string text, err;
    if (!read_text(L->dir + "/index.json", &text))
        return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot read %s/index.json", dir);
    json::Value cfg;
    if (!json::Parser(text.data(), text.size()).parse(&cfg, &err))
        return fail(LARQL_ERR_INVALID_ARG, "vindex: index.json: %s", err.c_str());
    if (cfg.kind != json::Value::kObj) return fail(LARQL_ERR_INVALID_ARG, "vindex: index.json is not an object");
    if (!as_size(cfg.get("num_layers"), &L->num_layers) || !as_size(cfg.get("hidden_size"), &L->hidden) ||
        L->num_layers == 0 || L->hidden == 0)
        return fail(LARQL_ERR_INVALID_ARG, "vindex: index.json needs positive num_layers and hidden_size");
    as_size(cfg.get("intermediate_size"), &L->inter);
    as_size(cfg.get("vocab_size"), &L->vocab);
    if (const json::Value* dt = cfg.get("dtype")) {  // StorageDtype, lowercase; F32 by default
        if (dt->kind != json::Value::kStr || (dt->str != "f32" && dt->str != "f16"))
            return fail(LARQL_ERR_INVALID_ARG, "vindex: index.json dtype must be \"f32\" or \"f16\"");
        L->gate_bits = dt->str == "f16" ? 16 : 32;
    }
    const size_t bpf = L->gate_bits / 8;
    const json::Value* layers = cfg.get("layers");
    if (!layers || layers->kind != json::Value::kArr)
        return fail(LARQL_ERR_INVALID_ARG, "vindex: index.json has no layers[] array");
    L->layers.assign(L->num_layers, LayerInfo{});
    for (const json::Value& li : layers->arr) {
        size_t layer, nf, off, len;
        if (!as_size(li.get("layer"), &layer) || !as_size(li.get("num_features"), &nf) ||
            !as_size(li.get("offset"), &off) || !as_size(li.get("length"), &len))
            return fail(LARQL_ERR_INVALID_ARG, "vindex: a layers[] entry lacks layer / num_features / offset / length");
        if (layer >= L->num_layers)
            return fail(LARQL_ERR_INVALID_ARG, "vindex: layers[] names layer %zu of %zu", layer, L->num_layers);
        if (off % bpf) return fail(LARQL_ERR_INVALID_ARG, "vindex: layer %zu offset %zu is not whole floats", layer, off);
        if (nf * L->hidden * bpf > len)
            return fail(LARQL_ERR_INVALID_ARG, "vindex: layer %zu holds %zu bytes, %zu features x %zu need %zu", layer,
                        len, nf, L->hidden, nf * L->hidden * bpf);
        L->layers[layer] = LayerInfo{nf, off, len};
        L->features_max = std::max(L->features_max, nf);
    }
    if (L->features_max == 0) return fail(LARQL_ERR_INVALID_ARG, "vindex: no layer has gate features");
    size_t gsz = 0;
    if (!file_size(L->dir + "/gate_vectors.bin", &gsz))
        return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot stat %s/gate_vectors.bin", dir);
    for (size_t l = 0; l < L->num_layers; ++l) {
        const LayerInfo& li = L->layers[l];
        if (li.features && li.offset + li.features * L->hidden * bpf > gsz)
            return fail(LARQL_ERR_INVALID_ARG, "vindex: layer %zu gate rows end past gate_vectors.bin (%zu bytes)", l,
                        gsz);
    }
    // Q4_0 gates (walk.rs:303-328): layer l holds num_features * hidden / 32 blocks of 18 bytes, layers contiguous
    size_t q4sz = 0;
    if (file_size(L->dir + "/gate_vectors_q4.bin", &q4sz)) {
        size_t need = 0;
        for (const LayerInfo& li : L->layers) need += li.features * L->hidden / 32 * 18;
        if (L->hidden % 32 || q4sz < need)
            return fail(LARQL_ERR_INVALID_ARG, "vindex: gate_vectors_q4.bin has %zu bytes, the layers need %zu (hidden "
                        "%zu must be a multiple of 32)", q4sz, need, L->hidden);
        L->gate_q4 = 1;
    }
    if (const json::Value* mc = cfg.get("model_config")) {
        as_size(mc->get("head_dim"), &L->head_dim);
        as_size(mc->get("num_q_heads"), &L->nq);
        as_size(mc->get("num_kv_heads"), &L->nkv);
    }
    // FFN: interleaved_q4k.bin, recognised by its size
    size_t fsz = 0;
    if (L->inter && file_size(L->dir + "/interleaved_q4k.bin", &fsz)) {
        const size_t q4 = q4k_bytes(L->inter * L->hidden), q6 = q6k_bytes(L->inter * L->hidden);
        if (fsz == L->num_layers * (2 * q4 + q6)) {
            L->ffn = 2;
        } else if (fsz == L->num_layers * 3 * q4) {
            L->ffn = 1;
        } else {
            return fail(LARQL_ERR_INVALID_ARG,
                        "vindex: interleaved_q4k.bin has %zu bytes; %zu layers need %zu (Q4_K / Q4_K / Q6_K) or %zu "
                        "(three Q4_K)", fsz, L->num_layers, L->num_layers * (2 * q4 + q6), L->num_layers * 3 * q4);
        }
        L->ffn_q4k_bytes = q4;
        L->ffn_down_bytes = L->ffn == 2 ? q6 : q4;
    }
    // attention: attn_weights_q4k.bin + manifest (an array of {key, shape, format, offset, length}, 4 per layer)
    size_t asz = 0;
    std::string mtext;
    if (file_size(L->dir + "/attn_weights_q4k.bin", &asz) &&
        read_text(L->dir + "/attn_weights_q4k_manifest.json", &mtext)) {
        json::Value man;
        if (!json::Parser(mtext.data(), mtext.size()).parse(&man, &err))
            return fail(LARQL_ERR_INVALID_ARG, "vindex: attn_weights_q4k_manifest.json: %s", err.c_str());
        if (man.kind != json::Value::kArr)
            return fail(LARQL_ERR_INVALID_ARG, "vindex: attn_weights_q4k_manifest.json is not an array");
        for (size_t i = 0; i < man.arr.size(); ++i) {
            const json::Value& e = man.arr[i];
            AttnEntry a;
            if (!as_size(e.get("offset"), &a.offset) || !as_size(e.get("length"), &a.length))
                return fail(LARQL_ERR_INVALID_ARG, "vindex: manifest entry %zu lacks offset / length", i);
            const json::Value* f = e.get("format");
            const std::string fmt = f && f->kind == json::Value::kStr ? f->str : "Q4_K";  // walk.rs:417
            a.format = fmt == "Q6_K" ? LARQL_FMT_Q6_K : LARQL_FMT_Q4_K;
            const json::Value* sh = e.get("shape");
            if (sh && sh->kind == json::Value::kArr && sh->arr.size() == 2) {
                if (!as_size(&sh->arr[0], &a.rows) || !as_size(&sh->arr[1], &a.cols))
                    return fail(LARQL_ERR_INVALID_ARG, "vindex: manifest entry %zu has a bad shape", i);
            } else if (L->head_dim && L->nq && L->nkv) {  // Q, K, V, O from the model config
                const size_t q = L->nq * L->head_dim, kv = L->nkv * L->head_dim;
                const size_t r[4] = {q, kv, kv, L->hidden}, c[4] = {L->hidden, L->hidden, L->hidden, q};
                a.rows = r[i % 4];
                a.cols = c[i % 4];
            } else {
                return fail(LARQL_ERR_INVALID_ARG, "vindex: manifest entry %zu has no shape", i);
            }
            const size_t need = a.format == LARQL_FMT_Q6_K ? q6k_bytes(a.rows * a.cols) : q4k_bytes(a.rows * a.cols);
            if (a.cols % 256 || a.length < need || a.offset + a.length > asz)
                return fail(LARQL_ERR_INVALID_ARG, "vindex: manifest entry %zu ([%zu x %zu] %s, %zu bytes at %zu) does "
                            "not fit attn_weights_q4k.bin (%zu bytes)", i, a.rows, a.cols, fmt.c_str(), a.length,
                            a.offset, asz);
            L->attn_entries.push_back(a);
        }
        L->attn = L->attn_entries.size() >= 4 * L->num_layers ? 1 : 0;
    }
    return LARQL_OK;
}

void fill_info(const Layout& L, size_t rank, size_t count, size_t per, larql_cuda_vindex_info* info) {
    info->num_layers = L.num_layers;
    info->hidden = L.hidden;
    info->intermediate = L.inter;
    info->vocab = L.vocab;
    info->features_max = L.features_max;
    info->gate_bits = L.gate_bits;
    info->ffn_q4k = L.ffn;
    info->attn_q4k = L.attn;
    info->gate_q4 = L.gate_q4;
    info->shard_rank = rank;
    info->shard_count = count;
    info->shard_row0 = rank * per;
    info->shard_rows = per;
}

// queries [batch][hidden] -> the walk's layout [batch][cols]: zeros past hidden (f16 rows), or for f32 rows
// [q | 0 | q * 2^-12 | 0] with halves of Dp = cols / 2 values
__global__ void vindex_query_kernel(const float* __restrict__ q, int batch, int hidden, int cols, int split,
                                    float* __restrict__ out) {
    const size_t n = static_cast<size_t>(batch) * cols;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int b = static_cast<int>(i / cols), c = static_cast<int>(i - static_cast<size_t>(b) * cols);
        const int half = split ? cols / 2 : cols;
        const int k = c < half ? c : c - half;
        float v = k < hidden ? q[static_cast<size_t>(b) * hidden + k] : 0.f;
        if (split && c >= half) v *= 1.0f / 4096.0f;
        out[i] = v;
    }
}

}  // namespace

}  // namespace larql

struct larql_cuda_vindex {
    larql_cuda_ctx* ctx = nullptr;
    larql::Layout L;
    size_t rank = 0, count = 1, per = 0, cols = 0;
    uint64_t gate = 0;  // the placed gate rows: num_layers * per rows of `cols` f16 values
    uint64_t gate_q4 = 0;  // the placed Q4_0 gate rows (num_layers * per rows of hidden values), when present
    std::vector<size_t> rows_here;  // real rows of each layer on this shard
    std::unique_ptr<larql::Mapped> ffn_map, attn_map;
    std::vector<std::array<uint64_t, 3>> ffn;  // per layer gate / up / down handles (0 = not placed yet)
    std::vector<std::array<uint64_t, 4>> attn;
    float* qbuf = nullptr;  // query staging in the walk's layout
    size_t qcap = 0;
};

using larql::fail;
using larql::cuda_fail;

namespace {

// Releases a weight this vindex placed and forgets its (pointer, length) registry entry.
void drop(larql::Ctx& c, uint64_t h) {
    if (!h) return;
    for (auto it = c.by_ptr.begin(); it != c.by_ptr.end();) it = it->second == h ? c.by_ptr.erase(it) : std::next(it);
    c.release_handle(h);
}

void release_all(larql_cuda_vindex* v) {
    larql::Ctx& c = v->ctx->impl;
    cudaStreamSynchronize(c.stream);
    drop(c, v->gate);
    drop(c, v->gate_q4);
    v->gate = v->gate_q4 = 0;
    for (auto& h : v->ffn)
        for (uint64_t& x : h) {
            drop(c, x);
            x = 0;
        }
    for (auto& h : v->attn)
        for (uint64_t& x : h) {
            drop(c, x);
            x = 0;
        }
    if (v->qbuf) cudaFree(v->qbuf);
    v->qbuf = nullptr;
    v->qcap = 0;
}

// A row range [r0, r1) of a [rows x cols] Q4_K / Q6_K matrix stored at `src` (whole rows are contiguous).
int place_rows(larql_cuda_vindex* v, const uint8_t* src, int format, size_t rows, size_t cols, uint64_t* h) {
    larql::Ctx& c = v->ctx->impl;
    const size_t per = (rows + v->count - 1) / v->count;
    const size_t r0 = std::min(rows, v->rank * per), r1 = std::min(rows, r0 + per);
    if (r1 <= r0) return fail(LARQL_ERR_BAD_SHAPE, "vindex: shard %zu of %zu holds no rows of a %zu-row matrix",
                              v->rank, v->count, rows);
    const size_t row_bytes = larql::format_bytes(format, 1, cols);
    return c.add_weight(src + r0 * row_bytes, false, (r1 - r0) * row_bytes, nullptr, false, format, r1 - r0, cols, h);
}

int ensure_query(larql_cuda_vindex* v, size_t batch) {
    const size_t need = batch * v->cols;
    if (need <= v->qcap) return LARQL_OK;
    if (v->qbuf) cudaFree(v->qbuf);
    v->qbuf = nullptr;
    v->qcap = 0;
    cudaError_t e = cudaMalloc(&v->qbuf, need * sizeof(float) + 256);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(vindex queries)");
    v->qcap = need;
    return LARQL_OK;
}

int walk_dev(larql_cuda_vindex* v, const float* q_dev, size_t batch, size_t top_k, uint32_t* oi, float* os,
             cudaStream_t s) {
    larql::Ctx& c = v->ctx->impl;
    if (batch == 0 || top_k == 0) return LARQL_OK;
    if (top_k > 16) return fail(LARQL_ERR_UNSUPPORTED, "vindex gate walk: top_k %zu > 16", top_k);
    int rc = ensure_query(v, batch);
    if (rc) return rc;
    const size_t n = batch * v->cols;
    const int grid = static_cast<int>(std::min<size_t>((n + 255) / 256, 4 * 148));
    larql::vindex_query_kernel<<<grid, 256, 0, s>>>(q_dev, static_cast<int>(batch), static_cast<int>(v->L.hidden),
                                                    static_cast<int>(v->cols), v->L.gate_bits == 32 ? 1 : 0, v->qbuf);
    larql::note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "vindex query layout launch");
    return c.gate_topk_dev(c.find(v->gate), v->L.num_layers, v->per, v->qbuf, batch, top_k, oi, os, s);
}

}  // namespace

extern "C" {

int larql_cuda_vindex_probe(const char* dir, larql_cuda_vindex_info* info) {
    if (!info) return fail(LARQL_ERR_INVALID_ARG, "null info");
    larql::Layout L;
    int rc = larql::probe(dir, &L);
    if (rc) return rc;
    larql::fill_info(L, 0, 1, L.features_max, info);
    return LARQL_OK;
}

int larql_cuda_vindex_open(larql_cuda_ctx* ctx, const char* dir, size_t shard_rank, size_t shard_count,
                           larql_cuda_vindex** out) {
    LARQL_CTX_GUARD(ctx);
    if (!out) return fail(LARQL_ERR_INVALID_ARG, "null output");
    *out = nullptr;
    if (shard_count == 0 || shard_rank >= shard_count)
        return fail(LARQL_ERR_INVALID_ARG, "vindex: shard %zu of %zu", shard_rank, shard_count);
    auto v = std::make_unique<larql_cuda_vindex>();
    v->ctx = ctx;
    int rc = larql::probe(dir, &v->L);
    if (rc) return rc;
    const larql::Layout& L = v->L;
    v->rank = shard_rank;
    v->count = shard_count;
    v->per = (L.features_max + shard_count - 1) / shard_count;
    const size_t dp = (L.hidden + 63) / 64 * 64;
    v->cols = L.gate_bits == 32 ? 2 * dp : dp;
    larql::Mapped gm;
    if (!gm.open(L.dir + "/gate_vectors.bin")) return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot map gate_vectors.bin");
    // stage this shard's rows in the walk's layout, then one copy to the device
    std::vector<uint16_t> stage(L.num_layers * v->per * v->cols, 0);
    v->rows_here.assign(L.num_layers, 0);
    bool too_large = false;
    for (size_t l = 0; l < L.num_layers; ++l) {
        const larql::LayerInfo& li = L.layers[l];
        const size_t r0 = std::min(li.features, shard_rank * v->per), r1 = std::min(li.features, r0 + v->per);
        v->rows_here[l] = r1 - r0;
        for (size_t r = r0; r < r1; ++r) {
            uint16_t* dst = stage.data() + (l * v->per + (r - r0)) * v->cols;
            if (L.gate_bits == 16) {
                memcpy(dst, gm.data + li.offset + r * L.hidden * 2, L.hidden * 2);
            } else {
                const float* src = reinterpret_cast<const float*>(gm.data + li.offset + r * L.hidden * 4);
                for (size_t k = 0; k < L.hidden; ++k) {
                    const float g = src[k];
                    if (!(std::fabs(g) < 32768.0f)) too_large = true;  // also NaN
                    const __half hi = __float2half_rn(g);
                    const float lo = (g - __half2float(hi)) * 4096.0f;
                    dst[k] = __half_as_ushort(hi);
                    dst[dp + k] = __half_as_ushort(__float2half_rn(lo));
                }
            }
        }
    }
    if (too_large)
        return fail(LARQL_ERR_UNSUPPORTED, "vindex: f32 gate values must be finite and below 32768 in magnitude");
    rc = ctx->impl.add_weight(stage.data(), false, stage.size() * 2, nullptr, false,
                              L.gate_bits == 16 ? LARQL_FMT_F16_HALFRS : LARQL_FMT_F16, L.num_layers * v->per, v->cols,
                              &v->gate);
    if (rc) return rc;
    // the staging buffer goes away: take the weight out of the (pointer, length) registry
    for (auto it = ctx->impl.by_ptr.begin(); it != ctx->impl.by_ptr.end();)
        it = it->second == v->gate ? ctx->impl.by_ptr.erase(it) : std::next(it);
    if (L.gate_q4) {  // this shard's Q4_0 rows of every layer, zero blocks after a short layer's end
        larql::Mapped qm;
        if (!qm.open(L.dir + "/gate_vectors_q4.bin")) {
            release_all(v.get());
            return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot map gate_vectors_q4.bin");
        }
        const size_t rb = L.hidden / 32 * 18;
        std::vector<uint8_t> q4(L.num_layers * v->per * rb, 0);
        size_t off = 0;
        for (size_t l = 0; l < L.num_layers; ++l) {
            const size_t f = L.layers[l].features;
            const size_t r0 = std::min(f, shard_rank * v->per), r1 = std::min(f, r0 + v->per);
            memcpy(q4.data() + l * v->per * rb, qm.data + off + r0 * rb, (r1 - r0) * rb);
            off += f * rb;
        }
        rc = ctx->impl.add_weight(q4.data(), false, q4.size(), nullptr, false, LARQL_FMT_Q4_0, L.num_layers * v->per,
                                  L.hidden, &v->gate_q4);
        if (rc) {
            release_all(v.get());
            return rc;
        }
        for (auto it = ctx->impl.by_ptr.begin(); it != ctx->impl.by_ptr.end();)
            it = it->second == v->gate_q4 ? ctx->impl.by_ptr.erase(it) : std::next(it);
    }
    if (L.ffn) {
        v->ffn_map = std::make_unique<larql::Mapped>();
        if (!v->ffn_map->open(L.dir + "/interleaved_q4k.bin")) {
            release_all(v.get());
            return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot map interleaved_q4k.bin");
        }
        v->ffn.assign(L.num_layers, {0, 0, 0});
    }
    if (L.attn) {
        v->attn_map = std::make_unique<larql::Mapped>();
        if (!v->attn_map->open(L.dir + "/attn_weights_q4k.bin")) {
            release_all(v.get());
            return fail(LARQL_ERR_INVALID_ARG, "vindex: cannot map attn_weights_q4k.bin");
        }
        v->attn.assign(L.num_layers, {0, 0, 0, 0});
    }
    *out = v.release();
    return LARQL_OK;
}

int larql_cuda_vindex_info_get(const larql_cuda_vindex* v, larql_cuda_vindex_info* info) {
    if (!v || !info) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    larql::fill_info(v->L, v->rank, v->count, v->per, info);
    return LARQL_OK;
}

int larql_cuda_vindex_gate_knn_dev(larql_cuda_vindex* v, const float* queries_dev, size_t batch, size_t top_k,
                                   uint32_t* out_idx_dev, float* out_score_dev, void* stream) {
    if (!v) return fail(LARQL_ERR_INVALID_ARG, "null vindex");
    LARQL_CTX_GUARD(v->ctx);
    if (!queries_dev || !out_idx_dev || !out_score_dev) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : v->ctx->impl.stream;
    return walk_dev(v, queries_dev, batch, top_k, out_idx_dev, out_score_dev, s);
}

}  // extern "C"

namespace {

// The host-buffer walk over the f16 / f32 gate rows or (q4) the Q4_0 ones; indices made global, empty slots set.
int knn_host(larql_cuda_vindex* v, const float* queries, size_t batch, size_t top_k, uint32_t* out_idx,
             float* out_score, bool q4) {
    if (!queries || !out_idx || !out_score) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    if (batch == 0 || top_k == 0) return LARQL_OK;
    larql::Ctx& c = v->ctx->impl;
    if (q4 && !v->gate_q4) return fail(LARQL_ERR_UNSUPPORTED, "vindex: no gate_vectors_q4.bin");
    const size_t nl = v->L.num_layers, nout = nl * batch * top_k;
    int rc = c.ensure_io(batch * v->L.hidden, 2 * nout);
    if (rc) return rc;
    uint32_t* di = reinterpret_cast<uint32_t*>(c.y_dev);
    float* ds = c.y_dev + nout;
    cudaError_t e = cudaMemcpyAsync(c.x_dev, queries, batch * v->L.hidden * sizeof(float), cudaMemcpyHostToDevice,
                                    c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "query upload");
    rc = q4 ? c.gate_topk_q4_dev(c.find(v->gate_q4), v->L.num_layers, v->per, c.x_dev, batch, top_k, di, ds, c.stream)
            : walk_dev(v, c.x_dev, batch, top_k, di, ds, c.stream);
    if (rc) return rc;
    e = cudaMemcpyAsync(out_idx, di, nout * sizeof(uint32_t), cudaMemcpyDeviceToHost, c.stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out_score, ds, nout * sizeof(float), cudaMemcpyDeviceToHost, c.stream);
    if (e != cudaSuccess) return cuda_fail(e, "top-k download");
    rc = c.finish();
    if (rc) return rc;
    // slots past a layer's rows on this shard are empty; the rest get the shard's first row added
    const uint32_t row0 = static_cast<uint32_t>(v->rank * v->per);
    for (size_t l = 0; l < nl; ++l)
        for (size_t i = 0; i < batch * top_k; ++i) {
            const size_t o = l * batch * top_k + i;
            if (out_idx[o] == 0xFFFFFFFFu || out_idx[o] >= v->rows_here[l]) {
                out_idx[o] = 0xFFFFFFFFu;
                out_score[o] = 0.f;
            } else {
                out_idx[o] += row0;
            }
        }
    return LARQL_OK;
}

}  // namespace

extern "C" {

int larql_cuda_vindex_gate_knn(larql_cuda_vindex* v, const float* queries, size_t batch, size_t top_k,
                               uint32_t* out_idx, float* out_score) {
    if (!v) return fail(LARQL_ERR_INVALID_ARG, "null vindex");
    LARQL_CTX_GUARD(v->ctx);
    return knn_host(v, queries, batch, top_k, out_idx, out_score, false);
}

int larql_cuda_vindex_gate_knn_q4(larql_cuda_vindex* v, const float* queries, size_t batch, size_t top_k,
                                  uint32_t* out_idx, float* out_score) {
    if (!v) return fail(LARQL_ERR_INVALID_ARG, "null vindex");
    LARQL_CTX_GUARD(v->ctx);
    return knn_host(v, queries, batch, top_k, out_idx, out_score, true);
}

int larql_cuda_vindex_ffn(larql_cuda_vindex* v, size_t layer, uint64_t* gate, uint64_t* up, uint64_t* down,
                          int* down_format) {
    if (!v) return fail(LARQL_ERR_INVALID_ARG, "null vindex");
    LARQL_CTX_GUARD(v->ctx);
    if (!gate || !up || !down) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    const larql::Layout& L = v->L;
    if (!L.ffn) return fail(LARQL_ERR_UNSUPPORTED, "vindex: no interleaved_q4k.bin");
    if (layer >= L.num_layers) return fail(LARQL_ERR_BAD_SHAPE, "vindex: layer %zu of %zu", layer, L.num_layers);
    if (L.hidden % 256 || L.inter % 256)
        return fail(LARQL_ERR_UNSUPPORTED, "vindex: FFN matrices need hidden and intermediate multiples of 256");
    auto& h = v->ffn[layer];
    const int dfmt = L.ffn == 2 ? LARQL_FMT_Q6_K : LARQL_FMT_Q4_K;
    if (!h[0]) {
        const uint8_t* base = v->ffn_map->data + layer * (2 * L.ffn_q4k_bytes + L.ffn_down_bytes);
        uint64_t g = 0, u = 0, d = 0;
        int rc = place_rows(v, base, LARQL_FMT_Q4_K, L.inter, L.hidden, &g);
        if (!rc) rc = place_rows(v, base + L.ffn_q4k_bytes, LARQL_FMT_Q4_K, L.inter, L.hidden, &u);
        if (!rc) rc = place_rows(v, base + 2 * L.ffn_q4k_bytes, dfmt, L.hidden, L.inter, &d);
        if (rc) {
            for (uint64_t x : {g, u, d}) drop(v->ctx->impl, x);
            return rc;
        }
        h = {g, u, d};
    }
    *gate = h[0];
    *up = h[1];
    *down = h[2];
    if (down_format) *down_format = dfmt;
    return LARQL_OK;
}

int larql_cuda_vindex_attn(larql_cuda_vindex* v, size_t layer, uint64_t handles[4], int formats[4]) {
    if (!v) return fail(LARQL_ERR_INVALID_ARG, "null vindex");
    LARQL_CTX_GUARD(v->ctx);
    if (!handles || !formats) return fail(LARQL_ERR_INVALID_ARG, "null argument");
    const larql::Layout& L = v->L;
    if (!L.attn) return fail(LARQL_ERR_UNSUPPORTED, "vindex: no attn_weights_q4k.bin with a manifest for every layer");
    if (layer >= L.num_layers) return fail(LARQL_ERR_BAD_SHAPE, "vindex: layer %zu of %zu", layer, L.num_layers);
    auto& h = v->attn[layer];
    for (int i = 0; i < 4; ++i) {
        const larql::AttnEntry& a = L.attn_entries[layer * 4 + i];
        if (!h[i]) {
            int rc = place_rows(v, v->attn_map->data + a.offset, a.format, a.rows, a.cols, &h[i]);
            if (rc) return rc;
        }
        handles[i] = h[i];
        formats[i] = a.format;
    }
    return LARQL_OK;
}

int larql_cuda_vindex_close(larql_cuda_vindex* v) {
    if (!v) return LARQL_OK;
    {
        std::lock_guard<std::recursive_mutex> lk(v->ctx->impl.mu);
        cudaSetDevice(v->ctx->impl.device);
        release_all(v);
    }
    delete v;
    return LARQL_OK;
}

}  // extern "C"
