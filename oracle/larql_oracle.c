/*
 * larql_oracle.c — CPU restatement of the LARQL reference algorithms on the
 * quantized-matvec / gate-walk path.  TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
 * load this library.  The product (the CUDA backend) never links or calls it.
 *
 * Every function names the reference file:line it restates (paths relative
 * to the larql-main workspace, `crates/` = larql-main/crates/).  Arithmetic
 * follows the Rust semantics exactly:
 *   - f32::round()      = round half away from zero  (C roundf)
 *   - `x as u8/i8/i32`  = truncate toward zero, saturate, NaN -> 0
 *   - f32::max / f32::min ignore NaN (C fmaxf / fminf)
 *   - no fused multiply-add (built with -ffp-contract=off), so every
 *     `a * b + c` rounds twice, as rustc emits it.
 * Accumulation order matches the reference loops where the reference is
 * sequential (q4k_matvec, q6k_matvec, q8_matvec, q4_0_matvec scalar path).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ───────────────────────── Rust numeric casts ───────────────────────── */

static inline int32_t rs_as_i32(float v) {
    if (v != v) return 0;
    if (v >= 2147483647.0f) return INT32_MAX;
    if (v <= -2147483648.0f) return INT32_MIN;
    return (int32_t)v;
}
static inline uint8_t rs_as_u8(float v) {
    if (v != v || v <= 0.0f) return 0;
    if (v >= 255.0f) return 255;
    return (uint8_t)v;
}
static inline int8_t rs_as_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}
/* f32::clamp: NaN passes through unchanged. */
static inline float rs_clamp(float v, float lo, float hi) {
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* ───────────────────────── f16 conversions ───────────────────────── */

/* crates/larql-models/src/quant/half.rs:4-20.  NOTE: for subnormal inputs
 * this decoder returns HALF the IEEE value (its exponent is one too small:
 * 127-15+1-e with e counting from 1); normals, zeros, inf and NaN are exact.
 * The reference uses it for f16 gate vectors (vindex gate.rs:91,287,762 via
 * half::decode_f16) and in the ggml dequantizers (quant/ggml.rs:99,143). */
EXPORT float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)(h >> 15)) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    if (exp == 0) {
        if (mant == 0) return bits_f32(sign);
        uint32_t e = 1, m = mant;
        while ((m & 0x400) == 0) { m <<= 1; e += 1; }
        return bits_f32(sign | ((127 - 15 + 1 - e) << 23) | ((m & 0x3FF) << 13));
    }
    if (exp == 31) return bits_f32(sign | (0xFFu << 23) | (mant << 13));
    return bits_f32(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

/* Exact IEEE half -> float: the decoders of q4k_matvec.rs:10-26,
 * q6k_matvec.rs:10-26, q4_common.rs:426-442 and csrc/q4_dot.c:9-35 (all
 * handle subnormals correctly). */
EXPORT float orc_f16_to_f32_ieee(uint16_t h) {
    uint32_t sign = ((uint32_t)(h >> 15)) << 31;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    if (exp == 0) {
        float v = (float)mant / 1024.0f * 0x1p-14f;
        return sign ? -v : v;
    }
    if (exp == 31) return bits_f32(sign | (0xFFu << 23) | (mant << 13));
    return bits_f32(sign | ((exp + 127 - 15) << 23) | (mant << 13));
}

/* crates/larql-compute/src/cpu/ops/q4_common.rs:83-94 — TRUNCATING f32->f16
 * (mantissa >> 13, no rounding; exponents below the f16 normal range flush to
 * signed zero).  Also the inline conversion of q4_common.rs:59-71. */
EXPORT uint16_t orc_f32_to_f16_trunc(float val) {
    uint32_t bits = f32_bits(val);
    uint32_t sign = (bits >> 16) & 0x8000;
    int32_t exp = (int32_t)((bits >> 23) & 0xFF);
    uint32_t mant = bits & 0x7FFFFF;
    if (exp == 0) return (uint16_t)sign;
    if (exp == 255) return (uint16_t)(sign | 0x7C00 | (mant >> 13));
    int32_t new_exp = exp - 127 + 15;
    if (new_exp >= 31) return (uint16_t)(sign | 0x7C00);
    if (new_exp <= 0) return (uint16_t)sign;
    return (uint16_t)(sign | ((uint32_t)new_exp << 10) | (mant >> 13));
}

/* crates/larql-models/src/quant/half.rs:28-41 — the larql-models variant
 * (identical to the above for finite inputs; NaN keeps a quiet-bit payload). */
EXPORT uint16_t orc_f32_to_f16_models(float value) {
    uint32_t bits = f32_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t exp = (int32_t)((bits >> 23) & 0xFF);
    uint32_t mant = bits & 0x007FFFFF;
    if (exp == 255) return (uint16_t)(sign | 0x7C00 | (mant != 0 ? 0x0200 : 0));
    int32_t exp16 = exp - 127 + 15;
    if (exp16 >= 31) return (uint16_t)(sign | 0x7C00);
    if (exp16 <= 0) return sign;
    return (uint16_t)(sign | ((uint16_t)exp16 << 10) | (uint16_t)(mant >> 13));
}

/* crates/larql-models/src/quant/half.rs:49-53 */
EXPORT void orc_decode_f16(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = orc_f16_to_f32(src[i]);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ───────────────────────── quantizers ───────────────────────── */

/* crates/larql-compute/src/cpu/ops/q4_common.rs:28-44 — x -> int8 + f32 scale
 * per 32 values (amax/127, round, clamp). */
EXPORT void orc_quantize_to_q8(const float* x, size_t n, int8_t* q8, float* scales) {
    size_t nb = n / 32;
    for (size_t b = 0; b < nb; b++) {
        const float* blk = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(blk[j]));
        float scale = amax / 127.0f;
        scales[b] = scale;
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        for (int j = 0; j < 32; j++)
            q8[b * 32 + j] = rs_as_i8(rs_clamp(roundf(blk[j] * inv), -128.0f, 127.0f));
    }
}

/* crates/larql-compute/src/cpu/ops/q4_common.rs:50-80 and the identical
 * crates/larql-models/src/quant/ggml.rs:310-337 — Q4_0, 18 B per 32 values:
 * f16 scale = amax/7 (truncating f16), nibble = round(v/scale)+8 in [0,15],
 * byte j = elem 2j | elem 2j+1 << 4. */
EXPORT void orc_quantize_q4_0(const float* data, size_t n, uint8_t* out) {
    size_t nb = n / 32;
    for (size_t i = 0; i < nb; i++) {
        const float* blk = data + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(blk[j]));
        float scale = amax / 7.0f;
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        uint16_t h = orc_f32_to_f16_trunc(scale);
        uint8_t* o = out + i * 18;
        o[0] = (uint8_t)(h & 0xFF);
        o[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 16; j++) {
            int32_t lo = rs_as_i32(roundf(blk[2 * j] * inv)) + 8;
            int32_t hi = rs_as_i32(roundf(blk[2 * j + 1] * inv)) + 8;
            lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
            hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
            o[2 + j] = (uint8_t)(lo | (hi << 4));
        }
    }
}

/* crates/larql-models/src/quant/ggml.rs:342-363 — GGUF Q8_0, 34 B per 32:
 * f16 scale = amax/127 (truncating, half.rs:28), int8 = round(v/scale). */
EXPORT void orc_quantize_q8_0(const float* data, size_t n, uint8_t* out) {
    size_t nb = n / 32;
    for (size_t i = 0; i < nb; i++) {
        const float* blk = data + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(blk[j]));
        float scale = amax / 127.0f;
        float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        uint16_t h = orc_f32_to_f16_models(scale);
        uint8_t* o = out + i * 34;
        o[0] = (uint8_t)(h & 0xFF);
        o[1] = (uint8_t)(h >> 8);
        for (int j = 0; j < 32; j++)
            o[2 + j] = (uint8_t)rs_as_i8(rs_clamp(roundf(blk[j] * inv), -128.0f, 127.0f));
    }
}

/* crates/larql-compute/src/cpu/ops/q8_matvec.rs:11-34 — compute-layout Q8:
 * int8 [rows*hidden] + f32 scale per 32 values. */
EXPORT void orc_quantize_weights_q8(const float* w, size_t rows, size_t hidden,
                                    int8_t* q8, float* scales) {
    size_t bpr = hidden / 32;
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < bpr; b++) {
            size_t off = r * hidden + b * 32;
            float amax = 0.0f;
            for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(w[off + j]));
            float scale = amax / 127.0f;
            float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
            scales[r * bpr + b] = scale;
            for (int j = 0; j < 32; j++)
                q8[off + j] = rs_as_i8(rs_clamp(roundf(w[off + j] * inv), -128.0f, 127.0f));
        }
}

/* crates/larql-compute/src/cpu/ops/q4_common.rs:104-170 — LARQL Q4_K, 148 B
 * per 256 values:
 *   [0..2) f16 d = max sub-block range / 63   (truncating f16)
 *   [2..4) f16 dmin = -min / 15               (truncating f16)
 *   [4..12) 8 x 6-bit scales, [12..16) zero
 *   [16..20) 8 x 4-bit mins (j<4 low nibble of byte j, j>=4 high nibble of j-4)
 *   [20..148) nibbles, byte i of sub-block j = elem 2i | elem 2i+1 << 4.
 * The nibble step uses the f32 d/dmin (not the f16-rounded ones) and is the
 * whole sub-block range, as in the reference. */
EXPORT void orc_quantize_q4_k(const float* data, size_t n, uint8_t* out) {
    size_t nsb = n / 256;
    for (size_t sb = 0; sb < nsb; sb++) {
        const float* blk = data + sb * 256;
        uint8_t* o = out + sb * 148;
        float smin[8], smax[8];
        for (int j = 0; j < 8; j++) {
            float mn = INFINITY, mx = -INFINITY;
            for (int i = 0; i < 32; i++) {
                mn = fminf(mn, blk[j * 32 + i]);
                mx = fmaxf(mx, blk[j * 32 + i]);
            }
            smin[j] = mn;
            smax[j] = mx;
        }
        float gmr = 0.0f, gmin = INFINITY;
        for (int j = 0; j < 8; j++) gmr = fmaxf(gmr, smax[j] - smin[j]);
        for (int j = 0; j < 8; j++) gmin = fminf(gmin, smin[j]);
        float d = gmr > 0.0f ? gmr / 63.0f : 0.0f;
        float dmin = gmin < 0.0f ? -gmin / 15.0f : 0.0f;
        uint16_t hd = orc_f32_to_f16_trunc(d), hm = orc_f32_to_f16_trunc(dmin);
        o[0] = (uint8_t)(hd & 0xFF); o[1] = (uint8_t)(hd >> 8);
        o[2] = (uint8_t)(hm & 0xFF); o[3] = (uint8_t)(hm >> 8);
        uint8_t qs[8], qm[8];
        for (int j = 0; j < 8; j++) {
            float range = smax[j] - smin[j];
            qs[j] = d > 0.0f ? rs_as_u8(rs_clamp(roundf(range / d), 0.0f, 63.0f)) : 0;
            qm[j] = dmin > 0.0f ? rs_as_u8(rs_clamp(roundf(-smin[j] / dmin), 0.0f, 15.0f)) : 0;
        }
        memset(o + 4, 0, 12);
        for (int j = 0; j < 8; j++) o[4 + j] = qs[j] & 0x3F;
        for (int j = 0; j < 4; j++) o[16 + j] = (uint8_t)((qm[j] & 0x0F) | ((qm[j + 4] & 0x0F) << 4));
        for (int j = 0; j < 8; j++) {
            float sc = d * (float)qs[j];
            float mn = dmin * (float)qm[j];
            float inv = sc > 0.0f ? 1.0f / sc : 0.0f;
            const float* sub = blk + j * 32;
            for (int i = 0; i < 16; i++) {
                uint8_t v0 = rs_as_u8(rs_clamp(roundf((sub[2 * i] + mn) * inv), 0.0f, 15.0f));
                uint8_t v1 = rs_as_u8(rs_clamp(roundf((sub[2 * i + 1] + mn) * inv), 0.0f, 15.0f));
                o[20 + j * 16 + i] = (uint8_t)(v0 | (v1 << 4));
            }
        }
    }
}

/* crates/larql-compute/src/cpu/ops/q4_common.rs:179-239 — Q6_K, 210 B per 256:
 * [0..128) low nibbles (sequential pairs), [128..192) high 2 bits (4 per byte,
 * element i at bits 2*(i%4) of byte i/4), [192..208) int8 scales per 16,
 * [208..210) f16 d = amax/32 (truncating). */
EXPORT void orc_quantize_q6_k(const float* data, size_t n, uint8_t* out) {
    size_t nsb = n / 256;
    for (size_t sb = 0; sb < nsb; sb++) {
        const float* blk = data + sb * 256;
        uint8_t* o = out + sb * 210;
        float amax = 0.0f;
        for (int i = 0; i < 256; i++) amax = fmaxf(amax, fabsf(blk[i]));
        float d = amax / 32.0f;
        int8_t ss[16];
        for (int j = 0; j < 16; j++) {
            float smax = 0.0f;
            for (int i = 0; i < 16; i++) smax = fmaxf(smax, fabsf(blk[j * 16 + i]));
            float sc = d > 0.0f ? smax / d : 0.0f;
            ss[j] = rs_as_i8(rs_clamp(roundf(sc), -128.0f, 127.0f));
        }
        uint8_t q6[256];
        for (int j = 0; j < 16; j++) {
            float sc = d * (float)ss[j];
            float inv = fabsf(sc) > 1e-10f ? 1.0f / sc : 0.0f;
            for (int i = 0; i < 16; i++) {
                int8_t q = rs_as_i8(rs_clamp(roundf(blk[j * 16 + i] * inv), -32.0f, 31.0f));
                q6[j * 16 + i] = (uint8_t)(q + 32);
            }
        }
        for (int i = 0; i < 128; i++) o[i] = (uint8_t)((q6[2 * i] & 0x0F) | ((q6[2 * i + 1] & 0x0F) << 4));
        memset(o + 128, 0, 64);
        for (int i = 0; i < 256; i++) o[128 + i / 4] |= (uint8_t)(((q6[i] >> 4) & 0x03) << ((i % 4) * 2));
        for (int j = 0; j < 16; j++) o[192 + j] = (uint8_t)ss[j];
        uint16_t hd = orc_f32_to_f16_trunc(d);
        o[208] = (uint8_t)(hd & 0xFF); o[209] = (uint8_t)(hd >> 8);
    }
}

/* ───────────────────────── dequantizers ───────────────────────── */

/* crates/larql-models/src/quant/ggml.rs:92-110 */
EXPORT void orc_dequantize_q4_0(const uint8_t* data, size_t n, float* out) {
    size_t nb = n / 32;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t* b = data + i * 18;
        float scale = orc_f16_to_f32(rd16(b));
        for (int j = 0; j < 16; j++) {
            int lo = (b[2 + j] & 0x0F) - 8, hi = ((b[2 + j] >> 4) & 0x0F) - 8;
            out[i * 32 + 2 * j] = (float)lo * scale;
            out[i * 32 + 2 * j + 1] = (float)hi * scale;
        }
    }
}

/* crates/larql-models/src/quant/ggml.rs:136-151 */
EXPORT void orc_dequantize_q8_0(const uint8_t* data, size_t n, float* out) {
    size_t nb = n / 32;
    for (size_t i = 0; i < nb; i++) {
        const uint8_t* b = data + i * 34;
        float scale = orc_f16_to_f32(rd16(b));
        for (int j = 0; j < 32; j++) out[i * 32 + j] = (float)(int8_t)b[2 + j] * scale;
    }
}

/* Dequantize one LARQL Q4_K (148 B) super-block stream to f32, element order
 * as consumed by crates/larql-compute/src/cpu/ops/q4k_matvec.rs:54-81
 * (value = d*sc_j*q - dmin*mn_j). */
EXPORT void orc_dequantize_q4_k(const uint8_t* data, size_t n, float* out) {
    size_t nsb = n / 256;
    for (size_t sb = 0; sb < nsb; sb++) {
        const uint8_t* b = data + sb * 148;
        float d = orc_f16_to_f32_ieee(rd16(b)), dmin = orc_f16_to_f32_ieee(rd16(b + 2));
        for (int j = 0; j < 8; j++) {
            float sc = d * (float)(b[4 + j] & 0x3F);
            float mn = dmin * (float)(j < 4 ? (b[16 + j] & 0x0F) : ((b[16 + j - 4] >> 4) & 0x0F));
            for (int i = 0; i < 16; i++) {
                uint8_t q = b[20 + j * 16 + i];
                out[sb * 256 + j * 32 + 2 * i] = sc * (float)(q & 0x0F) - mn;
                out[sb * 256 + j * 32 + 2 * i + 1] = sc * (float)((q >> 4) & 0x0F) - mn;
            }
        }
    }
}

/* crates/larql-models/src/quant/ggml.rs:228-273 (dequantize_q4_k, 144-byte GGUF super-blocks, the decoder the
 * GGUF loader applies, crates/larql-models/src/loading/gguf.rs:191): d, dmin by half.rs (:236-237); 6-bit
 * scales and mins from bytes 4..15 as llama.cpp's get_scale_min_k4 (:243-252); sub-block j's 16 bytes at
 * 16 + 16 j give its 16 low nibbles, then its 16 high nibbles (:255-270); value = d*sc*q - dmin*mn. */
EXPORT void orc_dequantize_q4_k_gguf(const uint8_t* data, size_t n, float* out) {
    size_t nsb = n / 256;
    for (size_t sb = 0; sb < nsb; sb++) {
        const uint8_t* b = data + sb * 144;
        const float d = orc_f16_to_f32(rd16(b)), dmin = orc_f16_to_f32(rd16(b + 2));
        const uint8_t* s = b + 4;
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            if (j < 4) {
                sc[j] = s[j] & 0x3F;
                mn[j] = s[j + 4] & 0x3F;
            } else {
                sc[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
                mn[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
            }
        }
        const uint8_t* q = b + 16;
        float* o = out + sb * 256;
        for (int j = 0; j < 8; j++) {
            const float sv = d * (float)sc[j], mv = dmin * (float)mn[j];
            for (int i = 0; i < 16; i++) o[32 * j + i] = sv * (float)(q[16 * j + i] & 0x0F) - mv;
            for (int i = 0; i < 16; i++) o[32 * j + 16 + i] = sv * (float)((q[16 * j + i] >> 4) & 0x0F) - mv;
        }
    }
}

/* GGUF-144 Q4_K x f32: the dequantized row (orc_dequantize_q4_k_gguf) dotted with x, sequential f32. */
EXPORT void orc_q4k_gguf_matvec_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    float* row = (float*)malloc(sizeof(float) * (hidden ? hidden : 1));
    const size_t bpr = hidden / 256 * 144;
    for (size_t r = 0; r < rows; r++) {
        orc_dequantize_q4_k_gguf(w + r * bpr, hidden, row);
        float acc = 0.0f;
        for (size_t k = 0; k < hidden; k++) acc += row[k] * x[k];
        y[r] = acc;
    }
    free(row);
}

/* GGUF-144 Q4_K in llama.cpp's layout, as the reference's Metal q4kf kernels read it
 * (crates/larql-compute/src/metal/shaders/q4kf_qkv_proj.rs:136-220, llama.cpp's mul_mv_q4_K): d, dmin IEEE f16
 * (Metal half); scales / mins as get_scale_min_k4 (as ggml.rs); the 128 quant bytes are four 32-byte chunks,
 * chunk c holding sub-block 2c in its low nibbles and 2c + 1 in its high ones, element e of a sub-block at byte e. */
EXPORT void orc_dequantize_q4_k_gguf_llama(const uint8_t* data, size_t n, float* out) {
    size_t nsb = n / 256;
    for (size_t sb = 0; sb < nsb; sb++) {
        const uint8_t* b = data + sb * 144;
        const float d = orc_f16_to_f32_ieee(rd16(b)), dmin = orc_f16_to_f32_ieee(rd16(b + 2));
        const uint8_t* s = b + 4;
        float* o = out + sb * 256;
        for (int j = 0; j < 8; j++) {
            uint8_t sc, mn;
            if (j < 4) {
                sc = s[j] & 0x3F;
                mn = s[j + 4] & 0x3F;
            } else {
                sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
                mn = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
            }
            const float sv = d * (float)sc, mv = dmin * (float)mn;
            const uint8_t* q = b + 16 + 32 * (j / 2);
            const int sh = 4 * (j & 1);
            for (int e = 0; e < 32; e++) o[32 * j + e] = sv * (float)((q[e] >> sh) & 0x0F) - mv;
        }
    }
}

/* The llama.cpp-layout row (orc_dequantize_q4_k_gguf_llama) dotted with x, sequential f32. */
EXPORT void orc_q4k_gguf_llama_matvec_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    float* row = (float*)malloc(sizeof(float) * (hidden ? hidden : 1));
    const size_t bpr = hidden / 256 * 144;
    for (size_t r = 0; r < rows; r++) {
        orc_dequantize_q4_k_gguf_llama(w + r * bpr, hidden, row);
        float acc = 0.0f;
        for (size_t k = 0; k < hidden; k++) acc += row[k] * x[k];
        y[r] = acc;
    }
    free(row);
}

/* ───────────────────────── matvecs ───────────────────────── */

/* crates/larql-compute/src/cpu/ops/q4k_matvec.rs:31-87 — rows [r0, r1). */
static void q4k_rows(const uint8_t* w, const float* x, float* y, size_t r0, size_t r1, size_t hidden) {
    size_t nsb = hidden / 256, bpr = nsb * 148;
    for (size_t row = r0; row < r1; row++) {
        const uint8_t* rp = w + row * bpr;
        float acc = 0.0f;
        for (size_t sb = 0; sb < nsb; sb++) {
            const uint8_t* b = rp + sb * 148;
            float d = orc_f16_to_f32_ieee(rd16(b)), dmin = orc_f16_to_f32_ieee(rd16(b + 2));
            float scales[8], mins[8];
            for (int j = 0; j < 4; j++) {
                scales[j] = (float)(b[4 + j] & 0x3F);
                scales[j + 4] = (float)(b[8 + j] & 0x3F);
                mins[j] = (float)(b[16 + j] & 0x0F);
                mins[j + 4] = (float)((b[16 + j] >> 4) & 0x0F);
            }
            const uint8_t* qs = b + 20;
            size_t xb = sb * 256;
            for (int j = 0; j < 8; j++) {
                float sc = d * scales[j], mn = dmin * mins[j];
                for (int i = 0; i < 16; i++) {
                    size_t xi = xb + j * 32 + i * 2;
                    uint8_t q = qs[j * 16 + i];
                    float lo = (float)(q & 0x0F), hi = (float)((q >> 4) & 0x0F);
                    acc += (sc * lo - mn) * x[xi];
                    acc += (sc * hi - mn) * x[xi + 1];
                }
            }
        }
        y[row] = acc;
    }
}

EXPORT void orc_q4k_matvec(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    q4k_rows(w, x, y, 0, rows, hidden);
}

/* crates/larql-compute/src/cpu/ops/q6k_matvec.rs:31-87 — rows [r0, r1). */
static void q6k_rows(const uint8_t* w, const float* x, float* y, size_t r0, size_t r1, size_t hidden) {
    size_t nsb = hidden / 256, bpr = nsb * 210;
    for (size_t row = r0; row < r1; row++) {
        float acc = 0.0f;
        for (size_t sb = 0; sb < nsb; sb++) {
            const uint8_t* b = w + row * bpr + sb * 210;
            const uint8_t *ql = b, *qh = b + 128, *sc8 = b + 192;
            float d = orc_f16_to_f32_ieee(rd16(b + 208));
            size_t xb = sb * 256;
            for (int j = 0; j < 16; j++) {
                float sc = d * (float)(int8_t)sc8[j];
                for (int i = 0; i < 8; i++) {
                    int qi = j * 16 + i * 2;
                    uint8_t lb = ql[qi / 2];
                    float lo0 = (float)(lb & 0x0F), lo1 = (float)((lb >> 4) & 0x0F);
                    float h0 = (float)((qh[qi / 4] >> ((qi % 4) * 2)) & 0x03);
                    float h1 = (float)((qh[(qi + 1) / 4] >> (((qi + 1) % 4) * 2)) & 0x03);
                    float v0 = sc * ((lo0 + h0 * 16.0f) - 32.0f);
                    float v1 = sc * ((lo1 + h1 * 16.0f) - 32.0f);
                    acc += v0 * x[xb + qi];
                    acc += v1 * x[xb + qi + 1];
                }
            }
        }
        y[row] = acc;
    }
}

EXPORT void orc_q6k_matvec(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    q6k_rows(w, x, y, 0, rows, hidden);
}

/* crates/larql-compute/csrc/q4_dot.c:169-199 (the x86 scalar q4_0_matvec_c,
 * reached through cpu/ops/q4_matvec.rs:18-31): per element
 * acc += (float)(nib-8) * (float)q8 * (f16 scale * q8 scale). */
static void q4_0_q8_rows(const uint8_t* w, const int8_t* q8, const float* q8s, float* y,
                         size_t r0, size_t r1, size_t hidden) {
    size_t nb = hidden / 32, bpr = nb * 18;
    for (size_t row = r0; row < r1; row++) {
        float acc = 0.0f;
        const uint8_t* rp = w + row * bpr;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* blk = rp + b * 18;
            float cs = orc_f16_to_f32_ieee(rd16(blk)) * q8s[b];
            const int8_t* qp = q8 + b * 32;
            for (int j = 0; j < 16; j++) {
                int lo = (blk[2 + j] & 0x0F) - 8, hi = ((blk[2 + j] >> 4) & 0x0F) - 8;
                acc += (float)lo * (float)qp[2 * j] * cs;
                acc += (float)hi * (float)qp[2 * j + 1] * cs;
            }
        }
        y[row] = acc;
    }
}

EXPORT void orc_q4_0_matvec_q8(const uint8_t* w, const int8_t* q8, const float* q8s, float* y,
                               size_t rows, size_t hidden) {
    q4_0_q8_rows(w, q8, q8s, y, 0, rows, hidden);
}

/* Q4_0 x f32: ggml.rs:92-110 dequantize (half.rs scale decode), then a sequential f32 dot per row
 * (the f32-activation semantics of the Metal q4_f32_matvec shader,
 * crates/larql-compute/src/metal/shaders/q4_f32_matvec.rs:10). */
static void q4_0_f32_rows(const uint8_t* w, const float* x, float* y, size_t r0, size_t r1, size_t hidden) {
    size_t nb = hidden / 32, bpr = nb * 18;
    for (size_t row = r0; row < r1; row++) {
        float acc = 0.0f;
        const uint8_t* rp = w + row * bpr;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* blk = rp + b * 18;
            float scale = orc_f16_to_f32(rd16(blk));
            for (int j = 0; j < 16; j++) {
                int lo = (blk[2 + j] & 0x0F) - 8, hi = ((blk[2 + j] >> 4) & 0x0F) - 8;
                acc += ((float)lo * scale) * x[b * 32 + 2 * j];
                acc += ((float)hi * scale) * x[b * 32 + 2 * j + 1];
            }
        }
        y[row] = acc;
    }
}

EXPORT void orc_q4_0_matvec_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    q4_0_f32_rows(w, x, y, 0, rows, hidden);
}

/* GGUF Q8_0 (34 B) x f32: ggml.rs:136-151 dequantize + sequential f32 dot. */
static void q8_0_f32_rows(const uint8_t* w, const float* x, float* y, size_t r0, size_t r1, size_t hidden) {
    size_t nb = hidden / 32, bpr = nb * 34;
    for (size_t row = r0; row < r1; row++) {
        float acc = 0.0f;
        const uint8_t* rp = w + row * bpr;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* blk = rp + b * 34;
            float scale = orc_f16_to_f32(rd16(blk));
            for (int j = 0; j < 32; j++) acc += ((float)(int8_t)blk[2 + j] * scale) * x[b * 32 + j];
        }
        y[row] = acc;
    }
}

EXPORT void orc_q8_0_matvec_f32(const uint8_t* w, const float* x, float* y, size_t rows, size_t hidden) {
    q8_0_f32_rows(w, x, y, 0, rows, hidden);
}

/* crates/larql-compute/src/cpu/ops/q8_matvec.rs:36-57 — compute-layout Q8
 * weights x Q8(x): int32 block sums, acc += isum * (w_scale * x_scale). */
EXPORT void orc_q8_matvec(const int8_t* wq, const float* ws, const int8_t* xq, const float* xs,
                          float* y, size_t rows, size_t hidden) {
    size_t nb = hidden / 32;
    for (size_t r = 0; r < rows; r++) {
        float acc = 0.0f;
        for (size_t b = 0; b < nb; b++) {
            float cs = ws[r * nb + b] * xs[b];
            int32_t isum = 0;
            for (int j = 0; j < 32; j++) isum += (int32_t)wq[r * hidden + b * 32 + j] * (int32_t)xq[b * 32 + j];
            acc += (float)isum * cs;
        }
        y[r] = acc;
    }
}

/* crates/larql-compute/csrc/q4_dot.c:201-232 — Q4_0 vecmat (scatter):
 * out[hidden] = act[inter] @ Q4[inter, hidden], rows with |act| < 1e-10 skipped. */
EXPORT void orc_q4_0_vecmat(const float* act, const uint8_t* w, float* out, size_t inter, size_t hidden) {
    size_t nb = hidden / 32, bpr = nb * 18;
    for (size_t j = 0; j < hidden; j++) out[j] = 0.0f;
    for (size_t row = 0; row < inter; row++) {
        float a = act[row];
        if (a > -1e-10f && a < 1e-10f) continue;
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* blk = w + row * bpr + b * 18;
            float scale = orc_f16_to_f32_ieee(rd16(blk)) * a;
            float* o = out + b * 32;
            for (int j = 0; j < 16; j++) {
                int lo = (blk[2 + j] & 0x0F) - 8, hi = ((blk[2 + j] >> 4) & 0x0F) - 8;
                o[2 * j] += (float)lo * scale;
                o[2 * j + 1] += (float)hi * scale;
            }
        }
    }
}

/* ───────────────────────── gate walk ───────────────────────── */

/* Scores for the gate walk: crates/larql-vindex/src/index/gate.rs:14-21 (gemv
 * = x[1,D] @ G[N,D]^T via CpuBackend::matmul_transb) on rows decoded from f16
 * (gate.rs:86-94, quant/half.rs:49).  The reference's f32 summation lives in
 * the third-party `matrixmultiply` 0.3 sgemm (order unpinned), so the oracle
 * accumulates in f64 and rounds once to f32. */
EXPORT void orc_gate_scores_f16(const uint16_t* gates, const float* q, float* scores,
                                size_t n_feat, size_t hidden) {
    for (size_t f = 0; f < n_feat; f++) {
        double acc = 0.0;
        const uint16_t* g = gates + f * hidden;
        for (size_t k = 0; k < hidden; k++) acc += (double)orc_f16_to_f32(g[k]) * (double)q[k];
        scores[f] = (float)acc;
    }
}

/* crates/larql-vindex/src/index/gate.rs:307-316 — top-K by |score|
 * descending.  The reference uses an unstable select + sort, so the order of
 * exact ties is unspecified; here ties break by ascending index. */
typedef struct { uint32_t idx; float score; } orc_hit;
static int cmp_hit(const void* a, const void* b) {
    const orc_hit *x = (const orc_hit*)a, *y = (const orc_hit*)b;
    float ax = fabsf(x->score), ay = fabsf(y->score);
    if (ax > ay) return -1;
    if (ax < ay) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}
EXPORT size_t orc_top_k_abs(const float* scores, size_t n, size_t k, uint32_t* idx, float* out_scores) {
    if (k > n) k = n;
    orc_hit* h = (orc_hit*)malloc(sizeof(orc_hit) * (n ? n : 1));
    for (size_t i = 0; i < n; i++) { h[i].idx = (uint32_t)i; h[i].score = scores[i]; }
    qsort(h, n, sizeof(orc_hit), cmp_hit);
    for (size_t i = 0; i < k; i++) { idx[i] = h[i].idx; out_scores[i] = h[i].score; }
    free(h);
    return k;
}

/* crates/larql-vindex/src/index/walk.rs:566-577 (lm_head_knn_backend's selection): k = min(top_k, n); when
 * 0 < k < n the k largest logits are kept (select_nth_unstable_by, descending), then sorted descending.  With
 * top_k == 0 or top_k >= n nothing is dropped, so every logit comes back sorted.  The order of exact ties is
 * unspecified there; here lower ids come first.  A NaN logit makes partial_cmp().unwrap() panic in the
 * reference: here the call returns (size_t)-1 and writes nothing. */
static int cmp_hit_signed(const void* a, const void* b) {
    const orc_hit *x = (const orc_hit*)a, *y = (const orc_hit*)b;
    if (x->score > y->score) return -1;
    if (x->score < y->score) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}
EXPORT size_t orc_top_k_signed(const float* scores, size_t n, size_t top_k, uint32_t* idx, float* out_scores) {
    for (size_t i = 0; i < n; i++)
        if (scores[i] != scores[i]) return (size_t)-1;
    size_t k = top_k < n ? top_k : n;
    if (k == 0) k = n;
    orc_hit* h = (orc_hit*)malloc(sizeof(orc_hit) * (n ? n : 1));
    for (size_t i = 0; i < n; i++) { h[i].idx = (uint32_t)i; h[i].score = scores[i]; }
    qsort(h, n, sizeof(orc_hit), cmp_hit_signed);
    for (size_t i = 0; i < k; i++) { idx[i] = h[i].idx; out_scores[i] = h[i].score; }
    free(h);
    return k;
}

/* The reference's f16 gate KNN as it runs after VectorIndex::warmup() (gate.rs:744-765 decodes each layer to
 * f32 once): scores = G_f32 . q with f32 products summed in f32 (matrixmultiply's sgemm behind
 * crates/larql-tensor/src/sgemm.rs:41-66; eight running partial sums here so the loop vectorises), then the
 * top-k by |score| (gate.rs:307-316) kept in a sorted array.  Timed as the CPU baseline of the gate walk;
 * parity uses orc_gate_scores_f16 (f64). */
#define ORC_GATE_KNN_BODY                                                                         \
    if (k > n_feat) k = n_feat;                                                                    \
    size_t have = 0;                                                                               \
    for (size_t f = 0; f < n_feat; f++) {                                                          \
        const float* r = g + f * hidden;                                                           \
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};                                                     \
        size_t d = 0;                                                                              \
        for (; d + 8 <= hidden; d += 8)                                                            \
            for (int j = 0; j < 8; j++) a[j] += r[d + j] * q[d + j];                               \
        float s = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));               \
        for (; d < hidden; d++) s += r[d] * q[d];                                                  \
        const float m = fabsf(s);                                                                  \
        if (have < k || m > fabsf(sc[have - 1])) {                                                 \
            size_t i = have < k ? have++ : k - 1;                                                  \
            while (i > 0 && m > fabsf(sc[i - 1])) { sc[i] = sc[i - 1]; idx[i] = idx[i - 1]; i--; } \
            sc[i] = s;                                                                             \
            idx[i] = (uint32_t)f;                                                                  \
        }                                                                                          \
    }                                                                                              \
    return have;

static size_t gate_knn_generic(const float* g, const float* q, size_t n_feat, size_t hidden, size_t k,
                               uint32_t* idx, float* sc) {
    ORC_GATE_KNN_BODY
}

/* matrixmultiply selects AVX2 + FMA kernels at run time where the CPU has them; so does this baseline. */
#if defined(__x86_64__)
#pragma GCC push_options
#pragma GCC optimize("O3", "fp-contract=fast")
__attribute__((target("avx2,fma"))) static size_t gate_knn_avx2(const float* g, const float* q, size_t n_feat,
                                                                size_t hidden, size_t k, uint32_t* idx,
                                                                float* sc) {
    ORC_GATE_KNN_BODY
}
#pragma GCC pop_options
#endif

EXPORT size_t orc_gate_knn_f32(const float* g, const float* q, size_t n_feat, size_t hidden, size_t k,
                               uint32_t* idx, float* sc) {
#if defined(__x86_64__)
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"))
        return gate_knn_avx2(g, q, n_feat, hidden, k, idx, sc);
#endif
    return gate_knn_generic(g, q, n_feat, hidden, k, idx, sc);
}

/* ───────────────────────── decode layer (composite) ─────────────────────────
 * The reference's CPU backend has no decode_token (backend.rs:115-124 returns None); this composes the CPU
 * pieces the Metal decode pipeline mirrors, for one Llama-style layer and one token at position `pos`:
 *   h = rms_norm_eps(x, input_norm, offset, eps)           larql-inference/src/residual.rs:17-35
 *   q, k, v = Q4_K matvecs of h                            larql-compute/src/cpu/ops/q4k_matvec.rs:31-87
 *   q, k = RoPE(pos, base), split-half rotation           larql-inference/src/attention/rope.rs:22-55
 *   K[pos], V[pos] = f16(k), f16(v) (round to nearest)    the f16 KV cache of the decode pipeline
 *   a = GQA over keys 0..pos (f32 dots, f64 exp sum)       larql-inference/src/attention/gqa.rs:29-110
 *   x += Q4_K(wo) a
 *   h = rms_norm_eps(x, post_attn_norm, offset, eps)
 *   x += Q4_K(down) (silu(Q4_K(gate) h) * Q4_K(up) h)      larql-inference/src/ffn/mod.rs:87-94
 * The caches are [max_seq][n_kv][head_dim] f16, updated in place at `pos`. */
static uint16_t f32_to_f16_rne(float f) {
    uint32_t x = f32_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  /* rounds to >= 65520 -> inf */
    if (ax < 0x38800000u) {                                      /* below the f16 normal range */
        float v = bits_f32(ax) * 16777216.0f;                    /* exact: scale to units of 2^-24 */
        uint32_t m = (uint32_t)v;
        float r = v - (float)m;
        if (r > 0.5f || (r == 0.5f && (m & 1u))) m++;
        return (uint16_t)(sign | m);
    }
    uint32_t e = (ax >> 23) - 112, mant = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static void rms_norm_row(const float* x, const float* w, float offset, double eps, size_t n, float* out) {
    double sq = 0.0;
    for (size_t j = 0; j < n; j++) sq += (double)x[j] * (double)x[j];
    float rms = (float)sqrt(sq / (double)n + eps);
    for (size_t j = 0; j < n; j++) out[j] = x[j] / rms * (offset + w[j]);
}

static void rope_row(float* v, size_t heads, size_t hd, double base, size_t pos) {
    size_t half = hd / 2;
    for (size_t h = 0; h < heads; h++) {
        float* p = v + h * hd;
        for (size_t i = 0; i < half; i++) {
            double inv = 1.0 / pow(base, 2.0 * (double)i / (double)hd);
            double th = (double)pos * inv;
            float c = (float)cos(th), s = (float)sin(th);
            float x0 = p[i], x1 = p[half + i];
            p[i] = x0 * c - x1 * s;
            p[half + i] = x0 * s + x1 * c;
        }
    }
}

EXPORT void orc_decode_layer(float* x, size_t hidden, size_t inter, size_t nq, size_t nkv, size_t hd,
                             const uint8_t* wq, const uint8_t* wk, const uint8_t* wv, const uint8_t* wo,
                             const uint8_t* wg, const uint8_t* wu, const uint8_t* wd,
                             const float* in_norm, const float* post_norm, float offset, float eps,
                             float attn_scale, double rope_base, uint16_t* kc, uint16_t* vc, size_t pos) {
    size_t qd = nq * hd, kvd = nkv * hd, reps = nq / nkv;
    float* h = (float*)malloc(sizeof(float) * (hidden > inter ? hidden : inter));
    float* q = (float*)malloc(sizeof(float) * qd);
    float* k = (float*)malloc(sizeof(float) * kvd);
    float* v = (float*)malloc(sizeof(float) * kvd);
    float* a = (float*)malloc(sizeof(float) * qd);
    float* o = (float*)malloc(sizeof(float) * hidden);
    float* g = (float*)malloc(sizeof(float) * inter);
    float* u = (float*)malloc(sizeof(float) * inter);
    float* sc = (float*)malloc(sizeof(float) * (pos + 1));
    rms_norm_row(x, in_norm, offset, (double)eps, hidden, h);
    orc_q4k_matvec(wq, h, q, qd, hidden);
    orc_q4k_matvec(wk, h, k, kvd, hidden);
    orc_q4k_matvec(wv, h, v, kvd, hidden);
    rope_row(q, nq, hd, rope_base, pos);
    rope_row(k, nkv, hd, rope_base, pos);
    for (size_t i = 0; i < kvd; i++) {
        kc[pos * kvd + i] = f32_to_f16_rne(k[i]);
        vc[pos * kvd + i] = f32_to_f16_rne(v[i]);
    }
    for (size_t hh = 0; hh < nq; hh++) {
        size_t kh = hh / reps;
        const float* qr = q + hh * hd;
        float mx = -INFINITY;
        for (size_t j = 0; j <= pos; j++) {
            const uint16_t* kr = kc + j * kvd + kh * hd;
            float s = 0.0f;
            for (size_t d = 0; d < hd; d++) s += orc_f16_to_f32_ieee(kr[d]) * qr[d];
            s *= attn_scale;
            sc[j] = s;
            if (s > mx) mx = s;
        }
        double sum = 0.0;
        for (size_t j = 0; j <= pos; j++) {
            double e = exp((double)(sc[j] - mx));
            sc[j] = (float)e;
            sum += e;
        }
        float inv = (float)(1.0 / sum);
        for (size_t j = 0; j <= pos; j++) sc[j] *= inv;
        for (size_t d = 0; d < hd; d++) {
            float acc = 0.0f;
            for (size_t j = 0; j <= pos; j++) acc += orc_f16_to_f32_ieee(vc[j * kvd + kh * hd + d]) * sc[j];
            a[hh * hd + d] = acc;
        }
    }
    orc_q4k_matvec(wo, a, o, hidden, qd);
    for (size_t i = 0; i < hidden; i++) x[i] += o[i];
    rms_norm_row(x, post_norm, offset, (double)eps, hidden, h);
    orc_q4k_matvec(wg, h, g, inter, hidden);
    orc_q4k_matvec(wu, h, u, inter, hidden);
    for (size_t i = 0; i < inter; i++) g[i] = g[i] * (1.0f / (1.0f + expf(-g[i]))) * u[i];
    orc_q4k_matvec(wd, g, o, hidden, inter);
    for (size_t i = 0; i < hidden; i++) x[i] += o[i];
    free(h); free(q); free(k); free(v); free(a); free(o); free(g); free(u); free(sc);
}

EXPORT uint16_t orc_f32_to_f16_rne(float f) { return f32_to_f16_rne(f); }

/* ───────────────────── threaded drivers (CPU baseline) ─────────────────────
 * The reference CPU path is single-threaded.  These split the same per-row
 * functions over contiguous row ranges so a baseline can use every host core;
 * per-row arithmetic is unchanged. */
typedef struct {
    int kind;
    const uint8_t* w; const float* x; const int8_t* q8; const float* q8s;
    float* y; size_t r0, r1, hidden;
} orc_job;

static void* run_job(void* p) {
    orc_job* j = (orc_job*)p;
    switch (j->kind) {
        case 0: q4k_rows(j->w, j->x, j->y, j->r0, j->r1, j->hidden); break;
        case 1: q4_0_q8_rows(j->w, j->q8, j->q8s, j->y, j->r0, j->r1, j->hidden); break;
        case 2: q4_0_f32_rows(j->w, j->x, j->y, j->r0, j->r1, j->hidden); break;
        case 3: q8_0_f32_rows(j->w, j->x, j->y, j->r0, j->r1, j->hidden); break;
        case 4: q6k_rows(j->w, j->x, j->y, j->r0, j->r1, j->hidden); break;
    }
    return NULL;
}

/* kind: 0 q4k(148) x f32, 1 q4_0 x q8, 2 q4_0 x f32, 3 q8_0(34) x f32, 4 q6k x f32. */
EXPORT int orc_matvec_mt(int kind, const uint8_t* w, const float* x, const int8_t* q8, const float* q8s,
                         float* y, size_t rows, size_t hidden, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    int created[256];
    orc_job jobs[256];
    size_t per = (rows + (size_t)nthreads - 1) / (size_t)nthreads;
    for (int t = 0; t < nthreads; t++) {
        created[t] = 0;
        size_t r0 = (size_t)t * per, r1 = r0 + per;
        if (r0 >= rows) continue;
        if (r1 > rows) r1 = rows;
        jobs[t] = (orc_job){kind, w, x, q8, q8s, y, r0, r1, hidden};
        if (nthreads > 1 && pthread_create(&th[t], NULL, run_job, &jobs[t]) == 0) created[t] = 1;
        else run_job(&jobs[t]);
    }
    for (int t = 0; t < nthreads; t++)
        if (created[t]) pthread_join(th[t], NULL);
    return 0;
}
