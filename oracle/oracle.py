"""ctypes binding of the CPU oracle (test infrastructure only).

The oracle is the C restatement in ``larql_oracle.c`` of the reference's CPU
algorithms (each C function cites its reference file:line) plus, when built,
the reference's own ``crates/larql-compute/csrc/q4_dot.c`` compiled unchanged
into ``_ref/libq4dot_ref.so``.  Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py`` import this module, and only as the
checker / the timed CPU baseline.  The CUDA product never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblarql_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libq4dot_ref.so")

_lib = None
_ref = None

u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
sz = C.c_size_t


def build() -> None:
    """Compile the oracle (and, where the reference tree exists, q4_dot.c)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32_ieee.restype = C.c_float
        L.orc_f16_to_f32_ieee.argtypes = [C.c_uint16]
        L.orc_f32_to_f16_trunc.restype = C.c_uint16
        L.orc_f32_to_f16_trunc.argtypes = [C.c_float]
        L.orc_f32_to_f16_models.restype = C.c_uint16
        L.orc_f32_to_f16_models.argtypes = [C.c_float]
        L.orc_decode_f16.argtypes = [u16p, f32p, sz]
        L.orc_quantize_to_q8.argtypes = [f32p, sz, i8p, f32p]
        L.orc_quantize_q4_0.argtypes = [f32p, sz, u8p]
        L.orc_quantize_q8_0.argtypes = [f32p, sz, u8p]
        L.orc_quantize_weights_q8.argtypes = [f32p, sz, sz, i8p, f32p]
        L.orc_quantize_q4_k.argtypes = [f32p, sz, u8p]
        L.orc_quantize_q6_k.argtypes = [f32p, sz, u8p]
        L.orc_dequantize_q4_0.argtypes = [u8p, sz, f32p]
        L.orc_dequantize_q8_0.argtypes = [u8p, sz, f32p]
        L.orc_dequantize_q4_k.argtypes = [u8p, sz, f32p]
        L.orc_dequantize_q4_k_gguf.argtypes = [u8p, sz, f32p]
        L.orc_q4k_gguf_matvec_f32.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_dequantize_q4_k_gguf_llama.argtypes = [u8p, sz, f32p]
        L.orc_q4k_gguf_llama_matvec_f32.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_q4k_matvec.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_q6k_matvec.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_q4_0_matvec_q8.argtypes = [u8p, i8p, f32p, f32p, sz, sz]
        L.orc_q4_0_matvec_f32.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_q8_0_matvec_f32.argtypes = [u8p, f32p, f32p, sz, sz]
        L.orc_q8_matvec.argtypes = [i8p, f32p, i8p, f32p, f32p, sz, sz]
        L.orc_q4_0_vecmat.argtypes = [f32p, u8p, f32p, sz, sz]
        L.orc_gate_scores_f16.argtypes = [u16p, f32p, f32p, sz, sz]
        L.orc_top_k_abs.restype = sz
        L.orc_top_k_abs.argtypes = [f32p, sz, sz, u32p, f32p]
        L.orc_top_k_signed.restype = sz
        L.orc_top_k_signed.argtypes = [f32p, sz, sz, u32p, f32p]
        L.orc_decode_layer.argtypes = [f32p, sz, sz, sz, sz, sz, u8p, u8p, u8p, u8p, u8p, u8p, u8p, f32p, f32p,
                                       C.c_float, C.c_float, C.c_float, C.c_double, u16p, u16p, sz]
        L.orc_f32_to_f16_rne.restype = C.c_uint16
        L.orc_f32_to_f16_rne.argtypes = [C.c_float]
        L.orc_gate_knn_f32.restype = sz
        L.orc_gate_knn_f32.argtypes = [f32p, f32p, sz, sz, sz, u32p, f32p]
        L.orc_matvec_mt.restype = C.c_int
        L.orc_matvec_mt.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, sz, sz, C.c_int]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own q4_dot.c (x86 scalar path), or None if not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        R = C.CDLL(REF_PATH)
        R.q4_0_matvec_c.argtypes = [u8p, i8p, f32p, f32p, sz, sz]
        R.q4_0_vecmat_c.argtypes = [f32p, u8p, f32p, sz, sz]
        _ref = R
    return _ref


METAL_PATH = os.path.join(HERE, "_ref", "libmetal_ref.so")
_metal = None


def metal_ref_lib():
    """The reference's Metal q4k_matvec / q6k_matvec shaders compiled for the CPU (Makefile target `metal`), or
    None if not built."""
    global _metal
    if _metal is None and os.path.exists(METAL_PATH):
        M = C.CDLL(METAL_PATH)
        for fn in (M.metal_q4k_matvec, M.metal_q6k_matvec, M.metal_q4kf_proj):
            fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint, C.c_uint]
            fn.restype = None
        _metal = M
    return _metal


def metal_q4k_matvec(w, x, rows, hidden):
    """crates/larql-compute/src/metal/shaders/q4k_matvec.rs run on the CPU (the reference's own shader code)."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(rows, np.float32)
    metal_ref_lib().metal_q4k_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, hidden)
    return y


def metal_q6k_matvec(w, x, rows, hidden):
    """crates/larql-compute/src/metal/shaders/q6k_matvec.rs run on the CPU (the reference's own shader code)."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(rows, np.float32)
    metal_ref_lib().metal_q6k_matvec(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, hidden)
    return y


def metal_q4kf_proj(w, x, rows, hidden):
    """crates/larql-compute/src/metal/shaders/q4kf_qkv_proj.rs q4kf_proj (GGUF-144 Q4_K as llama.cpp's mul_mv_q4_K
    reads it) run on the CPU."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(rows, np.float32)
    metal_ref_lib().metal_q4kf_proj(w.ctypes.data, x.ctypes.data, y.ctypes.data, rows, hidden)
    return y


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ── f16 ──

def f16_to_f32(bits: int) -> float:
    """larql-models half.rs:4-20 (subnormals come out at half their IEEE value)."""
    return lib().orc_f16_to_f32(bits)


def f16_to_f32_ieee(bits: int) -> float:
    """The exact decoders of q4k_matvec.rs / q6k_matvec.rs / q4_dot.c."""
    return lib().orc_f16_to_f32_ieee(bits)


def f32_to_f16_trunc(v: float) -> int:
    return lib().orc_f32_to_f16_trunc(v)


def decode_f16(bits: np.ndarray) -> np.ndarray:
    """larql-models half.rs:49-53 decode_f16 (the gate-vector decoder)."""
    bits = _c(bits, np.uint16).reshape(-1)
    out = np.empty(bits.size, np.float32)
    lib().orc_decode_f16(bits, out, bits.size)
    return out


# ── quantizers ──

def quantize_to_q8(x: np.ndarray):
    x = _c(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    s = np.empty(x.size // 32, np.float32)
    lib().orc_quantize_to_q8(x, x.size, q, s)
    return q, s


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).reshape(-1)
    assert w.size % 32 == 0
    out = np.empty(w.size // 32 * 18, np.uint8)
    lib().orc_quantize_q4_0(w, w.size, out)
    return out


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).reshape(-1)
    assert w.size % 32 == 0
    out = np.empty(w.size // 32 * 34, np.uint8)
    lib().orc_quantize_q8_0(w, w.size, out)
    return out


def quantize_weights_q8(w: np.ndarray, rows: int, hidden: int):
    w = _c(w, np.float32).reshape(-1)
    q = np.empty(rows * hidden, np.int8)
    s = np.empty(rows * hidden // 32, np.float32)
    lib().orc_quantize_weights_q8(w, rows, hidden, q, s)
    return q, s


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).reshape(-1)
    assert w.size % 256 == 0
    out = np.empty(w.size // 256 * 148, np.uint8)
    lib().orc_quantize_q4_k(w, w.size, out)
    return out


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    w = _c(w, np.float32).reshape(-1)
    assert w.size % 256 == 0
    out = np.empty(w.size // 256 * 210, np.uint8)
    lib().orc_quantize_q6_k(w, w.size, out)
    return out


# ── dequantizers ──

def dequantize_q4_0(data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q4_0(_c(data, np.uint8), n, out)
    return out


def dequantize_q8_0(data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q8_0(_c(data, np.uint8), n, out)
    return out


def dequantize_q4_k(data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q4_k(_c(data, np.uint8), n, out)
    return out


def dequantize_q4_k_gguf(data: np.ndarray, n: int) -> np.ndarray:
    """ggml.rs:228-273: GGUF 144-byte Q4_K super-blocks as the reference's GGUF loader decodes them."""
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q4_k_gguf(_c(data, np.uint8), n, out)
    return out


def dequantize_q4_k_gguf_llama(data: np.ndarray, n: int) -> np.ndarray:
    """GGUF 144-byte Q4_K in llama.cpp's layout, as the reference's Metal q4kf kernels read it."""
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q4_k_gguf_llama(_c(data, np.uint8), n, out)
    return out


# ── matvecs (one row of x at a time, as the reference) ──

def _batched(fn, x, rows, hidden):
    x = _c(x, np.float32)
    xb = x.reshape(-1, hidden)
    out = np.empty((xb.shape[0], rows), np.float32)
    for b in range(xb.shape[0]):
        y = np.empty(rows, np.float32)
        fn(np.ascontiguousarray(xb[b]), y)
        out[b] = y
    return out.reshape(rows) if x.ndim == 1 else out


def q4k_matvec(w, x, rows, hidden):
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q4k_matvec(w, xv, y, rows, hidden), x, rows, hidden)


def q6k_matvec(w, x, rows, hidden):
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q6k_matvec(w, xv, y, rows, hidden), x, rows, hidden)


def q4_0_matvec_f32(w, x, rows, hidden):
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q4_0_matvec_f32(w, xv, y, rows, hidden), x, rows, hidden)


def q4k_gguf_matvec_f32(w, x, rows, hidden):
    """GGUF-144 Q4_K (ggml.rs:228-273 dequantize) x f32, sequential f32 dot per row."""
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q4k_gguf_matvec_f32(w, xv, y, rows, hidden), x, rows, hidden)


def q4k_gguf_llama_matvec_f32(w, x, rows, hidden):
    """GGUF-144 Q4_K in llama.cpp's layout x f32, sequential f32 dot per row."""
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q4k_gguf_llama_matvec_f32(w, xv, y, rows, hidden), x, rows, hidden)


def q8_0_matvec_f32(w, x, rows, hidden):
    w = _c(w, np.uint8)
    return _batched(lambda xv, y: lib().orc_q8_0_matvec_f32(w, xv, y, rows, hidden), x, rows, hidden)


def q4_0_matvec_q8(w, q8x, q8s, rows, hidden):
    y = np.empty(rows, np.float32)
    lib().orc_q4_0_matvec_q8(_c(w, np.uint8), _c(q8x, np.int8), _c(q8s, np.float32), y, rows, hidden)
    return y


def q8_matvec(wq, ws, xq, xs, rows, hidden):
    y = np.empty(rows, np.float32)
    lib().orc_q8_matvec(_c(wq, np.int8), _c(ws, np.float32), _c(xq, np.int8), _c(xs, np.float32),
                        y, rows, hidden)
    return y


def q4_0_vecmat(act, w, inter, hidden):
    out = np.empty(hidden, np.float32)
    lib().orc_q4_0_vecmat(_c(act, np.float32), _c(w, np.uint8), out, inter, hidden)
    return out


def ref_q4_0_matvec_c(w, q8x, q8s, rows, hidden):
    """The reference's q4_0_matvec_c itself (csrc/q4_dot.c:169)."""
    R = ref_lib()
    if R is None:
        return None
    y = np.empty(rows, np.float32)
    R.q4_0_matvec_c(_c(w, np.uint8), _c(q8x, np.int8), _c(q8s, np.float32), y, rows, hidden)
    return y


def ref_q4_0_vecmat_c(act, w, inter, hidden):
    R = ref_lib()
    if R is None:
        return None
    out = np.empty(hidden, np.float32)
    R.q4_0_vecmat_c(_c(act, np.float32), _c(w, np.uint8), out, inter, hidden)
    return out


MT_KIND = {"q4k": 0, "q4_0_q8": 1, "q4_0": 2, "q8_0": 3, "q6k": 4}


def matvec_mt(kind: str, w, x, rows, hidden, threads, q8=None, q8s=None):
    """Row-split multi-threaded matvec (CPU baseline), same per-row arithmetic."""
    y = np.empty(rows, np.float32)
    L = lib()
    vp = lambda a: a.ctypes.data_as(C.c_void_p) if a is not None else None
    L.orc_matvec_mt(MT_KIND[kind], vp(w), vp(x), vp(q8), vp(q8s), vp(y), rows, hidden, threads)
    return y


# ── gate walk ──

def gate_scores_f16(gates_f16bits: np.ndarray, q: np.ndarray, n_feat: int, hidden: int) -> np.ndarray:
    g = _c(gates_f16bits, np.uint16)
    qb = _c(q, np.float32).reshape(-1, hidden)
    out = np.empty((qb.shape[0], n_feat), np.float32)
    for b in range(qb.shape[0]):
        s = np.empty(n_feat, np.float32)
        lib().orc_gate_scores_f16(g, np.ascontiguousarray(qb[b]), s, n_feat, hidden)
        out[b] = s
    return out


def gate_scores_f16_many(gates_f16bits: np.ndarray, q: np.ndarray, n_feat: int, hidden: int) -> np.ndarray:
    """gate.rs:108-134 scores of many queries against one layer at once: the rows decoded by half.rs
    (decode_f16, subnormals at half their IEEE value) times the queries, in f64 through one BLAS product.  The
    same math as orc_gate_scores_f16 up to the f64 summation order; used where the per-query C loop would take
    minutes (the 10240 x 2560 configs[4] layers at batch 1024)."""
    g = decode_f16(gates_f16bits).astype(np.float64).reshape(n_feat, hidden)
    qb = _c(q, np.float32).reshape(-1, hidden).astype(np.float64)
    return (qb @ g.T).astype(np.float32)


def top_k_abs(scores: np.ndarray, k: int):
    s = _c(scores, np.float32).reshape(-1)
    kk = min(k, s.size)
    idx = np.empty(max(kk, 1), np.uint32)
    sc = np.empty(max(kk, 1), np.float32)
    n = lib().orc_top_k_abs(s, s.size, k, idx, sc)
    return idx[:n].copy(), sc[:n].copy()


def top_k_signed(scores: np.ndarray, top_k: int):
    """walk.rs:566-577: the top_k logits by signed value, descending (top_k 0: all); ties by lower id.
    Raises ValueError on a NaN logit (the reference panics)."""
    s = _c(scores, np.float32).reshape(-1)
    idx = np.empty(max(s.size, 1), np.uint32)
    sc = np.empty(max(s.size, 1), np.float32)
    n = lib().orc_top_k_signed(s, s.size, top_k, idx, sc)
    if n == (1 << 64) - 1:
        raise ValueError("NaN logit")
    return idx[:n].copy(), sc[:n].copy()


def lm_head_knn(w_q4_0: np.ndarray, query: np.ndarray, vocab: int, hidden: int, top_k: int):
    """VectorIndex::lm_head_knn_backend's Q4 branch (walk.rs:549-583): quantize_to_q8(query), the Q4_0 x Q8
    matvec (q4_dot.c:169-199) over the vocab, then top_k_signed.  Returns (ids, logits, all logits)."""
    q8, s8 = quantize_to_q8(query)
    logits = q4_0_matvec_q8(w_q4_0, q8, s8, vocab, hidden)
    ids, vals = top_k_signed(logits, top_k)
    return ids, vals, logits


def decode_layer(x, hidden, inter, nq, nkv, hd, w, in_norm, post_norm, offset, eps, attn_scale, rope_base,
                 kc, vc, pos):
    """One decode step of one layer (composite of the reference CPU pieces).  w: dict of Q4_K byte arrays
    q, k, v, o, gate, up, down; kc / vc: uint16 [max_seq][nkv][hd] caches, updated in place at pos.
    Returns the new residual."""
    xx = _c(x, np.float32).copy()
    assert kc.dtype == np.uint16 and kc.flags.c_contiguous and vc.dtype == np.uint16 and vc.flags.c_contiguous
    lib().orc_decode_layer(xx, hidden, inter, nq, nkv, hd, _c(w["q"], np.uint8), _c(w["k"], np.uint8),
                           _c(w["v"], np.uint8), _c(w["o"], np.uint8), _c(w["gate"], np.uint8),
                           _c(w["up"], np.uint8), _c(w["down"], np.uint8), _c(in_norm, np.float32),
                           _c(post_norm, np.float32), offset, eps, attn_scale, rope_base, kc, vc, pos)
    return xx


def gate_knn_f32(gates_f32: np.ndarray, q: np.ndarray, n_feat: int, hidden: int, k: int):
    """The reference's gate KNN after warmup(): f32 dot products, top-k by |score| (CPU baseline)."""
    kk = min(k, n_feat)
    idx = np.empty(max(kk, 1), np.uint32)
    sc = np.empty(max(kk, 1), np.float32)
    n = lib().orc_gate_knn_f32(_c(gates_f32, np.float32), _c(q, np.float32), n_feat, hidden, k, idx, sc)
    return idx[:n].copy(), sc[:n].copy()


def gate_topk_f16(gates_f16bits, q, n_feat, hidden, k):
    """Per query: scores (f64-accumulated dot, rounded to f32), top-K by |score|."""
    scores = gate_scores_f16(gates_f16bits, q, n_feat, hidden)
    res = [top_k_abs(scores[b], k) for b in range(scores.shape[0])]
    return res, scores
