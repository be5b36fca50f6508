"""Python binding of the C ABI in include/larql_cuda.h (ctypes).

`CudaBackend` mirrors the reference trait `ComputeBackend`
(crates/larql-compute/src/backend.rs:24-164): the same method names, the same
argument meaning, and `None` where the trait returns `Option::None`
(operation not provided).  Other failures raise `LarqlCudaError`.

There is no CPU fallback: importing this module fails loudly if the CUDA
library has not been built, and every compute call runs the sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblarql_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "larql_cuda.h")

OK = 0
ERR_INVALID_ARG = 1
ERR_BAD_SHAPE = 2
ERR_UNSUPPORTED = 3
ERR_CUDA = 4
ERR_NCCL = 5
ERR_TIMEOUT = 6
ERR_OOM = 7
ERR_NOT_FOUND = 8

# crates/larql-compute/src/pipeline.rs:12-18 (QuantFormat), plus GGUF Q8_0 and f16 rows
FMT_Q4_0 = 0
FMT_Q4_K = 1
FMT_Q4_KF = 2
FMT_Q6_K = 3
FMT_Q8_0 = 4
FMT_Q8_0_GGUF = 5
FMT_F16 = 6
FMT_F16_HALFRS = 7  # f16 rows decoded like larql-models half.rs (vindex gate vectors)
FMT_Q4_K_GGUF = 8  # GGUF 144-byte Q4_K as larql-models ggml.rs dequantize_q4_k reads it
FMT_Q4_K_GGUF_LLAMA = 9  # GGUF 144-byte Q4_K in llama.cpp's layout, as the reference's Metal q4kf kernels read it
FORMAT_NAMES = {FMT_Q4_0: "Q4_0", FMT_Q4_K: "Q4_K", FMT_Q4_KF: "Q4_KF", FMT_Q6_K: "Q6_K", FMT_Q8_0: "Q8_0",
                FMT_Q8_0_GGUF: "Q8_0_GGUF", FMT_F16: "F16", FMT_F16_HALFRS: "F16_HALFRS",
                FMT_Q4_K_GGUF: "Q4_K_GGUF", FMT_Q4_K_GGUF_LLAMA: "Q4_K_GGUF_LLAMA"}


def format_bytes(fmt: int, rows: int, cols: int) -> int:
    n = rows * cols
    return {FMT_Q4_0: n // 32 * 18, FMT_Q4_K: n // 256 * 148, FMT_Q4_KF: n // 256 * 160,
            FMT_Q6_K: n // 256 * 210, FMT_Q8_0: n, FMT_Q8_0_GGUF: n // 32 * 34, FMT_F16: n * 2,
            FMT_F16_HALFRS: n * 2, FMT_Q4_K_GGUF: n // 256 * 144, FMT_Q4_K_GGUF_LLAMA: n // 256 * 144}[fmt]


# larql_cuda_reduce_fn: int (*)(void* user, float* buf, size_t n, void* stream)
REDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p)


class LayerDesc(C.Structure):
    """larql_cuda_layer_desc: the Llama / Q4_K subset of FullPipelineLayer (pipeline.rs:60-110)."""
    _fields_ = [("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("input_norm", C.c_void_p), ("post_attn_norm", C.c_void_p),
                ("norm_offset", C.c_float), ("eps", C.c_float), ("attn_scale", C.c_float)]


class VindexInfo(C.Structure):
    """larql_cuda_vindex_info: what index.json and the files of a vindex directory hold (VindexConfig,
    crates/larql-vindex/src/config/types.rs), plus the row shard an opened vindex holds."""
    _fields_ = [("num_layers", C.c_size_t), ("hidden", C.c_size_t), ("intermediate", C.c_size_t),
                ("vocab", C.c_size_t), ("features_max", C.c_size_t), ("gate_bits", C.c_int),
                ("ffn_q4k", C.c_int), ("attn_q4k", C.c_int), ("gate_q4", C.c_int), ("shard_rank", C.c_size_t),
                ("shard_count", C.c_size_t), ("shard_row0", C.c_size_t), ("shard_rows", C.c_size_t)]


class LarqlCudaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


_lib = None


def lib() -> C.CDLL:
    """The loaded C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python encoding-experiment_b200/build.py` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        vp, sz, i32, u64 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint64
        sigs = {
            "larql_cuda_version": ([], i32),
            "larql_cuda_last_error": ([C.c_char_p, sz], i32),
            "larql_cuda_status_string": ([i32], C.c_char_p),
            "larql_cuda_create": ([i32, C.POINTER(vp)], i32),
            "larql_cuda_destroy": ([vp], i32),
            "larql_cuda_name": ([vp, C.c_char_p, sz], i32),
            "larql_cuda_device_info": ([vp, C.c_char_p, sz], i32),
            "larql_cuda_has_q4": ([vp, C.POINTER(i32)], i32),
            "larql_cuda_stream": ([vp, C.POINTER(vp)], i32),
            "larql_cuda_sync": ([vp], i32),
            "larql_cuda_register_weight": ([vp, vp, sz, vp, i32, sz, sz, C.POINTER(u64)], i32),
            "larql_cuda_register_weight_device": ([vp, vp, sz, vp, i32, sz, sz, C.POINTER(u64)], i32),
            "larql_cuda_release_weight": ([vp, u64], i32),
            "larql_cuda_weight_device_ptr": ([vp, u64, C.POINTER(vp)], i32),
            "larql_cuda_q4k_matvec": ([vp, vp, sz, vp, sz, sz, vp], i32),
            "larql_cuda_q6k_matvec": ([vp, vp, sz, vp, sz, sz, vp], i32),
            "larql_cuda_q4_vecmat": ([vp, vp, vp, sz, sz, sz, vp], i32),
            "larql_cuda_q4_vecmat_dev": ([vp, u64, vp, vp, vp], i32),
            "larql_cuda_q4_matvec_pair_batch": ([vp, vp, sz, vp, sz, vp, sz, sz, sz, vp, vp], i32),
            "larql_cuda_q4_matvec_pair_batch_dev": ([vp, u64, u64, vp, sz, vp, vp, vp], i32),
            "larql_cuda_quantize_q6_k_dev": ([vp, vp, sz, vp, vp], i32),
            "larql_cuda_matvec": ([vp, u64, vp, sz, vp], i32),
            "larql_cuda_matvec_dev": ([vp, u64, vp, sz, vp, vp], i32),
            "larql_cuda_quantize_q4_k_dev": ([vp, vp, sz, vp, vp], i32),
            "larql_cuda_q4k_matvec_noalloc": ([vp, sz, sz, sz, vp, sz, vp, vp], i32),
            "larql_cuda_q4_matvec": ([vp, vp, sz, vp, vp, sz, sz, vp], i32),
            "larql_cuda_q4_matvec_dev": ([vp, u64, vp, vp, vp, vp], i32),
            "larql_cuda_quantize_to_q8_dev": ([vp, vp, sz, vp, vp, vp], i32),
            "larql_cuda_launch_count": ([C.POINTER(u64)], i32),
            "larql_cuda_describe_matvec": ([vp, u64, sz, C.c_char_p, sz], i32),
            "larql_cuda_gate_topk_f16": ([vp, vp, sz, sz, sz, sz, vp, sz, sz, vp, vp], i32),
            "larql_cuda_gate_topk_dev": ([vp, u64, sz, sz, vp, sz, sz, vp, vp, vp], i32),
            "larql_cuda_topk_merge_dev": ([vp, vp, vp, sz, sz, sz, vp, sz, vp, vp, vp], i32),
            "larql_cuda_lm_head_knn": ([vp, vp, sz, sz, sz, vp, sz, vp, vp, C.POINTER(sz)], i32),
            "larql_cuda_lm_head_knn_dev": ([vp, u64, vp, sz, vp, vp, vp], i32),
            "larql_cuda_logit_topk_dev": ([vp, vp, sz, sz, vp, vp, vp], i32),
            "larql_cuda_gate_scores_f16": ([vp, vp, sz, sz, sz, sz, vp, sz, vp], i32),
            "larql_cuda_gate_scores_dev": ([vp, u64, sz, sz, vp, sz, vp, vp], i32),
            "larql_cuda_gate_knn_batch_f16": ([vp, vp, sz, sz, sz, vp, sz, sz, vp, C.POINTER(sz)], i32),
            "larql_cuda_q4k_gemm_dev": ([vp, u64, vp, sz, vp, vp], i32),
            "larql_cuda_prefill_ffn_dev": ([vp, u64, u64, u64, vp, sz, vp, vp], i32),
            "larql_cuda_prefill_ffn": ([vp, vp, sz, vp, sz, vp, sz, sz, sz, vp, sz, vp], i32),
            "larql_cuda_layer_register": ([vp, C.POINTER(LayerDesc), sz, sz, sz, sz, sz, i32, C.POINTER(u64)], i32),
            "larql_cuda_layer_release": ([vp, u64], i32),
            "larql_cuda_kv_init": ([vp, sz, sz, sz, sz], i32),
            "larql_cuda_kv_populate": ([vp, sz, vp, vp, sz], i32),
            "larql_cuda_kv_populate_f16_dev": ([vp, sz, vp, vp, sz, vp], i32),
            "larql_cuda_kv_reset": ([vp], i32),
            "larql_cuda_kv_set_length": ([vp, sz], i32),
            "larql_cuda_decode_set_persistent": ([vp, C.c_int], i32),
            "larql_cuda_kv_length": ([vp, C.POINTER(sz)], i32),
            "larql_cuda_decode_token": ([vp, vp, sz, vp, C.c_float, vp], i32),
            "larql_cuda_decode_token_dev": ([vp, vp, sz, vp, sz, C.c_float, vp], i32),
            "larql_cuda_layer_register_shard": ([vp, C.POINTER(LayerDesc), sz, sz, sz, sz, sz, sz, sz, i32,
                                                 C.POINTER(u64)], i32),
            "larql_cuda_decode_token_sharded_dev": ([vp, vp, sz, vp, sz, C.c_float, vp, REDUCE_FN, vp, vp], i32),
            "larql_cuda_p2p_init": ([vp, sz, sz, sz, vp], i32),
            "larql_cuda_p2p_connect": ([vp, vp], i32),
            "larql_cuda_p2p_allreduce_dev": ([vp, vp, sz, vp], i32),
            "larql_cuda_quantize_q4_0_dev": ([vp, vp, sz, vp, vp], i32),
            "larql_cuda_quantize_q8_0_dev": ([vp, vp, sz, vp, vp], i32),
            "larql_cuda_gate_topk_q4": ([vp, vp, sz, sz, sz, sz, vp, sz, sz, vp, vp], i32),
            "larql_cuda_gate_topk_q4_dev": ([vp, u64, sz, sz, vp, sz, sz, vp, vp, vp], i32),
            "larql_cuda_vindex_probe": ([C.c_char_p, C.POINTER(VindexInfo)], i32),
            "larql_cuda_vindex_open": ([vp, C.c_char_p, sz, sz, C.POINTER(vp)], i32),
            "larql_cuda_vindex_info_get": ([vp, C.POINTER(VindexInfo)], i32),
            "larql_cuda_vindex_gate_knn": ([vp, vp, sz, sz, vp, vp], i32),
            "larql_cuda_vindex_gate_knn_q4": ([vp, vp, sz, sz, vp, vp], i32),
            "larql_cuda_vindex_gate_knn_dev": ([vp, vp, sz, sz, vp, vp, vp], i32),
            "larql_cuda_vindex_ffn": ([vp, sz, C.POINTER(u64), C.POINTER(u64), C.POINTER(u64), C.POINTER(i32)], i32),
            "larql_cuda_vindex_attn": ([vp, sz, C.POINTER(u64), C.POINTER(i32)], i32),
            "larql_cuda_vindex_close": ([vp], i32),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def header_functions() -> list[str]:
    """Names of every function declared in include/larql_cuda.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(larql_cuda_\w+)\s*\(", text)))


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().larql_cuda_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        raise LarqlCudaError(status, last_error())


def launch_count() -> int:
    """Kernel launches this library has enqueued in this process (host-side count)."""
    v = C.c_uint64()
    check(lib().larql_cuda_launch_count(C.byref(v)))
    return v.value


def _ptr(a) -> int:
    """Address of a numpy array or torch tensor's data."""
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    if a is None:
        return 0
    return int(a)


def _host_f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _host_u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


class Weight:
    """A weight placed on the device once (registry handle)."""

    def __init__(self, backend: "CudaBackend", handle: int, fmt: int, rows: int, cols: int, keepalive=None):
        self.backend, self.handle, self.format, self.rows, self.cols = backend, handle, fmt, rows, cols
        self._keepalive = keepalive

    def release(self) -> None:
        if self.handle:
            check(lib().larql_cuda_release_weight(self.backend.ctx, self.handle))
            self.handle = 0


class CudaBackend:
    """sm_100a implementation of the ComputeBackend methods on the hot path."""

    def __init__(self, device: int = 0):
        self.ctx = C.c_void_p()
        check(lib().larql_cuda_create(device, C.byref(self.ctx)))
        self.device = device
        self._pinned = []  # host buffers whose registry entries must outlive calls

    def close(self) -> None:
        if self.ctx:
            lib().larql_cuda_destroy(self.ctx)
            self.ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ── metadata (backend.rs:155-163) ──
    def name(self) -> str:
        buf = C.create_string_buffer(256)
        check(lib().larql_cuda_name(self.ctx, buf, 256))
        return buf.value.decode()

    def device_info(self) -> str:
        buf = C.create_string_buffer(512)
        check(lib().larql_cuda_device_info(self.ctx, buf, 512))
        return buf.value.decode()

    def has_q4(self) -> bool:
        v = C.c_int()
        check(lib().larql_cuda_has_q4(self.ctx, C.byref(v)))
        return bool(v.value)

    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().larql_cuda_stream(self.ctx, C.byref(s)))
        return s.value or 0

    def sync(self) -> None:
        check(lib().larql_cuda_sync(self.ctx))

    # ── registry ──
    def register_weight(self, data, fmt: int, rows: int, cols: int, scales=None) -> Weight:
        """Place host bytes (numpy) or a device tensor (torch, cuda) on the device once."""
        h = C.c_uint64()
        if hasattr(data, "is_cuda") and data.is_cuda:
            nbytes = data.numel() * data.element_size()
            check(lib().larql_cuda_register_weight_device(self.ctx, _ptr(data), nbytes, _ptr(scales), fmt, rows,
                                                          cols, C.byref(h)))
            return Weight(self, h.value, fmt, rows, cols)
        arr = np.ascontiguousarray(data)
        sc = None if scales is None else _host_f32(scales)
        check(lib().larql_cuda_register_weight(self.ctx, arr.ctypes.data, arr.nbytes,
                                               None if sc is None else sc.ctypes.data, fmt, rows, cols,
                                               C.byref(h)))
        return Weight(self, h.value, fmt, rows, cols, keepalive=(arr, sc))

    # ── trait mirrors (host slices in, owned Vec<f32> out) ──
    def q4k_matvec(self, q4k_data, x, num_rows: int, hidden: int):
        """ComputeBackend::q4k_matvec (backend.rs:126-130): scores[N] = Q4_K[N,K] @ x[K]."""
        w = _host_u8(q4k_data)
        xv = _host_f32(x)
        if xv.size != hidden:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"x has {xv.size} values, hidden={hidden}")
        out = np.empty(num_rows, np.float32)
        st = lib().larql_cuda_q4k_matvec(self.ctx, w.ctypes.data, w.nbytes, xv.ctypes.data, num_rows, hidden,
                                         out.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(w)  # the registry is keyed by this buffer's address
        return out

    def q6k_matvec(self, q6k_data, x, num_rows: int, hidden: int):
        """ComputeBackend::q6k_matvec (backend.rs:133-137): scores[N] = Q6_K[N,K] @ x[K]."""
        w = _host_u8(q6k_data)
        xv = _host_f32(x)
        if xv.size != hidden:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"x has {xv.size} values, hidden={hidden}")
        out = np.empty(num_rows, np.float32)
        st = lib().larql_cuda_q6k_matvec(self.ctx, w.ctypes.data, w.nbytes, xv.ctypes.data, num_rows, hidden,
                                         out.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(w)
        return out

    def q4_matvec(self, q4_data, q8_x, q8_scales, num_rows: int, hidden: int):
        """ComputeBackend::q4_matvec (backend.rs:49-53): scores[N] = Q4_0[N,K] @ Q8_x[K]."""
        w = _host_u8(q4_data)
        q = np.ascontiguousarray(q8_x, dtype=np.int8)
        sc = _host_f32(q8_scales)
        out = np.empty(num_rows, np.float32)
        st = lib().larql_cuda_q4_matvec(self.ctx, w.ctypes.data, w.nbytes, q.ctypes.data, sc.ctypes.data, num_rows,
                                        hidden, out.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(w)
        return out

    def q4_vecmat(self, activation, q4_data, intermediate: int, hidden: int):
        """ComputeBackend::q4_vecmat (backend.rs:56-60): out[hidden] = activation[intermediate] @ Q4_0[inter, hidden]."""
        w = _host_u8(q4_data)
        a = _host_f32(activation)
        if a.size != intermediate:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"activation has {a.size} values, intermediate={intermediate}")
        out = np.empty(hidden, np.float32)
        st = lib().larql_cuda_q4_vecmat(self.ctx, a.ctypes.data, w.ctypes.data, w.nbytes, intermediate, hidden,
                                        out.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(w)
        return out

    def q4_vecmat_dev(self, w: "Weight", act, out, stream=None) -> None:
        """Device q4_vecmat on a registered Q4_0 weight (rows = intermediate, cols = hidden)."""
        check(lib().larql_cuda_q4_vecmat_dev(self.ctx, w.handle, _ptr(act), _ptr(out),
                                             None if stream is None else C.c_void_p(int(stream))))

    def q4_matvec_pair_batch(self, gate_q4, up_q4, x_matrix, seq_len: int, num_rows: int, hidden: int):
        """ComputeBackend::q4_matvec_pair_batch (backend.rs:64-69): (gate, up), each [seq_len][num_rows]."""
        g = _host_u8(gate_q4)
        u = _host_u8(up_q4)
        x = _host_f32(x_matrix)
        if x.size != seq_len * hidden:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"x_matrix has {x.size} values, seq_len*hidden={seq_len * hidden}")
        go = np.empty((seq_len, num_rows), np.float32)
        uo = np.empty((seq_len, num_rows), np.float32)
        st = lib().larql_cuda_q4_matvec_pair_batch(self.ctx, g.ctypes.data, g.nbytes, u.ctypes.data, u.nbytes,
                                                   x.ctypes.data, seq_len, num_rows, hidden, go.ctypes.data,
                                                   uo.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.extend([g, u])
        return go, uo

    def q4_matvec_pair_batch_dev(self, gate: "Weight", up: "Weight", x, seq_len: int, gate_out, up_out,
                                 stream=None) -> None:
        check(lib().larql_cuda_q4_matvec_pair_batch_dev(self.ctx, gate.handle, up.handle, _ptr(x), seq_len,
                                                        _ptr(gate_out), _ptr(up_out),
                                                        None if stream is None else C.c_void_p(int(stream))))

    def gate_topk_f16(self, gates_f16bits, n_layers: int, n_feat: int, hidden: int, queries, top_k: int):
        """VectorIndex::gate_knn (gate.rs:108-134) for every layer and query: -> (idx, score), each
        [n_layers][batch][top_k] (index 0xFFFFFFFF / score 0 where a layer has fewer than top_k rows)."""
        g = np.ascontiguousarray(gates_f16bits, dtype=np.uint16)
        q = _host_f32(queries).reshape(-1, hidden)
        b = q.shape[0]
        idx = np.empty((n_layers, b, top_k), np.uint32)
        sc = np.empty((n_layers, b, top_k), np.float32)
        st = lib().larql_cuda_gate_topk_f16(self.ctx, g.ctypes.data, g.nbytes, n_layers, n_feat, hidden,
                                            q.ctypes.data, b, top_k, idx.ctypes.data, sc.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(g)
        return idx, sc

    def gate_knn_q4(self, gates_q4, n_layers: int, n_feat: int, hidden: int, queries, top_k: int):
        """VectorIndex::gate_knn_q4 (gate.rs:714-731) for every layer of Q4_0 gates and every query:
        (idx, score), each [n_layers][batch][top_k]; None where the trait would return None."""
        g = _host_u8(gates_q4)
        q = _host_f32(queries).reshape(-1, hidden)
        b = q.shape[0]
        idx = np.empty((n_layers, b, top_k), np.uint32)
        sc = np.empty((n_layers, b, top_k), np.float32)
        st = lib().larql_cuda_gate_topk_q4(self.ctx, g.ctypes.data, g.nbytes, n_layers, n_feat, hidden,
                                           q.ctypes.data, b, top_k, idx.ctypes.data, sc.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(g)
        return idx, sc

    def gate_topk_q4_dev(self, w: Weight, n_layers: int, n_feat: int, queries, batch: int, top_k: int, out_idx,
                         out_score, stream=None) -> None:
        """Device form of gate_knn_q4 on a registered Q4_0 weight of n_layers * n_feat rows."""
        check(lib().larql_cuda_gate_topk_q4_dev(self.ctx, w.handle, n_layers, n_feat, _ptr(queries), batch, top_k,
                                                _ptr(out_idx), _ptr(out_score),
                                                None if stream is None else C.c_void_p(int(stream))))

    def gate_topk_dev(self, w: Weight, n_layers: int, n_feat: int, queries, batch: int, top_k: int, out_idx,
                      out_score, stream=None) -> None:
        """Device-pointer gate walk on a registered FMT_F16_HALFRS weight."""
        check(lib().larql_cuda_gate_topk_dev(self.ctx, w.handle, n_layers, n_feat, _ptr(queries), batch, top_k,
                                             _ptr(out_idx), _ptr(out_score),
                                             None if stream is None else C.c_void_p(int(stream))))

    def gate_scores_f16(self, gates_f16bits, n_layers: int, n_feat: int, hidden: int, queries):
        """gate_scores_batch (gate.rs:545-559) for every layer: scores [n_layers][batch][n_feat] (or None)."""
        g = np.ascontiguousarray(gates_f16bits, dtype=np.uint16)
        q = _host_f32(queries).reshape(-1, hidden)
        b = q.shape[0]
        out = np.empty((n_layers, b, n_feat), np.float32)
        st = lib().larql_cuda_gate_scores_f16(self.ctx, g.ctypes.data, g.nbytes, n_layers, n_feat, hidden,
                                              q.ctypes.data, b, out.ctypes.data)
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(g)
        return out

    def gate_scores_dev(self, w: Weight, n_layers: int, n_feat: int, queries, batch: int, out, stream=None) -> None:
        """Device-pointer gate_scores_batch on a registered FMT_F16_HALFRS weight: out [n_layers][batch][n_feat]."""
        check(lib().larql_cuda_gate_scores_dev(self.ctx, w.handle, n_layers, n_feat, _ptr(queries), batch, _ptr(out),
                                               None if stream is None else C.c_void_p(int(stream))))

    def gate_knn_batch_f16(self, gates_f16bits, n_feat: int, hidden: int, x, top_k: int):
        """gate_knn_batch (gate.rs:500-537): sorted union of the per-position top-k features (or None)."""
        g = np.ascontiguousarray(gates_f16bits, dtype=np.uint16)
        q = _host_f32(x).reshape(-1, hidden)
        seq = q.shape[0]
        out = np.empty(max(1, seq * min(top_k, n_feat)), np.uint32)
        cnt = C.c_size_t(0)
        st = lib().larql_cuda_gate_knn_batch_f16(self.ctx, g.ctypes.data, g.nbytes, n_feat, hidden, q.ctypes.data,
                                                 seq, top_k, out.ctypes.data, C.byref(cnt))
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(g)
        return out[:cnt.value].astype(np.int64)

    def topk_merge_dev(self, idx_in, score_in, n_lists: int, rows: int, k_in: int, k_out: int, idx_out, score_out,
                       offsets=None, stream=None) -> None:
        """Merge [n_lists][rows][k_in] top-k lists (indices + offsets[list]) into [rows][k_out]."""
        check(lib().larql_cuda_topk_merge_dev(self.ctx, _ptr(idx_in), _ptr(score_in), n_lists, rows, k_in,
                                              None if offsets is None else _ptr(offsets), k_out, _ptr(idx_out),
                                              _ptr(score_out), None if stream is None else C.c_void_p(int(stream))))

    # ── lm-head KNN ──
    def lm_head_knn(self, q4_data, query, vocab: int, hidden: int, top_k: int):
        """VectorIndex::lm_head_knn_backend, Q4 branch (walk.rs:549-583): (token ids, logits) of the top_k logits
        by signed value, descending; None where the backend does not provide it (top_k 0 or > 32)."""
        w = _host_u8(q4_data)
        q = _host_f32(query)
        if q.size != hidden:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"query has {q.size} values, hidden={hidden}")
        k = max(1, min(top_k, vocab))
        ids = np.empty(k, np.uint32)
        vals = np.empty(k, np.float32)
        cnt = C.c_size_t(0)
        st = lib().larql_cuda_lm_head_knn(self.ctx, w.ctypes.data, w.nbytes, vocab, hidden, q.ctypes.data, top_k,
                                          ids.ctypes.data, vals.ctypes.data, C.byref(cnt))
        if st == ERR_UNSUPPORTED:
            return None
        check(st)
        self._pinned.append(w)
        return ids[:cnt.value].astype(np.int64), vals[:cnt.value]

    def lm_head_knn_dev(self, w: Weight, query, top_k: int, ids, logits, stream=None) -> None:
        """Device-pointer lm-head KNN on a registered Q4_0 weight (rows = vocab)."""
        check(lib().larql_cuda_lm_head_knn_dev(self.ctx, w.handle, _ptr(query), top_k, _ptr(ids), _ptr(logits),
                                               None if stream is None else C.c_void_p(int(stream))))

    def logit_topk_dev(self, logits, n: int, top_k: int, ids, out, stream=None) -> None:
        """The min(top_k, n) largest of n device logits, descending (equal logits by lower id)."""
        check(lib().larql_cuda_logit_topk_dev(self.ctx, _ptr(logits), n, top_k, _ptr(ids), _ptr(out),
                                              None if stream is None else C.c_void_p(int(stream))))

    # ── batched prefill ──
    def q4k_gemm_dev(self, w: Weight, x, n_tokens: int, y, stream=None) -> None:
        """Y[t][n] = W[n] . X[t] (tcgen05 dequant-GEMM)."""
        check(lib().larql_cuda_q4k_gemm_dev(self.ctx, w.handle, _ptr(x), n_tokens, _ptr(y),
                                            None if stream is None else C.c_void_p(int(stream))))

    def prefill_ffn_dev(self, gate: Weight, up: Weight, down: Weight, x, n_tokens: int, y, stream=None) -> None:
        """y[t] = down . (silu(gate . x[t]) * (up . x[t]))."""
        check(lib().larql_cuda_prefill_ffn_dev(self.ctx, gate.handle, up.handle, down.handle, _ptr(x), n_tokens,
                                               _ptr(y), None if stream is None else C.c_void_p(int(stream))))

    def prefill_ffn(self, gate, up, down, x, hidden: int, inter: int):
        """The FFN half of prefill_q4 (backend.rs:143-152) with host buffers: Q4_K gate / up [inter][hidden],
        down [hidden][inter] as uint8 arrays, x [n_tokens][hidden] f32 -> y [n_tokens][hidden] f32."""
        g, u, d = _host_u8(gate), _host_u8(up), _host_u8(down)
        xx = _host_f32(x).reshape(-1, hidden)
        y = np.empty_like(xx)
        check(lib().larql_cuda_prefill_ffn(self.ctx, g.ctypes.data, g.nbytes, u.ctypes.data, u.nbytes, d.ctypes.data,
                                           d.nbytes, hidden, inter, xx.ctypes.data, xx.shape[0], y.ctypes.data))
        self._pinned.extend([g, u, d])
        return y

    # ── decode (decode_token, backend.rs:99-124) ──
    def layer_register(self, w: dict, input_norm, post_attn_norm, hidden: int, inter: int, nq: int, nkv: int,
                       head_dim: int = 128, norm_offset: float = 0.0, eps: float = 1e-5, attn_scale=None) -> int:
        """w: Q4_K weights q, k, v, o, gate, up, down as numpy uint8 arrays or cuda tensors -> layer handle."""
        dev = hasattr(w["q"], "is_cuda") and w["q"].is_cuda
        keep = {k: (v if dev else np.ascontiguousarray(v, dtype=np.uint8)) for k, v in w.items()}
        ni = input_norm if (hasattr(input_norm, "is_cuda") and input_norm.is_cuda) else _host_f32(input_norm)
        npn = post_attn_norm if (hasattr(post_attn_norm, "is_cuda") and post_attn_norm.is_cuda) else _host_f32(post_attn_norm)
        d = LayerDesc(_ptr(keep["q"]), _ptr(keep["k"]), _ptr(keep["v"]), _ptr(keep["o"]), _ptr(keep["gate"]),
                      _ptr(keep["up"]), _ptr(keep["down"]), _ptr(ni), _ptr(npn), norm_offset, eps,
                      attn_scale if attn_scale is not None else 1.0 / np.sqrt(head_dim))
        h = C.c_uint64()
        check(lib().larql_cuda_layer_register(self.ctx, C.byref(d), hidden, inter, nq, nkv, head_dim, int(dev),
                                              C.byref(h)))
        return h.value

    def layer_release(self, h: int) -> None:
        check(lib().larql_cuda_layer_release(self.ctx, h))

    def kv_init(self, n_layers: int, max_seq: int, nkv: int, head_dim: int = 128) -> None:
        check(lib().larql_cuda_kv_init(self.ctx, n_layers, max_seq, nkv, head_dim))

    def kv_populate(self, layer: int, k, v, seq_len: int) -> None:
        """populate_kv_layer (backend.rs:103-107): k / v f32 [seq_len][nkv*head_dim] (host)."""
        kk, vv = _host_f32(k), _host_f32(v)
        check(lib().larql_cuda_kv_populate(self.ctx, layer, kk.ctypes.data, vv.ctypes.data, seq_len))

    def kv_populate_f16_dev(self, layer: int, k, v, seq_len: int, stream=None) -> None:
        check(lib().larql_cuda_kv_populate_f16_dev(self.ctx, layer, _ptr(k), _ptr(v), seq_len,
                                                   None if stream is None else C.c_void_p(int(stream))))

    def kv_reset(self) -> None:
        check(lib().larql_cuda_kv_reset(self.ctx))

    def decode_set_persistent(self, on: bool) -> None:
        """Run later decode tokens as one persistent launch where the layers allow it (decode_persist.cu)."""
        check(lib().larql_cuda_decode_set_persistent(self.ctx, 1 if on else 0))

    def kv_set_length(self, n: int) -> None:
        check(lib().larql_cuda_kv_set_length(self.ctx, n))

    def kv_length(self) -> int:
        v = C.c_size_t()
        check(lib().larql_cuda_kv_length(self.ctx, C.byref(v)))
        return v.value

    def decode_token(self, layers, x, rope_base: float) -> np.ndarray:
        """decode_token (backend.rs:115-124): one token through `layers` at position = kv_length()."""
        hs = (C.c_uint64 * len(layers))(*layers)
        xv = _host_f32(x)
        out = np.empty_like(xv)
        check(lib().larql_cuda_decode_token(self.ctx, hs, len(layers), xv.ctypes.data, rope_base, out.ctypes.data))
        return out

    def decode_token_dev(self, layers, x_dev, pos: int, rope_base: float, stream=None) -> None:
        hs = (C.c_uint64 * len(layers))(*layers)
        check(lib().larql_cuda_decode_token_dev(self.ctx, hs, len(layers), _ptr(x_dev), pos, rope_base,
                                                None if stream is None else C.c_void_p(int(stream))))

    def layer_register_shard(self, w: dict, input_norm, post_attn_norm, hidden: int, inter: int, nq: int, nkv: int,
                             rank: int, world: int, head_dim: int = 128, norm_offset: float = 0.0, eps: float = 1e-5,
                             attn_scale=None) -> int:
        """Rank `rank`'s share of a full layer (heads / FFN rows split over `world`) -> layer handle."""
        dev = hasattr(w["q"], "is_cuda") and w["q"].is_cuda
        keep = {k: (v if dev else np.ascontiguousarray(v, dtype=np.uint8)) for k, v in w.items()}
        ni = input_norm if (hasattr(input_norm, "is_cuda") and input_norm.is_cuda) else _host_f32(input_norm)
        npn = post_attn_norm if (hasattr(post_attn_norm, "is_cuda") and post_attn_norm.is_cuda) else _host_f32(post_attn_norm)
        d = LayerDesc(_ptr(keep["q"]), _ptr(keep["k"]), _ptr(keep["v"]), _ptr(keep["o"]), _ptr(keep["gate"]),
                      _ptr(keep["up"]), _ptr(keep["down"]), _ptr(ni), _ptr(npn), norm_offset, eps,
                      attn_scale if attn_scale is not None else 1.0 / np.sqrt(head_dim))
        h = C.c_uint64()
        check(lib().larql_cuda_layer_register_shard(self.ctx, C.byref(d), hidden, inter, nq, nkv, head_dim, rank,
                                                    world, int(dev), C.byref(h)))
        return h.value

    def decode_token_sharded_dev(self, layers, x_dev, pos: int, rope_base: float, red_dev, reduce, stream=None):
        """One token through sharded layers; `reduce(buf_ptr, n, stream_ptr)` must all-reduce the n floats at
        buf_ptr across ranks on that stream and return 0."""
        hs = (C.c_uint64 * len(layers))(*layers)
        cbs = self.__dict__.setdefault("_reduce_cbs", {})
        cb = cbs.get(id(reduce))
        if cb is None:  # one ctypes thunk per reduce callable, kept alive with the backend
            def thunk(user, buf, n, st):
                try:
                    return int(reduce(buf, n, st) or 0)
                except Exception:  # an exception cannot cross the C frame: report a failed reduction
                    import traceback
                    traceback.print_exc()
                    return 1
            cb = cbs[id(reduce)] = (REDUCE_FN(thunk), reduce)
        cb = cb[0]
        check(lib().larql_cuda_decode_token_sharded_dev(self.ctx, hs, len(layers), _ptr(x_dev), pos, rope_base,
                                                        _ptr(red_dev), cb, None,
                                                        None if stream is None else C.c_void_p(int(stream))))

    def p2p_init(self, rank: int, world: int, max_n: int) -> bytes:
        """Receive area of the peer-memory all-reduce; returns this rank's 64-byte IPC handle."""
        buf = (C.c_uint8 * 64)()
        check(lib().larql_cuda_p2p_init(self.ctx, rank, world, max_n, buf))
        return bytes(buf)

    def p2p_connect(self, handles) -> None:
        """Maps every rank's area (handles: `world` 64-byte IPC handles in rank order)."""
        blob = b"".join(handles)
        check(lib().larql_cuda_p2p_connect(self.ctx, blob))

    def p2p_allreduce_dev(self, buf, n: int, stream=None) -> None:
        """Sums `n` floats of the device buffer across the ranks, in place, enqueued on `stream`."""
        check(lib().larql_cuda_p2p_allreduce_dev(self.ctx, _ptr(buf) if not isinstance(buf, int) else C.c_void_p(buf),
                                                 n, None if stream is None else C.c_void_p(int(stream))))

    def quantize_to_q8_dev(self, x, q8, scales, stream=None) -> None:
        """Device quantize_to_q8 (bit-identical to q4_common.rs:28-44)."""
        check(lib().larql_cuda_quantize_to_q8_dev(self.ctx, _ptr(x), x.numel(), _ptr(q8), _ptr(scales),
                                                  None if stream is None else C.c_void_p(int(stream))))

    # ── handle API ──
    def matvec(self, w: Weight, x) -> np.ndarray:
        """y[b, r] = W[r, :] . x[b, :] (host arrays, synchronous)."""
        xv = _host_f32(x)
        batch = xv.size // w.cols
        if batch * w.cols != xv.size:
            raise LarqlCudaError(ERR_BAD_SHAPE, f"x size {xv.size} is not a multiple of cols={w.cols}")
        y = np.empty((batch, w.rows), np.float32)
        check(lib().larql_cuda_matvec(self.ctx, w.handle, xv.ctypes.data, batch, y.ctypes.data))
        return y.reshape(w.rows) if xv.ndim == 1 else y

    def matvec_dev(self, w: Weight, x, y, batch: int = 1, stream=None) -> None:
        """Device pointers / cuda tensors; enqueued on `stream` (int handle) or the context stream."""
        check(lib().larql_cuda_matvec_dev(self.ctx, w.handle, _ptr(x), batch, _ptr(y),
                                          None if stream is None else C.c_void_p(int(stream))))

    def describe_matvec(self, w: Weight, batch: int = 1) -> str:
        """The kernel(s) and launch plan matvec uses for this weight at this batch."""
        buf = C.create_string_buffer(256)
        check(lib().larql_cuda_describe_matvec(self.ctx, w.handle, batch, buf, 256))
        return buf.value.decode()

    def quantize_q4_0_dev(self, data, out, stream=None) -> None:
        """Device Q4_0 quantizer (bit-identical to q4_common.rs:50-80)."""
        check(lib().larql_cuda_quantize_q4_0_dev(self.ctx, _ptr(data), data.numel(), _ptr(out),
                                                 None if stream is None else C.c_void_p(int(stream))))

    def quantize_q8_0_dev(self, data, out, stream=None) -> None:
        """Device GGUF Q8_0 quantizer (bit-identical to ggml.rs:342-363)."""
        check(lib().larql_cuda_quantize_q8_0_dev(self.ctx, _ptr(data), data.numel(), _ptr(out),
                                                 None if stream is None else C.c_void_p(int(stream))))

    def quantize_q6_k_dev(self, data, out, stream=None) -> None:
        """Device Q6_K quantizer (bit-identical to q4_common.rs:179-239)."""
        check(lib().larql_cuda_quantize_q6_k_dev(self.ctx, _ptr(data), data.numel(), _ptr(out),
                                                 None if stream is None else C.c_void_p(int(stream))))

    def quantize_q4_k_dev(self, data, out, stream=None) -> None:
        """Device Q4_K quantizer (bit-identical to q4_common.rs:104-170)."""
        n = data.numel()
        check(lib().larql_cuda_quantize_q4_k_dev(self.ctx, _ptr(data), n, _ptr(out),
                                                 None if stream is None else C.c_void_p(int(stream))))


def vindex_probe(path: str) -> VindexInfo:
    """Reads and checks a .vindex directory on the host (no GPU): index.json and the files it names."""
    info = VindexInfo()
    check(lib().larql_cuda_vindex_probe(os.fsencode(path), C.byref(info)))
    return info


class Vindex:
    """A .vindex directory placed once on one GPU (VectorIndex::load_vindex, crates/larql-vindex/src/format/
    load.rs:19-87): the gate rows of every layer (this rank's row shard of them), and on request the Q4_K FFN
    and attention weights, as registered weights of `backend`."""

    def __init__(self, backend: CudaBackend, path: str, shard_rank: int = 0, shard_count: int = 1):
        self.backend = backend
        self.h = C.c_void_p()
        check(lib().larql_cuda_vindex_open(backend.ctx, os.fsencode(path), shard_rank, shard_count, C.byref(self.h)))
        self.info = VindexInfo()
        check(lib().larql_cuda_vindex_info_get(self.h, C.byref(self.info)))

    def gate_knn(self, queries, top_k: int):
        """gate_knn (gate.rs:108-134, 307-316) for every layer held: (idx, score), each [layers][batch][top_k];
        feature indices within the layer, 0xFFFFFFFF / 0 past a layer's rows."""
        q = _host_f32(queries).reshape(-1, self.info.hidden)
        b, nl = q.shape[0], self.info.num_layers
        idx = np.empty((nl, b, top_k), np.uint32)
        sc = np.empty((nl, b, top_k), np.float32)
        check(lib().larql_cuda_vindex_gate_knn(self.h, q.ctypes.data, b, top_k, idx.ctypes.data, sc.ctypes.data))
        return idx, sc

    def gate_knn_q4(self, queries, top_k: int):
        """gate_knn_q4 (gate.rs:714-731) over the placed Q4_0 gate rows; same layout as gate_knn."""
        q = _host_f32(queries).reshape(-1, self.info.hidden)
        b, nl = q.shape[0], self.info.num_layers
        idx = np.empty((nl, b, top_k), np.uint32)
        sc = np.empty((nl, b, top_k), np.float32)
        check(lib().larql_cuda_vindex_gate_knn_q4(self.h, q.ctypes.data, b, top_k, idx.ctypes.data, sc.ctypes.data))
        return idx, sc

    def gate_knn_dev(self, queries, batch: int, top_k: int, out_idx, out_score, stream=None) -> None:
        """Device form: shard-local indices, [layers][batch][top_k]."""
        check(lib().larql_cuda_vindex_gate_knn_dev(self.h, _ptr(queries), batch, top_k, _ptr(out_idx),
                                                   _ptr(out_score), None if stream is None else C.c_void_p(int(stream))))

    def ffn(self, layer: int):
        """(gate, up, down) Weights of a layer from interleaved_q4k.bin (this rank's rows)."""
        g, u, d, df = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_int()
        check(lib().larql_cuda_vindex_ffn(self.h, layer, C.byref(g), C.byref(u), C.byref(d), C.byref(df)))
        H, I = self.info.hidden, self.info.intermediate
        # owned by the vindex: released by close(), not by Weight.release
        return (Weight(self.backend, g.value, FMT_Q4_K, I, H), Weight(self.backend, u.value, FMT_Q4_K, I, H),
                Weight(self.backend, d.value, df.value, H, I))

    def attn(self, layer: int):
        """[(handle, format)] of Q, K, V, O from attn_weights_q4k.bin (this rank's rows)."""
        hs = (C.c_uint64 * 4)()
        fs = (C.c_int * 4)()
        check(lib().larql_cuda_vindex_attn(self.h, layer, hs, fs))
        return [(hs[i], fs[i]) for i in range(4)]

    def close(self) -> None:
        if self.h:
            check(lib().larql_cuda_vindex_close(self.h))
            self.h = C.c_void_p()

