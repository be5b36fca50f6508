"""GGUF-144 Q4_K x f32 matvec on the GPU vs the CPU oracle.

Reference: crates/larql-models/src/quant/ggml.rs:228-273 (dequantize_q4_k, the decoder the GGUF loader applies,
crates/larql-models/src/loading/gguf.rs:191) followed by an f32 dot.  The reference's own GGUF-144 encoder
(q4_common.rs:248-314) does not round-trip through this decoder, so the inputs are random-byte super-blocks
(every 6-bit scale and min, every nibble, random finite f16 d / dmin, subnormals included), read as the decoder
reads them.  Tolerance: max |err| <= 1e-3 * ||y_ref||_inf.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_f16_bits, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")


def _random_gguf_q4k(seed, rows, hidden, subnormal=False):
    rng = np.random.default_rng(seed)
    nsb = rows * hidden // 256
    b = rng.integers(0, 256, size=(nsb, 144), dtype=np.uint8)
    d = random_f16_bits(rng, nsb, -14, 1)
    dm = random_f16_bits(rng, nsb, -14, 1)
    if subnormal:
        d[::3] = rng.integers(1, 0x3FF, d[::3].size).astype(np.uint16)
        dm[1::3] = rng.integers(1, 0x3FF, dm[1::3].size).astype(np.uint16)
    b[:, 0:2] = d.view(np.uint8).reshape(nsb, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(nsb, 2)
    return b.reshape(-1)


def _cmp(got, ref, what):
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"{what}: max err {err} > {bound}"


@pytest.mark.parametrize("rows,hidden", [(64, 256), (37, 4096), (130, 2560), (20, 14336), (1000, 4096), (9, 30720)])
def test_gguf_q4k_random_blocks(backend, rows, hidden):
    w = _random_gguf_q4k(seed_for("gguf-q4k", rows, hidden), rows, hidden)
    x = normal(seed_for("gguf-q4k-x", rows, hidden), hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    _cmp(got, O.q4k_gguf_matvec_f32(w, x, rows, hidden), f"gguf q4k {rows}x{hidden}")


def test_gguf_q4k_subnormal_scales_follow_half_rs(backend):
    rows, hidden = 48, 2048
    w = _random_gguf_q4k(7, rows, hidden, subnormal=True)
    x = normal(8, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    _cmp(got, O.q4k_gguf_matvec_f32(w, x, rows, hidden), "gguf q4k subnormal d / dmin")


@pytest.mark.parametrize("batch", [2, 3, 8])
def test_gguf_q4k_batch_rows(backend, batch):
    rows, hidden = 300, 4096
    w = _random_gguf_q4k(11, rows, hidden)
    x = normal(12, batch * hidden).reshape(batch, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    ref = O.q4k_gguf_matvec_f32(w, x, rows, hidden)
    for b in range(batch):
        _cmp(got[b], ref[b], f"gguf q4k batch row {b}")


def test_gguf_q4k_matches_dequantized_weights_on_normal_data(backend):
    """Weights drawn N(0, 0.02) and packed with per-sub-block scales and mins (an encoder consistent with the
    decoder), against the dot of the dequantized matrix."""
    rows, hidden = 256, 4096
    rng = np.random.default_rng(21)
    w = _random_gguf_q4k(22, rows, hidden)
    blk = w.reshape(-1, 144)
    blk[:, 0:2] = np.full((blk.shape[0],), np.float16(0.002)).view(np.uint8).reshape(-1, 2)
    blk[:, 2:4] = np.full((blk.shape[0],), np.float16(0.001)).view(np.uint8).reshape(-1, 2)
    x = rng.standard_normal(hidden, dtype=np.float32)
    deq = O.dequantize_q4_k_gguf(w, rows * hidden).reshape(rows, hidden).astype(np.float64)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    _cmp(got, (deq @ x.astype(np.float64)).astype(np.float32), "gguf q4k vs f64 dot of the dequantized rows")


def test_gguf_q4k_shape_rules(backend):
    w = _random_gguf_q4k(31, 8, 512)
    with pytest.raises(L.LarqlCudaError):
        backend.register_weight(w[:-1], L.FMT_Q4_K_GGUF, 8, 512)  # size mismatch
    # cols not a multiple of 1024 (so not on the warp-MMA kernel) and above 30720: not provided
    wt = backend.register_weight(_random_gguf_q4k(32, 4, 32000), L.FMT_Q4_K_GGUF, 4, 32000)
    try:
        with pytest.raises(L.LarqlCudaError):
            backend.matvec(wt, normal(33, 32000))
    finally:
        wt.release()


@pytest.mark.parametrize("batch", [1, 4])
def test_gguf_q4k_mma_and_dp4a_paths_agree(monkeypatch, batch):
    """The warp-MMA kernel (default for cols % 1024 == 0) and the dp4a pair kernel (LARQL_CUDA_Q4K_PATH=dp4a)
    on the same weights, both against the oracle."""
    rows, hidden = 500, 4096
    w = _random_gguf_q4k(41, rows, hidden)
    x = normal(42, batch * hidden).reshape(batch, hidden)
    ref = O.q4k_gguf_matvec_f32(w, x, rows, hidden)
    outs = {}
    for path in ("mma", "dp4a"):
        monkeypatch.setenv("LARQL_CUDA_Q4K_PATH", path)
        be = L.CudaBackend(0)
        try:
            wt = be.register_weight(w, L.FMT_Q4_K_GGUF, rows, hidden)
            kern = be.describe_matvec(wt, batch)
            outs[path] = be.matvec(wt, x)
            wt.release()
        finally:
            be.close()
        assert ("q4k_mma_kernel" in kern) == (path == "mma"), kern
    for path, got in outs.items():
        for b in range(batch):
            _cmp(got[b], ref[b], f"gguf q4k {path} batch row {b}")


# ── GGUF-144 Q4_K in llama.cpp's layout (LARQL_FMT_Q4_K_GGUF_LLAMA): the layout the reference's Metal q4kf kernels
# read (crates/larql-compute/src/metal/shaders/q4kf_qkv_proj.rs:136-220), IEEE f16 d / dmin ──

@pytest.mark.parametrize("rows,hidden,batch", [(64, 1024, 1), (37, 4096, 1), (1000, 4096, 1), (20, 14336, 1),
                                               (130, 2048, 4), (300, 4096, 8), (33, 3072, 3)])
def test_gguf_llama_layout_random_blocks(backend, rows, hidden, batch):
    """Random bytes (every scale / min / nibble, f16 d / dmin over many exponents, subnormals included) against
    the oracle's restatement of the llama.cpp layout, every batch row."""
    w = _random_gguf_q4k(seed_for("gguf-llama", rows, hidden), rows, hidden, subnormal=True)
    x = normal(seed_for("gguf-llama-x", rows, hidden, batch), batch * hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF_LLAMA, rows, hidden)
    try:
        got = backend.matvec(wt, x.reshape(batch, hidden)).reshape(batch, rows)
    finally:
        wt.release()
    for b in range(batch):
        _cmp(got[b], O.q4k_gguf_llama_matvec_f32(w, x[b * hidden:(b + 1) * hidden], rows, hidden),
             f"gguf llama {rows}x{hidden} batch row {b}")


@pytest.mark.skipif(O.metal_ref_lib() is None, reason="reference Metal shaders not built here")
@pytest.mark.parametrize("rows,hidden", [(37, 4096), (256, 2048)])
def test_gguf_llama_layout_against_the_reference_metal_kernel(backend, rows, hidden):
    """The CUDA matvec against the reference's own q4kf_proj shader code run on the CPU (normal f16 d / dmin: the
    kernels decode f16 with the hardware's half type)."""
    w = _random_gguf_q4k(seed_for("gguf-llama-m", rows, hidden), rows, hidden)
    x = normal(seed_for("gguf-llama-mx", rows, hidden), hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF_LLAMA, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    _cmp(got, O.metal_q4kf_proj(w, x, rows, hidden), f"gguf llama vs Metal q4kf_proj {rows}x{hidden}")


def test_gguf_llama_layout_needs_k_multiple_of_1024(backend):
    w = _random_gguf_q4k(3, 8, 768)
    wt = backend.register_weight(w, L.FMT_Q4_K_GGUF_LLAMA, 8, 768)
    try:
        with pytest.raises(L.LarqlCudaError) as ei:
            backend.matvec(wt, normal(4, 768))
        assert ei.value.status == L.ERR_UNSUPPORTED
    finally:
        wt.release()
