"""Pins the CPU oracle to the reference's own known answers (CPU only).

Each test names the reference test or function whose answer it reproduces
(paths relative to the larql-main workspace).
"""
import math
import os

import numpy as np
import pytest

import oracle as O
from conftest import lcg_synth, normal, seed_for

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_0_ref.npz")


def _cos(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))


# ── f16: crates/larql-models/src/quant/half.rs:105-126 ──

def test_f16_known_values():
    assert O.f16_to_f32(0x3C00) == 1.0
    assert O.f16_to_f32(0x4000) == 2.0
    assert abs(O.f16_to_f32(0x3800) - 0.5) < 1e-6


def test_f16_special_values():
    assert O.f16_to_f32(0) == 0.0
    z = O.f16_to_f32(0x8000)
    assert z == 0.0 and math.copysign(1.0, z) < 0
    assert math.isinf(O.f16_to_f32(0x7C00)) and O.f16_to_f32(0x7C00) > 0
    assert math.isinf(O.f16_to_f32(0xFC00)) and O.f16_to_f32(0xFC00) < 0
    assert math.isnan(O.f16_to_f32(0x7E00))


def test_f16_decoders_for_all_bit_patterns():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ieee = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(ieee)
    sub = ((bits & 0x7C00) == 0) & ((bits & 0x3FF) != 0)
    # q4k_matvec.rs:10-26 / q4_dot.c:9-35: exact IEEE
    got_ieee = np.array([O.f16_to_f32_ieee(int(b)) for b in bits], np.float32)
    assert np.array_equal(got_ieee[finite].view(np.uint32), ieee[finite].view(np.uint32))
    # half.rs:4-20: exact for normals/zeros/inf, subnormals at half their value
    got = O.decode_f16(bits)
    norm = finite & ~sub
    assert np.array_equal(got[norm].view(np.uint32), ieee[norm].view(np.uint32))
    assert np.array_equal(got[sub], ieee[sub] * np.float32(0.5))
    assert np.all(np.isnan(got[np.isnan(ieee)]))


def test_f16_round_trip():
    for v in [0.0, 1.0, -1.0, 0.5, 100.0, 2.71]:
        back = O.f16_to_f32(O.f32_to_f16_trunc(v))
        assert abs(v - back) < 0.01 * max(abs(v), 0.001)


def test_f32_to_f16_truncates():
    # 1 + 2^-11 + 2^-12 rounds up under RNE but the reference truncates the mantissa
    v = np.float32(1.0 + 2.0 ** -11 + 2.0 ** -12)
    assert O.f32_to_f16_trunc(float(v)) == 0x3C00
    assert O.f32_to_f16_trunc(1e-8) == 0  # below the normal range -> signed zero
    assert O.f32_to_f16_trunc(-1e-8) == 0x8000
    assert O.f32_to_f16_trunc(1e6) == 0x7C00


# ── ggml dequant known answers: crates/larql-models/src/quant/ggml.rs:370-460 ──

def test_q4_0_basic():
    block = np.array([0x00, 0x3C] + [0x12] * 16, np.uint8)
    r = O.dequantize_q4_0(block, 32)
    assert abs(r[0] - (-6.0)) < 0.01 and abs(r[1] - (-7.0)) < 0.01


def test_q4_0_zero_scale():
    block = np.array([0x00, 0x00] + [0xFF] * 16, np.uint8)
    assert np.all(O.dequantize_q4_0(block, 32) == 0.0)


def test_q4_0_two_blocks():
    data = np.array([0x00, 0x3C] + [0x88] * 16 + [0x00, 0x40] + [0x19] * 16, np.uint8)
    r = O.dequantize_q4_0(data, 64)
    assert abs(r[0]) < 0.01 and abs(r[32] - 2.0) < 0.01 and abs(r[33] - (-14.0)) < 0.01


def test_q8_0_basic():
    block = np.array([0x00, 0x38] + [2, 0xFE] * 16, np.uint8)
    r = O.dequantize_q8_0(block, 32)
    assert abs(r[0] - 1.0) < 0.01 and abs(r[1] - (-1.0)) < 0.01


def test_q8_0_zero_scale():
    block = np.array([0x00, 0x00] + [127] * 32, np.uint8)
    assert np.all(O.dequantize_q8_0(block, 32) == 0.0)


def test_q8_0_full_range():
    block = np.array([0x00, 0x3C, 127, 0x81] + [0] * 30, np.uint8)
    r = O.dequantize_q8_0(block, 32)
    assert abs(r[0] - 127.0) < 0.01 and abs(r[1] + 127.0) < 0.01 and abs(r[2]) < 0.01


# ── quantizers: crates/larql-compute/src/cpu/ops/q4_common.rs:444-544 ──

def test_q8_quantize_sizes_and_zero():
    x = (np.arange(64, dtype=np.float32) - 32.0) * np.float32(0.1)
    q, s = O.quantize_to_q8(x)
    assert q.size == 64 and s.size == 2 and np.all(s >= 0)
    q, s = O.quantize_to_q8(np.zeros(32, np.float32))
    assert np.all(q == 0) and s[0] == 0.0


def test_q4_output_size_and_zero_input():
    assert O.quantize_q4_0(np.ones(64, np.float32)).size == 2 * 18
    assert O.quantize_q4_0(np.ones(256, np.float32)).size == 8 * 18
    z = O.quantize_q4_0(np.zeros(32, np.float32))
    assert z[0] == 0 and z[1] == 0 and np.all(z[2:] == 0x88)


def test_q4_round_trip_accuracy():
    data = (np.arange(32, dtype=np.float32) - 16.0) * np.float32(0.5)
    back = O.dequantize_q4_0(O.quantize_q4_0(data), 32)
    assert np.max(np.abs(back - data)) < 2.0


def test_q4_matvec_uses_quantized_data():
    hidden, rows = 256, 64
    m = np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    q8, s = O.quantize_to_q8(x)
    y = O.q4_0_matvec_q8(O.quantize_q4_0(m), q8, s, rows, hidden)
    assert np.any(np.abs(y) > 0.01)


# ── Q4_0 kernel pins: crates/larql-compute/tests/test_q4_x86_correctness.rs:81-170 ──

def _deq_q8(q8, s):
    return (q8.astype(np.float32).reshape(-1, 32) * s[:, None]).reshape(-1)


def test_q4_matvec_matches_dequant_reference():
    rows, hidden = 4, 64
    m = lcg_synth(rows * hidden, 0xC0FFEE)
    x = lcg_synth(hidden, 0xBEEF)
    q4 = O.quantize_q4_0(m)
    q8, s = O.quantize_to_q8(x)
    got = O.q4_0_matvec_q8(q4, q8, s, rows, hidden)
    ref = O.dequantize_q4_0(q4, rows * hidden).reshape(rows, hidden) @ _deq_q8(q8, s)
    rel = np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-6)
    assert rel < 1e-4 and _cos(got, ref) > 0.9999


def test_q4_vecmat_matches_dequant_reference():
    inter, hidden = 8, 64
    act = lcg_synth(inter, 0xDEADBEEF)
    m = lcg_synth(inter * hidden, 0xFEEDFACE)
    q4 = O.quantize_q4_0(m)
    got = O.q4_0_vecmat(act, q4, inter, hidden)
    ref = act @ O.dequantize_q4_0(q4, inter * hidden).reshape(inter, hidden)
    rel = np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-6)
    assert rel < 1e-4 and _cos(got, ref) > 0.9999


def test_q4_matvec_vs_raw_f32_quant_noise():
    rows, hidden = 4, 64
    m = lcg_synth(rows * hidden, 0x1234)
    x = lcg_synth(hidden, 0x5678)
    q8, s = O.quantize_to_q8(x)
    got = O.q4_0_matvec_q8(O.quantize_q4_0(m), q8, s, rows, hidden)
    assert _cos(got, m.reshape(rows, hidden) @ x) > 0.99


# ── golden vectors produced by the reference's own q4_dot.c (tests/golden/make_golden.py) ──

@pytest.mark.parametrize("case", ["x86_matvec", "normal_matvec"])
def test_restated_q4_0_matvec_bit_exact_vs_reference_c(case):
    g = np.load(GOLDEN)
    rows, hidden = int(g[f"{case}.rows"]), int(g[f"{case}.hidden"])
    x = g[f"{case}.x"]
    q8, s = O.quantize_to_q8(x)
    assert np.array_equal(q8, g[f"{case}.q8"]) and np.array_equal(s.view(np.uint32), g[f"{case}.q8s"].view(np.uint32))
    got = O.q4_0_matvec_q8(g[f"{case}.q4"], q8, s, rows, hidden)
    assert np.array_equal(got.view(np.uint32), g[f"{case}.y"].view(np.uint32))


def test_restated_q4_0_quantizer_matches_golden_bytes():
    g = np.load(GOLDEN)
    rows, hidden = int(g["x86_matvec.rows"]), int(g["x86_matvec.hidden"])
    assert np.array_equal(O.quantize_q4_0(lcg_synth(rows * hidden, 0xC0FFEE)), g["x86_matvec.q4"])
    assert np.array_equal(O.quantize_q4_0(normal(11, 96 * 1024, 0.02)), g["normal_matvec.q4"])


def test_restated_q4_0_vecmat_bit_exact_vs_reference_c():
    g = np.load(GOLDEN)
    inter, hidden = int(g["x86_vecmat.rows"]), int(g["x86_vecmat.hidden"])
    got = O.q4_0_vecmat(g["x86_vecmat.x"], g["x86_vecmat.q4"], inter, hidden)
    assert np.array_equal(got.view(np.uint32), g["x86_vecmat.y"].view(np.uint32))


@pytest.mark.skipif(O.ref_lib() is None, reason="reference q4_dot.c not built here")
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_restated_q4_0_vs_live_reference_random_bytes(seed):
    rng = np.random.default_rng(seed)
    rows, hidden = 33, 32 * 37
    q4 = rng.integers(0, 256, rows * hidden // 32 * 18, dtype=np.uint8).reshape(-1, 18)
    q4[:, 0:2] = np.float16(rng.uniform(-2, 2, q4.shape[0])).view(np.uint8).reshape(-1, 2)
    q4 = q4.reshape(-1)
    q8, s = O.quantize_to_q8(rng.standard_normal(hidden, dtype=np.float32))
    a = O.q4_0_matvec_q8(q4, q8, s, rows, hidden)
    b = O.ref_q4_0_matvec_c(q4, q8, s, rows, hidden)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ── Q8 compute layout: crates/larql-compute/src/cpu/ops/q8_matvec.rs:62-108 ──

def test_q8_vs_f32_high_cosine():
    hidden, rows = 256, 32
    w = np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    wq, ws = O.quantize_weights_q8(w, rows, hidden)
    xq, xs = O.quantize_to_q8(x)
    y = O.q8_matvec(wq, ws, xq, xs, rows, hidden)
    assert _cos(y, w.reshape(rows, hidden) @ x) > 0.999


# ── Q4_K (148 B): layout of q4_common.rs:96-103 as read by q4k_matvec.rs:43-81 ──

def _handmade_q4k_block():
    """d = 1.0, dmin = 0.5, sc_j = j + 1, mn_j = j, nibble byte i of sub-block j = (i, 15 - i)."""
    b = np.zeros(148, np.uint8)
    b[0:2] = [0x00, 0x3C]
    b[2:4] = [0x00, 0x38]
    for j in range(8):
        b[4 + j] = j + 1
    for j in range(4):
        b[16 + j] = (j & 0xF) | ((j + 4) << 4)
    for j in range(8):
        for i in range(16):
            b[20 + 16 * j + i] = (i & 0xF) | ((15 - i) << 4)
    expect = np.empty(256, np.float32)
    for j in range(8):
        for i in range(16):
            expect[32 * j + 2 * i] = 1.0 * (j + 1) * i - 0.5 * j
            expect[32 * j + 2 * i + 1] = 1.0 * (j + 1) * (15 - i) - 0.5 * j
    return b, expect


def test_q4k_handmade_block_dequant_and_matvec():
    b, expect = _handmade_q4k_block()
    assert np.array_equal(O.dequantize_q4_k(b, 256), expect)
    x = np.ones(256, np.float32)
    assert O.q4k_matvec(b, x, 1, 256)[0] == np.float32(expect.sum())


def test_q4k_produces_nonzero():  # q4k_matvec.rs:94-103
    hidden, rows = 256, 4
    m = np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    assert np.any(np.abs(O.q4k_matvec(O.quantize_q4_k(m), x, rows, hidden)) > 0.001)


def test_q4k_quantizer_layout_invariants():
    w = normal(0, 64 * 1024, 0.02)
    q = O.quantize_q4_k(w).reshape(-1, 148)
    assert q.shape[0] == 64 * 4
    assert np.all(q[:, 12:16] == 0)           # bytes 12..15 unused
    assert np.all(q[:, 4:12] <= 63)           # 6-bit scales
    # the reference's nibble step is the whole sub-block range: N(0, 0.02) data
    # only ever uses nibbles 0 and 1 (q4_common.rs:157-165)
    nib = np.concatenate([q[:, 20:] & 15, q[:, 20:] >> 4]).ravel()
    assert set(np.unique(nib).tolist()) <= {0, 1}


def test_q4k_matvec_matches_dequantized_dot():
    rows, hidden = 16, 1024
    w = normal(5, rows * hidden, 0.02)
    x = normal(6, hidden)
    q = O.quantize_q4_k(w)
    y = O.q4k_matvec(q, x, rows, hidden)
    ref = O.dequantize_q4_k(q, rows * hidden).reshape(rows, hidden).astype(np.float64) @ x.astype(np.float64)
    assert np.max(np.abs(y - ref)) < 1e-5 * max(1.0, np.max(np.abs(ref)))


def test_q6k_produces_nonzero():  # q6k_matvec.rs:94-103
    hidden, rows = 256, 4
    m = np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    assert np.any(np.abs(O.q6k_matvec(O.quantize_q6_k(m), x, rows, hidden)) > 0.001)


# ── gate KNN known answers: crates/larql-vindex/tests/test_vindex.rs:27-61,134-190 ──

def _vindex_gates():
    g0 = np.zeros((3, 4), np.float32)
    g0[0, 0] = g0[1, 1] = g0[2, 2] = 1.0
    g1 = np.zeros((3, 4), np.float32)
    g1[0, 3] = 1.0
    g1[1, 0] = g1[1, 1] = 0.5
    g1[2, 2] = -1.0
    return [g0.astype(np.float16).view(np.uint16), g1.astype(np.float16).view(np.uint16)]


def test_gate_knn_finds_best_match():
    g0, _ = _vindex_gates()
    (res,), _ = O.gate_topk_f16(g0, np.array([1, 0, 0, 0], np.float32), 3, 4, 1)
    assert res[0].tolist() == [0] and abs(res[1][0] - 1.0) < 0.01


def test_gate_knn_top_k_ordering():
    g0, _ = _vindex_gates()
    (res,), _ = O.gate_topk_f16(g0, np.array([0.8, 0.6, 0, 0], np.float32), 3, 4, 3)
    assert len(res[0]) == 3 and res[0][0] == 0 and res[0][1] == 1


def test_gate_walk_layer1_ranks_by_absolute_score():
    _, g1 = _vindex_gates()
    (res,), _ = O.gate_topk_f16(g1, np.array([1, 0, 0, 0], np.float32), 3, 4, 1)
    assert res[0].tolist() == [1]  # dim 0 contributes 0.5 (test_vindex.rs:188)
    (res,), _ = O.gate_topk_f16(g1, np.array([0, 0, 1, 0], np.float32), 3, 4, 1)
    assert res[0].tolist() == [2] and res[1][0] == -1.0  # |score| ranking (gate.rs:307-316)


def test_top_k_edge_cases():
    idx, sc = O.top_k_abs(np.array([], np.float32), 5)
    assert idx.size == 0
    idx, sc = O.top_k_abs(np.array([0.5, -3.0, 2.0], np.float32), 10)  # k > n returns n
    assert idx.tolist() == [1, 2, 0]
    idx, sc = O.top_k_abs(np.array([1.0, 2.0], np.float32), 0)
    assert idx.size == 0


def test_top_k_signed_follows_lm_head_selection():
    """walk.rs:566-577: k = min(top_k, n); 0 < k < n keeps the k largest logits, then sorts descending; top_k 0
    or >= n drops nothing (every logit, sorted); a NaN logit panics there (ValueError here)."""
    v = np.array([0.5, -3.0, 2.0, 2.0, -np.inf, np.inf, 0.0], np.float32)
    idx, sc = O.top_k_signed(v, 3)
    assert idx.tolist() == [5, 2, 3] and sc.tolist() == [np.inf, 2.0, 2.0]  # signed, ties by lower id
    idx, _ = O.top_k_signed(v, 0)
    assert idx.tolist() == [5, 2, 3, 0, 6, 1, 4]
    assert O.top_k_signed(v, 100)[0].tolist() == [5, 2, 3, 0, 6, 1, 4]
    assert O.top_k_signed(np.array([], np.float32), 4)[0].size == 0
    with pytest.raises(ValueError):
        O.top_k_signed(np.array([1.0, np.nan], np.float32), 1)
    rng = np.random.default_rng(5)
    r = rng.standard_normal(10000).astype(np.float32)
    idx, sc = O.top_k_signed(r, 25)
    assert idx.tolist() == np.argsort(-r.astype(np.float64), kind="stable")[:25].tolist()
    assert np.array_equal(sc, r[idx])


def test_lm_head_knn_composite_uses_q8_query():
    """lm_head_knn_backend quantizes the query to Q8 before the Q4_0 matvec (walk.rs:562-565)."""
    vocab, hidden = 300, 256
    w = O.quantize_q4_0(normal(31, vocab * hidden, 0.02))
    q = normal(32, hidden)
    ids, vals, logits = O.lm_head_knn(w, q, vocab, hidden, 5)
    q8, s8 = O.quantize_to_q8(q)
    assert np.array_equal(logits, O.q4_0_matvec_q8(w, q8, s8, vocab, hidden))
    assert ids.tolist() == np.argsort(-logits.astype(np.float64), kind="stable")[:5].tolist()


def _gguf_q4k_block(d, dmin, sc, mn, q):
    """One 144-byte GGUF Q4_K super-block packed so that ggml.rs:243-252 (get_scale_min_k4) reads back the
    given 6-bit sc / mn, and ggml.rs:255-270 reads q[32 j + i] (i < 16) from the low nibble of byte 16 j + i
    and q[32 j + 16 + i] from its high nibble."""
    b = np.zeros(144, np.uint8)
    b[0:2] = np.array([d], np.float16).view(np.uint8)
    b[2:4] = np.array([dmin], np.float16).view(np.uint8)
    s = np.zeros(12, np.int64)
    for j in range(4):
        s[j] |= sc[j] & 0x3F
        s[j + 4] |= mn[j] & 0x3F
    for j in range(4, 8):
        s[j + 4] |= (sc[j] & 0x0F) | ((mn[j] & 0x0F) << 4)
        s[j - 4] |= (sc[j] >> 4) << 6
        s[j] |= (mn[j] >> 4) << 6
    b[4:16] = s.astype(np.uint8)
    for j in range(8):
        for i in range(16):
            b[16 + 16 * j + i] = q[32 * j + i] | (q[32 * j + 16 + i] << 4)
    return b


def test_gguf_q4k_dequant_known_answer():
    """ggml.rs:228-273 restated: every 6-bit scale and min (the j >= 4 ones carry their top two bits in bytes
    0..7) and the 16-low-then-16-high nibble order of each sub-block."""
    rng = np.random.default_rng(3)
    sc = [1, 63, 17, 40, 33, 62, 5, 48]
    mn = [0, 9, 63, 21, 50, 3, 63, 16]
    q = rng.integers(0, 16, 256)
    blk = _gguf_q4k_block(0.5, 0.25, sc, mn, q)
    got = O.dequantize_q4_k_gguf(blk, 256)
    want = np.array([np.float32(0.5) * np.float32(sc[e // 32]) * np.float32(q[e]) - np.float32(0.25) * np.float32(mn[e // 32])
                     for e in range(256)], np.float32)
    assert np.array_equal(got, want)
    # d = dmin = a subnormal f16: half.rs decodes it at half its IEEE value
    sub = np.float16(np.float32(2.0) ** -20)
    got = O.dequantize_q4_k_gguf(_gguf_q4k_block(sub, sub, [1] * 8, [1] * 8, np.full(256, 3)), 256)
    h = np.float32(sub) * np.float32(0.5)
    assert np.all(got == h * 3 - h)


def _gguf_q4k_decode_numpy(data: np.ndarray, n: int) -> np.ndarray:
    """A second, vectorised restatement of ggml.rs:228-273, written independently of the C oracle."""
    b = data.reshape(-1, 144)[: n // 256]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dm = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    sub = lambda h, bits: np.where((bits & 0x7C00) == 0, h * np.float32(0.5), h)  # half.rs subnormals
    d = sub(d, b[:, 0].astype(np.uint16) | (b[:, 1].astype(np.uint16) << 8))
    dm = sub(dm, b[:, 2].astype(np.uint16) | (b[:, 3].astype(np.uint16) << 8))
    s = b[:, 4:16].astype(np.int64)
    sc = np.empty((b.shape[0], 8), np.int64)
    mn = np.empty((b.shape[0], 8), np.int64)
    sc[:, :4], mn[:, :4] = s[:, 0:4] & 63, s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    q = b[:, 16:144].reshape(-1, 8, 16).astype(np.int64)
    nib = np.concatenate([q & 15, q >> 4], axis=2).astype(np.float32)  # [sb][j][32]
    sv = (d[:, None] * sc.astype(np.float32))[:, :, None]
    mv = (dm[:, None] * mn.astype(np.float32))[:, :, None]
    return (sv * nib - mv).reshape(-1)


def test_gguf_q4k_dequant_random_blocks_two_restatements():
    """The C oracle and an independent numpy restatement of ggml.rs:228-273 agree bit for bit on random-byte
    super-blocks (every scale / min bit pattern, random f16 d / dmin with subnormals)."""
    rng = np.random.default_rng(17)
    nsb = 400
    b = rng.integers(0, 256, size=(nsb, 144), dtype=np.uint8)
    h = (rng.integers(0, 0x7C00, size=(nsb, 2)) | (rng.integers(0, 2, size=(nsb, 2)) << 15)).astype(np.uint16)
    b[:, 0:4] = h.view(np.uint8).reshape(nsb, 4)
    got = O.dequantize_q4_k_gguf(b.reshape(-1), nsb * 256)
    want = _gguf_q4k_decode_numpy(b.reshape(-1), nsb * 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ── a second, independent restatement of the LARQL Q4_K (148 B) and Q6_K (210 B) matvecs ──
# Written from q4k_matvec.rs:31-87 and q6k_matvec.rs:31-87 directly, vectorised over rows with numpy and
# sharing no code with oracle/larql_oracle.c.  numpy float32 arithmetic rounds every operation separately
# (no fused multiply-add), as rustc emits the reference's expressions, and numpy's f16 -> f32 conversion is
# the exact IEEE decode those two files implement.  Agreement bit for bit on random bytes pins the C oracle
# for the headline format to a second reading of the reference.

def _f16_le(b2: np.ndarray) -> np.ndarray:
    """[..., 2] little-endian f16 bytes -> f32 (exact IEEE decode, subnormals included)."""
    return np.ascontiguousarray(b2).view(np.float16)[..., 0].astype(np.float32)


def _sequential_f32_sum(t: np.ndarray) -> np.ndarray:
    """acc += t[:, e] for e in element order, in f32 (q4k_matvec.rs:79-80, q6k_matvec.rs:78-79)."""
    acc = np.zeros(t.shape[0], np.float32)
    for e in range(t.shape[1]):
        acc = acc + t[:, e]
    return acc


def _q4k_matvec_numpy(data: np.ndarray, x: np.ndarray, rows: int, hidden: int) -> np.ndarray:
    nsb = hidden // 256
    b = data.reshape(rows, nsb, 148)
    d, dmin = _f16_le(b[..., 0:2]), _f16_le(b[..., 2:4])                       # [rows, nsb]
    scales = (b[..., 4:12] & 0x3F).astype(np.float32)                          # j 0..7 from bytes 4..11
    mins = np.concatenate([b[..., 16:20] & 0x0F, b[..., 16:20] >> 4], axis=-1).astype(np.float32)
    q = b[..., 20:148].reshape(rows, nsb, 8, 16)
    nib = np.stack([q & 0x0F, q >> 4], axis=-1).reshape(rows, nsb, 8, 32).astype(np.float32)  # lo = 2i, hi = 2i+1
    sc = (d[..., None] * scales)[..., None]                                    # f32 d * scale_j
    mn = (dmin[..., None] * mins)[..., None]                                   # f32 dmin * min_j
    w = (sc * nib - mn).reshape(rows, hidden)                                  # (sc * q) - mn, each rounded
    return _sequential_f32_sum(w * x[None, :])


def _q6k_matvec_numpy(data: np.ndarray, x: np.ndarray, rows: int, hidden: int) -> np.ndarray:
    nsb = hidden // 256
    b = data.reshape(rows, nsb, 210)
    ql, qh = b[..., 0:128], b[..., 128:192]
    scales = np.ascontiguousarray(b[..., 192:208]).view(np.int8).astype(np.float32)   # [rows, nsb, 16]
    d = _f16_le(b[..., 208:210])
    e = np.arange(256)
    lo = np.where(e % 2 == 0, ql[..., e // 2] & 0x0F, ql[..., e // 2] >> 4).astype(np.float32)
    hi = ((qh[..., e // 4] >> ((e % 4) * 2)) & 0x03).astype(np.float32)
    sc = d[..., None] * scales                                                 # f32 d * (scale as i8)
    val = sc[..., e // 16] * ((lo + hi * np.float32(16.0)) - np.float32(32.0))
    return _sequential_f32_sum(val.reshape(rows, hidden) * x[None, :])


def _random_f16_scale_bytes(rng, n: int) -> np.ndarray:
    """n finite f16 values, every exponent including subnormals (exponent field 0), random sign; -> [n, 2] bytes."""
    h = (rng.integers(0, 0x7C00, size=n) | (rng.integers(0, 2, size=n) << 15)).astype(np.uint16)
    h[::7] = (rng.integers(1, 0x400, size=h[::7].size) | (rng.integers(0, 2, size=h[::7].size) << 15)).astype(np.uint16)
    return h.view(np.uint8).reshape(n, 2)


@pytest.mark.parametrize("rows,hidden,seed", [(48, 1024, 1), (9, 4096, 2), (130, 256, 3)])
def test_q4k_matvec_two_restatements_random_bytes(rows, hidden, seed):
    """C oracle vs the independent numpy restatement of q4k_matvec.rs:31-87, bit for bit: random bytes in every
    field (all nibbles, every 6-bit scale with random top bits, random unused bytes 12..15), f16 d / dmin over
    every exponent including subnormals, x ~ N(0, 1) with a spread of magnitudes."""
    rng = np.random.default_rng(seed)
    nsb = rows * hidden // 256
    b = rng.integers(0, 256, size=(nsb, 148), dtype=np.uint8)
    b[:, 0:2] = _random_f16_scale_bytes(rng, nsb)
    b[:, 2:4] = _random_f16_scale_bytes(rng, nsb)
    x = (rng.standard_normal(hidden) * np.exp2(rng.integers(-8, 8, hidden))).astype(np.float32)
    got = O.q4k_matvec(b.reshape(-1), x, rows, hidden)
    want = _q4k_matvec_numpy(b.reshape(-1), x, rows, hidden)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q4k_matvec_two_restatements_quantized():
    """The same agreement on weights from the reference quantizer (q4_common.rs:104-170)."""
    rows, hidden = 64, 2048
    w = O.quantize_q4_k(normal(41, rows * hidden, 0.02))
    x = normal(42, hidden)
    got = O.q4k_matvec(w, x, rows, hidden)
    assert np.array_equal(got.view(np.uint32), _q4k_matvec_numpy(w, x, rows, hidden).view(np.uint32))


@pytest.mark.parametrize("rows,hidden,seed", [(48, 1024, 4), (9, 4096, 5), (130, 256, 6)])
def test_q6k_matvec_two_restatements_random_bytes(rows, hidden, seed):
    """C oracle vs the independent numpy restatement of q6k_matvec.rs:31-87, bit for bit: random low / high
    bit planes, every int8 scale, f16 d over every exponent including subnormals."""
    rng = np.random.default_rng(seed)
    nsb = rows * hidden // 256
    b = rng.integers(0, 256, size=(nsb, 210), dtype=np.uint8)
    b[:, 208:210] = _random_f16_scale_bytes(rng, nsb)
    x = (rng.standard_normal(hidden) * np.exp2(rng.integers(-8, 8, hidden))).astype(np.float32)
    got = O.q6k_matvec(b.reshape(-1), x, rows, hidden)
    want = _q6k_matvec_numpy(b.reshape(-1), x, rows, hidden)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q6k_matvec_two_restatements_quantized():
    """The same agreement on weights from the reference quantizer (q4_common.rs:179-239)."""
    rows, hidden = 64, 2048
    w = O.quantize_q6_k(normal(43, rows * hidden, 0.02))
    x = normal(44, hidden)
    got = O.q6k_matvec(w, x, rows, hidden)
    assert np.array_equal(got.view(np.uint32), _q6k_matvec_numpy(w, x, rows, hidden).view(np.uint32))


def test_gate_scores_many_matches_per_query_loop():
    """oracle.gate_scores_f16_many (one f64 BLAS product) against the per-query C loop (orc_gate_scores_f16):
    the same f64 math up to summation order, on rows with half.rs subnormals."""
    nf, hidden, b = 300, 256, 6
    rng = np.random.default_rng(8)
    g = (rng.standard_normal(nf * hidden) * 0.02).astype(np.float16).view(np.uint16).copy()
    g[::53] = rng.integers(1, 0x400, size=g[::53].size).astype(np.uint16)
    q = rng.standard_normal((b, hidden)).astype(np.float32)
    a = O.gate_scores_f16(g, q, nf, hidden)
    m = O.gate_scores_f16_many(g, q, nf, hidden)
    np.testing.assert_allclose(m, a, rtol=1e-6, atol=1e-7)


# ── the reference's own Metal shaders, compiled for the CPU (oracle/Makefile target `metal`) ──
# crates/larql-compute/src/metal/shaders/q4k_matvec.rs and q6k_matvec.rs, extracted verbatim and run lane by lane:
# an execution of reference code for the Q4_K / Q6_K layouts.  The shaders sum in another order than the CPU
# matvecs (per sub-block, then across the 32 lanes), so agreement is to f32 rounding of the row's |terms|.

_metal = pytest.mark.skipif(O.metal_ref_lib() is None, reason="reference Metal shaders not built here")


def _q6k_abs_dequant(data, rows, hidden):
    nsb = hidden // 256
    b = data.reshape(rows, nsb, 210)
    ql, qh = b[..., 0:128], b[..., 128:192]
    scales = np.ascontiguousarray(b[..., 192:208]).view(np.int8).astype(np.float64)
    d = _f16_le(b[..., 208:210]).astype(np.float64)
    e = np.arange(256)
    lo = np.where(e % 2 == 0, ql[..., e // 2] & 0x0F, ql[..., e // 2] >> 4).astype(np.float64)
    hi = ((qh[..., e // 4] >> ((e % 4) * 2)) & 0x03).astype(np.float64)
    return np.abs((d[..., None] * scales)[..., e // 16] * (lo + 16 * hi - 32)).reshape(rows, hidden)


def _close_to_rounding(got, want, absterms, what):
    bound = 1e-5 * np.maximum(absterms, 1e-30)
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= bound), f"{what}: worst err {err.max()} (bound {bound[np.argmax(err - bound)]})"


@_metal
@pytest.mark.parametrize("rows,hidden,kind", [(37, 2048, "quantized"), (16, 4096, "random"), (130, 256, "random"),
                                              (9, 14336, "quantized")])
def test_q4k_oracle_matches_reference_metal_shader(rows, hidden, kind):
    rng = np.random.default_rng(seed_for("mq4k", rows, hidden))
    if kind == "quantized":
        w = O.quantize_q4_k(normal(seed_for("mq4kw", rows), rows * hidden, 0.02))
    else:  # every nibble / scale / min, random finite f16 d and dmin (subnormals included)
        nsb = rows * hidden // 256
        b = rng.integers(0, 256, size=(nsb, 148), dtype=np.uint8)
        b[:, 0:2] = _random_f16_scale_bytes(rng, nsb)
        b[:, 2:4] = _random_f16_scale_bytes(rng, nsb)
        w = b.reshape(-1)
    x = rng.standard_normal(hidden).astype(np.float32)
    absterms = np.abs(O.dequantize_q4_k(w, rows * hidden).reshape(rows, hidden).astype(np.float64)) @ np.abs(x)
    _close_to_rounding(O.q4k_matvec(w, x, rows, hidden), O.metal_q4k_matvec(w, x, rows, hidden), absterms,
                       f"Q4_K {kind} {rows}x{hidden}")


@_metal
@pytest.mark.parametrize("rows,hidden,kind", [(37, 2048, "quantized"), (16, 4096, "random"), (5, 256, "random")])
def test_q6k_oracle_matches_reference_metal_shader(rows, hidden, kind):
    """Random bytes use normal f16 d only: the shaders' decode_f16_metal (crates/larql-compute/src/metal/shaders/
    common.rs) flushes subnormal d to zero where the CPU q6k_matvec.rs decodes it (finding F16)."""
    rng = np.random.default_rng(seed_for("mq6k", rows, hidden))
    if kind == "quantized":
        w = O.quantize_q6_k(normal(seed_for("mq6kw", rows), rows * hidden, 0.02))
    else:
        nsb = rows * hidden // 256
        b = rng.integers(0, 256, size=(nsb, 210), dtype=np.uint8)
        h = (rng.integers(0x0400, 0x7C00, size=nsb) | (rng.integers(0, 2, size=nsb) << 15)).astype(np.uint16)
        b[:, 208:210] = h.view(np.uint8).reshape(nsb, 2)
        w = b.reshape(-1)
    x = rng.standard_normal(hidden).astype(np.float32)
    absterms = _q6k_abs_dequant(w, rows, hidden) @ np.abs(x).astype(np.float64)
    _close_to_rounding(O.q6k_matvec(w, x, rows, hidden), O.metal_q6k_matvec(w, x, rows, hidden), absterms,
                       f"Q6_K {kind} {rows}x{hidden}")


def _gguf144_llama_layout_dequant(data, n):
    """GGUF-144 Q4_K as llama.cpp lays it out: quants in four 32-byte chunks, chunk c holding sub-block 2c in its
    low nibbles and 2c+1 in its high ones; 6-bit scales / mins packed as get_scale_min_k4."""
    b = data.reshape(-1, 144)[: n // 256]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dm = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    s = b[:, 4:16].astype(np.int64)
    sc = np.empty((b.shape[0], 8), np.int64)
    mn = np.empty((b.shape[0], 8), np.int64)
    sc[:, :4], mn[:, :4] = s[:, 0:4] & 63, s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    q = b[:, 16:144].reshape(-1, 4, 32).astype(np.int64)
    nib = np.stack([q & 15, q >> 4], axis=2).reshape(-1, 8, 32).astype(np.float32)  # sub-block j = (chunk j//2, j&1)
    sv = (d[:, None] * sc.astype(np.float32))[:, :, None]      # f32 d * sc_j
    mv = (dm[:, None] * mn.astype(np.float32))[:, :, None]     # f32 dmin * mn_j
    return (sv * nib - mv).reshape(-1)


@_metal
def test_gguf144_reference_paths_disagree_by_execution():
    """Finding F6 checked by running reference code: the reference's Metal GGUF Q4_K kernel (q4kf_proj, llama.cpp's
    mul_mv_q4_K) reads the 144-byte blocks in llama.cpp's layout, while its CPU GGUF loader's dequantize_q4_k
    (crates/larql-models/src/quant/ggml.rs:228-273, the oracle here and the layout LARQL_FMT_Q4_K_GGUF follows)
    reads the quants as 16-byte runs per sub-block.  Random bytes with normal positive f16 d / dmin."""
    rng = np.random.default_rng(9)
    n, k = 8, 1024
    nsb = n * k // 256
    b = rng.integers(0, 256, size=(nsb, 144), dtype=np.uint8)
    b[:, 0:4] = rng.integers(0x2000, 0x3C00, size=(nsb, 2)).astype(np.uint16).view(np.uint8).reshape(nsb, 4)
    w = b.reshape(-1)
    x = rng.standard_normal(k).astype(np.float32)
    metal = O.metal_q4kf_proj(w, x, n, k)
    llama = _gguf144_llama_layout_dequant(w, n * k).reshape(n, k).astype(np.float64) @ x.astype(np.float64)
    absterms = np.abs(_gguf144_llama_layout_dequant(w, n * k).reshape(n, k).astype(np.float64)) @ np.abs(x)
    _close_to_rounding(metal, llama, absterms, "Metal q4kf_proj vs llama.cpp layout")
    cpu = O.q4k_gguf_matvec_f32(w, x, n, k)
    assert np.max(np.abs(cpu - metal)) > 0.05 * np.max(np.abs(metal))  # the two reference paths disagree


def test_gguf144_llama_layout_decoder_two_restatements():
    """The C decoder of the llama.cpp layout against the numpy one above, bit for bit, on random bytes (every
    scale / min bit pattern, normal and subnormal f16 d / dmin; IEEE decoding)."""
    rng = np.random.default_rng(21)
    nsb = 300
    b = rng.integers(0, 256, size=(nsb, 144), dtype=np.uint8)
    b[:, 0:2] = _random_f16_scale_bytes(rng, nsb)
    b[:, 2:4] = _random_f16_scale_bytes(rng, nsb)
    got = O.dequantize_q4_k_gguf_llama(b.reshape(-1), nsb * 256)
    want = _gguf144_llama_layout_dequant(b.reshape(-1), nsb * 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@_metal
@pytest.mark.parametrize("rows,hidden", [(37, 2048), (4, 4096), (9, 1024)])
def test_gguf144_llama_oracle_matches_reference_metal_shader(rows, hidden):
    """orc_q4k_gguf_llama_matvec_f32 against the reference's own q4kf_proj shader run on the CPU, random bytes
    (normal f16 d / dmin), to f32 rounding of the row's Σ|w·x|."""
    rng = np.random.default_rng(seed_for("mq4kf", rows, hidden))
    nsb = rows * hidden // 256
    b = rng.integers(0, 256, size=(nsb, 144), dtype=np.uint8)
    h = (rng.integers(0x0400, 0x7C00, size=(nsb, 2)) | (rng.integers(0, 2, size=(nsb, 2)) << 15)).astype(np.uint16)
    b[:, 0:4] = h.view(np.uint8).reshape(nsb, 4)
    w = b.reshape(-1)
    x = rng.standard_normal(hidden).astype(np.float32)
    deq = O.dequantize_q4_k_gguf_llama(w, rows * hidden).reshape(rows, hidden).astype(np.float64)
    _close_to_rounding(O.q4k_gguf_llama_matvec_f32(w, x, rows, hidden), O.metal_q4kf_proj(w, x, rows, hidden),
                       np.abs(deq) @ np.abs(x), f"GGUF-144 llama layout {rows}x{hidden}")
