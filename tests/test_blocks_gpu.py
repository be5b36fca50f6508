"""Q4_0 / Q8_0 / Q8 (compute layout) matvecs on the GPU vs the CPU oracle.

References: Q4_0 x Q8 = crates/larql-compute/csrc/q4_dot.c:169-199 (ComputeBackend::q4_matvec);
Q4_0 x f32 and GGUF Q8_0 x f32 = crates/larql-models/src/quant/ggml.rs dequantize (half.rs f16 decode) + dot;
Q8 compute layout = crates/larql-compute/src/cpu/ops/q8_matvec.rs:36-57 against quantize_to_q8(x).
Tolerance: max |err| <= 1e-3 * ||y_ref||_inf.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_f16_bits, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q4_0_ref.npz")
SHAPES = [(64, 512), (37, 1024), (96, 4096), (20, 14336), (130, 2560), (7, 64), (1000, 4096)]


def _random_q4_0(seed, rows, hidden, subnormal=False):
    rng = np.random.default_rng(seed)
    nb = rows * hidden // 32
    b = rng.integers(0, 256, size=(nb, 18), dtype=np.uint8)
    d = random_f16_bits(rng, nb, -12, 1)
    if subnormal:
        d[::3] = rng.integers(1, 0x3FF, d[::3].size).astype(np.uint16)
    b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def _random_q8_0(seed, rows, hidden, subnormal=False):
    rng = np.random.default_rng(seed)
    nb = rows * hidden // 32
    b = rng.integers(0, 256, size=(nb, 34), dtype=np.uint8)
    d = random_f16_bits(rng, nb, -12, 1)
    if subnormal:
        d[::3] = rng.integers(1, 0x3FF, d[::3].size).astype(np.uint16)
    b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    return b.reshape(-1)


def _cmp(got, ref, what):
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"{what}: max err {err} > {bound}"


@pytest.mark.parametrize("rows,hidden", SHAPES)
def test_q4_0_f32x_reference_quantized(backend, rows, hidden):
    w = O.quantize_q4_0(normal(seed_for("q40", rows, hidden), rows * hidden, 0.02))
    x = normal(seed_for("q40x", rows, hidden), hidden)
    wt = backend.register_weight(w, L.FMT_Q4_0, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    _cmp(got, O.q4_0_matvec_f32(w, x, rows, hidden), "q4_0 f32x")


@pytest.mark.parametrize("subnormal", [False, True])
def test_q4_0_f32x_random_bytes(backend, subnormal):
    rows, hidden = 77, 4096
    w = _random_q4_0(seed_for("q40r", subnormal), rows, hidden, subnormal)
    x = normal(seed_for("q40rx", subnormal), 3 * hidden).reshape(3, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_0, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    ref = O.q4_0_matvec_f32(w, x, rows, hidden)
    for b in range(3):
        _cmp(got[b], ref[b], f"q4_0 f32x random b{b}")


@pytest.mark.parametrize("rows,hidden", SHAPES)
def test_q4_0_q8x_trait_mirror_vs_reference_c(backend, rows, hidden):
    """ComputeBackend::q4_matvec with pre-quantized Q8 x, checked against q4_dot.c's q4_0_matvec_c semantics."""
    w = O.quantize_q4_0(normal(seed_for("q4q8", rows, hidden), rows * hidden, 0.02))
    q8, s8 = O.quantize_to_q8(normal(seed_for("q4q8x", rows, hidden), hidden))
    got = backend.q4_matvec(w, q8, s8, rows, hidden)
    _cmp(got, O.q4_0_matvec_q8(w, q8, s8, rows, hidden), "q4_0 q8x")


def test_q4_0_q8x_golden_from_reference_kernel(backend):
    g = np.load(GOLDEN)
    for case in ["x86_matvec", "normal_matvec"]:
        rows, hidden = int(g[f"{case}.rows"]), int(g[f"{case}.hidden"])
        got = backend.q4_matvec(g[f"{case}.q4"], g[f"{case}.q8"], g[f"{case}.q8s"], rows, hidden)
        _cmp(got, g[f"{case}.y"], case)


def test_q4_0_q8x_subnormal_scales_ieee(backend):
    """q4_dot.c decodes the f16 scale exactly (IEEE), unlike half.rs."""
    rows, hidden = 50, 2048
    w = _random_q4_0(5, rows, hidden, subnormal=True)
    q8, s8 = O.quantize_to_q8(normal(6, hidden))
    _cmp(backend.q4_matvec(w, q8, s8, rows, hidden), O.q4_0_matvec_q8(w, q8, s8, rows, hidden), "q4_0 q8x subnormal")


@pytest.mark.parametrize("rows,hidden", SHAPES)
def test_q8_0_gguf_reference_quantized(backend, rows, hidden):
    w = O.quantize_q8_0(normal(seed_for("q80", rows, hidden), rows * hidden, 0.02))
    x = normal(seed_for("q80x", rows, hidden), hidden)
    wt = backend.register_weight(w, L.FMT_Q8_0_GGUF, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    _cmp(got, O.q8_0_matvec_f32(w, x, rows, hidden), "q8_0 gguf")


@pytest.mark.parametrize("subnormal", [False, True])
def test_q8_0_gguf_random_bytes(backend, subnormal):
    rows, hidden = 61, 4096
    w = _random_q8_0(seed_for("q80r", subnormal), rows, hidden, subnormal)
    x = normal(seed_for("q80rx", subnormal), 2 * hidden).reshape(2, hidden)
    wt = backend.register_weight(w, L.FMT_Q8_0_GGUF, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    ref = O.q8_0_matvec_f32(w, x, rows, hidden)
    for b in range(2):
        _cmp(got[b], ref[b], f"q8_0 gguf random b{b}")


@pytest.mark.parametrize("rows,hidden", [(64, 512), (33, 4096), (20, 14336), (300, 1024)])
def test_q8_compute_layout(backend, rows, hidden):
    """q8_matvec.rs:36-57: int8 weights + f32 scales x quantize_to_q8(x), x quantized on the device."""
    wq, ws = O.quantize_weights_q8(normal(seed_for("q8c", rows, hidden), rows * hidden, 0.02), rows, hidden)
    x = normal(seed_for("q8cx", rows, hidden), 2 * hidden).reshape(2, hidden)
    wt = backend.register_weight(wq.view(np.uint8), L.FMT_Q8_0, rows, hidden, scales=ws)
    got = backend.matvec(wt, x)
    wt.release()
    for b in range(2):
        xq, xs = O.quantize_to_q8(x[b])
        _cmp(got[b], O.q8_matvec(wq, ws, xq, xs, rows, hidden), f"q8 compute b{b}")


def test_device_quantize_to_q8_bit_exact(backend):
    import torch
    rng = np.random.default_rng(3)
    for x in [normal(1, 4096), np.zeros(64, np.float32), rng.uniform(-1e5, 1e5, 1024).astype(np.float32),
              (rng.standard_normal(2048) * np.exp2(rng.integers(-40, 40, 2048))).astype(np.float32)]:
        wq, ws = O.quantize_to_q8(x)
        xd = torch.from_numpy(x).cuda()
        q = torch.empty(x.size, dtype=torch.int8, device="cuda")
        s = torch.empty(x.size // 32, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        backend.quantize_to_q8_dev(xd, q, s)
        backend.sync()
        assert np.array_equal(q.cpu().numpy(), wq)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), ws.view(np.uint32))


def test_q4_0_lm_head_rows_sample(backend):
    import torch
    rows, hidden = 128256, 4096
    rng = np.random.default_rng(9)
    w = O.quantize_q4_0(rng.standard_normal(rows * hidden, dtype=np.float32) * np.float32(0.02))
    x = normal(10, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_0, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    rb = hidden // 32 * 18
    for r0 in [0, 77777, rows - 40]:
        _cmp(got[r0:r0 + 40], O.q4_0_matvec_f32(w[r0 * rb:(r0 + 40) * rb], x, 40, hidden), f"lm-head rows {r0}")


def _special_values(seed, n):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * np.exp2(rng.integers(-30, 30, n))).astype(np.float32)
    x[:32] = 0.0                                   # zero block -> scale 0, nibbles 8 / int8 0
    x[40] = np.inf                                 # inf amax -> f16 inf scale, inv 0
    x[70] = np.nan                                 # NaN skipped by the f32::max fold
    x[96:128] = np.float32(3e38)                   # f16 overflow of the scale
    x[128:160] = np.float32(1e-30)                 # scale below the f16 normal range -> 0
    return x


@pytest.mark.parametrize("which", ["q4_0", "q8_0"])
def test_device_block32_quantizers_bit_exact(backend, which):
    import torch
    for x in [normal(11, 4096 * 33, 0.02), _special_values(12, 8192)]:
        ref = O.quantize_q4_0(x) if which == "q4_0" else O.quantize_q8_0(x)
        xd = torch.from_numpy(x).cuda()
        out = torch.empty(ref.size, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        (backend.quantize_q4_0_dev if which == "q4_0" else backend.quantize_q8_0_dev)(xd, out)
        backend.sync()
        got = out.cpu().numpy()
        bad = np.nonzero(got != ref)[0]
        assert bad.size == 0, f"{which}: {bad.size} bytes differ, first at {bad[:5]}"


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_f32x_nan_value_propagates(backend, fmt):
    """A NaN activation makes every output NaN, as the f32 dot of the dequantized rows does (the block's amax
    fold skips NaN, so the kernel tests each value)."""
    rows, hidden = 40, 1024
    src = normal(seed_for("nanx", fmt), rows * hidden, 0.02)
    w = O.quantize_q4_0(src) if fmt == "q4_0" else O.quantize_q8_0(src)
    x = normal(seed_for("nanxx", fmt), hidden)
    x[333] = np.nan
    wt = backend.register_weight(w, L.FMT_Q4_0 if fmt == "q4_0" else L.FMT_Q8_0_GGUF, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    ref = O.q4_0_matvec_f32(w, x, rows, hidden) if fmt == "q4_0" else O.q8_0_matvec_f32(w, x, rows, hidden)
    assert np.all(np.isnan(ref)) and np.all(np.isnan(got))


def _fmt_case(fmt, seed, rows, hidden, random_bytes=False):
    if fmt == "q4_0":
        w = _random_q4_0(seed, rows, hidden, True) if random_bytes else O.quantize_q4_0(normal(seed, rows * hidden, 0.02))
        return w, L.FMT_Q4_0, O.q4_0_matvec_f32
    w = _random_q8_0(seed, rows, hidden, True) if random_bytes else O.quantize_q8_0(normal(seed, rows * hidden, 0.02))
    return w, L.FMT_Q8_0_GGUF, O.q8_0_matvec_f32


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("batch", [2, 5, 8])
def test_block_f32x_warp_mma_all_batch_rows_in_one_pass(backend, fmt, batch):
    """Q4_0 / GGUF Q8_0 with K % 1024 == 0 at batch >= 2 run on the warp-MMA kernel (one weight pass for the
    whole batch; batch 1 stays on the block kernel for Q8_0 and takes the MMA kernel for Q4_0); 300 rows leave a
    partial row tile."""
    rows, hidden = 300, 4096
    w, F, ref_fn = _fmt_case(fmt, seed_for("blkb", fmt, batch), rows, hidden)
    x = normal(seed_for("blkbx", fmt, batch), batch * hidden).reshape(batch, hidden)
    wt = backend.register_weight(w, F, rows, hidden)
    assert "q4k_mma_kernel" in backend.describe_matvec(wt, batch)
    assert ("q4k_mma_kernel" if fmt == "q4_0" else "blk_matvec_kernel") in backend.describe_matvec(wt, 1)
    got = backend.matvec(wt, x)
    wt.release()
    ref = ref_fn(w, x, rows, hidden)
    for b in range(batch):
        _cmp(got[b], ref[b], f"{fmt} mma b{b}")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("cfg", ["8,1,0,1,0", "4,2,0,1,0", "4,1,0,3,0"])
def test_block_f32x_warp_mma_output_forms(monkeypatch, fmt, cfg):
    """Pinned plans (groups, K slices, stages, K parts) on random-byte blocks with subnormal scales: direct
    row-group stores, K slices summed in shared memory, K parts added by the last CTA of a tile."""
    monkeypatch.setenv("LARQL_CUDA_MMA_CFG", cfg)
    be = L.CudaBackend(0)
    try:
        rows, hidden = 200, 3072
        w, F, ref_fn = _fmt_case(fmt, seed_for("blkf", fmt, cfg), rows, hidden, random_bytes=True)
        x = normal(seed_for("blkfx", fmt, cfg), 3 * hidden).reshape(3, hidden)
        wt = be.register_weight(w, F, rows, hidden)
        got = be.matvec(wt, x)
        wt.release()
        ref = ref_fn(w, x, rows, hidden)
        for b in range(3):
            _cmp(got[b], ref[b], f"{fmt} {cfg} b{b}")
    finally:
        be.close()
