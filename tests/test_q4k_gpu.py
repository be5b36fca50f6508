"""Q4_K (LARQL 148 B) matvec on the GPU vs the CPU oracle (q4k_matvec.rs:31-87).

Tolerance (north star): max |err| <= 1e-3 * ||y_ref||_inf, f32 accumulate.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_q4k_blocks, seed_for

pytestmark = pytest.mark.gpu

L = pytest.importorskip("larql_cuda")


def _check(backend, w, x, rows, hidden):
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, hidden)
    try:
        got = backend.matvec(wt, x)
    finally:
        wt.release()
    ref = O.q4k_matvec(w, x, rows, hidden)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound} (rows={rows} hidden={hidden})"
    return got, ref


def test_reference_metal_test_shape(backend):
    """tests/test_metal_shaders.rs:1394-1411 inputs (32 x 256, cos/sin)."""
    rows, hidden = 32, 256
    m = np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32)
    x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    q = O.quantize_q4_k(m)
    got = backend.q4k_matvec(q, x, rows, hidden)
    ref = O.q4k_matvec(q, x, rows, hidden)
    assert np.max(np.abs(got - ref)) < 0.5  # the reference's own Metal-vs-CPU bound
    assert max_err_ok(got, ref)[0]
    assert np.any(np.abs(got) > 0.001)


@pytest.mark.skipif(O.metal_ref_lib() is None, reason="reference Metal shaders not built here")
@pytest.mark.parametrize("rows,hidden,kind", [(32, 256, "metal_test"), (300, 4096, "quantized"), (64, 2048, "random")])
def test_against_the_reference_metal_shader_run_on_cpu(backend, rows, hidden, kind):
    """The CUDA matvec against the reference's own q4k_matvec shader code (crates/larql-compute/src/metal/shaders/
    q4k_matvec.rs, compiled for the CPU by oracle/Makefile), not a restatement: the test_metal_shaders.rs inputs,
    quantized weights and random-byte blocks, within 1e-3 * |y|_inf."""
    if kind == "metal_test":
        w = O.quantize_q4_k(np.cos(np.arange(rows * hidden, dtype=np.float32) * np.float32(0.001)).astype(np.float32))
        x = np.sin(np.arange(hidden, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    else:
        w = (O.quantize_q4_k(normal(seed_for("mg", rows, hidden), rows * hidden, 0.02)) if kind == "quantized"
             else random_q4k_blocks(seed_for("mgr", rows), rows, hidden))
        x = normal(seed_for("mgx", rows, hidden), hidden)
    got = backend.q4k_matvec(w, x, rows, hidden)
    ok, err, bound = max_err_ok(got, O.metal_q4k_matvec(w, x, rows, hidden))
    assert ok, (kind, err, bound)


@pytest.mark.parametrize("rows,hidden", [(64, 512), (37, 1024), (5, 256), (130, 2560), (96, 4096), (20, 14336),
                                         (7, 17408), (3, 18432)])
def test_reference_quantized_weights(backend, rows, hidden):
    w = O.quantize_q4_k(normal(seed_for("q4k", rows, hidden), rows * hidden, 0.02))
    x = normal(seed_for("x", rows, hidden), hidden)
    _check(backend, w, x, rows, hidden)


@pytest.mark.parametrize("rows,hidden", [(64, 512), (33, 4096), (12, 14336), (9, 256)])
def test_random_byte_blocks(backend, rows, hidden):
    """All nibble values, all 6-bit scales, random signed f16 d/dmin (reference quantizer only emits 0/1 nibbles)."""
    w = random_q4k_blocks(seed_for("rand", rows, hidden), rows, hidden)
    x = normal(seed_for("xr", rows, hidden), hidden)
    _check(backend, w, x, rows, hidden)


def test_subnormal_scales(backend):
    rows, hidden = 16, 1024
    w = random_q4k_blocks(7, rows, hidden).reshape(-1, 148)
    rng = np.random.default_rng(8)
    w[:, 0:2] = rng.integers(1, 0x3FF, (w.shape[0], 1)).astype(np.uint16).view(np.uint8).reshape(-1, 2)  # subnormal d
    x = normal(9, hidden)
    _check(backend, w.reshape(-1), x, rows, hidden)


def test_config1_full_size(backend):
    """W 11008x4096 ~ N(0,0.02) seed 0 -> quantize_q4_k; x ~ N(0,1)."""
    rows, hidden = 11008, 4096
    w = O.quantize_q4_k(normal(0, rows * hidden, 0.02))
    x = normal(1, hidden)
    _check(backend, w, x, rows, hidden)


@pytest.mark.parametrize("rows,hidden,batch", [(200, 4096, 1), (200, 4096, 2), (200, 4096, 3), (200, 4096, 4),
                                               (200, 4096, 5), (200, 4096, 6), (200, 4096, 8), (37, 1024, 2),
                                               (130, 14336, 5), (130, 14336, 8), (1000, 2048, 7)])
def test_batched(backend, rows, hidden, batch):
    """Default routing: the warp-MMA kernel for K % 1024 == 0, the CUDA-core kernels otherwise."""
    w = O.quantize_q4_k(normal(seed_for("b", rows, hidden), rows * hidden, 0.02))
    x = normal(seed_for("bx", rows, hidden, batch), batch * hidden).reshape(batch, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    ref = O.q4k_matvec(w, x, rows, hidden)
    assert got.shape == (batch, rows)
    for b in range(batch):
        ok, err, bound = max_err_ok(got[b], ref[b])
        assert ok, (b, err, bound)


@pytest.mark.parametrize("batch", [2, 4, 8])
def test_batched_random_bytes(backend, batch):
    rows, hidden = 300, 4096
    w = random_q4k_blocks(seed_for("rb", batch), rows, hidden)
    x = normal(seed_for("rbx", batch), batch * hidden).reshape(batch, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, hidden)
    got = backend.matvec(wt, x)
    wt.release()
    ref = O.q4k_matvec(w, x, rows, hidden)
    for b in range(batch):
        ok, err, bound = max_err_ok(got[b], ref[b])
        assert ok, (b, err, bound)


def test_zero_and_constant_x(backend):
    rows, hidden = 40, 1024
    w = random_q4k_blocks(11, rows, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, hidden)
    assert np.all(backend.matvec(wt, np.zeros(hidden, np.float32)) == 0.0)
    x = np.full(hidden, 0.75, np.float32)
    ok, err, bound = max_err_ok(backend.matvec(wt, x), O.q4k_matvec(w, x, rows, hidden))
    wt.release()
    assert ok, (err, bound)


def test_trait_mirror_reuses_registered_weight(backend):
    rows, hidden = 64, 512
    w = O.quantize_q4_k(normal(21, rows * hidden, 0.02))
    x1, x2 = normal(22, hidden), normal(23, hidden)
    y1 = backend.q4k_matvec(w, x1, rows, hidden)
    y2 = backend.q4k_matvec(w, x2, rows, hidden)
    assert max_err_ok(y1, O.q4k_matvec(w, x1, rows, hidden))[0]
    assert max_err_ok(y2, O.q4k_matvec(w, x2, rows, hidden))[0]


def test_bad_shapes_are_errors(backend):
    w = np.zeros(148, np.uint8)
    with pytest.raises(L.LarqlCudaError) as e:
        backend.register_weight(w, L.FMT_Q4_K, 1, 255)
    assert e.value.status == L.ERR_BAD_SHAPE
    with pytest.raises(L.LarqlCudaError) as e:
        backend.register_weight(w, L.FMT_Q4_K, 2, 256)  # too few bytes
    assert e.value.status == L.ERR_BAD_SHAPE
    wt = backend.register_weight(w, L.FMT_Q4_K, 1, 256)
    with pytest.raises(L.LarqlCudaError) as e:
        backend.matvec(wt, np.zeros((9, 256), np.float32))  # batch > 8
    assert e.value.status == L.ERR_BAD_SHAPE
    wt.release()


def test_device_quantizer_bit_exact(backend):
    import torch
    rng = np.random.default_rng(5)
    cases = [normal(31, 64 * 4096, 0.02),
             rng.uniform(-3, 3, 256 * 40).astype(np.float32),
             np.zeros(256 * 3, np.float32),
             np.full(256 * 2, 0.5, np.float32),
             np.concatenate([np.full(256, -1.25, np.float32), rng.standard_normal(256).astype(np.float32) * 1e-6]),
             (rng.standard_normal(256 * 16) * np.exp2(rng.integers(-30, 30, 256 * 16))).astype(np.float32)]
    for data in cases:
        want = O.quantize_q4_k(data)
        src = torch.from_numpy(data).cuda()
        out = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        backend.quantize_q4_k_dev(src, out)
        backend.sync()
        got = out.cpu().numpy()
        assert np.array_equal(got, want), np.nonzero(got != want)[0][:10]


def test_lm_head_rows_sample_and_linearity(backend):
    """128256 x 4096 (303 MB): rows sampled against the oracle, linearity across the whole output."""
    import torch
    rows, hidden = 128256, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    wf = torch.randn(rows * hidden, generator=g, device="cuda", dtype=torch.float32) * 0.02
    q = torch.empty(rows * hidden // 256 * 148, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    backend.quantize_q4_k_dev(wf, q)
    backend.sync()
    del wf
    wt = backend.register_weight(q, L.FMT_Q4_K, rows, hidden)
    x1, x2 = normal(41, hidden), normal(42, hidden)
    xs = np.stack([x1, x2, x1 + x2])
    y = backend.matvec(wt, xs)
    wt.release()
    ok, err, bound = max_err_ok(y[2], y[0] + y[1], rel=2e-3)
    assert ok, (err, bound)
    qh = q.cpu().numpy()
    rb = hidden // 256 * 148
    for r0 in [0, 64000, rows - 50]:
        sub = qh[r0 * rb:(r0 + 50) * rb]
        ref = O.q4k_matvec(sub, x1, 50, hidden)
        assert max_err_ok(y[0][r0:r0 + 50], ref)[0]
