"""Batched prefill dequant-GEMM on tcgen05 vs the oracle: per token, the Q4_K matvec of q4k_matvec.rs:31-87 and
silu_gate_up (crates/larql-inference/src/ffn/mod.rs:87-94).  Tolerance: max |err| <= 1e-3 * ||Y_ref||_inf."""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_q4k_blocks, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")
torch = pytest.importorskip("torch")


def _q4k(seed, rows, cols):
    return O.quantize_q4_k(normal(seed, rows * cols, 0.02))


def _gemm(backend, w, n, k, x):
    wt = backend.register_weight(w, L.FMT_Q4_K, n, k)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.empty(x.shape[0] * n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.q4k_gemm_dev(wt, xd, x.shape[0], y)
    backend.sync()
    wt.release()
    return y.cpu().numpy().reshape(x.shape[0], n)


def _ref_rows(w, x, n, k, rows):
    return np.stack([O.q4k_matvec(w, x[t], n, k) for t in rows])


@pytest.mark.parametrize("n,k,m", [(300, 1024, 1), (300, 1024, 7), (256, 512, 64), (130, 2048, 129),
                                   (517, 1024, 300), (128, 256, 513)])
def test_gemm_vs_oracle(backend, n, k, m):
    w = _q4k(seed_for("pg", n, k), n, k)
    x = np.random.default_rng(seed_for("pgx", m)).standard_normal((m, k)).astype(np.float32)
    y = _gemm(backend, w, n, k, x)
    rows = range(m) if m <= 64 else sorted({0, 1, m // 2, m - 2, m - 1, 63, 64, 127, 128} & set(range(m)))
    ref = _ref_rows(w, x, n, k, rows)
    ok, err, bound = max_err_ok(y[list(rows)], ref)
    assert ok, f"max err {err} > {bound}"


def test_gemm_stream_k_many_contributors_repeatable(backend):
    """K = 8192 over 16 tiles: each tile is split across about ten CTAs, more than the owner's
    staging buffers, so the fixup refills them; two calls give identical bits."""
    n, k, m = 1000, 8192, 300
    w = _q4k(31, n, k)
    x = np.random.default_rng(32).standard_normal((m, k)).astype(np.float32)
    y1 = _gemm(backend, w, n, k, x)
    y2 = _gemm(backend, w, n, k, x)
    assert np.array_equal(y1, y2)
    rows = [0, 1, 150, 255, 256, 299]
    ok, err, bound = max_err_ok(y1[rows], _ref_rows(w, x, n, k, rows))
    assert ok, f"max err {err} > {bound}"


def test_gemm_misaligned_activations_and_nonfinite_token(backend):
    """Activations starting 4 bytes past a 16-byte boundary take the scalar prep path; a token holding a
    NaN gives non-finite outputs for that token only (the f32 reference sums NaN into every output)."""
    n, k, m = 300, 1024, 9
    w = _q4k(41, n, k)
    x = np.random.default_rng(42).standard_normal((m, k)).astype(np.float32)
    x[4, 17] = np.nan
    wt = backend.register_weight(w, L.FMT_Q4_K, n, k)
    buf = torch.empty(m * k + 4, dtype=torch.float32, device="cuda")
    buf[1:1 + m * k] = torch.from_numpy(x.ravel()).cuda()
    y = torch.empty(m * n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.q4k_gemm_dev(wt, buf[1:], m, y)
    backend.sync()
    wt.release()
    got = y.cpu().numpy().reshape(m, n)
    assert not np.isfinite(got[4]).any()
    for t in [0, 3, 5, 8]:
        ok, err, bound = max_err_ok(got[t], O.q4k_matvec(w, x[t], n, k))
        assert ok, f"token {t}: max err {err} > {bound}"


def test_gemm_random_byte_blocks_and_large_scales(backend):
    """Random bytes with f16 d / dmin up to 65504: the per-matrix power of two keeps the f16 tiles finite."""
    n, k, m = 200, 1024, 33
    w = random_q4k_blocks(5, n, k)
    x = np.random.default_rng(6).standard_normal((m, k)).astype(np.float32)
    y = _gemm(backend, w, n, k, x)
    ref = _ref_rows(w, x, n, k, range(m))
    ok, err, bound = max_err_ok(y, ref)
    assert ok, f"max err {err} > {bound}"


def test_gemm_wide_range_tokens(backend):
    n, k, m = 256, 1024, 4
    w = _q4k(7, n, k)
    rng = np.random.default_rng(8)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[1] *= np.float32(1e6)
    x[2] *= np.float32(1e-6)
    y = _gemm(backend, w, n, k, x)
    for t in range(m):
        ok, err, bound = max_err_ok(y[t], O.q4k_matvec(w, x[t], n, k))
        assert ok, f"token {t}: max err {err} > {bound}"


def _ffn_ref(wg, wu, wd, x, h, i, t):
    g = O.q4k_matvec(wg, x[t], i, h)
    u = O.q4k_matvec(wu, x[t], i, h)
    a = (g * (np.float32(1) / (np.float32(1) + np.exp(-g))) * u).astype(np.float32)
    return O.q4k_matvec(wd, a, h, i)


def _ffn(backend, wg, wu, wd, h, i, x):
    tg = backend.register_weight(wg, L.FMT_Q4_K, i, h)
    tu = backend.register_weight(wu, L.FMT_Q4_K, i, h)
    td = backend.register_weight(wd, L.FMT_Q4_K, h, i)
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.empty(x.shape[0] * h, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.prefill_ffn_dev(tg, tu, td, xd, x.shape[0], y)
    backend.sync()
    for t_ in (tg, tu, td):
        t_.release()
    return y.cpu().numpy().reshape(x.shape[0], h)


def test_ffn_small(backend):
    h, i, m = 1024, 2048, 40
    wg, wu, wd = _q4k(11, i, h), _q4k(12, i, h), _q4k(13, h, i)
    x = np.random.default_rng(14).standard_normal((m, h)).astype(np.float32)
    y = _ffn(backend, wg, wu, wd, h, i, x)
    ref = np.stack([_ffn_ref(wg, wu, wd, x, h, i, t) for t in range(m)])
    ok, err, bound = max_err_ok(y, ref)
    assert ok, f"max err {err} > {bound}"


def test_ffn_config4_sampled_tokens(backend):
    """512 tokens x 4096, gate/up 14336 x 4096 and down 4096 x 14336 in Q4_K."""
    h, i, m = 4096, 14336, 512
    wg, wu, wd = _q4k(21, i, h), _q4k(22, i, h), _q4k(23, h, i)
    x = np.random.default_rng(24).standard_normal((m, h)).astype(np.float32)
    y = _ffn(backend, wg, wu, wd, h, i, x)
    toks = [0, 127, 128, 255, 256, 511]
    ref = np.stack([_ffn_ref(wg, wu, wd, x, h, i, t) for t in toks])
    ok, err, bound = max_err_ok(y[toks], ref)
    assert ok, f"max err {err} > {bound}"
    assert np.all(np.isfinite(y))


def test_ffn_host_entry_borrowed_slices(backend):
    """larql_cuda_prefill_ffn: the prefill_q4 ownership form (host weights and activations in, host output out),
    twice on the same weights (found again by pointer and length), against the oracle composition."""
    h, i, m = 1024, 2048, 24
    wg, wu, wd = _q4k(51, i, h), _q4k(52, i, h), _q4k(53, h, i)
    for seed in (54, 55):
        x = np.random.default_rng(seed).standard_normal((m, h)).astype(np.float32)
        y = backend.prefill_ffn(wg, wu, wd, x, h, i)
        ref = np.stack([_ffn_ref(wg, wu, wd, x, h, i, t) for t in range(m)])
        ok, err, bound = max_err_ok(y, ref)
        assert ok, f"max err {err} > {bound}"

