"""Every Q4_K kernel family and MMA plan shape against the oracle (q4k_matvec.rs:31-87).

The context reads LARQL_CUDA_Q4K_PATH (mma | tc | dp4a | ts) and LARQL_CUDA_MMA_CFG
("groups,slices,stages,parts,prefetch"; 0 = planner's choice) when it is
created, so each case builds its own context.
Tolerance: max |err| <= 1e-3 * ||y_ref||_inf.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_q4k_blocks, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")


def _backend(path, cfg=None):
    old = {k: os.environ.get(k) for k in ("LARQL_CUDA_Q4K_PATH", "LARQL_CUDA_MMA_CFG")}
    os.environ["LARQL_CUDA_Q4K_PATH"] = path
    if cfg:
        os.environ["LARQL_CUDA_MMA_CFG"] = cfg
    else:
        os.environ.pop("LARQL_CUDA_MMA_CFG", None)
    try:
        return L.CudaBackend(0)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _run(be, w, x, rows, hidden):
    wt = be.register_weight(w, L.FMT_Q4_K, rows, hidden)
    try:
        return be.matvec(wt, x)
    finally:
        wt.release()


def _assert_close(got, ref, what):
    got = got.reshape(ref.shape)
    for b in range(ref.shape[0] if ref.ndim == 2 else 1):
        g, r = (got[b], ref[b]) if ref.ndim == 2 else (got, ref)
        ok, err, bound = max_err_ok(g, r)
        assert ok, f"{what} batch row {b}: max err {err} > {bound}"


# (16-row groups, K slices per group, stages, parts across CTAs): tile heights 16..128, 1-4 warps
# per row group, 2- to 8-stage rings, split-K across CTAs up to 16 parts (K = 16384) or 5 (K = 5120)
MMA_CFGS = ["8,1,2,1", "6,1,3,1", "4,1,4,1", "4,1,2,2", "8,1,2,4", "6,1,0,3", "4,1,3,16",
            "2,4,0,1", "4,2,0,1", "1,4,0,2", "2,2,3,4", "1,2,0,1", "2,4,0,16", "3,2,0,5"]
# x tables + stages above the 227 KB of shared memory (the library rejects a pinned plan that does not fit)
TOO_BIG = {("8,1,2,1", 8), ("6,1,3,1", 3), ("6,1,3,1", 5), ("6,1,3,1", 8), ("4,1,4,1", 8)}
MMA_CASES = [(c, b) for c in MMA_CFGS for b in (1, 2, 3, 5, 8) if (c, b) not in TOO_BIG]


@pytest.mark.parametrize("cfg,batch", MMA_CASES)
def test_mma_plans(cfg, batch):
    parts = int(cfg.split(",")[3])
    rows, hidden = 333, {16: 16384, 5: 5120}.get(parts, 4096)
    be = _backend("mma", cfg)
    try:
        w = O.quantize_q4_k(normal(seed_for("mp", rows, hidden), rows * hidden, 0.02))
        x = normal(seed_for("mpx", batch), batch * hidden).reshape(batch, hidden)
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), f"mma {cfg}")
    finally:
        be.close()


@pytest.mark.parametrize("path", ["mma", "tc", "dp4a", "ts"])
@pytest.mark.parametrize("rows,hidden,batch", [(4096, 4096, 1), (4096, 4096, 4), (130, 14336, 8), (517, 3072, 2),
                                               (16, 1024, 1), (1, 1024, 8), (2000, 2048, 6)])
def test_paths_agree_with_oracle(path, rows, hidden, batch):
    be = _backend(path)
    try:
        w = O.quantize_q4_k(normal(seed_for("pa", rows, hidden), rows * hidden, 0.02))
        x = normal(seed_for("pax", rows, batch), batch * hidden).reshape(batch, hidden)
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), f"{path} {rows}x{hidden}")
    finally:
        be.close()


@pytest.mark.parametrize("batch", [1, 4, 8])
@pytest.mark.parametrize("cfg", [None, "4,1,2,4", "2,4,0,2"])
def test_mma_random_byte_blocks(batch, cfg):
    """Every nibble, every 6-bit scale (bytes 4..11 with their top bits set), random finite f16 d / dmin."""
    rows, hidden = 250, 4096
    be = _backend("mma", cfg)
    try:
        w = random_q4k_blocks(seed_for("mrb", batch), rows, hidden)
        x = normal(seed_for("mrbx", batch), batch * hidden).reshape(batch, hidden)
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), "mma random bytes")
    finally:
        be.close()


def test_mma_wide_dynamic_range_x():
    """x spanning 2^-40..2^40 within a super-block exercises the per-super-block plane exponent."""
    rows, hidden, batch = 96, 2048, 2
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((batch, hidden)) * np.exp2(rng.integers(-40, 40, (batch, hidden)))).astype(np.float32)
    w = O.quantize_q4_k(normal(6, rows * hidden, 0.02))
    be = _backend("mma")
    try:
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), "wide range")
    finally:
        be.close()


def test_mma_split_k_repeatable():
    """Split-K sums parts in a fixed order: two launches give identical bits (tickets reset each launch)."""
    rows, hidden, batch = 700, 8192, 4
    be = _backend("mma", "4,2,2,8")
    try:
        w = O.quantize_q4_k(normal(7, rows * hidden, 0.02))
        x = normal(8, batch * hidden).reshape(batch, hidden)
        wt = be.register_weight(w, L.FMT_Q4_K, rows, hidden)
        a = be.matvec(wt, x)
        b = be.matvec(wt, x)
        wt.release()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        _assert_close(a, O.q4k_matvec(w, x, rows, hidden), "split-K")
    finally:
        be.close()


def test_pinned_plan_that_does_not_fit_is_unsupported():
    be = _backend("mma", "8,1,2,1")
    try:
        w = O.quantize_q4_k(normal(11, 64 * 4096, 0.02))
        wt = be.register_weight(w, L.FMT_Q4_K, 64, 4096)
        with pytest.raises(L.LarqlCudaError) as ei:
            be.matvec(wt, normal(12, 8 * 4096).reshape(8, 4096))
        assert ei.value.status == L.ERR_UNSUPPORTED
        wt.release()
    finally:
        be.close()


def test_mma_nonfinite_x_gives_nonfinite_rows():
    rows, hidden = 40, 1024
    w = O.quantize_q4_k(normal(9, rows * hidden, 0.02))
    x = normal(10, hidden)
    x[300] = np.nan
    be = _backend("mma")
    try:
        got = _run(be, w, x, rows, hidden)
    finally:
        be.close()
    ref = O.q4k_matvec(w, x, rows, hidden)
    assert np.all(~np.isfinite(ref)) and np.all(~np.isfinite(got))


# ── the tensor-memory kernel (q4k_ts.cu): sc*q in TMEM, x as f16 hi / lo planes ──

@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 6, 7, 8])
def test_ts_every_batch(batch):
    """Batch rows 0-3 are summed by warps 0-3, rows 4-7 by warps 4-7; 333 rows leave a ragged last tile."""
    rows, hidden = 333, 4096
    be = _backend("ts")
    try:
        w = O.quantize_q4_k(normal(seed_for("tsb", rows, hidden), rows * hidden, 0.02))
        x = normal(seed_for("tsbx", batch), batch * hidden).reshape(batch, hidden)
        wt = be.register_weight(w, L.FMT_Q4_K, rows, hidden)
        assert "q4k_ts_kernel" in be.describe_matvec(wt, batch)
        got = be.matvec(wt, x)
        wt.release()
        _assert_close(got, O.q4k_matvec(w, x, rows, hidden), f"ts batch {batch}")
    finally:
        be.close()


@pytest.mark.parametrize("batch", [1, 4, 8])
def test_ts_random_byte_blocks(batch):
    """Every nibble, every 6-bit scale with its top bits set, every min, random finite f16 d / dmin."""
    rows, hidden = 250, 4096
    be = _backend("ts")
    try:
        w = random_q4k_blocks(seed_for("tsrb", batch), rows, hidden)
        x = normal(seed_for("tsrbx", batch), batch * hidden).reshape(batch, hidden)
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), "ts random bytes")
    finally:
        be.close()


@pytest.mark.parametrize("rows,hidden,batch", [(4096, 14336, 8), (700, 8192, 4), (129, 1024, 3), (1, 2048, 8)])
def test_ts_split_k_shapes(rows, hidden, batch):
    """Shapes whose plan splits K across CTAs (ordered sum of the parts by the last CTA of a tile)."""
    be = _backend("ts")
    try:
        w = O.quantize_q4_k(normal(seed_for("tss", rows, hidden), rows * hidden, 0.02))
        x = normal(seed_for("tssx", rows, batch), batch * hidden).reshape(batch, hidden)
        wt = be.register_weight(w, L.FMT_Q4_K, rows, hidden)
        a = be.matvec(wt, x)
        b = be.matvec(wt, x)
        wt.release()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), "two launches differ"
        _assert_close(a, O.q4k_matvec(w, x, rows, hidden), f"ts {rows}x{hidden}")
    finally:
        be.close()


def test_ts_wide_dynamic_range_x():
    """x spanning 2^-40..2^40 within a super-block exercises the per-super-block power of two of the planes."""
    rows, hidden, batch = 96, 2048, 2
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((batch, hidden)) * np.exp2(rng.integers(-40, 40, (batch, hidden)))).astype(np.float32)
    w = O.quantize_q4_k(normal(6, rows * hidden, 0.02))
    be = _backend("ts")
    try:
        _assert_close(_run(be, w, x, rows, hidden), O.q4k_matvec(w, x, rows, hidden), "ts wide range")
    finally:
        be.close()


def test_ts_nonfinite_x_gives_nonfinite_rows():
    rows, hidden = 40, 1024
    w = O.quantize_q4_k(normal(9, rows * hidden, 0.02))
    x = normal(10, hidden)
    x[300] = np.nan
    be = _backend("ts")
    try:
        got = _run(be, w, x, rows, hidden)
    finally:
        be.close()
    ref = O.q4k_matvec(w, x, rows, hidden)
    assert np.all(~np.isfinite(ref)) and np.all(~np.isfinite(got))


def test_route_cache_alternating_batches():
    """The route (kernel, plan, tensor-map tile height) is cached per weight and batch; alternating batches on one
    weight, including a shape whose batch-1 and batch-8 plans use different tile heights, keeps every result right."""
    be = _backend("mma")
    try:
        for rows, hidden in [(4096, 4096), (700, 8192)]:
            w = O.quantize_q4_k(normal(seed_for("rc", rows, hidden), rows * hidden, 0.02))
            wt = be.register_weight(w, L.FMT_Q4_K, rows, hidden)
            try:
                plans = {}
                for batch in (1, 8, 4, 1, 8, 2, 4):
                    x = normal(seed_for("rcx", rows, batch), batch * hidden).reshape(batch, hidden)
                    plans.setdefault(batch, be.describe_matvec(wt, batch))
                    assert be.describe_matvec(wt, batch) == plans[batch]
                    _assert_close(be.matvec(wt, x), O.q4k_matvec(w, x, rows, hidden), f"route cache b{batch}")
            finally:
                wt.release()
    finally:
        be.close()
