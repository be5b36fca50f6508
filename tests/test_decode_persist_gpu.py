"""One-token decode in one persistent launch (csrc/decode_persist.cu, LARQL_CUDA_DECODE_PERSIST=1) vs the oracle
composite of the reference CPU pieces (rms_norm_eps residual.rs:17-35, q4k_matvec.rs:31-87, apply_rope rope.rs:22-55,
gqa_attention gqa.rs:29-110, silu_gate_up ffn/mod.rs:87-94).  Tolerance: max |err| <= 1e-3 * ||x_ref||_inf, as
the per-kernel decode tests."""
import numpy as np
import pytest

from conftest import max_err_ok
from test_decode_gpu import THETA, _oracle_token, _setup

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")


@pytest.fixture
def pbe(monkeypatch):
    monkeypatch.setenv("LARQL_CUDA_DECODE_PERSIST", "1")
    be = L.CudaBackend(0)
    yield be
    be.close()


def test_runtime_switch(backend):
    """larql_cuda_decode_set_persistent selects the persistent kernel on a context created without the variable."""
    hidden, inter, nq, nkv, seq = 1024, 1024, 8, 2, 64
    layers, handles, caches = _setup(backend, 1, hidden, inter, nq, nkv, seq, 128, 77)
    x = np.random.default_rng(78).standard_normal(hidden).astype(np.float32)
    backend.decode_set_persistent(True)
    try:
        n, got = _one_token(backend, handles, x, seq)
    finally:
        backend.decode_set_persistent(False)
    assert n == 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"
    n2, _ = _one_token(backend, handles, x, seq)
    assert n2 > 1
    for h in handles:
        backend.layer_release(h)


def _one_token(be, handles, x, seq):
    """One token through the device entry; returns (library kernel launches, new residual)."""
    import torch
    xd = torch.from_numpy(x.copy()).cuda()
    n0 = L.launch_count()
    be.decode_token_dev(handles, xd, seq, THETA)
    be.sync()
    return L.launch_count() - n0, xd.cpu().numpy()


def test_two_layers_three_tokens(pbe):
    hidden, inter, nq, nkv, seq = 1024, 2048, 8, 2, 37
    layers, handles, caches = _setup(pbe, 2, hidden, inter, nq, nkv, seq, 64, 1)
    rng = np.random.default_rng(2)
    for t in range(3):
        x = rng.standard_normal(hidden).astype(np.float32)
        got = pbe.decode_token(handles, x, THETA)
        ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq + t)
        ok, err, bound = max_err_ok(got, ref)
        assert ok, f"token {t}: max err {err} > {bound}"
        assert pbe.kv_length() == seq + t + 1


@pytest.mark.parametrize("nq,nkv", [(8, 8), (8, 4), (8, 2), (16, 2)])
def test_gqa_ratios(pbe, nq, nkv):
    hidden, inter, seq = 1024, 1024, 300
    layers, handles, caches = _setup(pbe, 1, hidden, inter, nq, nkv, seq, 512, nq * 10 + nkv)
    x = np.random.default_rng(3).standard_normal(hidden).astype(np.float32)
    n, got = _one_token(pbe, handles, x, seq)
    assert n == 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"


@pytest.mark.parametrize("seq", [1, 127, 128, 4501])
def test_cache_lengths(pbe, seq):
    """Two keys; 128 keys (one full range of 128); 129 keys (the second range holds only the new key); 36 ranges."""
    hidden, inter, nq, nkv = 1024, 1024, 8, 2
    layers, handles, caches = _setup(pbe, 1, hidden, inter, nq, nkv, seq, seq + 64, 40 + seq)
    x = np.random.default_rng(9).standard_normal(hidden).astype(np.float32)
    n, got = _one_token(pbe, handles, x, seq)
    assert n == 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"


def test_wide_layers_with_split_projections(pbe):
    """hidden 2048, FFN 9216, 4 layers: the down projection (9 chunks of 1024) split into three K parts, the O
    projection into two."""
    hidden, inter, nq, nkv, seq = 2048, 9216, 16, 4, 200
    layers, handles, caches = _setup(pbe, 4, hidden, inter, nq, nkv, seq, 256, 17)
    x = np.random.default_rng(18).standard_normal(hidden).astype(np.float32)
    n, got = _one_token(pbe, handles, x, seq)
    assert n == 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"


def test_config3_layer_at_position_2048(pbe):
    """hidden 4096, 32 / 8 heads of 128, FFN 14336, RoPE theta 500000 at position 2048 over a
    2048-token f16 cache ~ N(0, 1)."""
    hidden, inter, nq, nkv, seq = 4096, 14336, 32, 8, 2048
    layers, handles, caches = _setup(pbe, 1, hidden, inter, nq, nkv, seq, 2304, 7)
    x = np.random.default_rng(8).standard_normal(hidden).astype(np.float32)
    n, got = _one_token(pbe, handles, x, seq)
    assert n == 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"


def test_repeatable_and_replays_in_a_graph(pbe):
    """Bit-identical on repeated calls and in CUDA graph replays, and within the oracle bound."""
    import torch
    hidden, inter, nq, nkv, seq = 1024, 2048, 8, 2, 100
    layers, handles, caches = _setup(pbe, 2, hidden, inter, nq, nkv, seq, 128, 4)
    x0 = np.random.default_rng(5).standard_normal(hidden).astype(np.float32)
    outs = [_one_token(pbe, handles, x0, seq)[1] for _ in range(2)]
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    xd = torch.from_numpy(x0.copy()).cuda()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        pbe.decode_token_dev(handles, xd, seq, THETA, stream=stream.cuda_stream)
    for _ in range(2):
        xd.copy_(torch.from_numpy(x0))
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(xd.cpu().numpy().view(np.uint32), outs[0].view(np.uint32))
    del g
    ref = _oracle_token(layers, caches, x0, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(outs[0], ref)
    assert ok, f"max err {err} > {bound}"


def test_unserved_shapes_fall_back_to_the_pipeline(pbe):
    """hidden 1280 (not a multiple of 1024) runs the per-kernel pipeline: several launches, same bound."""
    hidden, inter, nq, nkv, seq = 1280, 1024, 8, 2, 20
    layers, handles, caches = _setup(pbe, 1, hidden, inter, nq, nkv, seq, 32, 6)
    x = np.random.default_rng(7).standard_normal(hidden).astype(np.float32)
    n, got = _one_token(pbe, handles, x, seq)
    assert n > 1
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"
