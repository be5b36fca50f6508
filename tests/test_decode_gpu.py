"""One-token decode through Llama-style Q4_K layers with an f16 KV cache, on the GPU vs the oracle composite of the
reference CPU pieces (rms_norm_eps residual.rs:17-35, q4k_matvec.rs:31-87, apply_rope_partial rope.rs:22-55,
gqa_attention gqa.rs:29-110, silu_gate_up ffn/mod.rs:87-94).  Tolerance: max |err| <= 1e-3 * ||x_ref||_inf."""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")
THETA = 500000.0


def _q4k(rng, rows, cols):
    out = np.empty(rows * cols // 256 * 148, np.uint8)
    step = max(1, (1 << 24) // cols) // 256 * 256 or 256
    for r in range(0, rows, step):
        m = min(step, rows - r)
        out[r * cols // 256 * 148:(r + m) * cols // 256 * 148] = O.quantize_q4_k(
            rng.standard_normal(m * cols, dtype=np.float32) * np.float32(0.02))
    return out


def _layer(rng, hidden, inter, nq, nkv, hd=128):
    qd, kvd = nq * hd, nkv * hd
    w = {"q": _q4k(rng, qd, hidden), "k": _q4k(rng, kvd, hidden), "v": _q4k(rng, kvd, hidden),
         "o": _q4k(rng, hidden, qd), "gate": _q4k(rng, inter, hidden), "up": _q4k(rng, inter, hidden),
         "down": _q4k(rng, hidden, inter)}
    norms = [(1.0 + rng.standard_normal(hidden) * 0.02).astype(np.float32) for _ in range(2)]
    return w, norms


def _setup(be, n_layers, hidden, inter, nq, nkv, seq, max_seq, seed):
    rng = np.random.default_rng(seed)
    hd, kvd = 128, nkv * 128
    layers, handles, caches = [], [], []
    be.kv_init(n_layers, max_seq, nkv, hd)
    for l in range(n_layers):
        w, (n1, n2) = _layer(rng, hidden, inter, nq, nkv)
        layers.append((w, n1, n2))
        handles.append(be.layer_register(w, n1, n2, hidden, inter, nq, nkv, hd, eps=1e-5))
        k = rng.standard_normal((seq, kvd), dtype=np.float32)
        v = rng.standard_normal((seq, kvd), dtype=np.float32)
        be.kv_populate(l, k, v, seq)
        kc = np.zeros((max_seq, kvd), np.uint16)
        vc = np.zeros((max_seq, kvd), np.uint16)
        kc[:seq] = k.astype(np.float16).view(np.uint16)
        vc[:seq] = v.astype(np.float16).view(np.uint16)
        caches.append((kc, vc))
    return layers, handles, caches


def _oracle_token(layers, caches, x, hidden, inter, nq, nkv, pos):
    for (w, n1, n2), (kc, vc) in zip(layers, caches):
        x = O.decode_layer(x, hidden, inter, nq, nkv, 128, w, n1, n2, 0.0, 1e-5, 1.0 / np.sqrt(128), THETA, kc, vc, pos)
    return x


def test_small_two_layers_three_tokens(backend):
    hidden, inter, nq, nkv, seq = 1024, 2048, 8, 2, 37
    be = backend
    layers, handles, caches = _setup(be, 2, hidden, inter, nq, nkv, seq, 64, 1)
    rng = np.random.default_rng(2)
    for t in range(3):
        x = rng.standard_normal(hidden).astype(np.float32)
        assert be.kv_length() == seq + t
        got = be.decode_token(handles, x, THETA)
        ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq + t)
        ok, err, bound = max_err_ok(got, ref)
        assert ok, f"token {t}: max err {err} > {bound}"
    for h in handles:
        be.layer_release(h)


@pytest.mark.parametrize("nq,nkv", [(8, 8), (8, 4), (16, 2)])
def test_gqa_ratios(backend, nq, nkv):
    hidden, inter, seq = 1024, 1024, 300
    layers, handles, caches = _setup(backend, 1, hidden, inter, nq, nkv, seq, 512, nq * 10 + nkv)
    x = np.random.default_rng(3).standard_normal(hidden).astype(np.float32)
    got = backend.decode_token(handles, x, THETA)
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"
    for h in handles:
        backend.layer_release(h)


@pytest.mark.parametrize("seq", [1, 4500])
def test_cache_lengths_short_and_multi_chunk(backend, seq):
    """Two keys (most of a KV head's CTAs hold none) and 4501 keys (each CTA walks several
    shared-memory sub-chunks with the online softmax)."""
    hidden, inter, nq, nkv = 1024, 1024, 8, 2
    layers, handles, caches = _setup(backend, 1, hidden, inter, nq, nkv, seq, seq + 64, 40 + seq)
    x = np.random.default_rng(9).standard_normal(hidden).astype(np.float32)
    got = backend.decode_token(handles, x, THETA)
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"
    for h in handles:
        backend.layer_release(h)


def test_unfused_path_on_the_cuda_core_matvec(monkeypatch):
    """With the CUDA-core Q4_K kernel selected (LARQL_CUDA_Q4K_PATH=dp4a) the layer runs as separate
    RMSNorm / SiLU kernels around the projections instead of the fused warp-MMA prologues."""
    monkeypatch.setenv("LARQL_CUDA_Q4K_PATH", "dp4a")
    be = L.CudaBackend(0)
    try:
        hidden, inter, nq, nkv, seq = 1024, 2048, 8, 2, 50
        layers, handles, caches = _setup(be, 2, hidden, inter, nq, nkv, seq, 64, 11)
        x = np.random.default_rng(12).standard_normal(hidden).astype(np.float32)
        got = be.decode_token(handles, x, THETA)
        ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
        ok, err, bound = max_err_ok(got, ref)
        assert ok, f"max err {err} > {bound}"
    finally:
        be.close()


@pytest.mark.parametrize("cfg", ["8,1,0,1,0", "4,2,0,1,0", "4,1,0,2,0"])
def test_fused_decode_on_each_epilogue_form(monkeypatch, cfg):
    """The norm / SiLU prologues and the residual + sum-of-squares epilogue on each output form of the MMA matvec
    (LARQL_CUDA_MMA_CFG pins groups, K slices, stages, K parts): one slice and one part (row groups write directly),
    two K slices (summed through shared memory), two K parts (the last CTA of a tile adds them)."""
    monkeypatch.setenv("LARQL_CUDA_MMA_CFG", cfg)
    monkeypatch.setenv("LARQL_CUDA_DECODE_FUSE", "3")
    be = L.CudaBackend(0)
    try:
        hidden, inter, nq, nkv, seq = 2048, 2048, 16, 4, 40
        layers, handles, caches = _setup(be, 2, hidden, inter, nq, nkv, seq, 64, 21)
        rng = np.random.default_rng(22)
        for t in range(2):
            x = rng.standard_normal(hidden).astype(np.float32)
            got = be.decode_token(handles, x, THETA)
            ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq + t)
            ok, err, bound = max_err_ok(got, ref)
            assert ok, f"{cfg} token {t}: max err {err} > {bound}"
    finally:
        be.close()


@pytest.mark.parametrize("mask", ["1", "2"])
def test_single_decode_fusions(monkeypatch, mask):
    """LARQL_CUDA_DECODE_FUSE=1 (SiLU into the down matvec only) and =2 (norm + residual only)."""
    monkeypatch.setenv("LARQL_CUDA_DECODE_FUSE", mask)
    be = L.CudaBackend(0)
    try:
        hidden, inter, nq, nkv, seq = 1024, 2048, 8, 2, 50
        layers, handles, caches = _setup(be, 2, hidden, inter, nq, nkv, seq, 64, 31)
        x = np.random.default_rng(32).standard_normal(hidden).astype(np.float32)
        got = be.decode_token(handles, x, THETA)
        ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
        ok, err, bound = max_err_ok(got, ref)
        assert ok, f"max err {err} > {bound}"
    finally:
        be.close()


def test_config3_layer_at_position_2048(backend):
    """hidden 4096, 32 / 8 heads of 128, FFN 14336, RoPE theta 500000 at position 2048 over a
    2048-token f16 cache ~ N(0, 1)."""
    hidden, inter, nq, nkv, seq = 4096, 14336, 32, 8, 2048
    layers, handles, caches = _setup(backend, 1, hidden, inter, nq, nkv, seq, 2304, 7)
    x = np.random.default_rng(8).standard_normal(hidden).astype(np.float32)
    got = backend.decode_token(handles, x, THETA)
    ref = _oracle_token(layers, caches, x, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(got, ref)
    assert ok, f"max err {err} > {bound}"
    for h in handles:
        backend.layer_release(h)


def test_device_form_is_repeatable_and_keeps_length(backend):
    import torch
    hidden, inter, nq, nkv, seq = 1024, 1024, 8, 2, 100
    layers, handles, caches = _setup(backend, 2, hidden, inter, nq, nkv, seq, 128, 4)
    x0 = np.random.default_rng(5).standard_normal(hidden).astype(np.float32)
    outs = []
    for _ in range(2):
        xd = torch.from_numpy(x0.copy()).cuda()
        backend.decode_token_dev(handles, xd, seq, THETA)
        backend.sync()
        outs.append(xd.cpu().numpy())
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert backend.kv_length() == seq
    ref = _oracle_token(layers, caches, x0, hidden, inter, nq, nkv, seq)
    ok, err, bound = max_err_ok(outs[0], ref)
    assert ok, f"max err {err} > {bound}"
    for h in handles:
        backend.layer_release(h)


def test_rejections(backend):
    rng = np.random.default_rng(6)
    w, (n1, n2) = _layer(rng, 1024, 1024, 8, 2)
    with pytest.raises(L.LarqlCudaError) as e:
        backend.layer_register(w, n1, n2, 1024, 1024, 8, 2, head_dim=64)
    assert e.value.status == L.ERR_UNSUPPORTED
    backend.kv_init(1, 16, 2)
    h = backend.layer_register(w, n1, n2, 1024, 1024, 8, 2)
    backend.kv_set_length(16)
    with pytest.raises(L.LarqlCudaError) as e:
        backend.decode_token([h], np.zeros(1024, np.float32), THETA)
    assert e.value.status == L.ERR_BAD_SHAPE
    backend.layer_release(h)


def test_sharded_decode_two_ranks_on_one_gpu():
    """Tensor-parallel decode (heads and FFN rows over 2 ranks) emulated on one GPU: two contexts, two host
    threads, the all-reduce done by the test (device sync, sum, copy back) between the ranks' partial sums."""
    import threading
    import torch
    hidden, inter, nq, nkv, seq, world = 1024, 2048, 8, 2, 40, 2
    rng = np.random.default_rng(21)
    full = [_layer(rng, hidden, inter, nq, nkv) for _ in range(2)]
    kvd, kvd_l = nkv * 128, nkv // world * 128
    caches = []
    for _ in full:
        k = rng.standard_normal((seq, kvd), dtype=np.float32)
        v = rng.standard_normal((seq, kvd), dtype=np.float32)
        caches.append((k, v))
    x0 = rng.standard_normal(hidden).astype(np.float32)
    bes, hss = [], []
    for r in range(world):
        be = L.CudaBackend(0)
        be.kv_init(2, seq + 8, nkv // world, 128)
        hs = []
        for l, (w, (n1, n2)) in enumerate(full):
            hs.append(be.layer_register_shard(w, n1, n2, hidden, inter, nq, nkv, r, world, eps=1e-5))
            k, v = caches[l]
            be.kv_populate(l, np.ascontiguousarray(k[:, r * kvd_l:(r + 1) * kvd_l]),
                           np.ascontiguousarray(v[:, r * kvd_l:(r + 1) * kvd_l]), seq)
        bes.append(be)
        hss.append(hs)
    xs = [torch.from_numpy(x0.copy()).cuda() for _ in range(world)]
    reds = [torch.zeros(hidden, dtype=torch.float32, device="cuda") for _ in range(world)]
    total = torch.zeros(hidden, dtype=torch.float32, device="cuda")
    bar = threading.Barrier(world, timeout=120)
    calls = [0, 0]

    def make_reduce(r):
        def reduce(buf, n, stream):
            assert n == hidden and buf == reds[r].data_ptr()
            calls[r] += 1
            torch.cuda.synchronize()  # this rank's partial is complete
            bar.wait()
            if r == 0:
                total.copy_(reds[0] + reds[1])
                torch.cuda.synchronize()
            bar.wait()
            reds[r].copy_(total)
            torch.cuda.synchronize()
            bar.wait()
            return 0
        return reduce

    errs = []

    def run(r):
        try:
            bes[r].decode_token_sharded_dev(hss[r], xs[r], seq, THETA, reds[r], make_reduce(r))
            bes[r].sync()
        except Exception as e:  # noqa: BLE001
            errs.append(e)
            bar.abort()

    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(300)
    try:
        assert not errs, errs
        assert calls == [4, 4]  # two reductions per layer
        got = [x.cpu().numpy() for x in xs]
        assert np.array_equal(got[0].view(np.uint32), got[1].view(np.uint32))
        kc = [np.zeros((seq + 8, kvd), np.uint16) for _ in full]
        vc = [np.zeros((seq + 8, kvd), np.uint16) for _ in full]
        for l, (k, v) in enumerate(caches):
            kc[l][:seq] = k.astype(np.float16).view(np.uint16)
            vc[l][:seq] = v.astype(np.float16).view(np.uint16)
        layers = [(w, n1, n2) for (w, (n1, n2)) in full]
        ref = _oracle_token(layers, list(zip(kc, vc)), x0, hidden, inter, nq, nkv, seq)
        ok, err, bound = max_err_ok(got[0], ref)
        assert ok, f"max err {err} > {bound}"
    finally:
        for be in bes:
            be.close()
