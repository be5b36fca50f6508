"""vindex gate walk on the GPU vs the CPU oracle.

Reference: crates/larql-vindex/src/index/gate.rs:108-134 (scores = G . r, G f16 rows decoded by
crates/larql-models/src/quant/half.rs) and :307-316 (top-K by |score| descending).
Parity (north star): top-K index sets identical except for ties within 1e-5; the oracle scores in f64.
"""
import numpy as np
import pytest

import oracle as O
from conftest import seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")
TIE = 1e-5


def _gates(seed, n, sigma=0.02, chunk=1 << 24):
    """n f16 gate values ~ N(0, sigma), generated in f32 chunks (the config-5 matrix is 891 M values)."""
    rng = np.random.default_rng(seed)
    out = np.empty(n, np.float16)
    for i in range(0, n, chunk):
        m = min(chunk, n - i)
        out[i:i + m] = rng.standard_normal(m, dtype=np.float32) * np.float32(sigma)
    return out.view(np.uint16)


def _check_layer(got_i, got_s, ref, k, what):
    """got_*: [k] for one (layer, query); ref: oracle scores [n_feat]."""
    a = np.abs(ref.astype(np.float64))
    n = a.size
    kk = min(k, n)
    order = np.argsort(-a, kind="stable")
    kth = a[order[kk - 1]]
    gi = got_i[:kk].astype(np.int64)
    assert np.all(gi < n), f"{what}: index out of range {gi}"
    assert len(set(gi.tolist())) == kk, f"{what}: duplicate indices {gi}"
    assert np.all(a[gi] >= kth - TIE), f"{what}: {gi[a[gi] < kth - TIE]} are not top-{k} (k-th |score| {kth})"
    must = set(np.nonzero(a > kth + TIE)[0].tolist())
    assert must <= set(gi.tolist()), f"{what}: missing {sorted(must - set(gi.tolist()))}"
    np.testing.assert_allclose(got_s[:kk], ref[gi], rtol=0, atol=2e-5 * max(1.0, a.max()), err_msg=what)
    assert np.all(np.diff(np.abs(got_s[:kk])) <= 1e-6 * max(1.0, a.max())), f"{what}: not sorted by |score|"
    if k > n:
        assert np.all(got_i[n:] == 0xFFFFFFFF)


def _run_and_check(backend, g, nl, nf, hidden, q, k, what, layers=None, queries=None):
    res = backend.gate_topk_f16(g, nl, nf, hidden, q, k)
    assert res is not None
    idx, sc = res
    b = q.reshape(-1, hidden).shape[0]
    assert idx.shape == (nl, b, k)
    g2 = g.reshape(nl, nf * hidden)
    for l in (range(nl) if layers is None else layers):
        qs = range(b) if queries is None else queries
        ref = O.gate_scores_f16(g2[l], q.reshape(-1, hidden)[list(qs)], nf, hidden)
        for j, qi in enumerate(qs):
            _check_layer(idx[l, qi], sc[l, qi], ref[j], k, f"{what} layer {l} query {qi}")
    return idx, sc


def test_vindex_known_answers_padded():
    """crates/larql-vindex/tests/test_vindex.rs:27-61,134-190, zero-padded from hidden 4 to 64."""
    be = L.CudaBackend(0)
    try:
        g0 = np.zeros((3, 64), np.float32)
        g0[0, 0] = g0[1, 1] = g0[2, 2] = 1.0
        g1 = np.zeros((3, 64), np.float32)
        g1[0, 3] = 1.0
        g1[1, 0] = g1[1, 1] = 0.5
        g1[2, 2] = -1.0
        g = np.concatenate([g0, g1]).astype(np.float16).view(np.uint16)
        q = np.zeros((3, 64), np.float32)
        q[0, 0] = 1.0
        q[1, :2] = [0.8, 0.6]
        q[2, 2] = 1.0
        idx, sc = be.gate_topk_f16(g, 2, 3, 64, q, 3)
        assert idx[0, 0, 0] == 0 and abs(sc[0, 0, 0] - 1.0) < 0.01          # best match
        assert idx[0, 1, :2].tolist() == [0, 1]                                # ordering
        assert idx[1, 0, 0] == 1                                               # layer 1, dim 0 -> 0.5
        assert idx[1, 2, 0] == 2 and sc[1, 2, 0] == -1.0                       # |score| ranking, sign kept
    finally:
        be.close()


@pytest.mark.parametrize("nl,nf,hidden,b,k", [(3, 1000, 2560, 1, 10), (2, 700, 512, 5, 16), (1, 300, 64, 130, 1),
                                              (2, 4096, 1024, 64, 10), (1, 257, 256, 300, 7), (2, 9, 128, 3, 16)])
def test_random_gates(backend, nl, nf, hidden, b, k):
    g = _gates(seed_for("gate", nl, nf, hidden), nl * nf * hidden)
    q = np.random.default_rng(seed_for("gq", b)).standard_normal((b, hidden)).astype(np.float32)
    _run_and_check(backend, g, nl, nf, hidden, q, k, f"random {nl}x{nf}x{hidden} b{b}",
                   queries=None if b <= 64 else list(range(0, b, 7)) + [b - 1])


def test_subnormal_gates_follow_half_rs(backend):
    """Gate values in the f16 subnormal range: half.rs decodes them to half their IEEE value (exact here: all
    |g| < 32768, so the device stores 2 g)."""
    nl, nf, hidden, b, k = 1, 600, 256, 4, 10
    rng = np.random.default_rng(3)
    g = rng.integers(1, 0x400, nl * nf * hidden).astype(np.uint16) | (rng.integers(0, 2, nl * nf * hidden).astype(np.uint16) << 15)
    q = rng.standard_normal((b, hidden)).astype(np.float32) * np.float32(1e4)
    _run_and_check(backend, g, nl, nf, hidden, q, k, "subnormal")


def test_large_gates_use_rounded_subnormals(backend):
    """A gate value >= 32768 rules out the doubled copy; subnormals are then rounded to their half.rs value
    (<= 2^-25 each), far inside the tie tolerance at these magnitudes."""
    nl, nf, hidden, b, k = 1, 300, 128, 2, 10
    rng = np.random.default_rng(6)
    g = (rng.standard_normal(nl * nf * hidden) * 0.02).astype(np.float16)
    g[rng.integers(0, g.size, 200)] = np.float16(3e-6)   # subnormal
    g[7] = np.float16(40000.0)
    q = rng.standard_normal((b, hidden)).astype(np.float32)
    _run_and_check(backend, g.view(np.uint16), nl, nf, hidden, q, k, "large gates")


def test_wide_range_queries(backend):
    nl, nf, hidden, b, k = 1, 512, 512, 3, 10
    g = _gates(4, nl * nf * hidden)
    rng = np.random.default_rng(5)
    q = (rng.standard_normal((b, hidden)) * np.exp2(rng.integers(-20, 20, (b, hidden)))).astype(np.float32)
    q[1] *= np.float32(1e20)
    q[2] *= np.float32(1e-20)
    _run_and_check(backend, g, nl, nf, hidden, q, k, "wide range")


C5 = dict(nl=34, nf=10240, hidden=2560, k=10)


@pytest.fixture(scope="module")
def config5_gates():
    """BASELINE configs[4] gates: 34 layers x 10240 rows x 2560 f16 ~ N(0, 0.02) (1.78 GB, generated once)."""
    return _gates(11, C5["nl"] * C5["nf"] * C5["hidden"])


def test_config5_sample(backend, config5_gates):
    """BASELINE configs[4] shape: 34 layers x 10240 gates x 2560 f16 ~ N(0, 0.02), batch 64, top-10;
    every layer for query 0, every query for two layers."""
    nl, nf, hidden, b, k = 34, 10240, 2560, 64, 10
    g = config5_gates
    q = np.random.default_rng(12).standard_normal((b, hidden)).astype(np.float32)
    idx, sc = _run_and_check(backend, g, nl, nf, hidden, q, k, "config5", layers=range(nl), queries=[0])
    g2 = g.reshape(nl, nf * hidden)
    for l in (5, 33):
        ref = O.gate_scores_f16(g2[l], q, nf, hidden)
        for qi in range(b):
            _check_layer(idx[l, qi], sc[l, qi], ref[qi], k, f"config5 layer {l} query {qi}")


def test_device_api_and_repeat(backend):
    import torch
    nl, nf, hidden, b, k = 2, 1000, 1024, 8, 10
    g = _gates(21, nl * nf * hidden)
    wt = backend.register_weight(g, L.FMT_F16_HALFRS, nl * nf, hidden)
    q = torch.randn(b, hidden, device="cuda")
    oi = torch.empty(nl * b * k, dtype=torch.int32, device="cuda")
    os_ = torch.empty(nl * b * k, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.gate_topk_dev(wt, nl, nf, q, b, k, oi, os_)
    backend.sync()
    i1, s1 = oi.cpu().numpy().copy(), os_.cpu().numpy().copy()
    backend.gate_topk_dev(wt, nl, nf, q, b, k, oi, os_)
    backend.sync()
    assert np.array_equal(i1, oi.cpu().numpy()) and np.array_equal(s1.view(np.uint32), os_.cpu().numpy().view(np.uint32))
    qh = q.cpu().numpy()
    g2 = g.reshape(nl, nf * hidden)
    for l in range(nl):
        ref = O.gate_scores_f16(g2[l], qh, nf, hidden)
        for qi in range(b):
            o = (l * b + qi) * k
            _check_layer(i1[o:o + k].view(np.uint32), s1[o:o + k], ref[qi], k, f"dev layer {l} query {qi}")
    wt.release()


def test_unsupported_shapes(backend):
    g = _gates(1, 2 * 100 * 96)
    assert backend.gate_topk_f16(g, 2, 100, 96, np.ones(96, np.float32), 10) is None      # hidden % 64
    g = _gates(1, 2 * 100 * 128)
    assert backend.gate_topk_f16(g, 2, 100, 128, np.ones(128, np.float32), 17) is None    # top_k > 16


def test_sharded_gate_walk_merge(backend):
    """Gate rows of every layer split into 4 row shards (one per GPU in the multi-GPU walk), each shard's
    top-k computed on its own, candidates merged with the shard offsets: equals the unsharded walk."""
    import torch
    nl, nf, hidden, b, k, shards = 3, 2048, 512, 5, 10, 4
    g = _gates(31, nl * nf * hidden).reshape(nl, nf, hidden)
    q = np.random.default_rng(32).standard_normal((b, hidden)).astype(np.float32)
    fs = nf // shards
    qd = torch.from_numpy(q).cuda()
    ci = torch.empty(shards * nl * b * k, dtype=torch.int32, device="cuda")
    cs = torch.empty(shards * nl * b * k, dtype=torch.float32, device="cuda")
    ws = []
    for s in range(shards):
        ws.append(backend.register_weight(np.ascontiguousarray(g[:, s * fs:(s + 1) * fs]).reshape(-1), L.FMT_F16_HALFRS,
                                          nl * fs, hidden))
        o = s * nl * b * k
        backend.gate_topk_dev(ws[-1], nl, fs, qd, b, k, ci[o:], cs[o:])
    offs = torch.tensor([s * fs for s in range(shards)], dtype=torch.int32, device="cuda")
    oi = torch.empty(nl * b * k, dtype=torch.int32, device="cuda")
    os_ = torch.empty(nl * b * k, dtype=torch.float32, device="cuda")
    backend.topk_merge_dev(ci, cs, shards, nl * b, k, k, oi, os_, offsets=offs)
    backend.sync()
    mi, ms = oi.cpu().numpy().view(np.uint32).reshape(nl, b, k), os_.cpu().numpy().reshape(nl, b, k)
    for l in range(nl):
        ref = O.gate_scores_f16(g[l].reshape(-1), q, nf, hidden)
        for qi in range(b):
            _check_layer(mi[l, qi], ms[l, qi], ref[qi], k, f"sharded layer {l} query {qi}")
    for w in ws:
        w.release()


def test_gate_scores_batch_matches_oracle(backend):
    """gate_scores_batch (gate.rs:545-559): every score of a partial query block against partial row tiles of
    two layers, including f16 subnormal gate values (half.rs decoding)."""
    nl, nf, hidden, b = 2, 300, 128, 37
    g = _gates(seed_for("gsb", nl, nf), nl * nf * hidden).copy()
    g[::97] = np.arange(len(g[::97]), dtype=np.uint16) % 1023 + 1  # subnormal bit patterns
    q = np.random.default_rng(5).standard_normal((b, hidden)).astype(np.float32)
    got = backend.gate_scores_f16(g, nl, nf, hidden, q)
    assert got is not None and got.shape == (nl, b, nf)
    g2 = g.reshape(nl, nf * hidden)
    for l in range(nl):
        ref = O.gate_scores_f16(g2[l], q, nf, hidden)
        np.testing.assert_allclose(got[l], ref, rtol=0, atol=2e-5 * max(1.0, float(np.abs(ref).max())))


def test_gate_scores_dev_on_registered_weight(backend):
    import torch
    nl, nf, hidden, b = 1, 520, 64, 5
    g = _gates(seed_for("gsd", nf), nf * hidden)
    q = np.random.default_rng(6).standard_normal((b, hidden)).astype(np.float32)
    w = backend.register_weight(g, L.FMT_F16_HALFRS, nl * nf, hidden)
    qd = torch.from_numpy(q).cuda()
    out = torch.empty(nl * b * nf, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.gate_scores_dev(w, nl, nf, qd, b, out)
    backend.sync()
    w.release()
    ref = O.gate_scores_f16(g, q, nf, hidden)
    np.testing.assert_allclose(out.cpu().numpy().reshape(b, nf), ref, rtol=0,
                               atol=2e-5 * max(1.0, float(np.abs(ref).max())))


@pytest.mark.parametrize("seq,top_k,nf", [(1, 10, 1000), (12, 10, 1000), (40, 16, 4096), (3, 8, 5)])
def test_gate_knn_batch_union(backend, seq, top_k, nf):
    """gate_knn_batch (gate.rs:500-537): the sorted union of the per-position top-k; membership may differ
    only for features within 1e-5 of a position's k-th |score|."""
    hidden = 128
    g = _gates(seed_for("gkb", seq, nf), nf * hidden)
    x = np.random.default_rng(seq + nf).standard_normal((seq, hidden)).astype(np.float32)
    got = backend.gate_knn_batch_f16(g, nf, hidden, x, top_k)
    assert got is not None
    assert np.all(np.diff(got) > 0), "not sorted and unique"
    ref = np.abs(O.gate_scores_f16(g, x, nf, hidden).astype(np.float64))
    k = min(top_k, nf)
    must, allowed = set(), set()
    for s in range(seq):
        kth = np.sort(ref[s])[::-1][k - 1]
        must |= set(np.nonzero(ref[s] > kth + TIE)[0].tolist())
        allowed |= set(np.nonzero(ref[s] >= kth - TIE)[0].tolist())
    gs = set(got.tolist())
    assert must <= gs, f"missing {sorted(must - gs)[:10]}"
    assert gs <= allowed, f"unexpected {sorted(gs - allowed)[:10]}"


@pytest.mark.parametrize("b", [1, 2, 3, 4])
@pytest.mark.parametrize("nf,hidden,k", [(1000, 2560, 10), (333, 512, 16), (5, 768, 8)])
def test_small_batches_on_cuda_cores(backend, b, nf, hidden, k):
    """One to four queries with hidden % 256 == 0 take the CUDA-core walk (gate_gemv.cu): uneven row ranges per
    part (1000, 333 rows) and a layer shorter than the top-k (5 rows)."""
    nl = 2
    g = _gates(seed_for("gv", b, nf, hidden), nl * nf * hidden)
    q = np.random.default_rng(seed_for("gvq", b, nf)).standard_normal(b * hidden).astype(np.float32)
    _run_and_check(backend, g, nl, nf, hidden, q, k, f"cuda-core walk b{b}")


def test_cuda_core_and_tensor_core_walks_agree(monkeypatch, backend):
    """The same small batch through both walks (LARQL_CUDA_GATE_GEMV=0 selects the tensor-core one): identical
    index sets, scores within the tie tolerance; doubled-copy gates with subnormals included."""
    nl, nf, hidden, b, k = 3, 2000, 1024, 3, 10
    g = _gates(21, nl * nf * hidden)
    rng = np.random.default_rng(22)
    g[rng.integers(0, g.size, 500)] = rng.integers(1, 0x400, 500).astype(np.uint16)  # subnormals
    q = rng.standard_normal((b, hidden)).astype(np.float32)
    i1, s1 = backend.gate_topk_f16(g, nl, nf, hidden, q, k)
    monkeypatch.setenv("LARQL_CUDA_GATE_GEMV", "0")
    be = L.CudaBackend(0)
    try:
        i2, s2 = be.gate_topk_f16(g, nl, nf, hidden, q, k)
    finally:
        be.close()
    for l in range(nl):
        for qi in range(b):
            assert set(i1[l, qi].tolist()) == set(i2[l, qi].tolist()), f"layer {l} query {qi}"
            np.testing.assert_allclose(s1[l, qi], s2[l, qi], rtol=0, atol=TIE)


def test_config5_full_shape_batch1(backend, config5_gates):
    """BASELINE configs[4] at batch 1, the timed CUDA-core route (gate_gemv.cu): the full 34 x 10240 x 2560
    walk for four separate single queries, every layer of each checked against the oracle's f64 scores
    (gate.rs:108-134) and top-10 by |score| (gate.rs:307-316), ties within 1e-5."""
    nl, nf, hidden, k = C5["nl"], C5["nf"], C5["hidden"], C5["k"]
    g2 = config5_gates.reshape(nl, nf * hidden)
    rng = np.random.default_rng(seed_for("c5b1"))
    qs = [rng.standard_normal((1, hidden)).astype(np.float32) for _ in range(4)]
    got = [backend.gate_topk_f16(config5_gates, nl, nf, hidden, q, k) for q in qs]
    for l in range(nl):
        ref = O.gate_scores_f16_many(g2[l], np.concatenate(qs), nf, hidden)
        for j, (idx, sc) in enumerate(got):
            _check_layer(idx[l, 0], sc[l, 0], ref[j], k, f"config5 batch 1 query {j} layer {l}")


def test_config5_full_shape_batch1024(backend, config5_gates):
    """BASELINE configs[4] at batch 1024, the timed tensor-core route (gate_tc.cu): one walk of 1024 queries
    over the full 34 x 10240 x 2560 gates; every layer for five queries (first, last, three inside) and every
    query for two layers, against the oracle's f64 scores and top-10 by |score|, ties within 1e-5."""
    nl, nf, hidden, k, b = C5["nl"], C5["nf"], C5["hidden"], C5["k"], 1024
    g2 = config5_gates.reshape(nl, nf * hidden)
    q = np.random.default_rng(seed_for("c5b1024")).standard_normal((b, hidden)).astype(np.float32)
    idx, sc = backend.gate_topk_f16(config5_gates, nl, nf, hidden, q, k)
    assert idx.shape == (nl, b, k)
    some = [0, 1, 333, 777, b - 1]
    for l in range(nl):
        every = l in (0, nl - 1)
        qs = list(range(b)) if every else some
        ref = O.gate_scores_f16_many(g2[l], q[qs], nf, hidden)
        for j, qi in enumerate(qs):
            _check_layer(idx[l, qi], sc[l, qi], ref[j], k, f"config5 batch 1024 layer {l} query {qi}")
