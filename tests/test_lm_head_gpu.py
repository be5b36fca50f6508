"""lm-head KNN on the GPU vs the CPU oracle.

Reference: VectorIndex::lm_head_knn_backend, its Q4 branch (crates/larql-vindex/src/index/walk.rs:549-583):
quantize_to_q8(query) (q4_common.rs:28-44), the Q4_0 x Q8 matvec over the vocab (q4_dot.c:169-199), then the
top_k logits by signed value, descending (walk.rs:566-577).

Parity: the selection is exact — the ids and logits the GPU returns equal, bit for bit, the oracle's top-k
(ties by lower id) of the logits the GPU's own Q4_0 x Q8 matvec produces; against the oracle's logits, the id
sets agree except for logits within TIE of the k-th, and the logits agree within 1e-3 * ||logits||_inf (the
matvec tolerance).
"""
import numpy as np
import pytest

import oracle as O
from conftest import normal, seed_for

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")

TIE = 1e-5


def _oracle_order(v: np.ndarray, k: int):
    """Ids of the k largest values, descending, ties by lower id, NaN below -inf (the kernel's order)."""
    ids = np.arange(v.size)
    nan = np.isnan(v)
    key = np.where(nan, -np.inf, v.astype(np.float64))
    order = np.lexsort((ids, nan, -key))  # last key sorts first: value desc, then non-NaN first, then id
    return order[:k]


def _check_against_oracle_logits(ids, vals, ref, k, what):
    a = ref.astype(np.float64)
    order = np.argsort(-a, kind="stable")
    kth = a[order[k - 1]]
    tie = TIE * max(1.0, float(np.max(np.abs(a))))
    gi = ids.astype(np.int64)
    assert len(set(gi.tolist())) == k, f"{what}: duplicate ids"
    assert np.all(a[gi] >= kth - tie), f"{what}: {gi[a[gi] < kth - tie]} are not in the top {k}"
    must = set(np.nonzero(a > kth + tie)[0].tolist())
    assert must <= set(gi.tolist()), f"{what}: missing {sorted(must - set(gi.tolist()))}"
    np.testing.assert_allclose(vals, ref[gi], rtol=0, atol=1e-3 * float(np.max(np.abs(a))), err_msg=what)
    assert np.all(np.diff(vals) <= 0), f"{what}: not descending"


@pytest.mark.parametrize("vocab,hidden,k", [(1000, 256, 10), (32000, 2048, 20), (50257, 768, 32), (7, 64, 10),
                                            (128256, 4096, 10)])
def test_lm_head_knn_matches_oracle(backend, vocab, hidden, k):
    w = O.quantize_q4_0(normal(seed_for("lmhead", vocab, hidden), vocab * hidden, 0.02))
    q = normal(seed_for("lmhead-q", vocab, hidden), hidden)
    res = backend.lm_head_knn(w, q, vocab, hidden, k)
    assert res is not None
    ids, vals = res
    kk = min(k, vocab)
    assert ids.shape == (kk,) and vals.shape == (kk,)
    # exact selection over the GPU's own logits (same device quantizer and matvec, deterministic)
    q8, s8 = O.quantize_to_q8(q)
    gpu_logits = backend.q4_matvec(w, q8, s8, vocab, hidden)
    ri, rv = O.top_k_signed(gpu_logits, k)
    assert np.array_equal(ids, ri.astype(np.int64)), f"ids {ids} vs {ri}"
    assert np.array_equal(vals.view(np.uint32), rv.view(np.uint32))
    # against the oracle's logits
    _, _, ref_logits = O.lm_head_knn(w, q, vocab, hidden, k)
    _check_against_oracle_logits(ids, vals, ref_logits, kk, f"lm-head {vocab}x{hidden} k{k}")


def test_lm_head_knn_device_api_repeats(backend):
    import torch
    vocab, hidden, k = 20000, 1024, 16
    w = O.quantize_q4_0(normal(3, vocab * hidden, 0.02))
    q = normal(4, hidden)
    wt = backend.register_weight(w, L.FMT_Q4_0, vocab, hidden)
    try:
        qd = torch.from_numpy(q).cuda()
        outs = []
        for _ in range(3):
            ids = torch.full((k,), 7, dtype=torch.int32, device="cuda")
            vals = torch.zeros(k, dtype=torch.float32, device="cuda")
            backend.lm_head_knn_dev(wt, qd, k, ids, vals)
            backend.sync()
            outs.append((ids.cpu().numpy().view(np.uint32).copy(), vals.cpu().numpy().copy()))
    finally:
        wt.release()
    for i, v in outs[1:]:
        assert np.array_equal(i, outs[0][0]) and np.array_equal(v.view(np.uint32), outs[0][1].view(np.uint32))
    q8, s8 = O.quantize_to_q8(q)
    ri, rv = O.top_k_signed(backend.q4_matvec(w, q8, s8, vocab, hidden), k)
    assert np.array_equal(outs[0][0], ri) and np.array_equal(outs[0][1].view(np.uint32), rv.view(np.uint32))


def _topk_dev(backend, v: np.ndarray, k: int):
    import torch
    kk = min(k, v.size)
    d = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).cuda()
    ids = torch.zeros(kk, dtype=torch.int32, device="cuda")
    out = torch.zeros(kk, dtype=torch.float32, device="cuda")
    backend.logit_topk_dev(d, v.size, k, ids, out)
    backend.sync()
    return ids.cpu().numpy().view(np.uint32).astype(np.int64), out.cpu().numpy()


def _cases():
    rng = np.random.default_rng(11)
    c = {}
    c["random_262144"] = rng.standard_normal(262144).astype(np.float32)
    c["ascending"] = np.arange(100000, dtype=np.float32)  # every candidate beats the list: worst-case insertions
    c["descending"] = -np.arange(100000, dtype=np.float32)
    c["all_equal"] = np.full(5000, 0.25, np.float32)  # ties by lower id: ids 0..k-1
    c["few_levels"] = rng.integers(0, 3, 70001).astype(np.float32)  # ties across warp ranges
    v = rng.standard_normal(4099).astype(np.float32)
    v[[5, 600, 4000]] = np.inf
    v[[7, 8]] = -np.inf
    v[100:3000:7] = np.nan
    c["specials"] = v
    c["signed_zeros"] = np.array([0.0, -0.0, 1e-45, -1e-45, 0.0, -0.0] * 10, np.float32)
    c["one"] = np.array([3.5], np.float32)
    c["tiny_vocab"] = rng.standard_normal(19).astype(np.float32)
    c["nan_heavy"] = np.where(rng.random(3000) < 0.999, np.nan, rng.standard_normal(3000)).astype(np.float32)
    return c


@pytest.mark.parametrize("name", list(_cases().keys()))
@pytest.mark.parametrize("k", [1, 10, 32])
def test_logit_topk_edges(backend, name, k):
    v = _cases()[name]
    ids, out = _topk_dev(backend, v, k)
    want = _oracle_order(v, min(k, v.size))
    assert np.array_equal(ids, want), f"{name} k{k}: {ids} vs {want}"
    ref = v[want]
    same = (out.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(out) & np.isnan(ref))
    assert np.all(same), f"{name} k{k}: values {out} vs {ref}"
    if not np.isnan(v).any():
        ri, rv = O.top_k_signed(v, k)
        assert np.array_equal(ids, ri.astype(np.int64))


def test_lm_head_knn_unsupported_and_shapes(backend):
    vocab, hidden = 100, 256
    w = O.quantize_q4_0(normal(21, vocab * hidden, 0.02))
    q = normal(22, hidden)
    assert backend.lm_head_knn(w, q, vocab, hidden, 0) is None  # the reference returns every logit sorted
    assert backend.lm_head_knn(w, q, vocab, hidden, 33) is None
    small = O.quantize_q4_0(normal(23, 20 * hidden, 0.02))
    ids, vals = backend.lm_head_knn(small, q, 20, hidden, 50)  # top_k >= vocab: every logit, sorted
    ri, rv = O.top_k_signed(backend.q4_matvec(small, *O.quantize_to_q8(q), 20, hidden), 50)
    assert ids.size == 20 and np.array_equal(ids, ri.astype(np.int64))
    odd = O.quantize_q4_0(normal(24, vocab * 96, 0.02))
    assert backend.lm_head_knn(odd, normal(25, 96), vocab, 96, 5) is None  # hidden % 64 != 0
