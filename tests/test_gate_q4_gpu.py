"""The Q4_0 gate walk (VectorIndex::gate_knn_q4 / gate_knn_adaptive's Q4 branch) on the GPU vs the oracle.

Reference: crates/larql-vindex/src/index/gate.rs:672-731 (quantize_to_q8 of the residual, q4_matvec over the
layer's Q4_0 gate rows, top_k_from_scores by |score|, :307-316), the Q4_0 file layout of
crates/larql-vindex/src/index/walk.rs:303-328.  Oracle: the restated quantize_to_q8 (q4_common.rs:28-44) and
q4_0_matvec_c (q4_dot.c:169-199, pinned bit-exact to the reference's compiled C), then top-K by |score|;
index sets equal except for ties within 1e-5.
"""
import numpy as np
import pytest

import oracle as O
from conftest import normal, seed_for
from vindex_util import check_topk

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")


def _layer_scores(w_layer, q, n_feat, hidden):
    q8, s8 = O.quantize_to_q8(q)
    return O.q4_0_matvec_q8(w_layer, q8, s8, n_feat, hidden)


@pytest.mark.parametrize("nl,nf,hidden,b,k", [(3, 700, 256, 1, 10), (2, 10240, 2560, 1, 10), (4, 33, 128, 5, 16),
                                              (2, 9, 64, 2, 16), (1, 5000, 1024, 3, 1)])
def test_gate_knn_q4_vs_oracle(backend, nl, nf, hidden, b, k):
    w = O.quantize_q4_0(normal(seed_for("gq4", nl, nf, hidden), nl * nf * hidden, 0.02))
    q = np.random.default_rng(seed_for("gq4x", b)).standard_normal((b, hidden)).astype(np.float32)
    res = backend.gate_knn_q4(w, nl, nf, hidden, q, k)
    assert res is not None
    idx, sc = res
    lb = nf * hidden // 32 * 18
    for l in range(nl):
        for qi in range(b):
            ref = _layer_scores(w[l * lb:(l + 1) * lb], q[qi], nf, hidden)
            check_topk(idx[l, qi], sc[l, qi], ref, k, f"Q4 gate layer {l} query {qi}")


def test_gate_knn_q4_device_form_repeatable(backend):
    import torch
    nl, nf, hidden, b, k = 2, 3000, 512, 4, 10
    w = O.quantize_q4_0(normal(seed_for("gq4d"), nl * nf * hidden, 0.02))
    wt = backend.register_weight(w, L.FMT_Q4_0, nl * nf, hidden)
    q = torch.randn(b, hidden, device="cuda")
    oi = torch.empty(nl * b * k, dtype=torch.int32, device="cuda")
    os_ = torch.empty(nl * b * k, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.gate_topk_q4_dev(wt, nl, nf, q, b, k, oi, os_)
    backend.sync()
    i1, s1 = oi.cpu().numpy().copy(), os_.cpu().numpy().copy()
    backend.gate_topk_q4_dev(wt, nl, nf, q, b, k, oi, os_)
    backend.sync()
    assert np.array_equal(i1, oi.cpu().numpy()) and np.array_equal(s1, os_.cpu().numpy())
    host_i, host_s = backend.gate_knn_q4(w, nl, nf, hidden, q.cpu().numpy(), k)
    assert np.array_equal(host_i.reshape(-1), i1.view(np.uint32)) and np.array_equal(host_s.reshape(-1), s1)
    wt.release()


def test_gate_knn_q4_unsupported_shapes(backend):
    w = O.quantize_q4_0(np.zeros(2 * 100 * 96, np.float32))
    assert backend.gate_knn_q4(w, 2, 100, 96, np.ones(96, np.float32), 10) is None       # hidden % 64
    w = O.quantize_q4_0(np.zeros(2 * 100 * 128, np.float32))
    assert backend.gate_knn_q4(w, 2, 100, 128, np.ones(128, np.float32), 17) is None     # top_k > 16
