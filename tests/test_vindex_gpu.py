"""The vindex loader on the GPU: gate rows placed once and walked, FFN / attention weights placed from the files.

Reference: crates/larql-vindex/src/format/load.rs:19-87 (load_vindex), index/gate.rs:108-134 and :307-316
(gate_knn: scores of the decoded rows, top-K by |score|), index/walk.rs:225 and :402-445 (interleaved_q4k.bin,
attn_weights_q4k.bin + manifest).  Oracle: f64 scores of the rows as the reference decodes them (f32 as stored;
f16 by half.rs), top-K index sets equal except for ties within 1e-5; matvecs within 1e-3 * |y|_inf of the
restated CPU matvecs (q4k_matvec.rs:31-87, q6k_matvec.rs:31-87).
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, seed_for
from vindex_util import check_topk, write_vindex

pytestmark = pytest.mark.gpu
L = pytest.importorskip("larql_cuda")
FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vindex_ui_walk_trace")


def _scores_f32(rows, q):
    return (q.astype(np.float64) @ rows.astype(np.float64).T).astype(np.float32)


def _scores_f16(rows_f32, q):
    bits = np.ascontiguousarray(rows_f32, dtype=np.float16).view(np.uint16)
    return O.gate_scores_f16_many(bits, q, rows_f32.shape[0], rows_f32.shape[1])


def test_reference_fixture_walk(backend):
    """The reference's ui_walk_trace vindex (2 layers x 4 f32 gate rows, hidden 8, rows e_i and 2 e_i): a unit
    query e_i scores feature i highest (1, then 2 in layer 1); random queries against the f64 oracle."""
    v = L.Vindex(backend, FIXTURE)
    try:
        g = np.fromfile(os.path.join(FIXTURE, "gate_vectors.bin"), np.float32).reshape(2, 4, 8)
        q = np.eye(8, dtype=np.float32)[:4]
        idx, sc = v.gate_knn(q, 4)
        for l in range(2):
            for i in range(4):
                assert idx[l, i, 0] == i and sc[l, i, 0] == np.float32(l + 1), (l, i, idx[l, i], sc[l, i])
        qr = np.random.default_rng(3).standard_normal((5, 8)).astype(np.float32)
        for k in (1, 3, 4, 6):
            idx, sc = v.gate_knn(qr, k)
            for l in range(2):
                ref = _scores_f32(g[l], qr)
                for b in range(5):
                    check_topk(idx[l, b], sc[l, b], ref[b], k, f"fixture layer {l} query {b} k {k}")
    finally:
        v.close()


@pytest.mark.parametrize("hidden,batch", [(320, 1), (320, 70), (512, 3), (512, 1), (2560, 2)])
def test_f16_vindex_uneven_layers(backend, tmp_path, hidden, batch):
    """f16 gates (half.rs decoding, subnormals included), layers of 700 / 500 / 13 rows (zero-row padding), hidden
    not a multiple of 64 (zero columns), batches on the CUDA-core and the tensor-core walk."""
    rng = np.random.default_rng(seed_for("vx16", hidden, batch))
    feats = (700, 500, 13)
    gates = [(rng.standard_normal((n, hidden)) * 0.02).astype(np.float32) for n in feats]
    gates[1].reshape(-1)[::97] = 3e-6  # f16 subnormal
    p = write_vindex(str(tmp_path / "v"), gates, "f16")
    q = rng.standard_normal((batch, hidden)).astype(np.float32)
    v = L.Vindex(backend, p)
    try:
        assert v.info.shard_rows == 700
        idx, sc = v.gate_knn(q, 16)
        for l, n in enumerate(feats):
            ref = _scores_f16(gates[l], q)
            for b in range(0, batch, max(1, batch // 7)):
                check_topk(idx[l, b], sc[l, b], ref[b], 16, f"layer {l} ({n} rows) query {b}")
    finally:
        v.close()


def test_f32_vindex_keeps_f32_rows(backend, tmp_path):
    """f32 gates that f16 cannot hold exactly: the high / scaled-low f16 pair keeps the scores within the 1e-5 tie
    window of the f32 rows' f64 scores."""
    rng = np.random.default_rng(7)
    gates = [(rng.standard_normal((600, 256)) * 0.02).astype(np.float32) for _ in range(2)]
    gates[0][:, :5] *= np.float32(1e-4)  # tiny entries (f16 subnormal / zero high parts)
    p = write_vindex(str(tmp_path / "v"), gates, "f32")
    q = rng.standard_normal((9, 256)).astype(np.float32)
    v = L.Vindex(backend, p)
    try:
        assert v.info.gate_bits == 32
        for k in (10, 16):
            idx, sc = v.gate_knn(q, k)
            for l in range(2):
                ref = _scores_f32(gates[l], q)
                for b in range(9):
                    check_topk(idx[l, b], sc[l, b], ref[b], k, f"f32 layer {l} query {b}")
    finally:
        v.close()


def test_row_shards_merge_to_the_whole_walk(backend, tmp_path):
    """Three row shards of every layer (shard_rank 0..2): the union of the shards' top-k, merged by |score|, is
    the top-k of the whole layer; each shard's indices are global (shard_row0 added)."""
    rng = np.random.default_rng(11)
    gates = [(rng.standard_normal((1000, 512)) * 0.02).astype(np.float32) for _ in range(2)]
    p = write_vindex(str(tmp_path / "v"), gates, "f16")
    q = rng.standard_normal((4, 512)).astype(np.float32)
    k = 10
    parts = []
    for r in range(3):
        v = L.Vindex(backend, p, r, 3)
        try:
            assert (v.info.shard_row0, v.info.shard_rows) == (r * 334, 334)
            parts.append(v.gate_knn(q, k))
        finally:
            v.close()
    for l in range(2):
        ref = _scores_f16(gates[l], q)
        for b in range(4):
            ci = np.concatenate([pi[l, b] for pi, _ in parts])
            cs = np.concatenate([ps[l, b] for _, ps in parts])
            ok = ci != 0xFFFFFFFF
            ci, cs = ci[ok], cs[ok]
            order = np.lexsort((ci, -np.abs(cs)))[:k]
            check_topk(ci[order], cs[order], ref[b], k, f"merged layer {l} query {b}")


def test_gate_knn_dev_matches_host(backend, tmp_path):
    import torch
    rng = np.random.default_rng(13)
    gates = [(rng.standard_normal((300, 256)) * 0.02).astype(np.float32) for _ in range(3)]
    p = write_vindex(str(tmp_path / "v"), gates, "f16")
    q = rng.standard_normal((5, 256)).astype(np.float32)
    v = L.Vindex(backend, p)
    try:
        hi, hs = v.gate_knn(q, 8)
        qd = torch.from_numpy(q).cuda()
        oi = torch.empty(3 * 5 * 8, dtype=torch.int32, device="cuda")
        os_ = torch.empty(3 * 5 * 8, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        v.gate_knn_dev(qd, 5, 8, oi, os_)
        backend.sync()
        assert np.array_equal(oi.cpu().numpy().view(np.uint32).reshape(3, 5, 8), hi)
        assert np.array_equal(os_.cpu().numpy().reshape(3, 5, 8), hs)
    finally:
        v.close()


@pytest.mark.parametrize("down_q6k", [True, False])
def test_ffn_weights_from_interleaved_file(backend, tmp_path, down_q6k):
    """interleaved_q4k.bin in the writer's layout (down in Q6_K) and in the reader's (three Q4_K): the placed
    gate / up / down of each layer give the oracle's matvecs; shard 1 of 2 holds the second half of the rows."""
    import torch
    rng = np.random.default_rng(17)
    H, I, nl = 512, 1024, 2
    mats = []
    for _ in range(nl):
        g = O.quantize_q4_k(rng.standard_normal(I * H, dtype=np.float32) * np.float32(0.02))
        u = O.quantize_q4_k(rng.standard_normal(I * H, dtype=np.float32) * np.float32(0.02))
        df = rng.standard_normal(H * I, dtype=np.float32) * np.float32(0.02)
        d = O.quantize_q6_k(df) if down_q6k else O.quantize_q4_k(df)
        mats.append((g, u, d))
    gates = [(rng.standard_normal((I, H)) * 0.02).astype(np.float32) for _ in range(nl)]
    p = write_vindex(str(tmp_path / "v"), gates, "f16", I, ffn=mats)
    xh = rng.standard_normal(H, dtype=np.float32)
    xi = rng.standard_normal(I, dtype=np.float32)
    for rank, count in ((0, 1), (1, 2)):
        v = L.Vindex(backend, p, rank, count)
        try:
            assert v.info.ffn_q4k == (2 if down_q6k else 1)
            for l in range(nl):
                wg, wu, wd = v.ffn(l)
                for w, data, x, rows, cols, fn in ((wg, mats[l][0], xh, I, H, O.q4k_matvec),
                                                   (wu, mats[l][1], xh, I, H, O.q4k_matvec),
                                                   (wd, mats[l][2], xi, H, I,
                                                    O.q6k_matvec if down_q6k else O.q4k_matvec)):
                    ref = fn(data, x, rows, cols)
                    per = rows // count
                    y = torch.empty(per, dtype=torch.float32, device="cuda")
                    xd = torch.from_numpy(x).cuda()
                    torch.cuda.synchronize()
                    backend.matvec_dev(w, xd, y, batch=1)
                    backend.sync()
                    ok, err, bound = max_err_ok(y.cpu().numpy(), ref[rank * per:(rank + 1) * per])
                    assert ok, (l, rows, cols, rank, err, bound)
        finally:
            v.close()


def test_attention_weights_from_manifest(backend, tmp_path):
    """attn_weights_q4k.bin + manifest (Q, K, O in Q4_K, V in Q6_K as the reference's writer does): the placed
    weights give the oracle's matvecs; shapes from the manifest and, without them, from the model config."""
    import torch
    rng = np.random.default_rng(19)
    H, hd, nq, nkv = 512, 64, 8, 2
    shapes = [(nq * hd, H), (nkv * hd, H), (nkv * hd, H), (H, nq * hd)]
    ent = []
    for i, (r, c) in enumerate(shapes * 2):
        wf = rng.standard_normal(r * c, dtype=np.float32) * np.float32(0.02)
        fmt = "Q6_K" if i % 4 == 2 else "Q4_K"
        ent.append((O.quantize_q6_k(wf) if fmt == "Q6_K" else O.quantize_q4_k(wf), r, c, fmt))
    gates = [(rng.standard_normal((64, H)) * 0.02).astype(np.float32) for _ in range(2)]
    mc = {"model_type": "llama", "head_dim": hd, "num_q_heads": nq, "num_kv_heads": nkv}
    for shapes_in_manifest in (True, False):
        p = write_vindex(str(tmp_path / f"v{int(shapes_in_manifest)}"), gates, "f16", 0, attn=ent, model_config=mc,
                         attn_shapes=shapes_in_manifest)
        v = L.Vindex(backend, p)
        try:
            for l in range(2):
                hs = v.attn(l)
                for i, (h, fmt) in enumerate(hs):
                    data, r, c, fs = ent[4 * l + i]
                    assert fmt == (L.FMT_Q6_K if fs == "Q6_K" else L.FMT_Q4_K)
                    x = rng.standard_normal(c, dtype=np.float32)
                    ref = (O.q6k_matvec if fs == "Q6_K" else O.q4k_matvec)(data, x, r, c)
                    w = L.Weight(backend, h, fmt, r, c)
                    y = torch.empty(r, dtype=torch.float32, device="cuda")
                    xd = torch.from_numpy(x).cuda()
                    torch.cuda.synchronize()
                    backend.matvec_dev(w, xd, y, batch=1)
                    backend.sync()
                    ok, err, bound = max_err_ok(y.cpu().numpy(), ref)
                    assert ok, (l, i, err, bound)
        finally:
            v.close()


@pytest.mark.parametrize("count", [1, 2])
def test_q4_gates_walk(backend, tmp_path, count):
    """gate_vectors_q4.bin (Q4_0 rows of layers of 900 / 600 features, hidden 256) placed at open and walked by
    gate_knn_q4: the oracle's quantize_to_q8 + q4_0_matvec_c scores, top-10 by |score|; two row shards merge
    to the whole walk."""
    rng = np.random.default_rng(23)
    H, feats, k = 256, (900, 600), 10
    gates = [(rng.standard_normal((n, H)) * 0.02).astype(np.float32) for n in feats]
    q4 = [O.quantize_q4_0(g.reshape(-1)) for g in gates]
    p = write_vindex(str(tmp_path / "v"), gates, "f16", gates_q4=q4)
    q = rng.standard_normal((3, H)).astype(np.float32)
    parts = []
    for r in range(count):
        v = L.Vindex(backend, p, r, count)
        try:
            assert v.info.gate_q4 == 1
            parts.append(v.gate_knn_q4(q, k))
        finally:
            v.close()
    for l, n in enumerate(feats):
        for b in range(3):
            q8, s8 = O.quantize_to_q8(q[b])
            ref = O.q4_0_matvec_q8(q4[l], q8, s8, n, H)
            ci = np.concatenate([pi[l, b] for pi, _ in parts])
            cs = np.concatenate([ps[l, b] for _, ps in parts])
            ok = ci != 0xFFFFFFFF
            ci, cs = ci[ok], cs[ok]
            order = np.lexsort((ci, -np.abs(cs)))[:k]
            check_topk(ci[order], cs[order], ref, k, f"Q4 vindex layer {l} query {b} shards {count}")

