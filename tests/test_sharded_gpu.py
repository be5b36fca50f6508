"""The row-sharded paths across two GPUs of one node over NCCL (skipped with fewer GPUs): one process per GPU.

* Q4_K matvec: each rank multiplies its row shard, the shards' outputs are all-gathered (the north star's
  row-shard + all-gather design); the gathered vector equals the oracle's (q4k_matvec.rs:31-87) within
  1e-3 * |y|_inf.
* lm-head KNN (lm_head_knn_backend, crates/larql-vindex/src/index/walk.rs:549-583): each rank takes the top-k
  logits of its vocabulary rows, the (id, logit) lists are all-gathered and the top-k of the candidates by signed
  logit is the whole head's top-k (oracle: quantize_to_q8, q4_0_matvec_c, top_k_signed; ties within 1e-5).
* gate walk through the vindex loader: each rank opens the same directory with its (rank, world) row shard, the
  per-rank top-k lists are all-gathered and merged with larql_cuda_topk_merge_dev at the shards' first rows;
  the merged lists equal the oracle's top-k by |score| (gate.rs:108-134, 307-316; ties within 1e-5).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
L = pytest.importorskip("larql_cuda")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, vdir):
    import datetime
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import oracle as O
    from conftest import max_err_ok, normal, seed_for
    from vindex_util import check_topk
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    be = L.CudaBackend(rank)
    try:
        # ── Q4_K matvec, row shards + all-gather ──
        n, k = 2000, 4096
        w = O.quantize_q4_k(normal(seed_for("sh-q4k", n, k), n * k, 0.02))
        x = normal(seed_for("sh-x", k), k)
        per = (n + world - 1) // world
        r0, r1 = rank * per, min(n, (rank + 1) * per)
        rb = k // 256 * 148
        wt = be.register_weight(np.ascontiguousarray(w[r0 * rb:r1 * rb]), L.FMT_Q4_K, r1 - r0, k)
        y = torch.zeros(per, dtype=torch.float32, device="cuda")
        xd = torch.from_numpy(x).cuda()
        torch.cuda.synchronize()
        be.matvec_dev(wt, xd, y[:r1 - r0], batch=1)
        be.sync()
        yall = torch.empty(per * world, dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(yall, y)
        ok, err, bound = max_err_ok(yall.cpu().numpy()[:n], O.q4k_matvec(w, x, n, k))
        assert ok, ("sharded matvec", err, bound)
        wt.release()

        # ── lm-head KNN, vocabulary shards ──
        vocab, hid, topk = 6000, 1024, 10
        wh = O.quantize_q4_0(normal(seed_for("sh-lm", vocab, hid), vocab * hid, 0.02))
        q = normal(seed_for("sh-q", hid), hid)
        vper = (vocab + world - 1) // world
        v0, v1 = rank * vper, min(vocab, (rank + 1) * vper)
        lb = hid // 32 * 18
        ht = be.register_weight(np.ascontiguousarray(wh[v0 * lb:v1 * lb]), L.FMT_Q4_0, v1 - v0, hid)
        ids = torch.empty(topk, dtype=torch.int32, device="cuda")
        vals = torch.empty(topk, dtype=torch.float32, device="cuda")
        qd = torch.from_numpy(q).cuda()
        torch.cuda.synchronize()
        be.lm_head_knn_dev(ht, qd, topk, ids, vals)
        be.sync()
        gids = torch.empty(world * topk, dtype=torch.int32, device="cuda")
        gvals = torch.empty(world * topk, dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(gids, ids + v0)
        dist.all_gather_into_tensor(gvals, vals)
        cv, ci = gvals.cpu().numpy(), gids.cpu().numpy()
        order = np.lexsort((ci, -cv))[:topk]
        got_i, got_v = ci[order], cv[order]
        q8, s8 = O.quantize_to_q8(q)
        logits = O.q4_0_matvec_q8(wh, q8, s8, vocab, hid).astype(np.float64)
        kth = np.sort(logits)[::-1][topk - 1]
        assert len(set(got_i.tolist())) == topk
        assert np.all(logits[got_i] >= kth - 1e-5), "sharded lm-head: not the top-k"
        assert set(np.nonzero(logits > kth + 1e-5)[0].tolist()) <= set(got_i.tolist())
        np.testing.assert_allclose(got_v, logits[got_i], rtol=0, atol=2e-5 * max(1.0, np.abs(logits).max()))
        ht.release()

        # ── gate walk through the vindex loader, row shards + merge ──
        v = L.Vindex(be, vdir, rank, world)
        try:
            nl, hidden, kk, b = v.info.num_layers, v.info.hidden, 10, 3
            qg = np.random.default_rng(5).standard_normal((b, hidden)).astype(np.float32)
            qgd = torch.from_numpy(qg).cuda()
            oi = torch.empty(nl * b * kk, dtype=torch.int32, device="cuda")
            osc = torch.empty(nl * b * kk, dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            v.gate_knn_dev(qgd, b, kk, oi, osc)
            be.sync()
            gi = torch.empty(world * nl * b * kk, dtype=torch.int32, device="cuda")
            gs = torch.empty(world * nl * b * kk, dtype=torch.float32, device="cuda")
            dist.all_gather_into_tensor(gi, oi)
            dist.all_gather_into_tensor(gs, osc)
            offs = torch.tensor([r * v.info.shard_rows for r in range(world)], dtype=torch.int32, device="cuda")
            mi = torch.empty(nl * b * kk, dtype=torch.int32, device="cuda")
            ms = torch.empty(nl * b * kk, dtype=torch.float32, device="cuda")
            be.topk_merge_dev(gi, gs, world, nl * b, kk, kk, mi, ms, offsets=offs)
            be.sync()
            mi_h = mi.cpu().numpy().view(np.uint32).reshape(nl, b, kk)
            ms_h = ms.cpu().numpy().reshape(nl, b, kk)
            gates = np.load(os.path.join(vdir, "gates.npy"))
            for l in range(nl):
                ref = O.gate_scores_f16_many(gates[l].astype(np.float16).view(np.uint16), qg, gates.shape[1], hidden)
                for qi in range(b):
                    check_topk(mi_h[l, qi], ms_h[l, qi], ref[qi], kk, f"sharded gate walk layer {l} query {qi}")
        finally:
            v.close()
        dist.barrier()
        open(os.path.join(out_dir, f"ok{rank}"), "w").close()
    finally:
        be.close()
        dist.destroy_process_group()


def test_row_sharded_paths_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from vindex_util import write_vindex
    rng = np.random.default_rng(3)
    gates = (rng.standard_normal((3, 1001, 512)) * 0.02).astype(np.float32)  # 1001 rows: uneven shards
    vdir = write_vindex(str(tmp_path / "vindex"), list(gates), "f16")
    np.save(os.path.join(vdir, "gates.npy"), gates)
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), vdir), nprocs=2, join=True)
    assert all((tmp_path / f"ok{r}").exists() for r in range(2))
