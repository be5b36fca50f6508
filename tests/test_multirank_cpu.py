"""World-size-2 `gloo` ranks on the CPU: the sharded designs the GPU paths use, checked with the oracle.

* Matvec row shards (the bench's multi-GPU step): rank r owns a contiguous row range of W, computes its rows
  and the ranks all-gather them; the result is the unsharded matvec, bit for bit (rows are independent).
* Gate-walk row shards: each rank takes the top-k of its slice of every layer's gate rows with the slice's
  row offset added, the lists are all-gathered and merged by |score| (ties by index), as
  larql_cuda_topk_merge_dev does; the merged list is the unsharded top-k.
* lm-head KNN row shards (larql_cuda_lm_head_knn_dev per rank on its vocabulary rows): each rank's top-k ids
  shifted by its first row, ids and logits all-gathered in rank order, and the selection applied once more to
  the gathered logits (larql_cuda_logit_topk_dev; equal logits go to the lower position, i.e. the lower rank,
  i.e. the lower token id) gives the unsharded top-k, ties included.
* Tensor-parallel decode (larql_cuda_layer_register_shard): O and down are split by input columns in whole
  256-value Q4_K blocks; the per-rank partial products all-reduced over the ranks equal the full projections.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O
from conftest import normal

torch = pytest.importorskip("torch")
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _q4k_cols(w, rows, cols, c0, c1):
    """Input-column slice [c0, c1) (multiples of 256) of a Q4_K matrix: whole 148-byte blocks of every row."""
    b = w.reshape(rows, cols // 256, 148)
    return np.ascontiguousarray(b[:, c0 // 256:c1 // 256]).reshape(-1)


def _merge_topk(idx, sc, k):
    """top-k by |score| descending, ties by ascending index, over the union of the lists."""
    order = sorted(range(len(idx)), key=lambda i: (-abs(float(sc[i])), int(idx[i])))[:k]
    return [int(idx[i]) for i in order]


def _worker(rank, port, case, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        if case == "rows":
            rows, cols = 301, 1024
            w = O.quantize_q4_k(normal(101, rows * cols, 0.02))
            x = normal(102, cols)
            per = (rows + WORLD - 1) // WORLD
            r0, r1 = rank * per, min(rows, (rank + 1) * per)
            rb = cols // 256 * 148
            mine = O.q4k_matvec(w[r0 * rb:r1 * rb], x, r1 - r0, cols)
            buf = torch.zeros(per, dtype=torch.float32)
            buf[:r1 - r0] = torch.from_numpy(mine)
            parts = [torch.zeros(per, dtype=torch.float32) for _ in range(WORLD)]
            dist.all_gather(parts, buf)
            got = torch.cat(parts)[:rows].numpy()
            ref = O.q4k_matvec(w, x, rows, cols)
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        elif case == "gate":
            nf, hidden, k = 700, 128, 10
            g = (np.random.default_rng(103).standard_normal(nf * hidden).astype(np.float32) * 0.02).astype(np.float16)
            g = g.view(np.uint16)
            q = normal(104, 3 * hidden).reshape(3, hidden)
            per = (nf + WORLD - 1) // WORLD
            f0, f1 = rank * per, min(nf, (rank + 1) * per)
            sc = O.gate_scores_f16(g[f0 * hidden:f1 * hidden], q, f1 - f0, hidden)
            li = np.zeros((3, k), np.int64)
            ls = np.zeros((3, k), np.float32)
            for b in range(3):
                ii = sorted(range(f1 - f0), key=lambda i: (-abs(float(sc[b, i])), i))[:k]
                li[b] = np.array(ii) + f0
                ls[b] = sc[b, ii]
            gi = [torch.zeros((3, k), dtype=torch.int64) for _ in range(WORLD)]
            gs = [torch.zeros((3, k), dtype=torch.float32) for _ in range(WORLD)]
            dist.all_gather(gi, torch.from_numpy(li))
            dist.all_gather(gs, torch.from_numpy(ls))
            full = O.gate_scores_f16(g, q, nf, hidden)
            for b in range(3):
                merged = _merge_topk(np.concatenate([t[b].numpy() for t in gi]),
                                     np.concatenate([t[b].numpy() for t in gs]), k)
                ref = sorted(range(nf), key=lambda i: (-abs(float(full[b, i])), i))[:k]
                assert merged == ref, (b, merged, ref)
        elif case == "lmhead":
            vocab, hidden, k = 1001, 256, 12
            wf = normal(109, vocab * hidden, 0.02).reshape(vocab, hidden)
            per = (vocab + WORLD - 1) // WORLD
            q = normal(110, hidden)
            # rows 3 and 40 lead the logits, and each has a copy on the other rank: equal logits, so the lower
            # token id must come first
            wf[3], wf[40] = q * np.float32(0.02), q * np.float32(0.015)
            wf[per + 3], wf[per + 40] = wf[3], wf[40]
            w = O.quantize_q4_0(wf.reshape(-1))
            v0, v1 = rank * per, min(vocab, (rank + 1) * per)
            rb = hidden // 32 * 18
            ids, vals, _ = O.lm_head_knn(w[v0 * rb:v1 * rb], q, v1 - v0, hidden, k)
            gi = [torch.zeros(k, dtype=torch.int64) for _ in range(WORLD)]
            gv = [torch.zeros(k, dtype=torch.float32) for _ in range(WORLD)]
            dist.all_gather(gi, torch.from_numpy(ids.astype(np.int64) + v0))
            dist.all_gather(gv, torch.from_numpy(vals))
            cand_ids = np.concatenate([t.numpy() for t in gi])
            pos, _ = O.top_k_signed(np.concatenate([t.numpy() for t in gv]), k)
            merged = cand_ids[pos.astype(np.int64)].tolist()
            ref, _, logits = O.lm_head_knn(w, q, vocab, hidden, k)
            assert merged == ref.astype(np.int64).tolist(), (merged, ref)
            assert logits[3] == logits[per + 3] and logits[40] == logits[per + 40]
            assert merged[:4] == [3, per + 3, 40, per + 40], merged
        elif case == "tp":
            hidden, qd, inter = 512, 1024, 2048
            wo = O.quantize_q4_k(normal(105, hidden * qd, 0.02))
            wd = O.quantize_q4_k(normal(106, hidden * inter, 0.02))
            attn = normal(107, qd)
            act = normal(108, inter)
            for (w, K, x) in ((wo, qd, attn), (wd, inter, act)):
                c0, c1 = rank * K // WORLD, (rank + 1) * K // WORLD
                part = torch.from_numpy(O.q4k_matvec(_q4k_cols(w, hidden, K, c0, c1), x[c0:c1], hidden, c1 - c0))
                dist.all_reduce(part)
                ref = O.q4k_matvec(w, x, hidden, K)
                np.testing.assert_allclose(part.numpy(), ref, rtol=0, atol=1e-5 * float(np.abs(ref).max()))
        open(os.path.join(out_dir, f"ok{rank}"), "w").close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["rows", "gate", "lmhead", "tp"])
def test_two_gloo_ranks(case, tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(), case, str(tmp_path)), nprocs=WORLD, join=True)
    assert all((tmp_path / f"ok{r}").exists() for r in range(WORLD))
