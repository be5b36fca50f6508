"""The vindex loader's host side (CPU only): index.json parsing and the layout checks of larql_cuda_vindex_probe.

Reference: crates/larql-vindex/src/format/load.rs:19-87 (VectorIndex::load_vindex), config/types.rs
(VindexConfig), config/dtype.rs (dtype, f32 by default), index/walk.rs:225 (interleaved_q4k.bin) and :402-445
(attn_weights_q4k.bin + manifest).  The reference's own fixture (tests/golden/vindex_ui_walk_trace, copied by
tests/golden/make_vindex_fixture.py) is probed as it lies on disk.
"""
import json
import os

import numpy as np
import pytest

import larql_cuda as L
import oracle as O
from vindex_util import write_vindex

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vindex_ui_walk_trace")


def _probe_fails(path, words):
    with pytest.raises(L.LarqlCudaError) as ei:
        L.vindex_probe(str(path))
    assert ei.value.status == L.ERR_INVALID_ARG
    for w in words:
        assert w in str(ei.value), str(ei.value)


def test_reference_fixture_probe():
    i = L.vindex_probe(FIXTURE)
    assert (i.num_layers, i.hidden, i.intermediate, i.vocab) == (2, 8, 4, 16)
    assert i.features_max == 4 and i.gate_bits == 32
    assert i.ffn_q4k == 0 and i.attn_q4k == 0
    assert (i.shard_rank, i.shard_count, i.shard_row0, i.shard_rows) == (0, 1, 0, 4)
    cfg = json.load(open(os.path.join(FIXTURE, "index.json")))
    assert [l["offset"] for l in cfg["layers"]] == [0, 128]
    assert os.path.getsize(os.path.join(FIXTURE, "gate_vectors.bin")) == 2 * 4 * 8 * 4


def test_synthetic_layouts(tmp_path):
    rng = np.random.default_rng(1)
    H, I = 256, 512
    gates = [rng.standard_normal((I, H)).astype(np.float32) * 0.02 for _ in range(2)]
    q4 = lambda r, c: O.quantize_q4_k(rng.standard_normal(r * c, dtype=np.float32) * np.float32(0.02))
    q6 = lambda r, c: O.quantize_q6_k(rng.standard_normal(r * c, dtype=np.float32) * np.float32(0.02))
    # the writer's layout: gate / up Q4_K, down Q6_K
    p = write_vindex(str(tmp_path / "a"), gates, "f16", I, ffn=[(q4(I, H), q4(I, H), q6(H, I))] * 2)
    i = L.vindex_probe(p)
    assert (i.num_layers, i.hidden, i.intermediate, i.features_max, i.gate_bits, i.ffn_q4k) == (2, H, I, I, 16, 2)
    # the reader's layout: three Q4_K matrices
    p = write_vindex(str(tmp_path / "b"), gates, "f32", I, ffn=[(q4(I, H), q4(I, H), q4(H, I))] * 2)
    assert L.vindex_probe(p).ffn_q4k == 1
    # attention manifest, with shapes and with shapes taken from the model config
    att = [(q4(H, H), H, H, "Q4_K"), (q4(128, H), 128, H, "Q4_K"), (q6(128, H), 128, H, "Q6_K"),
           (q4(H, H), H, H, "Q4_K")] * 2
    p = write_vindex(str(tmp_path / "c"), gates, "f16", I, attn=att)
    assert L.vindex_probe(p).attn_q4k == 1
    mc = {"model_type": "llama", "head_dim": 64, "num_q_heads": 4, "num_kv_heads": 2}
    p = write_vindex(str(tmp_path / "d"), gates, "f16", I, attn=att, model_config=mc, attn_shapes=False)
    assert L.vindex_probe(p).attn_q4k == 1


def test_layers_with_different_feature_counts(tmp_path):
    rng = np.random.default_rng(2)
    gates = [rng.standard_normal((n, 64)).astype(np.float32) for n in (30, 50, 10)]
    i = L.vindex_probe(write_vindex(str(tmp_path / "v"), gates, "f32"))
    assert i.features_max == 50 and i.num_layers == 3


def test_dtype_defaults_to_f32(tmp_path):
    p = write_vindex(str(tmp_path / "v"), [np.ones((4, 8), np.float32)], "f32")
    cfg = json.load(open(os.path.join(p, "index.json")))
    del cfg["dtype"]
    json.dump(cfg, open(os.path.join(p, "index.json"), "w"))
    assert L.vindex_probe(p).gate_bits == 32


def test_malformed_inputs_are_rejected_with_a_message(tmp_path):
    _probe_fails(tmp_path / "missing", ["index.json"])
    p = write_vindex(str(tmp_path / "v"), [np.ones((4, 8), np.float32)] * 2, "f32")
    ij = os.path.join(p, "index.json")
    good = open(ij).read()
    open(ij, "w").write(good[:-5])
    _probe_fails(p, ["index.json"])
    cfg = json.loads(good)
    for edit, words in [(lambda c: c.update(dtype="bf16"), ["dtype"]),
                        (lambda c: c["layers"][1].update(layer=7), ["layer 7"]),
                        (lambda c: c["layers"][0].update(length=8), ["layer 0"]),
                        (lambda c: c["layers"][1].update(offset=1000), ["gate_vectors.bin"]),
                        (lambda c: c.pop("layers"), ["layers"]),
                        (lambda c: c.update(num_layers=0), ["num_layers"])]:
        c = json.loads(good)
        edit(c)
        json.dump(c, open(ij, "w"))
        _probe_fails(p, words)
    json.dump(cfg, open(ij, "w"))
    assert L.vindex_probe(p).num_layers == 2


def test_ffn_and_manifest_size_checks(tmp_path):
    H, I = 256, 256
    gates = [np.zeros((I, H), np.float32)]
    blk = np.zeros(I * H // 256 * 148, np.uint8)
    p = write_vindex(str(tmp_path / "v"), gates, "f16", I, ffn=[(blk, blk, blk[:-148])])
    _probe_fails(p, ["interleaved_q4k.bin"])
    p = write_vindex(str(tmp_path / "w"), gates, "f16", I, attn=[(blk[:-148], I, H, "Q4_K")] * 4)
    _probe_fails(p, ["manifest entry 0"])


def test_q4_gate_file(tmp_path):
    rng = np.random.default_rng(3)
    gates = [rng.standard_normal((n, 128)).astype(np.float32) * 0.02 for n in (40, 24)]
    q4 = [O.quantize_q4_0(g.reshape(-1)) for g in gates]
    assert L.vindex_probe(write_vindex(str(tmp_path / "a"), gates, "f16", gates_q4=q4)).gate_q4 == 1
    assert L.vindex_probe(write_vindex(str(tmp_path / "b"), gates, "f16")).gate_q4 == 0
    _probe_fails(write_vindex(str(tmp_path / "c"), gates, "f16", gates_q4=[q4[0]]), ["gate_vectors_q4.bin"])

