"""Writes small .vindex directories in the reference's on-disk layout, for the loader tests.

Layout (crates/larql-vindex/src/config/types.rs VindexConfig; format/load.rs:19-87; index/walk.rs:225,402-445;
examples/build_q4k_weights.rs): index.json with num_layers / hidden_size / intermediate_size / dtype and
layers[] = {layer, num_features, offset, length} (byte offsets into gate_vectors.bin), gate_vectors.bin with each
layer's rows (f32 or f16), interleaved_q4k.bin with per layer gate, up (Q4_K) and down (Q6_K, or Q4_K in the
all-Q4_K layout), attn_weights_q4k.bin with attn_weights_q4k_manifest.json = [{key, shape, format, offset,
length}] four entries (Q, K, V, O) per layer.
"""
from __future__ import annotations

import json
import os

import numpy as np

TIE = 1e-5


def write_vindex(path, gates, dtype="f16", inter=0, ffn=None, attn=None, model_config=None, attn_shapes=True,
                 gates_q4=None):
    """gates: list of [features_l, hidden] f32 arrays (stored as f16 when dtype == "f16").
    ffn: list of (gate_bytes, up_bytes, down_bytes) per layer; attn: list of (bytes, rows, cols, "Q4_K"|"Q6_K"),
    four per layer; gates_q4: list of per-layer Q4_0 bytes (gate_vectors_q4.bin, walk.rs:303-328)."""
    os.makedirs(path, exist_ok=True)
    hidden = gates[0].shape[1]
    layers, blobs, off = [], [], 0
    for l, g in enumerate(gates):
        b = np.ascontiguousarray(g, dtype=np.float16 if dtype == "f16" else np.float32).tobytes()
        layers.append({"layer": l, "num_features": int(g.shape[0]), "offset": off, "length": len(b)})
        blobs.append(b)
        off += len(b)
    with open(os.path.join(path, "gate_vectors.bin"), "wb") as f:
        for b in blobs:
            f.write(b)
    cfg = {"version": 2, "model": "test/synthetic", "family": "llama", "num_layers": len(gates),
           "hidden_size": hidden, "intermediate_size": inter, "vocab_size": 0, "embed_scale": 1.0,
           "extract_level": "all", "dtype": dtype, "layers": layers, "down_top_k": 5, "has_model_weights": False}
    if model_config:
        cfg["model_config"] = model_config
    with open(os.path.join(path, "index.json"), "w") as f:
        json.dump(cfg, f, indent=2)
    if gates_q4 is not None:
        with open(os.path.join(path, "gate_vectors_q4.bin"), "wb") as f:
            for b in gates_q4:
                f.write(np.ascontiguousarray(b).tobytes())
    if ffn is not None:
        with open(os.path.join(path, "interleaved_q4k.bin"), "wb") as f:
            for (g, u, d) in ffn:
                f.write(np.ascontiguousarray(g).tobytes())
                f.write(np.ascontiguousarray(u).tobytes())
                f.write(np.ascontiguousarray(d).tobytes())
    if attn is not None:
        man, off = [], 0
        with open(os.path.join(path, "attn_weights_q4k.bin"), "wb") as f:
            for i, (data, rows, cols, fmt) in enumerate(attn):
                b = np.ascontiguousarray(data).tobytes()
                e = {"key": f"layers.{i // 4}.{'qkvo'[i % 4]}_proj", "format": fmt, "offset": off, "length": len(b)}
                if attn_shapes:
                    e["shape"] = [rows, cols]
                man.append(e)
                f.write(b)
                off += len(b)
        with open(os.path.join(path, "attn_weights_q4k_manifest.json"), "w") as f:
            json.dump(man, f, indent=2)
    return path


def check_topk(got_i, got_s, ref, k, what):
    """got_*: [k] for one (layer, query); ref: oracle scores of every row of that layer.  Index set equal to the
    top-k by |score| except for ties within 1e-5; scores within 2e-5 (relative to max(1, max |score|))."""
    a = np.abs(ref.astype(np.float64))
    n = a.size
    kk = min(k, n)
    order = np.argsort(-a, kind="stable")
    kth = a[order[kk - 1]]
    gi = got_i[:kk].astype(np.int64)
    assert np.all(gi < n), f"{what}: index out of range {gi}"
    assert len(set(gi.tolist())) == kk, f"{what}: duplicate indices {gi}"
    assert np.all(a[gi] >= kth - TIE), f"{what}: {gi[a[gi] < kth - TIE]} are not top-{k}"
    must = set(np.nonzero(a > kth + TIE)[0].tolist())
    assert must <= set(gi.tolist()), f"{what}: missing {sorted(must - set(gi.tolist()))}"
    np.testing.assert_allclose(got_s[:kk], ref[gi], rtol=0, atol=2e-5 * max(1.0, a.max()), err_msg=what)
    if k > n:
        assert np.all(got_i[n:] == 0xFFFFFFFF), f"{what}: slots past the layer's rows are not empty"
