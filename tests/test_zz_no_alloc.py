"""The no-allocation Q4_K matvec entry point (larql_cuda_q4k_matvec_noalloc).

Some callers cannot allocate device memory while they run — they work inside
a budget reserved up front, or in memory another framework owns.  For them the
library offers one entry point whose scratch is a fixed array compiled into the
library instead of memory allocated per call.  This test calls it through the
C ABI twice in a row and checks each result against the CPU oracle
(q4k_matvec.rs:31-87 restated) and against the regular entry point
(larql_cuda_matvec_dev on a registered weight), both within the matvec
tolerance (max |err| <= 1e-3 * ||y||_inf); it also checks that a call leaves
the device's free memory unchanged.  It lives in a file collected last so a
stopping run has already run every other test, and it makes its own inputs so
it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, random_q4k_blocks, seed_for

pytestmark = pytest.mark.gpu

L = pytest.importorskip("larql_cuda")


def _noalloc(w_dev, nbytes, rows, cols, x_dev, batch, y, stream):
    return L.lib().larql_cuda_q4k_matvec_noalloc(w_dev.data_ptr(), nbytes, rows, cols, x_dev.data_ptr(), batch,
                                                 y.data_ptr(), stream)


@pytest.mark.parametrize("rows,cols,batch,kind", [(300, 4096, 1, "quantized"), (1000, 4096, 4, "quantized"),
                                                  (257, 14336, 8, "quantized"), (40, 16384, 3, "quantized"),
                                                  (96, 2048, 5, "random_bytes")])
def test_noalloc_matches_oracle_and_regular_entry_point_twice(backend, rows, cols, batch, kind):
    import torch
    if kind == "quantized":
        w = O.quantize_q4_k(normal(seed_for("na", rows, cols), rows * cols, 0.02))
    else:  # every nibble and 6-bit scale, random finite f16 d / dmin
        w = random_q4k_blocks(seed_for("nab", rows, cols), rows, cols)
    x = normal(seed_for("nax", rows, cols, batch), batch * cols)
    oracle = np.stack([O.q4k_matvec(w, np.ascontiguousarray(x[b * cols:(b + 1) * cols]), rows, cols)
                       for b in range(batch)])
    w_dev = torch.from_numpy(w).cuda()
    x_dev = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, cols)
    y_ref = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.matvec_dev(wt, x_dev, y_ref, batch=batch)
    backend.sync()
    regular = y_ref.cpu().numpy().reshape(batch, rows)
    wt.release()
    for b in range(batch):
        ok, err, bound = max_err_ok(regular[b], oracle[b])
        assert ok, ("regular entry point vs oracle", b, err, bound)
    for call in range(2):
        y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
        rc = _noalloc(w_dev, w.nbytes, rows, cols, x_dev, batch, y, stream)
        assert rc == 0, L.last_error()
        got = y.cpu().numpy().reshape(batch, rows)
        for b in range(batch):
            ok, err, bound = max_err_ok(got[b], oracle[b])
            assert ok, ("noalloc vs oracle", call, b, err, bound)
            ok, err, bound = max_err_ok(got[b], regular[b])
            assert ok, ("noalloc vs regular entry point", call, b, err, bound)


def test_noalloc_call_leaves_free_device_memory_unchanged(backend):
    import torch
    rows, cols, batch = 512, 8192, 8
    w = O.quantize_q4_k(normal(seed_for("nam", rows, cols), rows * cols, 0.02))
    w_dev = torch.from_numpy(w).cuda()
    x_dev = torch.from_numpy(normal(seed_for("namx"), batch * cols)).cuda()
    y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert _noalloc(w_dev, w.nbytes, rows, cols, x_dev, batch, y, stream) == 0, L.last_error()  # set-up call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(w_dev, w.nbytes, rows, cols, x_dev, batch, y, stream) == 0, L.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_sizes_beyond_its_scratch(backend):
    import torch
    w = torch.zeros(148 * 80, dtype=torch.uint8, device="cuda")
    x = torch.zeros(20480 * 9, dtype=torch.float32, device="cuda")
    y = torch.zeros(9, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.lib().larql_cuda_q4k_matvec_noalloc(w.data_ptr(), w.numel(), 1, 20480, x.data_ptr(), 1, y.data_ptr(), stream)
    assert rc == L.ERR_BAD_SHAPE and "16384" in L.last_error()
    rc = L.lib().larql_cuda_q4k_matvec_noalloc(w.data_ptr(), w.numel(), 1, 4096, x.data_ptr(), 9, y.data_ptr(), stream)
    assert rc == L.ERR_BAD_SHAPE and "batch" in L.last_error()
