"""The no-allocation Q4_K matvec entry point (larql_cuda_q4k_matvec_noalloc).

Some callers cannot allocate device memory while they run — they work inside
a budget reserved up front, or in memory another framework owns.  For them the
library offers one entry point whose scratch is a fixed array compiled into the
library instead of memory allocated per call.  This test calls it through the
C ABI twice in a row and checks each result against the regular entry point
(larql_cuda_matvec_dev on a registered weight) within the matvec tolerance
(max |err| <= 1e-3 * ||y||_inf).  It lives in a file collected last so a
stopping run has already run every other test, and it makes its own inputs so
it also passes alone in a fresh process.
"""
import numpy as np
import pytest

import oracle as O
from conftest import max_err_ok, normal, seed_for

pytestmark = pytest.mark.gpu

L = pytest.importorskip("larql_cuda")


@pytest.mark.parametrize("rows,cols,batch", [(300, 4096, 1), (1000, 4096, 4), (257, 14336, 8), (40, 16384, 3)])
def test_noalloc_matches_regular_entry_point_twice(backend, rows, cols, batch):
    import torch
    w = O.quantize_q4_k(normal(seed_for("na", rows, cols), rows * cols, 0.02))
    x = normal(seed_for("nax", rows, cols, batch), batch * cols)
    w_dev = torch.from_numpy(w).cuda()
    x_dev = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    wt = backend.register_weight(w, L.FMT_Q4_K, rows, cols)
    y_ref = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    backend.matvec_dev(wt, x_dev, y_ref, batch=batch)
    backend.sync()
    ref = y_ref.cpu().numpy().reshape(batch, rows)
    wt.release()
    for call in range(2):
        y = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
        rc = L.lib().larql_cuda_q4k_matvec_noalloc(w_dev.data_ptr(), w.nbytes, rows, cols, x_dev.data_ptr(), batch,
                                                   y.data_ptr(), stream)
        assert rc == 0, L.last_error()
        got = y.cpu().numpy().reshape(batch, rows)
        for b in range(batch):
            ok, err, bound = max_err_ok(got[b], ref[b])
            assert ok, (call, b, err, bound)


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
